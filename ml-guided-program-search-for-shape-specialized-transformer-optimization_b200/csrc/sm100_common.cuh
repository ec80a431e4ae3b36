// sm100_common.cuh -- PTX building blocks shared by the sm_100a kernels of
// libb200tx: mbarriers with bounded waits, TMA tile loads, tcgen05 (TMEM
// allocation, UMMA issue, commit, TMEM loads/stores) and the shared-memory
// matrix descriptors the UMMA instructions consume.
//
// Every spin on an mbarrier is bounded in wall-clock time (%globaltimer).  A
// wait that runs out records a code in the library's device error word and
// reports failure to its caller, which then stops issuing work, drains what it
// has in flight (again with bounded waits) and releases its TMEM before the
// kernel returns.  No kernel in this library traps or asserts on the device.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace b200tx {

// Device error word: 0 = healthy.  Kernels write a code with atomicCAS so the
// first failure wins; the host reads and clears it through the C ABI.
__device__ unsigned int g_device_error = 0;

enum DeviceErrorCode : unsigned int {
  kErrNone = 0,
  kErrGemmProducerWait = 0x101,
  kErrGemmMmaWait = 0x102,
  kErrGemmEpilogueWait = 0x103,
  kErrAttnProducerWait = 0x201,
  kErrAttnMmaWait = 0x202,
  kErrAttnSoftmaxWait = 0x203,
  kErrPeerWait = 0x301,  // a tensor-parallel peer did not publish its partial in time
  kErrSeqWait = 0x401,   // the whole-forward kernel's copy or UMMA did not complete in time
};

// A single wait gives up after this many nanoseconds.  Every event waited on
// here completes within microseconds on a healthy GPU.
constexpr unsigned long long kWaitTimeoutNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_device_error(unsigned int code) {
  atomicCAS(&g_device_error, 0u, code);
}

__device__ __forceinline__ bool device_error_raised() {
  return *reinterpret_cast<volatile unsigned int*>(&g_device_error) != 0u;
}

// ------------------------------------------------- programmatic dependent launch
// Kernels of this library are launched with programmatic stream serialization:
// the next kernel of the stream may be scheduled as soon as every CTA of the
// running one has called griddep_launch_dependents(), so its launch and
// set-up (barrier init, TMEM allocation, tensor-map prefetch) overlap this
// kernel's tail.  griddep_wait() blocks until all preceding kernels of the
// stream have completed and their memory is visible; every kernel calls it
// after its set-up and before its first global-memory access.  Launched
// without the attribute, both are no-ops.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns false
// when the wait runs out (after recording `code`), when another role of this
// CTA has raised `abort_flag`, or when any CTA has recorded a device error.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int code,
                                          volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = global_timer_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++spins & 255u) == 0u) {
      if (*abort_flag != 0 || device_error_raised()) {
        *abort_flag = 1;
        return false;
      }
      if (global_timer_ns() - start > kWaitTimeoutNs) {
        record_device_error(code);
        *abort_flag = 1;
        return false;
      }
    }
  }
  return true;
}

// Drain wait before a CTA leaves: for copies this CTA issued, whatever the
// abort state or the device error word, bounded by the same timeout.
__device__ __forceinline__ void mbar_drain_wait(uint64_t* bar, uint32_t parity) {
  const unsigned long long start = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - start > kWaitTimeoutNs) return;
  }
}

// Round a dynamic shared-memory pointer up to the 1024-byte alignment that
// 128-byte-swizzled TMA tiles and UMMA descriptors (base offset 0) require.
__device__ __forceinline__ uint8_t* align_1024(uint8_t* p) {
  const uint32_t addr = smem_u32(p);
  return p + ((1024u - (addr & 1023u)) & 1023u);
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// Tiled TMA store of one box from this CTA's shared memory into global
// memory, tracked by the issuing thread's bulk async-groups.  Elements of the
// box outside the tensor are not written.  The shared source must have been
// made visible to the async proxy (fence_proxy_async_smem) by the threads
// that wrote it.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int32_t c0,
                                             int32_t c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem_src, int32_t c0, int32_t c1,
                                             int32_t c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}

// 1D bulk copy global -> this CTA's shared memory, counted on `bar`.  Both
// addresses 16-byte aligned, `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gmem_src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Closes the issuing thread's outstanding bulk stores into one group (an
// empty group when there are none).
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Waits until at most N of the thread's most recent bulk groups still read
// their shared-memory source (the older ones' sources may be overwritten).
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Waits until all of the thread's bulk groups have completed (their global
// writes performed).
__device__ __forceinline__ void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void prefetch_tensor_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void umma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16.  A (M x 16) sits in TMEM with
// row m in lane m and two bf16 values per 32-bit column (element k in column
// k/2, even k in the low half).
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05.mma issued so far by this thread
// has completed (implies tcgen05.fence::before_thread_sync).
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Each thread of the warp reads 32 consecutive 32-bit columns of its own lane.
__device__ __forceinline__ void tmem_ld_32cols(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
      " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31},"
      " [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st_32cols(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32"
      " [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16,"
      " %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st_16cols(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32"
      " [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// Shared-memory matrix descriptor for a tile stored with the 128-byte swizzle
// that TMA writes for a box whose inner extent is 128 bytes: rows of 128 B,
// eight-row atoms of 1024 B.  `smem_addr` must lie in a 1024-byte aligned
// atom; moving along K inside the 128-byte row is done by adding the byte
// offset to the start address.
//  K-major operand  (rows = M or N, 128 B of K per row):  SBO = 1024 B.
//  MN-major operand (rows = K, 64 MN elements per row):   SBO = 1024 B between
//  groups of eight K rows; LBO is the distance between 64-element MN blocks.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr, uint32_t lbo_bytes,
                                               uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(2) << 61;  // 128-byte swizzle
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 accumulation.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n, bool a_mn_major,
                                                       bool b_mn_major) {
  return (1u << 4)                                   // D format: f32
         | (1u << 7)                                 // A format: bf16
         | (1u << 10)                                // B format: bf16
         | (static_cast<uint32_t>(a_mn_major) << 15)  // A major
         | (static_cast<uint32_t>(b_mn_major) << 16)  // B major
         | (static_cast<uint32_t>(n >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);    // M / 16
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------- CTA pairs
// Building blocks for kernels launched as clusters of two CTAs whose tensor
// cores act as one (tcgen05 .cta_group::2): the even CTA of the pair (rank 0)
// issues the MMAs, which read both CTAs' shared memory at the same offsets and
// write both CTAs' TMEM.  Every tcgen05 instruction of such a kernel uses
// .cta_group::2.

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of this CTA's shared variable `ptr` in the shared memory of CTA
// `rank` of the cluster (a .shared::cluster address).
__device__ __forceinline__ uint32_t peer_smem_addr(const void* ptr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(ptr)), "r"(rank));
  return r;
}

// Arrive (release at cluster scope) on an mbarrier given by its cluster address.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// All threads of every CTA of the cluster.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// TMA tile load into this CTA's shared memory whose completion is counted on
// an mbarrier of the pair's leader CTA (bar_cluster_addr from peer_smem_addr).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster_addr, int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(c0), "r"(c1)
      : "memory");
}

// One warp in each CTA of the pair executes these together.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D (+)= A * B^T over the pair: M = 256 (rows 0..127 from the leader's A tile,
// 128..255 from the peer's), N columns split between the CTAs' B tiles; each
// CTA's TMEM receives its 128 rows.  Issued by one thread of the leader.
__device__ __forceinline__ void umma_bf16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                  uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on the mbarrier at this offset in every CTA of `cta_mask` when
// all MMAs issued so far by this thread have completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Two fp32 lanes in one 64-bit register, for the packed f32x2 FMA/ADD pipes.
__device__ __forceinline__ uint64_t f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ float2 unpack_f32x2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}

__device__ __forceinline__ uint64_t sub_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^x for a pair of fp32 values on the FMA pipe instead of MUFU, so that the
// softmax can split its exponentials between the two pipes.
// Method: Cody-Waite style range reduction x = n + f with n = round(x) and
// f in [-1/2, 1/2], then 2^f from a degree-3 polynomial and 2^n by adding n
// to the exponent field.  n is found with the round-to-nearest "magic number"
// addition: 1.5 * 2^23 + x holds round(x) in its low mantissa bits, so
// (bits << 23) is n << 23 modulo 2^32.  The polynomial
//     p(f) = 1 + f (c1 + f (c2 + f c3))
// is a relative-error minimax fit of 2^f on [-1/2, 1/2] with p(0) = 1 exactly
// (coefficients fitted for this library; max relative error 1.0e-4, well
// under the bf16 rounding of P).  Inputs are clamped to [-127, inf): at -127
// the result is exactly +0 (p(0) = 1 and n = -127 cancel the exponent bias),
// so masked (-inf) scores give p = 0 as with ex2; above -127 every result is
// a non-negative finite float.  Callers keep x <= 8 (the softmax slack).
__device__ __forceinline__ void exp2_poly_f32x2(uint64_t x2, float& r0, float& r1) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  constexpr float kC1 = 0.6932829022407532f;
  constexpr float kC2 = 0.24221037328243256f;
  constexpr float kC3 = 0.05500858277082443f;
  const float2 xv = unpack_f32x2(x2);
  const uint64_t x = f32x2(fmaxf(xv.x, -127.0f), fmaxf(xv.y, -127.0f));
  const uint64_t t = add_f32x2(x, f32x2(kMagic, kMagic));
  const uint64_t n = sub_f32x2(t, f32x2(kMagic, kMagic));
  const uint64_t f = sub_f32x2(x, n);
  uint64_t p = fma_f32x2(f32x2(kC3, kC3), f, f32x2(kC2, kC2));
  p = fma_f32x2(p, f, f32x2(kC1, kC1));
  p = fma_f32x2(p, f, f32x2(1.0f, 1.0f));
  const float2 tv = unpack_f32x2(t);
  const float2 pv = unpack_f32x2(p);
  uint32_t b0, b1;
  asm("mad.lo.u32 %0, %1, 8388608, %2;" : "=r"(b0) : "r"(__float_as_uint(tv.x)), "r"(__float_as_uint(pv.x)));
  asm("mad.lo.u32 %0, %1, 8388608, %2;" : "=r"(b1) : "r"(__float_as_uint(tv.y)), "r"(__float_as_uint(pv.y)));
  r0 = __uint_as_float(b0);
  r1 = __uint_as_float(b1);
}

// exp2 of two fp32 values, rounded to bf16 on the way in and computed by one
// MUFU operation for the pair; returns the packed bf16x2 (lo in bits 0..15).
__device__ __forceinline__ uint32_t exp2_bf16x2(uint64_t x) {
  const float2 v = unpack_f32x2(x);
  uint32_t packed, e;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(packed) : "f"(v.y), "f"(v.x));
  asm("ex2.approx.ftz.bf16x2 %0, %1;" : "=r"(e) : "r"(packed));
  return e;
}

// The two bf16 halves of a packed pair as an fp32 pair (exact widening).
__device__ __forceinline__ uint64_t bf16x2_to_f32x2(uint32_t v) {
  return f32x2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}

__device__ __forceinline__ void st_global_v4(void* ptr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(ptr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

}  // namespace b200tx
