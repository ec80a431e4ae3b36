// gemm_rownorm_kernels.cuh -- the projection that closes a block branch fused
// with the residual add and LayerNorm after it, for d_model 512, 768 and 1024,
// on the tcgen05 tensor cores:
//     u = round(x[rows, K] . w[cols, K]^T + bias)     (to the unfused program's update dtype)
//     r = residual_in + u;  normed = LayerNorm(r) * gamma + beta;  residual_out = r
// Replaces, for these widths, the reference's fused Linear residual-norm
// boundary (solution/kernels/boundary/triton_linear_residual_norm.py:33-112,
// built there for D 32 and 128) and, in the unfused program, the out-projection
// or FFN-out GEMM followed by the residual LayerNorm: the update never goes to
// memory, and the LayerNorm's loads and stores overlap the next tile's GEMM.
//
// A tile is 256 rows x all `cols` columns, computed by a cluster of
// 2 * P CTAs (P = cols / 256: clusters of 4, 6 or 8).  CTAs 2p and 2p+1 form a
// tensor-core pair (tcgen05 .cta_group::2, as the CTA-pair GEMM) computing
// columns [256p, 256p + 256) of all 256 rows: M = 256, N = 256 UMMAs whose A
// operand is the pair's two 128-row halves of x and whose B operand is the
// pair's two 128-row halves of w; CTA 2p + h holds rows [128h, 128h + 128) of
// the tile x the pair's 256 columns in its TMEM, in one of two accumulator
// stages (2 x 256 fp32 columns), so the epilogue of a tile runs while the
// pair's next tile accumulates.
//   warp 0       TMA: per 64-wide K slab, this CTA's 128 rows of x and 128
//                rows of w into a 4-stage ring (completion counted on the pair
//                leader's barrier, as the CTA-pair GEMM)
//   warp 1       in the pair leader, one thread issues the UMMAs
//   warps 2..9   epilogue, warp w reading TMEM lane quarter w % 4 (32 rows) and
//                column half (w - 2) / 4 (128 columns), one row per thread, in
//                32-column chunks staged through two 32 x 32 shared-memory
//                boxes per warp: TMA fills them with residual_in (pulled into
//                L2 one tile ahead); residual_out and normed are written into
//                them a row per lane and leave as whole 128-byte rows (8 lanes
//                a row), so that global memory is touched in whole lines.
//                Per tile:
//                pass 1: v = residual + round(acc + bias), written back over
//                        the accumulator in TMEM, and the (mean, M2) of the
//                        thread's 128 values (per 32-value chunk two passes over
//                        registers, chunks merged by Chan, Golub and LeVeque's
//                        pairwise update), handed to the exchange warp;
//                pass 2: residual_out = v, while the partials travel;
//                pass 3: normed = (v - mean) * rstd * gamma + beta; the
//                        accumulator stage is released once its last columns
//                        are in registers.
//   warp 10      exchange: the CTA's 256 partial (mean, M2) of a tile go to
//                slot [tile parity][p] of every CTA holding the same rows
//                (DSMEM stores), then one arrival (release, cluster scope) on
//                each one's barrier, made by P lanes at once.  Each CTA combines
//                the 2P partials of a row in the same order, so the CTAs of a
//                row agree bit for bit on its mean and variance.
// Measured (B200, 16384 rows): 49 us against 56 us for the out-projection GEMM
// plus residual LayerNorm at d_model 768 (K 768), 71 against 73 us at 1024
// (K 1024); slower than the unfused pair at K 3072-4096, where the GEMM alone
// runs at 1.5 PFLOP/s on 148 SMs while clusters of 8 CTAs occupy only 120.
// Padding-row modes as b200tx_residual_layer_norm_masked.  Every wait is
// bounded; a cluster barrier keeps all CTAs alive until the cluster is done.
#pragma once

#include "norm_kernels.cuh"
#include "sm100_common.cuh"

namespace b200tx {

constexpr int kRnBM = 256;  // rows per cluster tile (128 per CTA of a pair)
constexpr int kRnBN = 256;  // output columns per CTA pair
constexpr int kRnBK = 64;
constexpr int kRnStages = 4;
constexpr int kRnThreads = 352;
constexpr int kRnExchangeWarp = 10;
constexpr int kRnEpilogueThreads = 256;
constexpr int kRnMaxPairs = 4;           // d_model up to 1024 (a cluster of 8)
constexpr uint32_t kRnTmemCols = 512;    // two 256-column accumulator stages
constexpr uint32_t kRnTileBytes = 128 * kRnBK * 2;  // 16 KB: 128 rows of x or of w
constexpr uint32_t kRnStageBytes = 2 * kRnTileBytes;
constexpr uint32_t kRnBoxBytes = 32 * 32 * 4;       // one 32 x 32 staging box (fp32 at most)
constexpr uint32_t kRnStagingBytes = 8 * 2 * kRnBoxBytes;  // two boxes per epilogue warp: 64 KB
constexpr size_t kRnSmemBytes = 1024 + kRnStages * kRnStageBytes + kRnStagingBytes;  // 193 KB

struct RowNormArgs {
  const float* bias;         // [cols]
  const float* gamma;        // [cols]
  const float* beta;         // [cols]
  const uint8_t* row_valid;  // [rows] or null
  float* residual_out;       // [rows, cols] fp32, or null
  void* normed;              // [rows, cols] OutT
  int mask_mode;             // kNormMask* bits for rows whose flag is 0
  int rows, cols, inner;     // M, N (= d_model), K
  int pairs;                 // cols / 256 = CTA pairs per cluster
  int num_tiles;             // ceil(rows / 256)
  int round_update_bf16;     // the unfused program stores the update in bf16
  float eps;
};

__device__ __forceinline__ void st_shared_cluster_f32x4(uint32_t cluster_addr, float4 v) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

__device__ __forceinline__ float4 ld_shared_f32x4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// mbar_wait with acquire at cluster scope: the phase was completed by
// arrivals (release at cluster scope) of other CTAs of the cluster, whose
// shared-memory stores into this CTA must be visible after the wait.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, unsigned int code,
                                                  volatile int* abort_flag) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const unsigned long long start = global_timer_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait_cluster(bar, parity)) {
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

// Pulls one box of a tiled tensor into L2 (no shared memory, no completion).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int32_t c0, int32_t c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1)
               : "memory");
}

// Relaxed arrive on an mbarrier given by its cluster address: for a signal
// whose data dependency the caller has already enforced (the TMEM reads of an
// accumulator stage, completed by tcgen05.wait::ld), without a release that
// would wait for the thread's outstanding global stores.
__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// One row (this lane's) of a 32 x 32 staging box: 32 values of type T at
// 32 * sizeof(T) bytes per row, in the TMA's swizzled layout (128-byte rows:
// 16-byte chunk j at j ^ (row % 8); 64-byte rows: j ^ ((row / 2) % 4)).
template <typename T>
struct BoxRow;

template <>
struct BoxRow<float> {
  static __device__ __forceinline__ void load(uint32_t box, int row, float (&v)[32]) {
    const uint32_t base = box + static_cast<uint32_t>(row) * 128u;
    const uint32_t swz = static_cast<uint32_t>(row) & 7u;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 q = ld_shared_f32x4(base + ((static_cast<uint32_t>(j) ^ swz) << 4));
      v[4 * j] = q.x;
      v[4 * j + 1] = q.y;
      v[4 * j + 2] = q.z;
      v[4 * j + 3] = q.w;
    }
  }
  static __device__ __forceinline__ void store(uint32_t box, int row, const float (&v)[32]) {
    const uint32_t base = box + static_cast<uint32_t>(row) * 128u;
    const uint32_t swz = static_cast<uint32_t>(row) & 7u;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      st_shared_v4(base + ((static_cast<uint32_t>(j) ^ swz) << 4), __float_as_uint(v[4 * j]),
                   __float_as_uint(v[4 * j + 1]), __float_as_uint(v[4 * j + 2]), __float_as_uint(v[4 * j + 3]));
  }
  static __device__ __forceinline__ void store_bits(uint32_t box, int row, const uint32_t (&v)[32]) {
    const uint32_t base = box + static_cast<uint32_t>(row) * 128u;
    const uint32_t swz = static_cast<uint32_t>(row) & 7u;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      st_shared_v4(base + ((static_cast<uint32_t>(j) ^ swz) << 4), v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
  // The whole box to rows [row0, row0 + 32) x columns [col, col + 32) of a
  // row-major matrix: per instruction 8 lanes a row, 4 whole 128-byte rows.
  static __device__ __forceinline__ void to_global(uint32_t box, int lane, float* out, int64_t row0, int rows,
                                                   int cols, int col) {
    const int chunk = lane & 7;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int r = k * 4 + (lane >> 3);
      const float4 q =
          ld_shared_f32x4(box + static_cast<uint32_t>(r) * 128u + ((static_cast<uint32_t>(chunk ^ (r & 7))) << 4));
      if (row0 + r < rows)
        st_global_v4(out + (row0 + r) * cols + col + chunk * 4, __float_as_uint(q.x), __float_as_uint(q.y),
                     __float_as_uint(q.z), __float_as_uint(q.w));
    }
  }
};

template <>
struct BoxRow<__nv_bfloat16> {
  static __device__ __forceinline__ void load(uint32_t box, int row, float (&v)[32]) {
    const uint32_t base = box + static_cast<uint32_t>(row) * 64u;
    const uint32_t swz = (static_cast<uint32_t>(row) >> 1) & 3u;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 q = ld_shared_f32x4(base + ((static_cast<uint32_t>(j) ^ swz) << 4));
      const uint32_t w[4] = {__float_as_uint(q.x), __float_as_uint(q.y), __float_as_uint(q.z), __float_as_uint(q.w)};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[8 * j + 2 * i] = __uint_as_float(w[i] << 16);
        v[8 * j + 2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      }
    }
  }
  static __device__ __forceinline__ void store(uint32_t box, int row, const float (&v)[32]) {
    const uint32_t base = box + static_cast<uint32_t>(row) * 64u;
    const uint32_t swz = (static_cast<uint32_t>(row) >> 1) & 3u;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      st_shared_v4(base + ((static_cast<uint32_t>(j) ^ swz) << 4), pack_bf16x2(v[8 * j], v[8 * j + 1]),
                   pack_bf16x2(v[8 * j + 2], v[8 * j + 3]), pack_bf16x2(v[8 * j + 4], v[8 * j + 5]),
                   pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
  }
  // As BoxRow<float>::to_global for 64-byte rows: 4 lanes a row, 8 rows per instruction.
  static __device__ __forceinline__ void to_global(uint32_t box, int lane, __nv_bfloat16* out, int64_t row0,
                                                   int rows, int cols, int col) {
    const int chunk = lane & 3;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int r = k * 8 + (lane >> 2);
      const float4 q = ld_shared_f32x4(box + static_cast<uint32_t>(r) * 64u +
                                       ((static_cast<uint32_t>(chunk ^ ((r >> 1) & 3))) << 4));
      if (row0 + r < rows)
        st_global_v4(out + (row0 + r) * cols + col + chunk * 8, __float_as_uint(q.x), __float_as_uint(q.y),
                     __float_as_uint(q.z), __float_as_uint(q.w));
    }
  }
};

template <typename InT, typename OutT>
__global__ void __launch_bounds__(kRnThreads, 1)
    gemm_residual_layernorm_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                   const __grid_constant__ CUtensorMap tmap_w,
                                   const __grid_constant__ CUtensorMap tmap_rin, RowNormArgs args) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full_bar[kRnStages];
  __shared__ uint64_t empty_bar[kRnStages];
  __shared__ uint64_t acc_full_bar[2];
  __shared__ uint64_t acc_empty_bar[2];
  __shared__ uint64_t box_bar[8][2];  // residual_in box of each epilogue warp landed
  __shared__ uint64_t stat_ready;     // this CTA's partial statistics of the tile written (8 warps)
  __shared__ uint64_t stat_bar;       // the rows' partial statistics of every CTA present
  __shared__ uint64_t drain_bar;
  // Partial (mean, M2) of 128 columns of a row: [tile parity][pair][column half][row].
  // 16-byte aligned: the exchange warp moves them in 16-byte vectors.
  __shared__ __align__(16) float2 stat_part[2][kRnMaxPairs][2][128];
  __shared__ __align__(16) float2 stat_local[2][128];  // this CTA's partials of the tile: [column half][row]
  __shared__ __align__(16) float col_bias[kRnBN];  // read as float4
  __shared__ __align__(16) float col_gamma[kRnBN];
  __shared__ __align__(16) float col_beta[kRnBN];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  uint8_t* smem = align_1024(smem_raw);
  uint8_t* smem_a = smem;
  uint8_t* smem_w = smem + kRnStages * kRnTileBytes;
  uint8_t* smem_boxes = smem + kRnStages * kRnStageBytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t half = rank & 1u;                 // rows [128 half, 128 half + 128) of a tile
  const int pair_idx = static_cast<int>(rank >> 1);  // columns [256 pair_idx, ...)
  const bool leader = half == 0;
  const int pairs = args.pairs;
  const int cluster_ctas = 2 * pairs;
  const int cluster_id = static_cast<int>(blockIdx.x) / cluster_ctas;
  const int num_clusters = static_cast<int>(gridDim.x) / cluster_ctas;
  const int col_base = pair_idx * kRnBN;
  const int num_kb = (args.inner + kRnBK - 1) / kRnBK;
  const uint16_t pair_mask = static_cast<uint16_t>(0x3u << (2 * pair_idx));

  if (threadIdx.x == 0) {
    prefetch_tensor_map(&tmap_x);
    prefetch_tensor_map(&tmap_w);
    prefetch_tensor_map(&tmap_rin);
    for (int s = 0; s < kRnStages; ++s) {
      mbar_init(&full_bar[s], 1);  // the leader's arrive.expect_tx
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full_bar[a], 1);
      mbar_init(&acc_empty_bar[a], 16);  // 8 epilogue warps in each CTA of the pair
    }
    for (int w = 0; w < 8; ++w) {
      mbar_init(&box_bar[w][0], 1);
      mbar_init(&box_bar[w][1], 1);
    }
    mbar_init(&stat_ready, kRnEpilogueThreads / 32);
    mbar_init(&stat_bar, pairs);  // one arrival from the exchange warp of each CTA of the rows
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&tmem_slot, kRnTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  // Every CTA's barriers are initialised before any CTA arrives remotely.
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      const uint32_t full_leader_base = peer_smem_addr(&full_bar[0], rank & ~1u);
      for (int tile = cluster_id; tile < args.num_tiles && !abort_flag; tile += num_clusters) {
        const int a_row = tile * kRnBM + static_cast<int>(half) * 128;
        const int w_row = col_base + static_cast<int>(half) * 128;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, kErrGemmProducerWait, &abort_flag)) break;
          if (leader) {
            mbar_arrive_expect_tx(&full_bar[stage], 2 * kRnStageBytes);
            tma_load_2d(smem_a + stage * kRnTileBytes, &tmap_x, &full_bar[stage], kb * kRnBK, a_row);
            tma_load_2d(smem_w + stage * kRnTileBytes, &tmap_w, &full_bar[stage], kb * kRnBK, w_row);
          } else {
            const uint32_t full_leader = full_leader_base + stage * static_cast<uint32_t>(sizeof(uint64_t));
            tma_load_2d_pair(smem_a + stage * kRnTileBytes, &tmap_x, full_leader, kb * kRnBK, a_row);
            tma_load_2d_pair(smem_w + stage * kRnTileBytes, &tmap_w, full_leader, kb * kRnBK, w_row);
          }
          ++issued;
          if (++stage == kRnStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // The leader waits for the pair's last loads (complete already on the
      // normal path) so that no TMA write is in flight when the pair leaves.
      if (leader) {
        const int outstanding = issued < kRnStages ? issued : kRnStages;
        for (int i = 0; i < outstanding; ++i) {
          if (--stage < 0) {
            stage = kRnStages - 1;
            phase ^= 1u;
          }
          mbar_drain_wait(&full_bar[stage], phase);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (leader && elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16(kRnBM, kRnBN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int t = 0;
      bool issued_any = false;
      for (int tile = cluster_id; tile < args.num_tiles && !abort_flag; tile += num_clusters, ++t) {
        const int acc = t & 1;
        const uint32_t acc_phase = (t >> 1) & 1;
        if (!mbar_wait(&acc_empty_bar[acc], acc_phase ^ 1u, kErrGemmMmaWait, &abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kRnBN;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, kErrGemmMmaWait, &abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem_a + stage * kRnTileBytes);
          const uint32_t w_addr = smem_u32(smem_w + stage * kRnTileBytes);
#pragma unroll
          for (int k = 0; k < kRnBK / 16; ++k) {
            umma_bf16_ss_pair(d_tmem, sw128_desc(a_addr + k * 32, 16, 1024),
                              sw128_desc(w_addr + k * 32, 16, 1024), idesc, (kb | k) != 0 ? 1u : 0u);
          }
          issued_any = true;
          umma_commit_pair(&empty_bar[stage], pair_mask);
          if (++stage == kRnStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(&acc_full_bar[acc], pair_mask);
      }
      if (issued_any) {
        umma_commit_pair(&drain_bar, static_cast<uint16_t>(1u << (2 * pair_idx)));
        mbar_drain_wait(&drain_bar, 0);
      }
    }
  } else if (warp == kRnExchangeWarp) {
    // ------------------------------------------------------------ exchange
    // Per tile: this CTA's 256 partial (mean, M2) from the epilogue warps to
    // slot [tile parity][pair_idx] of every CTA holding the same rows (ranks
    // 2p + half), then one arrival (release, cluster scope) on each one's
    // barrier, made by P lanes at once.  The arrivals wait for the stores to
    // land (about a microsecond while the pair MMAs load the SM-to-SM links);
    // this warp absorbs that wait, the epilogue warps meanwhile write v.
    // Two slot sets alternate by tile: a CTA that has passed tile t's
    // exchange may send tile t + 1's while the others still read t's.
    constexpr uint32_t kStatParityStride = kRnMaxPairs * 2 * 128 * sizeof(float2);
    uint32_t dst[kRnMaxPairs];
#pragma unroll
    for (int p = 0; p < kRnMaxPairs; ++p)
      dst[p] = peer_smem_addr(&stat_part[0][pair_idx][0][0], static_cast<uint32_t>(2 * (p < pairs ? p : 0)) + half);
    const uint32_t bar_mine = peer_smem_addr(&stat_bar, static_cast<uint32_t>(2 * (lane < pairs ? lane : 0)) + half);
    const float4* src = reinterpret_cast<const float4*>(&stat_local[0][0]) + lane * 4;  // 8 partials a lane
    int t = 0;
    for (int tile = cluster_id; tile < args.num_tiles; tile += num_clusters, ++t) {
      const bool ok = mbar_wait(&stat_ready, static_cast<uint32_t>(t) & 1u, kErrGemmEpilogueWait, &abort_flag);
      if (__any_sync(0xffffffffu, !ok)) break;
      float4 q[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) q[j] = src[j];
      const uint32_t off = static_cast<uint32_t>(t & 1) * kStatParityStride + static_cast<uint32_t>(lane) * 64u;
#pragma unroll
      for (int p = 0; p < kRnMaxPairs; ++p) {
        if (p < pairs) {
#pragma unroll
          for (int j = 0; j < 4; ++j) st_shared_cluster_f32x4(dst[p] + off + j * 16, q[j]);
        }
      }
      __syncwarp();
      if (lane < pairs) mbar_arrive_cluster(bar_mine);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;  // epilogue warp 0..7
    const int quarter = warp & 3;
    const int ch = ew >> 2;   // column half: 128 of the pair's 256 columns
    const int row_in_cta = quarter * 32 + lane;
    uint8_t* const box_ptr = smem_boxes + ew * 2 * kRnBoxBytes;
    const uint32_t box0 = smem_u32(box_ptr);
    const uint32_t box1 = box0 + kRnBoxBytes;
    const int col_warp = col_base + ch * 128;  // first column of this warp
    constexpr uint32_t kInBoxBytes = 32 * 32 * sizeof(InT);
    OutT* const normed = static_cast<OutT*>(args.normed);
    // Column constants of the pair's 256 columns, staged once.
    for (int i = static_cast<int>(threadIdx.x) - 64; i < kRnBN; i += kRnEpilogueThreads) {
      col_bias[i] = args.bias != nullptr ? __ldg(args.bias + col_base + i) : 0.f;
      col_gamma[i] = __ldg(args.gamma + col_base + i);
      col_beta[i] = __ldg(args.beta + col_base + i);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kRnEpilogueThreads) : "memory");
    // This thread's partial statistics go to slot [parity][pair_idx][ch][row]
    // of every CTA that holds these rows (ranks 2p + half) and arrive on that
    // CTA's barrier.  Two slot sets alternate by tile: a CTA that has passed
    // tile t's exchange may write tile t + 1's while the others still read t's.

    const uint32_t acc_empty_leader0 = peer_smem_addr(&acc_empty_bar[0], rank & ~1u);
    const uint32_t acc_empty_leader1 = peer_smem_addr(&acc_empty_bar[1], rank & ~1u);
    const float inv_cols = 1.0f / static_cast<float>(args.cols);  // M2 -> variance
    // residual_in boxes: loads issued (by lane 2) and waited (by all lanes) per
    // box.  Lane 0 makes the accumulator and exchange arrivals, lane 1 the L2
    // prefetches, so that none of them queues behind another.
    constexpr int kBoxLane = 2;
    int box_loads[2] = {0, 0};
    int box_waits[2] = {0, 0};
    auto load_box = [&](int b, int tile, int chunk) {
      if (lane == kBoxLane) {
        uint64_t* bar = &box_bar[ew][b];
        mbar_arrive_expect_tx(bar, kInBoxBytes);
        tma_load_2d(box_ptr + b * kRnBoxBytes, &tmap_rin, bar, col_warp + chunk * 32,
                    tile * kRnBM + static_cast<int>(half) * 128 + quarter * 32);
      }
      ++box_loads[b];
    };
    // L2 prefetch of a tile's residual boxes of this warp.
    auto prefetch_tile = [&](int tile, int first_chunk) {
      if (lane == 1 && tile < args.num_tiles)
        for (int c = first_chunk; c < 4; ++c)
          tma_prefetch_l2_2d(&tmap_rin, col_warp + c * 32, tile * kRnBM + static_cast<int>(half) * 128 + quarter * 32);
    };
    if (cluster_id < args.num_tiles) {
      load_box(0, cluster_id, 0);
      load_box(1, cluster_id, 1);
      prefetch_tile(cluster_id, 2);
    }
    bool ok = true;
    int t = 0;
    for (int tile = cluster_id; tile < args.num_tiles; tile += num_clusters, ++t) {
      const int acc = t & 1;
      const uint32_t acc_phase = (t >> 1) & 1;
      const int row0 = tile * kRnBM + static_cast<int>(half) * 128 + quarter * 32;  // the warp's first row
      const int64_t row = static_cast<int64_t>(row0) + lane;
      const bool in_range = row < args.rows;
      const bool valid = !in_range || args.row_valid == nullptr || args.row_valid[row] != 0;
      const bool add_update = valid || !(args.mask_mode & kNormMaskDropUpdate);
      const bool zero_residual = !valid && (args.mask_mode & kNormMaskZeroResidual);
      const bool zero_normed = !valid && (args.mask_mode & kNormMaskZeroNormed);
      // The next tile's residual travels to L2 while this one is processed.
      prefetch_tile(tile + num_clusters, 0);
      ok = mbar_wait(&acc_full_bar[acc], acc_phase, kErrGemmEpilogueWait, &abort_flag);
      if (__any_sync(0xffffffffu, !ok)) {
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kRnBN + ch * 128;
      // Pass 1: v = residual + round(acc + bias) over the accumulator, and the
      // statistics of this thread's 128 values: per 32-value chunk the mean and
      // the sum of squared deviations (two passes over registers), merged
      // chunk by chunk (Chan, Golub and LeVeque's pairwise update).
      float mean = 0.f, m2 = 0.f;
      uint32_t accv[2][32];
      tmem_ld_32cols(taddr, accv[0]);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int b = c & 1;
        ok = mbar_wait(&box_bar[ew][b], static_cast<uint32_t>(box_waits[b]) & 1u, kErrGemmEpilogueWait,
                       &abort_flag);
        if (ok) ++box_waits[b];  // a load not seen to land is drained before the CTA leaves
        float r[32];
        BoxRow<InT>::load(b ? box1 : box0, lane, r);
        tmem_wait_ld();
        if (__any_sync(0xffffffffu, !ok)) {
          ok = false;
          break;
        }
        if (c + 2 < 4) {
          // The box has been read: refill it with chunk c + 2.
          fence_proxy_async_smem();
          __syncwarp();
          load_box(b, tile, c + 2);
        }
        if (c + 1 < 4) tmem_ld_32cols(taddr + (c + 1) * 32, accv[(c + 1) & 1]);
        const float4* bias4 = reinterpret_cast<const float4*>(col_bias + ch * 128 + c * 32);
        float csum = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 bb = bias4[q];
          float u0 = __uint_as_float(accv[c & 1][4 * q]) + bb.x;
          float u1 = __uint_as_float(accv[c & 1][4 * q + 1]) + bb.y;
          float u2 = __uint_as_float(accv[c & 1][4 * q + 2]) + bb.z;
          float u3 = __uint_as_float(accv[c & 1][4 * q + 3]) + bb.w;
          if (args.round_update_bf16) {
            const __nv_bfloat162 lo = __floats2bfloat162_rn(u0, u1);
            const __nv_bfloat162 hi = __floats2bfloat162_rn(u2, u3);
            u0 = __low2float(lo);
            u1 = __high2float(lo);
            u2 = __low2float(hi);
            u3 = __high2float(hi);
          }
          const float u[4] = {u0, u1, u2, u3};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float rv = r[4 * q + e];
            r[4 * q + e] = zero_residual ? 0.f : (add_update ? rv + u[e] : rv);
            csum += r[4 * q + e];
          }
        }
        uint32_t vbits[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) vbits[i] = __float_as_uint(r[i]);
        tmem_st_32cols(taddr + c * 32, vbits);
        const float cmean = csum * (1.0f / 32.0f);
        float cm2 = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float d = r[i] - cmean;
          cm2 = fmaf(d, d, cm2);
        }
        if (c == 0) {
          mean = cmean;
          m2 = cm2;
        } else {
          // n = 32c values so far, 32 more: weights 1/(c+1) and 32c/(c+1).
          const float delta = cmean - mean;
          const float inv = 1.0f / static_cast<float>(c + 1);
          mean = fmaf(delta, inv, mean);
          m2 += cm2 + delta * delta * (32.0f * static_cast<float>(c) * inv);
        }
      }
      if (!ok) break;
      tmem_wait_st();
      // Hand this thread's (mean, M2) to the exchange warp, and write
      // residual_out = v while the partials travel to the row's CTAs.
      stat_local[ch][row_in_cta] = make_float2(mean, m2);
      __syncwarp();
      if (lane == 0) mbar_arrive(&stat_ready);
      if (args.residual_out != nullptr) {
        uint32_t vv[2][32];
        tmem_ld_32cols(taddr, vv[0]);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          tmem_wait_ld();
          if (c + 1 < 4) tmem_ld_32cols(taddr + (c + 1) * 32, vv[(c + 1) & 1]);
          const uint32_t box = (c & 1) ? box1 : box0;
          __syncwarp();  // the reads of this box two chunks ago are done
          BoxRow<float>::store_bits(box, lane, vv[c & 1]);
          __syncwarp();
          BoxRow<float>::to_global(box, lane, args.residual_out, row0, args.rows, args.cols, col_warp + c * 32);
        }
      }
      const int par = t & 1;
      ok = mbar_wait_cluster(&stat_bar, static_cast<uint32_t>(t) & 1u, kErrGemmEpilogueWait, &abort_flag);
      if (__any_sync(0xffffffffu, !ok)) {
        ok = false;
        break;
      }
      // Every CTA of the row combines the partials in the same order, so they
      // agree bit for bit: mean of the means, M2 = sum M2_i + 128 sum (mean_i - mean)^2.
      float2 part[kRnMaxPairs][2];
      float msum = 0.f;
#pragma unroll
      for (int p = 0; p < kRnMaxPairs; ++p) {
        if (p < pairs) {
          part[p][0] = stat_part[par][p][0][row_in_cta];
          part[p][1] = stat_part[par][p][1][row_in_cta];
          msum += part[p][0].x + part[p][1].x;
        }
      }
      const float row_mean = msum / static_cast<float>(2 * pairs);
      float row_m2 = 0.f, spread = 0.f;
#pragma unroll
      for (int p = 0; p < kRnMaxPairs; ++p) {
        if (p < pairs) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float d = part[p][h].x - row_mean;
            row_m2 += part[p][h].y;
            spread = fmaf(d, d, spread);
          }
        }
      }
      const float rstd = rsqrtf(fmaf(spread, 128.0f, row_m2) * inv_cols + args.eps);
      // Pass 2: normed, each chunk through a box (one row per lane, boxes
      // alternating) and out to global memory in whole rows.
      uint32_t vv[2][32];
      tmem_ld_32cols(taddr, vv[0]);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tmem_wait_ld();
        if (c + 1 < 4) {
          tmem_ld_32cols(taddr + (c + 1) * 32, vv[(c + 1) & 1]);
        } else {
          // Every column of the accumulator stage this warp reads is in
          // registers: release the stage to the pair's MMA issuer.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster_relaxed(acc ? acc_empty_leader1 : acc_empty_leader0);
        }
        const float4* gamma4 = reinterpret_cast<const float4*>(col_gamma + ch * 128 + c * 32);
        const float4* beta4 = reinterpret_cast<const float4*>(col_beta + ch * 128 + c * 32);
        float n[32];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 gg = gamma4[q];
          const float4 bb = beta4[q];
          const float g[4] = {gg.x, gg.y, gg.z, gg.w};
          const float be[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
          for (int e = 0; e < 4; ++e)
            n[4 * q + e] =
                zero_normed ? 0.f : (__uint_as_float(vv[c & 1][4 * q + e]) - row_mean) * rstd * g[e] + be[e];
        }
        const uint32_t box = (c & 1) ? box1 : box0;
        __syncwarp();  // the reads of this box two chunks ago are done
        BoxRow<OutT>::store(box, lane, n);
        __syncwarp();
        BoxRow<OutT>::to_global(box, lane, normed, row0, args.rows, args.cols, col_warp + c * 32);
      }
      // The next tile's first two residual boxes (the boxes' generic reads and
      // writes are ordered before the TMA writes).
      const int next = tile + num_clusters;
      if (next < args.num_tiles) {
        fence_proxy_async_smem();
        __syncwarp();
        load_box(0, next, 0);
        load_box(1, next, 1);
      }
    }
    // No box load in flight when the CTA leaves.
    if (lane == kBoxLane) {
      for (int b = 0; b < 2; ++b)
        for (; box_waits[b] < box_loads[b]; ++box_waits[b])
          mbar_drain_wait(&box_bar[ew][b], static_cast<uint32_t>(box_waits[b]) & 1u);
    }
    __syncwarp();
  }

  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kRnTmemCols);
  }
}

}  // namespace b200tx
