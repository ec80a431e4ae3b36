// norm_kernels.cuh -- residual add + LayerNorm + cast, one warp per row.
//
// Replaces the reference's residual/LayerNorm primitives:
//   initial LayerNorm      solution/kernels/norm/triton_initial.py:38-66
//   fp32 residual + LN     solution/kernels/norm/triton_residual.py:38-73
//   mixed residual + LN    solution/kernels/norm/triton_mixed_residual.py:40-77
// Semantics (official/torch_transformer_benchmark.py:125-145, nn.LayerNorm):
//   r = residual_in + update            (fp32)
//   n = (r - mean(r)) * rsqrt(var(r) + eps) * gamma + beta
// with the biased variance over the row, computed two-pass in registers.
//
// Padding masks (official/torch_transformer_benchmark.py:119-121, 143-144,
// 170-171): with `row_valid`, a row whose flag is 0 follows `mask_mode`:
//   kNormMaskDropUpdate   r = residual_in           (attention output zeroed)
//   kNormMaskZeroResidual r = 0                     (block output zeroed)
//   kNormMaskZeroNormed   normed = 0                (final output zeroed)
// The branch is per row, so uniform across the row's warp.
//
// Layout: row-major [rows, cols].  For cols % 128 == 0 (every BASELINE width)
// each lane owns cols/128 groups of four consecutive columns, so each warp
// instruction touches 512 contiguous bytes of fp32 (256 of bf16): 128-bit
// loads and stores, no shared memory, two butterfly reductions per row.
#pragma once

#include "sm100_common.cuh"

namespace b200tx {

constexpr int kNormMaskDropUpdate = 1;
constexpr int kNormMaskZeroResidual = 2;
constexpr int kNormMaskZeroNormed = 4;

struct NormArgs {
  const void* residual_in;  // [rows, cols] fp32 or bf16
  const void* update;       // [rows, cols] bf16 or fp32; null for a plain LayerNorm
  float* residual_out;      // [rows, cols] fp32; null when the sum is not kept
  void* normed;             // [rows, cols] bf16 or fp32
  const float* gamma;       // [cols]
  const float* beta;        // [cols]
  const uint8_t* row_valid; // [rows] 0/1 or null (every row valid)
  int mask_mode;            // kNormMask* bits applied to rows whose flag is 0
  int64_t rows;
  int cols;
  float eps;
};

// Which of the masked behaviours apply to this row.
struct RowMask {
  bool add_update;
  bool zero_residual;
  bool zero_normed;
};

__device__ __forceinline__ RowMask row_mask(const NormArgs& a, int64_t row) {
  const bool valid = a.row_valid == nullptr || a.row_valid[row] != 0;
  RowMask m;
  m.add_update = valid || !(a.mask_mode & kNormMaskDropUpdate);
  m.zero_residual = !valid && (a.mask_mode & kNormMaskZeroResidual);
  m.zero_normed = !valid && (a.mask_mode & kNormMaskZeroNormed);
  return m;
}

template <typename T>
__device__ __forceinline__ float4 load4(const T* base, int64_t idx);

template <>
__device__ __forceinline__ float4 load4<float>(const float* base, int64_t idx) {
  return __ldg(reinterpret_cast<const float4*>(base + idx));
}

template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* base, int64_t idx) {
  const uint2 raw = __ldg(reinterpret_cast<const uint2*>(base + idx));
  const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
  const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
  const float2 a = __bfloat1622float2(lo);
  const float2 b = __bfloat1622float2(hi);
  return make_float4(a.x, a.y, b.x, b.y);
}

template <typename T>
__device__ __forceinline__ void store4(T* base, int64_t idx, float4 v);

template <>
__device__ __forceinline__ void store4<float>(float* base, int64_t idx, float4 v) {
  *reinterpret_cast<float4*>(base + idx) = v;
}

template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* base, int64_t idx,
                                                      float4 v) {
  uint2 raw;
  raw.x = pack_bf16x2(v.x, v.y);
  raw.y = pack_bf16x2(v.z, v.w);
  *reinterpret_cast<uint2*>(base + idx) = raw;
}

template <typename T>
__device__ __forceinline__ float load1(const T* base, int64_t idx);
template <>
__device__ __forceinline__ float load1<float>(const float* base, int64_t idx) {
  return base[idx];
}
template <>
__device__ __forceinline__ float load1<__nv_bfloat16>(const __nv_bfloat16* base, int64_t idx) {
  return __bfloat162float(base[idx]);
}
template <typename T>
__device__ __forceinline__ void store1(T* base, int64_t idx, float v);
template <>
__device__ __forceinline__ void store1<float>(float* base, int64_t idx, float v) {
  base[idx] = v;
}
template <>
__device__ __forceinline__ void store1<__nv_bfloat16>(__nv_bfloat16* base, int64_t idx, float v) {
  base[idx] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int offset = 16; offset > 0; offset >>= 1) v += __shfl_xor_sync(0xffffffffu, v, offset);
  return v;
}

constexpr int kNormWarpsPerBlock = 8;

// Vectorised path: cols == 128 * NV.
template <int NV, typename InT, typename UpdT, typename OutT>
__global__ void __launch_bounds__(kNormWarpsPerBlock * 32)
    residual_layernorm_vec_kernel(NormArgs args) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kNormWarpsPerBlock + (threadIdx.x >> 5);
  griddep_wait();
  griddep_launch_dependents();
  if (row >= args.rows) return;
  const int cols = 128 * NV;
  const int64_t base = row * cols;
  const InT* rin = static_cast<const InT*>(args.residual_in);

  const RowMask mask = row_mask(args, row);
  float4 v[NV];
  if (mask.zero_residual) {
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  } else {
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = load4<InT>(rin, base + (i * 32 + lane) * 4);
    if constexpr (!std::is_same<UpdT, void>::value) {
      if (mask.add_update) {
        const UpdT* upd = static_cast<const UpdT*>(args.update);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          const float4 u = load4<UpdT>(upd, base + (i * 32 + lane) * 4);
          v[i].x += u.x;
          v[i].y += u.y;
          v[i].z += u.z;
          v[i].w += u.w;
        }
      }
    }
  }
  if (args.residual_out != nullptr) {
#pragma unroll
    for (int i = 0; i < NV; ++i) store4<float>(args.residual_out, base + (i * 32 + lane) * 4, v[i]);
  }

  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  const float mean = warp_sum(s) * (1.0f / cols);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
    q += (a * a + b * b) + (c * c + d * d);
  }
  const float var = warp_sum(q) * (1.0f / cols);
  const float rstd = rsqrtf(var + args.eps);

  OutT* out = static_cast<OutT*>(args.normed);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 4;
    const float4 g = __ldg(reinterpret_cast<const float4*>(args.gamma + c));
    const float4 b = __ldg(reinterpret_cast<const float4*>(args.beta + c));
    float4 o;
    o.x = (v[i].x - mean) * rstd * g.x + b.x;
    o.y = (v[i].y - mean) * rstd * g.y + b.y;
    o.z = (v[i].z - mean) * rstd * g.z + b.z;
    o.w = (v[i].w - mean) * rstd * g.w + b.w;
    if (mask.zero_normed) o = make_float4(0.f, 0.f, 0.f, 0.f);
    store4<OutT>(out, base + c, o);
  }
}

// Generic path for any width: three passes over the row in global memory
// (sum, centred sum of squares, normalise), still one warp per row.
template <typename InT, typename UpdT, typename OutT>
__global__ void __launch_bounds__(kNormWarpsPerBlock * 32)
    residual_layernorm_generic_kernel(NormArgs args) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kNormWarpsPerBlock + (threadIdx.x >> 5);
  griddep_wait();
  griddep_launch_dependents();
  if (row >= args.rows) return;
  const int cols = args.cols;
  const int64_t base = row * cols;
  const InT* rin = static_cast<const InT*>(args.residual_in);
  const UpdT* upd = static_cast<const UpdT*>(args.update);
  const RowMask mask = row_mask(args, row);
  auto value_at = [&](int c) -> float {
    if (mask.zero_residual) return 0.f;
    float x = load1<InT>(rin, base + c);
    if constexpr (!std::is_same<UpdT, void>::value) {
      if (mask.add_update) x += load1<UpdT>(upd, base + c);
    }
    return x;
  };
  float s = 0.f;
  for (int c = lane; c < cols; c += 32) s += value_at(c);
  const float mean = warp_sum(s) / cols;
  float q = 0.f;
  for (int c = lane; c < cols; c += 32) {
    const float d = value_at(c) - mean;
    q += d * d;
  }
  const float rstd = rsqrtf(warp_sum(q) / cols + args.eps);
  OutT* out = static_cast<OutT*>(args.normed);
  for (int c = lane; c < cols; c += 32) {
    const float x = value_at(c);
    // Every lane reads its own columns before writing them, so an in-place
    // residual update (residual_out == residual_in) stays exact.
    if (args.residual_out != nullptr) args.residual_out[base + c] = x;
    store1<OutT>(out, base + c,
                 mask.zero_normed ? 0.f : (x - mean) * rstd * args.gamma[c] + args.beta[c]);
  }
}

// ---------------------------------------------------------------------------
// Tensor-parallel reduction fused into the residual LayerNorm.  Each rank of a
// tensor-parallel group writes its partial sum of a row-parallel projection
// (out-proj, FFN-out) into a buffer its peers can read over NVLink; this
// kernel adds the partials of all `count` ranks (its own and the peers') to the
// residual and normalises, in one pass, so no separate all-reduce moves the
// partials.  Before reading, one thread per CTA waits until every peer has
// published the epoch (peer_signal_kernel after its GEMM) with a bounded
// acquire spin at system scope; a wait that runs out records
// kErrPeerWait and the CTA stops without writing.
// ---------------------------------------------------------------------------
constexpr int kMaxPeers = 8;

struct PeerSumArgs {
  const __nv_bfloat16* partials[kMaxPeers];  // [rows, cols] bf16, index = group rank
  int count;                                 // ranks in the group
  int self;                                  // this rank (its partial is local)
  const uint32_t* flags;                     // [count] local slots written by the peers
  uint32_t epoch;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait for every peer's epoch; one thread per CTA, then the CTA syncs.
__device__ __forceinline__ bool wait_peer_epoch(const PeerSumArgs& p) {
  __shared__ int ok_shared;
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned long long start = global_timer_ns();
    for (int r = 0; r < p.count && ok; ++r) {
      if (r == p.self) continue;
      uint32_t spins = 0;
      while (static_cast<int32_t>(ld_acquire_sys(p.flags + r) - p.epoch) < 0) {
        if ((++spins & 63u) == 0u &&
            (device_error_raised() || global_timer_ns() - start > kWaitTimeoutNs)) {
          record_device_error(kErrPeerWait);
          ok = 0;
          break;
        }
      }
    }
    ok_shared = ok;
  }
  __syncthreads();
  return ok_shared != 0;
}

template <int NV, typename OutT>
__global__ void __launch_bounds__(kNormWarpsPerBlock * 32)
    residual_layernorm_peer_kernel(NormArgs args, PeerSumArgs peers) {
  griddep_wait();
  griddep_launch_dependents();
  if (!wait_peer_epoch(peers)) return;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kNormWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= args.rows) return;
  const int cols = 128 * NV;
  const int64_t base = row * cols;
  const float* rin = static_cast<const float*>(args.residual_in);
  const RowMask mask = row_mask(args, row);
  float4 v[NV];
  if (mask.zero_residual) {
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  } else if (peers.count == 2 && mask.add_update) {
    // Two ranks (the common tensor-parallel group): issue the NVLink loads of
    // the peer's partial first, so their latency overlaps the local loads.
    const __nv_bfloat16* remote = peers.partials[peers.self ^ 1];
    const __nv_bfloat16* local = peers.partials[peers.self];
    uint2 rraw[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) rraw[i] = __ldcg(reinterpret_cast<const uint2*>(remote + base + (i * 32 + lane) * 4));
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t idx = base + (i * 32 + lane) * 4;
      v[i] = load4<float>(rin, idx);
      const uint2 lraw = __ldg(reinterpret_cast<const uint2*>(local + idx));
      const float2 la = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&lraw.x));
      const float2 lb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&lraw.y));
      const float2 ra = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rraw[i].x));
      const float2 rb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rraw[i].y));
      // Rank order of the sum is kept (partial 0 first) so both ranks agree bit for bit.
      const float2 a0 = peers.self == 0 ? la : ra, a1 = peers.self == 0 ? ra : la;
      const float2 b0 = peers.self == 0 ? lb : rb, b1 = peers.self == 0 ? rb : lb;
      v[i].x += a0.x;
      v[i].y += a0.y;
      v[i].z += b0.x;
      v[i].w += b0.y;
      v[i].x += a1.x;
      v[i].y += a1.y;
      v[i].z += b1.x;
      v[i].w += b1.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = load4<float>(rin, base + (i * 32 + lane) * 4);
    if (mask.add_update) {
      for (int r = 0; r < peers.count; ++r) {
        const __nv_bfloat16* part = peers.partials[r];
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          const int64_t idx = base + (i * 32 + lane) * 4;
          // Peer partials bypass L1 (written by another GPU during this
          // program); the local one may use the read-only path.
          uint2 raw;
          if (r == peers.self) {
            raw = __ldg(reinterpret_cast<const uint2*>(part + idx));
          } else {
            raw = __ldcg(reinterpret_cast<const uint2*>(part + idx));
          }
          const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
          const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
          v[i].x += a.x;
          v[i].y += a.y;
          v[i].z += b.x;
          v[i].w += b.y;
        }
      }
    }
  }
  if (args.residual_out != nullptr) {
#pragma unroll
    for (int i = 0; i < NV; ++i) store4<float>(args.residual_out, base + (i * 32 + lane) * 4, v[i]);
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  const float mean = warp_sum(s) * (1.0f / cols);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
    q += (a * a + b * b) + (c * c + d * d);
  }
  const float rstd = rsqrtf(warp_sum(q) * (1.0f / cols) + args.eps);
  OutT* out = static_cast<OutT*>(args.normed);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 4;
    const float4 g = __ldg(reinterpret_cast<const float4*>(args.gamma + c));
    const float4 b = __ldg(reinterpret_cast<const float4*>(args.beta + c));
    float4 o;
    o.x = (v[i].x - mean) * rstd * g.x + b.x;
    o.y = (v[i].y - mean) * rstd * g.y + b.y;
    o.z = (v[i].z - mean) * rstd * g.z + b.z;
    o.w = (v[i].w - mean) * rstd * g.w + b.w;
    if (mask.zero_normed) o = make_float4(0.f, 0.f, 0.f, 0.f);
    store4<OutT>(out, base + c, o);
  }
}

// Reduce-scatter + all-gather form for groups of three or more ranks: each
// rank sums the group's partials only for its own slice of rows [row_begin,
// row_begin + rows), adds the residual, normalises, keeps residual_out for
// those rows and writes the normalised rows into every rank's output buffer
// (`outs`, its own local, the others peer memory).  NVLink traffic per rank:
// (P - 1)/P of the rows' partials in and as many normalised rows out, instead
// of every peer's whole partial.  After a CTA barrier (which orders every
// thread's stores before thread 0), thread 0 fences at system scope (a
// cumulative fence) and counts the CTA done on a local counter; the CTA that
// completes the launch's count publishes `epoch` into this rank's slot of every
// peer's done flags (release, system scope).  peer_wait_kernel then holds the
// stream until every peer's slice has landed here.  Rows are independent, so
// each row is computed by one rank only and the ranks agree by construction.
struct PeerGatherArgs {
  void* outs[kMaxPeers];            // [rows_total, cols] OutT of every rank, index = group rank
  uint32_t* done_slots[kMaxPeers];  // this rank's slot in each peer's done flags (null: none)
  uint32_t* counter;                // this rank's CTA counter (monotonic)
  uint32_t counter_target;          // its value once every CTA of this launch is done
  int64_t row_begin;
};

template <int NV, typename OutT>
__global__ void __launch_bounds__(kNormWarpsPerBlock * 32)
    residual_layernorm_peer_rs_kernel(NormArgs args, PeerSumArgs peers, PeerGatherArgs g) {
  griddep_wait();
  griddep_launch_dependents();
  // A CTA that gives up here never counts itself done: the peers' waits for
  // this rank's slice run out and record the error too.
  if (!wait_peer_epoch(peers)) return;
  const int lane = threadIdx.x & 31;
  const int64_t local_row = static_cast<int64_t>(blockIdx.x) * kNormWarpsPerBlock + (threadIdx.x >> 5);
  if (local_row < args.rows) {
    const int cols = 128 * NV;
    const int64_t base = (g.row_begin + local_row) * cols;
    const float* rin = static_cast<const float*>(args.residual_in);
    float4 v[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = load4<float>(rin, base + (i * 32 + lane) * 4);
    // Partials added in rank order (the rank loop unrolled, so that the next
    // rank's loads can be issued while this one's are added).
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r) {
      if (r >= peers.count) break;
      const __nv_bfloat16* part = peers.partials[r];
      uint2 raw[NV];
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int64_t idx = base + (i * 32 + lane) * 4;
        raw[i] = r == peers.self ? __ldg(reinterpret_cast<const uint2*>(part + idx))
                                 : __ldcg(reinterpret_cast<const uint2*>(part + idx));
      }
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw[i].x));
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw[i].y));
        v[i].x += a.x;
        v[i].y += a.y;
        v[i].z += b.x;
        v[i].w += b.y;
      }
    }
    if (args.residual_out != nullptr) {
#pragma unroll
      for (int i = 0; i < NV; ++i) store4<float>(args.residual_out, base + (i * 32 + lane) * 4, v[i]);
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    const float mean = warp_sum(s) * (1.0f / cols);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
      q += (a * a + b * b) + (c * c + d * d);
    }
    const float rstd = rsqrtf(warp_sum(q) * (1.0f / cols) + args.eps);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 4;
      const float4 gm = __ldg(reinterpret_cast<const float4*>(args.gamma + c));
      const float4 bt = __ldg(reinterpret_cast<const float4*>(args.beta + c));
      float4 o;
      o.x = (v[i].x - mean) * rstd * gm.x + bt.x;
      o.y = (v[i].y - mean) * rstd * gm.y + bt.y;
      o.z = (v[i].z - mean) * rstd * gm.z + bt.z;
      o.w = (v[i].w - mean) * rstd * gm.w + bt.w;
      // The peers' copies first (NVLink), then this rank's.
      for (int k = 1; k <= peers.count; ++k) {
        const int r = (peers.self + k) % peers.count;
        store4<OutT>(static_cast<OutT*>(g.outs[r]), base + c, o);
      }
    }
  }
  // The CTA's stores (every thread's, ordered before thread 0 by the barrier)
  // are visible system-wide before the CTA counts itself.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t done = atomicAdd(g.counter, 1u) + 1u;
    if (done == g.counter_target) {
      __threadfence_system();
      for (int r = 0; r < peers.count; ++r)
        if (g.done_slots[r] != nullptr) st_release_sys(g.done_slots[r], peers.epoch);
    }
  }
}

// Holds the stream until every peer has published `epoch` into this rank's
// done flags (bounded acquire spin at system scope, one thread; a wait that
// runs out records kErrPeerWait).
__global__ void peer_wait_kernel(const uint32_t* flags, int count, int self, uint32_t epoch) {
  griddep_wait();
  griddep_launch_dependents();
  if (threadIdx.x != 0) return;
  const unsigned long long start = global_timer_ns();
  for (int r = 0; r < count; ++r) {
    if (r == self) continue;
    uint32_t spins = 0;
    while (static_cast<int32_t>(ld_acquire_sys(flags + r) - epoch) < 0) {
      if ((++spins & 63u) == 0u && (device_error_raised() || global_timer_ns() - start > kWaitTimeoutNs)) {
        record_device_error(kErrPeerWait);
        return;
      }
    }
  }
}

// Publishes `epoch` to the peers after this rank's partial is complete: the
// kernel runs after the GEMM on the stream, fences at system scope and stores
// the epoch with release semantics into this rank's slot of every peer's flag
// array (peer memory over NVLink).
struct PeerSignalArgs {
  uint32_t* slots[kMaxPeers];  // this rank's slot in each peer's flag array
  int count;
  uint32_t epoch;
};

__global__ void peer_signal_kernel(PeerSignalArgs args) {
  griddep_wait();
  griddep_launch_dependents();
  const int i = threadIdx.x;
  if (i < args.count && args.slots[i] != nullptr) {
    __threadfence_system();
    st_release_sys(args.slots[i], args.epoch);
  }
}

}  // namespace b200tx
