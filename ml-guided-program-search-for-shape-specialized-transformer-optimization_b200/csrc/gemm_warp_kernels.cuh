// gemm_warp_kernels.cuh -- the projection GEMM for small problems on the
// warp-level tensor-core instruction mma.sync.m16n8k16 (bf16 in, fp32 out).
//
// The tcgen05 GEMMs (gemm_kernels.cuh) are persistent pipelines built for
// large M: each launch allocates TMEM, initialises mbarriers, fetches tensor
// maps, runs a TMA ring and drains its epilogue through TMA stores, which costs
// a few microseconds of fixed latency.  The reference's official shapes have
// as few as 128 tokens with D = F = 128 (official/test_shapes.json), where that
// latency is the whole projection.  This variant has none of it: a CTA of four
// warps computes a 64 x 64 output tile, staging 64 x 64 slices of A and W in
// shared memory with 16-byte loads (padded rows: conflict-free fragment loads)
// and issuing m16n8k16 MMAs, then applies the same epilogue (fp32 bias, exact
// erf GELU, cast) and stores straight from registers.  Same function as the
// other variants: out[M, N] = epilogue(a[M, K] . w[N, K]^T + bias).
//
// Warp w owns rows [16w, 16w + 16) of the tile and all 64 columns (8 n-tiles
// of 8); the fragment layouts are those of attention_mma_kernels.cuh.
#pragma once

#include "attention_mma_kernels.cuh"
#include "gemm_kernels.cuh"

namespace b200tx {

constexpr int kWarpGemmBM = 64;
constexpr int kWarpGemmBN = 64;
constexpr int kWarpGemmBK = 64;
constexpr int kWarpGemmThreads = 128;

struct WarpGemmArgs {
  const __nv_bfloat16* a;  // [M, K]
  const __nv_bfloat16* w;  // [N, K]
  const float* bias;       // [N] or null
  void* out;               // [M, N] bf16 or fp32
  int M, N, K;
  int n_tiles;             // ceil(N / kWarpGemmBN)
};

template <typename OutT>
__device__ __forceinline__ void store_pair(OutT* p, float v0, float v1);
template <>
__device__ __forceinline__ void store_pair<__nv_bfloat16>(__nv_bfloat16* p, float v0, float v1) {
  *reinterpret_cast<uint32_t*>(p) = pack_bf16x2(v0, v1);
}
template <>
__device__ __forceinline__ void store_pair<float>(float* p, float v0, float v1) {
  *reinterpret_cast<float2*>(p) = make_float2(v0, v1);
}

template <int EPI, typename OutT>
__global__ void __launch_bounds__(kWarpGemmThreads) gemm_bf16_tn_warp_kernel(WarpGemmArgs args) {
  constexpr int STR = kWarpGemmBK + 8;                    // padded row (elements)
  constexpr int CHUNKS = kWarpGemmBM * kWarpGemmBK / 8;   // 16-byte chunks per operand slice
  __shared__ __align__(16) __nv_bfloat16 a_s[kWarpGemmBM * STR];
  __shared__ __align__(16) __nv_bfloat16 w_s[kWarpGemmBN * STR];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;
  const int t = lane & 3;
  const int m0 = static_cast<int>(blockIdx.x / args.n_tiles) * kWarpGemmBM;
  const int n0 = static_cast<int>(blockIdx.x % args.n_tiles) * kWarpGemmBN;
  const int M = args.M, N = args.N, K = args.K;
  // W is not written by the previous kernel: its first slice is fetched while
  // that kernel drains (programmatic dependent launch).
  copy_chunks<CHUNKS, kWarpGemmThreads>(
      [&](int i) {
        const int row = i / (kWarpGemmBK / 8);
        const int c = (i % (kWarpGemmBK / 8)) * 8;
        if (c >= K || n0 + row >= N) return make_uint4(0u, 0u, 0u, 0u);
        return *reinterpret_cast<const uint4*>(args.w + static_cast<int64_t>(n0 + row) * K + c);
      },
      [&](int i, uint4 v) {
        *reinterpret_cast<uint4*>(&w_s[(i / (kWarpGemmBK / 8)) * STR + (i % (kWarpGemmBK / 8)) * 8]) = v;
      });
  griddep_wait();
  griddep_launch_dependents();

  float acc[kWarpGemmBN / 8][4];
#pragma unroll
  for (int n = 0; n < kWarpGemmBN / 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;

  for (int k0 = 0; k0 < K; k0 += kWarpGemmBK) {
    if (k0 > 0) __syncthreads();  // the previous slice's fragments have been read
    // Chunks [0, CHUNKS) are A's, [CHUNKS, 2 CHUNKS) W's (W's first slice is
    // already staged); K is a multiple of 8, so a chunk is all inside K or all
    // outside.
    copy_chunks<2 * CHUNKS, kWarpGemmThreads>(
        [&](int i) {
          const bool is_w = i >= CHUNKS;
          const int ci = is_w ? i - CHUNKS : i;
          const int row = ci / (kWarpGemmBK / 8);
          const int c = (ci % (kWarpGemmBK / 8)) * 8;
          const int grow = (is_w ? n0 : m0) + row;
          if ((is_w && k0 == 0) || k0 + c >= K || grow >= (is_w ? N : M)) return make_uint4(0u, 0u, 0u, 0u);
          return *reinterpret_cast<const uint4*>((is_w ? args.w : args.a) + static_cast<int64_t>(grow) * K + k0 + c);
        },
        [&](int i, uint4 v) {
          const bool is_w = i >= CHUNKS;
          if (is_w && k0 == 0) return;  // staged before the wait
          const int ci = is_w ? i - CHUNKS : i;
          __nv_bfloat16* dst = is_w ? w_s : a_s;
          *reinterpret_cast<uint4*>(&dst[(ci / (kWarpGemmBK / 8)) * STR + (ci % (kWarpGemmBK / 8)) * 8]) = v;
        });
    __syncthreads();
#pragma unroll
    for (int ks = 0; ks < kWarpGemmBK / 16; ++ks) {
      const __nv_bfloat16* a0 = &a_s[(warp * 16 + g) * STR + ks * 16 + 2 * t];
      const __nv_bfloat16* a1 = a0 + 8 * STR;
      const uint32_t af[4] = {ld_u32(a0), ld_u32(a1), ld_u32(a0 + 8), ld_u32(a1 + 8)};
#pragma unroll
      for (int n = 0; n < kWarpGemmBN / 8; ++n) {
        const __nv_bfloat16* wr = &w_s[(n * 8 + g) * STR + ks * 16 + 2 * t];
        mma_m16n8k16_bf16(acc[n], af, ld_u32(wr), ld_u32(wr + 8));
      }
    }
  }

  OutT* out = static_cast<OutT*>(args.out);
  const int r0 = m0 + warp * 16 + g;
  const int r1 = r0 + 8;
  // Bias (read-only path) and epilogue for every column before the first
  // store: loads after a possibly aliasing store could not be hoisted.
#pragma unroll
  for (int n = 0; n < kWarpGemmBN / 8; ++n) {
    const int col = n0 + n * 8 + 2 * t;
    float2 bb = make_float2(0.f, 0.f);
    if (args.bias != nullptr && col < N) bb = make_float2(__ldg(args.bias + col), __ldg(args.bias + col + 1));
    acc[n][0] += bb.x;
    acc[n][1] += bb.y;
    acc[n][2] += bb.x;
    acc[n][3] += bb.y;
    if constexpr (EPI == kEpiBiasGelu) {
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[n][e] = gelu_erf(acc[n][e]);
    }
  }
#pragma unroll
  for (int n = 0; n < kWarpGemmBN / 8; ++n) {
    const int col = n0 + n * 8 + 2 * t;
    if (col >= N) continue;  // N is a multiple of 8: col + 1 < N whenever col < N
    if (r0 < M) store_pair<OutT>(out + static_cast<int64_t>(r0) * N + col, acc[n][0], acc[n][1]);
    if (r1 < M) store_pair<OutT>(out + static_cast<int64_t>(r1) * N + col, acc[n][2], acc[n][3]);
  }
}

}  // namespace b200tx
