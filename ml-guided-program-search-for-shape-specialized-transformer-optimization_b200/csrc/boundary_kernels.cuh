// boundary_kernels.cuh -- the projection that closes a block branch, fused with
// the residual add and the LayerNorm that follow it, for d_model 32, 64 or 128.
//
// The reference fuses these boundaries for its small official shapes
// (solution/kernels/boundary/triton_linear_residual_norm.py:33-112, D in {32,
// 128}: Linear + bias -> rounded update -> + fp32 residual -> LayerNorm;
// solution/kernels/boundary/triton_ffn_residual_norm.py:43-136, D = F = 128:
// the whole MLP through the same boundary, the hidden row never written to
// memory).  At those shapes every launch costs more than its arithmetic, and
// fusing takes the block from seven launches to four.  Two kernels:
//
//   linear:  r = residual_in + round(x[M,K] . W[D,K]^T + b);  normed = LN(r)
//   MLP:     h = round_bf16(GELU(n[M,D] . W1[F,D]^T + b1))     (never stored)
//            r = residual_in + round(h . W2[D,F]^T + b2);      normed = LN(r)
//
// "round" is the update dtype the unfused program writes between the GEMM and
// the LayerNorm (bf16, or fp32 = no rounding), so both paths take the same
// rounding points.  Padding-row behaviour (row_valid, mask_mode) is the
// residual LayerNorm kernel's: drop the update, zero the residual, zero the
// normalised output.
//
// A CTA of four warps owns 16 rows, so that small problems still spread over
// many warps: for the Linear boundary warp w computes output columns
// [w D/4, (w + 1) D/4); for the MLP it computes 16 of every 64 hidden columns
// and their contribution to all outputs, and the four partial outputs are
// summed through shared memory.  Products are mma.sync.m16n8k16 (bf16 in,
// fp32 out; the fragment layouts of attention_mma_kernels.cuh) on operands
// staged in shared memory with 16-byte loads (rows padded by 8 elements:
// conflict-free fragment loads).  The LayerNorm statistics are summed over a
// row group's four lanes by shuffles and over the warps through shared
// memory.  No waits other than __syncthreads.
#pragma once

#include "attention_mma_kernels.cuh"
#include "gemm_kernels.cuh"
#include "norm_kernels.cuh"

namespace b200tx {

constexpr int kBoundaryRows = 16;  // rows per CTA; its 4 warps split the columns (or the hidden dim)
constexpr int kBoundaryThreads = 128;
constexpr int kBoundaryK = 64;       // K slice per iteration (linear)
constexpr int kBoundaryHidden = 64;  // hidden columns per iteration (MLP): 16 per warp

struct BoundaryArgs {
  const __nv_bfloat16* x;   // linear: [M, K]; MLP: the normalised input [M, D]
  const __nv_bfloat16* w;   // linear: [D, K]; MLP: W1 [F, D]
  const float* bias;        // linear: [D]; MLP: b1 [F]
  const __nv_bfloat16* w2;  // MLP: W2 [D, F]
  const float* bias2;       // MLP: b2 [D]
  const void* residual_in;  // [M, D] fp32 or bf16
  float* residual_out;      // [M, D] fp32, or null when the sum is not kept
  void* normed;             // [M, D] bf16 or fp32
  const float* gamma;       // [D]
  const float* beta;        // [D]
  const uint8_t* row_valid; // [M] or null
  int mask_mode;            // kNormMask* bits for rows whose flag is 0
  int M;
  int K;                    // linear: inner dimension; MLP: F
  float eps;
  int update_bf16;          // round the branch update to bf16 before the add
};

// Stage rows [row0, row0 + ROWS) x columns [c0, c0 + COLS) of a row-major bf16
// matrix with `ld` columns into smem (row stride STR); zero outside
// rows_total x cols_total.  COLS and the column bound are multiples of 8.
template <int ROWS, int COLS, int STR>
__device__ __forceinline__ void stage_bf16(__nv_bfloat16* dst, const __nv_bfloat16* src, int64_t ld,
                                           int row0, int rows_total, int c0, int cols_total) {
  constexpr int CPR = COLS / 8;  // 16-byte chunks per row
  copy_chunks<ROWS * CPR, kBoundaryThreads>(
      [&](int i) {
        const int r = i / CPR;
        const int c = (i % CPR) * 8;
        if (row0 + r >= rows_total || c0 + c >= cols_total) return make_uint4(0u, 0u, 0u, 0u);
        return *reinterpret_cast<const uint4*>(src + static_cast<int64_t>(row0 + r) * ld + c0 + c);
      },
      [&](int i, uint4 v) { *reinterpret_cast<uint4*>(dst + (i / CPR) * STR + (i % CPR) * 8) = v; });
}

template <typename T>
__device__ __forceinline__ float2 load_pair(const T* p);
template <>
__device__ __forceinline__ float2 load_pair<float>(const float* p) {
  return *reinterpret_cast<const float2*>(p);
}
template <>
__device__ __forceinline__ float2 load_pair<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}

template <typename T>
__device__ __forceinline__ void store_pair_out(T* p, float v0, float v1);
template <>
__device__ __forceinline__ void store_pair_out<float>(float* p, float v0, float v1) {
  *reinterpret_cast<float2*>(p) = make_float2(v0, v1);
}
template <>
__device__ __forceinline__ void store_pair_out<__nv_bfloat16>(__nv_bfloat16* p, float v0, float v1) {
  *reinterpret_cast<uint32_t*>(p) = pack_bf16x2(v0, v1);
}

__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Bias, rounding, residual add and LayerNorm of the CTA's 16 rows.  Warp w
// holds columns [w D/4, (w + 1) D/4) of rows g and g + 8 (acc[n][0..1] and
// acc[n][2..3] at columns w D/4 + 8n + 2t, + 1); the row statistics are summed
// over the row group's four lanes by shuffles and over the four warps through
// shared memory (`stats`, 2 x 4 x 16 floats).
template <int D, typename InT, typename OutT>
__device__ __forceinline__ void boundary_epilogue(const BoundaryArgs& a, const float (&acc)[D / 32][4], int row0,
                                                  const float* bias_out, float* stats) {
  constexpr int NT = D / 32;  // n-tiles of this warp's column slice
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;
  const int t = lane & 3;
  const int cbase = warp * (D / 4);
  float v[2][NT][2];
  float sum[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = row0 + g + 8 * h;
    const bool in_range = row < a.M;
    bool valid = true;
    if (in_range && a.row_valid != nullptr) valid = a.row_valid[row] != 0;
    const bool add_update = valid || !(a.mask_mode & kNormMaskDropUpdate);
    const bool zero_residual = !valid && (a.mask_mode & kNormMaskZeroResidual);
    const InT* rin = static_cast<const InT*>(a.residual_in) + static_cast<int64_t>(row) * D;
    sum[h] = 0.f;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int c = cbase + n * 8 + 2 * t;
      float u0 = acc[n][2 * h] + __ldg(bias_out + c);
      float u1 = acc[n][2 * h + 1] + __ldg(bias_out + c + 1);
      if (a.update_bf16) {
        u0 = round_bf16(u0);
        u1 = round_bf16(u1);
      }
      float2 r = make_float2(0.f, 0.f);
      if (in_range && !zero_residual) {
        r = load_pair<InT>(rin + c);
        if (add_update) {
          r.x += u0;
          r.y += u1;
        }
      }
      v[h][n][0] = r.x;
      v[h][n][1] = r.y;
      sum[h] += r.x + r.y;
    }
    sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 1);
    sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 2);
  }
  if (t == 0) {
    stats[warp * 16 + g] = sum[0];
    stats[warp * 16 + g + 8] = sum[1];
  }
  __syncthreads();
  float mean[2], sq[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = g + 8 * h;
    mean[h] = (stats[r] + stats[16 + r] + stats[32 + r] + stats[48 + r]) * (1.0f / D);
    sq[h] = 0.f;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const float d0 = v[h][n][0] - mean[h], d1 = v[h][n][1] - mean[h];
      sq[h] += d0 * d0 + d1 * d1;
    }
    sq[h] += __shfl_xor_sync(0xffffffffu, sq[h], 1);
    sq[h] += __shfl_xor_sync(0xffffffffu, sq[h], 2);
  }
  if (t == 0) {
    stats[64 + warp * 16 + g] = sq[0];
    stats[64 + warp * 16 + g + 8] = sq[1];
  }
  __syncthreads();
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = g + 8 * h;
    const int row = row0 + r;
    if (row >= a.M) continue;
    const float var = (stats[64 + r] + stats[80 + r] + stats[96 + r] + stats[112 + r]) * (1.0f / D);
    const float rstd = rsqrtf(var + a.eps);
    const bool zero_normed =
        a.row_valid != nullptr && a.row_valid[row] == 0 && (a.mask_mode & kNormMaskZeroNormed);
    if (a.residual_out != nullptr) {
      float* rout = a.residual_out + static_cast<int64_t>(row) * D;
#pragma unroll
      for (int n = 0; n < NT; ++n)
        *reinterpret_cast<float2*>(rout + cbase + n * 8 + 2 * t) = make_float2(v[h][n][0], v[h][n][1]);
    }
    // All gamma / beta loads (read-only path) before any store of the row: a
    // load that follows a store through a pointer that may alias it cannot be
    // hoisted, and would wait a memory round trip per column pair.
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int c = cbase + n * 8 + 2 * t;
      const float g0 = __ldg(a.gamma + c), g1 = __ldg(a.gamma + c + 1);
      const float b0 = __ldg(a.beta + c), b1 = __ldg(a.beta + c + 1);
      v[h][n][0] = zero_normed ? 0.f : (v[h][n][0] - mean[h]) * rstd * g0 + b0;
      v[h][n][1] = zero_normed ? 0.f : (v[h][n][1] - mean[h]) * rstd * g1 + b1;
    }
    OutT* out = static_cast<OutT*>(a.normed) + static_cast<int64_t>(row) * D;
#pragma unroll
    for (int n = 0; n < NT; ++n) store_pair_out<OutT>(out + cbase + n * 8 + 2 * t, v[h][n][0], v[h][n][1]);
  }
}

// out-proj / FFN-out + bias + rounding + residual add + LayerNorm.  A CTA owns
// 16 rows; warp w computes their columns [w D/4, (w + 1) D/4).
template <int D, typename InT, typename OutT>
__global__ void __launch_bounds__(kBoundaryThreads) linear_residual_layernorm_kernel(BoundaryArgs a) {
  constexpr int STR = kBoundaryK + 8;
  constexpr int NT = D / 32;
  __shared__ __align__(16) __nv_bfloat16 x_s[kBoundaryRows * STR];
  __shared__ __align__(16) __nv_bfloat16 w_s[D * STR];
  __shared__ float stats[128];
  // The weights do not depend on the previous kernel: their first slice is
  // fetched while that kernel drains (programmatic dependent launch).
  stage_bf16<D, kBoundaryK, STR>(w_s, a.w, a.K, 0, D, 0, a.K);
  griddep_wait();
  griddep_launch_dependents();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;
  const int t = lane & 3;
  const int row0 = static_cast<int>(blockIdx.x) * kBoundaryRows;

  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  for (int k0 = 0; k0 < a.K; k0 += kBoundaryK) {
    if (k0 > 0) {
      __syncthreads();  // the previous slice's fragments have been read
      stage_bf16<D, kBoundaryK, STR>(w_s, a.w, a.K, 0, D, k0, a.K);
    }
    stage_bf16<kBoundaryRows, kBoundaryK, STR>(x_s, a.x, a.K, row0, a.M, k0, a.K);
    __syncthreads();
#pragma unroll
    for (int ks = 0; ks < kBoundaryK / 16; ++ks) {
      const __nv_bfloat16* x0 = &x_s[g * STR + ks * 16 + 2 * t];
      const __nv_bfloat16* x1 = x0 + 8 * STR;
      const uint32_t af[4] = {ld_u32(x0), ld_u32(x1), ld_u32(x0 + 8), ld_u32(x1 + 8)};
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const __nv_bfloat16* wr = &w_s[(warp * (D / 4) + n * 8 + g) * STR + ks * 16 + 2 * t];
        mma_m16n8k16_bf16(acc[n], af, ld_u32(wr), ld_u32(wr + 8));
      }
    }
  }
  boundary_epilogue<D, InT, OutT>(a, acc, row0, a.bias, stats);
}

// FFN-in + bias + GELU + bf16 hidden, FFN-out + bias + rounding + residual add
// + LayerNorm; the hidden rows never leave the chip.  A CTA owns 16 rows; per
// 64-column hidden chunk warp w computes hidden columns [16w, 16w + 16) and
// their contribution to all D outputs; the four partial outputs are summed
// through shared memory before the epilogue.
template <int D, typename InT, typename OutT>
__global__ void __launch_bounds__(kBoundaryThreads) mlp_residual_layernorm_kernel(BoundaryArgs a) {
  constexpr int XSTR = D + 8;
  constexpr int HSTR = kBoundaryHidden + 8;
  constexpr int RSTR = D + 8;  // partial-output row stride (floats)
  constexpr int W1_BYTES = kBoundaryHidden * XSTR * 2;
  constexpr int W2_BYTES = D * HSTR * 2;
  constexpr int RED_BYTES = 4 * kBoundaryRows * RSTR * 4;
  constexpr int POOL = (W1_BYTES + W2_BYTES) > RED_BYTES ? (W1_BYTES + W2_BYTES) : RED_BYTES;
  __shared__ __align__(16) __nv_bfloat16 x_s[kBoundaryRows * XSTR];
  __shared__ __align__(16) unsigned char pool[POOL];  // W1 + W2 chunks, then the partial outputs
  __shared__ float stats[128];
  __nv_bfloat16* w1_s = reinterpret_cast<__nv_bfloat16*>(pool);
  __nv_bfloat16* w2_s = reinterpret_cast<__nv_bfloat16*>(pool + W1_BYTES);
  float* red = reinterpret_cast<float*>(pool);
  const int F = a.K;
  // The first hidden chunk's weights are fetched before waiting for the
  // previous kernel (they do not depend on it).
  stage_bf16<kBoundaryHidden, D, XSTR>(w1_s, a.w, D, 0, F, 0, D);
  stage_bf16<D, kBoundaryHidden, HSTR>(w2_s, a.w2, F, 0, D, 0, F);
  griddep_wait();
  griddep_launch_dependents();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;
  const int t = lane & 3;
  const int row0 = static_cast<int>(blockIdx.x) * kBoundaryRows;

  stage_bf16<kBoundaryRows, D, XSTR>(x_s, a.x, D, row0, a.M, 0, D);
  __syncthreads();
  uint32_t xf[D / 16][4];
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
    const __nv_bfloat16* x0 = &x_s[g * XSTR + ks * 16 + 2 * t];
    const __nv_bfloat16* x1 = x0 + 8 * XSTR;
    xf[ks][0] = ld_u32(x0);
    xf[ks][1] = ld_u32(x1);
    xf[ks][2] = ld_u32(x0 + 8);
    xf[ks][3] = ld_u32(x1 + 8);
  }

  float acc[D / 8][4];  // this warp's partial output over its hidden columns
#pragma unroll
  for (int n = 0; n < D / 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  for (int h0 = 0; h0 < F; h0 += kBoundaryHidden) {
    if (h0 > 0) {
      __syncthreads();  // the previous chunk's fragments have been read
      stage_bf16<kBoundaryHidden, D, XSTR>(w1_s, a.w, D, h0, F, 0, D);
      stage_bf16<D, kBoundaryHidden, HSTR>(w2_s, a.w2, F, 0, D, h0, F);
      __syncthreads();
    }
    float hacc[2][4];
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      hacc[n][0] = hacc[n][1] = hacc[n][2] = hacc[n][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const __nv_bfloat16* wr = &w1_s[(warp * 16 + n * 8 + g) * XSTR + ks * 16 + 2 * t];
        mma_m16n8k16_bf16(hacc[n], xf[ks], ld_u32(wr), ld_u32(wr + 8));
      }
    }
    // Bias, exact-erf GELU and the bf16 hidden rounding of the unfused program,
    // packed straight into the A fragment of the second product.  Hidden
    // columns past F have zero weights and bias, so they contribute GELU(0) = 0.
    uint32_t af[4];
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      const int c = h0 + warp * 16 + n * 8 + 2 * t;
      const float b0 = c < F ? __ldg(a.bias + c) : 0.f;
      const float b1 = c < F ? __ldg(a.bias + c + 1) : 0.f;
      af[2 * n] = pack_bf16x2(gelu_erf(hacc[n][0] + b0), gelu_erf(hacc[n][1] + b1));
      af[2 * n + 1] = pack_bf16x2(gelu_erf(hacc[n][2] + b0), gelu_erf(hacc[n][3] + b1));
    }
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      const __nv_bfloat16* wr = &w2_s[(n * 8 + g) * HSTR + warp * 16 + 2 * t];
      mma_m16n8k16_bf16(acc[n], af, ld_u32(wr), ld_u32(wr + 8));
    }
  }
  // Sum the four warps' partial outputs; warp w keeps columns [w D/4, (w+1) D/4).
  __syncthreads();  // the last chunk's weights have been read: the pool is free
#pragma unroll
  for (int n = 0; n < D / 8; ++n) {
    float* p = red + (warp * kBoundaryRows + g) * RSTR + n * 8 + 2 * t;
    *reinterpret_cast<float2*>(p) = make_float2(acc[n][0], acc[n][1]);
    *reinterpret_cast<float2*>(p + 8 * RSTR) = make_float2(acc[n][2], acc[n][3]);
  }
  __syncthreads();
  float out[D / 32][4];
#pragma unroll
  for (int n = 0; n < D / 32; ++n) {
    const int c = warp * (D / 4) + n * 8 + 2 * t;
    float2 s0 = make_float2(0.f, 0.f), s1 = make_float2(0.f, 0.f);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float2 p0 = *reinterpret_cast<const float2*>(red + (w * kBoundaryRows + g) * RSTR + c);
      const float2 p1 = *reinterpret_cast<const float2*>(red + (w * kBoundaryRows + g + 8) * RSTR + c);
      s0.x += p0.x;
      s0.y += p0.y;
      s1.x += p1.x;
      s1.y += p1.y;
    }
    out[n][0] = s0.x;
    out[n][1] = s0.y;
    out[n][2] = s1.x;
    out[n][3] = s1.y;
  }
  boundary_epilogue<D, InT, OutT>(a, out, row0, a.bias2, stats);
}

}  // namespace b200tx
