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

}  // namespace b200tx
