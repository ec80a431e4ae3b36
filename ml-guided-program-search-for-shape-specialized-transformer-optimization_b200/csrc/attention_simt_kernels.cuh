// attention_simt_kernels.cuh -- flash attention for any head_dim in
// {8, 16, 32, 64, 128, 256} on the CUDA cores, for the shapes the tcgen05
// kernels (head_dim 64) do not cover: the reference's official benchmark
// shapes (official/test_shapes.json) have head dims 8, 32, 128 and 256.
//
// Semantics as the tensor-core kernels (official/torch_transformer_benchmark.py
// :95-118): softmax(q k^T * scale, causal -inf, key-padding -inf) in fp32, the
// probabilities rounded to bf16 before P.V as the reference casts them to the
// activation dtype, fp32 accumulation; reads the packed [B, S, 3, H, Dh]
// projection, writes [B, S, H, Dh].  A query that sees no valid key writes a
// zero row.
//
// One CTA = 32 query rows of one (batch, head).  Each query row is owned by
// T = max(1, Dh/16) consecutive threads; thread t of a row holds dims
// [16t, 16t+16) of q and of the output accumulator in registers.  Per KV tile
// of 32 keys (K and V staged in shared memory as bf16): partial dot products
// over the thread's 16 dims are summed across the row's T lanes by xor
// shuffles, the 32 scores are masked, the online softmax updates the running
// max / sum (fp32), and P.V accumulates the thread's 16 output dims.
#pragma once

#include "sm100_common.cuh"

namespace b200tx {

constexpr int kSimtRows = 32;  // query rows per CTA
constexpr int kSimtKeys = 32;  // keys per KV tile

struct SimtAttnArgs {
  const __nv_bfloat16* qkv;   // [B, S, 3, H, Dh]
  const uint8_t* key_valid;   // [B, S] or null
  __nv_bfloat16* out;         // [B, S, H, Dh]
  int batch, seq, heads;
  float scale_log2;           // scale * log2(e)
  int causal;
};

template <int DH>
__global__ void attention_simt_kernel(SimtAttnArgs args) {
  constexpr int W = DH < 16 ? DH : 16;  // dims per thread
  constexpr int T = DH / W;             // threads per query row
  constexpr int VEC = W / 8;            // 16-byte vectors per thread slice
  __shared__ __align__(16) __nv_bfloat16 k_tile[kSimtKeys][DH];
  __shared__ __align__(16) __nv_bfloat16 v_tile[kSimtKeys][DH];
  __shared__ uint8_t valid_tile[kSimtKeys];

  griddep_wait();
  griddep_launch_dependents();

  const int tid = threadIdx.x;
  const int row_in_block = tid / T;
  const int part = tid % T;
  const int num_q_blocks = (args.seq + kSimtRows - 1) / kSimtRows;
  const int q_block = static_cast<int>(blockIdx.x % num_q_blocks);
  const int bh = static_cast<int>(blockIdx.x / num_q_blocks);
  const int head = bh % args.heads;
  const int b = bh / args.heads;
  const int q_idx = q_block * kSimtRows + row_in_block;
  const int64_t row_stride = 3LL * args.heads * DH;  // elements per token in qkv
  const int d_model = args.heads * DH;
  const __nv_bfloat16* base = args.qkv + static_cast<int64_t>(b) * args.seq * row_stride;

  float q[W];
  {
    const int qi = q_idx < args.seq ? q_idx : args.seq - 1;  // rows past S compute, never store
    const __nv_bfloat16* qp = base + qi * row_stride + head * DH + part * W;
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      const uint4 raw = *reinterpret_cast<const uint4*>(qp + v * 8);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        q[v * 8 + 2 * i] = f.x * args.scale_log2;
        q[v * 8 + 2 * i + 1] = f.y * args.scale_log2;
      }
    }
  }
  float o[W];
#pragma unroll
  for (int i = 0; i < W; ++i) o[i] = 0.f;
  float m_run = -INFINITY;
  float l_run = 0.f;

  const int last_row = (q_block + 1) * kSimtRows - 1;
  const int kv_end = args.causal ? (last_row < args.seq - 1 ? last_row + 1 : args.seq) : args.seq;
  const int n_tiles = (kv_end + kSimtKeys - 1) / kSimtKeys;

  for (int t = 0; t < n_tiles; ++t) {
    const int k0 = t * kSimtKeys;
    __syncthreads();  // previous tile fully consumed
    // Stage K and V (16-byte vectors) and the keys' validity.
    constexpr int kVecPerRow = DH / 8;
    for (int idx = tid; idx < kSimtKeys * kVecPerRow; idx += blockDim.x) {
      const int kr = idx / kVecPerRow;
      const int c = (idx % kVecPerRow) * 8;
      const int key = k0 + kr;
      uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (key < args.seq) {
        const __nv_bfloat16* tok = base + key * row_stride;
        kv = *reinterpret_cast<const uint4*>(tok + d_model + head * DH + c);
        vv = *reinterpret_cast<const uint4*>(tok + 2 * d_model + head * DH + c);
      }
      *reinterpret_cast<uint4*>(&k_tile[kr][c]) = kv;
      *reinterpret_cast<uint4*>(&v_tile[kr][c]) = vv;
    }
    for (int kr = tid; kr < kSimtKeys; kr += blockDim.x) {
      const int key = k0 + kr;
      valid_tile[kr] = key < args.seq && (args.key_valid == nullptr ||
                                          args.key_valid[static_cast<int64_t>(b) * args.seq + key] != 0);
    }
    __syncthreads();

    float s[kSimtKeys];
#pragma unroll
    for (int kr = 0; kr < kSimtKeys; ++kr) {
      float acc = 0.f;
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        const uint4 raw = *reinterpret_cast<const uint4*>(&k_tile[kr][part * W + v * 8]);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(h[i]);
          acc = fmaf(q[v * 8 + 2 * i], f.x, acc);
          acc = fmaf(q[v * 8 + 2 * i + 1], f.y, acc);
        }
      }
#pragma unroll
      // The row's T lanes are consecutive and T divides 32, so xor offsets
      // below T stay inside the row.
      for (int off = 1; off < T; off <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
      const int key = k0 + kr;
      const bool masked = !valid_tile[kr] || (args.causal && key > q_idx);
      s[kr] = masked ? -INFINITY : acc;
    }
    float mx = -INFINITY;
#pragma unroll
    for (int kr = 0; kr < kSimtKeys; ++kr) mx = fmaxf(mx, s[kr]);
    const float m_new = fmaxf(m_run, mx);
    const float m_use = m_new == -INFINITY ? 0.f : m_new;
    const float alpha = fast_exp2(m_run - m_use);  // 0 when m_run = -inf
    l_run *= alpha;
#pragma unroll
    for (int i = 0; i < W; ++i) o[i] *= alpha;
#pragma unroll
    for (int kr = 0; kr < kSimtKeys; ++kr) {
      const float p_exact = fast_exp2(s[kr] - m_use);
      l_run += p_exact;
      // P is rounded to bf16 before P.V (the reference casts probabilities
      // to the activation dtype); the row sum keeps fp32.
      const float p = __bfloat162float(__float2bfloat16_rn(p_exact));
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        const uint4 raw = *reinterpret_cast<const uint4*>(&v_tile[kr][part * W + v * 8]);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(h[i]);
          o[v * 8 + 2 * i] = fmaf(p, f.x, o[v * 8 + 2 * i]);
          o[v * 8 + 2 * i + 1] = fmaf(p, f.y, o[v * 8 + 2 * i + 1]);
        }
      }
    }
    m_run = m_new;
  }

  if (q_idx < args.seq) {
    const float inv_l = l_run > 0.f ? 1.0f / l_run : 0.f;
    __nv_bfloat16* op = args.out + (static_cast<int64_t>(b) * args.seq + q_idx) * d_model + head * DH + part * W;
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      uint4 raw;
      raw.x = pack_bf16x2(o[v * 8 + 0] * inv_l, o[v * 8 + 1] * inv_l);
      raw.y = pack_bf16x2(o[v * 8 + 2] * inv_l, o[v * 8 + 3] * inv_l);
      raw.z = pack_bf16x2(o[v * 8 + 4] * inv_l, o[v * 8 + 5] * inv_l);
      raw.w = pack_bf16x2(o[v * 8 + 6] * inv_l, o[v * 8 + 7] * inv_l);
      *reinterpret_cast<uint4*>(op + v * 8) = raw;
    }
  }
}

}  // namespace b200tx
