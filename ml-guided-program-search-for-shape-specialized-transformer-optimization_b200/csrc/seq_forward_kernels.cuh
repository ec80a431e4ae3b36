// seq_forward_kernels.cuh -- the whole forward of a small model in one launch:
// every layer of the reference's official block (pre-norm: x += attention(LN1(x));
// x += FFN(LN2(x)); final LayerNorm) for d_model = ffn_dim = 128 and sequences
// of at most 128 tokens, one CTA per tile of 128 rows holding whole sequences.
// Replaces, for the reference's small official shapes (official/test_shapes.json:
// B x S x 128 with 1, 2 or 4 heads), the per-primitive program of
// solution/transformer.py:1346-1513 (_forward_eager): about seven launches per
// layer become none, and no activation leaves the SM between the input load
// and the output store.
//
// On-chip state of a tile (16 warps; thread (w, l) works on row 32 (w % 4) + l,
// its TMEM lane, and on the 32 columns [32 (w / 4), 32 (w / 4) + 32)):
//   TMEM   R  [0, 128)    fp32 residual stream
//          T1 [128, 256)  accumulators: Q, then scores of even heads, out-proj, FFN-out
//          T2 [256, 384)  K, then scores of odd heads, FFN-in
//          T3 [384, 512)  V, then the attention output of all heads
//   smem   six 32 KB [128 x 128] bf16 operand images in the UMMA K-major
//          128-byte-swizzled layout (two 64-column panels of 128 rows):
//          A   the normalised input of a projection (n, ctx, n2, the FFN
//              hidden row), or the probabilities of odd heads
//          Q, K, VT (V transposed: dims x tokens, so that P . V has K = tokens)
//          W0, W1  weight slots, filled by 1D bulk copies of weight images
//              pre-swizzled in global memory (b200tx_seq_weight_image); W0
//              holds the probabilities of even heads during attention (W1's
//              copy waits until the last P . V is done)
// Per layer: Q, K, V projections (UMMA M128 N128 K128) with bias and bf16
// rounding; per head S = Q_h K_h^T (K = head_dim), causal softmax within each
// sequence in fp32 (probabilities normalised, then rounded to bf16, as the
// unfused program), O_h = P V_h into T3; ctx = bf16(O); u = ctx Wo^T + bo,
// rounded to bf16, r += u, n2 = LN2(r); h = bf16(GELU(n2 W1^T + b1));
// u = h W2^T + b2 rounded, r += u, n = LN(r) with the next layer's norm1 (bf16)
// or the final norm (fp32, the output).  Thread 0 issues the bulk copies and
// the UMMAs; every asynchronous event has its own mbarrier, so no barrier ever
// has two phases outstanding; every wait is bounded and its outcome voted
// CTA-wide, so the CTA leaves together.
#pragma once

#include "gemm_kernels.cuh"
#include "sm100_common.cuh"

namespace b200tx {

constexpr int kSfD = 128;            // d_model = ffn_dim
constexpr int kSfRows = 128;         // rows per tile
constexpr int kSfThreads = 512;  // 16 warps: 4 lane quarters x 4 column groups
constexpr int kSfMaxLayers = 8;
constexpr uint32_t kSfMatBytes = kSfRows * kSfD * 2;  // 32 KB operand image
constexpr uint32_t kSfPanelBytes = kSfMatBytes / 2;   // 64 columns x 128 rows
constexpr int kSfWeightImages = 6;                    // Wq, Wk, Wv, Wo, W1, W2 per layer
constexpr size_t kSfSmemBytes = 1024 + 6 * static_cast<size_t>(kSfMatBytes);  // 193 KB

struct SeqLayer {
  const uint8_t* w_img;           // kSfWeightImages pre-swizzled images of kSfMatBytes each
  const float* b_qkv;             // [384]: q, k, v
  const float* b_o;               // [128]
  const float* b_1;               // [128]
  const float* b_2;               // [128]
  const float* ln2_g;             // norm2 of this layer
  const float* ln2_b;
  const float* next_g;            // norm1 of the next layer, or the final norm
  const float* next_b;
};

struct SeqForwardArgs {
  const float* x;                 // [rows, 128] fp32
  float* out;                     // [rows, 128] fp32
  const float* ln0_g;             // norm1 of layer 0
  const float* ln0_b;
  SeqLayer layers[kSfMaxLayers];
  int num_layers;
  int rows;                       // B * S
  int seq;                        // S, a divisor of 128
  int heads;                      // head_dim = 128 / heads in {32, 64, 128}
  int num_tiles;
  float scale_log2;               // head_dim^-1/2 * log2(e)
  float eps;
};

// Byte offset of element (row, col) of a [128 x 128] bf16 operand image:
// panel col / 64, row pitch 128 bytes, 16-byte chunk (col % 64) / 8 swizzled
// with row % 8.
__device__ __forceinline__ uint32_t sf_offset(int row, int col) {
  const uint32_t panel = static_cast<uint32_t>(col) >> 6;
  const uint32_t chunk = (static_cast<uint32_t>(col) >> 3) & 7u;
  return panel * kSfPanelBytes + static_cast<uint32_t>(row) * 128u + ((chunk ^ (static_cast<uint32_t>(row) & 7u)) << 4) +
         (static_cast<uint32_t>(col) & 7u) * 2u;
}

// Eight consecutive columns [col, col + 8) of this thread's row, as bf16.
__device__ __forceinline__ void sf_store8(uint32_t image, int row, int col, const float* v) {
  st_shared_v4(image + sf_offset(row, col), pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
               pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}

// UMMA shared-memory descriptor of the K-step at column k0 (a multiple of 16)
// of rows [row0, row0 + n) of an operand image (row0 a multiple of 8).
__device__ __forceinline__ uint64_t sf_desc(uint32_t image, int row0, int k0) {
  return sw128_desc(image + (static_cast<uint32_t>(k0) >> 6) * kSfPanelBytes + static_cast<uint32_t>(row0) * 128u +
                        (static_cast<uint32_t>(k0) & 63u) * 2u,
                    16, 1024);
}

// D[128 x n] (+)= A[128 x K] . B[n x K]^T over K columns [k0, k0 + K) of both
// images; one thread issues.
__device__ __forceinline__ void sf_mma(uint32_t d_tmem, uint32_t a_img, uint32_t b_img, int b_row0, int n, int k0,
                                       int k_len) {
  const uint32_t idesc = umma_idesc_bf16(128, n, false, false);
  for (int k = 0; k < k_len; k += 16)
    umma_bf16_ss(d_tmem, sf_desc(a_img, 0, k0 + k), sf_desc(b_img, b_row0, k0 + k), idesc, k != 0 ? 1u : 0u);
}

// One [128 x 128] bf16 row-major weight (torch Linear layout [out, in]) into
// its operand image: 16-byte chunk (r, j) of the source to sf_offset(r, 8 j).
// 2048 chunks, one per thread.
__global__ void seq_weight_image_kernel(const __nv_bfloat16* w, uint8_t* image) {
  const int i = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= kSfRows * (kSfD / 8)) return;
  const int r = i / (kSfD / 8), j = i % (kSfD / 8);
  const uint4 v = *reinterpret_cast<const uint4*>(w + r * kSfD + j * 8);
  *reinterpret_cast<uint4*>(image + sf_offset(r, j * 8)) = v;
}

// Every weight image of a model in one launch (the allocation-free entry
// point's images): block (x, y) moves 256 of the 2048 sixteen-byte chunks of
// image y (layer y / 6, matrix y % 6) from its row-major source.  It waits for
// the previous launch on the stream to complete before its first access, so
// that it never rewrites images a previous forward is still reading.
struct SeqImageSources {
  const __nv_bfloat16* w[kSfMaxLayers * kSfWeightImages];
};

__global__ void seq_weight_images_kernel(const __grid_constant__ SeqImageSources src, uint8_t* images) {
  griddep_wait();
  griddep_launch_dependents();
  const int i = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= kSfRows * (kSfD / 8)) return;
  const int r = i / (kSfD / 8), j = i % (kSfD / 8);
  const uint4 v = *reinterpret_cast<const uint4*>(src.w[blockIdx.y] + r * kSfD + j * 8);
  *reinterpret_cast<uint4*>(images + static_cast<size_t>(blockIdx.y) * kSfMatBytes + sf_offset(r, j * 8)) = v;
}

// The per-row phases.  Thread (warp w, lane l) owns row 32 (w % 4) + l (its
// TMEM lane) and the 32 columns [32 (w / 4), 32 (w / 4) + 32): one 32-column
// TMEM load per phase.  Row reductions (LayerNorm statistics, softmax max and
// sum) combine the four column groups' partials, one (a, b) pair per group and
// one CTA barrier per reduction, through `red2` (two buffers used in turn).
struct SfRow {
  int row;       // tile row = TMEM lane
  int grp;       // column group 0..3
  int col0;      // first column of the group
  float2* red2;  // [2][4][128] paired partials
  int turn;      // buffer of the next reduction
};

// The row's four column groups' (a, b) partials, in group order (one CTA
// barrier).  The two buffers alternate, so a buffer is rewritten only after
// the next reduction's barrier, which follows every read of it.
__device__ __forceinline__ void sf_row_pairs(SfRow& r, float a, float b, float2 (&p)[4]) {
  float2* buf = r.red2 + r.turn * 4 * kSfRows;
  r.turn ^= 1;
  buf[r.grp * kSfRows + r.row] = make_float2(a, b);
  __syncthreads();
#pragma unroll
  for (int g = 0; g < 4; ++g) p[g] = buf[g * kSfRows + r.row];
}

__device__ __forceinline__ void sf_load_bias32(const float* p, float* b) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p) + q);
    b[4 * q] = v.x;
    b[4 * q + 1] = v.y;
    b[4 * q + 2] = v.z;
    b[4 * q + 3] = v.w;
  }
}

// image[row, group columns] = bf16(acc + bias).
__device__ __forceinline__ void sf_epilogue_proj(uint32_t t_addr, const float* bias, uint32_t image, const SfRow& r) {
  uint32_t a[32];
  tmem_ld_32cols(t_addr + r.col0, a);
  float b[32];
  sf_load_bias32(bias + r.col0, b);
  tmem_wait_ld();
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(a[i]) + b[i];
#pragma unroll
  for (int q = 0; q < 4; ++q) sf_store8(image, r.row, r.col0 + 8 * q, v + 8 * q);
}

// VT[d, row] = bf16(acc[d] + bias[d]) for the group's 32 dims (V transposed).
__device__ __forceinline__ void sf_epilogue_vt(uint32_t t_addr, const float* bias, uint32_t image, const SfRow& r) {
  uint32_t a[32];
  tmem_ld_32cols(t_addr + r.col0, a);
  float b[32];
  sf_load_bias32(bias + r.col0, b);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const __nv_bfloat16 h = __float2bfloat16_rn(__uint_as_float(a[i]) + b[i]);
    asm volatile("st.shared.b16 [%0], %1;" ::"r"(image + sf_offset(r.col0 + i, r.row)),
                 "h"(*reinterpret_cast<const unsigned short*>(&h))
                 : "memory");
  }
}

// image[row, group columns] = bf16(GELU(acc + bias)).
__device__ __forceinline__ void sf_epilogue_gelu(uint32_t t_addr, const float* bias, uint32_t image, const SfRow& r) {
  uint32_t a[32];
  tmem_ld_32cols(t_addr + r.col0, a);
  float v[32];
  sf_load_bias32(bias + r.col0, v);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] += __uint_as_float(a[i]);
#pragma unroll
  for (int i = 0; i < 32; i += 2) gelu_erf_x2(v[i], v[i + 1]);
#pragma unroll
  for (int q = 0; q < 4; ++q) sf_store8(image, r.row, r.col0 + 8 * q, v + 8 * q);
}

// image[row, group columns] = bf16(acc) (the attention output).
__device__ __forceinline__ void sf_epilogue_copy(uint32_t t_addr, uint32_t image, const SfRow& r) {
  uint32_t a[32];
  tmem_ld_32cols(t_addr + r.col0, a);
  tmem_wait_ld();
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(a[i]);
#pragma unroll
  for (int q = 0; q < 4; ++q) sf_store8(image, r.row, r.col0 + 8 * q, v + 8 * q);
}

// LayerNorm of the row whose group columns are v (two-pass, as the standalone
// kernel), into the row of an operand image (bf16) or of an fp32 global row.
// Packed f32x2 arithmetic: each lane of a packed op is one IEEE fp32 operation.
template <bool kToGlobal>
__device__ __forceinline__ void sf_layer_norm(SfRow& r, const float* v, float eps, const float* gamma,
                                              const float* beta, uint32_t image, float* out_row) {
  // Each group's sum and squared deviations about its own mean (two passes
  // in registers), then one exchange: the row's mean and M2 by the pairwise
  // merge of Chan, Golub and LeVeque for four groups of 32.
  uint64_t s2 = f32x2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 32; i += 2) s2 = add_f32x2(s2, f32x2(v[i], v[i + 1]));
  const float2 sv = unpack_f32x2(s2);
  const float gsum = sv.x + sv.y;
  const float gmean = gsum * (1.0f / 32);
  const uint64_t gmean2 = f32x2(gmean, gmean);
  uint64_t q2 = f32x2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    const uint64_t d = sub_f32x2(f32x2(v[i], v[i + 1]), gmean2);
    q2 = fma_f32x2(d, d, q2);
  }
  const float2 qv = unpack_f32x2(q2);
  float2 part[4];
  sf_row_pairs(r, gsum, qv.x + qv.y, part);
  const float mean = ((part[0].x + part[1].x) + (part[2].x + part[3].x)) * (1.0f / kSfD);
  float m2 = 0.f;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const float dm = part[g].x * (1.0f / 32) - mean;
    m2 += part[g].y + 32.0f * dm * dm;
  }
  const uint64_t mean2 = f32x2(mean, mean);
  const float rstd = rsqrtf(m2 * (1.0f / kSfD) + eps);
  const uint64_t rstd2 = f32x2(rstd, rstd);
  float g[32], b[32];
  sf_load_bias32(gamma + r.col0, g);
  sf_load_bias32(beta + r.col0, b);
  float n[32];
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    const uint64_t t = mul_f32x2(sub_f32x2(f32x2(v[i], v[i + 1]), mean2), rstd2);
    const float2 o = unpack_f32x2(fma_f32x2(t, f32x2(g[i], g[i + 1]), f32x2(b[i], b[i + 1])));
    n[i] = o.x;
    n[i + 1] = o.y;
  }
  if constexpr (kToGlobal) {
    if (out_row != nullptr) {  // null: a padding row past the input (every thread joins the reductions)
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(out_row + r.col0 + i) = make_float4(n[i], n[i + 1], n[i + 2], n[i + 3]);
    }
  } else {
#pragma unroll
    for (int qd = 0; qd < 4; ++qd) sf_store8(image, r.row, r.col0 + 8 * qd, n + 8 * qd);
  }
}

// r += bf16(acc + bias) in the residual's group columns; the new values in v.
__device__ __forceinline__ void sf_residual_add(uint32_t t_acc, uint32_t t_res, const float* bias, const SfRow& r,
                                                float* v) {
  uint32_t a[32], res[32];
  tmem_ld_32cols(t_acc + r.col0, a);
  tmem_ld_32cols(t_res + r.col0, res);
  float b[32];
  sf_load_bias32(bias + r.col0, b);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    const float2 u = unpack_f32x2(
        add_f32x2(f32x2(__uint_as_float(a[i]), __uint_as_float(a[i + 1])), f32x2(b[i], b[i + 1])));
    const float2 ur = __bfloat1622float2(__floats2bfloat162_rn(u.x, u.y));  // the update as the program stores it
    const float2 o = unpack_f32x2(
        add_f32x2(f32x2(__uint_as_float(res[i]), __uint_as_float(res[i + 1])), f32x2(ur.x, ur.y)));
    v[i] = o.x;
    v[i + 1] = o.y;
    res[i] = __float_as_uint(o.x);
    res[i + 1] = __float_as_uint(o.y);
  }
  tmem_st_32cols(t_res + r.col0, res);
  tmem_wait_st();
}

// Causal softmax of the row's scores within its sequence, normalised and
// rounded to bf16, into the probability image.  The group's 32 keys are read
// only if they lie in the warp's sequences (warp-uniform: the sequence length
// is a multiple of 32); only the diagonal group holds keys past the row.  The
// other groups write zeros.  The max is taken on the raw scores (the scale is
// positive) and the scale folded into the exponent: 2^(s * scale - max * scale).
__device__ __forceinline__ void sf_softmax(uint32_t t_addr, uint32_t image, SfRow& r, int quarter, int seq,
                                           float scale_log2) {
  const int c_lo = ((quarter * 32) / seq) * seq / 32;
  const bool needed = r.grp >= c_lo && r.grp <= quarter;
  float x[32];
  float mx = -INFINITY;
  if (needed) {
    uint32_t a[32];
    tmem_ld_32cols(t_addr + r.col0, a);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) x[i] = __uint_as_float(a[i]);
    if (r.grp == quarter) {
      const int last = r.row - r.col0;  // keys col0 + i allowed for i <= last
#pragma unroll
      for (int i = 0; i < 32; ++i) x[i] = i <= last ? x[i] : -INFINITY;
    }
    float m0 = x[0], m1 = x[1];
#pragma unroll
    for (int i = 2; i < 32; i += 2) {
      m0 = fmaxf(m0, x[i]);
      m1 = fmaxf(m1, x[i + 1]);
    }
    mx = fmaxf(m0, m1);
  }
  // Exponentials and their sum against the group's own maximum, then one
  // exchange of (max, sum) per group: the row's maximum M, its sum
  // l = sum_g l_g 2^((m_g - M) scale) and this group's factor
  // 2^((m_g - M) scale) / l.  The diagonal group is never empty, so M is
  // finite; a group above the diagonal has m_g = -inf and l_g = 0.
  uint64_t sum2 = f32x2(0.f, 0.f);
  if (needed) {
    const uint64_t sc = f32x2(scale_log2, scale_log2);
    const uint64_t off = f32x2(-mx * scale_log2, -mx * scale_log2);
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      const float2 t = unpack_f32x2(fma_f32x2(f32x2(x[i], x[i + 1]), sc, off));
      x[i] = fast_exp2(t.x);
      x[i + 1] = fast_exp2(t.y);
      sum2 = add_f32x2(sum2, f32x2(x[i], x[i + 1]));
    }
  }
  const float2 sv = unpack_f32x2(sum2);
  float2 part[4];
  sf_row_pairs(r, mx, sv.x + sv.y, part);
  const float row_max = fmaxf(fmaxf(part[0].x, part[1].x), fmaxf(part[2].x, part[3].x));
  float total = 0.f;
#pragma unroll
  for (int g = 0; g < 4; ++g) total += part[g].y * fast_exp2((part[g].x - row_max) * scale_log2);
  const float inv = needed ? fast_exp2((mx - row_max) * scale_log2) / total : 0.f;
  const uint64_t inv2 = f32x2(inv, inv);
  float p[32];
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    const float2 o = needed ? unpack_f32x2(mul_f32x2(f32x2(x[i], x[i + 1]), inv2)) : make_float2(0.f, 0.f);
    p[i] = o.x;
    p[i + 1] = o.y;
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) sf_store8(image, r.row, r.col0 + 8 * q, p + 8 * q);
}

__global__ void __launch_bounds__(kSfThreads, 1) seq_forward_kernel(const __grid_constant__ SeqForwardArgs args) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t wbar[2];  // weight slot s landed
  __shared__ uint64_t tbar[3];  // UMMA into T1 / T2 / T3 complete
  __shared__ uint64_t pbar[2];  // P . V of the head using probability image 0 (P) / 1 (A) complete
  __shared__ uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  __shared__ float2 red2[2 * 4 * kSfRows];  // row-reduction partials, (a, b) per group

  uint8_t* smem = align_1024(smem_raw);
  const uint32_t img_a = smem_u32(smem);
  const uint32_t img_q = img_a + kSfMatBytes;
  const uint32_t img_k = img_a + 2 * kSfMatBytes;
  const uint32_t img_vt = img_a + 3 * kSfMatBytes;
  uint8_t* const w_ptr[2] = {smem + 4 * kSfMatBytes, smem + 5 * kSfMatBytes};
  const uint32_t img_w[2] = {img_a + 4 * kSfMatBytes, img_a + 5 * kSfMatBytes};
  const uint32_t img_p = img_w[0];  // even heads' probabilities, while slot 0 is idle

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int quarter = warp & 3;  // TMEM lane quarter this warp may access
  SfRow rw;
  rw.row = quarter * 32 + (tid & 31);
  rw.grp = warp >> 2;
  rw.col0 = rw.grp * 32;
  rw.red2 = red2;
  rw.turn = 0;
  const int row = rw.row;

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&wbar[i], 1);
      mbar_init(&pbar[i], 1);
    }
    for (int i = 0; i < 3; ++i) mbar_init(&tbar[i], 1);
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t lanes = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
  const uint32_t tR = lanes, tT1 = lanes + 128, tT2 = lanes + 256, tT3 = lanes + 384;
  const uint32_t dT1 = tmem + 128, dT2 = tmem + 256, dT3 = tmem + 384;  // UMMA destinations
  griddep_wait();
  griddep_launch_dependents();

  const int head_dim = kSfD / args.heads;
  uint32_t wph[2] = {0u, 0u}, tph[3] = {0u, 0u, 0u}, pph[2] = {0u, 0u};
  int w_issued[2] = {0, 0}, w_waited[2] = {0, 0};
  bool mma_issued = false;
  bool failed = false;
  // Every thread waits for every event, in program order; the outcome is
  // voted CTA-wide, so a wait that runs out ends the tile loop everywhere.
  // A phase this thread saw complete is counted as passed even when the vote
  // fails, so the drain below waits only for what did not land.
  bool seen = false;
  auto wait_on = [&](uint64_t* bar, uint32_t& phase) -> bool {
    seen = mbar_wait(bar, phase, kErrSeqWait, &abort_flag);
    if (seen) phase ^= 1u;
    return __syncthreads_or(seen ? 0 : 1) == 0;
  };
  auto wait_w = [&](int s) -> bool {
    const bool ok = wait_on(&wbar[s], wph[s]);
    if (seen) ++w_waited[s];
    return ok;
  };
  auto load_w = [&](int s, const uint8_t* image) {
    if (tid == 0) {
      mbar_arrive_expect_tx(&wbar[s], kSfMatBytes);
      bulk_load(w_ptr[s], image, kSfMatBytes, &wbar[s]);
    }
    ++w_issued[s];
  };
  // Writes of this thread to operand images (generic proxy) and reads of
  // TMEM are complete and visible before thread 0 issues the next UMMA.
  auto operands_ready = [&]() {
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  };
  auto issue = [&](uint32_t d, uint32_t a, uint32_t b, int b_row0, int n, int k0, int k_len, uint64_t* bar) {
    if (tid == 0) {
      sf_mma(d, a, b, b_row0, n, k0, k_len);
      umma_commit(bar);
    }
    mma_issued = true;
  };
  const uint8_t* first_images = args.layers[0].w_img;
  for (int tile = static_cast<int>(blockIdx.x); tile < args.num_tiles && !failed; tile += gridDim.x) {
    const int64_t grow = static_cast<int64_t>(tile) * kSfRows + row;
    const bool in_range = grow < args.rows;
    const bool first_tile = tile == static_cast<int>(blockIdx.x);
    if (first_tile) {
      load_w(0, first_images + 0 * kSfMatBytes);  // layer 0: Wq, Wk
      load_w(1, first_images + 1 * kSfMatBytes);
    }
    // Input row -> residual (TMEM) and LN1 of layer 0 -> A.
    {
      float v[32];
      uint32_t r[32];
      const float4* xin = reinterpret_cast<const float4*>(args.x + grow * kSfD + rw.col0);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 q = in_range ? __ldg(xin + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        v[4 * i] = q.x;
        v[4 * i + 1] = q.y;
        v[4 * i + 2] = q.z;
        v[4 * i + 3] = q.w;
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(v[i]);
      tmem_st_32cols(tR + rw.col0, r);
      tmem_wait_st();
      sf_layer_norm<false>(rw, v, args.eps, args.ln0_g, args.ln0_b, img_a, nullptr);
    }
    operands_ready();
    for (int l = 0; l < args.num_layers && !failed; ++l) {
      const SeqLayer& L = args.layers[l];
      const bool last_layer = l + 1 == args.num_layers;
      // Next images for slots 0 / 1 after this layer: the next layer's Wq /
      // Wk, or layer 0's of this CTA's next tile, or none.
      const uint8_t* next_images =
          !last_layer ? args.layers[l + 1].w_img
                      : (tile + static_cast<int>(gridDim.x) < args.num_tiles ? first_images : nullptr);
      // --- Q and K projections
      if (!wait_w(0) || !wait_w(1)) { failed = true; break; }
      issue(dT1, img_a, img_w[0], 0, 128, 0, kSfD, &tbar[0]);
      issue(dT2, img_a, img_w[1], 0, 128, 0, kSfD, &tbar[1]);
      if (!wait_on(&tbar[0], tph[0])) { failed = true; break; }
      load_w(0, L.w_img + 2 * kSfMatBytes);  // Wv
      sf_epilogue_proj(tT1, L.b_qkv, img_q, rw);
      // --- V projection (A still holds n), running under K's epilogue
      if (!wait_w(0)) { failed = true; break; }
      issue(dT3, img_a, img_w[0], 0, 128, 0, kSfD, &tbar[2]);
      if (!wait_on(&tbar[1], tph[1])) { failed = true; break; }
      load_w(1, L.w_img + 3 * kSfMatBytes);  // Wo
      sf_epilogue_proj(tT2, L.b_qkv + kSfD, img_k, rw);
      if (!wait_on(&tbar[2], tph[2])) { failed = true; break; }
      sf_epilogue_vt(tT3, L.b_qkv + 2 * kSfD, img_vt, rw);
      operands_ready();
      // --- attention: S_h into T1 / T2 alternately, P_h into P / A alternately
      issue(dT1, img_q, img_k, 0, 128, 0, head_dim, &tbar[0]);
      if (args.heads > 1) issue(dT2, img_q, img_k, 0, 128, head_dim, head_dim, &tbar[1]);
      for (int h = 0; h < args.heads; ++h) {
        const int b = h & 1;
        if (!wait_on(&tbar[b], tph[b])) { failed = true; break; }
        if (h >= 2 && !wait_on(&pbar[b], pph[b])) { failed = true; break; }  // P . V of head h - 2
        const uint32_t img_prob = b ? img_a : img_p;
        sf_softmax(b ? tT2 : tT1, img_prob, rw, quarter, args.seq, args.scale_log2);
        operands_ready();
        issue(dT3 + h * head_dim, img_prob, img_vt, h * head_dim, head_dim, 0, kSfRows, &pbar[b]);
        if (h + 2 < args.heads) issue(b ? dT2 : dT1, img_q, img_k, 0, 128, (h + 2) * head_dim, head_dim, &tbar[b]);
      }
      if (failed) break;
      for (int h = args.heads >= 2 ? args.heads - 2 : 0; h < args.heads; ++h)
        if (!wait_on(&pbar[h & 1], pph[h & 1])) { failed = true; break; }
      if (failed) break;
      load_w(0, L.w_img + 4 * kSfMatBytes);  // W1, into the slot the even heads' probabilities used
      // --- ctx = bf16(O) -> A (odd heads' probabilities are consumed)
      sf_epilogue_copy(tT3, img_a, rw);
      operands_ready();
      // --- out-projection, residual add, LN2 -> A
      if (!wait_w(1)) { failed = true; break; }
      issue(dT1, img_a, img_w[1], 0, 128, 0, kSfD, &tbar[0]);
      if (!wait_on(&tbar[0], tph[0])) { failed = true; break; }
      load_w(1, L.w_img + 5 * kSfMatBytes);  // W2
      {
        float v[32];
        sf_residual_add(tT1, tR, L.b_o, rw, v);
        sf_layer_norm<false>(rw, v, args.eps, L.ln2_g, L.ln2_b, img_a, nullptr);
      }
      operands_ready();
      // --- FFN in: A = bf16(GELU(n2 W1^T + b1))
      if (!wait_w(0)) { failed = true; break; }
      issue(dT2, img_a, img_w[0], 0, 128, 0, kSfD, &tbar[1]);
      if (!wait_on(&tbar[1], tph[1])) { failed = true; break; }
      if (next_images != nullptr) load_w(0, next_images + 0 * kSfMatBytes);
      sf_epilogue_gelu(tT2, L.b_1, img_a, rw);
      operands_ready();
      // --- FFN out, residual add, next LN -> A (or the output)
      if (!wait_w(1)) { failed = true; break; }
      issue(dT1, img_a, img_w[1], 0, 128, 0, kSfD, &tbar[0]);
      if (!wait_on(&tbar[0], tph[0])) { failed = true; break; }
      if (next_images != nullptr) load_w(1, next_images + 1 * kSfMatBytes);
      {
        float v[32];
        sf_residual_add(tT1, tR, L.b_2, rw, v);
        if (!last_layer)
          sf_layer_norm<false>(rw, v, args.eps, L.next_g, L.next_b, img_a, nullptr);
        else
          sf_layer_norm<true>(rw, v, args.eps, L.next_g, L.next_b, 0u, in_range ? args.out + grow * kSfD : nullptr);
      }
      operands_ready();
    }
  }
  // Leave with nothing in flight: the weight copies not yet waited for, and
  // every UMMA issued (a commit after them all).
  if (tid == 0) {
    for (int s = 0; s < 2; ++s)
      for (; w_waited[s] < w_issued[s]; ++w_waited[s]) {
        mbar_drain_wait(&wbar[s], wph[s]);
        wph[s] ^= 1u;
      }
    if (mma_issued) {
      umma_commit(&drain_bar);
      mbar_drain_wait(&drain_bar, 0);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}
}  // namespace b200tx
