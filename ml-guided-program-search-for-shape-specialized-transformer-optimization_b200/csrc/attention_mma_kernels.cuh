// attention_mma_kernels.cuh -- flash attention for head_dim 8, 16, 32, 64 and 128
// on the warp-level tensor-core instruction mma.sync.m16n8k16 (bf16 in, fp32
// out).
//
// The tcgen05 kernels are built for head_dim 64 and sized for long sequences.
// The reference's official benchmark shapes (official/test_shapes.json) use
// head dims 8, 32, 64 and 128 on short sequences (S <= 1024), where the
// CUDA-core kernel is latency-bound (one query row per one to eight threads,
// keys walked serially).  For these shapes each warp
// keeps its 16 query rows' Q fragments in registers and issues m16n8k16 MMAs:
// the scores of a 64-key tile are 8 accumulator tiles, the probabilities go
// back into A fragments without leaving registers (an accumulator's row/column
// layout is the A operand's), and P.V accumulates the 16 x Dh output.
//
// Semantics as the other attention kernels (official/torch_transformer_
// benchmark.py:95-118): softmax(q k^T * scale, causal -inf, key-padding -inf)
// in fp32 with an online running max and sum, probabilities rounded to bf16
// before P.V (the reference casts them to the activation dtype), fp32
// accumulation; reads the packed [B, S, 3, H, Dh] projection and writes
// [B, S, H, Dh].  A query that sees no valid key writes a zero row.
//
// Layout: CTA = 64 query rows (4 warps x 16) of one (batch, head); KV tiles of
// 64 keys are staged in shared memory, K and V row-major (key, dim): K's B
// fragments are single 32-bit loads, V's come transposed from ldmatrix .trans.
// Row strides are padded by 8 elements, which makes both free of bank
// conflicts.  The grid lists all heads' last query blocks first, so that
// under a causal mask the longest blocks start first.  There are no waits on
// other CTAs or on asynchronous copies: only __syncthreads.
//
// Fragment layouts (PTX ISA, mma.m16n8k16 with .bf16): g = lane / 4,
// t = lane % 4.  A (16 x 16, row-major): reg0 = (row g, cols 2t, 2t+1),
// reg1 = (row g+8, cols 2t..), reg2 = (row g, cols 2t+8..), reg3 = (row g+8,
// cols 2t+8..).  B (16 x 8, k x n): reg0 = (k 2t, 2t+1; n g), reg1 = (k 2t+8,
// 2t+9; n g).  C (16 x 8): c0, c1 = (row g, cols 2t, 2t+1), c2, c3 = (row g+8).
#pragma once

#include "sm100_common.cuh"

namespace b200tx {

constexpr int kMmaAttnRows = 64;  // query rows per CTA (4 warps x 16)
constexpr int kMmaAttnKeys = 64;  // keys per KV tile
constexpr int kMmaAttnThreads = 128;

struct MmaAttnArgs {
  const __nv_bfloat16* qkv;  // [B, S, 3, H, Dh]
  const uint8_t* key_valid;  // [B, S] or null
  __nv_bfloat16* out;        // [B, S, H, Dh]
  int batch, seq, heads;
  int q_blocks;              // ceil(seq / kMmaAttnRows)
  float scale_log2;          // scale * log2(e)
  int causal;
};

__device__ __forceinline__ void mma_m16n8k16_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                  uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t ld_u32(const __nv_bfloat16* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}

// Copy N 16-byte chunks with THREADS threads, every load of this thread in
// flight before its first store: load(i) returns chunk i (zero-filled out of
// range), store(i, v) writes it.  A loop that stores each chunk right after
// loading it waits one memory round trip per chunk, since the store stalls on
// its load and instructions issue in order.
template <int N, int THREADS, typename Load, typename Store>
__device__ __forceinline__ void copy_chunks(Load load, Store store) {
  constexpr int PER = (N + THREADS - 1) / THREADS;
  uint4 v[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int i = static_cast<int>(threadIdx.x) + j * THREADS;
    v[j] = (N % THREADS == 0 || i < N) ? load(i) : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int i = static_cast<int>(threadIdx.x) + j * THREADS;
    if (N % THREADS == 0 || i < N) store(i, v[j]);
  }
}

template <int DH>
__global__ void __launch_bounds__(kMmaAttnThreads) attention_mma_kernel(MmaAttnArgs args) {
  static_assert(DH == 8 || DH == 16 || DH == 32 || DH == 64 || DH == 128,
                "built for head_dim 8, 16, 32, 64 and 128");
  constexpr int KSTEPS = (DH + 15) / 16;    // k-steps of Q.K^T (DH = 8 is zero-padded to 16)
  constexpr int OUT_TILES = DH / 8;          // n-tiles of the 16 x DH output
  constexpr int S_TILES = kMmaAttnKeys / 8;  // n-tiles of the 16 x 64 scores
  constexpr int KSTR = DH + 8;               // K row stride (elements)
  constexpr int CHUNKS = kMmaAttnKeys * DH / 8;  // 16-byte chunks per K (or V) tile
  __shared__ __align__(16) __nv_bfloat16 k_s[kMmaAttnKeys * KSTR];
  __shared__ __align__(16) __nv_bfloat16 v_s[kMmaAttnKeys * KSTR];
  __shared__ float key_bias[kMmaAttnKeys];  // 0, or -inf for a padding key or one past S

  griddep_wait();
  griddep_launch_dependents();

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;
  const int t = lane & 3;
  const int bh_count = args.batch * args.heads;
  const int q_block = args.q_blocks - 1 - static_cast<int>(blockIdx.x / bh_count);
  const int bh = static_cast<int>(blockIdx.x % bh_count);
  const int head = bh % args.heads;
  const int b = bh / args.heads;
  const int S = args.seq;
  const int d_model = args.heads * DH;
  const int64_t tok = 3LL * d_model;  // elements per token of the packed projection
  const __nv_bfloat16* q_base = args.qkv + static_cast<int64_t>(b) * S * tok + head * DH;
  const __nv_bfloat16* k_base = q_base + d_model;
  const __nv_bfloat16* v_base = q_base + 2 * d_model;
  const uint8_t* valid = args.key_valid != nullptr ? args.key_valid + static_cast<int64_t>(b) * S : nullptr;

  const int q0 = q_block * kMmaAttnRows;
  const int r0 = q0 + warp * 16 + g;  // this thread's two query rows
  const int r1 = r0 + 8;

  // Q fragments for the whole KV loop (zero beyond S and beyond DH).
  uint32_t qf[KSTEPS][4];
#pragma unroll
  for (int ks = 0; ks < KSTEPS; ++ks) {
    const int c = ks * 16 + 2 * t;
    qf[ks][0] = (r0 < S && c < DH) ? ld_u32(q_base + r0 * tok + c) : 0u;
    qf[ks][1] = (r1 < S && c < DH) ? ld_u32(q_base + r1 * tok + c) : 0u;
    qf[ks][2] = (r0 < S && c + 8 < DH) ? ld_u32(q_base + r0 * tok + c + 8) : 0u;
    qf[ks][3] = (r1 < S && c + 8 < DH) ? ld_u32(q_base + r1 * tok + c + 8) : 0u;
  }

  float o[OUT_TILES][4];
#pragma unroll
  for (int i = 0; i < OUT_TILES; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY;  // running row max (log2 domain)
  float l0 = 0.f, l1 = 0.f;              // this thread's share of the running row sums

  const int kv_tiles = (S + kMmaAttnKeys - 1) / kMmaAttnKeys;
  const int last_tile = args.causal ? min(kv_tiles - 1, q_block) : kv_tiles - 1;
  for (int j = 0; j <= last_tile; ++j) {
    const int k0 = j * kMmaAttnKeys;
    __syncthreads();  // the previous tile's fragments have been read
    // Chunk i < CHUNKS is K's, i >= CHUNKS is V's (same key / column split).
    copy_chunks<2 * CHUNKS, kMmaAttnThreads>(
        [&](int i) {
          const bool is_v = i >= CHUNKS;
          const int ci = is_v ? i - CHUNKS : i;
          const int key = ci / (DH / 8);
          const int c = (ci % (DH / 8)) * 8;
          if (k0 + key >= S) return make_uint4(0u, 0u, 0u, 0u);
          return *reinterpret_cast<const uint4*>((is_v ? v_base : k_base) +
                                                 static_cast<int64_t>(k0 + key) * tok + c);
        },
        [&](int i, uint4 v) {
          const bool is_v = i >= CHUNKS;
          const int ci = is_v ? i - CHUNKS : i;
          const int key = ci / (DH / 8);
          const int c = (ci % (DH / 8)) * 8;
          *reinterpret_cast<uint4*>(&(is_v ? v_s : k_s)[key * KSTR + c]) = v;
        });
    if (threadIdx.x < kMmaAttnKeys) {
      const int key = k0 + threadIdx.x;
      const bool ok = key < S && (valid == nullptr || valid[key] != 0);
      key_bias[threadIdx.x] = ok ? 0.f : -INFINITY;
    }
    __syncthreads();

    // Scores of 16 rows x 64 keys.
    float s[S_TILES][4];
#pragma unroll
    for (int n = 0; n < S_TILES; ++n) {
      s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
      const __nv_bfloat16* krow = &k_s[(n * 8 + g) * KSTR];
#pragma unroll
      for (int ks = 0; ks < KSTEPS; ++ks) {
        const uint32_t b0 = ld_u32(krow + ks * 16 + 2 * t);
        const uint32_t b1 = (ks * 16 + 8 < DH) ? ld_u32(krow + ks * 16 + 8 + 2 * t) : 0u;
        mma_m16n8k16_bf16(s[n], qf[ks], b0, b1);
      }
    }
    // Scale into the log2 domain; padding, beyond-S and causal keys to -inf.
    const bool diagonal = args.causal && k0 + kMmaAttnKeys - 1 > q0 + warp * 16;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int n = 0; n < S_TILES; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kk = n * 8 + 2 * t + (e & 1);
        float v = fmaf(s[n][e], args.scale_log2, key_bias[kk]);
        if (diagonal && k0 + kk > ((e < 2) ? r0 : r1)) v = -INFINITY;
        s[n][e] = v;
      }
      mx0 = fmaxf(mx0, fmaxf(s[n][0], s[n][1]));
      mx1 = fmaxf(mx1, fmaxf(s[n][2], s[n][3]));
    }
    // The four lanes of a row group hold its 64 scores.
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0);
    const float mn1 = fmaxf(m1, mx1);
    // A row that has seen no valid key keeps m = -inf and exponentiates
    // against 0, so every p is 0 (no inf - inf).
    const float base0 = mn0 == -INFINITY ? 0.f : mn0;
    const float base1 = mn1 == -INFINITY ? 0.f : mn1;
    const float corr0 = fast_exp2(m0 - base0);  // 0 while m0 = -inf
    const float corr1 = fast_exp2(m1 - base1);
    m0 = mn0;
    m1 = mn1;
    l0 *= corr0;
    l1 *= corr1;
#pragma unroll
    for (int i = 0; i < OUT_TILES; ++i) {
      o[i][0] *= corr0;
      o[i][1] *= corr0;
      o[i][2] *= corr1;
      o[i][3] *= corr1;
    }
    // P (bf16) straight into A fragments: key k-step kk covers score tiles
    // 2kk (cols 2t..) and 2kk+1 (cols 2t+8..).
    uint32_t pf[S_TILES][2];
#pragma unroll
    for (int n = 0; n < S_TILES; ++n) {
      const float p0 = fast_exp2(s[n][0] - base0);
      const float p1 = fast_exp2(s[n][1] - base0);
      const float p2 = fast_exp2(s[n][2] - base1);
      const float p3 = fast_exp2(s[n][3] - base1);
      l0 += p0 + p1;
      l1 += p2 + p3;
      pf[n][0] = pack_bf16x2(p0, p1);
      pf[n][1] = pack_bf16x2(p2, p3);
    }
#pragma unroll
    for (int kk = 0; kk < kMmaAttnKeys / 16; ++kk) {
      const uint32_t a[4] = {pf[2 * kk][0], pf[2 * kk][1], pf[2 * kk + 1][0], pf[2 * kk + 1][1]};
#pragma unroll
      for (int i = 0; i < OUT_TILES; ++i) {
        // V is row-major (key, dim) in shared memory; ldmatrix .trans hands each
        // lane the (2t, 2t+1; g) key pairs of the B fragment.  Lanes 0-7 give the
        // rows of keys kk*16 + 0..7, lanes 8-15 those of kk*16 + 8..15.
        uint32_t b0, b1;
        const uint32_t addr = smem_u32(&v_s[(kk * 16 + (lane & 15)) * KSTR + i * 8]);
        asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];\n"
                     : "=r"(b0), "=r"(b1)
                     : "r"(addr));
        mma_m16n8k16_bf16(o[i], a, b0, b1);
      }
    }
  }

  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? 1.0f / l0 : 0.f;
  const float inv1 = l1 > 0.f ? 1.0f / l1 : 0.f;
  __nv_bfloat16* out0 = args.out + (static_cast<int64_t>(b) * S + r0) * d_model + head * DH + 2 * t;
  __nv_bfloat16* out1 = out0 + 8LL * d_model;
#pragma unroll
  for (int i = 0; i < OUT_TILES; ++i) {
    if (r0 < S) *reinterpret_cast<uint32_t*>(out0 + i * 8) = pack_bf16x2(o[i][0] * inv0, o[i][1] * inv0);
    if (r1 < S) *reinterpret_cast<uint32_t*>(out1 + i * 8) = pack_bf16x2(o[i][2] * inv1, o[i][3] * inv1);
  }
}

}  // namespace b200tx
