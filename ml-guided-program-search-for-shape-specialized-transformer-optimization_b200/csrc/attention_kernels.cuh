// attention_kernels.cuh -- causal flash attention forward for head_dim 64 on the
// sm_100 tensor cores, reading Q/K/V straight out of the packed QKV projection
// and writing the context in [B, S, H*64] (BSD) order for the out-projection.
//
// Replaces the reference's attention primitives:
//   streaming Dh64 kernel   solution/shape14/triton_streaming_dh64.py:68-190
//   shape13 Dh32 kernel     solution/kernels/attention/triton_s1024_dh32.py:72-265
//   query-blocked reference solution/operators/attention/sdpa.py:116-170
// Semantics (official/torch_transformer_benchmark.py:95-118):
//   softmax(Q K^T * Dh^-1/2, causal -inf above the diagonal) computed in fp32,
//   probabilities cast to the activation dtype (bf16 here), times V.
// No [S, S] tensor exists anywhere: scores live in TMEM one 128x128 tile at a
// time and the softmax keeps its running max and sum in registers.
//
// One CTA = one 128-row query tile of one (batch, head); 192 threads, two CTAs
// per SM so one CTA's softmax overlaps the other's MMAs.
//   warp 0      TMA: Q once, then K_j, V_j through a 3-slot ring of 16 KB tiles
//   warp 1      one thread issues S = Q K_j^T (4 x 128x128x16 UMMAs) and
//               O += P_j V_j (8 x 128x64x16 UMMAs, V consumed MN-major)
//   warps 2..5  softmax, one query row per thread: two passes over the S row in
//               TMEM (max, then exp2 / sum / bf16 P into swizzled shared memory)
// TMEM: S in columns [0,128), O in columns [128,192) of a 256-column allocation.
// The running max is only moved when a row's maximum grows by more than 8 (in
// log2 units); until then P may reach 2^8, which fp32 O and l absorb exactly as
// if the max had been moved, and O is rescaled in TMEM only for such warps.
// Query tiles are dispatched longest-first (diagonal tile index descending)
// so the causal triangle balances across the grid.
#pragma once

#include "sm100_common.cuh"

namespace b200tx {

constexpr int kAttnBM = 128;
constexpr int kAttnBN = 128;
constexpr int kAttnDh = 64;
constexpr int kAttnRing = 3;
constexpr int kAttnThreads = 192;
constexpr uint32_t kAttnTmemCols = 256;
constexpr uint32_t kAttnTmemO = 128;
constexpr uint32_t kAttnTileBytes = kAttnBM * kAttnDh * 2;  // 16 KB (Q, K or V tile)
constexpr uint32_t kAttnPHalfBytes = kAttnBM * 64 * 2;      // 16 KB: 64 key columns of P
constexpr size_t kAttnSmemBytes =
    1024 + kAttnTileBytes * (1 + kAttnRing) + 2 * kAttnPHalfBytes;  // 97 KB

struct AttnArgs {
  __nv_bfloat16* out;  // [B, S, H*64]
  // [B, S] 0/1 padding mask of the keys (official/torch_transformer_benchmark.py:
  // 105-108), or null when every key is valid.  Read by the masked quad build.
  const uint8_t* key_valid;
  int batch;
  int seq;
  int heads;
  int num_q_tiles;
  float scale_log2;  // Dh^-1/2 * log2(e)
  int causal;
};

__global__ void __launch_bounds__(kAttnThreads, 2)
    attention_fwd_dh64_kernel(const __grid_constant__ CUtensorMap tmap_qkv, AttnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t q_full_bar;
  __shared__ uint64_t ring_full_bar[kAttnRing];
  __shared__ uint64_t ring_empty_bar[kAttnRing];
  __shared__ uint64_t s_full_bar;
  __shared__ uint64_t p_full_bar;
  __shared__ uint64_t o_done_bar;
  __shared__ uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  uint8_t* smem = align_1024(smem_raw);
  uint8_t* smem_q = smem;
  uint8_t* smem_ring = smem + kAttnTileBytes;
  uint8_t* smem_p = smem_ring + kAttnRing * kAttnTileBytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Longest query tiles first.
  const int hb_count = args.heads * args.batch;
  const int q_tile = args.num_q_tiles - 1 - static_cast<int>(blockIdx.x / hb_count);
  const int hb = static_cast<int>(blockIdx.x % hb_count);
  const int head = hb % args.heads;
  const int batch = hb / args.heads;
  const int kv_tiles_total = (args.seq + kAttnBN - 1) / kAttnBN;
  const int n_kv = args.causal ? (q_tile + 1) : kv_tiles_total;
  const int d_model = args.heads * kAttnDh;

  if (threadIdx.x == 0) {
    prefetch_tensor_map(&tmap_qkv);
    mbar_init(&q_full_bar, 1);
    for (int s = 0; s < kAttnRing; ++s) {
      mbar_init(&ring_full_bar[s], 1);
      mbar_init(&ring_empty_bar[s], 1);
    }
    mbar_init(&s_full_bar, 1);
    mbar_init(&p_full_bar, 128);
    mbar_init(&o_done_bar, 1);
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, kAttnTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(&q_full_bar, kAttnTileBytes);
      tma_load_3d(smem_q, &tmap_qkv, &q_full_bar, head * kAttnDh, q_tile * kAttnBM, batch);
      const int items = 2 * n_kv;  // K_0, V_0, K_1, V_1, ...
      int issued = 0;
      for (int i = 0; i < items; ++i) {
        const int slot = i % kAttnRing;
        const uint32_t ph = (i / kAttnRing) & 1;
        if (!mbar_wait(&ring_empty_bar[slot], ph ^ 1u, kErrAttnProducerWait, &abort_flag)) break;
        mbar_arrive_expect_tx(&ring_full_bar[slot], kAttnTileBytes);
        const int j = i >> 1;
        const int col = (i & 1 ? 2 * d_model : d_model) + head * kAttnDh;
        tma_load_3d(smem_ring + slot * kAttnTileBytes, &tmap_qkv, &ring_full_bar[slot], col,
                    j * kAttnBN, batch);
        ++issued;
      }
      // Wait for the loads still in flight (complete already on the normal path).
      volatile int no_abort = 0;
      mbar_wait(&q_full_bar, 0, kErrAttnProducerWait, &no_abort);
      const int first = issued > kAttnRing ? issued - kAttnRing : 0;
      for (int i = first; i < issued; ++i) {
        mbar_wait(&ring_full_bar[i % kAttnRing], (i / kAttnRing) & 1, kErrAttnProducerWait,
                  &no_abort);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_qk = umma_idesc_bf16(kAttnBM, kAttnBN, false, false);
      constexpr uint32_t idesc_pv = umma_idesc_bf16(kAttnBM, kAttnDh, false, true);
      const uint32_t q_addr = smem_u32(smem_q);
      const uint32_t p_addr = smem_u32(smem_p);
      const uint32_t s_tmem = tmem_base;
      const uint32_t o_tmem = tmem_base + kAttnTmemO;
      bool issued_any = false;
      auto issue_qk = [&](int j) -> bool {
        const int i = 2 * j;
        const int slot = i % kAttnRing;
        if (!mbar_wait(&ring_full_bar[slot], (i / kAttnRing) & 1, kErrAttnMmaWait, &abort_flag))
          return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem_ring + slot * kAttnTileBytes);
#pragma unroll
        for (int k = 0; k < kAttnDh / 16; ++k) {
          umma_bf16_ss(s_tmem, sw128_desc(q_addr + k * 32, 16, 1024),
                       sw128_desc(k_addr + k * 32, 16, 1024), idesc_qk, k != 0 ? 1u : 0u);
        }
        issued_any = true;
        umma_commit(&ring_empty_bar[slot]);
        umma_commit(&s_full_bar);
        return true;
      };
      bool ok = mbar_wait(&q_full_bar, 0, kErrAttnMmaWait, &abort_flag);
      if (ok) {
        tc_fence_after();
        ok = issue_qk(0);
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        // Softmax of tile j finished: S is free, P_j is in shared memory and O
        // has been rescaled where needed.
        if (!mbar_wait(&p_full_bar, j & 1, kErrAttnMmaWait, &abort_flag)) break;
        tc_fence_after();
        if (j + 1 < n_kv && !issue_qk(j + 1)) break;
        const int i = 2 * j + 1;
        const int slot = i % kAttnRing;
        if (!mbar_wait(&ring_full_bar[slot], (i / kAttnRing) & 1, kErrAttnMmaWait, &abort_flag))
          break;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem_ring + slot * kAttnTileBytes);
#pragma unroll
        for (int k = 0; k < kAttnBN / 16; ++k) {
          const uint32_t pa = p_addr + (k >> 2) * kAttnPHalfBytes + (k & 3) * 32;
          const uint32_t vb = v_addr + k * 16 * 128;  // 16 key rows of 128 B
          umma_bf16_ss(o_tmem, sw128_desc(pa, 16, 1024), sw128_desc(vb, kAttnTileBytes, 1024),
                       idesc_pv, (j | k) != 0 ? 1u : 0u);
        }
        umma_commit(&ring_empty_bar[slot]);
        umma_commit(&o_done_bar);
      }
      if (issued_any) {
        umma_commit(&drain_bar);
        volatile int no_abort = 0;
        mbar_wait(&drain_bar, 0, kErrAttnMmaWait, &no_abort);
      }
    }
  } else {
    // Softmax warps: warp w owns TMEM lanes 32*(w%4) .. +31 = query rows.
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int q_idx = q_tile * kAttnBM + row;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t p_row = smem_u32(smem_p) + row * 128;
    const uint32_t swz = row & 7;
    const float c = args.scale_log2;
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      ok = mbar_wait(&s_full_bar, j & 1, kErrAttnSoftmaxWait, &abort_flag);
      if (__any_sync(0xffffffffu, !ok)) {
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after();
      // Columns at or beyond `limit` are masked: above the diagonal on the
      // diagonal tile, beyond the sequence on a non-causal ragged last tile.
      int limit = kAttnBN;
      if (args.causal) {
        if (j == q_tile) limit = row + 1;
      } else if ((j + 1) * kAttnBN > args.seq) {
        limit = args.seq - j * kAttnBN;
      }
      // Pass 1: row maximum.
      float mx = -INFINITY;
#pragma unroll 1
      for (int cc = 0; cc < kAttnBN / 32; ++cc) {
        uint32_t r[32];
        tmem_ld_32cols(lane_base + cc * 32, r);
        tmem_wait_ld();
        if (limit >= (cc + 1) * 32) {
#pragma unroll
          for (int i = 0; i < 32; ++i) mx = fmaxf(mx, __uint_as_float(r[i]));
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (cc * 32 + i < limit) mx = fmaxf(mx, __uint_as_float(r[i]));
        }
      }
      const float mx_scaled = mx * c;
      const bool need = mx_scaled > m_run + 8.0f;
      const float m_new = need ? mx_scaled : m_run;
      // P_{j-1} and O are busy until the previous P.V has completed.
      if (j > 0) {
        ok = mbar_wait(&o_done_bar, (j - 1) & 1, kErrAttnSoftmaxWait, &abort_flag);
        if (__any_sync(0xffffffffu, !ok)) {
          ok = false;
          break;
        }
        __syncwarp();
        tc_fence_after();
      }
      // Pass 2: probabilities, row sum, bf16 P in the 128-byte-swizzled
      // K-major layout the UMMA descriptor expects.
      float sum = 0.f;
#pragma unroll 1
      for (int cc = 0; cc < kAttnBN / 32; ++cc) {
        uint32_t r[32];
        tmem_ld_32cols(lane_base + cc * 32, r);
        tmem_wait_ld();
        float p[32];
        if (limit >= (cc + 1) * 32) {
#pragma unroll
          for (int i = 0; i < 32; ++i) p[i] = fast_exp2(fmaf(__uint_as_float(r[i]), c, -m_new));
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            p[i] = (cc * 32 + i < limit) ? fast_exp2(fmaf(__uint_as_float(r[i]), c, -m_new)) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) sum += p[i];
        const uint32_t half_base = p_row + (cc >> 1) * kAttnPHalfBytes;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t chunk = (cc & 1) * 4 + q;  // 16-byte chunk within the 128-byte row
          const int b = q * 8;
          st_shared_v4(half_base + ((chunk ^ swz) << 4), pack_bf16x2(p[b], p[b + 1]),
                       pack_bf16x2(p[b + 2], p[b + 3]), pack_bf16x2(p[b + 4], p[b + 5]),
                       pack_bf16x2(p[b + 6], p[b + 7]));
        }
      }
      fence_proxy_async_smem();
      const float alpha = need ? fast_exp2(m_run - m_new) : 1.0f;  // exp2(-inf) = 0 on j == 0
      if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int cc = 0; cc < kAttnDh / 32; ++cc) {
          uint32_t r[32];
          tmem_ld_32cols(lane_base + kAttnTmemO + cc * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st_32cols(lane_base + kAttnTmemO + cc * 32, r);
        }
        tmem_wait_st();
      }
      l_run = l_run * alpha + sum;
      m_run = m_new;
      tc_fence_before();
      mbar_arrive(&p_full_bar);
    }
    if (ok) {
      ok = mbar_wait(&o_done_bar, (n_kv - 1) & 1, kErrAttnSoftmaxWait, &abort_flag);
      const bool all_ok = !__any_sync(0xffffffffu, !ok);
      __syncwarp();
      if (all_ok) {
        tc_fence_after();
        const float inv_l = 1.0f / l_run;
        __nv_bfloat16* out_row =
            args.out + (static_cast<int64_t>(batch) * args.seq + q_idx) * d_model + head * kAttnDh;
#pragma unroll 1
        for (int cc = 0; cc < kAttnDh / 32; ++cc) {
          uint32_t r[32];
          tmem_ld_32cols(lane_base + kAttnTmemO + cc * 32, r);
          tmem_wait_ld();
          if (q_idx < args.seq) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              st_global_v4(out_row + cc * 32 + i,
                           pack_bf16x2(__uint_as_float(r[i]) * inv_l, __uint_as_float(r[i + 1]) * inv_l),
                           pack_bf16x2(__uint_as_float(r[i + 2]) * inv_l, __uint_as_float(r[i + 3]) * inv_l),
                           pack_bf16x2(__uint_as_float(r[i + 4]) * inv_l, __uint_as_float(r[i + 5]) * inv_l),
                           pack_bf16x2(__uint_as_float(r[i + 6]) * inv_l, __uint_as_float(r[i + 7]) * inv_l));
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kAttnTmemCols);
  }
}


// ---------------------------------------------------------------------------
// Paired-tile variant: one CTA = two consecutive 128-row query tiles of one
// (batch, head), one CTA per SM, 320 threads.
//   warp 0      TMA: Q0/Q1 once; K_j and V_j through separate 3-slot rings
//   warp 1      one thread issues, per query tile w, S_w = Q_w K_j^T (SS UMMA)
//               and O_w += P_w V_j (TS UMMA: P read straight from TMEM),
//               ping-ponging the two tiles so one tile's MMAs run while the
//               other tile's softmax works
//   warps 2..5  softmax of query tile 0, warps 6..9 of query tile 1: one row per
//               thread, the whole 128-column S row loaded into registers in one
//               pass, bf16 P written back over S in TMEM (tcgen05.st)
// TMEM (512 columns): S0/P0 [0,128), S1/P1 [128,256), O0 [256,320), O1 [320,384).
// tcgen05.mma operations of one thread execute in issue order, so the
// S_w(j+1) UMMA, issued after O_w += P_w(j) V_j, never overwrites P_w(j) early,
// and the commit that signals S_w(j+1) also proves that P_w(j) V_j is done.
// ---------------------------------------------------------------------------
constexpr int kAttn2Threads = 320;
// The running max moves only once a row maximum exceeds it by this much (log2
// units): P may then reach 2^8, which fp32 exp2, fp32 O and fp32 l carry
// exactly, and O is rescaled in TMEM only on those rare steps.
constexpr float kAttnMaxSlack = 8.0f;
constexpr int kAttn2Ring = 3;
constexpr uint32_t kAttn2TmemCols = 512;
constexpr size_t kAttn2SmemBytes = 1024 + kAttnTileBytes * (2 + 2 * kAttn2Ring);  // 129 KB

__global__ void __launch_bounds__(kAttn2Threads, 1)
    attention_fwd_dh64_pair_kernel(const __grid_constant__ CUtensorMap tmap_qkv, AttnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t q_full_bar;
  __shared__ uint64_t k_full_bar[kAttn2Ring];
  __shared__ uint64_t k_empty_bar[kAttn2Ring];
  __shared__ uint64_t v_full_bar[kAttn2Ring];
  __shared__ uint64_t v_empty_bar[kAttn2Ring];
  __shared__ uint64_t s_full_bar[2];
  __shared__ uint64_t p_full_bar[2];
  __shared__ uint64_t o_final_bar[2];
  __shared__ uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  uint8_t* smem = align_1024(smem_raw);
  uint8_t* smem_q = smem;                                  // Q0, Q1
  uint8_t* smem_k = smem + 2 * kAttnTileBytes;             // K ring
  uint8_t* smem_v = smem_k + kAttn2Ring * kAttnTileBytes;  // V ring

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int num_pairs = (args.num_q_tiles + 1) >> 1;
  const int hb_count = args.heads * args.batch;
  const int pair = num_pairs - 1 - static_cast<int>(blockIdx.x / hb_count);  // longest first
  const int hb = static_cast<int>(blockIdx.x % hb_count);
  const int head = hb % args.heads;
  const int batch = hb / args.heads;
  const int kv_tiles_total = (args.seq + kAttnBN - 1) / kAttnBN;
  const int q_tile0 = 2 * pair;
  const bool active1 = q_tile0 + 1 < args.num_q_tiles;
  const int n_kv0 = args.causal ? q_tile0 + 1 : kv_tiles_total;
  const int n_kv1 = active1 ? (args.causal ? q_tile0 + 2 : kv_tiles_total) : 0;
  const int n_kv = n_kv0 > n_kv1 ? n_kv0 : n_kv1;
  const int d_model = args.heads * kAttnDh;

  if (threadIdx.x == 0) {
    prefetch_tensor_map(&tmap_qkv);
    mbar_init(&q_full_bar, 1);
    for (int s = 0; s < kAttn2Ring; ++s) {
      mbar_init(&k_full_bar[s], 1);
      mbar_init(&k_empty_bar[s], 1);
      mbar_init(&v_full_bar[s], 1);
      mbar_init(&v_empty_bar[s], 1);
    }
    for (int w = 0; w < 2; ++w) {
      mbar_init(&s_full_bar[w], 1);
      mbar_init(&p_full_bar[w], 128);
      mbar_init(&o_final_bar[w], 1);
    }
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, kAttn2TmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(&q_full_bar, (active1 ? 2u : 1u) * kAttnTileBytes);
      tma_load_3d(smem_q, &tmap_qkv, &q_full_bar, head * kAttnDh, q_tile0 * kAttnBM, batch);
      if (active1)
        tma_load_3d(smem_q + kAttnTileBytes, &tmap_qkv, &q_full_bar, head * kAttnDh,
                    (q_tile0 + 1) * kAttnBM, batch);
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int slot = j % kAttn2Ring;
        const uint32_t ph = (j / kAttn2Ring) & 1;
        if (!mbar_wait(&k_empty_bar[slot], ph ^ 1u, kErrAttnProducerWait, &abort_flag)) break;
        mbar_arrive_expect_tx(&k_full_bar[slot], kAttnTileBytes);
        tma_load_3d(smem_k + slot * kAttnTileBytes, &tmap_qkv, &k_full_bar[slot],
                    d_model + head * kAttnDh, j * kAttnBN, batch);
        if (!mbar_wait(&v_empty_bar[slot], ph ^ 1u, kErrAttnProducerWait, &abort_flag)) {
          ++issued;  // K_j is in flight
          break;
        }
        mbar_arrive_expect_tx(&v_full_bar[slot], kAttnTileBytes);
        tma_load_3d(smem_v + slot * kAttnTileBytes, &tmap_qkv, &v_full_bar[slot],
                    2 * d_model + head * kAttnDh, j * kAttnBN, batch);
        ++issued;
      }
      // Wait for the loads still in flight (complete already on the normal path).
      volatile int no_abort = 0;
      mbar_wait(&q_full_bar, 0, kErrAttnProducerWait, &no_abort);
      const int first = issued > kAttn2Ring ? issued - kAttn2Ring : 0;
      for (int j = first; j < issued; ++j) {
        const uint32_t ph = (j / kAttn2Ring) & 1;
        mbar_wait(&k_full_bar[j % kAttn2Ring], ph, kErrAttnProducerWait, &no_abort);
        mbar_wait(&v_full_bar[j % kAttn2Ring], ph, kErrAttnProducerWait, &no_abort);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_qk = umma_idesc_bf16(kAttnBM, kAttnBN, false, false);
      constexpr uint32_t idesc_pv = umma_idesc_bf16(kAttnBM, kAttnDh, false, true);
      const uint32_t q_addr = smem_u32(smem_q);
      bool issued_any = false;
      // S_w = Q_w K_j^T; commits s_full[w] and, when K_j has no further user,
      // frees its ring slot.
      auto issue_qk = [&](int w, int j) -> bool {
        const int slot = j % kAttn2Ring;
        if (w == 0 || !(j < n_kv0)) {  // first user of K_j waits for it
          if (!mbar_wait(&k_full_bar[slot], (j / kAttn2Ring) & 1, kErrAttnMmaWait, &abort_flag))
            return false;
          tc_fence_after();
        }
        const uint32_t k_addr = smem_u32(smem_k + slot * kAttnTileBytes);
        const uint32_t qa = q_addr + w * kAttnTileBytes;
        const uint32_t s_tmem = tmem_base + w * kAttnBN;
#pragma unroll
        for (int k = 0; k < kAttnDh / 16; ++k) {
          umma_bf16_ss(s_tmem, sw128_desc(qa + k * 32, 16, 1024), sw128_desc(k_addr + k * 32, 16, 1024),
                       idesc_qk, k != 0 ? 1u : 0u);
        }
        issued_any = true;
        umma_commit(&s_full_bar[w]);
        const bool last_user = (w == 1) || !(j < n_kv1);
        if (last_user) umma_commit(&k_empty_bar[slot]);
        return true;
      };
      bool ok = mbar_wait(&q_full_bar, 0, kErrAttnMmaWait, &abort_flag);
      if (ok) tc_fence_after();
      if (ok && n_kv0 > 0) ok = issue_qk(0, 0);
      if (ok && n_kv1 > 0) ok = issue_qk(1, 0);
      for (int j = 0; ok && j < n_kv; ++j) {
        const int slot = j % kAttn2Ring;
        bool v_ready = false;
        for (int w = 0; w < 2 && ok; ++w) {
          const int n_kv_this = w == 0 ? n_kv0 : n_kv1;
          if (!(j < n_kv_this)) continue;
          // Softmax of (w, j) done: P_w(j) is in TMEM, O_w rescaled.
          if (!mbar_wait(&p_full_bar[w], j & 1, kErrAttnMmaWait, &abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (!v_ready) {
            if (!mbar_wait(&v_full_bar[slot], (j / kAttn2Ring) & 1, kErrAttnMmaWait, &abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            v_ready = true;
          }
          const uint32_t v_addr = smem_u32(smem_v + slot * kAttnTileBytes);
          const uint32_t p_tmem = tmem_base + w * kAttnBN;
          const uint32_t o_tmem = tmem_base + 2 * kAttnBN + w * kAttnDh;
#pragma unroll
          for (int k = 0; k < kAttnBN / 16; ++k) {
            umma_bf16_ts(o_tmem, p_tmem + k * 8, sw128_desc(v_addr + k * 16 * 128, kAttnTileBytes, 1024),
                         idesc_pv, (j | k) != 0 ? 1u : 0u);
          }
          const bool last_v_user = (w == 1) || !(j < n_kv1);
          if (last_v_user) umma_commit(&v_empty_bar[slot]);
          if (j + 1 < n_kv_this) {
            ok = issue_qk(w, j + 1);
          } else {
            umma_commit(&o_final_bar[w]);
          }
        }
      }
      if (issued_any) {
        umma_commit(&drain_bar);
        volatile int no_abort = 0;
        mbar_wait(&drain_bar, 0, kErrAttnMmaWait, &no_abort);
      }
    }
  } else {
    // Softmax warpgroup w = (warp - 2) / 4 owns query tile q_tile0 + w; warp
    // `warp` reads TMEM lanes 32*(warp%4) .. +31 = its 32 query rows.
    const int w = (warp - 2) >> 2;
    const int n_kv_mine = w == 0 ? n_kv0 : n_kv1;
    const int q_tile = q_tile0 + w;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int q_idx = q_tile * kAttnBM + row;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_tmem = tmem_base + lane_off + w * kAttnBN;
    const uint32_t o_tmem = tmem_base + lane_off + 2 * kAttnBN + w * kAttnDh;
    const float c = args.scale_log2;
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = n_kv_mine > 0;
    for (int j = 0; ok && j < n_kv_mine; ++j) {
      ok = mbar_wait(&s_full_bar[w], j & 1, kErrAttnSoftmaxWait, &abort_flag);
      if (__any_sync(0xffffffffu, !ok)) {
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after();
      uint32_t s[kAttnBN];
      tmem_ld_32cols(s_tmem + 0, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
      tmem_ld_32cols(s_tmem + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
      tmem_ld_32cols(s_tmem + 64, *reinterpret_cast<uint32_t(*)[32]>(&s[64]));
      tmem_ld_32cols(s_tmem + 96, *reinterpret_cast<uint32_t(*)[32]>(&s[96]));
      tmem_wait_ld();
      int limit = kAttnBN;
      if (args.causal) {
        if (j == q_tile) limit = row + 1;
      } else if ((j + 1) * kAttnBN > args.seq) {
        limit = args.seq - j * kAttnBN;
      }
      if (limit < kAttnBN) {
#pragma unroll
        for (int i = 0; i < kAttnBN; ++i)
          if (i >= limit) s[i] = __float_as_uint(-INFINITY);
      }
      // Row maximum: eight independent max3 chains, then a short tree.
      float mp[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mp[k] = __uint_as_float(s[k]);
#pragma unroll
      for (int i = 8; i < kAttnBN; i += 16) {
#pragma unroll
        for (int k = 0; k < 8; ++k) mp[k] = max3(mp[k], __uint_as_float(s[i + k]), __uint_as_float(s[i + 8 + k]));
      }
      const float mx = fmaxf(max3(mp[0], mp[1], mp[2]), max3(max3(mp[3], mp[4], mp[5]), mp[6], mp[7]));
      const float mx_scaled = mx * c;
      const bool need = mx_scaled > m_run + kAttnMaxSlack;
      const float m_new = need ? mx_scaled : m_run;
      const float alpha = need ? fast_exp2(m_run - m_new) : 1.0f;  // 0 on the first tile
      // P = exp2(s * c - m): one f32x2 FMA per pair, one MUFU ex2 per element,
      // packed to bf16 and stored straight back over S; the row sum adds the
      // fp32 probabilities in four independent f32x2 chains.
      const uint64_t c2 = f32x2(c, c);
      const uint64_t neg_m2 = f32x2(-m_new, -m_new);
      uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll
      for (int quarter_row = 0; quarter_row < 4; ++quarter_row) {
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int e = quarter_row * 32 + 2 * i;
          const float2 x = unpack_f32x2(
              fma_f32x2(f32x2(__uint_as_float(s[e]), __uint_as_float(s[e + 1])), c2, neg_m2));
          const float p0 = fast_exp2(x.x);
          const float p1 = fast_exp2(x.y);
          packed[i] = pack_bf16x2(p0, p1);
          acc[i & 3] = add_f32x2(acc[i & 3], f32x2(p0, p1));
        }
        tmem_st_16cols(s_tmem + quarter_row * 16, packed);
      }
      // Rescale O_w now that S is dead (fewer live registers).  O_w is idle here: the commit behind s_full also covers O_w += P_w(j-1) V.
      if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int cc = 0; cc < kAttnDh / 32; ++cc) {
          uint32_t r[32];
          tmem_ld_32cols(o_tmem + cc * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st_32cols(o_tmem + cc * 32, r);
        }
      }
      const float2 a01 = unpack_f32x2(add_f32x2(add_f32x2(acc[0], acc[1]), add_f32x2(acc[2], acc[3])));
      const float row_sum = a01.x + a01.y;
      tmem_wait_st();
      l_run = l_run * alpha + row_sum;
      m_run = m_new;
      tc_fence_before();
      mbar_arrive(&p_full_bar[w]);
    }
    if (ok) {
      ok = mbar_wait(&o_final_bar[w], 0, kErrAttnSoftmaxWait, &abort_flag);
      const bool all_ok = !__any_sync(0xffffffffu, !ok);
      __syncwarp();
      if (all_ok) {
        tc_fence_after();
        const float inv_l = 1.0f / l_run;
        __nv_bfloat16* out_row =
            args.out + (static_cast<int64_t>(batch) * args.seq + q_idx) * d_model + head * kAttnDh;
#pragma unroll 1
        for (int cc = 0; cc < kAttnDh / 32; ++cc) {
          uint32_t r[32];
          tmem_ld_32cols(o_tmem + cc * 32, r);
          tmem_wait_ld();
          if (q_idx < args.seq) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              st_global_v4(out_row + cc * 32 + i,
                           pack_bf16x2(__uint_as_float(r[i]) * inv_l, __uint_as_float(r[i + 1]) * inv_l),
                           pack_bf16x2(__uint_as_float(r[i + 2]) * inv_l, __uint_as_float(r[i + 3]) * inv_l),
                           pack_bf16x2(__uint_as_float(r[i + 4]) * inv_l, __uint_as_float(r[i + 5]) * inv_l),
                           pack_bf16x2(__uint_as_float(r[i + 6]) * inv_l, __uint_as_float(r[i + 7]) * inv_l));
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kAttn2TmemCols);
  }
}

// ---------------------------------------------------------------------------
// Quad-tile variant: one CTA = four consecutive 128-row query tiles of one
// (batch, head) against 64-row KV tiles; one CTA per SM, 576 threads.
//   warp 0       TMA: Q0..Q3 once; K_j, V_j (64 x 64) through a 6-slot ring each
//   warp 1       one thread issues, per query tile w, S_w = Q_w K_j^T
//                (4 x 128x64x16 SS UMMAs) and O_w += P_w V_j (4 x 128x64x16 TS
//                UMMAs, P read from TMEM), cycling over the four tiles
//   warps 2..17  softmax: warps 2+4w .. 5+4w own query tile w, one row per
//                thread, 64 scores per step
// With four tiles in flight, the serial chain of one tile (softmax ->
// P.V and next Q.K^T on the tensor core -> TMEM load) overlaps the exp2 work
// of the other three, so the MUFU pipe, not latency, bounds the kernel.
// TMEM (512 columns): S_w/P_w at 64w .. 64w+63 (P packed into the first 32),
// O_w at 256 + 64w .. +63.
//
// Duo variant: the same kernel with two query tiles per CTA (320 threads,
// 256 TMEM columns, 4-slot KV rings, 97 KB shared memory), so that two CTAs
// share an SM. The four tiles in flight then belong to two independent CTAs:
// one CTA's prologue, epilogue and causal tail (tiles that end before the
// CTA's longest one) overlap the other's main loop, at the cost of loading
// each K/V tile for two query tiles instead of four.
// ---------------------------------------------------------------------------
constexpr int kAttn4BN = 64;
constexpr uint32_t kAttn4KvBytes = kAttn4BN * kAttnDh * 2;  // 8 KB
constexpr float kAttn4MaxSlack = 8.0f;

template <int kTiles>
struct QuadShape {
  static_assert(kTiles == 2 || kTiles == 4, "two or four query tiles per CTA");
  static constexpr int kRing = kTiles == 4 ? 6 : 4;
  static constexpr int kThreads = 64 + kTiles * 128;
  static constexpr int kCtasPerSm = 4 / kTiles;
  static constexpr uint32_t kTmemCols = kTiles * 128;
  static constexpr size_t kSmemBytes =
      1024 + kTiles * kAttnTileBytes + 2 * kRing * kAttn4KvBytes;  // 161 KB / 97 KB
};

// kMasked: the build that reads args.key_valid (padding masks); the unmasked
// build carries none of that code. kTiles: query tiles per CTA (4 = QUAD,
// 2 = DUO).
template <bool kMasked, int kTiles>
__global__ void __launch_bounds__(QuadShape<kTiles>::kThreads, QuadShape<kTiles>::kCtasPerSm)
    attention_fwd_dh64_quad_kernel(const __grid_constant__ CUtensorMap tmap_q,
                                   const __grid_constant__ CUtensorMap tmap_kv,
                                   const __grid_constant__ CUtensorMap tmap_out, AttnArgs args) {
  constexpr int kAttn4Tiles = kTiles;
  constexpr int kAttn4Ring = QuadShape<kTiles>::kRing;
  constexpr uint32_t kAttn4TmemCols = QuadShape<kTiles>::kTmemCols;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t q_full_bar;
  __shared__ uint64_t k_full_bar[kAttn4Ring];
  __shared__ uint64_t k_empty_bar[kAttn4Ring];
  __shared__ uint64_t v_full_bar[kAttn4Ring];
  __shared__ uint64_t v_empty_bar[kAttn4Ring];
  __shared__ uint64_t s_full_bar[kAttn4Tiles];
  __shared__ uint64_t p_full_bar[kAttn4Tiles];
  __shared__ uint64_t o_final_bar[kAttn4Tiles];
  __shared__ uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  uint8_t* smem = align_1024(smem_raw);
  uint8_t* smem_q = smem;
  uint8_t* smem_k = smem + kAttn4Tiles * kAttnTileBytes;
  uint8_t* smem_v = smem_k + kAttn4Ring * kAttn4KvBytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int num_quads = (args.num_q_tiles + kAttn4Tiles - 1) / kAttn4Tiles;
  const int hb_count = args.heads * args.batch;
  const int quad = num_quads - 1 - static_cast<int>(blockIdx.x / hb_count);  // longest first
  const int hb = static_cast<int>(blockIdx.x % hb_count);
  const int head = hb % args.heads;
  const int batch = hb / args.heads;
  const int kv_total = (args.seq + kAttn4BN - 1) / kAttn4BN;
  const int q_tile0 = kAttn4Tiles * quad;
  auto n_kv_of = [&](int w) -> int {
    const int q = q_tile0 + w;
    if (q >= args.num_q_tiles) return 0;
    if (!args.causal) return kv_total;
    const int n = 2 * q + 2;
    return n < kv_total ? n : kv_total;
  };
  int n_kv = 0;
#pragma unroll
  for (int w = 0; w < kAttn4Tiles; ++w) n_kv = n_kv > n_kv_of(w) ? n_kv : n_kv_of(w);
  const int d_model = args.heads * kAttnDh;

  if (threadIdx.x == 0) {
    prefetch_tensor_map(&tmap_q);
    prefetch_tensor_map(&tmap_kv);
    prefetch_tensor_map(&tmap_out);
    mbar_init(&q_full_bar, 1);
    for (int s = 0; s < kAttn4Ring; ++s) {
      mbar_init(&k_full_bar[s], 1);
      mbar_init(&k_empty_bar[s], 1);
      mbar_init(&v_full_bar[s], 1);
      mbar_init(&v_empty_bar[s], 1);
    }
    for (int w = 0; w < kAttn4Tiles; ++w) {
      mbar_init(&s_full_bar[w], 1);
      mbar_init(&p_full_bar[w], 128);
      mbar_init(&o_final_bar[w], 1);
    }
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, kAttn4TmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    if (elect_one()) {
      int active = 0;
      for (int w = 0; w < kAttn4Tiles; ++w) active += n_kv_of(w) > 0 ? 1 : 0;
      mbar_arrive_expect_tx(&q_full_bar, static_cast<uint32_t>(active) * kAttnTileBytes);
      for (int w = 0; w < kAttn4Tiles; ++w) {
        if (n_kv_of(w) > 0)
          tma_load_3d(smem_q + w * kAttnTileBytes, &tmap_q, &q_full_bar, head * kAttnDh,
                      (q_tile0 + w) * kAttnBM, batch);
      }
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int slot = j % kAttn4Ring;
        const uint32_t ph = (j / kAttn4Ring) & 1;
        if (!mbar_wait(&k_empty_bar[slot], ph ^ 1u, kErrAttnProducerWait, &abort_flag)) break;
        mbar_arrive_expect_tx(&k_full_bar[slot], kAttn4KvBytes);
        tma_load_3d(smem_k + slot * kAttn4KvBytes, &tmap_kv, &k_full_bar[slot],
                    d_model + head * kAttnDh, j * kAttn4BN, batch);
        if (!mbar_wait(&v_empty_bar[slot], ph ^ 1u, kErrAttnProducerWait, &abort_flag)) {
          ++issued;
          break;
        }
        mbar_arrive_expect_tx(&v_full_bar[slot], kAttn4KvBytes);
        tma_load_3d(smem_v + slot * kAttn4KvBytes, &tmap_kv, &v_full_bar[slot],
                    2 * d_model + head * kAttnDh, j * kAttn4BN, batch);
        ++issued;
      }
      volatile int no_abort = 0;
      mbar_wait(&q_full_bar, 0, kErrAttnProducerWait, &no_abort);
      const int first = issued > kAttn4Ring ? issued - kAttn4Ring : 0;
      for (int j = first; j < issued; ++j) {
        const uint32_t ph = (j / kAttn4Ring) & 1;
        mbar_wait(&k_full_bar[j % kAttn4Ring], ph, kErrAttnProducerWait, &no_abort);
        mbar_wait(&v_full_bar[j % kAttn4Ring], ph, kErrAttnProducerWait, &no_abort);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_qk = umma_idesc_bf16(kAttnBM, kAttn4BN, false, false);
      constexpr uint32_t idesc_pv = umma_idesc_bf16(kAttnBM, kAttnDh, false, true);
      const uint32_t q_addr = smem_u32(smem_q);
      int nk[kAttn4Tiles];
#pragma unroll
      for (int w = 0; w < kAttn4Tiles; ++w) nk[w] = n_kv_of(w);
      bool issued_any = false;
      // First / last tile (in issue order) that uses KV tile j.
      auto first_user = [&](int j) -> int {
#pragma unroll
        for (int w = 0; w < kAttn4Tiles; ++w)
          if (j < nk[w]) return w;
        return kAttn4Tiles;
      };
      auto last_user = [&](int j) -> int {
        int u = -1;
#pragma unroll
        for (int w = 0; w < kAttn4Tiles; ++w)
          if (j < nk[w]) u = w;
        return u;
      };
      auto issue_qk = [&](int w, int j) -> bool {
        const int slot = j % kAttn4Ring;
        if (w == first_user(j)) {
          if (!mbar_wait(&k_full_bar[slot], (j / kAttn4Ring) & 1, kErrAttnMmaWait, &abort_flag))
            return false;
          tc_fence_after();
        }
        const uint32_t k_addr = smem_u32(smem_k + slot * kAttn4KvBytes);
        const uint32_t qa = q_addr + w * kAttnTileBytes;
        const uint32_t s_tmem = tmem_base + w * kAttn4BN;
#pragma unroll
        for (int k = 0; k < kAttnDh / 16; ++k) {
          umma_bf16_ss(s_tmem, sw128_desc(qa + k * 32, 16, 1024), sw128_desc(k_addr + k * 32, 16, 1024),
                       idesc_qk, k != 0 ? 1u : 0u);
        }
        issued_any = true;
        umma_commit(&s_full_bar[w]);
        if (w == last_user(j)) umma_commit(&k_empty_bar[slot]);
        return true;
      };
      bool ok = mbar_wait(&q_full_bar, 0, kErrAttnMmaWait, &abort_flag);
      if (ok) tc_fence_after();
      for (int w = 0; ok && w < kAttn4Tiles; ++w)
        if (nk[w] > 0) ok = issue_qk(w, 0);
      for (int j = 0; ok && j < n_kv; ++j) {
        const int slot = j % kAttn4Ring;
        const int last = last_user(j);
        bool v_ready = false;
        for (int w = 0; ok && w < kAttn4Tiles; ++w) {
          if (!(j < nk[w])) continue;
          if (!mbar_wait(&p_full_bar[w], j & 1, kErrAttnMmaWait, &abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (!v_ready) {
            if (!mbar_wait(&v_full_bar[slot], (j / kAttn4Ring) & 1, kErrAttnMmaWait, &abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            v_ready = true;
          }
          const uint32_t v_addr = smem_u32(smem_v + slot * kAttn4KvBytes);
          const uint32_t p_tmem = tmem_base + w * kAttn4BN;
          const uint32_t o_tmem = tmem_base + kAttn4Tiles * kAttn4BN + w * kAttnDh;
#pragma unroll
          for (int k = 0; k < kAttn4BN / 16; ++k) {
            umma_bf16_ts(o_tmem, p_tmem + k * 8, sw128_desc(v_addr + k * 16 * 128, kAttn4KvBytes, 1024),
                         idesc_pv, (j | k) != 0 ? 1u : 0u);
          }
          if (w == last) umma_commit(&v_empty_bar[slot]);
          if (j + 1 < nk[w]) {
            ok = issue_qk(w, j + 1);
          } else {
            umma_commit(&o_final_bar[w]);
          }
        }
      }
      if (issued_any) {
        umma_commit(&drain_bar);
        volatile int no_abort = 0;
        mbar_wait(&drain_bar, 0, kErrAttnMmaWait, &no_abort);
      }
    }
  } else {
    const int w = (warp - 2) >> 2;
    const int n_kv_mine = n_kv_of(w);
    const int q_tile = q_tile0 + w;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int q_idx = q_tile * kAttnBM + row;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_tmem = tmem_base + lane_off + w * kAttn4BN;
    const uint32_t o_tmem = tmem_base + lane_off + kAttn4Tiles * kAttn4BN + w * kAttnDh;
    const float c = args.scale_log2;
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = n_kv_mine > 0;
    const uint8_t* key_valid =
        kMasked ? args.key_valid + static_cast<int64_t>(batch) * args.seq : nullptr;
    for (int j = 0; ok && j < n_kv_mine; ++j) {
      // Padding flags of this KV tile's 64 keys (two per lane), loaded before
      // the wait so that their latency overlaps it.
      bool kv0 = true, kv1 = true;
      if (kMasked) {
        const int c0 = j * kAttn4BN + lane;
        kv0 = c0 < args.seq && key_valid[c0] != 0;
        kv1 = c0 + 32 < args.seq && key_valid[c0 + 32] != 0;
      }
      ok = mbar_wait(&s_full_bar[w], j & 1, kErrAttnSoftmaxWait, &abort_flag);
      if (__any_sync(0xffffffffu, !ok)) {
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after();
      uint32_t s[kAttn4BN];
      tmem_ld_32cols(s_tmem + 0, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
      tmem_ld_32cols(s_tmem + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
      tmem_wait_ld();
      // Columns at or beyond `limit` are masked: above the diagonal, or past
      // the sequence on a ragged non-causal tile.
      int limit = kAttn4BN;
      if (args.causal) {
        const int lim = q_idx - j * kAttn4BN + 1;
        limit = lim < kAttn4BN ? lim : kAttn4BN;
      } else if ((j + 1) * kAttn4BN > args.seq) {
        limit = args.seq - j * kAttn4BN;
      }
      if (limit < kAttn4BN) {
#pragma unroll
        for (int i = 0; i < kAttn4BN; ++i)
          if (i >= limit) s[i] = __float_as_uint(-INFINITY);
      }
      if (kMasked) {
        const uint32_t lo = __ballot_sync(0xffffffffu, kv0);
        const uint32_t hi = __ballot_sync(0xffffffffu, kv1);
        if ((lo & hi) != 0xffffffffu) {
#pragma unroll
          for (int i = 0; i < kAttn4BN; ++i)
            if (!(((i < 32 ? lo : hi) >> (i & 31)) & 1u)) s[i] = __float_as_uint(-INFINITY);
        }
      }
      float mp[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) mp[k] = __uint_as_float(s[k]);
#pragma unroll
      for (int i = 4; i < kAttn4BN - 8; i += 8) {
#pragma unroll
        for (int k = 0; k < 4; ++k) mp[k] = max3(mp[k], __uint_as_float(s[i + k]), __uint_as_float(s[i + 4 + k]));
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) mp[k] = fmaxf(mp[k], __uint_as_float(s[kAttn4BN - 4 + k]));
      const float mx = fmaxf(max3(mp[0], mp[1], mp[2]), mp[3]);
      const float mx_scaled = mx * c;
      // A fully masked row (the upper half of a diagonal block) has mx = -inf:
      // it keeps its running max and contributes p = 0.
      const bool need = mx_scaled > m_run + kAttn4MaxSlack;
      const float m_new = need ? mx_scaled : m_run;
      const float alpha = need ? fast_exp2(m_run - m_new) : 1.0f;  // 0 on the first tile
      // A row that has seen no valid key yet (padding) keeps m = -inf; its
      // scores are all -inf, so any finite offset gives p = 0 without NaN.
      const float m_use = (kMasked && m_new == -INFINITY) ? 0.0f : m_new;
      const uint64_t c2 = f32x2(c, c);
      const uint64_t neg_m2 = f32x2(-m_use, -m_use);
      uint64_t acc[2] = {0, 0};
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int e = part * 32 + 2 * i;
          const float2 x = unpack_f32x2(
              fma_f32x2(f32x2(__uint_as_float(s[e]), __uint_as_float(s[e + 1])), c2, neg_m2));
          const float p0 = fast_exp2(x.x);
          const float p1 = fast_exp2(x.y);
          packed[i] = pack_bf16x2(p0, p1);
          acc[i & 1] = add_f32x2(acc[i & 1], f32x2(p0, p1));
        }
        tmem_st_16cols(s_tmem + part * 16, packed);
      }
      // O_w is idle here: the commit behind s_full also covers O_w += P_w(j-1) V.
      if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int cc = 0; cc < kAttnDh / 32; ++cc) {
          uint32_t r[32];
          tmem_ld_32cols(o_tmem + cc * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st_32cols(o_tmem + cc * 32, r);
        }
      }
      const float2 a = unpack_f32x2(add_f32x2(acc[0], acc[1]));
      tmem_wait_st();
      l_run = l_run * alpha + (a.x + a.y);
      m_run = m_new;
      tc_fence_before();
      mbar_arrive(&p_full_bar[w]);
    }
    if (ok) {
      ok = mbar_wait(&o_final_bar[w], 0, kErrAttnSoftmaxWait, &abort_flag);
      const bool all_ok = !__any_sync(0xffffffffu, !ok);
      __syncwarp();
      if (all_ok) {
        tc_fence_after();
        // l = 0 only for a padding query that sees no valid key: zero row.
        const float inv_l = (!kMasked || l_run > 0.0f) ? 1.0f / l_run : 0.0f;
        // The warp's 32 output rows leave through its tile's Q slot, idle once
        // the tile's UMMAs are complete: one 128-byte row per lane in the
        // 128-byte-swizzled layout of a [32 x 64] box (4 KB-aligned, so row i
        // swizzles by i % 8), then one TMA store (rows past the sequence are
        // clipped by the tensor map) instead of 16-byte stores into 32 rows.
        uint8_t* const box = smem_q + w * kAttnTileBytes + quarter * 32 * 128;
        const uint32_t row_addr = smem_u32(box) + static_cast<uint32_t>(lane) * 128u;
        const uint32_t swz = static_cast<uint32_t>(lane) & 7u;
#pragma unroll 1
        for (int cc = 0; cc < kAttnDh / 32; ++cc) {
          uint32_t r[32];
          tmem_ld_32cols(o_tmem + cc * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            const uint32_t chunk = static_cast<uint32_t>(cc * 4 + i / 8);
            st_shared_v4(row_addr + ((chunk ^ swz) << 4),
                         pack_bf16x2(__uint_as_float(r[i]) * inv_l, __uint_as_float(r[i + 1]) * inv_l),
                         pack_bf16x2(__uint_as_float(r[i + 2]) * inv_l, __uint_as_float(r[i + 3]) * inv_l),
                         pack_bf16x2(__uint_as_float(r[i + 4]) * inv_l, __uint_as_float(r[i + 5]) * inv_l),
                         pack_bf16x2(__uint_as_float(r[i + 6]) * inv_l, __uint_as_float(r[i + 7]) * inv_l));
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        const int row0 = q_tile * kAttnBM + quarter * 32;
        if (lane == 0 && row0 < args.seq) {
          tma_store_3d(&tmap_out, box, head * kAttnDh, row0, batch);
          bulk_commit_group();
          // The store has read the box and written its rows before the CTA
          // (and its shared memory) goes away.
          bulk_wait_group_all();
        }
        __syncwarp();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kAttn4TmemCols);
  }
}

}  // namespace b200tx
