// attention_persistent.cuh -- persistent causal flash attention for head_dim 64
// with double-buffered scores, so that the softmax never waits for the
// tensor-core chain of its own query tile.
//
// Same function and semantics as the kernels in attention_kernels.cuh (the
// reference's attention primitives, official/torch_transformer_benchmark.py:
// 95-118: softmax(Q K^T * Dh^-1/2, causal) in fp32, probabilities cast to the
// activation dtype, times V), same packed [B, S, 3*H*64] input and [B, S, H*64]
// output, optional [B, S] key-padding flags.
//
// Work item = two consecutive 128-row query tiles (slots 0 and 1) of one
// (batch, head); items are ordered longest-first and a grid of at most one
// CTA per SM walks them in snake order (CTA c takes items c, 2G-1-c, 2G+c, ...),
// so the causal triangle balances without one launch wave per item.
//   warp 0      TMA: Q of both slots into one of two Q buffers (the next
//               item's Q lands while the current item runs), then the item's
//               64-row K and V tiles through two 8-slot rings
//   warp 1      one thread issues, per slot w and step j,
//               S_w(j) = Q_w K_j^T into S buffer j%2 of the slot and, once the
//               slot's softmax has written P_w(j), O_w += P_w(j) V_j followed
//               at once by S_w(j+2) into the buffer P_w(j) occupied
//   warps 2..9  softmax, warps 2+4w .. 5+4w own slot w, one query row per
//               thread, 64 scores per step; they also normalise and store O
// Because S_w(j+1) is computed while the softmax works on S_w(j), a slot's
// softmax waits on the tensor core only for the first step of an item.
// TMEM (512 columns): S_w buffers at 128w and 128w + 64 (P packed bf16 into
// the first 32 columns of its buffer), O_w at 256 + 64w.
// Barrier phases run on per-slot step counters that continue across items.
#pragma once

#include "attention_kernels.cuh"

namespace b200tx {

constexpr int kAttnPSlots = 2;
constexpr int kAttnPBN = 64;
constexpr int kAttnPRing = 8;
constexpr int kAttnPThreads = 64 + kAttnPSlots * 128;  // 320
constexpr uint32_t kAttnPTmemCols = 512;
constexpr uint32_t kAttnPKvBytes = kAttnPBN * kAttnDh * 2;      // 8 KB
constexpr uint32_t kAttnPQBytes = kAttnPSlots * kAttnTileBytes;  // 32 KB per Q buffer
constexpr size_t kAttnPSmemBytes =
    1024 + 2 * kAttnPQBytes + 2 * kAttnPRing * kAttnPKvBytes;  // 193 KB
constexpr float kAttnPMaxSlack = 8.0f;

struct AttnPItem {
  int batch;
  int head;
  int q_tile0;
  int n0, n1;  // 64-key steps of slots 0 and 1 (0: the slot has no query tile)
  int n_max;
};

__host__ __device__ __forceinline__ int attn_p_num_items(int num_q_tiles, int heads, int batch) {
  return ((num_q_tiles + 1) / 2) * heads * batch;
}

__device__ __forceinline__ int attn_p_steps(const AttnArgs& args, int q) {
  if (q >= args.num_q_tiles) return 0;
  const int kv_total = (args.seq + kAttnPBN - 1) / kAttnPBN;
  if (!args.causal) return kv_total;
  const int diag = 2 * q + 2;  // KV tiles holding keys <= the tile's last row
  return diag < kv_total ? diag : kv_total;
}

__device__ __forceinline__ AttnPItem attn_p_item(const AttnArgs& args, int i) {
  const int hb_count = args.heads * args.batch;
  const int num_pairs = (args.num_q_tiles + 1) >> 1;
  const int rank = i / hb_count;
  const int pair = num_pairs - 1 - rank;  // longest first
  const int hb = i - rank * hb_count;
  AttnPItem item;
  item.head = hb % args.heads;
  item.batch = hb / args.heads;
  item.q_tile0 = 2 * pair;
  item.n0 = attn_p_steps(args, item.q_tile0);
  item.n1 = attn_p_steps(args, item.q_tile0 + 1);
  item.n_max = item.n0 > item.n1 ? item.n0 : item.n1;
  return item;
}

// The k-th item of CTA `cta` in snake order, or -1 past the end.
__device__ __forceinline__ int attn_p_item_index(int k, int cta, int grid, int num_items) {
  const int i = (k & 1) ? k * grid + (grid - 1 - cta) : k * grid + cta;
  return i < num_items ? i : -1;
}

template <bool kMasked>
__global__ void __launch_bounds__(kAttnPThreads, 1)
    attention_fwd_dh64_persistent_kernel(const __grid_constant__ CUtensorMap tmap_q,
                                         const __grid_constant__ CUtensorMap tmap_kv, AttnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t q_full_bar[2];
  __shared__ uint64_t q_empty_bar[2];
  __shared__ uint64_t k_full_bar[kAttnPRing];
  __shared__ uint64_t k_empty_bar[kAttnPRing];
  __shared__ uint64_t v_full_bar[kAttnPRing];
  __shared__ uint64_t v_empty_bar[kAttnPRing];
  __shared__ uint64_t s_full_bar[kAttnPSlots][2];
  __shared__ uint64_t p_full_bar[kAttnPSlots][2];
  __shared__ uint64_t pv_done_bar[kAttnPSlots];
  __shared__ uint64_t o_final_bar[kAttnPSlots];
  __shared__ uint64_t o_free_bar[kAttnPSlots];
  __shared__ uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  uint8_t* smem = align_1024(smem_raw);
  uint8_t* smem_q = smem;                                 // [2 buffers][2 slots] x 16 KB
  uint8_t* smem_k = smem + 2 * kAttnPQBytes;              // ring of 8 KB K tiles
  uint8_t* smem_v = smem_k + kAttnPRing * kAttnPKvBytes;  // ring of 8 KB V tiles

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int grid = static_cast<int>(gridDim.x);
  const int cta = static_cast<int>(blockIdx.x);
  const int num_items = attn_p_num_items(args.num_q_tiles, args.heads, args.batch);
  const int rounds = (num_items + grid - 1) / grid;
  const int d_model = args.heads * kAttnDh;

  if (threadIdx.x == 0) {
    prefetch_tensor_map(&tmap_q);
    prefetch_tensor_map(&tmap_kv);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&q_full_bar[b], 1);
      mbar_init(&q_empty_bar[b], 1);
    }
    for (int s = 0; s < kAttnPRing; ++s) {
      mbar_init(&k_full_bar[s], 1);
      mbar_init(&k_empty_bar[s], 1);
      mbar_init(&v_full_bar[s], 1);
      mbar_init(&v_empty_bar[s], 1);
    }
    for (int w = 0; w < kAttnPSlots; ++w) {
      for (int b = 0; b < 2; ++b) {
        mbar_init(&s_full_bar[w][b], 1);
        mbar_init(&p_full_bar[w][b], 128);
      }
      mbar_init(&pv_done_bar[w], 1);
      mbar_init(&o_final_bar[w], 1);
      mbar_init(&o_free_bar[w], 128);
    }
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, kAttnPTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int kv_seq = 0;    // position in this CTA's stream of K/V tiles
      int v_issued = 0;  // V tiles issued (kv_seq, or one less after an abort)
      int kk = 0;        // items loaded so far
      for (int k = 0; k < rounds && !abort_flag; ++k) {
        const int i = attn_p_item_index(k, cta, grid, num_items);
        if (i < 0) continue;
        const AttnPItem item = attn_p_item(args, i);
        const int qb = kk & 1;
        if (!mbar_wait(&q_empty_bar[qb], ((kk >> 1) & 1) ^ 1u, kErrAttnProducerWait, &abort_flag)) break;
        const int active = (item.n0 > 0 ? 1 : 0) + (item.n1 > 0 ? 1 : 0);
        mbar_arrive_expect_tx(&q_full_bar[qb], static_cast<uint32_t>(active) * kAttnTileBytes);
        if (item.n0 > 0)
          tma_load_3d(smem_q + qb * kAttnPQBytes, &tmap_q, &q_full_bar[qb], item.head * kAttnDh,
                      item.q_tile0 * kAttnBM, item.batch);
        if (item.n1 > 0)
          tma_load_3d(smem_q + qb * kAttnPQBytes + kAttnTileBytes, &tmap_q, &q_full_bar[qb],
                      item.head * kAttnDh, (item.q_tile0 + 1) * kAttnBM, item.batch);
        ++kk;
        bool ok = true;
        for (int j = 0; j < item.n_max; ++j) {
          const int slot = kv_seq % kAttnPRing;
          const uint32_t ph = (kv_seq / kAttnPRing) & 1;
          if (!mbar_wait(&k_empty_bar[slot], ph ^ 1u, kErrAttnProducerWait, &abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full_bar[slot], kAttnPKvBytes);
          tma_load_3d(smem_k + slot * kAttnPKvBytes, &tmap_kv, &k_full_bar[slot],
                      d_model + item.head * kAttnDh, j * kAttnPBN, item.batch);
          ++kv_seq;
          if (!mbar_wait(&v_empty_bar[slot], ph ^ 1u, kErrAttnProducerWait, &abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&v_full_bar[slot], kAttnPKvBytes);
          tma_load_3d(smem_v + slot * kAttnPKvBytes, &tmap_kv, &v_full_bar[slot],
                      2 * d_model + item.head * kAttnDh, j * kAttnPBN, item.batch);
          ++v_issued;
        }
        if (!ok) break;
      }
      // No TMA write may be in flight when the CTA leaves: wait for the last
      // Q buffers and ring slots issued (complete already on the normal path).
      volatile int no_abort = 0;
      for (int b = kk > 2 ? kk - 2 : 0; b < kk; ++b)
        mbar_wait(&q_full_bar[b & 1], (b >> 1) & 1, kErrAttnProducerWait, &no_abort);
      for (int s = kv_seq > kAttnPRing ? kv_seq - kAttnPRing : 0; s < kv_seq; ++s)
        mbar_wait(&k_full_bar[s % kAttnPRing], (s / kAttnPRing) & 1, kErrAttnProducerWait, &no_abort);
      for (int s = v_issued > kAttnPRing ? v_issued - kAttnPRing : 0; s < v_issued; ++s)
        mbar_wait(&v_full_bar[s % kAttnPRing], (s / kAttnPRing) & 1, kErrAttnProducerWait, &no_abort);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc_qk = umma_idesc_bf16(kAttnBM, kAttnPBN, false, false);
      constexpr uint32_t idesc_pv = umma_idesc_bf16(kAttnBM, kAttnDh, false, true);
      // Per slot: steps before this item, and items finished (o_free phases).
      int gs0 = 0, gs1 = 0;
      int done0 = 0, done1 = 0;
      int kv_base = 0;
      int kk = 0;
      bool issued_any = false;
      bool ok = true;
      for (int k = 0; ok && k < rounds; ++k) {
        const int i = attn_p_item_index(k, cta, grid, num_items);
        if (i < 0) continue;
        const AttnPItem item = attn_p_item(args, i);
        const int qb = kk & 1;
        ok = mbar_wait(&q_full_bar[qb], (kk >> 1) & 1, kErrAttnMmaWait, &abort_flag);
        if (!ok) break;
        tc_fence_after();
        // Slot 1 (the later query tile) uses every KV tile slot 0 uses.
        auto steps = [&](int w) -> int { return w == 0 ? item.n0 : item.n1; };
        auto first_user = [&](int j) -> int { return j < item.n0 ? 0 : 1; };
        auto last_user = [&](int j) -> int { return j < item.n1 ? 1 : 0; };
        auto issue_qk = [&](int w, int j) -> bool {
          const int s = kv_base + j;
          const int slot = s % kAttnPRing;
          if (w == first_user(j)) {
            if (!mbar_wait(&k_full_bar[slot], (s / kAttnPRing) & 1, kErrAttnMmaWait, &abort_flag)) return false;
            tc_fence_after();
          }
          const int b = ((w == 0 ? gs0 : gs1) + j) & 1;
          const uint32_t s_tmem = tmem_base + w * 128 + b * kAttnPBN;
          const uint32_t q_addr = smem_u32(smem_q + qb * kAttnPQBytes + w * kAttnTileBytes);
          const uint32_t k_addr = smem_u32(smem_k + slot * kAttnPKvBytes);
#pragma unroll
          for (int kx = 0; kx < kAttnDh / 16; ++kx) {
            umma_bf16_ss(s_tmem, sw128_desc(q_addr + kx * 32, 16, 1024), sw128_desc(k_addr + kx * 32, 16, 1024),
                         idesc_qk, kx != 0 ? 1u : 0u);
          }
          issued_any = true;
          umma_commit(&s_full_bar[w][b]);
          if (w == last_user(j)) umma_commit(&k_empty_bar[slot]);
          return true;
        };
        for (int j = 0; ok && j < 2; ++j)
          for (int w = 0; ok && w < kAttnPSlots; ++w)
            if (j < steps(w)) ok = issue_qk(w, j);
        for (int j = 0; ok && j < item.n_max; ++j) {
          for (int w = 0; ok && w < kAttnPSlots; ++w) {
            if (!(j < steps(w))) continue;
            const int g = (w == 0 ? gs0 : gs1) + j;
            const int b = g & 1;
            const int done = w == 0 ? done0 : done1;
            if (!mbar_wait(&p_full_bar[w][b], (g >> 1) & 1, kErrAttnMmaWait, &abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            if (j == 0 && done > 0) {
              // The slot's previous item has read its O out of TMEM.
              if (!mbar_wait(&o_free_bar[w], (done - 1) & 1, kErrAttnMmaWait, &abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
            }
            const int s = kv_base + j;
            const int slot = s % kAttnPRing;
            if (w == first_user(j)) {
              if (!mbar_wait(&v_full_bar[slot], (s / kAttnPRing) & 1, kErrAttnMmaWait, &abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
            }
            const uint32_t v_addr = smem_u32(smem_v + slot * kAttnPKvBytes);
            const uint32_t p_tmem = tmem_base + w * 128 + b * kAttnPBN;
            const uint32_t o_tmem = tmem_base + 256 + w * kAttnDh;
#pragma unroll
            for (int kx = 0; kx < kAttnPBN / 16; ++kx) {
              umma_bf16_ts(o_tmem, p_tmem + kx * 8, sw128_desc(v_addr + kx * 16 * 128, kAttnPKvBytes, 1024),
                           idesc_pv, (j | kx) != 0 ? 1u : 0u);
            }
            umma_commit(&pv_done_bar[w]);
            // One o_final phase per item: the slot's epilogue waits on it
            // (pv_done may be two phases ahead of any one P.V by then).
            if (j == steps(w) - 1) umma_commit(&o_final_bar[w]);
            if (w == last_user(j)) umma_commit(&v_empty_bar[slot]);
            // S_w(j+2) goes into the buffer P_w(j) occupies: the tensor pipe
            // runs in issue order, so the P.V above has read it first.
            if (j + 2 < steps(w)) ok = issue_qk(w, j + 2);
          }
        }
        if (!ok) break;
        umma_commit(&q_empty_bar[qb]);
        if (item.n0 > 0) {
          gs0 += item.n0;
          ++done0;
        }
        if (item.n1 > 0) {
          gs1 += item.n1;
          ++done1;
        }
        kv_base += item.n_max;
        ++kk;
      }
      if (issued_any) {
        umma_commit(&drain_bar);
        volatile int no_abort = 0;
        mbar_wait(&drain_bar, 0, kErrAttnMmaWait, &no_abort);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int w = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t o_tmem = tmem_base + lane_off + 256 + w * kAttnDh;
    const float c = args.scale_log2;
    int gs = 0;
    int items_done = 0;  // items this slot has finished (o_final phases)
    bool ok = true;
    for (int k = 0; ok && k < rounds; ++k) {
      const int i = attn_p_item_index(k, cta, grid, num_items);
      if (i < 0) continue;
      const AttnPItem item = attn_p_item(args, i);
      const int n = w == 0 ? item.n0 : item.n1;
      if (n == 0) continue;
      const int q_idx = (item.q_tile0 + w) * kAttnBM + row;
      const uint8_t* key_valid =
          kMasked ? args.key_valid + static_cast<int64_t>(item.batch) * args.seq : nullptr;
      float m_run = -INFINITY;
      float l_run = 0.f;
      for (int j = 0; ok && j < n; ++j) {
        const int g = gs + j;
        const int b = g & 1;
        // Padding flags of this step's 64 keys (two per lane), loaded before
        // the wait so that their latency overlaps it.
        bool kv0 = true, kv1 = true;
        if (kMasked) {
          const int c0 = j * kAttnPBN + lane;
          kv0 = c0 < args.seq && key_valid[c0] != 0;
          kv1 = c0 + 32 < args.seq && key_valid[c0 + 32] != 0;
        }
        ok = mbar_wait(&s_full_bar[w][b], (g >> 1) & 1, kErrAttnSoftmaxWait, &abort_flag);
        if (__any_sync(0xffffffffu, !ok)) {
          ok = false;
          break;
        }
        __syncwarp();
        tc_fence_after();
        const uint32_t s_tmem = tmem_base + lane_off + w * 128 + b * kAttnPBN;
        uint32_t s[kAttnPBN];
        tmem_ld_32cols(s_tmem + 0, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
        tmem_ld_32cols(s_tmem + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
        tmem_wait_ld();
        // Columns at or beyond `limit` are masked: above the diagonal, or past
        // the sequence on a ragged non-causal tile.
        int limit = kAttnPBN;
        if (args.causal) {
          const int lim = q_idx - j * kAttnPBN + 1;
          limit = lim < kAttnPBN ? lim : kAttnPBN;
        } else if ((j + 1) * kAttnPBN > args.seq) {
          limit = args.seq - j * kAttnPBN;
        }
        if (limit < kAttnPBN) {
#pragma unroll
          for (int x = 0; x < kAttnPBN; ++x)
            if (x >= limit) s[x] = __float_as_uint(-INFINITY);
        }
        if (kMasked) {
          const uint32_t lo = __ballot_sync(0xffffffffu, kv0);
          const uint32_t hi = __ballot_sync(0xffffffffu, kv1);
          if ((lo & hi) != 0xffffffffu) {
#pragma unroll
            for (int x = 0; x < kAttnPBN; ++x)
              if (!(((x < 32 ? lo : hi) >> (x & 31)) & 1u)) s[x] = __float_as_uint(-INFINITY);
          }
        }
        float mp[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) mp[t] = __uint_as_float(s[t]);
#pragma unroll
        for (int x = 4; x < kAttnPBN - 8; x += 8) {
#pragma unroll
          for (int t = 0; t < 4; ++t) mp[t] = max3(mp[t], __uint_as_float(s[x + t]), __uint_as_float(s[x + 4 + t]));
        }
#pragma unroll
        for (int t = 0; t < 4; ++t) mp[t] = fmaxf(mp[t], __uint_as_float(s[kAttnPBN - 4 + t]));
        const float mx = fmaxf(max3(mp[0], mp[1], mp[2]), mp[3]);
        const float mx_scaled = mx * c;
        // A fully masked row (the upper half of a diagonal tile) has mx = -inf:
        // it keeps its running max and contributes p = 0.
        const bool need = mx_scaled > m_run + kAttnPMaxSlack;
        const float m_new = need ? mx_scaled : m_run;
        const float alpha = need ? fast_exp2(m_run - m_new) : 1.0f;  // 0 on the first step
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
          for (int x = 0; x < 16; ++x) {
            const int e = part * 32 + 2 * x;
            const float2 xv = unpack_f32x2(
                fma_f32x2(f32x2(__uint_as_float(s[e]), __uint_as_float(s[e + 1])), c2, neg_m2));
            const float p0 = fast_exp2(xv.x);
            const float p1 = fast_exp2(xv.y);
            packed[x] = pack_bf16x2(p0, p1);
            acc[x & 1] = add_f32x2(acc[x & 1], f32x2(p0, p1));
          }
          tmem_st_16cols(s_tmem + part * 16, packed);
        }
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          // O_w holds P_w(j-1) V once that P.V has completed; rescale it
          // before P_w(j) V is added.  pv_done completes one phase per P.V of
          // the slot.  S(g) completing implies P.V(g-2) has (S(g) was issued
          // after it), and P.V(g) waits for this step: the barrier is at
          // phase g-1 or g, so the parity wait for g-1 is unambiguous.
          const bool pv_ok = mbar_wait(&pv_done_bar[w], (g - 1) & 1, kErrAttnSoftmaxWait, &abort_flag);
          if (__any_sync(0xffffffffu, !pv_ok)) {
            ok = false;
            break;
          }
          __syncwarp();
          tc_fence_after();
#pragma unroll 1
          for (int cc = 0; cc < kAttnDh / 32; ++cc) {
            uint32_t r[32];
            tmem_ld_32cols(o_tmem + cc * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int x = 0; x < 32; ++x) r[x] = __float_as_uint(__uint_as_float(r[x]) * alpha);
            tmem_st_32cols(o_tmem + cc * 32, r);
          }
        }
        const float2 a = unpack_f32x2(add_f32x2(acc[0], acc[1]));
        tmem_wait_st();
        l_run = l_run * alpha + (a.x + a.y);
        m_run = m_new;
        tc_fence_before();
        mbar_arrive(&p_full_bar[w][b]);
      }
      if (!ok) break;
      // The item's last P.V into O_w: one o_final phase per item (pv_done
      // can be two phases past any given P.V by now, which a parity wait
      // cannot tell apart).
      ok = mbar_wait(&o_final_bar[w], items_done & 1, kErrAttnSoftmaxWait, &abort_flag);
      if (__any_sync(0xffffffffu, !ok)) {
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after();
      // l = 0 only for a padding query that sees no valid key: zero row.
      const float inv_l = (!kMasked || l_run > 0.0f) ? 1.0f / l_run : 0.0f;
      __nv_bfloat16* out_row =
          args.out + (static_cast<int64_t>(item.batch) * args.seq + q_idx) * d_model + item.head * kAttnDh;
#pragma unroll 1
      for (int cc = 0; cc < kAttnDh / 32; ++cc) {
        uint32_t r[32];
        tmem_ld_32cols(o_tmem + cc * 32, r);
        tmem_wait_ld();
        if (q_idx < args.seq) {
#pragma unroll
          for (int x = 0; x < 32; x += 8) {
            st_global_v4(out_row + cc * 32 + x,
                         pack_bf16x2(__uint_as_float(r[x]) * inv_l, __uint_as_float(r[x + 1]) * inv_l),
                         pack_bf16x2(__uint_as_float(r[x + 2]) * inv_l, __uint_as_float(r[x + 3]) * inv_l),
                         pack_bf16x2(__uint_as_float(r[x + 4]) * inv_l, __uint_as_float(r[x + 5]) * inv_l),
                         pack_bf16x2(__uint_as_float(r[x + 6]) * inv_l, __uint_as_float(r[x + 7]) * inv_l));
          }
        }
      }
      // O_w has been read: the slot's next item may overwrite it.
      tc_fence_before();
      mbar_arrive(&o_free_bar[w]);
      gs += n;
      ++items_done;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kAttnPTmemCols);
  }
}

}  // namespace b200tx
