// attention_pingpong.cuh -- persistent causal flash attention for head_dim 64
// whose softmax never waits for the tensor core of its own query tile.
//
// Same function and semantics as the other attention kernels of this library
// (the reference's attention primitives, official/torch_transformer_benchmark.py:
// 95-118: softmax(Q K^T * Dh^-1/2, causal) in fp32, probabilities cast to the
// activation dtype, times V), same packed [B, S, 3*H*64] input, [B, S, H*64]
// output and optional [B, S] key-padding flags.
//
// Work item = two consecutive 128-row query tiles (w = 0, 1) of one
// (batch, head), streamed against 128-key K/V tiles.  Items are ordered
// longest-first and a grid of at most one CTA per SM walks them in snake
// order (CTA c: items c, 2G-1-c, 2G+c, ...).
//   warp 0       TMA: both Q tiles of an item into one of two Q buffers (the
//                next item's Q lands while the current one runs), then the
//                item's K_j and V_j through two 4-slot rings
//   warp 1       one thread issues the UMMAs: S_w(j+1) = Q_w K_{j+1}^T as soon
//                as the softmax of tile w has LOADED S_w(j) (not when it has
//                finished with it), and O_w += P_w(j) V_j once P_w(j) is written
//   warps 2..17  softmax, eight warps per query tile: warp 2 + 8w + 4h + k
//                reads TMEM lane quarter (warp % 4) and score columns
//                [64h, 64h + 64) of those 32 rows, so each query row is split
//                between two warps (halves h = 0, 1); the two halves of a row
//                exchange their partial row maxima through shared memory once
//                per step (an mbarrier per warp pair, waited with the same
//                bound as every other wait) and keep separate partial row
//                sums, exchanged once in the epilogue, where each half
//                normalises and stores 32 of the row's 64 output columns
// TMEM (512 columns), per tile w: S_w at 256w (128 fp32 columns), P_w at
// 256w + 128 (128 bf16 keys packed into 64 columns), O_w at 256w + 192.
// Because P_w(j) and S_w(j+1) occupy different columns, S_w(j+1) is computed
// while the softmax is still turning S_w(j) into P_w(j), and sixteen softmax
// warps (four per SM sub-partition) hide each other's latency.
//
// The exponentials are split between the MUFU (ex2.approx) and the FMA pipe
// (exp2_poly_f32x2, a degree-3 minimax polynomial after Cody-Waite range
// reduction, max relative error 1.0e-4 -- far below the bf16 rounding of P):
// kPolyPairs of every 16 score pairs take the polynomial.
//
// The running max only moves when a row maximum exceeds it by more than 8
// (log2 units); P may then reach 2^8, carried exactly by bf16 P, fp32 O and
// fp32 l.  When it moves, the warps of those rows rescale their columns of
// O_w in TMEM (after the previous P.V finished, before the next is issued).
//
// Barrier phases run on counters that continue across a CTA's items.  Every
// wait is bounded (sm100_common.cuh): a wait that runs out records its code in
// the device error word, every role stops issuing, drains what it has in
// flight and the TMEM is freed before the kernel returns.
#pragma once

#include "attention_kernels.cuh"

namespace b200tx {

constexpr int kPpSoftmaxWarp0 = 2;
constexpr uint32_t kPpTileCols = 256;  // TMEM columns per query tile
constexpr uint32_t kPpColP = 128;      // P_w offset inside the tile's columns
constexpr uint32_t kPpColO = 192;      // O_w offset inside the tile's columns
constexpr float kPpMaxSlack = 8.0f;

// Launch shape of the kernel with kTiles query tiles per CTA: two tiles and
// one CTA per SM (512 TMEM columns), or one tile and two CTAs per SM (256
// each, smaller K/V rings so that two CTAs' shared memory fits).
template <int kTiles>
struct PpShape {
  static_assert(kTiles == 1 || kTiles == 2, "one or two query tiles per CTA");
  static constexpr int kThreads = 64 + 256 * kTiles;
  static constexpr int kCtasPerSm = 2 / kTiles;
  static constexpr int kRing = kTiles == 2 ? 4 : 2;
  static constexpr uint32_t kTmemCols = kPpTileCols * kTiles;
  static constexpr uint32_t kQBufBytes = kTiles * kAttnTileBytes;
  static constexpr size_t kSmemBytes = 1024 + 2 * kQBufBytes + 2 * kRing * kAttnTileBytes;  // 193 / 97 KB
};

struct PpItem {
  int batch;
  int head;
  int q_tile0;
  int n[2];  // 128-key steps of tiles 0 and 1 (0: the item has no tile 1)
  int n_max;
};

// The r-th item (kTiles consecutive query tiles of one batch row and head) of
// this CTA in snake order, or false when it has no more.
template <int kTiles>
__device__ __forceinline__ bool pp_item(const AttnArgs& args, int r, PpItem& it) {
  const int grid = static_cast<int>(gridDim.x);
  const int c = static_cast<int>(blockIdx.x);
  const int64_t t64 = static_cast<int64_t>(r) * grid + ((r & 1) ? (grid - 1 - c) : c);
  const int hb_count = args.heads * args.batch;
  const int num_groups = (args.num_q_tiles + kTiles - 1) / kTiles;
  if (t64 >= static_cast<int64_t>(num_groups) * hb_count) return false;
  const int t = static_cast<int>(t64);
  const int group = num_groups - 1 - t / hb_count;  // longest first
  const int hb = t % hb_count;
  it.head = hb % args.heads;
  it.batch = hb / args.heads;
  it.q_tile0 = kTiles * group;
  const int kv_total = (args.seq + kAttnBN - 1) / kAttnBN;
  const int q1 = it.q_tile0 + 1;
  it.n[0] = args.causal ? (it.q_tile0 + 1 < kv_total ? it.q_tile0 + 1 : kv_total) : kv_total;
  it.n[1] = (kTiles == 1 || q1 >= args.num_q_tiles)
                ? 0
                : (args.causal ? (q1 + 1 < kv_total ? q1 + 1 : kv_total) : kv_total);
  it.n_max = it.n[0] > it.n[1] ? it.n[0] : it.n[1];
  return true;
}

template <bool kMasked, int kPolyPairs, int kTiles>
__global__ void __launch_bounds__(PpShape<kTiles>::kThreads, PpShape<kTiles>::kCtasPerSm)
    attention_fwd_dh64_pingpong_kernel(const __grid_constant__ CUtensorMap tmap_qkv, AttnArgs args) {
  static_assert(kPolyPairs >= 0 && kPolyPairs <= 16, "poly pairs per 16");
  constexpr int kPpRing = PpShape<kTiles>::kRing;
  constexpr uint32_t kPpTmemCols = PpShape<kTiles>::kTmemCols;
  constexpr uint32_t kPpQBufBytes = PpShape<kTiles>::kQBufBytes;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t q_full_bar[2];
  __shared__ uint64_t q_empty_bar[2];
  __shared__ uint64_t k_full_bar[kPpRing];
  __shared__ uint64_t k_empty_bar[kPpRing];
  __shared__ uint64_t v_full_bar[kPpRing];
  __shared__ uint64_t v_empty_bar[kPpRing];
  __shared__ uint64_t s_full_bar[2];   // S_w(j) computed (UMMA commit)
  __shared__ uint64_t s_empty_bar[2];  // S_w(j) loaded by the softmax (8 warp arrivals)
  __shared__ uint64_t p_full_bar[2];   // P_w(j) stored, O_w rescaled (8 warp arrivals)
  __shared__ uint64_t pv_done_bar[2];  // O_w += P_w(j) V_j complete (UMMA commit)
  __shared__ uint64_t o_final_bar[2];  // the item's last P.V of tile w complete
  __shared__ uint64_t o_empty_bar[2];  // O_w read by the epilogue (8 warp arrivals)
  __shared__ uint64_t drain_bar;
  // Exchange between the two warps that share rows: each thread writes its
  // value (a partial row max, or at the end of an item its partial row sum)
  // into slot [exchange parity][tile][half][row]; after __syncwarp one lane
  // per warp arrives on the pair's barrier (2 arrivals), and the partner's
  // value is read after the phase completes.  Two slots suffice: a warp can only write a slot again after
  // the exchange in between, which its partner joins after reading it.
  __shared__ uint64_t pair_bar[2][4];  // [tile][lane quarter]
  __shared__ float xchg[2][2][2][kAttnBM];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  uint8_t* smem = align_1024(smem_raw);
  uint8_t* smem_q = smem;                               // 2 buffers x 2 tiles
  uint8_t* smem_k = smem + 2 * kPpQBufBytes;            // K ring
  uint8_t* smem_v = smem_k + kPpRing * kAttnTileBytes;  // V ring

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int d_model = args.heads * kAttnDh;

  if (threadIdx.x == 0) {
    prefetch_tensor_map(&tmap_qkv);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&q_full_bar[b], 1);
      mbar_init(&q_empty_bar[b], 1);
    }
    for (int s = 0; s < kPpRing; ++s) {
      mbar_init(&k_full_bar[s], 1);
      mbar_init(&k_empty_bar[s], 1);
      mbar_init(&v_full_bar[s], 1);
      mbar_init(&v_empty_bar[s], 1);
    }
    for (int w = 0; w < 2; ++w) {
      mbar_init(&s_full_bar[w], 1);
      mbar_init(&s_empty_bar[w], 8);
      mbar_init(&p_full_bar[w], 8);
      mbar_init(&pv_done_bar[w], 1);
      mbar_init(&o_final_bar[w], 1);
      mbar_init(&o_empty_bar[w], 8);
      for (int k = 0; k < 4; ++k) mbar_init(&pair_bar[w][k], 2);
    }
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, kPpTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      int kv = 0;        // ring positions whose K and V were both issued
      int q_loaded = 0;  // items whose Q load was issued
      bool ok = true;
      PpItem it;
      for (int r = 0; ok && pp_item<kTiles>(args, r, it); ++r) {
        const int buf = r & 1;
        if (r >= 2 && !mbar_wait(&q_empty_bar[buf], ((r >> 1) - 1) & 1, kErrAttnProducerWait, &abort_flag)) {
          ok = false;
          break;
        }
        uint8_t* q_dst = smem_q + buf * kPpQBufBytes;
        mbar_arrive_expect_tx(&q_full_bar[buf], (it.n[1] > 0 ? 2u : 1u) * kAttnTileBytes);
        tma_load_3d(q_dst, &tmap_qkv, &q_full_bar[buf], it.head * kAttnDh, it.q_tile0 * kAttnBM, it.batch);
        if (it.n[1] > 0)
          tma_load_3d(q_dst + kAttnTileBytes, &tmap_qkv, &q_full_bar[buf], it.head * kAttnDh,
                      (it.q_tile0 + 1) * kAttnBM, it.batch);
        ++q_loaded;
        for (int j = 0; j < it.n_max; ++j, ++kv) {
          const int slot = kv % kPpRing;
          const uint32_t ph = (kv / kPpRing) & 1;
          if (!mbar_wait(&k_empty_bar[slot], ph ^ 1u, kErrAttnProducerWait, &abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full_bar[slot], kAttnTileBytes);
          tma_load_3d(smem_k + slot * kAttnTileBytes, &tmap_qkv, &k_full_bar[slot], d_model + it.head * kAttnDh,
                      j * kAttnBN, it.batch);
          if (!mbar_wait(&v_empty_bar[slot], ph ^ 1u, kErrAttnProducerWait, &abort_flag)) {
            ok = false;
            // K of this position is in flight; V is not.
            volatile int no_abort = 0;
            mbar_wait(&k_full_bar[slot], ph, kErrAttnProducerWait, &no_abort);
            break;
          }
          mbar_arrive_expect_tx(&v_full_bar[slot], kAttnTileBytes);
          tma_load_3d(smem_v + slot * kAttnTileBytes, &tmap_qkv, &v_full_bar[slot],
                      2 * d_model + it.head * kAttnDh, j * kAttnBN, it.batch);
        }
      }
      // Drain: wait (bounded) until every load this thread issued has landed
      // (already true on the normal path: the MMA thread consumed them all).
      volatile int no_abort = 0;
      for (int q = q_loaded > 2 ? q_loaded - 2 : 0; q < q_loaded; ++q)
        mbar_wait(&q_full_bar[q & 1], (q >> 1) & 1, kErrAttnProducerWait, &no_abort);
      for (int p = kv > kPpRing ? kv - kPpRing : 0; p < kv; ++p) {
        mbar_wait(&k_full_bar[p % kPpRing], (p / kPpRing) & 1, kErrAttnProducerWait, &no_abort);
        mbar_wait(&v_full_bar[p % kPpRing], (p / kPpRing) & 1, kErrAttnProducerWait, &no_abort);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc_qk = umma_idesc_bf16(kAttnBM, kAttnBN, false, false);
      constexpr uint32_t idesc_pv = umma_idesc_bf16(kAttnBM, kAttnDh, false, true);
      int kv = 0;
      int s_issued0 = 0, s_issued1 = 0;      // S_w UMMAs issued (s_empty phases to wait for)
      int pv_issued0 = 0, pv_issued1 = 0;    // P.V UMMAs issued (p_full phases to wait for)
      int items_done0 = 0, items_done1 = 0;  // items whose O_w went to the epilogue
      bool issued_any = false;
      bool ok = true;
      PpItem it;
      for (int r = 0; ok && pp_item<kTiles>(args, r, it); ++r) {
        const int buf = r & 1;
        if (!mbar_wait(&q_full_bar[buf], (r >> 1) & 1, kErrAttnMmaWait, &abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t q_addr = smem_u32(smem_q + buf * kPpQBufBytes);
        // S_w(j) = Q_w K_j^T once the softmax has loaded S_w(j-1).  The first
        // user of K_j waits for its load; the last one frees its slot.
        auto issue_qk = [&](int w, int j) -> bool {
          int& issued = w == 0 ? s_issued0 : s_issued1;
          if (issued > 0 && !mbar_wait(&s_empty_bar[w], (issued - 1) & 1, kErrAttnMmaWait, &abort_flag))
            return false;
          const int pos = kv + j;
          const int slot = pos % kPpRing;
          if (w == 0 || j >= it.n[0]) {
            if (!mbar_wait(&k_full_bar[slot], (pos / kPpRing) & 1, kErrAttnMmaWait, &abort_flag)) return false;
          }
          tc_fence_after();
          const uint32_t k_addr = smem_u32(smem_k + slot * kAttnTileBytes);
          const uint32_t qa = q_addr + w * kAttnTileBytes;
          const uint32_t s_tmem = tmem_base + w * kPpTileCols;
#pragma unroll
          for (int k = 0; k < kAttnDh / 16; ++k) {
            umma_bf16_ss(s_tmem, sw128_desc(qa + k * 32, 16, 1024), sw128_desc(k_addr + k * 32, 16, 1024), idesc_qk,
                         k != 0 ? 1u : 0u);
          }
          issued_any = true;
          umma_commit(&s_full_bar[w]);
          ++issued;
          if (w == 1 || j >= it.n[1]) umma_commit(&k_empty_bar[slot]);
          return true;
        };
        // O_w += P_w(j) V_j once the softmax has stored P_w(j); the first
        // P.V of an item overwrites O_w, so the previous item's epilogue must
        // have read it.
        auto issue_pv = [&](int w, int j, bool& v_ready) -> bool {
          int& issued = w == 0 ? pv_issued0 : pv_issued1;
          int& done = w == 0 ? items_done0 : items_done1;
          if (!mbar_wait(&p_full_bar[w], issued & 1, kErrAttnMmaWait, &abort_flag)) return false;
          if (j == 0 && done > 0 && !mbar_wait(&o_empty_bar[w], (done - 1) & 1, kErrAttnMmaWait, &abort_flag))
            return false;
          const int pos = kv + j;
          const int slot = pos % kPpRing;
          if (!v_ready) {
            if (!mbar_wait(&v_full_bar[slot], (pos / kPpRing) & 1, kErrAttnMmaWait, &abort_flag)) return false;
            v_ready = true;
          }
          tc_fence_after();
          const uint32_t v_addr = smem_u32(smem_v + slot * kAttnTileBytes);
          const uint32_t p_tmem = tmem_base + w * kPpTileCols + kPpColP;
          const uint32_t o_tmem = tmem_base + w * kPpTileCols + kPpColO;
#pragma unroll
          for (int k = 0; k < kAttnBN / 16; ++k) {
            umma_bf16_ts(o_tmem, p_tmem + k * 8, sw128_desc(v_addr + k * 16 * 128, kAttnTileBytes, 1024), idesc_pv,
                         (j | k) != 0 ? 1u : 0u);
          }
          umma_commit(&pv_done_bar[w]);
          ++issued;
          if (w == 1 || j >= it.n[1]) umma_commit(&v_empty_bar[slot]);
          if (j + 1 == it.n[w]) {
            umma_commit(&o_final_bar[w]);
            ++done;
          }
          return true;
        };
        if (it.n[0] > 0) ok = issue_qk(0, 0);
        if (ok && it.n[1] > 0) ok = issue_qk(1, 0);
        for (int j = 0; ok && j < it.n_max; ++j) {
          if (j + 1 < it.n[0]) ok = issue_qk(0, j + 1);
          if (ok && j + 1 < it.n[1]) ok = issue_qk(1, j + 1);
          bool v_ready = false;
          if (ok && j < it.n[0]) ok = issue_pv(0, j, v_ready);
          if (ok && j < it.n[1]) ok = issue_pv(1, j, v_ready);
        }
        if (!ok) break;
        kv += it.n_max;
        // Every UMMA that reads this Q buffer has been issued.
        umma_commit(&q_empty_bar[buf]);
      }
      if (issued_any) {
        umma_commit(&drain_bar);
        volatile int no_abort = 0;
        mbar_wait(&drain_bar, 0, kErrAttnMmaWait, &no_abort);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int sw = warp - kPpSoftmaxWarp0;
    const int w = sw >> 3;        // query tile
    const int h = (sw >> 2) & 1;  // half of the score row: columns [64h, 64h + 64)
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    uint64_t* const pair = &pair_bar[w][quarter];  // shared with the other half of these rows
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_tmem = tmem_base + lane_off + w * kPpTileCols + 64 * h;
    const uint32_t p_tmem = tmem_base + lane_off + w * kPpTileCols + kPpColP + 32 * h;
    const uint32_t o_tmem = tmem_base + lane_off + w * kPpTileCols + kPpColO + 32 * h;
    const float c = args.scale_log2;
    const uint64_t c2 = f32x2(c, c);
    int s_seen = 0;   // S_w arrivals consumed
    int pv_seen = 0;  // P.V completions accounted for
    int items = 0;    // items of this tile finished
    int exchanges = 0;  // completed phases of this warp pair's barrier
    bool ok = true;
    PpItem it;
    for (int r = 0; ok && pp_item<kTiles>(args, r, it); ++r) {
      const int n = it.n[w];
      if (n == 0) continue;
      const int q_tile = it.q_tile0 + w;
      const int q_idx = q_tile * kAttnBM + row;
      const uint8_t* kv_flags = kMasked ? args.key_valid + static_cast<int64_t>(it.batch) * args.seq : nullptr;
      float m_run = -INFINITY;
      float l_run = 0.f;  // this half's partial row sum
      for (int j = 0; j < n; ++j) {
        const int key0 = j * kAttnBN + 64 * h;  // first key of this half's columns
        // Key flags of this half's 64 keys (masked build): two 32-key ballots.
        uint32_t kbits0 = ~0u, kbits1 = ~0u;
        if constexpr (kMasked) {
          const int ka = key0 + lane, kb = key0 + 32 + lane;
          kbits0 = __ballot_sync(0xffffffffu, ka < args.seq && kv_flags[ka] != 0);
          kbits1 = __ballot_sync(0xffffffffu, kb < args.seq && kv_flags[kb] != 0);
        }
        ok = mbar_wait(&s_full_bar[w], s_seen & 1, kErrAttnSoftmaxWait, &abort_flag);
        if (__any_sync(0xffffffffu, !ok)) {
          ok = false;
          break;
        }
        ++s_seen;
        __syncwarp();
        tc_fence_after();
        uint32_t s[64];
        tmem_ld_32cols(s_tmem + 0, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
        tmem_ld_32cols(s_tmem + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
        tmem_wait_ld();
        // This half of S_w(j) is in registers: once all eight warps have
        // arrived, the tensor core may write S_w(j+1).
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty_bar[w]);
        // Keys at or beyond `limit` (relative to key0) are masked: above the
        // diagonal, or past the sequence on the last tile.
        int limit = 64;
        if (args.causal && j == q_tile) {
          limit = row + 1 - 64 * h;
        } else if (key0 + 64 > args.seq) {
          limit = args.seq - key0;
        }
        if (limit < 64) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (i >= limit) s[i] = __float_as_uint(-INFINITY);
        }
        if constexpr (kMasked) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (!(((i < 32 ? kbits0 : kbits1) >> (i & 31)) & 1u)) s[i] = __float_as_uint(-INFINITY);
        }
        // Partial row maximum (four max3 chains), then the other half's.
        float mp[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) mp[k] = __uint_as_float(s[k]);
#pragma unroll
        for (int i = 4; i < 60; i += 8) {
#pragma unroll
          for (int k = 0; k < 4; ++k) mp[k] = max3(mp[k], __uint_as_float(s[i + k]), __uint_as_float(s[i + 4 + k]));
        }
        const float mine = fmaxf(max3(mp[0], mp[1], mp[2]), max3(mp[3], __uint_as_float(s[60]), __uint_as_float(s[61])));
        const float mine2 = max3(mine, __uint_as_float(s[62]), __uint_as_float(s[63]));
        const int slot = exchanges & 1;
        xchg[slot][w][h][row] = mine2;
        __syncwarp();
        if (lane == 0) mbar_arrive(pair);
        ok = mbar_wait(pair, exchanges & 1, kErrAttnSoftmaxWait, &abort_flag);
        if (__any_sync(0xffffffffu, !ok)) {
          ok = false;
          break;
        }
        ++exchanges;
        const float mx = fmaxf(mine2, xchg[slot][w][h ^ 1][row]);
        const float mx_scaled = mx * c;
        const bool need = mx_scaled > m_run + kPpMaxSlack;
        const float m_new = need ? mx_scaled : m_run;
        const float alpha = need ? fast_exp2(m_run - m_new) : 1.0f;  // 0 on the first step
        // A row that has seen no valid key keeps m = -inf: a finite offset
        // gives p = 0 instead of NaN.
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const uint64_t neg_m2 = f32x2(-m_use, -m_use);
        uint64_t acc[2] = {0, 0};
#pragma unroll
        for (int chunk = 0; chunk < 2; ++chunk) {
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int e = chunk * 32 + 2 * i;
            const uint64_t x = fma_f32x2(f32x2(__uint_as_float(s[e]), __uint_as_float(s[e + 1])), c2, neg_m2);
            float p0, p1;
            if (i < kPolyPairs) {
              exp2_poly_f32x2(x, p0, p1);
            } else {
              const float2 xv = unpack_f32x2(x);
              p0 = fast_exp2(xv.x);
              p1 = fast_exp2(xv.y);
            }
            packed[i] = pack_bf16x2(p0, p1);
            acc[i & 1] = add_f32x2(acc[i & 1], f32x2(p0, p1));
          }
          if (chunk == 0 && j > 0) {
            // P_w(j-1) V_{j-1} must have read P_w before it is overwritten
            // (and have written O_w before a rescale).
            const bool got = mbar_wait(&pv_done_bar[w], pv_seen & 1, kErrAttnSoftmaxWait, &abort_flag);
            if (__any_sync(0xffffffffu, !got)) ok = false;
            ++pv_seen;
            tc_fence_after();
          }
          if (!ok) break;
          tmem_st_16cols(p_tmem + chunk * 16, packed);
        }
        if (!ok) break;
        // Rescale this warp's columns of O_w for its rows whose maximum moved.
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          uint32_t o[32];
          tmem_ld_32cols(o_tmem, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st_32cols(o_tmem, o);
        }
        const float2 a01 = unpack_f32x2(add_f32x2(acc[0], acc[1]));
        l_run = l_run * alpha + (a01.x + a01.y);
        m_run = m_new;
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full_bar[w]);
      }
      if (!ok) break;
      // Epilogue: this half's 32 output columns, O_w / l in bf16.
      ok = mbar_wait(&o_final_bar[w], items & 1, kErrAttnSoftmaxWait, &abort_flag);
      if (__any_sync(0xffffffffu, !ok)) {
        ok = false;
        break;
      }
      ++pv_seen;  // the item's last P.V, complete before o_final
      __syncwarp();
      tc_fence_after();
      uint32_t o[32];
      tmem_ld_32cols(o_tmem, o);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty_bar[w]);
      ++items;
      const int slot = exchanges & 1;
      xchg[slot][w][h][row] = l_run;
      __syncwarp();
      if (lane == 0) mbar_arrive(pair);
      ok = mbar_wait(pair, exchanges & 1, kErrAttnSoftmaxWait, &abort_flag);
      if (__any_sync(0xffffffffu, !ok)) {
        ok = false;
        break;
      }
      ++exchanges;
      const float l_row = l_run + xchg[slot][w][h ^ 1][row];
      const float inv_l = l_row > 0.f ? 1.0f / l_row : 0.f;
      if (q_idx < args.seq) {
        __nv_bfloat16* out_row = args.out + (static_cast<int64_t>(it.batch) * args.seq + q_idx) * d_model +
                                 it.head * kAttnDh + 32 * h;
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          st_global_v4(out_row + i, pack_bf16x2(__uint_as_float(o[i]) * inv_l, __uint_as_float(o[i + 1]) * inv_l),
                       pack_bf16x2(__uint_as_float(o[i + 2]) * inv_l, __uint_as_float(o[i + 3]) * inv_l),
                       pack_bf16x2(__uint_as_float(o[i + 4]) * inv_l, __uint_as_float(o[i + 5]) * inv_l),
                       pack_bf16x2(__uint_as_float(o[i + 6]) * inv_l, __uint_as_float(o[i + 7]) * inv_l));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kPpTmemCols);
  }
}

}  // namespace b200tx
