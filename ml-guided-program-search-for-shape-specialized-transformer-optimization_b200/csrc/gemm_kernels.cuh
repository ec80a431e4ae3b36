// gemm_kernels.cuh -- C[M,N] = A[M,K] . W[N,K]^T + bias[N] (optional exact GELU)
// on the sm_100 tensor cores (tcgen05.mma kind::f16, bf16 in, fp32 accumulate).
//
// Replaces the reference's projection kernels and the cuBLAS linears they sit
// beside:
//   packed QKV projection   solution/kernels/projection/triton_qkv_layout.py:59-113
//   attention out-proj      solution/kernels/projection/triton_attention_output.py:69-147
//   FFN in + exact GELU     solution/kernels/ffn/triton_linear_exact_gelu.py:68-132
//   fp16 shadow F.linear    solution/transformer.py:333-353
// Both operands are K-major (nn.Linear weight layout), so one kernel covers
// every projection of the block.
//
// Structure: persistent CTAs (one per SM), 320 threads.
//   warp 0      TMA producer: A tile 128x64 and W tile 256x64 per stage, 4-stage ring
//   warp 1      one elected thread issues 4 UMMAs (128x256x16) per stage
//   warps 2..9  epilogue: two warps per TMEM lane quarter, each owning 128 of the
//               256 accumulator columns: TMEM -> registers (tcgen05.ld 32x32b,
//               double-buffered), + bias (staged once per tile in shared memory),
//               optional GELU, cast, 16-byte global stores
// The fp32 accumulator for a 128x256 tile uses 256 TMEM columns; two of them
// (all 512 columns) let the epilogue of tile t overlap the MMAs of tile t+1.
// Tiles are walked N-fastest so all CTAs stream the same row block of A while
// the weight matrix (<= 32 MB for every BASELINE shape) stays in L2.
#pragma once

#include "sm100_common.cuh"

namespace b200tx {

constexpr int kGemmBM = 128;
constexpr int kGemmBN = 256;
constexpr int kGemmBK = 64;  // 64 bf16 = one 128-byte swizzle row
constexpr int kGemmStages = 4;
constexpr int kGemmThreads = 320;
constexpr int kGemmEpilogueThreads = 256;
constexpr uint32_t kGemmTmemCols = 512;
constexpr uint32_t kGemmTileABytes = kGemmBM * kGemmBK * 2;  // 16 KB
constexpr uint32_t kGemmTileBBytes = kGemmBN * kGemmBK * 2;  // 32 KB
constexpr uint32_t kGemmStageBytes = kGemmTileABytes + kGemmTileBBytes;
constexpr size_t kGemmSmemBytes = 1024 + kGemmStages * kGemmStageBytes;

enum GemmEpilogue : int { kEpiBias = 0, kEpiBiasGelu = 1 };

struct GemmArgs {
  const float* bias;  // [N] fp32 or null
  void* out;          // [M, N] row-major, bf16 or fp32
  int M, N, K;
  int num_m_tiles, num_n_tiles;
  // Pair kernel only: work units are the first `full_units` tiles, then the
  // remaining tiles each split into two 128-column halves (num_units in all).
  int full_units, num_units;
  int bias_vec4;  // bias is 16-byte aligned: whole 32-column chunks read it as float4
};

// Exact-erf GELU, 0.5 x (1 + erf(x / sqrt 2)), with erf from Abramowitz &
// Stegun, Handbook of Mathematical Functions, formula 7.1.26:
//   erf(z) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-z^2),
//   t = 1 / (1 + p z), z >= 0, |error| <= 1.5e-7.
// With h = 0.5 |x| poly(t) exp(-z^2):  GELU(x) = x - h for x >= 0, and -h for
// x < 0 (odd symmetry of erf: 1 + erf(-z) = poly(t) exp(-z^2)).  One reciprocal and one exp2 on MUFU, the rest on FMA;
// the approximation error is ~70x below one bf16 rounding of the output.
__device__ __forceinline__ float gelu_erf(float x) {
  constexpr float kP = 0.3275911f;
  constexpr float kA1 = 0.254829592f;
  constexpr float kA2 = -0.284496736f;
  constexpr float kA3 = 1.421413741f;
  constexpr float kA4 = -1.453152027f;
  constexpr float kA5 = 1.061405429f;
  constexpr float kInvSqrt2 = 0.70710678118654752f;
  constexpr float kLog2e = 1.4426950408889634f;
  const float z = fabsf(x) * kInvSqrt2;
  float t;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(fmaf(kP, z, 1.0f)));
  const float poly = t * fmaf(fmaf(fmaf(fmaf(kA5, t, kA4), t, kA3), t, kA2), t, kA1);
  const float e = fast_exp2(-(z * z) * kLog2e);
  const float h = 0.5f * fabsf(x) * poly * e;
  return x >= 0.0f ? x - h : -h;
}

// gelu_erf on two values with the packed f32x2 FMA/MUL pipes: the same
// operations in the same order (each lane of a packed op is one IEEE fp32
// operation), so the results equal gelu_erf bit for bit, with about a third
// fewer issued instructions.  The reciprocal and exp2 stay per value on MUFU.
__device__ __forceinline__ void gelu_erf_x2(float& x0, float& x1) {
  constexpr float kP = 0.3275911f;
  constexpr float kA1 = 0.254829592f;
  constexpr float kA2 = -0.284496736f;
  constexpr float kA3 = 1.421413741f;
  constexpr float kA4 = -1.453152027f;
  constexpr float kA5 = 1.061405429f;
  constexpr float kInvSqrt2 = 0.70710678118654752f;
  constexpr float kLog2e = 1.4426950408889634f;
  const uint64_t ax = f32x2(fabsf(x0), fabsf(x1));
  const uint64_t z = mul_f32x2(ax, f32x2(kInvSqrt2, kInvSqrt2));
  const float2 d = unpack_f32x2(fma_f32x2(f32x2(kP, kP), z, f32x2(1.0f, 1.0f)));
  float t0, t1;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t0) : "f"(d.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t1) : "f"(d.y));
  const uint64_t t = f32x2(t0, t1);
  uint64_t q = fma_f32x2(f32x2(kA5, kA5), t, f32x2(kA4, kA4));
  q = fma_f32x2(q, t, f32x2(kA3, kA3));
  q = fma_f32x2(q, t, f32x2(kA2, kA2));
  q = fma_f32x2(q, t, f32x2(kA1, kA1));
  const uint64_t poly = mul_f32x2(t, q);
  const uint64_t zz = mul_f32x2(z, z);
  const float2 arg = unpack_f32x2(mul_f32x2(f32x2(-unpack_f32x2(zz).x, -unpack_f32x2(zz).y), f32x2(kLog2e, kLog2e)));
  const uint64_t e = f32x2(fast_exp2(arg.x), fast_exp2(arg.y));
  const uint64_t half_ax = mul_f32x2(f32x2(0.5f, 0.5f), ax);
  const float2 h = unpack_f32x2(mul_f32x2(mul_f32x2(half_ax, poly), e));
  x0 = x0 >= 0.0f ? x0 - h.x : -h.x;
  x1 = x1 >= 0.0f ? x1 - h.y : -h.y;
}

template <int EPI, typename OutT>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap tmap_a,
                        const __grid_constant__ CUtensorMap tmap_w, GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full_bar[kGemmStages];
  __shared__ uint64_t empty_bar[kGemmStages];
  __shared__ uint64_t acc_full_bar[2];
  __shared__ uint64_t acc_empty_bar[2];
  __shared__ uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  __shared__ float bias_tile[8][kGemmBN / 2];  // one 128-column slice per epilogue warp

  uint8_t* smem = align_1024(smem_raw);
  uint8_t* smem_a = smem;
  uint8_t* smem_w = smem + kGemmStages * kGemmTileABytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = args.num_m_tiles * args.num_n_tiles;
  const int num_kb = (args.K + kGemmBK - 1) / kGemmBK;

  if (threadIdx.x == 0) {
    prefetch_tensor_map(&tmap_a);
    prefetch_tensor_map(&tmap_w);
    for (int s = 0; s < kGemmStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full_bar[a], 1);
      mbar_init(&acc_empty_bar[a], kGemmEpilogueThreads);
    }
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, kGemmTmemCols);
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
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !abort_flag; tile += gridDim.x) {
        const int m_tile = tile / args.num_n_tiles;
        const int n_tile = tile - m_tile * args.num_n_tiles;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, kErrGemmProducerWait, &abort_flag)) break;
          mbar_arrive_expect_tx(&full_bar[stage], kGemmStageBytes);
          tma_load_2d(smem_a + stage * kGemmTileABytes, &tmap_a, &full_bar[stage], kb * kGemmBK,
                      m_tile * kGemmBM);
          tma_load_2d(smem_w + stage * kGemmTileBBytes, &tmap_w, &full_bar[stage], kb * kGemmBK,
                      n_tile * kGemmBN);
          ++issued;
          if (++stage == kGemmStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Never leave a TMA write in flight into shared memory this CTA is
      // about to release: wait for the last loads issued (already complete on
      // the normal path, so these waits return at once).
      const int outstanding = issued < kGemmStages ? issued : kGemmStages;
      for (int i = 0; i < outstanding; ++i) {
        if (--stage < 0) {
          stage = kGemmStages - 1;
          phase ^= 1u;
        }
        volatile int no_abort = 0;
        mbar_wait(&full_bar[stage], phase, kErrGemmProducerWait, &no_abort);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16(kGemmBM, kGemmBN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int t = 0;
      bool issued_any = false;
      for (int tile = blockIdx.x; tile < num_tiles && !abort_flag; tile += gridDim.x, ++t) {
        const int acc = t & 1;
        const uint32_t acc_phase = (t >> 1) & 1;
        if (!mbar_wait(&acc_empty_bar[acc], acc_phase ^ 1u, kErrGemmMmaWait, &abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kGemmBN;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, kErrGemmMmaWait, &abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem_a + stage * kGemmTileABytes);
          const uint32_t w_addr = smem_u32(smem_w + stage * kGemmTileBBytes);
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k) {
            const uint64_t a_desc = sw128_desc(a_addr + k * 32, 16, 1024);
            const uint64_t w_desc = sw128_desc(w_addr + k * 32, 16, 1024);
            umma_bf16_ss(d_tmem, a_desc, w_desc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          issued_any = true;
          umma_commit(&empty_bar[stage]);
          if (++stage == kGemmStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&acc_full_bar[acc]);
      }
      if (issued_any) {
        // All MMAs of this thread retire before TMEM is released.
        umma_commit(&drain_bar);
        volatile int no_abort = 0;
        mbar_wait(&drain_bar, 0, kErrGemmMmaWait, &no_abort);
      }
    }
  } else {
    // Epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 (its lane quarter) and
    // the column half (w-2)/4 of the 256-column accumulator.
    const int quarter = warp & 3;
    const int col_half = (warp - 2) >> 2;
    const int row_in_tile = quarter * 32 + lane;
    int t = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++t) {
      const int acc = t & 1;
      const uint32_t acc_phase = (t >> 1) & 1;
      const int m_tile = tile / args.num_n_tiles;
      const int n_tile = tile - m_tile * args.num_n_tiles;
      // Stage this warp's 128 bias values for the tile before waiting for the
      // accumulator.  Each warp owns its slice, so only warp-level
      // synchronisation is needed (no CTA barrier that an aborting warp could
      // leave the others stuck on).
      float* warp_bias = bias_tile[warp - 2];
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int col = n_tile * kGemmBN + col_half * (kGemmBN / 2) + i * 32 + lane;
        warp_bias[i * 32 + lane] = (args.bias != nullptr && col < args.N) ? __ldg(args.bias + col) : 0.f;
      }
      __syncwarp();
      bool ok = mbar_wait(&acc_full_bar[acc], acc_phase, kErrGemmEpilogueWait, &abort_flag);
      if (__any_sync(0xffffffffu, !ok)) break;
      __syncwarp();
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(m_tile) * kGemmBM + row_in_tile;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             acc * kGemmBN + col_half * (kGemmBN / 2);
      constexpr int kChunks = kGemmBN / 2 / 32;  // 4 chunks of 32 columns
      uint32_t buf[2][32];
      tmem_ld_32cols(taddr, buf[0]);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        if (c + 1 < kChunks) tmem_ld_32cols(taddr + (c + 1) * 32, buf[(c + 1) & 1]);
        const uint32_t (&r)[32] = buf[c & 1];
        const int col_in_tile = col_half * (kGemmBN / 2) + c * 32;
        const int col0 = n_tile * kGemmBN + col_in_tile;
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) + warp_bias[c * 32 + i];
        if constexpr (EPI == kEpiBiasGelu) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) gelu_erf_x2(v[i], v[i + 1]);
        }
        if (row < args.M) {
          // N % 8 == 0 (checked on the host): each group of eight columns is
          // either entirely inside the matrix or entirely past its edge.
          OutT* out_row = static_cast<OutT*>(args.out) + row * args.N + col0;
          if constexpr (std::is_same<OutT, __nv_bfloat16>::value) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              if (col0 + i < args.N)
                st_global_v4(out_row + i, pack_bf16x2(v[i], v[i + 1]), pack_bf16x2(v[i + 2], v[i + 3]),
                             pack_bf16x2(v[i + 4], v[i + 5]), pack_bf16x2(v[i + 6], v[i + 7]));
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              if (col0 + i < args.N)
                st_global_v4(out_row + i, __float_as_uint(v[i]), __float_as_uint(v[i + 1]),
                             __float_as_uint(v[i + 2]), __float_as_uint(v[i + 3]));
            }
          }
        }
        if (c + 1 < kChunks) tmem_wait_ld();
      }
      // Every column of this thread's lane has been read: release the buffer.
      tc_fence_before();
      mbar_arrive(&acc_empty_bar[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kGemmTmemCols);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant: clusters of two CTAs (one per SM) share 256x256 output
// tiles through the tcgen05 .cta_group::2 MMA.  CTA r of the pair loads rows
// 128r..128r+127 of the tile's A block and rows 128r..128r+127 of its 256-row
// W block, 32 KB per stage, so a 6-stage ring fits where the single-CTA kernel
// holds 4 stages of 48 KB, and every SM streams a third less operand data per
// FLOP out of L2.  The leader (rank 0) issues 256x256x16 UMMAs that read both
// CTAs' shared memory and write both CTAs' TMEM (each CTA keeps its 128 rows
// x 256 fp32 columns, double-buffered in its 512 columns).
//   warp 0      TMA producer in each CTA; all loads of a stage complete on
//               the leader's full barrier: the leader arms it with the bytes
//               of both CTAs (its one arrival) and loads with a plain TMA,
//               the peer's .cta_group::2 TMA loads report their bytes to it
//               (no remote arrival, which would serialise the peer's loop)
//   warp 1      leader only: one elected thread issues the UMMAs; commits are
//               multicast to both CTAs (stage free, accumulator ready)
//   warps 2..9  epilogue in each CTA as in the single-CTA kernel; each warp
//               releases an accumulator on the leader's barrier (16 arrivals)
// Both CTAs walk the same pair-tile sequence.  A cluster barrier orders the
// barrier initialisation before any remote use and keeps both CTAs (their
// shared memory and TMEM) alive until the pair has finished.
// ---------------------------------------------------------------------------
constexpr int kGemm2BM = 256;  // rows per pair tile (128 per CTA)
constexpr int kGemm2BN = 256;  // columns per pair tile (W rows: 128 per CTA)
constexpr int kGemm2Stages = 6;
constexpr uint32_t kGemm2TileABytes = 128 * kGemmBK * 2;  // 16 KB
constexpr uint32_t kGemm2TileBBytes = 128 * kGemmBK * 2;  // 16 KB
constexpr uint32_t kGemm2StageBytes = kGemm2TileABytes + kGemm2TileBBytes;
// Epilogue staging for the TMA stores of bf16 outputs: per epilogue warp two
// 2 KB buffers of 32 rows x 32 columns (64-byte rows, 64-byte swizzle).
constexpr uint32_t kGemm2StoreBoxBytes = 32 * 32 * 2;
constexpr uint32_t kGemm2StoreBytes = 8 * 2 * kGemm2StoreBoxBytes;  // 32 KB
constexpr size_t kGemm2SmemBytes =
    1024 + kGemm2Stages * kGemm2StageBytes + kGemm2StoreBytes;  // 225 KB

// Work unit u of the pair kernel: a whole 256 x 256 tile, or (in the last,
// partial wave) one 256 x 128 half of a tile.  Halving the tail tiles lets a
// wave of R < pairs/2 leftover tiles occupy 2R pairs for half as long.
struct PairUnit {
  int m_tile;
  int col_base;  // first output column
  int width;     // 256 or 128 columns
};

__device__ __forceinline__ PairUnit pair_unit(const GemmArgs& args, int u) {
  int tile = u;
  int half = -1;
  if (u >= args.full_units) {
    const int h = u - args.full_units;
    tile = args.full_units + (h >> 1);
    half = h & 1;
  }
  const int m_tile = tile / args.num_n_tiles;
  const int n_tile = tile - m_tile * args.num_n_tiles;
  PairUnit unit;
  unit.m_tile = m_tile;
  unit.col_base = n_tile * kGemm2BN + (half > 0 ? kGemm2BN / 2 : 0);
  unit.width = half >= 0 ? kGemm2BN / 2 : kGemm2BN;
  return unit;
}

template <int EPI, typename OutT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_tn_pair_kernel(const __grid_constant__ CUtensorMap tmap_a,
                             const __grid_constant__ CUtensorMap tmap_w,
                             const __grid_constant__ CUtensorMap tmap_out, GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full_bar[kGemm2Stages];
  __shared__ uint64_t empty_bar[kGemm2Stages];
  __shared__ uint64_t acc_full_bar[2];
  __shared__ uint64_t acc_empty_bar[2];
  __shared__ uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  uint8_t* smem = align_1024(smem_raw);
  uint8_t* smem_a = smem;
  uint8_t* smem_w = smem + kGemm2Stages * kGemm2TileABytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int num_pairs = static_cast<int>(gridDim.x >> 1);
  const int num_units = args.num_units;  // pair tiles (256 x 256) and tail halves (256 x 128)
  const int num_kb = (args.K + kGemmBK - 1) / kGemmBK;

  if (threadIdx.x == 0) {
    prefetch_tensor_map(&tmap_a);
    prefetch_tensor_map(&tmap_w);
    if constexpr (std::is_same<OutT, __nv_bfloat16>::value) prefetch_tensor_map(&tmap_out);
    for (int s = 0; s < kGemm2Stages; ++s) {
      mbar_init(&full_bar[s], 1);  // the leader's arrive.expect_tx
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full_bar[a], 1);
      mbar_init(&acc_empty_bar[a], 16);  // 8 epilogue warps in each CTA
    }
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&tmem_slot, kGemmTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      const uint32_t full_leader_base = peer_smem_addr(&full_bar[0], 0);
      for (int u = pair; u < num_units && !abort_flag; u += num_pairs) {
        const PairUnit unit = pair_unit(args, u);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, kErrGemmProducerWait, &abort_flag)) break;
          const int a_row = unit.m_tile * kGemm2BM + static_cast<int>(rank) * 128;
          // A half-width unit uses the first 64 of the 128 W rows loaded.
          const int w_row = unit.col_base + static_cast<int>(rank) * (unit.width / 2);
          if (leader) {
            mbar_arrive_expect_tx(&full_bar[stage], 2 * kGemm2StageBytes);
            tma_load_2d(smem_a + stage * kGemm2TileABytes, &tmap_a, &full_bar[stage], kb * kGemmBK, a_row);
            tma_load_2d(smem_w + stage * kGemm2TileBBytes, &tmap_w, &full_bar[stage], kb * kGemmBK, w_row);
          } else {
            const uint32_t full_leader = full_leader_base + stage * static_cast<uint32_t>(sizeof(uint64_t));
            tma_load_2d_pair(smem_a + stage * kGemm2TileABytes, &tmap_a, full_leader, kb * kGemmBK, a_row);
            tma_load_2d_pair(smem_w + stage * kGemm2TileBBytes, &tmap_w, full_leader, kb * kGemmBK, w_row);
          }
          ++issued;
          if (++stage == kGemm2Stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // The leader waits for the pair's last loads (complete already on the
      // normal path) so that no TMA write is in flight when the pair leaves.
      if (leader) {
        const int outstanding = issued < kGemm2Stages ? issued : kGemm2Stages;
        for (int i = 0; i < outstanding; ++i) {
          if (--stage < 0) {
            stage = kGemm2Stages - 1;
            phase ^= 1u;
          }
          volatile int no_abort = 0;
          mbar_wait(&full_bar[stage], phase, kErrGemmProducerWait, &no_abort);
        }
      }
    }
  } else if (warp == 1) {
    if (leader && elect_one()) {
      constexpr uint32_t idesc_full = umma_idesc_bf16(kGemm2BM, kGemm2BN, false, false);
      constexpr uint32_t idesc_half = umma_idesc_bf16(kGemm2BM, kGemm2BN / 2, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int t = 0;
      bool issued_any = false;
      for (int u = pair; u < num_units && !abort_flag; u += num_pairs, ++t) {
        const uint32_t idesc = u < args.full_units ? idesc_full : idesc_half;
        const int acc = t & 1;
        const uint32_t acc_phase = (t >> 1) & 1;
        if (!mbar_wait(&acc_empty_bar[acc], acc_phase ^ 1u, kErrGemmMmaWait, &abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kGemm2BN;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, kErrGemmMmaWait, &abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem_a + stage * kGemm2TileABytes);
          const uint32_t w_addr = smem_u32(smem_w + stage * kGemm2TileBBytes);
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k) {
            umma_bf16_ss_pair(d_tmem, sw128_desc(a_addr + k * 32, 16, 1024),
                              sw128_desc(w_addr + k * 32, 16, 1024), idesc, (kb | k) != 0 ? 1u : 0u);
          }
          issued_any = true;
          umma_commit_pair(&empty_bar[stage], 0x3);
          if (++stage == kGemm2Stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(&acc_full_bar[acc], 0x3);
      }
      if (issued_any) {
        umma_commit_pair(&drain_bar, 0x1);
        volatile int no_abort = 0;
        mbar_wait(&drain_bar, 0, kErrGemmMmaWait, &no_abort);
      }
    }
  } else {
    const int quarter = warp & 3;
    const int col_half = (warp - 2) >> 2;
    const int row_in_tile = static_cast<int>(rank) * 128 + quarter * 32 + lane;
    const uint32_t acc_empty_leader0 = peer_smem_addr(&acc_empty_bar[0], 0);
    const uint32_t acc_empty_leader1 = peer_smem_addr(&acc_empty_bar[1], 0);
    // bf16 outputs leave through shared memory and TMA stores: this warp's two
    // staging boxes alternate, one store group per 32 x 32 chunk.
    uint8_t* const stage_out = smem + kGemm2Stages * kGemm2StageBytes + (warp - 2) * 2 * kGemm2StoreBoxBytes;
    uint32_t store_seq = 0;
    int t = 0;
    for (int u = pair; u < num_units; u += num_pairs, ++t) {
      const int acc = t & 1;
      const uint32_t acc_phase = (t >> 1) & 1;
      const PairUnit unit = pair_unit(args, u);
      const int m_tile = unit.m_tile;
      bool ok = mbar_wait(&acc_full_bar[acc], acc_phase, kErrGemmEpilogueWait, &abort_flag);
      if (__any_sync(0xffffffffu, !ok)) break;
      __syncwarp();
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(m_tile) * kGemm2BM + row_in_tile;
      const int row_base = m_tile * kGemm2BM + static_cast<int>(rank) * 128 + quarter * 32;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             acc * kGemm2BN + col_half * (unit.width / 2);
      constexpr int kMaxChunks = kGemm2BN / 2 / 32;
      const int chunks = unit.width / 2 / 32;
      uint32_t buf[2][32];
      tmem_ld_32cols(taddr, buf[0]);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < kMaxChunks; ++c) {
        if (c >= chunks) break;
        if (c + 1 < chunks) tmem_ld_32cols(taddr + (c + 1) * 32, buf[(c + 1) & 1]);
        const uint32_t (&r)[32] = buf[c & 1];
        const int col0 = unit.col_base + col_half * (unit.width / 2) + c * 32;
        // N % 8 == 0 (checked on the host): each group of eight columns is
        // either entirely inside the matrix or entirely past its edge.
        float v[32];
        if (args.bias_vec4 && col0 + 32 <= args.N) {
          // Eight broadcast 16-byte loads (every lane reads the same columns).
          const float4* b4 = reinterpret_cast<const float4*>(args.bias + col0);
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4) {
            const float4 bb = __ldg(b4 + q4);
            v[4 * q4 + 0] = __uint_as_float(r[4 * q4 + 0]) + bb.x;
            v[4 * q4 + 1] = __uint_as_float(r[4 * q4 + 1]) + bb.y;
            v[4 * q4 + 2] = __uint_as_float(r[4 * q4 + 2]) + bb.z;
            v[4 * q4 + 3] = __uint_as_float(r[4 * q4 + 3]) + bb.w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float b = (args.bias != nullptr && col0 + (i & ~7) < args.N) ? __ldg(args.bias + col0 + i) : 0.f;
            v[i] = __uint_as_float(r[i]) + b;
          }
        }
        if constexpr (EPI == kEpiBiasGelu) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) gelu_erf_x2(v[i], v[i + 1]);
        }
        if constexpr (std::is_same<OutT, __nv_bfloat16>::value) {
          // The store that last read this staging box (two groups ago) is done.
          if (lane == 0) bulk_wait_group_read<1>();
          __syncwarp();
          uint8_t* const box = stage_out + (store_seq & 1u) * kGemm2StoreBoxBytes;
          const uint32_t row_addr = smem_u32(box) + static_cast<uint32_t>(lane) * 64u;
          const uint32_t swz = (static_cast<uint32_t>(lane) >> 1) & 3u;  // 64-byte swizzle
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            st_shared_v4(row_addr + ((static_cast<uint32_t>(j) ^ swz) << 4), pack_bf16x2(v[8 * j], v[8 * j + 1]),
                         pack_bf16x2(v[8 * j + 2], v[8 * j + 3]), pack_bf16x2(v[8 * j + 4], v[8 * j + 5]),
                         pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (row_base < args.M && col0 < args.N) tma_store_2d(&tmap_out, box, col0, row_base);
            bulk_commit_group();
          }
          ++store_seq;
        } else if (row < args.M) {
          float* out_row = static_cast<float*>(args.out) + row * args.N + col0;
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            if (col0 + i < args.N)
              st_global_v4(out_row + i, __float_as_uint(v[i]), __float_as_uint(v[i + 1]), __float_as_uint(v[i + 2]),
                           __float_as_uint(v[i + 3]));
          }
        }
        if (c + 1 < chunks) tmem_wait_ld();
      }
      // This warp has read its columns of the accumulator: one arrival on the
      // leader's barrier (remote for the peer CTA).
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? acc_empty_leader1 : acc_empty_leader0);
    }
    // No store may still read the staging boxes (or be unperformed) when the
    // CTA leaves.
    if constexpr (std::is_same<OutT, __nv_bfloat16>::value) {
      if (lane == 0) bulk_wait_group_all();
      __syncwarp();
    }
  }

  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kGemmTmemCols);
  }
}

}  // namespace b200tx
