// gemm_rownorm_kernels.cuh -- the projection that closes a block branch fused
// with the residual add and LayerNorm after it, for d_model 512, 768 and 1024,
// on the tcgen05 tensor cores:
//     u = round(x[rows, K] . w[cols, K]^T + bias)     (to the unfused program's update dtype)
//     r = residual_in + u;  normed = LayerNorm(r) * gamma + beta;  residual_out = r
// Replaces, for these widths, the reference's fused Linear residual-norm
// boundary (solution/kernels/boundary/triton_linear_residual_norm.py:33-112,
// built there for D 32 and 128) and, in the unfused program, the out-projection
// or FFN-out GEMM followed by the residual LayerNorm.  The update never goes to
// memory: the row is complete in the tensor memory of one CTA pair.
//
// A tile is 128 rows x all `cols` columns, computed by a cluster of two CTAs:
// CTA c owns columns [c * cols/2, (c + 1) * cols/2) (256, 384 or 512 of them),
// accumulated in its TMEM as fp32 (up to all 512 columns).  Both CTAs read the
// same 128 rows of x.  The UMMAs are cta_group::1, M = 128, N = 128, one per
// 128-row piece of the CTA's w rows and 16-wide K step.
//   warp 0       TMA: per 64-wide K slab, the x tile into a 3-slot ring and
//                the w pieces (128 rows each) into a 10-slot ring
//   warp 1       one thread issues the UMMAs and commits the ring slots; the
//                accumulator is released by the epilogue after each tile
//   warps 2..9   epilogue, warp w reading TMEM lane quarter w % 4 (32 rows) and
//                column half (w - 2) / 4 of the CTA's columns, one row per thread:
//                pass 1: v = residual + round(acc + bias), written back over the
//                        accumulator in TMEM, partial row sums;
//                pass 2: partial sums of (v - mean)^2 (two-pass variance, as
//                        the standalone LayerNorm kernel);
//                pass 3: residual_out = v, normed = (v - mean) * rstd * gamma + beta.
//                The four partial sums of a row (two column halves x two CTAs)
//                are exchanged through shared memory: each thread writes its
//                partial into its own and the partner CTA's exchange slots and
//                arrives on both CTAs' exchange barrier (512 arrivals: every
//                thread of the pair), whose bounded wait then reads all four.
// Padding-row modes as b200tx_residual_layer_norm_masked.  Every wait is
// bounded; a cluster barrier keeps both CTAs alive until the pair is done.
#pragma once

#include "norm_kernels.cuh"
#include "sm100_common.cuh"

namespace b200tx {

constexpr int kRnBM = 128;
constexpr int kRnBK = 64;
constexpr int kRnPieceRows = 128;  // w rows per ring slot and UMMA N
constexpr int kRnARing = 3;
constexpr int kRnWRing = 10;
constexpr int kRnThreads = 320;
constexpr int kRnEpilogueThreads = 256;
constexpr int kRnMaxHalf = 512;  // columns per CTA
constexpr uint32_t kRnTmemCols = 512;
constexpr uint32_t kRnATileBytes = kRnBM * kRnBK * 2;         // 16 KB
constexpr uint32_t kRnWTileBytes = kRnPieceRows * kRnBK * 2;  // 16 KB
constexpr size_t kRnSmemBytes = 1024 + kRnARing * kRnATileBytes + kRnWRing * kRnWTileBytes;  // 209 KB

struct RowNormArgs {
  const float* bias;         // [cols]
  const void* residual_in;   // [rows, cols] fp32 or bf16
  float* residual_out;       // [rows, cols] fp32, or null
  void* normed;              // [rows, cols] bf16 or fp32
  const float* gamma;        // [cols]
  const float* beta;         // [cols]
  const uint8_t* row_valid;  // [rows] or null
  int mask_mode;             // kNormMask* bits for rows whose flag is 0
  int rows, cols, inner;     // M, N (= d_model), K
  int num_tiles;
  int round_update_bf16;     // the unfused program stores the update in bf16
  float eps;
};

__device__ __forceinline__ void st_shared_cluster_f32(uint32_t cluster_addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cluster_addr), "f"(v) : "memory");
}

// mbar_wait with acquire at cluster scope: the phase was completed by
// arrivals (release at cluster scope) of the partner CTA, whose shared-memory
// stores into this CTA must be visible after the wait.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, unsigned int code,
                                                  volatile int* abort_flag) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const unsigned long long start = global_timer_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait_cluster(bar, parity)) {
    if ((++spins & 255u) == 0u) {
      if (*abort_flag != 0 || device_error_raised()) {
        *abort_flag = 1;
        return false;
      }
      if (global_timer_ns() - start > kWaitTimeoutNs) {
        record_device_error(code);
        *abort_flag = 1;
        return false;
      }
    }
  }
  return true;
}

template <typename InT, typename OutT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kRnThreads, 1)
    gemm_residual_layernorm_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                   const __grid_constant__ CUtensorMap tmap_w, RowNormArgs args) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t a_full_bar[kRnARing];
  __shared__ uint64_t a_empty_bar[kRnARing];
  __shared__ uint64_t w_full_bar[kRnWRing];
  __shared__ uint64_t w_empty_bar[kRnWRing];
  __shared__ uint64_t acc_full_bar;
  __shared__ uint64_t acc_empty_bar;
  __shared__ uint64_t sum_bar;  // partial row sums of both CTAs present (512 arrivals)
  __shared__ uint64_t sq_bar;   // partial centred squares of both CTAs present (512 arrivals)
  __shared__ uint64_t drain_bar;
  __shared__ float sum_part[2][2][kRnBM];  // [cta][column half][row]
  __shared__ float sq_part[2][2][kRnBM];
  __shared__ float col_bias[kRnMaxHalf];
  __shared__ float col_gamma[kRnMaxHalf];
  __shared__ float col_beta[kRnMaxHalf];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  uint8_t* smem = align_1024(smem_raw);
  uint8_t* smem_a = smem;
  uint8_t* smem_w = smem + kRnARing * kRnATileBytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cta = cluster_ctarank();
  const uint32_t partner = cta ^ 1u;
  const int half_cols = args.cols / 2;            // this CTA's columns
  const int pieces = half_cols / kRnPieceRows;    // 2, 3 or 4
  const int col_base = static_cast<int>(cta) * half_cols;
  const int num_kb = (args.inner + kRnBK - 1) / kRnBK;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int num_pairs = static_cast<int>(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    prefetch_tensor_map(&tmap_x);
    prefetch_tensor_map(&tmap_w);
    for (int s = 0; s < kRnARing; ++s) {
      mbar_init(&a_full_bar[s], 1);
      mbar_init(&a_empty_bar[s], 1);
    }
    for (int s = 0; s < kRnWRing; ++s) {
      mbar_init(&w_full_bar[s], 1);
      mbar_init(&w_empty_bar[s], 1);
    }
    mbar_init(&acc_full_bar, 1);
    mbar_init(&acc_empty_bar, kRnEpilogueThreads);
    mbar_init(&sum_bar, 2 * kRnEpilogueThreads);
    mbar_init(&sq_bar, 2 * kRnEpilogueThreads);
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, kRnTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  // Both CTAs' barriers are initialised before either arrives remotely.
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      int a_pos = 0, w_pos = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < args.num_tiles; tile += num_pairs) {
        for (int kb = 0; ok && kb < num_kb; ++kb) {
          const int as = a_pos % kRnARing;
          if (!mbar_wait(&a_empty_bar[as], ((a_pos / kRnARing) & 1) ^ 1u, kErrGemmProducerWait, &abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&a_full_bar[as], kRnATileBytes);
          tma_load_2d(smem_a + as * kRnATileBytes, &tmap_x, &a_full_bar[as], kb * kRnBK, tile * kRnBM);
          ++a_pos;
          for (int p = 0; p < pieces; ++p) {
            const int ws = w_pos % kRnWRing;
            if (!mbar_wait(&w_empty_bar[ws], ((w_pos / kRnWRing) & 1) ^ 1u, kErrGemmProducerWait, &abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&w_full_bar[ws], kRnWTileBytes);
            tma_load_2d(smem_w + ws * kRnWTileBytes, &tmap_w, &w_full_bar[ws], kb * kRnBK,
                        col_base + p * kRnPieceRows);
            ++w_pos;
          }
        }
      }
      // Drain: every load issued has landed before the CTA may exit.
      volatile int no_abort = 0;
      for (int p = a_pos > kRnARing ? a_pos - kRnARing : 0; p < a_pos; ++p)
        mbar_wait(&a_full_bar[p % kRnARing], (p / kRnARing) & 1, kErrGemmProducerWait, &no_abort);
      for (int p = w_pos > kRnWRing ? w_pos - kRnWRing : 0; p < w_pos; ++p)
        mbar_wait(&w_full_bar[p % kRnWRing], (p / kRnWRing) & 1, kErrGemmProducerWait, &no_abort);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16(kRnBM, kRnPieceRows, false, false);
      int a_pos = 0, w_pos = 0, t = 0;
      bool issued_any = false;
      bool ok = true;
      for (int tile = pair; ok && tile < args.num_tiles; tile += num_pairs, ++t) {
        // The epilogue has read the previous tile's accumulator.
        if (t > 0 && !mbar_wait(&acc_empty_bar, (t - 1) & 1, kErrGemmMmaWait, &abort_flag)) break;
        tc_fence_after();
        for (int kb = 0; ok && kb < num_kb; ++kb) {
          const int as = a_pos % kRnARing;
          if (!mbar_wait(&a_full_bar[as], (a_pos / kRnARing) & 1, kErrGemmMmaWait, &abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t a_addr = smem_u32(smem_a + as * kRnATileBytes);
          for (int p = 0; p < pieces; ++p) {
            const int ws = w_pos % kRnWRing;
            if (!mbar_wait(&w_full_bar[ws], (w_pos / kRnWRing) & 1, kErrGemmMmaWait, &abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t w_addr = smem_u32(smem_w + ws * kRnWTileBytes);
            const uint32_t d_tmem = tmem_base + p * kRnPieceRows;
#pragma unroll
            for (int k = 0; k < kRnBK / 16; ++k) {
              umma_bf16_ss(d_tmem, sw128_desc(a_addr + k * 32, 16, 1024), sw128_desc(w_addr + k * 32, 16, 1024),
                           idesc, (kb | k) != 0 ? 1u : 0u);
            }
            issued_any = true;
            umma_commit(&w_empty_bar[ws]);
            ++w_pos;
          }
          if (!ok) break;
          umma_commit(&a_empty_bar[as]);
          ++a_pos;
        }
        if (!ok) break;
        umma_commit(&acc_full_bar);
      }
      if (issued_any) {
        umma_commit(&drain_bar);
        volatile int no_abort = 0;
        mbar_wait(&drain_bar, 0, kErrGemmMmaWait, &no_abort);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int ch = (warp - 2) >> 2;                     // column half of this CTA's columns
    const int row_in_tile = quarter * 32 + lane;
    const int per_thread = half_cols / 2;               // 128, 192 or 256 columns
    const int lc0 = ch * per_thread;                    // first local column of this thread
    const int chunks = per_thread / 32;
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    // Column constants of this CTA, staged once (only epilogue threads use them).
    for (int i = static_cast<int>(threadIdx.x) - 64; i < half_cols; i += kRnEpilogueThreads) {
      col_bias[i] = args.bias != nullptr ? __ldg(args.bias + col_base + i) : 0.f;
      col_gamma[i] = __ldg(args.gamma + col_base + i);
      col_beta[i] = __ldg(args.beta + col_base + i);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kRnEpilogueThreads) : "memory");
    const InT* rin = static_cast<const InT*>(args.residual_in);
    OutT* nout = static_cast<OutT*>(args.normed);
    const uint32_t remote_sum = peer_smem_addr(&sum_part[cta][ch][row_in_tile], partner);
    const uint32_t remote_sq = peer_smem_addr(&sq_part[cta][ch][row_in_tile], partner);
    const uint32_t remote_sum_bar = peer_smem_addr(&sum_bar, partner);
    const uint32_t remote_sq_bar = peer_smem_addr(&sq_bar, partner);
    const float inv_cols = 1.0f / static_cast<float>(args.cols);
    int t = 0;
    for (int tile = pair; tile < args.num_tiles; tile += num_pairs, ++t) {
      const int64_t row = static_cast<int64_t>(tile) * kRnBM + row_in_tile;
      const bool in_range = row < args.rows;
      const bool valid = !in_range || args.row_valid == nullptr || args.row_valid[row] != 0;
      const bool add_update = valid || !(args.mask_mode & kNormMaskDropUpdate);
      const bool zero_residual = !valid && (args.mask_mode & kNormMaskZeroResidual);
      const bool zero_normed = !valid && (args.mask_mode & kNormMaskZeroNormed);
      const int64_t base = row * args.cols + col_base + lc0;
      bool ok = mbar_wait(&acc_full_bar, t & 1, kErrGemmEpilogueWait, &abort_flag);
      if (__any_sync(0xffffffffu, !ok)) break;
      __syncwarp();
      tc_fence_after();
      // Pass 1: v = residual + round(acc + bias), written back over the
      // accumulator; partial row sum.
      float sum = 0.f;
      for (int c = 0; c < chunks; ++c) {
        uint32_t acc[32];
        tmem_ld_32cols(t_row + lc0 + c * 32, acc);
        float res[32];
        if (in_range && !zero_residual) {
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const float4 r4 = load4<InT>(rin, base + c * 32 + i);
            res[i] = r4.x;
            res[i + 1] = r4.y;
            res[i + 2] = r4.z;
            res[i + 3] = r4.w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) res[i] = 0.f;
        }
        __syncwarp();
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float u = __uint_as_float(acc[i]) + col_bias[lc0 + c * 32 + i];
          if (args.round_update_bf16) u = __bfloat162float(__float2bfloat16_rn(u));
          const float v = zero_residual ? 0.f : (add_update ? res[i] + u : res[i]);
          sum += v;
          acc[i] = __float_as_uint(v);
        }
        tmem_st_32cols(t_row + lc0 + c * 32, acc);
      }
      tmem_wait_st();
      // Exchange 1: the four partial sums of this row.
      sum_part[cta][ch][row_in_tile] = sum;
      st_shared_cluster_f32(remote_sum, sum);
      mbar_arrive(&sum_bar);
      mbar_arrive_cluster(remote_sum_bar);
      ok = mbar_wait_cluster(&sum_bar, t & 1, kErrGemmEpilogueWait, &abort_flag);
      if (__any_sync(0xffffffffu, !ok)) break;
      const float mean = ((sum_part[0][0][row_in_tile] + sum_part[0][1][row_in_tile]) +
                          (sum_part[1][0][row_in_tile] + sum_part[1][1][row_in_tile])) * inv_cols;
      // Pass 2: partial sum of centred squares.
      float sq = 0.f;
      for (int c = 0; c < chunks; ++c) {
        uint32_t v[32];
        tmem_ld_32cols(t_row + lc0 + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float d = __uint_as_float(v[i]) - mean;
          sq += d * d;
        }
      }
      sq_part[cta][ch][row_in_tile] = sq;
      st_shared_cluster_f32(remote_sq, sq);
      mbar_arrive(&sq_bar);
      mbar_arrive_cluster(remote_sq_bar);
      ok = mbar_wait_cluster(&sq_bar, t & 1, kErrGemmEpilogueWait, &abort_flag);
      if (__any_sync(0xffffffffu, !ok)) break;
      const float var = ((sq_part[0][0][row_in_tile] + sq_part[0][1][row_in_tile]) +
                         (sq_part[1][0][row_in_tile] + sq_part[1][1][row_in_tile])) * inv_cols;
      const float rstd = rsqrtf(var + args.eps);
      // Pass 3: the new residual and the normalised row.
      for (int c = 0; c < chunks; ++c) {
        uint32_t v[32];
        __syncwarp();
        tmem_ld_32cols(t_row + lc0 + c * 32, v);
        tmem_wait_ld();
        const int lc = lc0 + c * 32;
        if (in_range && args.residual_out != nullptr) {
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            st_global_v4(args.residual_out + base + c * 32 + i, v[i], v[i + 1], v[i + 2], v[i + 3]);
        }
        float n[32];
#pragma unroll
        for (int i = 0; i < 32; ++i)
          n[i] = zero_normed ? 0.f
                             : (__uint_as_float(v[i]) - mean) * rstd * col_gamma[lc + i] + col_beta[lc + i];
        if (in_range) {
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            store4<OutT>(nout, base + c * 32 + i, make_float4(n[i], n[i + 1], n[i + 2], n[i + 3]));
        }
      }
      // Every column of this thread's row has been read: release the accumulator.
      tc_fence_before();
      mbar_arrive(&acc_empty_bar);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kRnTmemCols);
  }
  // The partner may still arrive on this CTA's barriers until it is done.
  cluster_sync();
}

}  // namespace b200tx
