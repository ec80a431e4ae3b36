// b200tx.cu -- the single translation unit of libb200tx: host-side argument
// checks, TMA descriptor encoding and launches for the sm_100a kernels in the
// *.cuh files next to it, behind the C ABI declared in include/b200tx.h.
//
// One translation unit keeps the device error word a plain __device__ variable
// (no relocatable device code) and lets every kernel see it.

#include "b200tx.h"

#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>
#include <utility>

#include "attention_kernels.cuh"
#include "attention_mma_kernels.cuh"
#include "attention_persistent.cuh"
#include "attention_pingpong.cuh"
#include "attention_simt_kernels.cuh"
#include "boundary_kernels.cuh"
#include "gemm_kernels.cuh"
#include "gemm_rownorm_kernels.cuh"
#include "gemm_warp_kernels.cuh"
#include "norm_kernels.cuh"
#include "seq_forward_kernels.cuh"
#include "sm100_common.cuh"

// Weight images of b200tx_sequence_forward_noalloc, the library's only fixed
// scratch array: B200TX_SEQ_NOALLOC_MAX_LAYERS layers x 6 images x 32 KB =
// 768 KB of global memory on every device that loads the library, held until
// the process exits.  In host code this name is not a device address; the
// entry point looks the address up once per device (cudaGetSymbolAddress).
static __device__ __align__(256) uint8_t
    g_seq_noalloc_images[static_cast<size_t>(B200TX_SEQ_NOALLOC_MAX_LAYERS) * b200tx::kSfWeightImages *
                         b200tx::kSfMatBytes];

namespace {

constexpr int kAbiVersion = 2;
constexpr int kMaxDevices = 64;

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t err, const char* what) {
  return fail(B200TX_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(err), cudaGetErrorString(err));
}

// Attention variant codes run 0 .. kAttnVariants-1 (B200TX_ATTN_*).
constexpr int kAttnVariants = 6;

// PINGPONG attention build: two query tiles per CTA (one CTA per SM; one
// tile with two CTAs per SM measured slower at every shape), and 2 of every
// 16 score pairs exponentiated on the FMA pipe (the measured best of 0..8).
constexpr int kPpTiles = 2;
constexpr int kPpPolyPairs = 2;

struct DeviceState {
  bool probed = false;
  int sm_count = 0;
  int cc_major = 0;
  int cc_minor = 0;
  bool gemm_attr[8] = {false, false, false, false, false, false, false, false};
  bool attn_attr[2 * kAttnVariants] = {};  // unmasked builds by variant, then the masked builds
  bool rownorm_attr[4] = {};               // GEMM + residual LayerNorm builds by (in, out) dtype
  int rownorm_clusters[4][5] = {};         // their co-resident clusters by CTA pairs per cluster
  bool seq_forward_attr = false;           // whole-forward kernel's shared-memory size set
  uint8_t* seq_noalloc_images = nullptr;   // device address of g_seq_noalloc_images on this device
};

std::mutex g_mutex;
DeviceState g_devices[kMaxDevices];
PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;

// Looks up the current device, checks it is an sm_100 part and fills `state`.
int current_device(DeviceState** state) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(B200TX_ERR_UNSUPPORTED, "device index %d", dev);
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState& s = g_devices[dev];
  if (!s.probed) {
    err = cudaDeviceGetAttribute(&s.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (err != cudaSuccess) return cuda_fail(err, "cudaDeviceGetAttribute(SM count)");
    err = cudaDeviceGetAttribute(&s.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
    if (err != cudaSuccess) return cuda_fail(err, "cudaDeviceGetAttribute(cc major)");
    err = cudaDeviceGetAttribute(&s.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (err != cudaSuccess) return cuda_fail(err, "cudaDeviceGetAttribute(cc minor)");
    s.probed = true;
  }
  if (s.cc_major != 10 || s.cc_minor != 0) {
    return fail(B200TX_ERR_UNSUPPORTED,
                "libb200tx is built for sm_100a only; device %d has compute capability %d.%d", dev,
                s.cc_major, s.cc_minor);
  }
  *state = &s;
  return B200TX_OK;
}

int encoder(PFN_cuTensorMapEncodeTiled_v12000* out) {
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_encode_tiled == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    cudaError_t err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (err != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr) {
      return fail(B200TX_ERR_DRIVER, "driver entry point cuTensorMapEncodeTiled unavailable");
    }
    g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  *out = g_encode_tiled;
  return B200TX_OK;
}

// Tiled bf16 tensor map (128-byte swizzle unless given); out-of-range elements
// of a box read as zero and are not written by stores.  dims/strides innermost
// first; strides in bytes for dims 1..
int encode_tiled_map(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, int rank,
                     const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                     CUtensorMapSwizzle swizzle) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  int rc = encoder(&encode);
  if (rc != B200TX_OK) return rc;
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t bx[5];
  cuuint32_t es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  CUresult res = encode(map, dtype, static_cast<cuuint32_t>(rank),
                        const_cast<void*>(base), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) {
    return fail(B200TX_ERR_DRIVER, "cuTensorMapEncodeTiled failed with CUresult %d", int(res));
  }
  return B200TX_OK;
}

int encode_bf16_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box,
                    CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  return encode_tiled_map(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, rank, dims, strides_bytes, box, swizzle);
}

// A [rows, cols] row-major matrix of fp32 or bf16 in 32 x 32 boxes (128- or
// 64-byte rows, swizzled to match).
int encode_box32_map(CUtensorMap* map, const void* base, bool fp32, int64_t rows, int64_t cols) {
  const uint64_t dims[2] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows)};
  const uint64_t strides[1] = {static_cast<uint64_t>(cols) * (fp32 ? 4 : 2)};
  const uint32_t box[2] = {32u, 32u};
  return encode_tiled_map(map, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, 2,
                          dims, strides, box, fp32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Every kernel goes out with programmatic stream serialization (see
// griddep_wait in sm100_common.cuh): the next launch of the stream may start
// its set-up while this one drains.  Compile-time cluster dimensions of a
// kernel are kept.
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                   cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// As launch, for kernels whose cluster size is chosen at run time.
template <typename... KArgs, typename... Args>
cudaError_t launch_clustered(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, unsigned cluster_x,
                             cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ------------------------------------------------------------------ norms
template <int NV, typename InT, typename UpdT, typename OutT>
cudaError_t launch_norm_vec(const b200tx::NormArgs& a, cudaStream_t stream) {
  const unsigned grid =
      static_cast<unsigned>((a.rows + b200tx::kNormWarpsPerBlock - 1) / b200tx::kNormWarpsPerBlock);
  return launch(b200tx::residual_layernorm_vec_kernel<NV, InT, UpdT, OutT>, dim3(grid),
                dim3(b200tx::kNormWarpsPerBlock * 32), 0, stream, a);
}

template <typename InT, typename UpdT, typename OutT>
cudaError_t launch_norm(const b200tx::NormArgs& a, bool vec_ok, cudaStream_t stream) {
  if (vec_ok && a.cols % 128 == 0) {
    switch (a.cols / 128) {
      case 1: return launch_norm_vec<1, InT, UpdT, OutT>(a, stream);
      case 2: return launch_norm_vec<2, InT, UpdT, OutT>(a, stream);
      case 4: return launch_norm_vec<4, InT, UpdT, OutT>(a, stream);
      case 6: return launch_norm_vec<6, InT, UpdT, OutT>(a, stream);
      case 8: return launch_norm_vec<8, InT, UpdT, OutT>(a, stream);
      case 12: return launch_norm_vec<12, InT, UpdT, OutT>(a, stream);
      case 16: return launch_norm_vec<16, InT, UpdT, OutT>(a, stream);
      case 24: return launch_norm_vec<24, InT, UpdT, OutT>(a, stream);
      case 32: return launch_norm_vec<32, InT, UpdT, OutT>(a, stream);
      default: break;
    }
  }
  const unsigned grid =
      static_cast<unsigned>((a.rows + b200tx::kNormWarpsPerBlock - 1) / b200tx::kNormWarpsPerBlock);
  return launch(b200tx::residual_layernorm_generic_kernel<InT, UpdT, OutT>, dim3(grid),
                dim3(b200tx::kNormWarpsPerBlock * 32), 0, stream, a);
}

template <typename InT, typename UpdT>
cudaError_t launch_norm_out(const b200tx::NormArgs& a, int out_dtype, bool vec_ok,
                            cudaStream_t stream) {
  if (out_dtype == B200TX_BF16) return launch_norm<InT, UpdT, __nv_bfloat16>(a, vec_ok, stream);
  return launch_norm<InT, UpdT, float>(a, vec_ok, stream);
}

}  // namespace

extern "C" {

int b200tx_abi_version(void) { return kAbiVersion; }

const char* b200tx_last_error(void) { return g_last_error.c_str(); }

int b200tx_device_check(int* sm_count_out, int* cc_major_out, int* cc_minor_out) {
  DeviceState* s = nullptr;
  int rc = current_device(&s);
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices) {
    const DeviceState& d = g_devices[dev];
    if (sm_count_out) *sm_count_out = d.sm_count;
    if (cc_major_out) *cc_major_out = d.cc_major;
    if (cc_minor_out) *cc_minor_out = d.cc_minor;
  }
  return rc;
}

int b200tx_device_error(int clear, unsigned int* code_out) {
  cudaError_t err = cudaDeviceSynchronize();
  if (err != cudaSuccess) return cuda_fail(err, "cudaDeviceSynchronize");
  unsigned int code = 0;
  err = cudaMemcpyFromSymbol(&code, b200tx::g_device_error, sizeof(code));
  if (err != cudaSuccess) return cuda_fail(err, "reading the device error word");
  if (clear) {
    const unsigned int zero = 0;
    err = cudaMemcpyToSymbol(b200tx::g_device_error, &zero, sizeof(zero));
    if (err != cudaSuccess) return cuda_fail(err, "clearing the device error word");
  }
  if (code_out) *code_out = code;
  return B200TX_OK;
}

int b200tx_device_error_async(unsigned int* word, cudaStream_t stream) {
  if (word == nullptr) return fail(B200TX_ERR_INVALID_ARGUMENT, "device_error_async: null destination");
  cudaError_t err = cudaMemcpyFromSymbolAsync(word, b200tx::g_device_error, sizeof(unsigned int), 0,
                                              cudaMemcpyDefault, stream);
  if (err != cudaSuccess) return cuda_fail(err, "device_error_async: cudaMemcpyFromSymbolAsync");
  return B200TX_OK;
}

}  // extern "C"

namespace {

int residual_layer_norm_impl(const void* residual_in, int in_dtype, const void* update,
                             int update_dtype, float* residual_out, void* normed, int out_dtype,
                             const float* gamma, const float* beta, const uint8_t* row_valid,
                             int mask_mode, int64_t rows, int64_t cols, float eps,
                             cudaStream_t stream) {
  if (mask_mode < 0 || mask_mode > 7)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "residual_layer_norm: mask_mode %d", mask_mode);
  if (residual_in == nullptr || normed == nullptr || gamma == nullptr || beta == nullptr)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "residual_layer_norm: null tensor pointer");
  if (rows <= 0 || cols <= 0 || cols > (1 << 20))
    return fail(B200TX_ERR_INVALID_ARGUMENT, "residual_layer_norm: bad shape [%lld, %lld]",
                (long long)rows, (long long)cols);
  if ((rows + b200tx::kNormWarpsPerBlock - 1) / b200tx::kNormWarpsPerBlock > 0x7fffffffLL)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "residual_layer_norm: too many rows");
  if (in_dtype != B200TX_F32 && in_dtype != B200TX_BF16)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "residual_layer_norm: in_dtype %d", in_dtype);
  if (out_dtype != B200TX_F32 && out_dtype != B200TX_BF16)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "residual_layer_norm: out_dtype %d", out_dtype);
  if (update != nullptr && update_dtype != B200TX_F32 && update_dtype != B200TX_BF16)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "residual_layer_norm: update_dtype %d", update_dtype);
  DeviceState* dev = nullptr;
  int rc = current_device(&dev);
  if (rc != B200TX_OK) return rc;

  b200tx::NormArgs a;
  a.residual_in = residual_in;
  a.update = update;
  a.residual_out = residual_out;
  a.normed = normed;
  a.gamma = gamma;
  a.beta = beta;
  a.row_valid = row_valid;
  a.mask_mode = row_valid != nullptr ? mask_mode : 0;
  a.rows = rows;
  a.cols = static_cast<int>(cols);
  a.eps = eps;
  const bool vec_ok = aligned16(residual_in) && aligned16(normed) && aligned16(gamma) &&
                      aligned16(beta) && (update == nullptr || aligned16(update)) &&
                      (residual_out == nullptr || aligned16(residual_out));
  cudaError_t err;
  if (in_dtype == B200TX_F32) {
    if (update == nullptr)
      err = launch_norm_out<float, void>(a, out_dtype, vec_ok, stream);
    else if (update_dtype == B200TX_BF16)
      err = launch_norm_out<float, __nv_bfloat16>(a, out_dtype, vec_ok, stream);
    else
      err = launch_norm_out<float, float>(a, out_dtype, vec_ok, stream);
  } else {
    if (update == nullptr)
      err = launch_norm_out<__nv_bfloat16, void>(a, out_dtype, vec_ok, stream);
    else if (update_dtype == B200TX_BF16)
      err = launch_norm_out<__nv_bfloat16, __nv_bfloat16>(a, out_dtype, vec_ok, stream);
    else
      err = launch_norm_out<__nv_bfloat16, float>(a, out_dtype, vec_ok, stream);
  }
  if (err != cudaSuccess) return cuda_fail(err, "residual_layer_norm launch");
  return B200TX_OK;
}

}  // namespace

extern "C" {

int b200tx_residual_layer_norm(const void* residual_in, int in_dtype, const void* update,
                               int update_dtype, float* residual_out, void* normed,
                               int out_dtype, const float* gamma, const float* beta,
                               int64_t rows, int64_t cols, float eps, cudaStream_t stream) {
  return residual_layer_norm_impl(residual_in, in_dtype, update, update_dtype, residual_out, normed,
                                  out_dtype, gamma, beta, nullptr, 0, rows, cols, eps, stream);
}

int b200tx_residual_layer_norm_masked(const void* residual_in, int in_dtype, const void* update,
                                      int update_dtype, float* residual_out, void* normed,
                                      int out_dtype, const float* gamma, const float* beta,
                                      const uint8_t* row_valid, int mask_mode, int64_t rows,
                                      int64_t cols, float eps, cudaStream_t stream) {
  if (row_valid == nullptr)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "residual_layer_norm_masked: null row_valid");
  return residual_layer_norm_impl(residual_in, in_dtype, update, update_dtype, residual_out, normed,
                                  out_dtype, gamma, beta, row_valid, mask_mode, rows, cols, eps,
                                  stream);
}

}  // extern "C"

namespace {

int linear_impl(const void* a, const void* w, const float* bias, void* out, int out_dtype,
                int64_t M, int64_t N, int64_t K, int epilogue, int variant, cudaStream_t stream) {
  if (variant != B200TX_GEMM_1SM && variant != B200TX_GEMM_PAIR && variant != B200TX_GEMM_WARP)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "linear: variant %d", variant);
  if (a == nullptr || w == nullptr || out == nullptr)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "linear: null tensor pointer");
  if (M <= 0 || N <= 0 || K <= 0 || M > 0x7fffffffLL || N > 0x7fffffffLL || K > 0x7fffffffLL)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "linear: bad shape M=%lld N=%lld K=%lld",
                (long long)M, (long long)N, (long long)K);
  if (K % 8 != 0 || N % 8 != 0)
    return fail(B200TX_ERR_UNSUPPORTED, "linear: K (%lld) and N (%lld) must be multiples of 8",
                (long long)K, (long long)N);
  if (!aligned16(a) || !aligned16(w) || !aligned16(out) ||
      (bias != nullptr && (reinterpret_cast<uintptr_t>(bias) & 3u) != 0))
    return fail(B200TX_ERR_INVALID_ARGUMENT, "linear: operands must be 16-byte aligned");
  if (epilogue != B200TX_EPI_BIAS && epilogue != B200TX_EPI_BIAS_GELU)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "linear: epilogue %d", epilogue);
  if (out_dtype != B200TX_F32 && out_dtype != B200TX_BF16)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "linear: out_dtype %d", out_dtype);
  DeviceState* dev = nullptr;
  int rc = current_device(&dev);
  if (rc != B200TX_OK) return rc;

  if (variant == B200TX_GEMM_WARP) {
    // No tensor maps, no TMEM: one 64 x 64 output tile per CTA.
    b200tx::WarpGemmArgs wa;
    wa.a = static_cast<const __nv_bfloat16*>(a);
    wa.w = static_cast<const __nv_bfloat16*>(w);
    wa.bias = bias;
    wa.out = out;
    wa.M = static_cast<int>(M);
    wa.N = static_cast<int>(N);
    wa.K = static_cast<int>(K);
    wa.n_tiles = static_cast<int>((N + b200tx::kWarpGemmBN - 1) / b200tx::kWarpGemmBN);
    const int64_t blocks = ((M + b200tx::kWarpGemmBM - 1) / b200tx::kWarpGemmBM) * wa.n_tiles;
    if (blocks > 0x7fffffffLL) return fail(B200TX_ERR_UNSUPPORTED, "linear: too many tiles");
    const dim3 grid(static_cast<unsigned>(blocks));
    const dim3 block(b200tx::kWarpGemmThreads);
    const bool gelu = epilogue == B200TX_EPI_BIAS_GELU;
    cudaError_t err;
    if (out_dtype == B200TX_BF16)
      err = gelu ? launch(b200tx::gemm_bf16_tn_warp_kernel<b200tx::kEpiBiasGelu, __nv_bfloat16>, grid, block, 0, stream, wa)
                 : launch(b200tx::gemm_bf16_tn_warp_kernel<b200tx::kEpiBias, __nv_bfloat16>, grid, block, 0, stream, wa);
    else
      err = gelu ? launch(b200tx::gemm_bf16_tn_warp_kernel<b200tx::kEpiBiasGelu, float>, grid, block, 0, stream, wa)
                 : launch(b200tx::gemm_bf16_tn_warp_kernel<b200tx::kEpiBias, float>, grid, block, 0, stream, wa);
    if (err != cudaSuccess) return cuda_fail(err, "linear (warp) launch");
    return B200TX_OK;
  }

  const bool paired = variant == B200TX_GEMM_PAIR;
  const int tile_m = paired ? b200tx::kGemm2BM : b200tx::kGemmBM;
  const int tile_n = paired ? b200tx::kGemm2BN : b200tx::kGemmBN;
  CUtensorMap map_a, map_w;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
    const uint32_t box[2] = {b200tx::kGemmBK, 128u};  // 128 A rows per CTA in both variants
    rc = encode_bf16_map(&map_a, a, 2, dims, strides, box);
    if (rc != B200TX_OK) return rc;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
    // W rows per CTA: the whole 256-row block, or one CTA's half of it.
    const uint32_t box[2] = {b200tx::kGemmBK, paired ? 128u : static_cast<uint32_t>(b200tx::kGemmBN)};
    rc = encode_bf16_map(&map_w, w, 2, dims, strides, box);
    if (rc != B200TX_OK) return rc;
  }
  b200tx::GemmArgs args;
  args.bias = bias;
  args.bias_vec4 = (bias != nullptr && aligned16(bias)) ? 1 : 0;
  args.out = out;
  args.M = static_cast<int>(M);
  args.N = static_cast<int>(N);
  args.K = static_cast<int>(K);
  args.num_m_tiles = static_cast<int>((M + tile_m - 1) / tile_m);
  args.num_n_tiles = static_cast<int>((N + tile_n - 1) / tile_n);
  const int64_t tiles = static_cast<int64_t>(args.num_m_tiles) * args.num_n_tiles;
  if (tiles > 0x3fffffffLL) return fail(B200TX_ERR_UNSUPPORTED, "linear: too many tiles");
  // Persistent grid: one CTA per SM, or one CTA pair per two SMs.
  const int64_t slots = paired ? dev->sm_count / 2 : dev->sm_count;
  // Pair kernel: when the last wave holds at most half as many tiles as there
  // are pairs, those tiles run as two 128-column halves each, on twice as many
  // pairs for half as long.
  int64_t units = tiles;
  int64_t full_units = tiles;
  if (paired) {
    const int64_t tail = tiles % slots;
    if (tail > 0 && 2 * tail <= slots) {
      full_units = tiles - tail;
      units = tiles + tail;
    }
  }
  args.full_units = static_cast<int>(full_units);
  args.num_units = static_cast<int>(units);
  const unsigned grid =
      static_cast<unsigned>((units < slots ? units : slots) * (paired ? 2 : 1));

  const int instance = (paired ? 4 : 0) + epilogue * 2 + (out_dtype == B200TX_F32 ? 1 : 0);
  const size_t smem = paired ? b200tx::kGemm2SmemBytes : b200tx::kGemmSmemBytes;
  auto set_smem = [&](const void* fn) -> int {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!dev->gemm_attr[instance]) {
      cudaError_t err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
      if (err != cudaSuccess) return cuda_fail(err, "linear: cudaFuncSetAttribute");
      dev->gemm_attr[instance] = true;
    }
    return B200TX_OK;
  };
  cudaError_t err = cudaSuccess;
  if (!paired) {
    using KernelFn = void (*)(CUtensorMap, CUtensorMap, b200tx::GemmArgs);
    KernelFn kernel;
    switch (instance) {
      case 0: kernel = b200tx::gemm_bf16_tn_kernel<b200tx::kEpiBias, __nv_bfloat16>; break;
      case 1: kernel = b200tx::gemm_bf16_tn_kernel<b200tx::kEpiBias, float>; break;
      case 2: kernel = b200tx::gemm_bf16_tn_kernel<b200tx::kEpiBiasGelu, __nv_bfloat16>; break;
      default: kernel = b200tx::gemm_bf16_tn_kernel<b200tx::kEpiBiasGelu, float>; break;
    }
    rc = set_smem(reinterpret_cast<const void*>(kernel));
    if (rc != B200TX_OK) return rc;
    err = launch(kernel, dim3(grid), dim3(b200tx::kGemmThreads), smem, stream, map_a, map_w, args);
  } else {
    // bf16 outputs are written by TMA stores of 32 x 32 boxes (64-byte rows,
    // 64-byte swizzle); fp32 outputs by the threads (the map is not read).
    CUtensorMap map_out = map_a;
    if (out_dtype == B200TX_BF16) {
      const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(M)};
      const uint64_t strides[1] = {static_cast<uint64_t>(N) * 2};
      const uint32_t box[2] = {32u, 32u};
      rc = encode_bf16_map(&map_out, out, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
      if (rc != B200TX_OK) return rc;
    }
    using PairFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, b200tx::GemmArgs);
    PairFn kernel;
    switch (instance) {
      case 4: kernel = b200tx::gemm_bf16_tn_pair_kernel<b200tx::kEpiBias, __nv_bfloat16>; break;
      case 5: kernel = b200tx::gemm_bf16_tn_pair_kernel<b200tx::kEpiBias, float>; break;
      case 6: kernel = b200tx::gemm_bf16_tn_pair_kernel<b200tx::kEpiBiasGelu, __nv_bfloat16>; break;
      default: kernel = b200tx::gemm_bf16_tn_pair_kernel<b200tx::kEpiBiasGelu, float>; break;
    }
    rc = set_smem(reinterpret_cast<const void*>(kernel));
    if (rc != B200TX_OK) return rc;
    err = launch(kernel, dim3(grid), dim3(b200tx::kGemmThreads), smem, stream, map_a, map_w, map_out, args);
  }
  if (err != cudaSuccess) return cuda_fail(err, "linear launch");
  return B200TX_OK;
}

}  // namespace

extern "C" {

int b200tx_linear(const void* a, const void* w, const float* bias, void* out, int out_dtype,
                  int64_t M, int64_t N, int64_t K, int epilogue, cudaStream_t stream) {
  return linear_impl(a, w, bias, out, out_dtype, M, N, K, epilogue, B200TX_GEMM_PAIR, stream);
}

int b200tx_linear_ex(const void* a, const void* w, const float* bias, void* out, int out_dtype,
                     int64_t M, int64_t N, int64_t K, int epilogue, int variant,
                     cudaStream_t stream) {
  return linear_impl(a, w, bias, out, out_dtype, M, N, K, epilogue, variant, stream);
}

}  // extern "C"

namespace {

int attention_impl(const void* qkv, const uint8_t* key_valid, void* out, int64_t batch,
                   int64_t seq, int64_t heads, int64_t head_dim, float scale, int causal,
                   int variant, cudaStream_t stream) {
  if (qkv == nullptr || out == nullptr)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "attention: null tensor pointer");
  if (batch <= 0 || seq <= 0 || heads <= 0)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "attention: bad shape B=%lld S=%lld H=%lld",
                (long long)batch, (long long)seq, (long long)heads);
  if (head_dim != b200tx::kAttnDh)
    return fail(B200TX_ERR_UNSUPPORTED, "attention: head_dim %lld (only 64 is built)",
                (long long)head_dim);
  if (variant < 0 || variant >= kAttnVariants)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "attention: variant %d", variant);
  if (!aligned16(qkv) || !aligned16(out))
    return fail(B200TX_ERR_INVALID_ARGUMENT, "attention: operands must be 16-byte aligned");
  if (key_valid != nullptr && variant != B200TX_ATTN_QUAD && variant != B200TX_ATTN_PERSISTENT &&
      variant != B200TX_ATTN_DUO && variant != B200TX_ATTN_PINGPONG)
    return fail(B200TX_ERR_UNSUPPORTED,
                "attention: padding masks are built into the QUAD, DUO, PERSISTENT and PINGPONG variants "
                "only (variant %d)",
                variant);
  if (!(scale > 0.0f)) return fail(B200TX_ERR_INVALID_ARGUMENT, "attention: scale must be > 0");
  const int64_t q_tiles = (seq + b200tx::kAttnBM - 1) / b200tx::kAttnBM;
  const int64_t units = variant == B200TX_ATTN_PAIRED       ? (q_tiles + 1) / 2
                        : variant == B200TX_ATTN_QUAD       ? (q_tiles + 3) / 4
                        : variant == B200TX_ATTN_PERSISTENT ? (q_tiles + 1) / 2
                        : variant == B200TX_ATTN_DUO        ? (q_tiles + 1) / 2
                        : variant == B200TX_ATTN_PINGPONG   ? (q_tiles + 1) / 2
                                                            : q_tiles;
  const int64_t blocks = units * heads * batch;
  if (blocks > 0x7fffffffLL || seq > 0x7fffffffLL || batch > 0x7fffffffLL)
    return fail(B200TX_ERR_UNSUPPORTED, "attention: problem too large for one launch");
  DeviceState* dev = nullptr;
  int rc = current_device(&dev);
  if (rc != B200TX_OK) return rc;

  const int64_t d_model = heads * head_dim;
  CUtensorMap map_qkv;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(3 * d_model), static_cast<uint64_t>(seq),
                              static_cast<uint64_t>(batch)};
    const uint64_t strides[2] = {static_cast<uint64_t>(3 * d_model) * 2,
                                 static_cast<uint64_t>(3 * d_model) * 2 * static_cast<uint64_t>(seq)};
    const uint32_t box[3] = {b200tx::kAttnDh, b200tx::kAttnBM, 1};
    rc = encode_bf16_map(&map_qkv, qkv, 3, dims, strides, box);
    if (rc != B200TX_OK) return rc;
  }
  b200tx::AttnArgs args;
  args.out = static_cast<__nv_bfloat16*>(out);
  args.key_valid = key_valid;
  args.batch = static_cast<int>(batch);
  args.seq = static_cast<int>(seq);
  args.heads = static_cast<int>(heads);
  args.num_q_tiles = static_cast<int>(q_tiles);
  args.scale_log2 = scale * 1.4426950408889634f;
  args.causal = causal ? 1 : 0;
  if (variant == B200TX_ATTN_PINGPONG) {
    // Persistent: at most one CTA per SM walks the items (pairs of query
    // tiles); Q, K and V tiles are all 128 x 64 boxes of the one map.
    using PpFn = void (*)(CUtensorMap, b200tx::AttnArgs);
    using Shape = b200tx::PpShape<kPpTiles>;
    const PpFn kernel =
        key_valid != nullptr
            ? b200tx::attention_fwd_dh64_pingpong_kernel<true, kPpPolyPairs, kPpTiles>
            : b200tx::attention_fwd_dh64_pingpong_kernel<false, kPpPolyPairs, kPpTiles>;
    const int attr_slot = key_valid != nullptr ? kAttnVariants + variant : variant;
    {
      std::lock_guard<std::mutex> lock(g_mutex);
      if (!dev->attn_attr[attr_slot]) {
        cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(Shape::kSmemBytes));
        if (err != cudaSuccess) return cuda_fail(err, "attention: cudaFuncSetAttribute");
        dev->attn_attr[attr_slot] = true;
      }
    }
    const int64_t items = ((q_tiles + kPpTiles - 1) / kPpTiles) * heads * batch;
    const int64_t slots = static_cast<int64_t>(dev->sm_count) * Shape::kCtasPerSm;
    const int64_t grid = items < slots ? items : slots;
    cudaError_t err = launch(kernel, dim3(static_cast<unsigned>(grid)), dim3(Shape::kThreads),
                             Shape::kSmemBytes, stream, map_qkv, args);
    if (err != cudaSuccess) return cuda_fail(err, "attention launch");
    return B200TX_OK;
  }
  if (variant == B200TX_ATTN_PERSISTENT) {
    CUtensorMap map_kv;
    const uint64_t dims[3] = {static_cast<uint64_t>(3 * d_model), static_cast<uint64_t>(seq),
                              static_cast<uint64_t>(batch)};
    const uint64_t strides[2] = {static_cast<uint64_t>(3 * d_model) * 2,
                                 static_cast<uint64_t>(3 * d_model) * 2 * static_cast<uint64_t>(seq)};
    const uint32_t box[3] = {b200tx::kAttnDh, b200tx::kAttnPBN, 1};
    rc = encode_bf16_map(&map_kv, qkv, 3, dims, strides, box);
    if (rc != B200TX_OK) return rc;
    using PersistFn = void (*)(CUtensorMap, CUtensorMap, b200tx::AttnArgs);
    const PersistFn kernel = key_valid != nullptr ? b200tx::attention_fwd_dh64_persistent_kernel<true>
                                                  : b200tx::attention_fwd_dh64_persistent_kernel<false>;
    const int attr_slot = key_valid != nullptr ? kAttnVariants + variant : variant;
    {
      std::lock_guard<std::mutex> lock(g_mutex);
      if (!dev->attn_attr[attr_slot]) {
        cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(b200tx::kAttnPSmemBytes));
        if (err != cudaSuccess) return cuda_fail(err, "attention: cudaFuncSetAttribute");
        dev->attn_attr[attr_slot] = true;
      }
    }
    // Persistent: at most one CTA per SM walks the work items.
    const int64_t grid = blocks < dev->sm_count ? blocks : dev->sm_count;
    cudaError_t err = launch(kernel, dim3(static_cast<unsigned>(grid)), dim3(b200tx::kAttnPThreads),
                             b200tx::kAttnPSmemBytes, stream, map_qkv, map_kv, args);
    if (err != cudaSuccess) return cuda_fail(err, "attention launch");
    return B200TX_OK;
  }
  if (variant == B200TX_ATTN_QUAD || variant == B200TX_ATTN_DUO) {
    CUtensorMap map_kv;
    const uint64_t dims[3] = {static_cast<uint64_t>(3 * d_model), static_cast<uint64_t>(seq),
                              static_cast<uint64_t>(batch)};
    const uint64_t strides[2] = {static_cast<uint64_t>(3 * d_model) * 2,
                                 static_cast<uint64_t>(3 * d_model) * 2 * static_cast<uint64_t>(seq)};
    const uint32_t box[3] = {b200tx::kAttnDh, b200tx::kAttn4BN, 1};
    rc = encode_bf16_map(&map_kv, qkv, 3, dims, strides, box);
    if (rc != B200TX_OK) return rc;
    // The context [batch, seq, d_model] in [32 x 64] boxes: one per softmax
    // warp's rows of one head.
    CUtensorMap map_out;
    const uint64_t out_dims[3] = {static_cast<uint64_t>(d_model), static_cast<uint64_t>(seq),
                                  static_cast<uint64_t>(batch)};
    const uint64_t out_strides[2] = {static_cast<uint64_t>(d_model) * 2,
                                     static_cast<uint64_t>(d_model) * 2 * static_cast<uint64_t>(seq)};
    const uint32_t out_box[3] = {b200tx::kAttnDh, 32, 1};
    rc = encode_bf16_map(&map_out, out, 3, out_dims, out_strides, out_box);
    if (rc != B200TX_OK) return rc;
    using QuadFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, b200tx::AttnArgs);
    const bool duo = variant == B200TX_ATTN_DUO;
    const QuadFn quad_kernel =
        duo ? (key_valid != nullptr ? b200tx::attention_fwd_dh64_quad_kernel<true, 2>
                                    : b200tx::attention_fwd_dh64_quad_kernel<false, 2>)
            : (key_valid != nullptr ? b200tx::attention_fwd_dh64_quad_kernel<true, 4>
                                    : b200tx::attention_fwd_dh64_quad_kernel<false, 4>);
    const size_t smem = duo ? b200tx::QuadShape<2>::kSmemBytes : b200tx::QuadShape<4>::kSmemBytes;
    const int threads = duo ? b200tx::QuadShape<2>::kThreads : b200tx::QuadShape<4>::kThreads;
    const int attr_slot = key_valid != nullptr ? kAttnVariants + variant : variant;
    {
      std::lock_guard<std::mutex> lock(g_mutex);
      if (!dev->attn_attr[attr_slot]) {
        cudaError_t err = cudaFuncSetAttribute(quad_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
        if (err != cudaSuccess) return cuda_fail(err, "attention: cudaFuncSetAttribute");
        dev->attn_attr[attr_slot] = true;
      }
    }
    cudaError_t err = launch(quad_kernel, dim3(static_cast<unsigned>(blocks)), dim3(threads), smem,
                             stream, map_qkv, map_kv, map_out, args);
    if (err != cudaSuccess) return cuda_fail(err, "attention launch");
    return B200TX_OK;
  }
  using KernelFn = void (*)(CUtensorMap, b200tx::AttnArgs);
  const KernelFn kernel = variant == B200TX_ATTN_PAIRED ? b200tx::attention_fwd_dh64_pair_kernel
                                                        : b200tx::attention_fwd_dh64_kernel;
  const size_t smem = variant == B200TX_ATTN_PAIRED ? b200tx::kAttn2SmemBytes : b200tx::kAttnSmemBytes;
  const int threads = variant == B200TX_ATTN_PAIRED ? b200tx::kAttn2Threads : b200tx::kAttnThreads;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!dev->attn_attr[variant]) {
      cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
      if (err != cudaSuccess) return cuda_fail(err, "attention: cudaFuncSetAttribute");
      dev->attn_attr[variant] = true;
    }
  }
  cudaError_t err = launch(kernel, dim3(static_cast<unsigned>(blocks)), dim3(threads), smem, stream,
                           map_qkv, args);
  if (err != cudaSuccess) return cuda_fail(err, "attention launch");
  return B200TX_OK;
}

}  // namespace

extern "C" {

int b200tx_attention_ex(const void* qkv, void* out, int64_t batch, int64_t seq, int64_t heads,
                        int64_t head_dim, float scale, int causal, int variant, cudaStream_t stream) {
  return attention_impl(qkv, nullptr, out, batch, seq, heads, head_dim, scale, causal, variant,
                        stream);
}

int b200tx_attention_masked(const void* qkv, const uint8_t* key_valid, void* out, int64_t batch,
                            int64_t seq, int64_t heads, int64_t head_dim, float scale, int causal,
                            int variant, cudaStream_t stream) {
  if (key_valid == nullptr)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "attention_masked: null key_valid");
  return attention_impl(qkv, key_valid, out, batch, seq, heads, head_dim, scale, causal, variant,
                        stream);
}

int b200tx_peer_alloc(size_t bytes, void** device_ptr_out, void* ipc_handle_out) {
  if (device_ptr_out == nullptr || ipc_handle_out == nullptr || bytes == 0)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "peer_alloc: null output or zero size");
  void* p = nullptr;
  cudaError_t err = cudaMalloc(&p, bytes);
  if (err != cudaSuccess) return cuda_fail(err, "peer_alloc: cudaMalloc");
  err = cudaMemset(p, 0, bytes);
  if (err == cudaSuccess) {
    cudaIpcMemHandle_t h;
    err = cudaIpcGetMemHandle(&h, p);
    if (err == cudaSuccess) {
      static_assert(sizeof(h) == B200TX_IPC_HANDLE_BYTES, "IPC handle size");
      std::memcpy(ipc_handle_out, &h, sizeof(h));
      *device_ptr_out = p;
      return B200TX_OK;
    }
  }
  cudaFree(p);
  return cuda_fail(err, "peer_alloc: zero fill / cudaIpcGetMemHandle");
}

int b200tx_peer_open(const void* ipc_handle, void** device_ptr_out) {
  if (ipc_handle == nullptr || device_ptr_out == nullptr)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "peer_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t err = cudaIpcOpenMemHandle(device_ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) return cuda_fail(err, "peer_open: cudaIpcOpenMemHandle");
  return B200TX_OK;
}

int b200tx_peer_close(void* device_ptr) {
  cudaError_t err = cudaIpcCloseMemHandle(device_ptr);
  if (err != cudaSuccess) return cuda_fail(err, "peer_close: cudaIpcCloseMemHandle");
  return B200TX_OK;
}

int b200tx_peer_free(void* device_ptr) {
  cudaError_t err = cudaFree(device_ptr);
  if (err != cudaSuccess) return cuda_fail(err, "peer_free: cudaFree");
  return B200TX_OK;
}

int b200tx_peer_signal(uint32_t* const* peer_slots, int count, uint32_t epoch, cudaStream_t stream) {
  if (peer_slots == nullptr || count <= 0 || count > b200tx::kMaxPeers)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "peer_signal: count %d (1..%d)", count, b200tx::kMaxPeers);
  DeviceState* dev = nullptr;
  int rc = current_device(&dev);
  if (rc != B200TX_OK) return rc;
  b200tx::PeerSignalArgs a = {};
  for (int i = 0; i < count; ++i) a.slots[i] = peer_slots[i];
  a.count = count;
  a.epoch = epoch;
  cudaError_t err = launch(b200tx::peer_signal_kernel, dim3(1), dim3(32), 0, stream, a);
  if (err != cudaSuccess) return cuda_fail(err, "peer_signal launch");
  return B200TX_OK;
}

int b200tx_residual_layer_norm_peer(const float* residual_in, const void* const* partials, int count,
                                    int self, const uint32_t* flags, uint32_t epoch,
                                    float* residual_out, void* normed, int out_dtype,
                                    const float* gamma, const float* beta, const uint8_t* row_valid,
                                    int mask_mode, int64_t rows, int64_t cols, float eps,
                                    cudaStream_t stream) {
  if (residual_in == nullptr || partials == nullptr || flags == nullptr || normed == nullptr ||
      gamma == nullptr || beta == nullptr)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "residual_layer_norm_peer: null pointer");
  if (count < 1 || count > b200tx::kMaxPeers || self < 0 || self >= count)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "residual_layer_norm_peer: count %d self %d", count, self);
  if (rows <= 0 || cols <= 0 || cols % 128 != 0 || (rows + 7) / 8 > 0x7fffffffLL)
    return fail(B200TX_ERR_UNSUPPORTED, "residual_layer_norm_peer: shape [%lld, %lld] (cols %% 128 == 0)",
                (long long)rows, (long long)cols);
  if (out_dtype != B200TX_F32 && out_dtype != B200TX_BF16)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "residual_layer_norm_peer: out_dtype %d", out_dtype);
  if (mask_mode < 0 || mask_mode > 7)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "residual_layer_norm_peer: mask_mode %d", mask_mode);
  bool ok = aligned16(residual_in) && aligned16(normed) && aligned16(gamma) && aligned16(beta) &&
            (residual_out == nullptr || aligned16(residual_out));
  b200tx::PeerSumArgs p = {};
  for (int i = 0; i < count; ++i) {
    if (partials[i] == nullptr || (reinterpret_cast<uintptr_t>(partials[i]) & 7u) != 0) ok = false;
    p.partials[i] = static_cast<const __nv_bfloat16*>(partials[i]);
  }
  if (!ok) return fail(B200TX_ERR_INVALID_ARGUMENT, "residual_layer_norm_peer: misaligned or null operand");
  p.count = count;
  p.self = self;
  p.flags = flags;
  p.epoch = epoch;
  DeviceState* dev = nullptr;
  int rc = current_device(&dev);
  if (rc != B200TX_OK) return rc;
  b200tx::NormArgs a;
  a.residual_in = residual_in;
  a.update = nullptr;
  a.residual_out = residual_out;
  a.normed = normed;
  a.gamma = gamma;
  a.beta = beta;
  a.row_valid = row_valid;
  a.mask_mode = row_valid != nullptr ? mask_mode : 0;
  a.rows = rows;
  a.cols = static_cast<int>(cols);
  a.eps = eps;
  const dim3 grid(static_cast<unsigned>((rows + b200tx::kNormWarpsPerBlock - 1) / b200tx::kNormWarpsPerBlock));
  const dim3 block(b200tx::kNormWarpsPerBlock * 32);
  const bool bf16 = out_dtype == B200TX_BF16;
  cudaError_t err;
#define B200TX_PEER_NV(NV)                                                                         \
  case NV:                                                                                        \
    err = bf16 ? launch(b200tx::residual_layernorm_peer_kernel<NV, __nv_bfloat16>, grid, block, 0, \
                        stream, a, p)                                                             \
               : launch(b200tx::residual_layernorm_peer_kernel<NV, float>, grid, block, 0, stream, a, p); \
    break;
  switch (cols / 128) {
    B200TX_PEER_NV(1)
    B200TX_PEER_NV(2)
    B200TX_PEER_NV(4)
    B200TX_PEER_NV(6)
    B200TX_PEER_NV(8)
    B200TX_PEER_NV(12)
    B200TX_PEER_NV(16)
    default:
      return fail(B200TX_ERR_UNSUPPORTED, "residual_layer_norm_peer: cols %lld not built", (long long)cols);
  }
#undef B200TX_PEER_NV
  if (err != cudaSuccess) return cuda_fail(err, "residual_layer_norm_peer launch");
  return B200TX_OK;
}

int b200tx_residual_layer_norm_peer_rs(const float* residual_in, const void* const* partials, int count,
                                       int self, const uint32_t* flags, uint32_t epoch, int64_t row_begin,
                                       int64_t row_count, float* residual_out, void* const* outs,
                                       int out_dtype, const float* gamma, const float* beta,
                                       uint32_t* const* done_slots, uint32_t* counter, uint32_t counter_base,
                                       uint32_t* counter_after, int64_t rows, int64_t cols, float eps,
                                       cudaStream_t stream) {
  if (residual_in == nullptr || partials == nullptr || flags == nullptr || outs == nullptr ||
      done_slots == nullptr || counter == nullptr || gamma == nullptr || beta == nullptr)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "residual_layer_norm_peer_rs: null pointer");
  if (count < 2 || count > b200tx::kMaxPeers || self < 0 || self >= count)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "residual_layer_norm_peer_rs: count %d self %d", count, self);
  if (rows <= 0 || cols <= 0 || cols % 128 != 0 || row_begin < 0 || row_count <= 0 ||
      row_begin + row_count > rows || (row_count + 7) / 8 > 0x7fffffffLL)
    return fail(B200TX_ERR_UNSUPPORTED,
                "residual_layer_norm_peer_rs: rows [%lld, %lld) of [%lld, %lld] (cols %% 128 == 0)",
                (long long)row_begin, (long long)(row_begin + row_count), (long long)rows, (long long)cols);
  if (out_dtype != B200TX_F32 && out_dtype != B200TX_BF16)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "residual_layer_norm_peer_rs: out_dtype %d", out_dtype);
  bool ok = aligned16(residual_in) && aligned16(gamma) && aligned16(beta) &&
            (residual_out == nullptr || aligned16(residual_out)) &&
            (reinterpret_cast<uintptr_t>(counter) & 3u) == 0;
  b200tx::PeerSumArgs p = {};
  b200tx::PeerGatherArgs g = {};
  for (int i = 0; i < count; ++i) {
    if (partials[i] == nullptr || (reinterpret_cast<uintptr_t>(partials[i]) & 7u) != 0) ok = false;
    if (outs[i] == nullptr || !aligned16(outs[i])) ok = false;
    if (i != self && done_slots[i] == nullptr) ok = false;
    p.partials[i] = static_cast<const __nv_bfloat16*>(partials[i]);
    g.outs[i] = outs[i];
    g.done_slots[i] = i == self ? nullptr : done_slots[i];
  }
  if (!ok) return fail(B200TX_ERR_INVALID_ARGUMENT, "residual_layer_norm_peer_rs: misaligned or null operand");
  p.count = count;
  p.self = self;
  p.flags = flags;
  p.epoch = epoch;
  DeviceState* dev = nullptr;
  int rc = current_device(&dev);
  if (rc != B200TX_OK) return rc;
  b200tx::NormArgs a;
  a.residual_in = residual_in;
  a.update = nullptr;
  a.residual_out = residual_out;
  a.normed = outs[self];
  a.gamma = gamma;
  a.beta = beta;
  a.row_valid = nullptr;
  a.mask_mode = 0;
  a.rows = row_count;
  a.cols = static_cast<int>(cols);
  a.eps = eps;
  const unsigned ctas = static_cast<unsigned>((row_count + b200tx::kNormWarpsPerBlock - 1) / b200tx::kNormWarpsPerBlock);
  g.counter = counter;
  g.counter_target = counter_base + ctas;
  g.row_begin = row_begin;
  const dim3 block(b200tx::kNormWarpsPerBlock * 32);
  const bool bf16 = out_dtype == B200TX_BF16;
  cudaError_t err;
#define B200TX_PEER_RS_NV(NV)                                                                            \
  case NV:                                                                                              \
    err = bf16 ? launch(b200tx::residual_layernorm_peer_rs_kernel<NV, __nv_bfloat16>, dim3(ctas), block, 0, \
                        stream, a, p, g)                                                                \
               : launch(b200tx::residual_layernorm_peer_rs_kernel<NV, float>, dim3(ctas), block, 0, stream, a, \
                        p, g);                                                                          \
    break;
  switch (cols / 128) {
    B200TX_PEER_RS_NV(1)
    B200TX_PEER_RS_NV(2)
    B200TX_PEER_RS_NV(4)
    B200TX_PEER_RS_NV(6)
    B200TX_PEER_RS_NV(8)
    B200TX_PEER_RS_NV(12)
    B200TX_PEER_RS_NV(16)
    default:
      return fail(B200TX_ERR_UNSUPPORTED, "residual_layer_norm_peer_rs: cols %lld not built", (long long)cols);
  }
#undef B200TX_PEER_RS_NV
  if (err != cudaSuccess) return cuda_fail(err, "residual_layer_norm_peer_rs launch");
  if (counter_after != nullptr) *counter_after = g.counter_target;
  return B200TX_OK;
}

int b200tx_peer_wait(const uint32_t* flags, int count, int self, uint32_t epoch, cudaStream_t stream) {
  if (flags == nullptr || count < 1 || count > b200tx::kMaxPeers || self < 0 || self >= count)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "peer_wait: count %d self %d", count, self);
  DeviceState* dev = nullptr;
  int rc = current_device(&dev);
  if (rc != B200TX_OK) return rc;
  cudaError_t err = launch(b200tx::peer_wait_kernel, dim3(1), dim3(32), 0, stream, flags, count, self, epoch);
  if (err != cudaSuccess) return cuda_fail(err, "peer_wait launch");
  return B200TX_OK;
}

int b200tx_seq_weight_image(const void* weight, void* image, cudaStream_t stream) {
  if (weight == nullptr || image == nullptr || !aligned16(weight) || !aligned16(image))
    return fail(B200TX_ERR_INVALID_ARGUMENT, "seq_weight_image: null or misaligned pointer");
  DeviceState* dev = nullptr;
  int rc = current_device(&dev);
  if (rc != B200TX_OK) return rc;
  cudaError_t err = launch(b200tx::seq_weight_image_kernel, dim3(b200tx::kSfRows * (b200tx::kSfD / 8) / 256),
                           dim3(256), 0, stream, static_cast<const __nv_bfloat16*>(weight),
                           static_cast<uint8_t*>(image));
  if (err != cudaSuccess) return cuda_fail(err, "seq_weight_image launch");
  return B200TX_OK;
}

int b200tx_sequence_forward(const float* x, float* out, int64_t batch, int64_t seq, int64_t d_model,
                            int64_t heads, int64_t ffn_dim, int num_layers, const b200tx_seq_layer* layers,
                            const float* ln0_gamma, const float* ln0_beta, float eps, cudaStream_t stream) {
  if (x == nullptr || out == nullptr || layers == nullptr || ln0_gamma == nullptr || ln0_beta == nullptr)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "sequence_forward: null pointer");
  if (d_model != b200tx::kSfD || ffn_dim != b200tx::kSfD)
    return fail(B200TX_ERR_UNSUPPORTED, "sequence_forward: d_model %lld ffn_dim %lld (built: 128, 128)",
                (long long)d_model, (long long)ffn_dim);
  if (heads != 1 && heads != 2 && heads != 4)
    return fail(B200TX_ERR_UNSUPPORTED, "sequence_forward: %lld heads (built: 1, 2, 4)", (long long)heads);
  if (seq != 32 && seq != 64 && seq != 128)
    return fail(B200TX_ERR_UNSUPPORTED, "sequence_forward: seq_len %lld (built: 32, 64, 128)", (long long)seq);
  if (num_layers < 1 || num_layers > b200tx::kSfMaxLayers)
    return fail(B200TX_ERR_UNSUPPORTED, "sequence_forward: %d layers (1..%d)", num_layers, b200tx::kSfMaxLayers);
  if (batch <= 0 || batch * seq > 0x7fffffffLL)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "sequence_forward: batch %lld", (long long)batch);
  bool ok = aligned16(x) && aligned16(out) && aligned16(ln0_gamma) && aligned16(ln0_beta);
  b200tx::SeqForwardArgs a = {};
  for (int l = 0; l < num_layers; ++l) {
    const b200tx_seq_layer& s = layers[l];
    const void* ptrs[] = {s.weight_images, s.b_qkv, s.b_o, s.b_1, s.b_2, s.ln2_gamma, s.ln2_beta, s.next_gamma,
                          s.next_beta};
    for (const void* q : ptrs) ok = ok && q != nullptr && aligned16(q);
    a.layers[l].w_img = static_cast<const uint8_t*>(s.weight_images);
    a.layers[l].b_qkv = s.b_qkv;
    a.layers[l].b_o = s.b_o;
    a.layers[l].b_1 = s.b_1;
    a.layers[l].b_2 = s.b_2;
    a.layers[l].ln2_g = s.ln2_gamma;
    a.layers[l].ln2_b = s.ln2_beta;
    a.layers[l].next_g = s.next_gamma;
    a.layers[l].next_b = s.next_beta;
  }
  if (!ok) return fail(B200TX_ERR_INVALID_ARGUMENT, "sequence_forward: null or misaligned operand");
  DeviceState* dev = nullptr;
  int rc = current_device(&dev);
  if (rc != B200TX_OK) return rc;
  a.x = x;
  a.out = out;
  a.ln0_g = ln0_gamma;
  a.ln0_b = ln0_beta;
  a.num_layers = num_layers;
  a.rows = static_cast<int>(batch * seq);
  a.seq = static_cast<int>(seq);
  a.heads = static_cast<int>(heads);
  a.num_tiles = (a.rows + b200tx::kSfRows - 1) / b200tx::kSfRows;
  a.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(b200tx::kSfD / heads));
  a.eps = eps;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!dev->seq_forward_attr) {
      cudaError_t err = cudaFuncSetAttribute(b200tx::seq_forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(b200tx::kSfSmemBytes));
      if (err != cudaSuccess) return cuda_fail(err, "sequence_forward: cudaFuncSetAttribute");
      dev->seq_forward_attr = true;
    }
  }
  const int ctas = a.num_tiles < dev->sm_count ? a.num_tiles : dev->sm_count;
  cudaError_t err = launch(b200tx::seq_forward_kernel, dim3(static_cast<unsigned>(ctas)), dim3(b200tx::kSfThreads),
                           b200tx::kSfSmemBytes, stream, a);
  if (err != cudaSuccess) return cuda_fail(err, "sequence_forward launch");
  return B200TX_OK;
}

// The whole forward without any allocation: the weight images go into
// g_seq_noalloc_images (rewritten by every call, on the stream, before its
// forward reads them) instead of caller-allocated memory.
int b200tx_sequence_forward_noalloc(const float* x, float* out, int64_t batch, int64_t seq, int64_t d_model,
                                    int64_t heads, int64_t ffn_dim, int num_layers,
                                    const b200tx_seq_layer_weights* layers, const float* ln0_gamma,
                                    const float* ln0_beta, float eps, cudaStream_t stream) {
  if (x == nullptr || out == nullptr || layers == nullptr || ln0_gamma == nullptr || ln0_beta == nullptr)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "sequence_forward_noalloc: null pointer");
  if (d_model != b200tx::kSfD || ffn_dim != b200tx::kSfD)
    return fail(B200TX_ERR_UNSUPPORTED, "sequence_forward_noalloc: d_model %lld ffn_dim %lld (built: 128, 128)",
                (long long)d_model, (long long)ffn_dim);
  if (heads != 1 && heads != 2 && heads != 4)
    return fail(B200TX_ERR_UNSUPPORTED, "sequence_forward_noalloc: %lld heads (built: 1, 2, 4)", (long long)heads);
  if (seq != 32 && seq != 64 && seq != 128)
    return fail(B200TX_ERR_UNSUPPORTED, "sequence_forward_noalloc: seq_len %lld (built: 32, 64, 128)",
                (long long)seq);
  if (num_layers < 1 || num_layers > B200TX_SEQ_NOALLOC_MAX_LAYERS)
    return fail(B200TX_ERR_UNSUPPORTED,
                "sequence_forward_noalloc: %d layers; its fixed image array holds 1..%d (%zu KB per device); "
                "use b200tx_sequence_forward with caller-allocated images for more",
                num_layers, B200TX_SEQ_NOALLOC_MAX_LAYERS, sizeof(g_seq_noalloc_images) / 1024);
  if (batch <= 0 || batch * seq > 0x7fffffffLL)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "sequence_forward_noalloc: batch %lld", (long long)batch);
  bool ok = aligned16(x) && aligned16(out) && aligned16(ln0_gamma) && aligned16(ln0_beta);
  for (int l = 0; l < num_layers; ++l) {
    const b200tx_seq_layer_weights& w = layers[l];
    const void* ptrs[] = {w.w_qkv, w.w_o,       w.w_1,      w.w_2,        w.b_qkv,    w.b_o,
                          w.b_1,   w.b_2,       w.ln2_gamma, w.ln2_beta, w.next_gamma, w.next_beta};
    for (const void* q : ptrs) ok = ok && q != nullptr && aligned16(q);
  }
  if (!ok) return fail(B200TX_ERR_INVALID_ARGUMENT, "sequence_forward_noalloc: null or misaligned operand");
  DeviceState* dev = nullptr;
  int rc = current_device(&dev);
  if (rc != B200TX_OK) return rc;
  {
    // Set-up, once per device, with that device current (current_device).
    std::lock_guard<std::mutex> lock(g_mutex);
    if (dev->seq_noalloc_images == nullptr) {
      void* images = nullptr;
      cudaError_t err = cudaGetSymbolAddress(&images, g_seq_noalloc_images);
      if (err != cudaSuccess) return cuda_fail(err, "sequence_forward_noalloc: cudaGetSymbolAddress");
      dev->seq_noalloc_images = static_cast<uint8_t*>(images);
    }
    if (!dev->seq_forward_attr) {
      cudaError_t err = cudaFuncSetAttribute(b200tx::seq_forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(b200tx::kSfSmemBytes));
      if (err != cudaSuccess) return cuda_fail(err, "sequence_forward_noalloc: cudaFuncSetAttribute");
      dev->seq_forward_attr = true;
    }
  }
  uint8_t* const images = dev->seq_noalloc_images;
  constexpr size_t kLayerBytes = static_cast<size_t>(b200tx::kSfWeightImages) * b200tx::kSfMatBytes;
  b200tx::SeqImageSources src = {};
  b200tx::SeqForwardArgs a = {};
  for (int l = 0; l < num_layers; ++l) {
    const b200tx_seq_layer_weights& w = layers[l];
    const auto* qkv = static_cast<const __nv_bfloat16*>(w.w_qkv);
    const __nv_bfloat16* mats[b200tx::kSfWeightImages] = {
        qkv, qkv + b200tx::kSfD * b200tx::kSfD, qkv + 2 * b200tx::kSfD * b200tx::kSfD,
        static_cast<const __nv_bfloat16*>(w.w_o), static_cast<const __nv_bfloat16*>(w.w_1),
        static_cast<const __nv_bfloat16*>(w.w_2)};
    for (int m = 0; m < b200tx::kSfWeightImages; ++m) src.w[l * b200tx::kSfWeightImages + m] = mats[m];
    a.layers[l].w_img = images + l * kLayerBytes;
    a.layers[l].b_qkv = w.b_qkv;
    a.layers[l].b_o = w.b_o;
    a.layers[l].b_1 = w.b_1;
    a.layers[l].b_2 = w.b_2;
    a.layers[l].ln2_g = w.ln2_gamma;
    a.layers[l].ln2_b = w.ln2_beta;
    a.layers[l].next_g = w.next_gamma;
    a.layers[l].next_b = w.next_beta;
  }
  cudaError_t err = launch(b200tx::seq_weight_images_kernel,
                           dim3(b200tx::kSfRows * (b200tx::kSfD / 8) / 256,
                                static_cast<unsigned>(num_layers * b200tx::kSfWeightImages)),
                           dim3(256), 0, stream, src, images);
  if (err != cudaSuccess) return cuda_fail(err, "sequence_forward_noalloc: weight image launch");
  a.x = x;
  a.out = out;
  a.ln0_g = ln0_gamma;
  a.ln0_b = ln0_beta;
  a.num_layers = num_layers;
  a.rows = static_cast<int>(batch * seq);
  a.seq = static_cast<int>(seq);
  a.heads = static_cast<int>(heads);
  a.num_tiles = (a.rows + b200tx::kSfRows - 1) / b200tx::kSfRows;
  a.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(b200tx::kSfD / heads));
  a.eps = eps;
  const int ctas = a.num_tiles < dev->sm_count ? a.num_tiles : dev->sm_count;
  err = launch(b200tx::seq_forward_kernel, dim3(static_cast<unsigned>(ctas)), dim3(b200tx::kSfThreads),
               b200tx::kSfSmemBytes, stream, a);
  if (err != cudaSuccess) return cuda_fail(err, "sequence_forward_noalloc: forward launch");
  return B200TX_OK;
}

int b200tx_attention_generic(const void* qkv, const uint8_t* key_valid, void* out, int64_t batch,
                             int64_t seq, int64_t heads, int64_t head_dim, float scale, int causal,
                             cudaStream_t stream) {
  if (qkv == nullptr || out == nullptr)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "attention_generic: null tensor pointer");
  if (batch <= 0 || seq <= 0 || heads <= 0)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "attention_generic: bad shape B=%lld S=%lld H=%lld",
                (long long)batch, (long long)seq, (long long)heads);
  if (head_dim != 8 && head_dim != 16 && head_dim != 32 && head_dim != 64 && head_dim != 128 &&
      head_dim != 256)
    return fail(B200TX_ERR_UNSUPPORTED, "attention_generic: head_dim %lld (built: 8..256, powers of 2)",
                (long long)head_dim);
  if (!aligned16(qkv) || !aligned16(out))
    return fail(B200TX_ERR_INVALID_ARGUMENT, "attention_generic: operands must be 16-byte aligned");
  if (!(scale > 0.0f)) return fail(B200TX_ERR_INVALID_ARGUMENT, "attention_generic: scale must be > 0");
  const int64_t q_blocks = (seq + b200tx::kSimtRows - 1) / b200tx::kSimtRows;
  const int64_t blocks = q_blocks * heads * batch;
  if (blocks > 0x7fffffffLL || seq > 0x7fffffffLL || heads * head_dim * 3 * seq > (1LL << 62))
    return fail(B200TX_ERR_UNSUPPORTED, "attention_generic: problem too large for one launch");
  DeviceState* dev = nullptr;
  int rc = current_device(&dev);
  if (rc != B200TX_OK) return rc;
  b200tx::SimtAttnArgs a;
  a.qkv = static_cast<const __nv_bfloat16*>(qkv);
  a.key_valid = key_valid;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.batch = static_cast<int>(batch);
  a.seq = static_cast<int>(seq);
  a.heads = static_cast<int>(heads);
  a.scale_log2 = scale * 1.4426950408889634f;
  a.causal = causal ? 1 : 0;
  const dim3 grid(static_cast<unsigned>(blocks));
  const int t = head_dim < 16 ? 1 : static_cast<int>(head_dim / 16);
  const dim3 block(static_cast<unsigned>(b200tx::kSimtRows * t));
  cudaError_t err;
  switch (head_dim) {
    case 8: err = launch(b200tx::attention_simt_kernel<8>, grid, block, 0, stream, a); break;
    case 16: err = launch(b200tx::attention_simt_kernel<16>, grid, block, 0, stream, a); break;
    case 32: err = launch(b200tx::attention_simt_kernel<32>, grid, block, 0, stream, a); break;
    case 64: err = launch(b200tx::attention_simt_kernel<64>, grid, block, 0, stream, a); break;
    case 128: err = launch(b200tx::attention_simt_kernel<128>, grid, block, 0, stream, a); break;
    default: err = launch(b200tx::attention_simt_kernel<256>, grid, block, 0, stream, a); break;
  }
  if (err != cudaSuccess) return cuda_fail(err, "attention_generic launch");
  return B200TX_OK;
}

int b200tx_attention_mma(const void* qkv, const uint8_t* key_valid, void* out, int64_t batch,
                         int64_t seq, int64_t heads, int64_t head_dim, float scale, int causal,
                         cudaStream_t stream) {
  if (qkv == nullptr || out == nullptr)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "attention_mma: null tensor pointer");
  if (batch <= 0 || seq <= 0 || heads <= 0)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "attention_mma: bad shape B=%lld S=%lld H=%lld",
                (long long)batch, (long long)seq, (long long)heads);
  if (head_dim != 8 && head_dim != 16 && head_dim != 32 && head_dim != 64 && head_dim != 128)
    return fail(B200TX_ERR_UNSUPPORTED, "attention_mma: head_dim %lld (built: 8, 16, 32, 64, 128)",
                (long long)head_dim);
  if (!aligned16(qkv) || !aligned16(out))
    return fail(B200TX_ERR_INVALID_ARGUMENT, "attention_mma: operands must be 16-byte aligned");
  if (!(scale > 0.0f)) return fail(B200TX_ERR_INVALID_ARGUMENT, "attention_mma: scale must be > 0");
  const int64_t q_blocks = (seq + b200tx::kMmaAttnRows - 1) / b200tx::kMmaAttnRows;
  const int64_t blocks = q_blocks * heads * batch;
  if (blocks > 0x7fffffffLL || batch * heads > 0x7fffffffLL ||
      batch * seq * heads * head_dim * 3 > (1LL << 62))
    return fail(B200TX_ERR_UNSUPPORTED, "attention_mma: problem too large for one launch");
  DeviceState* dev = nullptr;
  int rc = current_device(&dev);
  if (rc != B200TX_OK) return rc;
  b200tx::MmaAttnArgs a;
  a.qkv = static_cast<const __nv_bfloat16*>(qkv);
  a.key_valid = key_valid;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.batch = static_cast<int>(batch);
  a.seq = static_cast<int>(seq);
  a.heads = static_cast<int>(heads);
  a.q_blocks = static_cast<int>(q_blocks);
  a.scale_log2 = scale * 1.4426950408889634f;
  a.causal = causal ? 1 : 0;
  const dim3 grid(static_cast<unsigned>(blocks));
  const dim3 block(b200tx::kMmaAttnThreads);
  cudaError_t err;
  switch (head_dim) {
    case 8: err = launch(b200tx::attention_mma_kernel<8>, grid, block, 0, stream, a); break;
    case 16: err = launch(b200tx::attention_mma_kernel<16>, grid, block, 0, stream, a); break;
    case 32: err = launch(b200tx::attention_mma_kernel<32>, grid, block, 0, stream, a); break;
    case 64: err = launch(b200tx::attention_mma_kernel<64>, grid, block, 0, stream, a); break;
    default: err = launch(b200tx::attention_mma_kernel<128>, grid, block, 0, stream, a); break;
  }
  if (err != cudaSuccess) return cuda_fail(err, "attention_mma launch");
  return B200TX_OK;
}

}  // extern "C"

namespace {

// The Linear boundary at d_model 512 / 768 / 1024: a tcgen05 GEMM whose
// clusters of CTA pairs hold whole rows and apply the residual LayerNorm in
// their epilogue (gemm_rownorm_kernels.cuh).
int launch_gemm_rownorm(const b200tx::BoundaryArgs& a, DeviceState* dev, int in_dtype, int out_dtype,
                        int64_t rows, int64_t cols, int64_t inner, cudaStream_t stream) {
  if (!aligned16(a.residual_in) || (a.residual_out != nullptr && !aligned16(a.residual_out)) ||
      !aligned16(a.normed) || (reinterpret_cast<uintptr_t>(a.bias) & 3u) != 0)
    return fail(B200TX_ERR_INVALID_ARGUMENT,
                "linear_residual_layer_norm: at d_model %lld residual_in, residual_out and normed must be "
                "16-byte aligned",
                (long long)cols);
  const bool in_f32 = in_dtype == B200TX_F32;
  const bool out_f32 = out_dtype == B200TX_F32;
  CUtensorMap map_x, map_w, map_rin;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(inner), static_cast<uint64_t>(rows)};
    const uint64_t strides[1] = {static_cast<uint64_t>(inner) * 2};
    const uint32_t box[2] = {static_cast<uint32_t>(b200tx::kRnBK), 128u};
    int rc = encode_bf16_map(&map_x, a.x, 2, dims, strides, box);
    if (rc != B200TX_OK) return rc;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(inner), static_cast<uint64_t>(cols)};
    const uint64_t strides[1] = {static_cast<uint64_t>(inner) * 2};
    const uint32_t box[2] = {static_cast<uint32_t>(b200tx::kRnBK), 128u};
    int rc = encode_bf16_map(&map_w, a.w, 2, dims, strides, box);
    if (rc != B200TX_OK) return rc;
  }
  int rc = encode_box32_map(&map_rin, a.residual_in, in_f32, rows, cols);
  if (rc != B200TX_OK) return rc;
  b200tx::RowNormArgs r;
  r.bias = a.bias;
  r.gamma = a.gamma;
  r.beta = a.beta;
  r.row_valid = a.row_valid;
  r.residual_out = a.residual_out;
  r.normed = a.normed;
  r.mask_mode = a.mask_mode;
  r.rows = static_cast<int>(rows);
  r.cols = static_cast<int>(cols);
  r.inner = static_cast<int>(inner);
  r.pairs = static_cast<int>(cols / b200tx::kRnBN);
  r.num_tiles = static_cast<int>((rows + b200tx::kRnBM - 1) / b200tx::kRnBM);
  r.round_update_bf16 = a.update_bf16;
  r.eps = a.eps;
  using KernelFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, b200tx::RowNormArgs);
  KernelFn kernel;
  const int instance = (in_f32 ? 2 : 0) + (out_f32 ? 1 : 0);
  switch (instance) {
    case 0: kernel = b200tx::gemm_residual_layernorm_kernel<__nv_bfloat16, __nv_bfloat16>; break;
    case 1: kernel = b200tx::gemm_residual_layernorm_kernel<__nv_bfloat16, float>; break;
    case 2: kernel = b200tx::gemm_residual_layernorm_kernel<float, __nv_bfloat16>; break;
    default: kernel = b200tx::gemm_residual_layernorm_kernel<float, float>; break;
  }
  const unsigned cluster = static_cast<unsigned>(2 * r.pairs);
  int max_clusters = 0;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!dev->rownorm_attr[instance]) {
      cudaError_t err = cudaFuncSetAttribute(reinterpret_cast<const void*>(kernel),
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(b200tx::kRnSmemBytes));
      if (err != cudaSuccess) return cuda_fail(err, "linear_residual_layer_norm: cudaFuncSetAttribute");
      dev->rownorm_attr[instance] = true;
    }
    int& cached = dev->rownorm_clusters[instance][r.pairs];
    if (cached == 0) {
      // How many clusters of this size the device holds at once (one CTA per SM).
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(cluster * 64);
      cfg.blockDim = dim3(b200tx::kRnThreads);
      cfg.dynamicSmemBytes = b200tx::kRnSmemBytes;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = cluster;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      cudaError_t err = cudaOccupancyMaxActiveClusters(&cached, reinterpret_cast<const void*>(kernel), &cfg);
      if (err != cudaSuccess) return cuda_fail(err, "linear_residual_layer_norm: cudaOccupancyMaxActiveClusters");
      if (cached <= 0)
        return fail(B200TX_ERR_UNSUPPORTED, "linear_residual_layer_norm: no cluster of %u CTAs fits the device",
                    cluster);
    }
    max_clusters = cached;
  }
  // Persistent: as many clusters as are co-resident, walking the 256-row tiles.
  const int clusters = r.num_tiles < max_clusters ? r.num_tiles : max_clusters;
  cudaError_t err = launch_clustered(kernel, dim3(static_cast<unsigned>(clusters) * cluster),
                                     dim3(b200tx::kRnThreads), b200tx::kRnSmemBytes, cluster, stream, map_x, map_w,
                                     map_rin, r);
  if (err != cudaSuccess) return cuda_fail(err, "linear_residual_layer_norm (row-complete GEMM) launch");
  return B200TX_OK;
}

template <bool MLP, int D, typename InT, typename OutT>
cudaError_t launch_boundary_typed(const b200tx::BoundaryArgs& a, cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>((a.M + b200tx::kBoundaryRows - 1) / b200tx::kBoundaryRows));
  const dim3 block(b200tx::kBoundaryThreads);
  if constexpr (MLP)
    return launch(b200tx::mlp_residual_layernorm_kernel<D, InT, OutT>, grid, block, 0, stream, a);
  else
    return launch(b200tx::linear_residual_layernorm_kernel<D, InT, OutT>, grid, block, 0, stream, a);
}

template <bool MLP, int D>
cudaError_t launch_boundary_d(const b200tx::BoundaryArgs& a, int in_dtype, int out_dtype, cudaStream_t stream) {
  if (in_dtype == B200TX_F32)
    return out_dtype == B200TX_BF16 ? launch_boundary_typed<MLP, D, float, __nv_bfloat16>(a, stream)
                                    : launch_boundary_typed<MLP, D, float, float>(a, stream);
  return out_dtype == B200TX_BF16 ? launch_boundary_typed<MLP, D, __nv_bfloat16, __nv_bfloat16>(a, stream)
                                  : launch_boundary_typed<MLP, D, __nv_bfloat16, float>(a, stream);
}

// Shared checks and launch of the two fused boundary entry points.
template <bool MLP>
int boundary_impl(const char* name, b200tx::BoundaryArgs& a, int in_dtype, int out_dtype, int update_dtype,
                  int64_t rows, int64_t cols, int64_t inner, cudaStream_t stream) {
  if (a.x == nullptr || a.w == nullptr || a.bias == nullptr || a.residual_in == nullptr ||
      a.normed == nullptr || a.gamma == nullptr || a.beta == nullptr ||
      (MLP && (a.w2 == nullptr || a.bias2 == nullptr)))
    return fail(B200TX_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (rows <= 0 || rows > 0x7fffffffLL || inner <= 0 || inner > 0x7fffffffLL)
    return fail(B200TX_ERR_INVALID_ARGUMENT, "%s: bad shape rows=%lld inner=%lld", name, (long long)rows,
                (long long)inner);
  const bool wide = !MLP && (cols == 512 || cols == 768 || cols == 1024);
  if (cols != 32 && cols != 64 && cols != 128 && !wide)
    return fail(B200TX_ERR_UNSUPPORTED, "%s: cols (d_model) %lld (built: 32, 64, 128%s)", name, (long long)cols,
                MLP ? "" : ", 512, 768, 1024");
  if (MLP ? inner % 16 != 0 : inner % 8 != 0)
    return fail(B200TX_ERR_UNSUPPORTED, "%s: inner dimension %lld must be a multiple of %d", name,
                (long long)inner, MLP ? 16 : 8);
  if ((in_dtype != B200TX_F32 && in_dtype != B200TX_BF16) || (out_dtype != B200TX_F32 && out_dtype != B200TX_BF16) ||
      (update_dtype != B200TX_F32 && update_dtype != B200TX_BF16))
    return fail(B200TX_ERR_INVALID_ARGUMENT, "%s: dtype codes in=%d out=%d update=%d", name, in_dtype, out_dtype,
                update_dtype);
  if (!aligned16(a.x) || !aligned16(a.w) || (MLP && !aligned16(a.w2)) ||
      (reinterpret_cast<uintptr_t>(a.residual_in) & 7u) != 0 || (reinterpret_cast<uintptr_t>(a.normed) & 7u) != 0 ||
      (a.residual_out != nullptr && (reinterpret_cast<uintptr_t>(a.residual_out) & 7u) != 0))
    return fail(B200TX_ERR_INVALID_ARGUMENT, "%s: misaligned operand", name);
  DeviceState* dev = nullptr;
  int rc = current_device(&dev);
  if (rc != B200TX_OK) return rc;
  a.M = static_cast<int>(rows);
  a.K = static_cast<int>(inner);
  a.update_bf16 = update_dtype == B200TX_BF16 ? 1 : 0;
  if (a.row_valid == nullptr) a.mask_mode = 0;
  if (wide) return launch_gemm_rownorm(a, dev, in_dtype, out_dtype, rows, cols, inner, stream);
  cudaError_t err;
  switch (cols) {
    case 32: err = launch_boundary_d<MLP, 32>(a, in_dtype, out_dtype, stream); break;
    case 64: err = launch_boundary_d<MLP, 64>(a, in_dtype, out_dtype, stream); break;
    default: err = launch_boundary_d<MLP, 128>(a, in_dtype, out_dtype, stream); break;
  }
  if (err != cudaSuccess) return cuda_fail(err, name);
  return B200TX_OK;
}

}  // namespace

extern "C" {

int b200tx_linear_residual_layer_norm(const void* x, const void* w, const float* bias, int64_t inner,
                                      const void* residual_in, int in_dtype, float* residual_out,
                                      void* normed, int out_dtype, const float* gamma, const float* beta,
                                      const uint8_t* row_valid, int mask_mode, int update_dtype,
                                      int64_t rows, int64_t cols, float eps, cudaStream_t stream) {
  b200tx::BoundaryArgs a{};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.w = static_cast<const __nv_bfloat16*>(w);
  a.bias = bias;
  a.residual_in = residual_in;
  a.residual_out = residual_out;
  a.normed = normed;
  a.gamma = gamma;
  a.beta = beta;
  a.row_valid = row_valid;
  a.mask_mode = mask_mode;
  a.eps = eps;
  return boundary_impl<false>("linear_residual_layer_norm", a, in_dtype, out_dtype, update_dtype, rows, cols,
                              inner, stream);
}

int b200tx_mlp_residual_layer_norm(const void* x, const void* w1, const float* b1, const void* w2,
                                   const float* b2, int64_t ffn_dim, const void* residual_in, int in_dtype,
                                   float* residual_out, void* normed, int out_dtype, const float* gamma,
                                   const float* beta, const uint8_t* row_valid, int mask_mode,
                                   int update_dtype, int64_t rows, int64_t cols, float eps,
                                   cudaStream_t stream) {
  b200tx::BoundaryArgs a{};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.w = static_cast<const __nv_bfloat16*>(w1);
  a.bias = b1;
  a.w2 = static_cast<const __nv_bfloat16*>(w2);
  a.bias2 = b2;
  a.residual_in = residual_in;
  a.residual_out = residual_out;
  a.normed = normed;
  a.gamma = gamma;
  a.beta = beta;
  a.row_valid = row_valid;
  a.mask_mode = mask_mode;
  a.eps = eps;
  return boundary_impl<true>("mlp_residual_layer_norm", a, in_dtype, out_dtype, update_dtype, rows, cols,
                             ffn_dim, stream);
}

int b200tx_attention(const void* qkv, void* out, int64_t batch, int64_t seq, int64_t heads,
                     int64_t head_dim, float scale, int causal, cudaStream_t stream) {
  return b200tx_attention_ex(qkv, out, batch, seq, heads, head_dim, scale, causal,
                             B200TX_ATTN_QUAD, stream);
}

}  // extern "C"
