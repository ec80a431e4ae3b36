/*
 * b200tx.h -- C ABI of libb200tx, the sm_100a (B200) kernels behind the
 * Transformer forward of the `solution` package.
 *
 * The reference (Wendystar0628/ML-Guided-Program-Search-for-Shape-Specialized-
 * Transformer-Optimization) is pure Python: its hot path calls Triton kernels
 * through Python wrappers that return `(tensor, marker)`.  Each entry point
 * below replaces one of those operators; the reference file:line it stands in
 * for is cited beside it.  The Python wrappers in solution/kernels/ bind these
 * symbols with ctypes.
 *
 * Conventions
 *   - Plain device pointers, element counts and a cudaStream_t; no framework
 *     types.  Tensors are dense row-major with the shapes given per function.
 *   - Nothing here allocates device memory, synchronises the device or the
 *     stream, or launches on any stream other than the one passed in, so every
 *     call can be captured in a CUDA graph.
 *   - Return value 0 = launched.  A negative value is an error; the message is
 *     in b200tx_last_error() (thread-local).  Argument errors are detected on
 *     the host before anything is launched.
 *   - Kernels never trap.  A device-side wait that runs out (a hung pipeline)
 *     records a code that b200tx_device_error() returns.
 */
#ifndef B200TX_H_
#define B200TX_H_

#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types accepted by the dtype arguments. */
#define B200TX_F32 0
#define B200TX_BF16 1

/* Epilogues of b200tx_linear. */
#define B200TX_EPI_BIAS 0
#define B200TX_EPI_BIAS_GELU 1

/* GEMM kernel variants (b200tx_linear_ex). */
#define B200TX_GEMM_1SM 0  /* one CTA per SM, 128x256 tiles, 4-stage 48 KB ring */
#define B200TX_GEMM_PAIR 1 /* CTA pairs (cta_group::2), 256x256 tiles, 6-stage 32 KB ring */
#define B200TX_GEMM_WARP 2 /* small problems: 64x64 tiles on warp-level MMAs (mma.sync), no TMA/TMEM */

/* Attention kernel variants (b200tx_attention_ex). */
#define B200TX_ATTN_PAIRED 0 /* two 128-row query tiles per CTA, P kept in TMEM */
#define B200TX_ATTN_SINGLE 1 /* one 128-row query tile per CTA, P through shared memory */
#define B200TX_ATTN_QUAD 2   /* four 128-row query tiles per CTA, 64-row KV tiles, P in TMEM */
#define B200TX_ATTN_PERSISTENT 3 /* persistent grid, two query tiles per item, double-buffered S */
#define B200TX_ATTN_DUO 4    /* two 128-row query tiles per CTA, 64-row KV tiles, two CTAs per SM */
#define B200TX_ATTN_PINGPONG 5 /* persistent; two 128-row query tiles x 128-row KV tiles, S, P and O
                                  in separate TMEM columns so S(j+1) overlaps the softmax of S(j) */

/* Status codes. */
#define B200TX_OK 0
#define B200TX_ERR_INVALID_ARGUMENT -1
#define B200TX_ERR_UNSUPPORTED -2
#define B200TX_ERR_CUDA -3
#define B200TX_ERR_DRIVER -4

/* ABI version of this header; bumped when a signature changes. */
int b200tx_abi_version(void);

/* Message describing the last failed call on this host thread ("" if none). */
const char* b200tx_last_error(void);

/* Reads (and, if `clear` != 0, resets) the device error word of the current
 * device: 0 when healthy, else the code of the first kernel wait that ran out.
 * Synchronises the device; diagnostic use only. */
int b200tx_device_error(int clear, unsigned int* code_out);

/* Stream-ordered read of the current device's error word: copies it into
 * *word (pinned host or device memory) on `stream`, after the work queued
 * before it.  Does not clear it and does not synchronise; the caller waits on
 * the stream (or an event) before reading *word.  The word is sticky: once a
 * wait has run out, later kernels on the device stop early until
 * b200tx_device_error(clear = 1) resets it.  No reference counterpart (the
 * reference's Triton kernels have no device-side waits). */
int b200tx_device_error_async(unsigned int* word, cudaStream_t stream);

/* Multiprocessor count and compute capability of the current device; returns
 * B200TX_ERR_UNSUPPORTED unless it is a compute capability 10.0 device. */
int b200tx_device_check(int* sm_count_out, int* cc_major_out, int* cc_minor_out);

/*
 * LayerNorm of each row, optionally after a residual add:
 *     r = residual_in + update            (update may be NULL)
 *     normed = (r - mean(r)) / sqrt(var(r) + eps) * gamma + beta
 *     residual_out = r                    (if residual_out != NULL)
 * residual_in  [rows, cols] in_dtype (F32 or BF16)
 * update       [rows, cols] update_dtype (F32 or BF16), or NULL
 * residual_out [rows, cols] F32, or NULL; may equal residual_in (in place)
 * normed       [rows, cols] out_dtype (F32 or BF16)
 * gamma, beta  [cols] F32
 * Replaces: solution/kernels/norm/triton_initial.py:38-66 (initial LN, no
 * update), solution/kernels/norm/triton_residual.py:38-73 and
 * solution/kernels/norm/triton_mixed_residual.py:40-77 (residual + LN; the
 * `final_boundary` fp32 output is out_dtype = F32), and the torch path
 * residual_add + nn.LayerNorm at solution/transformer.py:1629-1632.
 */
int b200tx_residual_layer_norm(const void* residual_in, int in_dtype, const void* update,
                               int update_dtype, float* residual_out, void* normed,
                               int out_dtype, const float* gamma, const float* beta,
                               int64_t rows, int64_t cols, float eps, cudaStream_t stream);

/* mask_mode bits of b200tx_residual_layer_norm_masked, applied to rows whose
 * row_valid flag is 0 (the reference's masked_fill of padding tokens,
 * official/torch_transformer_benchmark.py:119-121, 143-144, 170-171). */
#define B200TX_MASK_DROP_UPDATE 1   /* r = residual_in: the update is ignored */
#define B200TX_MASK_ZERO_RESIDUAL 2 /* r = 0 (residual_out, and the LN input) */
#define B200TX_MASK_ZERO_NORMED 4   /* normed = 0 */

/*
 * b200tx_residual_layer_norm with a padding mask: row_valid [rows] uint8
 * (0 = padding token, non-null); mask_mode is a combination of B200TX_MASK_*
 * bits.  Replaces the masked LayerNorm path of the reference
 * (solution/kernels/norm/triton_masked.py:47-118) and the masked_fill calls
 * of official/torch_transformer_benchmark.py:119-121, 143-144, 170-171.
 */
int b200tx_residual_layer_norm_masked(const void* residual_in, int in_dtype, const void* update,
                                      int update_dtype, float* residual_out, void* normed,
                                      int out_dtype, const float* gamma, const float* beta,
                                      const uint8_t* row_valid, int mask_mode, int64_t rows,
                                      int64_t cols, float eps, cudaStream_t stream);

/*
 * out[M, N] = epilogue(a[M, K] . w[N, K]^T + bias[N]) on the tcgen05 tensor
 * cores, bf16 inputs, fp32 accumulation, output F32 or BF16.
 * a, w: BF16, row-major, K contiguous; bias: F32 [N] or NULL.
 * epilogue: B200TX_EPI_BIAS or B200TX_EPI_BIAS_GELU (exact erf GELU).
 * Requires K % 8 == 0 and N % 8 == 0 (16-byte TMA row pitch); 16-byte
 * aligned a, w and out.
 * Replaces: solution/kernels/projection/triton_qkv_layout.py:59-113 (packed
 * QKV), solution/kernels/projection/triton_attention_output.py:69-147
 * (out-proj), solution/kernels/ffn/triton_linear_exact_gelu.py:68-132 (FFN in
 * + GELU), and the fp16-shadow F.linear at solution/transformer.py:333-353.
 */
int b200tx_linear(const void* a, const void* w, const float* bias, void* out, int out_dtype,
                  int64_t M, int64_t N, int64_t K, int epilogue, cudaStream_t stream);

/*
 * b200tx_linear with an explicit kernel variant (B200TX_GEMM_PAIR, the variant
 * of b200tx_linear, B200TX_GEMM_1SM, or B200TX_GEMM_WARP for problems too small
 * to amortise the tcgen05 pipelines' set-up).  All compute the same function;
 * the execution plan's GEMM launch records pick one per projection.  Replaces the
 * same reference operators as b200tx_linear; the variant is the sm100
 * counterpart of the reference's GEMM launch parameters
 * (TritonGemmParams, solution/config.py:279-325).
 */
int b200tx_linear_ex(const void* a, const void* w, const float* bias, void* out, int out_dtype,
                     int64_t M, int64_t N, int64_t K, int epilogue, int variant,
                     cudaStream_t stream);

/*
 * Causal (or full) multi-head attention over the packed projection output.
 * qkv  [batch, seq, 3, heads, head_dim] BF16 -- the [B, S, 3D] output of the
 *      packed QKV linear (rows q;k;v of W_qkv), D = heads * head_dim
 * out  [batch, seq, heads, head_dim] BF16 -- the [B, S, D] context, ready for
 *      the out-projection
 * softmax(q k^T * scale (+ causal mask)) v with fp32 softmax statistics.
 * head_dim must be 64.
 * Replaces: solution/shape14/triton_streaming_dh64.py:68-190 (streaming
 * Dh64, BSD output), solution/kernels/attention/triton_s1024_dh32.py:72-265,
 * solution/operators/attention/sdpa.py:76-170 (SDPA / query-blocked
 * reference attention) together with split_qkv
 * (solution/operators/projection/qkv_layout.py:22-50).
 */
int b200tx_attention(const void* qkv, void* out, int64_t batch, int64_t seq, int64_t heads,
                     int64_t head_dim, float scale, int causal, cudaStream_t stream);

/*
 * b200tx_attention with an explicit kernel variant (B200TX_ATTN_QUAD, the
 * default of b200tx_attention, B200TX_ATTN_DUO, B200TX_ATTN_PERSISTENT,
 * B200TX_ATTN_PINGPONG, B200TX_ATTN_PAIRED or B200TX_ATTN_SINGLE).  All compute the same function; the execution plan's
 * attention launch record picks one.
 * Replaces the same reference operators as b200tx_attention; the variant is the
 * sm100 counterpart of the reference's attention launch parameters
 * (TritonAttentionParams, solution/config.py:189-234).
 */
int b200tx_attention_ex(const void* qkv, void* out, int64_t batch, int64_t seq, int64_t heads,
                        int64_t head_dim, float scale, int causal, int variant,
                        cudaStream_t stream);

/*
 * b200tx_attention_ex with a key padding mask: key_valid [batch, seq] uint8
 * (non-null), 0 = padding key, whose scores are -inf for every query (the
 * reference's invalid_keys masked_fill, official/torch_transformer_benchmark.py:
 * 105-108).  A query that sees no valid key gets a zero context row.  Built
 * into B200TX_ATTN_QUAD, B200TX_ATTN_DUO, B200TX_ATTN_PERSISTENT and
 * B200TX_ATTN_PINGPONG; other variants return B200TX_ERR_UNSUPPORTED.
 */
int b200tx_attention_masked(const void* qkv, const uint8_t* key_valid, void* out, int64_t batch,
                            int64_t seq, int64_t heads, int64_t head_dim, float scale, int causal,
                            int variant, cudaStream_t stream);

/*
 * Causal (or full) attention for head_dim 8, 16, 32, 64, 128 or 256 on the CUDA
 * cores, with an optional key padding mask (key_valid [batch, seq] uint8 or
 * NULL); same layouts and semantics as b200tx_attention_masked.  It covers the
 * head dims the tensor-core kernels (head_dim 64) do not, e.g. the reference's
 * official benchmark shapes (official/test_shapes.json: head dims 8, 32, 128,
 * 256).  Replaces the same reference operators as b200tx_attention
 * (solution/operators/attention/sdpa.py:76-170 for those shapes).
 */
int b200tx_attention_generic(const void* qkv, const uint8_t* key_valid, void* out, int64_t batch,
                             int64_t seq, int64_t heads, int64_t head_dim, float scale, int causal,
                             cudaStream_t stream);

/*
 * The same attention as b200tx_attention_generic for head_dim 8, 16, 32, 64 or
 * 128 on warp-level tensor-core MMAs (mma.sync m16n8k16, bf16 inputs, fp32
 * accumulation): 64 query rows per CTA, 64-key tiles, P kept in registers.
 * Same layouts, masks and semantics.  Replaces, for the reference's official
 * shapes (official/test_shapes.json: head dims 8, 32, 64, 128), its
 * small-head kernels solution/kernels/attention/triton_dh8.py:72-260 and
 * solution/kernels/attention/triton_s1024_dh32.py:72-366, and the SDPA
 * operators solution/operators/attention/sdpa.py:76-170.
 */
int b200tx_attention_mma(const void* qkv, const uint8_t* key_valid, void* out, int64_t batch,
                         int64_t seq, int64_t heads, int64_t head_dim, float scale, int causal,
                         cudaStream_t stream);

/*
 * The projection that closes a block branch fused with the residual add and
 * LayerNorm after it, for d_model (cols) 32, 64 or 128 (CTAs of 16 rows whose
 * four warps split the columns; warp-level tensor-core MMAs) and 512, 768 or
 * 1024 (tcgen05 CTA pairs in clusters of 2 * cols / 256 CTAs holding 256 whole
 * rows; residual_in, residual_out and normed 16-byte aligned there):
 *     u = x[rows, inner] . w[cols, inner]^T + bias[cols]   (rounded to update_dtype)
 *     r = residual_in + u;  normed = LayerNorm(r) * gamma + beta
 * x, w BF16 row-major; bias, gamma, beta F32; residual_in in_dtype (F32 or
 * BF16); residual_out F32 or NULL (not kept); normed out_dtype; inner a
 * multiple of 8.  row_valid (uint8 [rows] or NULL) and mask_mode as in
 * b200tx_residual_layer_norm_masked.  The update is rounded to update_dtype
 * (BF16 or F32) before the add, as the unfused program stores it.
 * Replaces the reference's fused Linear residual-norm boundary
 * solution/kernels/boundary/triton_linear_residual_norm.py:33-112 (D 32 and
 * 128) for the out-projection and the FFN-out projection.
 */
int b200tx_linear_residual_layer_norm(const void* x, const void* w, const float* bias, int64_t inner,
                                      const void* residual_in, int in_dtype, float* residual_out,
                                      void* normed, int out_dtype, const float* gamma, const float* beta,
                                      const uint8_t* row_valid, int mask_mode, int update_dtype,
                                      int64_t rows, int64_t cols, float eps, cudaStream_t stream);

/*
 * The whole MLP fused through the same boundary, d_model 32, 64 or 128:
 *     h = bf16(GELU_erf(x[rows, cols] . w1[ffn_dim, cols]^T + b1))   (never stored)
 *     u = h . w2[cols, ffn_dim]^T + b2                              (rounded to update_dtype)
 *     r = residual_in + u;  normed = LayerNorm(r) * gamma + beta
 * ffn_dim a multiple of 16; the other arguments as in
 * b200tx_linear_residual_layer_norm.  Replaces the reference's fused MLP
 * boundary solution/kernels/boundary/triton_ffn_residual_norm.py:43-136
 * (D = F = 128).
 */
int b200tx_mlp_residual_layer_norm(const void* x, const void* w1, const float* b1, const void* w2,
                                   const float* b2, int64_t ffn_dim, const void* residual_in, int in_dtype,
                                   float* residual_out, void* normed, int out_dtype, const float* gamma,
                                   const float* beta, const uint8_t* row_valid, int mask_mode,
                                   int update_dtype, int64_t rows, int64_t cols, float eps,
                                   cudaStream_t stream);

/* ------------------------------------------------------------------------
 * The whole forward of a small model in one launch (d_model = ffn_dim = 128,
 * 1, 2 or 4 heads, sequences of 32, 64 or 128 tokens, 1-8 layers): one CTA per
 * 128 rows (whole sequences) runs every layer on chip -- tcgen05 UMMAs with the
 * residual and the accumulators in TMEM, weights streamed by bulk copies from
 * pre-swizzled images.  Replaces, for the reference's small official shapes
 * (official/test_shapes.json), the per-primitive forward of
 * solution/transformer.py:1346-1513; no padding mask.
 * ------------------------------------------------------------------------ */

/* One [128, 128] BF16 row-major weight (a Linear's [out, in]) into its 32 KB
 * operand image (16-byte aligned).  A layer's images are six consecutive
 * images: Wq, Wk, Wv (the rows of the packed QKV weight), Wo, W1, W2. */
int b200tx_seq_weight_image(const void* weight, void* image, cudaStream_t stream);

typedef struct b200tx_seq_layer {
  const void* weight_images;  /* 6 x 32 KB images (b200tx_seq_weight_image) */
  const float* b_qkv;         /* [384] q, k, v biases */
  const float* b_o;           /* [128] */
  const float* b_1;           /* [128] */
  const float* b_2;           /* [128] */
  const float* ln2_gamma;     /* norm2 of this layer */
  const float* ln2_beta;
  const float* next_gamma;    /* norm1 of the next layer, or the final norm */
  const float* next_beta;
} b200tx_seq_layer;

/* out = forward(x), x and out F32 [batch, seq, 128]; ln0 = norm1 of layer 0.
 * Every pointer 16-byte aligned; causal attention; the unfused program's
 * rounding points (bf16 projections, probabilities and updates). */
int b200tx_sequence_forward(const float* x, float* out, int64_t batch, int64_t seq, int64_t d_model,
                            int64_t heads, int64_t ffn_dim, int num_layers, const b200tx_seq_layer* layers,
                            const float* ln0_gamma, const float* ln0_beta, float eps, cudaStream_t stream);

/* ------------------------------------------------------------------------
 * The same whole forward for callers that cannot allocate device memory.
 * No counterpart in the reference.  b200tx_sequence_forward needs 192 KB of
 * weight images per layer that the caller allocates and fills; some callers
 * cannot: a process whose device memory is all handed out by its framework's
 * own pool (a serving engine that reserves the GPU at start-up), or code that
 * must not call cudaMalloc because it synchronizes the device.  This entry
 * point takes the plain weights instead and builds the images, on the
 * stream, in a fixed array that the library holds in device memory for up to
 * B200TX_SEQ_NOALLOC_MAX_LAYERS layers (768 KB on every GPU that loads the
 * library, until the process exits); more layers are rejected with
 * B200TX_ERR_UNSUPPORTED.  It allocates nothing.
 * - The first call on a device looks up the array's device address
 *   (cudaGetSymbolAddress) with that device current; make that first call
 *   before any stream capture.
 * - Every call on a device shares the one array and rewrites the images of
 *   the layers it runs before its forward reads them, so nothing in it needs
 *   clearing.  Calls whose work overlaps on the GPU (different streams, or
 *   host threads) race on it: serialize them.
 * - Same shapes, results and pointer rules as b200tx_sequence_forward, with
 *   each weight a BF16 row-major [out, in] matrix, 16-byte aligned.
 * ------------------------------------------------------------------------ */
#define B200TX_SEQ_NOALLOC_MAX_LAYERS 4

typedef struct b200tx_seq_layer_weights {
  const void* w_qkv;          /* [384, 128] BF16: the q, k and v weights stacked by rows */
  const void* w_o;            /* [128, 128] BF16 out-projection */
  const void* w_1;            /* [128, 128] BF16 FFN in */
  const void* w_2;            /* [128, 128] BF16 FFN out */
  const float* b_qkv;         /* [384] q, k, v biases */
  const float* b_o;           /* [128] */
  const float* b_1;           /* [128] */
  const float* b_2;           /* [128] */
  const float* ln2_gamma;     /* norm2 of this layer */
  const float* ln2_beta;
  const float* next_gamma;    /* norm1 of the next layer, or the final norm */
  const float* next_beta;
} b200tx_seq_layer_weights;

int b200tx_sequence_forward_noalloc(const float* x, float* out, int64_t batch, int64_t seq, int64_t d_model,
                                    int64_t heads, int64_t ffn_dim, int num_layers,
                                    const b200tx_seq_layer_weights* layers, const float* ln0_gamma,
                                    const float* ln0_beta, float eps, cudaStream_t stream);

/* ------------------------------------------------------------------------
 * Tensor-parallel reduction over NVLink peer memory.  The reference is
 * single-GPU; these entry points implement the head-sharded runtime's
 * reduction after the row-parallel projections (out-proj and FFN-out) without
 * a separate all-reduce: each rank's GEMM writes its partial into a buffer the
 * peers opened through CUDA IPC, b200tx_peer_signal publishes an epoch into
 * each peer's flag array, and b200tx_residual_layer_norm_peer sums every
 * rank's partial into the residual and normalises in one pass.
 * ------------------------------------------------------------------------ */
#define B200TX_IPC_HANDLE_BYTES 64

/* Set-up only (these allocate and map memory): a zero-filled device buffer of
 * `bytes` and its IPC handle (B200TX_IPC_HANDLE_BYTES) for the peers; opening a
 * peer's handle in this process; closing / freeing. */
int b200tx_peer_alloc(size_t bytes, void** device_ptr_out, void* ipc_handle_out);
int b200tx_peer_open(const void* ipc_handle, void** device_ptr_out);
int b200tx_peer_close(void* device_ptr);
int b200tx_peer_free(void* device_ptr);

/* After this rank's partial is complete on `stream`: store `epoch` (release,
 * system scope) into peer_slots[i], this rank's slot in each peer's flag array
 * (count <= 8; a NULL slot is skipped). */
int b200tx_peer_signal(uint32_t* const* peer_slots, int count, uint32_t epoch, cudaStream_t stream);

/*
 * b200tx_residual_layer_norm_masked with update = the sum of `count` bf16
 * partials [rows, cols] (partials[self] local, the others peers' buffers):
 * waits (bounded, system-scope acquire) until flags[r] >= epoch for every peer
 * r, then r = residual_in + sum_r partials[r], normalised.  residual_in F32;
 * cols a multiple of 128 up to 2048; row_valid may be NULL.  A wait that runs
 * out records its code in b200tx_device_error and writes nothing.
 */
int b200tx_residual_layer_norm_peer(const float* residual_in, const void* const* partials, int count,
                                    int self, const uint32_t* flags, uint32_t epoch,
                                    float* residual_out, void* normed, int out_dtype,
                                    const float* gamma, const float* beta, const uint8_t* row_valid,
                                    int mask_mode, int64_t rows, int64_t cols, float eps,
                                    cudaStream_t stream);

/*
 * Reduce-scatter + all-gather form of b200tx_residual_layer_norm_peer for
 * groups of three or more ranks (count 2..8): after the same epoch wait, this
 * rank sums the partials only for its rows [row_begin, row_begin + row_count)
 * of the [rows, cols] tensors, writes residual_out for those rows (may be NULL)
 * and the normalised rows into outs[r] for every rank r (outs[self] local, the
 * others peers' buffers, out_dtype F32 or BF16).  When every CTA is done (a
 * count on *counter, which starts at counter_base and ends at *counter_after,
 * returned), epoch is published into done_slots[r], this rank's slot in each
 * peer's done flags (done_slots[self] unused).  No padding-row mask.  No
 * reference counterpart (the reference runs on one GPU); it serves the
 * head-sharded runtime as b200tx_residual_layer_norm_peer does.
 */
int b200tx_residual_layer_norm_peer_rs(const float* residual_in, const void* const* partials, int count,
                                       int self, const uint32_t* flags, uint32_t epoch, int64_t row_begin,
                                       int64_t row_count, float* residual_out, void* const* outs,
                                       int out_dtype, const float* gamma, const float* beta,
                                       uint32_t* const* done_slots, uint32_t* counter, uint32_t counter_base,
                                       uint32_t* counter_after, int64_t rows, int64_t cols, float eps,
                                       cudaStream_t stream);

/* Holds the stream (one thread, bounded system-scope acquire spin) until
 * flags[r] >= epoch for every r != self; a wait that runs out records its code
 * in b200tx_device_error. */
int b200tx_peer_wait(const uint32_t* flags, int count, int self, uint32_t epoch, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* B200TX_H_ */
