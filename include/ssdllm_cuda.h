/*
 * ssdllm_cuda.h — C ABI of the B200 (sm_100a) compute backend for ssd-llm.
 *
 * This is the drop-in boundary for ssd-llm's compute backend (`src/metal`): the
 * operator surface that `src/inference` calls on `MetalCompute` / `MetalGpu`.
 * Every entry point below names the reference interface it replaces
 * (path:line inside quantumnic/ssd-llm). The Rust side binds these with an
 * `extern "C"` block and keeps the `MetalCompute` method signatures.
 *
 * Conventions
 *  - Every call returns an int status: SSD_OK (0) or one of SSD_ERR_*. No call
 *    returns silent zeros for an unsupported type (the reference does,
 *    src/metal/compute.rs:672-675); it returns SSD_ERR_TYPE instead.
 *    ssd_last_error() gives a message for the calling thread's last failure.
 *  - Pointers named *_dev are device pointers; `stream` is a cudaStream_t
 *    (NULL = CUDA's default stream, as in every CUDA API; the context's own stream
 *    is available from ssd_ctx_stream). Device-pointer calls are stream-ordered
 *    and asynchronous; they allocate nothing on the hot path.
 *  - Calls named *_host take host slices, copy in, compute, copy out and
 *    synchronise: they keep the reference's synchronous semantics
 *    (src/metal/gpu.rs:531-532).
 *  - Weights are uploaded once (ssd_weight_upload) in the reference's GGUF block
 *    layout and stay HBM-resident in a library-owned layout until freed.
 *  - Quantized block layouts are the reference's own (not llama.cpp's): Q4_0
 *    element 2j is the low nibble of byte j, 2j+1 the high nibble
 *    (src/metal/compute.rs:693-699); Q4_K as src/metal/compute.rs:718-744.
 */
#ifndef SSDLLM_CUDA_H
#define SSDLLM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SSD_ABI_VERSION 1

/* status codes */
#define SSD_OK 0
#define SSD_ERR_ARG 1     /* null pointer, bad size */
#define SSD_ERR_TYPE 2    /* unsupported GgmlType */
#define SSD_ERR_SHAPE 3   /* dimensions inconsistent with the type's block size */
#define SSD_ERR_CUDA 4    /* a CUDA runtime call failed */
#define SSD_ERR_TIMEOUT 5 /* a bounded device-side wait gave up */
#define SSD_ERR_NCCL 6    /* an NCCL call failed */
#define SSD_ERR_NOMEM 7   /* device allocation failed */
#define SSD_ERR_STATE 8   /* call out of order (e.g. engine not built) */

/* GgmlType ids, src/model/gguf.rs:16-47 */
#define SSD_TYPE_F32 0
#define SSD_TYPE_F16 1
#define SSD_TYPE_Q4_0 2
#define SSD_TYPE_Q8_0 8
#define SSD_TYPE_Q4_K 12
/* Q5_K in the reference's block layout (matvec_q5_k_cpu, src/metal/compute.rs:845-899):
 * 256 weights in 176 bytes, f16 d, f16 dmin, 12 bytes of 6-bit (scale, min) as Q4_K, 32 B
 * of high bits, 128 B of low nibbles; weight = d * sc * (low4 | hbit << 4) - dmin * m. */
#define SSD_TYPE_Q5_K 13
/* Q6_K in the reference's own block layout (matvec_q6_k_cpu, src/metal/compute.rs:752-790):
 * 256 weights in 210 bytes, ql[128] low nibbles, qh[64] 2-bit high parts, 16 int8 scales,
 * f16 d; weight = (d * scale) * ((high2 << 4 | low4) - 32). Q5_K, Q6_K and Q8_K are accepted by
 * ssd_weight_upload, ssd_dequantize, the matvec entry points and the prefill matmul. */
#define SSD_TYPE_Q6_K 14
/* Q8_K in the reference's block layout (matvec_q8_k_cpu, src/metal/compute.rs:971-993):
 * 256 weights in 292 bytes, f32 d, 256 int8, 32 bytes of block sums (not read by the
 * matvec, kept for the download); weight = d * q. */
#define SSD_TYPE_Q8_K 15
/* 16-bit dense weights, row-major, 2 bytes each: F16 (IEEE half, matvec_f16_cpu,
 * src/metal/compute.rs:2272-2285) and BF16 (the top half of an f32, matvec_bf16_cpu,
 * :2250-2269). Accepted by ssd_weight_upload, ssd_dequantize and the plain matvec entry
 * points (any column count). F32 weights (row-major, 4 bytes each; matvec_f32_simd,
 * :378-424) are accepted by the same calls. ssd_fused_swiglu takes dense gate / up weights
 * with norm_w NULL (no fused norm). */
#define SSD_TYPE_BF16 30
/* Low-bit formats in the reference's own block layouts (matvec_*_cpu, src/metal/compute.rs:
 * 793-1075, 1964-2240), kept as uploaded: Q2_K (256 weights in 84 B), Q3_K (110 B), IQ2_XXS
 * (66 B), IQ2_XS (74 B), IQ3_XXS (98 B), IQ4_NL (32 weights in 18 B), IQ3_S (110 B), IQ4_XS
 * (148 B). Accepted by ssd_weight_upload / _download, ssd_dequantize (the reference's element
 * values, bit-exact), ssd_matvec, ssd_matvec_residual and ssd_matvec_quantized_host (columns a
 * multiple of the block, x 16-byte aligned). */
#define SSD_TYPE_Q2_K 10
#define SSD_TYPE_Q3_K 11
#define SSD_TYPE_IQ2_XXS 16
#define SSD_TYPE_IQ2_XS 17
#define SSD_TYPE_IQ3_XXS 18
#define SSD_TYPE_IQ4_NL 20
#define SSD_TYPE_IQ3_S 21
#define SSD_TYPE_IQ4_XS 23

typedef struct ssd_ctx ssd_ctx;
typedef struct ssd_weight ssd_weight;
typedef struct ssd_kv_cache ssd_kv_cache;
typedef struct ssd_model ssd_model;

/* ---------------------------------------------------------------- basics */
int ssd_abi_version(void);
const char* ssd_status_str(int status);
/* Message of the calling thread's last failed call ("" if none). */
const char* ssd_last_error(void);

/* Context: one per device, owns a stream.
 * Replaces MetalCompute::new (src/metal/compute.rs:47-72) and MetalGpu::new
 * (src/metal/gpu.rs:73-160), which the reference constructs per forward pass
 * and per token (src/inference/transformer.rs:301-302, :704). ssd_ctx_get()
 * returns a process-wide cached context for the device, so per-token
 * construction costs nothing; ssd_ctx_create() makes a private one. */
int ssd_ctx_create(int device, ssd_ctx** out);
int ssd_ctx_get(int device, ssd_ctx** out);
int ssd_ctx_destroy(ssd_ctx* ctx);
int ssd_ctx_stream(ssd_ctx* ctx, void** stream_out);
int ssd_ctx_sync(ssd_ctx* ctx);
/* Reads and clears the device status word: SSD_ERR_TIMEOUT if a kernel's bounded
 * wait (TMA barrier, peer flag) gave up since the last call, else SSD_OK. Synchronises
 * the device. No reference counterpart (Metal calls block until completion,
 * src/metal/gpu.rs:531-532). */
int ssd_ctx_device_status(ssd_ctx* ctx, int* status);
/* Launch the context's standalone kernels (ssd_matvec and the fused matvecs) with
 * programmatic dependent launch, so a kernel's weight prefetch overlaps the tail
 * of the kernel before it on the same stream (default off). The decode engine
 * always uses it. No reference counterpart (Metal commits each dispatch and waits,
 * src/metal/gpu.rs:531-532). */
int ssd_ctx_set_pdl(ssd_ctx* ctx, int on);
/* Number of SMs and device name. No reference counterpart (reports only). */
int ssd_ctx_info(ssd_ctx* ctx, int* num_sms, char* name, size_t name_len);
/* Synchronous copies between host memory and device memory of the context. The
 * reference copies every operand per call (src/metal/gpu.rs:499-505, :1253); here
 * callers copy explicitly, once. */
int ssd_copy_to_device(ssd_ctx* ctx, void* dst_dev, const void* src_host, size_t bytes);
int ssd_copy_to_host(ssd_ctx* ctx, void* dst_host, const void* src_dev, size_t bytes);

/* --------------------------------------------------------------- weights */
/* Upload a [rows x cols] tensor given in the reference block layout.
 * Replaces the per-call weight copies of MetalGpu (src/metal/gpu.rs:499-505,
 * :770-785): the weight is uploaded once and stays HBM-resident.
 * Supported: Q4_0, Q8_0, Q4_K, F32. cols must be a multiple of the block size. */
int ssd_weight_upload(ssd_ctx* ctx, const void* host_raw, size_t bytes, int ggml_type, int rows,
                      int cols, ssd_weight** out);
/* Same as ssd_weight_upload (src/metal/gpu.rs:499-505), from a device buffer in the
 * reference block layout (stream-ordered). */
int ssd_weight_upload_device(ssd_ctx* ctx, const void* raw_dev, size_t bytes, int ggml_type,
                             int rows, int cols, ssd_weight** out, void* stream);
/* Copy the weight back in the reference block layout (host buffer of raw_bytes), free
 * it, query it. No reference counterpart (the reference never keeps device weights). */
int ssd_weight_download(ssd_ctx* ctx, const ssd_weight* w, void* host_raw, size_t bytes);
int ssd_weight_free(ssd_weight* w);
int ssd_weight_info(const ssd_weight* w, int* ggml_type, int* rows, int* cols,
                    size_t* raw_bytes);
/* Bytes of one row of `cols` elements in the reference layout (0 if unsupported). */
size_t ssd_row_bytes(int ggml_type, int64_t cols);

/* Synthetic weights for benchmarks: element (r, c) of a [total_rows x total_cols]
 * matrix is N(0, std^2) drawn from a counter-based hash of (seed, tensor_id, r, c)
 * and quantized per block with ssd_quantize's rules. The [row0, row0+rows) x
 * [col0, col0+cols) window is materialised, so tensor-parallel shards are exact
 * slices of the same global matrix. No reference counterpart (test inputs). */
int ssd_weight_synth(ssd_ctx* ctx, int ggml_type, uint64_t seed, uint32_t tensor_id,
                     float std_dev, int64_t total_cols, int row0, int rows, int col0, int cols,
                     ssd_weight** out, void* stream);
/* f32 N(mean, std^2) values of the same generator, row-major window.
 * No reference counterpart (test and benchmark inputs). */
int ssd_synth_f32(ssd_ctx* ctx, uint64_t seed, uint32_t tensor_id, float mean, float std_dev,
                  int64_t total_cols, int row0, int rows, int col0, int cols, float* out_dev,
                  void* stream);

/* -------------------------------------------------- quantize / dequantize */
/* f32 rows -> reference block layout (device). No reference counterpart: the
 * reference ships no quantizer for these formats; this is the inverse of its
 * decoders src/metal/compute.rs:680-750, :904-925 (builder's rule:
 * Q4_0 d = m/-8 with m the signed value of largest magnitude; Q8_0 d = amax/127;
 * Q4_K 6-bit scales/mins over 32-wide sub-blocks). */
int ssd_quantize(ssd_ctx* ctx, const float* x_dev, int rows, int cols, int ggml_type,
                 void* raw_out_dev, void* stream);
/* Packed -> f32 [rows x cols], bit-exact with dequantize_to_f32
 * (src/ssd/streamer.rs:93-180) and the Q4_K element formula of
 * matvec_q4_k_cpu (src/metal/compute.rs:718-744). */
int ssd_dequantize(ssd_ctx* ctx, const ssd_weight* w, float* out_dev, void* stream);

/* ------------------------------------------------------- batch prefill */
/* y[t] = W x[t] for n_tokens prompt tokens at once (x [n_tokens][cols], y
 * [n_tokens][rows], row-major device arrays): the per-token matvec_quantized calls of the
 * layer-major batch_prefill_lora loop (src/inference/transformer.rs:120-250) as one
 * tensor-core GEMM (tcgen05, fp16 hi/lo operand splits, three passes, fp32 accumulation in
 * TMEM). n_tokens and rows multiples of 128, cols a multiple of 64. Uses the context's
 * scratch buffer (4 bytes per weight + 4 per activation). */
int ssd_prefill_matmul(ssd_ctx* ctx, const ssd_weight* w, const float* x_dev, int n_tokens,
                       float* y_dev, void* stream);

/* ------------------------------------------------------------- matvecs */
/* y = W x. Replaces MetalCompute::matvec_quantized (src/metal/compute.rs:157-191)
 * and the matvec_q4_0 / matvec_q8_0 / matvec_q4_k Metal kernels
 * (src/metal/shaders/kernels.metal:166-273, :575-604). */
int ssd_matvec(ssd_ctx* ctx, const ssd_weight* w, const float* x_dev, float* y_dev, void* stream);
/* ssd_matvec for a series of matvecs that do not feed each other (the reference calls
 * matvec_quantized, src/metal/compute.rs:157-191, once per matrix, each on inputs already in
 * memory): the caller guarantees that no kernel enqueued before this call on the stream writes
 * x_dev or touches y_dev. The kernel then streams its weights and x without waiting for its
 * predecessor, so consecutive launches overlap; it waits for the predecessor at its end, so
 * later kernels see everything before it completed. Results are identical to ssd_matvec. */
int ssd_matvec_independent(ssd_ctx* ctx, const ssd_weight* w, const float* x_dev, float* y_dev,
                           void* stream);
/* y = base + W x (base may alias y): matvec plus the residual add of
 * src/inference/transformer.rs:369-371. */
int ssd_matvec_residual(ssd_ctx* ctx, const ssd_weight* w, const float* x_dev,
                        const float* base_dev, float* y_dev, void* stream);
/* logits = W rmsnorm(x, norm_w): MetalCompute::fused_rmsnorm_linear_f32
 * (src/metal/compute.rs:348-372, CPU :557-577) with a quantized W. eps as given
 * (the reference hard-codes 1e-5). */
int ssd_fused_rmsnorm_matvec(ssd_ctx* ctx, const ssd_weight* w, const float* x_dev,
                             const float* norm_w_dev, float eps, float* y_dev, void* stream);
/* Q,K,V = (Wq,Wk,Wv) rmsnorm(x) with RoPE on Q and K at `position`:
 * MetalCompute::fused_qkv_rope_f32 (src/metal/compute.rs:296-326, CPU :509-529)
 * with the attention pre-norm of transformer.rs:323-326 folded in when
 * norm_w_dev is non-NULL. */
int ssd_fused_qkv_rope(ssd_ctx* ctx, const ssd_weight* wq, const ssd_weight* wk,
                       const ssd_weight* wv, const float* x_dev, const float* norm_w_dev,
                       float eps, int head_dim, int position, float theta, float* q_dev,
                       float* k_dev, float* v_dev, void* stream);
/* act = silu(Wg n) * (Wu n), n = rmsnorm(x, norm_w) (or x when norm_w is NULL):
 * the fused SwiGLU of MetalGpu::feed_forward_f32 (src/metal/gpu.rs:789-841,
 * src/inference/feed_forward.rs:17-44). */
int ssd_fused_swiglu(ssd_ctx* ctx, const ssd_weight* w_gate, const ssd_weight* w_up,
                     const float* x_dev, const float* norm_w_dev, float eps, float* act_dev,
                     void* stream);

/* ------------------------------------------------------ elementwise ops */
/* In-place RMSNorm: MetalCompute::rmsnorm_f32 (src/metal/compute.rs:193-202, :580-588). */
int ssd_rmsnorm(ssd_ctx* ctx, float* x_dev, const float* w_dev, int n, float eps, void* stream);
/* hidden += attn; out = rmsnorm(hidden, w): MetalCompute::fused_post_attn_norm_f32
 * (src/metal/compute.rs:328-346, :536-555). */
int ssd_fused_post_attn_norm(ssd_ctx* ctx, float* hidden_dev, const float* attn_dev,
                             const float* w_dev, int n, float eps, float* out_dev, void* stream);
/* In-place softmax: MetalCompute::softmax_f32 (src/metal/compute.rs:204-213, :604-620). */
int ssd_softmax(ssd_ctx* ctx, float* x_dev, int n, void* stream);
/* In-place multi-head RoPE (src/metal/compute.rs:482-506). */
int ssd_rope(ssd_ctx* ctx, float* x_dev, int len, int head_dim, int n_heads, int position,
             float theta, void* stream);
/* In-place SiLU (src/metal/compute.rs:641-645). */
int ssd_silu(ssd_ctx* ctx, float* x_dev, int n, void* stream);
/* Greedy argmax, LAST index on ties (src/inference/sampler.rs:572-578). */
int ssd_argmax(ssd_ctx* ctx, const float* v_dev, int n, int32_t* idx_dev, void* stream);

/* ------------------------------------------------------ INT8 KV + attention */
/* Device INT8 KV cache for one layer: K and V [capacity][kv_dim] int8 plus one
 * f32 scale per (position, K or V) spanning all KV heads, as
 * QuantizedLayerKvCache (src/inference/quantized_kv_cache.rs:88-130). */
int ssd_kv_create(ssd_ctx* ctx, int capacity, int n_head_kv, int head_dim, ssd_kv_cache** out);
int ssd_kv_free(ssd_kv_cache* kv);
/* Device pointers of the cache arrays (QuantizedLayerKvCache's keys/values/scales,
 * src/inference/quantized_kv_cache.rs:88-95), for tests and direct filling. */
int ssd_kv_pointers(ssd_kv_cache* kv, int8_t** k_dev, int8_t** v_dev, float** k_scale_dev,
                    float** v_scale_dev);
/* Quantize k, v [kv_dim] into row `position`: QuantizedLayerKvCache::append
 * (src/inference/quantized_kv_cache.rs:107-110) with QuantizedVec::quantize (:23-41),
 * bit-exact. */
int ssd_kv_append(ssd_ctx* ctx, ssd_kv_cache* kv, const float* k_dev, const float* v_dev,
                  int position, void* stream);
/* ssd_kv_append for `rows` consecutive positions from [rows][kv_dim] f32 (cache
 * filling; src/inference/quantized_kv_cache.rs:107-110 per row). */
int ssd_kv_append_rows(ssd_ctx* ctx, ssd_kv_cache* kv, const float* k_dev, const float* v_dev,
                       int position, int rows, void* stream);
/* Decode attention of q [n_head*head_dim] over cache positions [0, seq_len):
 * MetalCompute::flash_attention_f32 (src/metal/compute.rs:217-258) over the INT8
 * cache, with the math of flash_attention_cached
 * (src/inference/flash_attention.rs:68-135): split-K online softmax, GQA
 * kv_h = h / (n_head / n_head_kv). out [n_head*head_dim]. */
int ssd_attention_int8(ssd_ctx* ctx, const ssd_kv_cache* kv, const float* q_dev, int n_head,
                       int seq_len, float* out_dev, void* stream);

/* ssd_attention_int8 for callers that cannot allocate device memory (code running
 * beside a CUDA graph capture, hosts whose framework owns the device allocator, loops
 * that must never block in cudaMalloc/cudaFree). No reference counterpart.
 * Same arguments and results as ssd_attention_int8, but the split-K partials live in
 * a fixed 4 MiB device array inside the library (held on every GPU that loads the
 * library until the process exits) instead of the context's scratch buffer; this
 * call allocates nothing. Limit: n_head * ceil(seq_len / 128) * (head_dim + 2) must
 * be at most 1,048,576 floats (e.g. 64 heads x 16,128 positions at head_dim 128);
 * larger calls return SSD_ERR_SHAPE. The first call on a device looks up the array's
 * device address and loads every attention kernel this call may launch (each head_dim
 * and GQA group), so make that first call, of any shape, before any stream capture;
 * later calls of every shape only launch. All calls share
 * the one array: calls whose kernels overlap on the GPU (different streams, or
 * different threads without ordering) race and must be serialised by the caller. */
int ssd_attention_int8_noalloc(ssd_ctx* ctx, const ssd_kv_cache* kv, const float* q_dev,
                               int n_head, int seq_len, float* out_dev, void* stream);

/* Causal attention of a prompt batch: n_q queries (rows of q_dev, q_stride floats apart,
 * n_head x head_dim each, RoPE applied) at positions pos0 .. pos0 + n_q - 1, each over
 * the cache positions 0 .. its own (already appended). Replaces the per-token attention
 * of batch_prefill_lora (src/inference/transformer.rs:120-250, attention.rs:172-240)
 * with one call; runs on the tcgen05 tensor cores when head_dim is 128 and n_q a
 * multiple of 128. */
int ssd_attention_prefill(ssd_ctx* ctx, const ssd_kv_cache* kv, const float* q_dev, int n_q,
                          int q_stride, int pos0, int n_head, float* out_dev, int out_stride,
                          void* stream);

/* ------------------------------------------------- host-slice operators */
/* The consumer side of the tensor-parallel peer all-reduce as an operator:
 * y = W (x + sum over r < n_ranks of partials[r * cols ..]), the partials added in rank
 * order once every rank's flag (flags[r], device memory) reaches *epoch + call + 1. Each
 * wait is bounded (well under a second): a flag that is never raised leaves y undefined and
 * SSD_ERR_TIMEOUT for ssd_ctx_device_status, and later peer waits of the context return at
 * once until that status is read. No reference counterpart (the reference's thread row
 * split has no reduction, src/inference/tensor_parallel.rs:33-105). */
int ssd_matvec_peer_input(ssd_ctx* ctx, const ssd_weight* w, const float* x_dev,
                          const float* partials_dev, int n_ranks,
                          const unsigned long long* flags_dev,
                          const unsigned long long* epoch_dev, int call, float* y_dev,
                          void* stream);
/* MetalCompute::matvec_quantized (src/metal/compute.rs:157-191) with its exact
 * signature semantics: raw weight bytes, x and y on the host; uploads, computes,
 * downloads and synchronises. */
int ssd_matvec_quantized_host(ssd_ctx* ctx, const uint8_t* w_raw, size_t w_bytes,
                              const float* x, float* y, int out_dim, int in_dim, int ggml_type);

/* ------------------------------------------------ host-slice f32 operators */
/* The remaining MetalCompute methods (src/metal/compute.rs:145-375) with their slice
 * semantics: row-major f32 weights [out][in] and vectors on the host; each call copies its
 * operands to the device, computes on the context's stream, copies the results back and
 * synchronises (src/metal/gpu.rs:169-205 uploads its weights per call the same way).
 * Outputs are caller-provided arrays of the sizes the reference returns. */
/* MetalCompute::matvec_f32 (src/metal/compute.rs:145-153): y[out_dim] = W x. */
int ssd_matvec_f32_host(ssd_ctx* ctx, const float* w, const float* x, float* y, int out_dim,
                        int in_dim);
/* MetalCompute::rmsnorm_f32 (src/metal/compute.rs:193-202), x updated in place. */
int ssd_rmsnorm_f32_host(ssd_ctx* ctx, float* x, const float* weight, int n, float eps);
/* MetalCompute::softmax_f32 (src/metal/compute.rs:204-215), x updated in place; n == 0 is a
 * no-op. */
int ssd_softmax_f32_host(ssd_ctx* ctx, float* x, int n);
/* MetalCompute::flash_attention_f32 (src/metal/compute.rs:217-259; the shader
 * src/metal/shaders/kernels.metal:1360-1440): q [n_head][head_dim], k and v
 * [seq_len][n_head_kv * head_dim]; each head attends to positions
 * [window_start, min(window_end, seq_len)) with GQA group n_head / n_head_kv; a head whose
 * window is empty gets zeros; head_dim <= 256. Only the window's K / V rows are copied.
 * Where the reference returns None (seq_len < 4 without a GPU) this call still computes. */
int ssd_flash_attention_f32_host(ssd_ctx* ctx, const float* q, const float* k, const float* v,
                                 int n_head, int n_head_kv, int head_dim, int seq_len,
                                 int window_start, int window_end, float* out);
/* The same attention on device pointers (the kernel behind the host call, for callers that
 * keep an f32 cache resident; src/inference/flash_attention.rs:146-229 is its CPU twin).
 * Uses the context scratch for split partials when the window is long. */
int ssd_flash_attention_f32(ssd_ctx* ctx, const float* q_dev, const float* k_dev,
                            const float* v_dev, int n_head, int n_head_kv, int head_dim,
                            int seq_len, int window_start, int window_end, float* out_dev,
                            void* stream);
/* MetalCompute::fused_qkv_f32 (src/metal/compute.rs:273-292): q[q_dim], k[kv_dim],
 * v[kv_dim] from one x[n_embd]. */
int ssd_fused_qkv_f32_host(ssd_ctx* ctx, const float* wq, const float* wk, const float* wv,
                           const float* x, int q_dim, int kv_dim, int n_embd, float* q, float* k,
                           float* v);
/* MetalCompute::fused_qkv_rope_f32 (src/metal/compute.rs:296-323): as fused_qkv_f32, then
 * RoPE at `position` on Q and K (rope_f32_multi_head, :482-506). */
int ssd_fused_qkv_rope_f32_host(ssd_ctx* ctx, const float* wq, const float* wk, const float* wv,
                                const float* x, int q_dim, int kv_dim, int n_embd, int head_dim,
                                int position, float theta, float* q, float* k, float* v);
/* MetalCompute::fused_post_attn_norm_f32 (src/metal/compute.rs:328-343): hidden += attn in
 * place, out = rmsnorm(hidden) * norm_w. */
int ssd_fused_post_attn_norm_f32_host(ssd_ctx* ctx, float* hidden, const float* attn,
                                      const float* norm_w, int n, float eps, float* out);
/* MetalCompute::fused_rmsnorm_linear_f32 (src/metal/compute.rs:348-374):
 * logits[vocab] = W_out (x * inv_rms * norm_w), eps 1e-5 as the reference fixes it. */
int ssd_fused_rmsnorm_linear_f32_host(ssd_ctx* ctx, const float* x, const float* norm_w,
                                      const float* out_w, int vocab, int n_embd, float* logits);
/* MetalGpu::feed_forward_f32 (src/metal/gpu.rs:789-838; src/inference/feed_forward.rs:17-43):
 * out[n_embd] = W_down (silu(W_gate x) * (W_up x)); W_gate and W_up [n_ff][n_embd], W_down
 * [n_embd][n_ff]. Gate and up rows share one pass over x. n_ff == 0 gives zeros. */
int ssd_feed_forward_f32_host(ssd_ctx* ctx, const float* x, const float* w_gate,
                              const float* w_up, const float* w_down, int n_embd, int n_ff,
                              float* out);

/* ------------------------------------------------------- decode engine */
/* Llama-shaped decoder with HBM-resident quantized weights, INT8 KV cache and
 * optional row-sharded tensor parallelism. Replaces forward_pass / generate's
 * per-token loop (src/inference/transformer.rs:283-399, :681-770).
 * tp_size > 1 needs ssd_model_tp_init before building. */
typedef struct {
    int n_layers, n_embd, n_head, n_head_kv, head_dim, n_ff, vocab;
    int wtype;        /* layer weight type: Q4_0, Q8_0, Q4_K, Q5_K, Q6_K or Q8_K; at tp_size 1
                         also F16, BF16, F32 and the low-bit Q2_K, Q3_K, IQ4_NL, IQ4_XS,
                         IQ3_XXS, IQ3_S, IQ2_XXS, IQ2_XS (decode step only: the batch
                         prefill refuses low-bit weights) */
    int out_type;     /* output.weight type: as wtype */
    int embd_type;    /* token_embd type: Q4_0 .. Q8_K, or F32 / F16 / BF16 */
    int kv_capacity;  /* INT8 KV positions */
    float theta, eps;
    int tp_rank, tp_size;
} ssd_model_config;

int ssd_model_create(ssd_ctx* ctx, const ssd_model_config* cfg, ssd_model** out);
/* The [row0, row0+nrows) x [col0, col0+ncols) slice of global tensor `name` that
 * rank cfg->tp_rank keeps (host only, needs no device). Row-sharded: attn_q,
 * ffn_gate, ffn_up, output; column-sharded: attn_output, ffn_down; replicated:
 * attn_k, attn_v, token_embd. Replaces the row split of parallel_matvec
 * (src/inference/tensor_parallel.rs:47-64), which only split rows. */
int ssd_shard_range(const ssd_model_config* cfg, const char* name, int layer, int* row0,
                    int* nrows, int* col0, int* ncols);
int ssd_model_free(ssd_model* m);
/* NCCL communicator for tensor parallelism: unique_id is the 128-byte
 * ncclUniqueId rank 0 got from ssd_tp_unique_id and shared out of band. Replaces the
 * thread spawn/join of src/inference/tensor_parallel.rs:69-103 (one process per GPU). */
int ssd_tp_unique_id(uint8_t out[128]);
int ssd_model_tp_init(ssd_model* m, const uint8_t unique_id[128]);
/* Peer-memory all-reduce for tensor parallelism. No reference counterpart: the
 * reference's "tensor parallelism" is a thread row-split with no reduction
 * (src/inference/tensor_parallel.rs:33-105). After ssd_model_tp_init, each rank calls
 * ssd_model_p2p_handle (allocates its receive buffer and returns the 64-byte CUDA IPC
 * handle), the handles are exchanged out of band, and each rank calls ssd_model_p2p_open
 * with all tp_size handles in rank order. From then on the decode step sums the o_proj
 * and down partials over NVLink peer memory inside its own kernels (bounded waits;
 * a peer that never arrives is reported as SSD_ERR_TIMEOUT by ssd_ctx_device_status)
 * instead of calling ncclAllReduce. One process per GPU, GPUs with peer access. */
int ssd_model_p2p_handle(ssd_model* m, uint8_t out[64]);
int ssd_model_p2p_open(ssd_model* m, const uint8_t* handles);
/* Fill every weight with ssd_weight_synth (this rank's shard of the global tensors).
 * No reference counterpart (benchmark inputs; the reference loads GGUF files). */
int ssd_model_synth_weights(ssd_model* m, uint64_t seed, float std_dev);
/* Set one tensor from host data in the reference layout (full, unsharded tensor;
 * the rank keeps its shard). name: attn_q, attn_k, attn_v, attn_output,
 * ffn_gate, ffn_up, ffn_down, attn_norm, ffn_norm (layer >= 0) or token_embd,
 * output_norm, output (layer = -1): the GGUF names of src/model/gguf.rs:410-416. */
int ssd_model_set_tensor(ssd_model* m, const char* name, int layer, const void* host_raw,
                         size_t bytes);
/* Same, with the tensor's own ggml type (-1: the type the model config gives that name).
 * A file may mix types per tensor; the reference reads each tensor's dtype from its GGUF
 * tensor info (src/model/gguf.rs:284-291) and dispatches the matvec on it
 * (src/metal/compute.rs:648-675). attn_q / attn_k and ffn_gate / ffn_up must share a type
 * (each pair is one fused launch); an attn_v of another type gets a launch of its own. */
int ssd_model_set_tensor_typed(ssd_model* m, const char* name, int layer, const void* host_raw,
                               size_t bytes, int ggml_type);
/* Fill the KV cache of every layer at positions [0, n) (both K and V rows drawn
 * N(0,1) by the synthetic generator, then INT8-quantized) and set the position.
 * No reference counterpart (benchmark inputs). */
int ssd_model_synth_kv(ssd_model* m, uint64_t seed, int n);
/* Sequence position (the `position` argument of forward_pass,
 * src/inference/transformer.rs:283-291); cache rows beyond it are ignored. */
int ssd_model_set_position(ssd_model* m, int pos);
int ssd_model_get_position(ssd_model* m, int* pos);
/* One decode step (one iteration of generate's loop, src/inference/transformer.rs:681-770)
 * from the token id in the model's device token slot: embed, all layers at the current
 * position, final norm, logits, argmax -> next token in the slot; position += 1.
 * Captured into a CUDA graph on first use when use_graph != 0. */
int ssd_model_decode_step(ssd_model* m, int use_graph);
/* Host token in, host token out: ssd_model_decode_step with the H2D and D2H copies
 * (generate's embed -> forward_pass -> sample, src/inference/transformer.rs:732-770). */
int ssd_model_decode_token(ssd_model* m, int32_t token_in, int32_t* token_out, int use_graph);
/* Layer-major batch prefill of n prompt tokens (host array) at the current position:
 * batch_prefill_lora (src/inference/transformer.rs:120-250) followed by the logits and
 * greedy argmax of the last token (generate, :681-741). Every layer's projections run as
 * tensor-core GEMMs over the n token rows, attention is causal over the INT8 cache (the
 * tokens' K/V rows are appended first); the first call prepares fp16 hi/lo splits of the
 * layer weights (4 bytes per weight, kept by the model). Leaves the decode state as after
 * n decode steps: position += n, the next token in the token slot and *next_token.
 * tp_size 1; n a multiple of 128; n_embd, n_ff and the QKV rows multiples of 128. */
int ssd_model_prefill(ssd_model* m, const int32_t* tokens, int n, int32_t* next_token);
/* Device pointers of the decode state: hidden [n_embd] (generate's hidden_state,
 * src/inference/transformer.rs:637), logits [vocab/tp], token. */
int ssd_model_state(ssd_model* m, float** hidden_dev, float** logits_dev, int32_t** token_dev);
/* This rank's shard of a model tensor (names as ssd_model_set_tensor), owned by the
 * model: for timing a layer's kernels in isolation. No reference counterpart. */
int ssd_model_weight(ssd_model* m, const char* name, int layer, ssd_weight** out);
/* Device pointer of a layer norm weight ("attn_norm", "ffn_norm") or "output_norm"
 * (layer -1); the RMSNorm weights of src/inference/transformer.rs:323-357. */
int ssd_model_norm(ssd_model* m, const char* name, int layer, float** out);
/* The INT8 KV cache of one layer, all KV heads (QuantizedKvCache::layer,
 * src/inference/quantized_kv_cache.rs:160-237). */
int ssd_model_kv(ssd_model* m, int layer, ssd_kv_cache** out);
/* One layer of forward_pass (src/inference/transformer.rs:312-394) on the model's
 * hidden state at the current position (layer parity tests). */
int ssd_model_layer_step(ssd_model* m, int layer);
/* Kernel launches issued by one decode step. No reference counterpart (reports). */
int ssd_model_launches_per_step(ssd_model* m, int* launches);

/* ------------------------------------------------ continuous-batch decode */
/* Sixteen decode slots over one model's weights: BatchScheduler (src/inference/
 * batch_scheduler.rs:24-129), whose step (:149-403) runs its decoding requests layer-major
 * (:236-296), each with its own KV cache and position. A slot holds one request; between
 * steps the caller may give a slot a new request (ssd_batch_set_position to its start,
 * then its prompt tokens as the slot's input of the next steps), which is the scheduler's
 * admission of queued requests (:157-166). One GPU (tp_size 1); layer and output weights
 * Q4_0 / Q8_0 / Q4_K with widths multiple of 256, head_dim <= 128. */
typedef struct ssd_batch ssd_batch;
/* BatchScheduler::new with its slots' caches (src/inference/batch_scheduler.rs:89-100,
 * the per-request KvCache of submit, :103-129);
 * capacity: INT8 KV positions per slot (every layer, every slot). */
int ssd_batch_create(ssd_model* m, int capacity, ssd_batch** out);
int ssd_batch_free(ssd_batch* b);
int ssd_batch_slots(ssd_batch* b, int* slots);
/* One step of every slot (BatchScheduler::step's decode phase and sampling,
 * src/inference/batch_scheduler.rs:225-363): tokens_in (host, one per slot) or NULL to feed
 * each slot its last output; the greedy next tokens into tokens_out (host, may be NULL); every slot's position
 * += 1 (stopping at the capacity). Captured into a CUDA graph on first use when
 * use_graph != 0. */
int ssd_batch_step(ssd_batch* b, const int32_t* tokens_in, int32_t* tokens_out, int use_graph);
/* A slot's position (a request's `position`, src/inference/batch_scheduler.rs:231, :350). */
int ssd_batch_set_position(ssd_batch* b, int slot, int pos);
int ssd_batch_positions(ssd_batch* b, int* pos);
/* Fill every slot's cache at positions [0, n) (K / V rows N(0,1), INT8-quantized) and set
 * every position to n. No reference counterpart (benchmark inputs). */
int ssd_batch_synth_kv(ssd_batch* b, uint64_t seed, int n);
/* Device pointers of one (layer, slot) INT8 cache: the layer cache of the slot's request
 * (src/inference/quantized_kv_cache.rs:101-130). */
int ssd_batch_kv_pointers(ssd_batch* b, int layer, int slot, int8_t** k, int8_t** v, float** ks,
                          float** vs);
/* Device pointer of the slots' hidden states [16][n_embd] after a step (each request's
 * hidden_state, src/inference/batch_scheduler.rs:300-303). */
int ssd_batch_state(ssd_batch* b, float** hidden_dev);
/* Kernel launches issued by one batch step. No reference counterpart (reports). */
int ssd_batch_launches_per_step(ssd_batch* b, int* launches);

/* ------------------------------------------------------------ GGUF files */
typedef struct ssd_gguf ssd_gguf;
/* GgufFile::open (src/model/gguf.rs:233-315): parses the header, metadata and tensor
 * infos (magic "GGUF", version 2-3, strings <= 1 MiB, data at the next multiple of
 * general.alignment, default 32). Host only. Bad files fail with SSD_ERR_ARG. */
int ssd_gguf_open(const char* path, ssd_gguf** out);
/* Frees the parsed file (the GgufFile value of src/model/gguf.rs:224-231 going out of
 * scope). */
int ssd_gguf_close(ssd_gguf* g);
/* GgufHeader fields and GgufFile::data_offset (src/model/gguf.rs:139-143, :224-231). */
int ssd_gguf_info(const ssd_gguf* g, uint32_t* version, uint64_t* n_tensors, uint64_t* n_kv,
                  uint64_t* data_offset);
/* TensorInfo i (src/model/gguf.rs:216-222): name (NUL-terminated, truncated to cap),
 * dims (ne0 = columns first), ggml type, offset in the data section, size in bytes. */
int ssd_gguf_tensor(const ssd_gguf* g, uint64_t i, char* name, size_t cap, uint32_t* n_dims,
                    uint64_t dims[8], uint32_t* type, uint64_t* offset, uint64_t* size_bytes);
/* GgufFile::find_tensor (src/model/gguf.rs:405-407): index, or -1 if absent. */
int ssd_gguf_find(const ssd_gguf* g, const char* name, int64_t* index);
/* GgufFile::get_u32 / get_f32 and MetadataValue::as_u32 / as_f32 / as_string
 * (src/model/gguf.rs:427-435, :183-212): *found = 0 when the key is absent or of another
 * type. The array length is what vocab_size reads from tokenizer.ggml.tokens
 * (src/model/gguf.rs:371-379). */
int ssd_gguf_get_u32(const ssd_gguf* g, const char* key, int* found, uint32_t* value);
int ssd_gguf_get_f32(const ssd_gguf* g, const char* key, int* found, float* value);
int ssd_gguf_get_str(const ssd_gguf* g, const char* key, int* found, char* out, size_t cap);
int ssd_gguf_array_len(const ssd_gguf* g, const char* key, int* found, uint64_t* n);
/* Raw bytes of tensor i in the file's block format (what the layer streamer reads,
 * src/ssd/streamer.rs:34-91); bytes must equal its size. */
int ssd_gguf_read(const ssd_gguf* g, uint64_t i, void* dst, size_t bytes);
/* Decode-engine config from the file's {arch}.* metadata (GgufFile::architecture ..
 * vocab_size, src/model/gguf.rs:318-379; RoPE base default 10000 as
 * src/inference/transformer.rs:20-21; eps default 1e-5), the layer / output / embedding
 * types from blk.0.attn_q, output (or token_embd) and token_embd. */
int ssd_gguf_model_config(const ssd_gguf* g, int kv_capacity, int tp_rank, int tp_size,
                          ssd_model_config* cfg);
/* Loads every tensor of the first n_layers layers plus token_embd, output_norm and
 * output (token_embd if absent, src/inference/transformer.rs:690-700) into the model:
 * this rank's shard, HBM-resident (the layer lookups of transformer.rs:171-180, :557). */
int ssd_model_load_gguf(ssd_model* m, const ssd_gguf* g, int n_layers);

/* ---------------------------------------------------- SSD -> HBM streaming tier
 * For models whose layers do not all fit the HBM budget: the layer matrices stay in the GGUF
 * file and pass through n_slots = hbm_budget / slot_bytes HBM layer slots. */
typedef struct ssd_stream ssd_stream;
/* LayerCache's CacheStats (src/model/cache.rs: hits, misses, evictions, prefetch_hits) plus
 * the loads made, the file bytes read, and the slot count and size the budget bought. */
typedef struct {
    uint64_t hits, misses, evictions, prefetch_hits, loads, bytes_read;
    int n_slots;
    size_t slot_bytes;
} ssd_stream_stats;
/* SsdStreamer::new + Prefetcher::new(LookAhead(lookahead)) + LayerCache::new(budget)
 * (src/ssd/streamer.rs:19-32, src/ssd/prefetch.rs:24-31, src/model/cache.rs): opens the
 * file, loads every layer's attn_norm / ffn_norm and token_embd, output_norm, output
 * (token_embd if absent) into the model, and allocates the slots (each sized for the
 * largest layer's seven matrices in the library layout), two pinned staging buffers and a
 * copy stream. The model (from ssd_gguf_model_config of the same file, tp_size 1) must
 * not hold layer matrices of its own (SSD_ERR_STATE). SSD_ERR_NOMEM if the budget is below
 * one layer. */
int ssd_stream_open(ssd_model* m, const char* gguf_path, size_t hbm_budget, int lookahead,
                    ssd_stream** out);
/* LayerCache::pin (src/model/cache.rs): loads the layer now if needed and never evicts it;
 * refused (SSD_ERR_NOMEM) if it would leave no slot for the other layers. */
int ssd_stream_pin(ssd_stream* s, int layer);
/* ssd_model_decode_token with streamed layers (the layer loop of forward_pass with
 * layer_cache.get / streamer.load_layer on a miss and prefetcher.on_layer_start before each
 * layer, src/inference/transformer.rs:151-163): eager launches, each layer's kernels after
 * its slot is loaded; after them the next `lookahead` layers are loaded. */
int ssd_stream_decode_token(ssd_stream* s, int32_t token_in, int32_t* token_out);
/* Counters since ssd_stream_open (LayerCache::stats, src/model/cache.rs). */
int ssd_stream_stats_get(const ssd_stream* s, ssd_stream_stats* out);
/* Waits for the model's stream and frees the slots, staging buffers and copy stream; the
 * model stays usable for ssd_model_free. No reference counterpart beyond Drop. */
int ssd_stream_close(ssd_stream* s);

#ifdef __cplusplus
}
#endif
#endif /* SSDLLM_CUDA_H */
