/*
 * oracle.h — CPU restatement of ssd-llm's CPU compute path (TEST INFRASTRUCTURE ONLY).
 *
 * This library is the parity checker for the CUDA backend. Only tests/, the
 * smoke() check in __graft_entry__.py and bench.py's cpu_baseline / reference
 * arm may load it. The product path never calls it.
 *
 * Every function restates one function of the reference (Rust, quantumnic/ssd-llm)
 * with the same loop nesting, the same accumulator structure and the same
 * operation order, in `float`, compiled with -ffp-contract=off and without
 * fast-math, so that results are bitwise what the reference's x86 scalar path
 * computes (glibc libm stands in for Rust std's libm calls on Linux).
 * Citations are path:line inside the reference project.
 */
#ifndef SSD_ORACLE_H
#define SSD_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GgmlType ids: src/model/gguf.rs:16-47 */
enum { ORA_F32 = 0, ORA_F16 = 1, ORA_Q4_0 = 2, ORA_Q8_0 = 8, ORA_Q2_K = 10, ORA_Q3_K = 11,
       ORA_Q4_K = 12, ORA_Q5_K = 13, ORA_Q6_K = 14, ORA_Q8_K = 15, ORA_IQ2_XXS = 16,
       ORA_IQ2_XS = 17, ORA_IQ3_XXS = 18, ORA_IQ4_NL = 20, ORA_IQ3_S = 21, ORA_IQ4_XS = 23,
       ORA_BF16 = 30 };

/* Low-bit formats in the reference's block layouts (oracle_iq.c, compute.rs:793-1075,
 * 1964-2240): block size / bytes, one matvec row (-1 for other types), dequantize (the
 * per-element weight value the reference multiplies x by). */
int ora_lowbit_block(int type);
size_t ora_lowbit_block_bytes(int type);
int ora_row_lowbit(int type, const uint8_t* w, const float* x, int in_dim, int row, float* y);
int ora_dequant_lowbit(const uint8_t* w, int type, int64_t n, float* out);

/* f16 -> f32 (half::f16::to_f32, used by f16_to_f32 src/metal/compute.rs:2244-2247). */
float ora_f16_to_f32(uint16_t h);
/* f32 -> f16 round-to-nearest-even (half::f16::from_f32, used by the reference tests). */
uint16_t ora_f32_to_f16(float f);

/* Bytes per row for a type (src/model/gguf.rs block sizes). 0 if unsupported. */
size_t ora_row_bytes(int type, int64_t n_cols);

/* Builder's quantizers: exact inverses of the reference decoders. Input rows of
 * n elements (n a multiple of the block size) -> reference block layout. */
void ora_quantize_q4_0(const float* w, int64_t n, uint8_t* out);
void ora_quantize_q8_0(const float* w, int64_t n, uint8_t* out);
void ora_quantize_q4_k(const float* w, int64_t n, uint8_t* out);

/* Dequantize to f32: src/ssd/streamer.rs:93-180 (Q4_0, Q8_0, F16, F32); Q4_K uses
 * the element formula of matvec_q4_k_cpu src/metal/compute.rs:707-750, Q6_K that of
 * matvec_q6_k_cpu src/metal/compute.rs:752-790 ((d * scale) * q), Q5_K that of
 * matvec_q5_k_cpu src/metal/compute.rs:845-899 (scale * q - min), Q8_K that of
 * matvec_q8_k_cpu src/metal/compute.rs:971-993 (d * q). Returns 0,
 * or -1 for an unsupported type. */
int ora_dequantize(const uint8_t* w, int type, int64_t n, float* out);

/* Quantized matvec, src/metal/compute.rs:648-790, :904-925. Unsupported type:
 * writes zeros and returns -1 (the reference returns zeros, :672-675). */
int ora_matvec_quantized(const uint8_t* w, const float* x, int out_dim, int in_dim,
                         int type, float* y);
/* Same result, rows split over `threads` pthreads (tensor_parallel.rs:33-105 split;
 * per-row arithmetic unchanged, so bitwise equal to threads=1). */
int ora_matvec_quantized_mt(const uint8_t* w, const float* x, int out_dim, int in_dim,
                            int type, float* y, int threads);

/* f32 matvec with 4 accumulators: matvec_f32_simd_scalar src/metal/compute.rs:390-424. */
void ora_matvec_f32(const float* w, const float* x, int out_dim, int in_dim, float* y);

/* rmsnorm_f32_fast_scalar src/metal/compute.rs:580-588 (in place). */
void ora_rmsnorm(float* x, const float* w, int n, float eps);
/* fused_residual_rmsnorm_f32 src/metal/compute.rs:444-460 (in place). */
void ora_fused_residual_rmsnorm(float* x, const float* residual, const float* w, int n, float eps);
/* fused_post_attn_norm_f32_cpu src/metal/compute.rs:536-555: h += a; out = norm(h). */
void ora_fused_post_attn_norm(float* hidden, const float* attn, const float* w, int n, float eps,
                              float* out);
/* fused_rmsnorm_linear_f32_cpu src/metal/compute.rs:557-577 (eps fixed at 1e-5). */
void ora_fused_rmsnorm_linear(const float* x, const float* norm_w, const float* out_w,
                              int vocab, int n_embd, float* logits);

/* rope_f32_multi_head src/metal/compute.rs:482-506 (in place). */
void ora_rope_multi_head(float* x, int len, int head_dim, int n_heads, int position, float theta);
/* softmax_f32_fast_scalar src/metal/compute.rs:604-620 (in place). */
void ora_softmax(float* x, int n);
/* silu_f32 src/metal/compute.rs:641-645 (in place). */
void ora_silu(float* x, int n);
/* argmax src/inference/sampler.rs:572-578: ties keep the LAST index. */
int ora_argmax(const float* v, int n);

/* INT8 KV row quantizer QuantizedVec::quantize src/inference/quantized_kv_cache.rs:23-41. */
void ora_kv_quantize(const float* v, int n, int8_t* q, float* scale);
/* QuantizedVec::dequantize_into src/inference/quantized_kv_cache.rs:48-53. */
void ora_kv_dequantize(const int8_t* q, float scale, int n, float* out);

/* Decode attention over an INT8 KV cache.
 * K/V cache: [seq_len][kv_dim] int8 + one f32 scale per (position, K or V)
 * (QuantizedLayerKvCache, src/inference/quantized_kv_cache.rs:107-130).
 * ora_attention_int8 restates the score/softmax/weighted-sum loops of
 * multi_head_attention_fused_rope src/inference/attention.rs:198-236 (no wo);
 * ora_flash_attention_int8 restates the online-softmax loop of
 * flash_attention_cached src/inference/flash_attention.rs:68-135 (no wo). */
void ora_attention_int8(const float* q, const int8_t* k, const float* ks, const int8_t* v,
                        const float* vs, int seq_len, int n_head, int n_head_kv, int head_dim,
                        float* out);
void ora_flash_attention_int8(const float* q, const int8_t* k, const float* ks, const int8_t* v,
                              const float* vs, int seq_len, int n_head, int n_head_kv,
                              int head_dim, float* out);

/* f32 K/V windowed attention: flash_attention_f32 (src/metal/shaders/kernels.metal:1360-1440,
 * flash_attention_windowed src/inference/flash_attention.rs:146-229). */
void ora_flash_attention_f32(const float* q, const float* k, const float* v, int n_head,
                             int n_head_kv, int head_dim, int seq_len, int window_start,
                             int window_end, float* out);
/* SwiGLU feed-forward, src/inference/feed_forward.rs:17-43. */
void ora_feed_forward_f32(const float* x, const float* w_gate, const float* w_up,
                          const float* w_down, int n_embd, int n_ff, float* out);

/* One decoder layer decode step: forward_pass body src/inference/transformer.rs:312-394
 * with multi_head_attention_fused_rope (attention.rs:172-240) over the INT8 cache and
 * feed_forward (feed_forward.rs:17-44). Weights are packed in `wtype` (reference layout).
 * matvec_mode 0: the reference's live path (dequantize to f32, matvec_f32_simd);
 * matvec_mode 1: the operator path (matvec_quantized_cpu).
 * The K/V of `position` are quantized into the cache row `position`; attention runs
 * over positions 0..position. `hidden` is updated in place. */
typedef struct {
    int n_embd, n_head, n_head_kv, head_dim, n_ff;
    int wtype;
    const uint8_t *wq, *wk, *wv, *wo, *w_gate, *w_up, *w_down;
    const float *attn_norm, *ffn_norm;
    float theta, eps;
    /* per-matrix types (wq, wk, wv, wo, w_gate, w_up, w_down) where the file mixes them,
     * as the reference's per-tensor dispatch allows (compute.rs:648-675); -1 = wtype */
    int wtypes[7];
} ora_layer;

int ora_layer_step(const ora_layer* L, float* hidden, int position, int8_t* k_cache,
                   float* k_scales, int8_t* v_cache, float* v_scales, int matvec_mode,
                   int threads);

#ifdef __cplusplus
}
#endif
#endif
