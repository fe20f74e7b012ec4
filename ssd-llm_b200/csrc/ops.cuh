// ops.cuh — launchers for the non-matvec operators (internal interface).
#pragma once
#include "common.cuh"

namespace ssd {

// INT8 KV append of one position (k and v rows of kv_dim floats). The position is
// read from pos_dev when non-null (graph replay), else `pos`.
int launch_kv_append(const ssd_kv_cache* kv, const float* k, const float* v, int pos,
                     const int* pos_dev, int rows, cudaStream_t s, bool pdl);

// Split-K decode attention over the INT8 cache. seq_len = (*pos_dev + 1) when pos_dev
// is non-null, else seq_len. kv_head0 / n_kv_local select this rank's KV heads;
// q holds n_kv_local * group heads. partial must hold attn_partial_floats() floats.
struct AttnArgs {
    const int8_t* k;
    const int8_t* v;
    const float* ks;
    const float* vs;
    int kv_dim, head_dim, group, kv_head0, n_kv_local;
    const float* q;
    float* out;
    float* partial;
    int seq_len;
    const int* pos_dev;
    int max_seq;  // grid is sized for max_seq positions (graph-stable)
    // Batch of causal queries (prefill): when n_q > 1, query i (q + i * q_stride, out +
    // i * out_stride) attends to positions [0, seq0 + i], its partials at
    // partial + i * attn_partial_floats(heads, max_seq, head_dim).
    int n_q;
    int q_stride, out_stride;
    int seq0;
    // Decode with the KV append fused (n_q 1, pos_dev set): when k_new is non-null the
    // CTAs of the new position's chunk quantize k_new / v_new (kv_dim floats each) into the
    // cache at *pos_dev (their own heads' bytes; local head 0 also the scales) first.
    const float* k_new;
    const float* v_new;
    int* status;  // device status word for bounded waits (default: the context's)
    // Tensor-core prefill kernel only: when set, the output rows are written as fp16 hi /
    // lo splits (hi = fp16(o), lo = fp16(o - hi), row stride out_stride: the A operand of
    // the output-projection GEMM) instead of fp32 out.
    __half* out_hi;
    __half* out_lo;
    // Continuous-batch decode (n_slots > 0, with the fused append): query z = slot z, whose
    // cache is k / v + z * slot_kv bytes and ks / vs + z * slot_sc floats, whose position is
    // pos_dev[z] and whose new rows are k_new / v_new + z * slot_new floats.
    int n_slots;
    size_t slot_kv;
    int slot_sc, slot_new;
    // K / V sharded by heads over tensor-parallel ranks (fused append): the INT8 row scale
    // spans every rank's heads (quantized_kv_cache.rs:107-110), so the global absmax of the
    // new K and V rows is needed. Either amax_in holds it (K, V; computed and max-reduced
    // by the caller), or xch_n > 1 ranks exchange their local pair in the kernel: the CTA of
    // local head 0 in the new position's chunk writes word 2j+w = (absmax bits << 32) | tag
    // to xch_out[r] for every rank r, and the chunk's CTAs wait (bounded) until all xch_n
    // pairs of xch_in carry the tag (uint32)(*xch_epoch + xch_call) + 1.
    const float* amax_in;
    int xch_n;
    int xch_call;
    const unsigned long long* xch_epoch;
    const unsigned long long* xch_in;
    unsigned long long* xch_out[8];
    // Set by launch_attention (decode): CTAs per KV head; each takes group / hsplit of its
    // query heads over the chunk's positions.
    int hsplit;
};
// Local absmax pair (K, V) of the n-float rows k, v into out[0..1] (one CTA).
int launch_kv_absmax(const float* k, const float* v, int n, float* out, cudaStream_t s, bool pdl);
// Quantizes `rows` full K / V rows of src_dim floats (row scale over the whole row) and
// stores columns [col0, col0 + kv->kv_dim) of each at positions pos.. of the cache (a rank's
// head slice under tensor parallelism; col0 0 and src_dim kv->kv_dim for a whole row).
int launch_kv_append_slice(const ssd_kv_cache* kv, const float* k, const float* v, int src_dim,
                           int col0, int pos, int rows, cudaStream_t s);
// Causal attention of a prompt batch on the tcgen05 tensor cores (attn_tc.cu): n_q
// queries (a multiple of 128, head_dim 128) at positions seq0 .., over the cache rows
// [0, seq0 + n_q) already appended. Same arguments as the batched launch_attention.
int launch_attention_prefill_tc(ssd_ctx* ctx, const AttnArgs& a, cudaStream_t s, bool pdl);
// The prompt-batch attention: the tensor-core kernel where it covers the shape, else
// launch_attention's batched per-query kernels (which need a.partial).
int launch_prefill_attention(ssd_ctx* ctx, const AttnArgs& a, cudaStream_t s, bool pdl);
// Whether launch_prefill_attention takes the tensor-core kernel for these arguments.
bool prefill_attention_uses_tc(const AttnArgs& a);
size_t attn_partial_floats(int n_heads, int max_seq, int head_dim);
int launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl);

// Embedding row gather (token from *token_dev, or from the argmax key when
// key_dev is non-null) into hidden.
int launch_embed(const ssd_weight* emb, const int32_t* token_dev, float* hidden, cudaStream_t s,
                 bool pdl);
// Embedding rows of n tokens (tokens_dev[n]) into hidden [n][n_embd].
int launch_embed_rows(const ssd_weight* emb, const int32_t* tokens_dev, int n, float* hidden,
                      cudaStream_t s);
// token = low 32 bits of *key; *key = 0; *pos += 1; *epoch += epoch_inc (if epoch).
int launch_finalize(unsigned long long* key, int32_t* token, int* pos, unsigned long long* epoch,
                    int epoch_inc, cudaStream_t s, bool pdl);

}  // namespace ssd
