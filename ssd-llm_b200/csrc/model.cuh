// model.cuh — decode-engine hooks for the SSD -> HBM streaming tier (internal interface).
#pragma once
#include "common.cuh"

struct ssd_model;

namespace ssd {

// Layer weights supplied per step instead of held by the model: before layer l's kernels
// are enqueued on stream s, acquire(user, l, s, w) returns its seven matrices (attn_q,
// attn_k, attn_v, attn_output, ffn_gate, ffn_up, ffn_down) and makes s wait until they are
// on the device; after them, release(user, l, s) may record that s is done with them.
struct LayerHooks {
    int (*acquire)(void* user, int layer, cudaStream_t s, ssd_weight* const* (&w));
    int (*release)(void* user, int layer, cudaStream_t s);
    void* user;
};

// One greedy decode step like ssd_model_decode_token, launched eagerly (no graph: the
// weight pointers change from step to step), with the layer matrices from `hk`. The model
// itself must hold the norms and the global tensors; tp_size 1.
int model_decode_token_hooked(ssd_model* m, int32_t token_in, int32_t* token_out,
                              const LayerHooks& hk);
ssd_ctx* model_ctx(const ssd_model* m);
// True if any layer holds one of its seven matrices (set_tensor / synth / GGUF load).
bool model_has_layer_matrices(const ssd_model* m);
const ssd_model_config& model_cfg(const ssd_model* m);

}  // namespace ssd
