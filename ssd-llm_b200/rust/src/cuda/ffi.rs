//! Raw bindings of `libssdllm_cuda.so`, the B200 (sm_100a) compute backend: one
//! declaration per entry point of `include/ssdllm_cuda.h`, with the same names, argument
//! order and types (opaque handles, plain pointers, sizes, `c_int` status codes). The safe
//! `CudaCompute` wrapper with `MetalCompute`'s signatures is in `compute.rs`.
//!
//! Every call returns `SSD_OK` (0) or an `SSD_ERR_*` code; `ssd_last_error()` gives the
//! calling thread's last message. `*_dev` pointers are device pointers and `stream` is a
//! `cudaStream_t` (null = CUDA's default stream); `*_host` calls take host slices and
//! synchronise before returning.
#![allow(non_camel_case_types, dead_code)]

use std::os::raw::{c_char, c_float, c_int, c_void};

#[repr(C)]
pub struct SsdCtx {
    _p: [u8; 0],
}
#[repr(C)]
pub struct SsdWeight {
    _p: [u8; 0],
}
#[repr(C)]
pub struct SsdKvCache {
    _p: [u8; 0],
}
#[repr(C)]
pub struct SsdModel {
    _p: [u8; 0],
}
#[repr(C)]
pub struct SsdBatch {
    _p: [u8; 0],
}
#[repr(C)]
pub struct SsdGguf {
    _p: [u8; 0],
}
#[repr(C)]
pub struct SsdStream {
    _p: [u8; 0],
}

/// `ssd_stream_stats`: LayerCache's counters plus the loads, file bytes read and slots.
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct SsdStreamStats {
    pub hits: u64,
    pub misses: u64,
    pub evictions: u64,
    pub prefetch_hits: u64,
    pub loads: u64,
    pub bytes_read: u64,
    pub n_slots: c_int,
    pub slot_bytes: usize,
}

/// `ssd_model_config`: the decode engine's shape (layer weights in one quantized type).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct SsdModelConfig {
    pub n_layers: c_int,
    pub n_embd: c_int,
    pub n_head: c_int,
    pub n_head_kv: c_int,
    pub head_dim: c_int,
    pub n_ff: c_int,
    pub vocab: c_int,
    pub wtype: c_int,
    pub out_type: c_int,
    pub embd_type: c_int,
    pub kv_capacity: c_int,
    pub theta: c_float,
    pub eps: c_float,
    pub tp_rank: c_int,
    pub tp_size: c_int,
}

pub const SSD_ABI_VERSION: c_int = 1;

pub const SSD_OK: c_int = 0;
pub const SSD_ERR_ARG: c_int = 1;
pub const SSD_ERR_TYPE: c_int = 2;
pub const SSD_ERR_SHAPE: c_int = 3;
pub const SSD_ERR_CUDA: c_int = 4;
pub const SSD_ERR_TIMEOUT: c_int = 5;
pub const SSD_ERR_NCCL: c_int = 6;
pub const SSD_ERR_NOMEM: c_int = 7;
pub const SSD_ERR_STATE: c_int = 8;

/// GgmlType ids (src/model/gguf.rs:16-47) the library accepts.
pub const SSD_TYPE_F32: c_int = 0;
pub const SSD_TYPE_F16: c_int = 1;
pub const SSD_TYPE_Q4_0: c_int = 2;
pub const SSD_TYPE_Q8_0: c_int = 8;
pub const SSD_TYPE_Q4_K: c_int = 12;
pub const SSD_TYPE_Q5_K: c_int = 13;
pub const SSD_TYPE_Q6_K: c_int = 14;
pub const SSD_TYPE_Q8_K: c_int = 15;
pub const SSD_TYPE_BF16: c_int = 30;

#[link(name = "ssdllm_cuda")]
extern "C" {
    // ---- basics: version, status strings, contexts, copies
    pub fn ssd_abi_version() -> c_int;
    pub fn ssd_status_str(status: c_int) -> *const c_char;
    pub fn ssd_last_error() -> *const c_char;
    pub fn ssd_ctx_create(device: c_int, out: *mut *mut SsdCtx) -> c_int;
    pub fn ssd_ctx_get(device: c_int, out: *mut *mut SsdCtx) -> c_int;
    pub fn ssd_ctx_destroy(ctx: *mut SsdCtx) -> c_int;
    pub fn ssd_ctx_stream(ctx: *mut SsdCtx, stream_out: *mut *mut c_void) -> c_int;
    pub fn ssd_ctx_sync(ctx: *mut SsdCtx) -> c_int;
    pub fn ssd_ctx_device_status(ctx: *mut SsdCtx, status: *mut c_int) -> c_int;
    pub fn ssd_ctx_set_pdl(ctx: *mut SsdCtx, on: c_int) -> c_int;
    pub fn ssd_ctx_info(
        ctx: *mut SsdCtx,
        num_sms: *mut c_int,
        name: *mut c_char,
        name_len: usize,
    ) -> c_int;
    pub fn ssd_copy_to_device(
        ctx: *mut SsdCtx,
        dst_dev: *mut c_void,
        src_host: *const c_void,
        bytes: usize,
    ) -> c_int;
    pub fn ssd_copy_to_host(
        ctx: *mut SsdCtx,
        dst_host: *mut c_void,
        src_dev: *const c_void,
        bytes: usize,
    ) -> c_int;

    // ---- HBM-resident weights (replace the per-call uploads of src/metal/gpu.rs:396-490)
    pub fn ssd_weight_upload(
        ctx: *mut SsdCtx,
        host_raw: *const c_void,
        bytes: usize,
        ggml_type: c_int,
        rows: c_int,
        cols: c_int,
        out: *mut *mut SsdWeight,
    ) -> c_int;
    pub fn ssd_weight_upload_device(
        ctx: *mut SsdCtx,
        raw_dev: *const c_void,
        bytes: usize,
        ggml_type: c_int,
        rows: c_int,
        cols: c_int,
        out: *mut *mut SsdWeight,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_weight_download(
        ctx: *mut SsdCtx,
        w: *const SsdWeight,
        host_raw: *mut c_void,
        bytes: usize,
    ) -> c_int;
    pub fn ssd_weight_free(w: *mut SsdWeight) -> c_int;
    pub fn ssd_weight_info(
        w: *const SsdWeight,
        ggml_type: *mut c_int,
        rows: *mut c_int,
        cols: *mut c_int,
        raw_bytes: *mut usize,
    ) -> c_int;
    pub fn ssd_row_bytes(ggml_type: c_int, cols: i64) -> usize;
    pub fn ssd_weight_synth(
        ctx: *mut SsdCtx,
        ggml_type: c_int,
        seed: u64,
        tensor_id: u32,
        std_dev: c_float,
        total_cols: i64,
        row0: c_int,
        rows: c_int,
        col0: c_int,
        cols: c_int,
        out: *mut *mut SsdWeight,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_synth_f32(
        ctx: *mut SsdCtx,
        seed: u64,
        tensor_id: u32,
        mean: c_float,
        std_dev: c_float,
        total_cols: i64,
        row0: c_int,
        rows: c_int,
        col0: c_int,
        cols: c_int,
        out_dev: *mut c_float,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_quantize(
        ctx: *mut SsdCtx,
        x_dev: *const c_float,
        rows: c_int,
        cols: c_int,
        ggml_type: c_int,
        raw_out_dev: *mut c_void,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_dequantize(
        ctx: *mut SsdCtx,
        w: *const SsdWeight,
        out_dev: *mut c_float,
        stream: *mut c_void,
    ) -> c_int;

    // ---- device-pointer operators (MetalGpu kernels, src/metal/gpu.rs:169-1258)
    pub fn ssd_prefill_matmul(
        ctx: *mut SsdCtx,
        w: *const SsdWeight,
        x_dev: *const c_float,
        n_tokens: c_int,
        y_dev: *mut c_float,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_matvec(
        ctx: *mut SsdCtx,
        w: *const SsdWeight,
        x_dev: *const c_float,
        y_dev: *mut c_float,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_matvec_residual(
        ctx: *mut SsdCtx,
        w: *const SsdWeight,
        x_dev: *const c_float,
        base_dev: *const c_float,
        y_dev: *mut c_float,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_fused_rmsnorm_matvec(
        ctx: *mut SsdCtx,
        w: *const SsdWeight,
        x_dev: *const c_float,
        norm_w_dev: *const c_float,
        eps: c_float,
        y_dev: *mut c_float,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_fused_qkv_rope(
        ctx: *mut SsdCtx,
        wq: *const SsdWeight,
        wk: *const SsdWeight,
        wv: *const SsdWeight,
        x_dev: *const c_float,
        norm_w_dev: *const c_float,
        eps: c_float,
        head_dim: c_int,
        position: c_int,
        theta: c_float,
        q_dev: *mut c_float,
        k_dev: *mut c_float,
        v_dev: *mut c_float,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_fused_swiglu(
        ctx: *mut SsdCtx,
        w_gate: *const SsdWeight,
        w_up: *const SsdWeight,
        x_dev: *const c_float,
        norm_w_dev: *const c_float,
        eps: c_float,
        act_dev: *mut c_float,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_rmsnorm(
        ctx: *mut SsdCtx,
        x_dev: *mut c_float,
        w_dev: *const c_float,
        n: c_int,
        eps: c_float,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_fused_post_attn_norm(
        ctx: *mut SsdCtx,
        hidden_dev: *mut c_float,
        attn_dev: *const c_float,
        w_dev: *const c_float,
        n: c_int,
        eps: c_float,
        out_dev: *mut c_float,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_softmax(
        ctx: *mut SsdCtx,
        x_dev: *mut c_float,
        n: c_int,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_rope(
        ctx: *mut SsdCtx,
        x_dev: *mut c_float,
        len: c_int,
        head_dim: c_int,
        n_heads: c_int,
        position: c_int,
        theta: c_float,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_silu(ctx: *mut SsdCtx, x_dev: *mut c_float, n: c_int, stream: *mut c_void) -> c_int;
    pub fn ssd_argmax(
        ctx: *mut SsdCtx,
        v_dev: *const c_float,
        n: c_int,
        idx_dev: *mut i32,
        stream: *mut c_void,
    ) -> c_int;

    // ---- INT8 KV cache and attention (src/inference/quantized_kv_cache.rs, attention.rs)
    pub fn ssd_kv_create(
        ctx: *mut SsdCtx,
        capacity: c_int,
        n_head_kv: c_int,
        head_dim: c_int,
        out: *mut *mut SsdKvCache,
    ) -> c_int;
    pub fn ssd_kv_free(kv: *mut SsdKvCache) -> c_int;
    pub fn ssd_kv_pointers(
        kv: *mut SsdKvCache,
        k_dev: *mut *mut i8,
        v_dev: *mut *mut i8,
        k_scale_dev: *mut *mut c_float,
        v_scale_dev: *mut *mut c_float,
    ) -> c_int;
    pub fn ssd_kv_append(
        ctx: *mut SsdCtx,
        kv: *mut SsdKvCache,
        k_dev: *const c_float,
        v_dev: *const c_float,
        position: c_int,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_kv_append_rows(
        ctx: *mut SsdCtx,
        kv: *mut SsdKvCache,
        k_dev: *const c_float,
        v_dev: *const c_float,
        position: c_int,
        rows: c_int,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_attention_int8(
        ctx: *mut SsdCtx,
        kv: *const SsdKvCache,
        q_dev: *const c_float,
        n_head: c_int,
        seq_len: c_int,
        out_dev: *mut c_float,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_attention_int8_noalloc(
        ctx: *mut SsdCtx,
        kv: *const SsdKvCache,
        q_dev: *const c_float,
        n_head: c_int,
        seq_len: c_int,
        out_dev: *mut c_float,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_attention_prefill(
        ctx: *mut SsdCtx,
        kv: *const SsdKvCache,
        q_dev: *const c_float,
        n_q: c_int,
        q_stride: c_int,
        pos0: c_int,
        n_head: c_int,
        out_dev: *mut c_float,
        out_stride: c_int,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_matvec_peer_input(
        ctx: *mut SsdCtx,
        w: *const SsdWeight,
        x_dev: *const c_float,
        partials_dev: *const c_float,
        n_ranks: c_int,
        flags_dev: *const u64,
        epoch_dev: *const u64,
        call: c_int,
        y_dev: *mut c_float,
        stream: *mut c_void,
    ) -> c_int;

    // ---- host-slice operators: the MetalCompute methods (src/metal/compute.rs:145-375)
    pub fn ssd_matvec_quantized_host(
        ctx: *mut SsdCtx,
        w_raw: *const u8,
        w_bytes: usize,
        x: *const c_float,
        y: *mut c_float,
        out_dim: c_int,
        in_dim: c_int,
        ggml_type: c_int,
    ) -> c_int;
    pub fn ssd_matvec_f32_host(
        ctx: *mut SsdCtx,
        w: *const c_float,
        x: *const c_float,
        y: *mut c_float,
        out_dim: c_int,
        in_dim: c_int,
    ) -> c_int;
    pub fn ssd_rmsnorm_f32_host(
        ctx: *mut SsdCtx,
        x: *mut c_float,
        weight: *const c_float,
        n: c_int,
        eps: c_float,
    ) -> c_int;
    pub fn ssd_softmax_f32_host(ctx: *mut SsdCtx, x: *mut c_float, n: c_int) -> c_int;
    pub fn ssd_flash_attention_f32_host(
        ctx: *mut SsdCtx,
        q: *const c_float,
        k: *const c_float,
        v: *const c_float,
        n_head: c_int,
        n_head_kv: c_int,
        head_dim: c_int,
        seq_len: c_int,
        window_start: c_int,
        window_end: c_int,
        out: *mut c_float,
    ) -> c_int;
    pub fn ssd_flash_attention_f32(
        ctx: *mut SsdCtx,
        q_dev: *const c_float,
        k_dev: *const c_float,
        v_dev: *const c_float,
        n_head: c_int,
        n_head_kv: c_int,
        head_dim: c_int,
        seq_len: c_int,
        window_start: c_int,
        window_end: c_int,
        out_dev: *mut c_float,
        stream: *mut c_void,
    ) -> c_int;
    pub fn ssd_fused_qkv_f32_host(
        ctx: *mut SsdCtx,
        wq: *const c_float,
        wk: *const c_float,
        wv: *const c_float,
        x: *const c_float,
        q_dim: c_int,
        kv_dim: c_int,
        n_embd: c_int,
        q: *mut c_float,
        k: *mut c_float,
        v: *mut c_float,
    ) -> c_int;
    pub fn ssd_fused_qkv_rope_f32_host(
        ctx: *mut SsdCtx,
        wq: *const c_float,
        wk: *const c_float,
        wv: *const c_float,
        x: *const c_float,
        q_dim: c_int,
        kv_dim: c_int,
        n_embd: c_int,
        head_dim: c_int,
        position: c_int,
        theta: c_float,
        q: *mut c_float,
        k: *mut c_float,
        v: *mut c_float,
    ) -> c_int;
    pub fn ssd_fused_post_attn_norm_f32_host(
        ctx: *mut SsdCtx,
        hidden: *mut c_float,
        attn: *const c_float,
        norm_w: *const c_float,
        n: c_int,
        eps: c_float,
        out: *mut c_float,
    ) -> c_int;
    pub fn ssd_fused_rmsnorm_linear_f32_host(
        ctx: *mut SsdCtx,
        x: *const c_float,
        norm_w: *const c_float,
        out_w: *const c_float,
        vocab: c_int,
        n_embd: c_int,
        logits: *mut c_float,
    ) -> c_int;
    pub fn ssd_feed_forward_f32_host(
        ctx: *mut SsdCtx,
        x: *const c_float,
        w_gate: *const c_float,
        w_up: *const c_float,
        w_down: *const c_float,
        n_embd: c_int,
        n_ff: c_int,
        out: *mut c_float,
    ) -> c_int;

    // ---- decode engine (forward_pass / generate, src/inference/transformer.rs:283-399, :681-770)
    pub fn ssd_model_create(
        ctx: *mut SsdCtx,
        cfg: *const SsdModelConfig,
        out: *mut *mut SsdModel,
    ) -> c_int;
    pub fn ssd_shard_range(
        cfg: *const SsdModelConfig,
        name: *const c_char,
        layer: c_int,
        row0: *mut c_int,
        nrows: *mut c_int,
        col0: *mut c_int,
        ncols: *mut c_int,
    ) -> c_int;
    pub fn ssd_model_free(m: *mut SsdModel) -> c_int;
    pub fn ssd_tp_unique_id(out: *mut u8) -> c_int;
    pub fn ssd_model_tp_init(m: *mut SsdModel, unique_id: *const u8) -> c_int;
    pub fn ssd_model_p2p_handle(m: *mut SsdModel, out: *mut u8) -> c_int;
    pub fn ssd_model_p2p_open(m: *mut SsdModel, handles: *const u8) -> c_int;
    pub fn ssd_model_synth_weights(m: *mut SsdModel, seed: u64, std_dev: c_float) -> c_int;
    pub fn ssd_model_set_tensor(
        m: *mut SsdModel,
        name: *const c_char,
        layer: c_int,
        host_raw: *const c_void,
        bytes: usize,
    ) -> c_int;
    pub fn ssd_model_set_tensor_typed(
        m: *mut SsdModel,
        name: *const c_char,
        layer: c_int,
        host_raw: *const c_void,
        bytes: usize,
        ggml_type: c_int,
    ) -> c_int;
    pub fn ssd_model_synth_kv(m: *mut SsdModel, seed: u64, n: c_int) -> c_int;
    pub fn ssd_model_set_position(m: *mut SsdModel, pos: c_int) -> c_int;
    pub fn ssd_model_get_position(m: *mut SsdModel, pos: *mut c_int) -> c_int;
    pub fn ssd_model_decode_step(m: *mut SsdModel, use_graph: c_int) -> c_int;
    pub fn ssd_model_decode_token(
        m: *mut SsdModel,
        token_in: i32,
        token_out: *mut i32,
        use_graph: c_int,
    ) -> c_int;
    pub fn ssd_model_prefill(
        m: *mut SsdModel,
        tokens: *const i32,
        n: c_int,
        next_token: *mut i32,
    ) -> c_int;
    pub fn ssd_model_state(
        m: *mut SsdModel,
        hidden_dev: *mut *mut c_float,
        logits_dev: *mut *mut c_float,
        token_dev: *mut *mut i32,
    ) -> c_int;
    pub fn ssd_model_weight(
        m: *mut SsdModel,
        name: *const c_char,
        layer: c_int,
        out: *mut *mut SsdWeight,
    ) -> c_int;
    pub fn ssd_model_norm(
        m: *mut SsdModel,
        name: *const c_char,
        layer: c_int,
        out: *mut *mut c_float,
    ) -> c_int;
    pub fn ssd_model_kv(m: *mut SsdModel, layer: c_int, out: *mut *mut SsdKvCache) -> c_int;
    pub fn ssd_model_layer_step(m: *mut SsdModel, layer: c_int) -> c_int;
    pub fn ssd_model_launches_per_step(m: *mut SsdModel, launches: *mut c_int) -> c_int;

    // ---- continuous batch (BatchScheduler, src/inference/batch_scheduler.rs:149-403)
    pub fn ssd_batch_create(m: *mut SsdModel, capacity: c_int, out: *mut *mut SsdBatch) -> c_int;
    pub fn ssd_batch_free(b: *mut SsdBatch) -> c_int;
    pub fn ssd_batch_slots(b: *mut SsdBatch, slots: *mut c_int) -> c_int;
    pub fn ssd_batch_step(
        b: *mut SsdBatch,
        tokens_in: *const i32,
        tokens_out: *mut i32,
        use_graph: c_int,
    ) -> c_int;
    pub fn ssd_batch_set_position(b: *mut SsdBatch, slot: c_int, pos: c_int) -> c_int;
    pub fn ssd_batch_positions(b: *mut SsdBatch, pos: *mut c_int) -> c_int;
    pub fn ssd_batch_synth_kv(b: *mut SsdBatch, seed: u64, n: c_int) -> c_int;
    pub fn ssd_batch_kv_pointers(
        b: *mut SsdBatch,
        layer: c_int,
        slot: c_int,
        k: *mut *mut i8,
        v: *mut *mut i8,
        ks: *mut *mut c_float,
        vs: *mut *mut c_float,
    ) -> c_int;
    pub fn ssd_batch_state(b: *mut SsdBatch, hidden_dev: *mut *mut c_float) -> c_int;
    pub fn ssd_batch_launches_per_step(b: *mut SsdBatch, launches: *mut c_int) -> c_int;

    // ---- GGUF files (src/model/gguf.rs)
    pub fn ssd_gguf_open(path: *const c_char, out: *mut *mut SsdGguf) -> c_int;
    pub fn ssd_gguf_close(g: *mut SsdGguf) -> c_int;
    pub fn ssd_gguf_info(
        g: *const SsdGguf,
        version: *mut u32,
        n_tensors: *mut u64,
        n_kv: *mut u64,
        data_offset: *mut u64,
    ) -> c_int;
    pub fn ssd_gguf_tensor(
        g: *const SsdGguf,
        i: u64,
        name: *mut c_char,
        cap: usize,
        n_dims: *mut u32,
        dims: *mut u64,
        ty: *mut u32,
        offset: *mut u64,
        size_bytes: *mut u64,
    ) -> c_int;
    pub fn ssd_gguf_find(g: *const SsdGguf, name: *const c_char, index: *mut i64) -> c_int;
    pub fn ssd_gguf_get_u32(
        g: *const SsdGguf,
        key: *const c_char,
        found: *mut c_int,
        value: *mut u32,
    ) -> c_int;
    pub fn ssd_gguf_get_f32(
        g: *const SsdGguf,
        key: *const c_char,
        found: *mut c_int,
        value: *mut c_float,
    ) -> c_int;
    pub fn ssd_gguf_get_str(
        g: *const SsdGguf,
        key: *const c_char,
        found: *mut c_int,
        out: *mut c_char,
        cap: usize,
    ) -> c_int;
    pub fn ssd_gguf_array_len(
        g: *const SsdGguf,
        key: *const c_char,
        found: *mut c_int,
        n: *mut u64,
    ) -> c_int;
    pub fn ssd_gguf_read(g: *const SsdGguf, i: u64, dst: *mut c_void, bytes: usize) -> c_int;
    pub fn ssd_gguf_model_config(
        g: *const SsdGguf,
        kv_capacity: c_int,
        tp_rank: c_int,
        tp_size: c_int,
        cfg: *mut SsdModelConfig,
    ) -> c_int;
    pub fn ssd_model_load_gguf(m: *mut SsdModel, g: *const SsdGguf, n_layers: c_int) -> c_int;

    // SSD -> HBM streaming tier (src/ssd/streamer.rs, src/ssd/prefetch.rs, src/model/cache.rs)
    pub fn ssd_stream_open(
        m: *mut SsdModel,
        gguf_path: *const c_char,
        hbm_budget: usize,
        lookahead: c_int,
        out: *mut *mut SsdStream,
    ) -> c_int;
    pub fn ssd_stream_pin(s: *mut SsdStream, layer: c_int) -> c_int;
    pub fn ssd_stream_decode_token(s: *mut SsdStream, token_in: i32, token_out: *mut i32) -> c_int;
    pub fn ssd_stream_stats_get(s: *const SsdStream, out: *mut SsdStreamStats) -> c_int;
    pub fn ssd_stream_close(s: *mut SsdStream) -> c_int;

    pub fn ssd_matvec_independent(
        ctx: *mut SsdCtx,
        w: *const SsdWeight,
        x_dev: *const c_float,
        y_dev: *mut c_float,
        stream: *mut c_void,
    ) -> c_int;
}
