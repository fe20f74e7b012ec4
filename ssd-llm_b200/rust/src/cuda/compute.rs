//! `CudaCompute`: the B200 backend behind `MetalCompute`'s method signatures
//! (src/metal/compute.rs:18-375), plus `MetalGpu::feed_forward_f32` (src/metal/gpu.rs:789-838)
//! and safe handles for the HBM-resident decode engine and continuous batch.
//!
//! Every method keeps the reference's argument meaning and result shape (`Vec<f32>`
//! results, tuples for QKV, `Option` for construction and flash attention). The reference
//! falls back to CPU code or returns silent zeros when the GPU path cannot run
//! (compute.rs:672-675); here a non-zero library status panics with the library's message,
//! so a failure is never mistaken for a result. There is no CPU fallback.
use std::ffi::{CStr, CString};
use std::os::raw::c_int;
use std::ptr;

use super::ffi;
use crate::model::gguf::GgmlType;

fn check(st: c_int) {
    if st != ffi::SSD_OK {
        let msg = unsafe { CStr::from_ptr(ffi::ssd_last_error()) };
        panic!("ssdllm_cuda status {st}: {}", msg.to_string_lossy());
    }
}

/// The GGUF id of a `GgmlType` (src/model/gguf.rs:16-47), the `ggml_type` argument of the
/// C entry points.
pub fn ggml_id(t: GgmlType) -> c_int {
    let id: u32 = match t {
        GgmlType::F32 => 0,
        GgmlType::F16 => 1,
        GgmlType::Q4_0 => 2,
        GgmlType::Q4_1 => 3,
        GgmlType::Q5_0 => 6,
        GgmlType::Q5_1 => 7,
        GgmlType::Q8_0 => 8,
        GgmlType::Q8_1 => 9,
        GgmlType::Q2K => 10,
        GgmlType::Q3K => 11,
        GgmlType::Q4K => 12,
        GgmlType::Q5K => 13,
        GgmlType::Q6K => 14,
        GgmlType::Q8K => 15,
        GgmlType::IQ2XXS => 16,
        GgmlType::IQ2XS => 17,
        GgmlType::IQ3XXS => 18,
        GgmlType::IQ1S => 19,
        GgmlType::IQ4NL => 20,
        GgmlType::IQ3S => 21,
        GgmlType::IQ2S => 22,
        GgmlType::IQ4XS => 23,
        GgmlType::I8 => 24,
        GgmlType::I16 => 25,
        GgmlType::I32 => 26,
        GgmlType::I64 => 27,
        GgmlType::F64 => 28,
        GgmlType::IQ1M => 29,
        GgmlType::BF16 => 30,
        GgmlType::Unknown(v) => v,
    };
    id as c_int
}

/// Compute context (replaces `MetalCompute`). One cached library context per device, so
/// the per-token construction in src/inference/transformer.rs:704 costs nothing.
pub struct CudaCompute {
    ctx: *mut ffi::SsdCtx,
}

unsafe impl Send for CudaCompute {}
unsafe impl Sync for CudaCompute {}

impl CudaCompute {
    /// compute.rs:31-45: whether a CUDA device can be opened.
    pub fn is_available() -> bool {
        let mut ctx = ptr::null_mut();
        unsafe { ffi::ssd_ctx_get(0, &mut ctx) == ffi::SSD_OK }
    }

    /// compute.rs:47-138: a context on device 0, or None when no device is usable.
    pub fn new() -> Option<Self> {
        Self::on_device(0)
    }

    /// A context on `device` (one process per GPU under tensor parallelism).
    pub fn on_device(device: i32) -> Option<Self> {
        let mut ctx = ptr::null_mut();
        (unsafe { ffi::ssd_ctx_get(device, &mut ctx) } == ffi::SSD_OK).then(|| Self { ctx })
    }

    /// compute.rs:140-143. Every call runs on the GPU; there is no size threshold.
    pub fn should_use_gpu(&self, _elements: usize) -> bool {
        true
    }

    /// compute.rs:261-264.
    pub fn has_gpu(&self) -> bool {
        true
    }

    /// compute.rs:266-269: no runtime-compiled shader library (the kernels are sm_100a
    /// code inside libssdllm_cuda.so).
    pub fn shader_library_path(&self) -> Option<&str> {
        None
    }

    /// compute.rs:145-153: y = W x, W row-major [out_dim][in_dim].
    pub fn matvec_f32(&self, w: &[f32], x: &[f32], out_dim: usize, in_dim: usize) -> Vec<f32> {
        assert!(w.len() >= out_dim * in_dim && x.len() >= in_dim);
        let mut y = vec![0.0f32; out_dim];
        check(unsafe {
            ffi::ssd_matvec_f32_host(self.ctx, w.as_ptr(), x.as_ptr(), y.as_mut_ptr(),
                                     out_dim as c_int, in_dim as c_int)
        });
        y
    }

    /// compute.rs:157-191. Q4_0, Q8_0, Q4_K, Q5_K, Q6_K, Q8_K, F16 and BF16 run on the GPU in
    /// the reference's block layouts; other types panic with SSD_ERR_TYPE instead of the
    /// reference's silent zeros.
    pub fn matvec_quantized(&self, w_raw: &[u8], x: &[f32], out_dim: usize, in_dim: usize,
                            dtype: GgmlType) -> Vec<f32> {
        assert!(x.len() >= in_dim);
        let mut y = vec![0.0f32; out_dim];
        check(unsafe {
            ffi::ssd_matvec_quantized_host(self.ctx, w_raw.as_ptr(), w_raw.len(), x.as_ptr(),
                                           y.as_mut_ptr(), out_dim as c_int, in_dim as c_int,
                                           ggml_id(dtype))
        });
        y
    }

    /// compute.rs:193-202 (in place).
    pub fn rmsnorm_f32(&self, x: &mut [f32], weight: &[f32], eps: f32) {
        assert!(weight.len() >= x.len());
        check(unsafe {
            ffi::ssd_rmsnorm_f32_host(self.ctx, x.as_mut_ptr(), weight.as_ptr(),
                                      x.len() as c_int, eps)
        });
    }

    /// compute.rs:204-215 (in place).
    pub fn softmax_f32(&self, x: &mut [f32]) {
        check(unsafe { ffi::ssd_softmax_f32_host(self.ctx, x.as_mut_ptr(), x.len() as c_int) });
    }

    /// compute.rs:217-259: attention of n_head query heads over f32 K/V rows
    /// [seq_len][n_head_kv * head_dim], positions [window_start, min(window_end, seq_len)).
    /// Always Some (the reference returns None without a GPU or below 4 positions).
    #[allow(clippy::too_many_arguments)]
    pub fn flash_attention_f32(&self, q_heads: &[f32], k_cache: &[f32], v_cache: &[f32],
                               n_head: usize, n_head_kv: usize, head_dim: usize,
                               seq_len: usize, window_start: usize,
                               window_end: usize) -> Option<Vec<f32>> {
        assert!(q_heads.len() >= n_head * head_dim);
        assert!(k_cache.len() >= seq_len * n_head_kv * head_dim);
        assert!(v_cache.len() >= seq_len * n_head_kv * head_dim);
        let mut out = vec![0.0f32; n_head * head_dim];
        check(unsafe {
            ffi::ssd_flash_attention_f32_host(self.ctx, q_heads.as_ptr(), k_cache.as_ptr(),
                                              v_cache.as_ptr(), n_head as c_int,
                                              n_head_kv as c_int, head_dim as c_int,
                                              seq_len as c_int, window_start as c_int,
                                              window_end as c_int, out.as_mut_ptr())
        });
        Some(out)
    }

    /// compute.rs:273-292 -> (Q, K, V).
    #[allow(clippy::too_many_arguments)]
    pub fn fused_qkv_f32(&self, wq: &[f32], wk: &[f32], wv: &[f32], x: &[f32], q_dim: usize,
                         kv_dim: usize, n_embd: usize) -> (Vec<f32>, Vec<f32>, Vec<f32>) {
        assert!(wq.len() >= q_dim * n_embd && wk.len() >= kv_dim * n_embd);
        assert!(wv.len() >= kv_dim * n_embd && x.len() >= n_embd);
        let (mut q, mut k, mut v) = (vec![0.0f32; q_dim], vec![0.0f32; kv_dim],
                                     vec![0.0f32; kv_dim]);
        check(unsafe {
            ffi::ssd_fused_qkv_f32_host(self.ctx, wq.as_ptr(), wk.as_ptr(), wv.as_ptr(),
                                        x.as_ptr(), q_dim as c_int, kv_dim as c_int,
                                        n_embd as c_int, q.as_mut_ptr(), k.as_mut_ptr(),
                                        v.as_mut_ptr())
        });
        (q, k, v)
    }

    /// compute.rs:296-323 -> (Q_rope, K_rope, V).
    #[allow(clippy::too_many_arguments)]
    pub fn fused_qkv_rope_f32(&self, wq: &[f32], wk: &[f32], wv: &[f32], x: &[f32],
                              q_dim: usize, kv_dim: usize, n_embd: usize, head_dim: usize,
                              position: usize,
                              theta_base: f32) -> (Vec<f32>, Vec<f32>, Vec<f32>) {
        assert!(wq.len() >= q_dim * n_embd && wk.len() >= kv_dim * n_embd);
        assert!(wv.len() >= kv_dim * n_embd && x.len() >= n_embd);
        let (mut q, mut k, mut v) = (vec![0.0f32; q_dim], vec![0.0f32; kv_dim],
                                     vec![0.0f32; kv_dim]);
        check(unsafe {
            ffi::ssd_fused_qkv_rope_f32_host(self.ctx, wq.as_ptr(), wk.as_ptr(), wv.as_ptr(),
                                             x.as_ptr(), q_dim as c_int, kv_dim as c_int,
                                             n_embd as c_int, head_dim as c_int,
                                             position as c_int, theta_base, q.as_mut_ptr(),
                                             k.as_mut_ptr(), v.as_mut_ptr())
        });
        (q, k, v)
    }

    /// compute.rs:328-343: hidden += attn_output in place; returns rmsnorm(hidden) * weight.
    pub fn fused_post_attn_norm_f32(&self, hidden: &mut [f32], attn_output: &[f32],
                                    norm_weight: &[f32], eps: f32) -> Vec<f32> {
        assert!(attn_output.len() >= hidden.len() && norm_weight.len() >= hidden.len());
        let mut out = vec![0.0f32; hidden.len()];
        check(unsafe {
            ffi::ssd_fused_post_attn_norm_f32_host(self.ctx, hidden.as_mut_ptr(),
                                                   attn_output.as_ptr(), norm_weight.as_ptr(),
                                                   hidden.len() as c_int, eps,
                                                   out.as_mut_ptr())
        });
        out
    }

    /// compute.rs:348-374: logits = W_out (x * inv_rms * norm_weight), eps 1e-5.
    pub fn fused_rmsnorm_linear_f32(&self, x: &[f32], norm_weight: &[f32], out_weight: &[f32],
                                    vocab_size: usize, n_embd: usize) -> Vec<f32> {
        assert!(x.len() >= n_embd && norm_weight.len() >= n_embd);
        assert!(out_weight.len() >= vocab_size * n_embd);
        let mut logits = vec![0.0f32; vocab_size];
        check(unsafe {
            ffi::ssd_fused_rmsnorm_linear_f32_host(self.ctx, x.as_ptr(), norm_weight.as_ptr(),
                                                   out_weight.as_ptr(), vocab_size as c_int,
                                                   n_embd as c_int, logits.as_mut_ptr())
        });
        logits
    }

    /// MetalGpu::feed_forward_f32 (gpu.rs:789-838): W_down (silu(W_gate x) * (W_up x)),
    /// n_ff = w_gate.len() / n_embd (zeros when that is 0, feed_forward.rs:25-28).
    pub fn feed_forward_f32(&self, x: &[f32], w_gate: &[f32], w_up: &[f32], w_down: &[f32],
                            n_embd: usize) -> Vec<f32> {
        let n_ff = w_gate.len() / n_embd;
        assert!(w_up.len() >= n_ff * n_embd && w_down.len() >= n_embd * n_ff);
        let mut out = vec![0.0f32; n_embd];
        check(unsafe {
            ffi::ssd_feed_forward_f32_host(self.ctx, x.as_ptr(), w_gate.as_ptr(), w_up.as_ptr(),
                                           w_down.as_ptr(), n_embd as c_int, n_ff as c_int,
                                           out.as_mut_ptr())
        });
        out
    }

    /// The raw context, for the device-pointer entry points of `ffi`.
    pub fn raw(&self) -> *mut ffi::SsdCtx {
        self.ctx
    }
}

/// The HBM-resident decode engine: `forward_pass` and `generate`'s token loop
/// (src/inference/transformer.rs:283-399, :681-770) with the weights uploaded once from the
/// GGUF file (instead of SsdStreamer::load_layer's per-token dequantization,
/// src/ssd/streamer.rs:34-66) and an INT8 KV cache per layer.
pub struct CudaModel {
    m: *mut ffi::SsdModel,
}

unsafe impl Send for CudaModel {}

impl CudaModel {
    /// Opens `path`, derives the config (kv_capacity positions; rank `tp_rank` of
    /// `tp_size`) and uploads `n_layers` layers (all when negative).
    pub fn from_gguf(cc: &CudaCompute, path: &str, kv_capacity: i32, n_layers: i32) -> Self {
        let p = CString::new(path).expect("path");
        let mut g = ptr::null_mut();
        check(unsafe { ffi::ssd_gguf_open(p.as_ptr(), &mut g) });
        let mut cfg = ffi::SsdModelConfig::default();
        check(unsafe { ffi::ssd_gguf_model_config(g, kv_capacity, 0, 1, &mut cfg) });
        let mut m = ptr::null_mut();
        check(unsafe { ffi::ssd_model_create(cc.raw(), &cfg, &mut m) });
        let st = unsafe { ffi::ssd_model_load_gguf(m, g, n_layers) };
        unsafe { ffi::ssd_gguf_close(g) };
        check(st);
        Self { m }
    }

    /// Prompt prefill (batch_prefill, transformer.rs:120-250): every prompt token through
    /// every layer, KV cached; returns the greedy next token.
    pub fn prefill(&mut self, tokens: &[i32]) -> i32 {
        let mut next = 0i32;
        check(unsafe {
            ffi::ssd_model_prefill(self.m, tokens.as_ptr(), tokens.len() as c_int, &mut next)
        });
        next
    }

    /// One greedy decode step (generate's loop body, transformer.rs:681-770); the step runs
    /// as one CUDA graph replay when `use_graph`.
    pub fn decode_token(&mut self, token: i32, use_graph: bool) -> i32 {
        let mut out = 0i32;
        check(unsafe { ffi::ssd_model_decode_token(self.m, token, &mut out, use_graph as c_int) });
        out
    }

    pub fn position(&self) -> i32 {
        let mut p = 0;
        check(unsafe { ffi::ssd_model_get_position(self.m, &mut p) });
        p
    }

    pub fn raw(&self) -> *mut ffi::SsdModel {
        self.m
    }
}

impl Drop for CudaModel {
    fn drop(&mut self) {
        unsafe { ffi::ssd_model_free(self.m) };
    }
}

/// SSD -> HBM streaming tier (SsdStreamer + Prefetcher + LayerCache, src/ssd/streamer.rs,
/// src/ssd/prefetch.rs, src/model/cache.rs): a model whose layer matrices stay in the GGUF
/// file and pass through `hbm_budget` bytes of HBM layer slots, `lookahead` layers ahead.
pub struct CudaStream {
    s: *mut ffi::SsdStream,
    _model: CudaModel,
}

unsafe impl Send for CudaStream {}

impl CudaStream {
    pub fn open(cc: &CudaCompute, path: &str, kv_capacity: i32, hbm_budget: usize,
                lookahead: i32) -> Self {
        let p = CString::new(path).expect("path");
        let mut g = ptr::null_mut();
        check(unsafe { ffi::ssd_gguf_open(p.as_ptr(), &mut g) });
        let mut cfg = ffi::SsdModelConfig::default();
        let st = unsafe { ffi::ssd_gguf_model_config(g, kv_capacity, 0, 1, &mut cfg) };
        unsafe { ffi::ssd_gguf_close(g) };
        check(st);
        let mut m = ptr::null_mut();
        check(unsafe { ffi::ssd_model_create(cc.raw(), &cfg, &mut m) });
        let model = CudaModel { m };
        let mut s = ptr::null_mut();
        check(unsafe { ffi::ssd_stream_open(m, p.as_ptr(), hbm_budget, lookahead, &mut s) });
        Self { s, _model: model }
    }

    /// LayerCache::pin: the layer stays in HBM.
    pub fn pin(&mut self, layer: i32) {
        check(unsafe { ffi::ssd_stream_pin(self.s, layer) });
    }

    /// One greedy decode step with streamed layers.
    pub fn decode_token(&mut self, token: i32) -> i32 {
        let mut out = 0i32;
        check(unsafe { ffi::ssd_stream_decode_token(self.s, token, &mut out) });
        out
    }

    pub fn stats(&self) -> ffi::SsdStreamStats {
        let mut st = ffi::SsdStreamStats::default();
        check(unsafe { ffi::ssd_stream_stats_get(self.s, &mut st) });
        st
    }
}

impl Drop for CudaStream {
    fn drop(&mut self) {
        unsafe { ffi::ssd_stream_close(self.s) };
    }
}

/// Continuous batch (BatchScheduler::step, src/inference/batch_scheduler.rs:149-403): up
/// to `capacity` sequences decode together, each weight byte streamed once per step for all
/// of them; a slot joins by setting its position and leaves by being ignored.
pub struct CudaBatch {
    b: *mut ffi::SsdBatch,
}

impl CudaBatch {
    pub fn new(model: &CudaModel, capacity: i32) -> Self {
        let mut b = ptr::null_mut();
        check(unsafe { ffi::ssd_batch_create(model.raw(), capacity, &mut b) });
        Self { b }
    }

    /// One decode step of every slot: tokens_in[slot] -> returned greedy tokens.
    pub fn step(&mut self, tokens_in: &[i32], use_graph: bool) -> Vec<i32> {
        let mut n = 0;
        check(unsafe { ffi::ssd_batch_slots(self.b, &mut n) });
        assert!(tokens_in.len() >= n as usize);
        let mut out = vec![0i32; n as usize];
        check(unsafe {
            ffi::ssd_batch_step(self.b, tokens_in.as_ptr(), out.as_mut_ptr(), use_graph as c_int)
        });
        out
    }

    /// A request joins slot `slot` at position `pos` (0 for a fresh sequence).
    pub fn set_position(&mut self, slot: i32, pos: i32) {
        check(unsafe { ffi::ssd_batch_set_position(self.b, slot, pos) });
    }
}

impl Drop for CudaBatch {
    fn drop(&mut self) {
        unsafe { ffi::ssd_batch_free(self.b) };
    }
}
