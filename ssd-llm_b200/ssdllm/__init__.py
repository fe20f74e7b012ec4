"""Python binding of the sm_100a backend (ctypes over include/ssdllm_cuda.h).

`CudaCompute` mirrors the operator surface of ssd-llm's `MetalCompute`
(src/metal/compute.rs:18-373): same method names and argument meaning, host
slices in, host results out. The device-pointer functions (`matvec`, `kv_append`,
`attention_int8`, ...) take torch CUDA tensors and run on torch's current stream.
Everything runs through libssdllm_cuda.so; there is no CPU fallback: if the
library or a GPU is missing, loading fails with an error.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(HERE, "libssdllm_cuda.so")

F32, F16, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K, Q8_K, BF16 = 0, 1, 2, 8, 12, 13, 14, 15, 30
BLOCK = {Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210),
         Q8_K: (256, 292), F16: (1, 2), BF16: (1, 2), F32: (1, 4)}
STATUS = {0: "ok", 1: "invalid argument", 2: "unsupported ggml type", 3: "shape mismatch",
          4: "CUDA error", 5: "device wait timed out", 6: "NCCL error",
          7: "out of device memory", 8: "invalid state"}

_lib = None
_vp = ctypes.c_void_p


class SsdError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status


class ModelConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "n_layers", "n_embd", "n_head", "n_head_kv", "head_dim", "n_ff", "vocab", "wtype",
        "out_type", "embd_type", "kv_capacity")] + [
        ("theta", ctypes.c_float), ("eps", ctypes.c_float), ("tp_rank", ctypes.c_int),
        ("tp_size", ctypes.c_int)]


class StreamStats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in (
        "hits", "misses", "evictions", "prefetch_hits", "loads", "bytes_read")] + [
        ("n_slots", ctypes.c_int), ("slot_bytes", ctypes.c_size_t)]


_u32p = ctypes.POINTER(ctypes.c_uint32)
_u64p = ctypes.POINTER(ctypes.c_uint64)
_ip = ctypes.POINTER(ctypes.c_int)

# name -> (argtypes, restype); the set is checked against include/ssdllm_cuda.h by tests
_SIGS = {
    "ssd_abi_version": ([], ctypes.c_int),
    "ssd_status_str": ([ctypes.c_int], ctypes.c_char_p),
    "ssd_last_error": ([], ctypes.c_char_p),
    "ssd_ctx_create": ([ctypes.c_int, ctypes.POINTER(_vp)], ctypes.c_int),
    "ssd_ctx_get": ([ctypes.c_int, ctypes.POINTER(_vp)], ctypes.c_int),
    "ssd_ctx_destroy": ([_vp], ctypes.c_int),
    "ssd_ctx_stream": ([_vp, ctypes.POINTER(_vp)], ctypes.c_int),
    "ssd_ctx_sync": ([_vp], ctypes.c_int),
    "ssd_ctx_info": ([_vp, ctypes.POINTER(ctypes.c_int), ctypes.c_char_p, ctypes.c_size_t],
                     ctypes.c_int),
    "ssd_ctx_set_pdl": ([_vp, ctypes.c_int], ctypes.c_int),
    "ssd_ctx_device_status": ([_vp, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "ssd_copy_to_device": ([_vp, _vp, _vp, ctypes.c_size_t], ctypes.c_int),
    "ssd_copy_to_host": ([_vp, _vp, _vp, ctypes.c_size_t], ctypes.c_int),
    "ssd_weight_upload": ([_vp, _vp, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                           ctypes.POINTER(_vp)], ctypes.c_int),
    "ssd_weight_upload_device": ([_vp, _vp, ctypes.c_size_t, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_int, ctypes.POINTER(_vp), _vp], ctypes.c_int),
    "ssd_weight_download": ([_vp, _vp, _vp, ctypes.c_size_t], ctypes.c_int),
    "ssd_weight_free": ([_vp], ctypes.c_int),
    "ssd_weight_info": ([_vp, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                         ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_size_t)],
                        ctypes.c_int),
    "ssd_row_bytes": ([ctypes.c_int, ctypes.c_int64], ctypes.c_size_t),
    "ssd_weight_synth": ([_vp, ctypes.c_int, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_float,
                          ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                          ctypes.POINTER(_vp), _vp], ctypes.c_int),
    "ssd_synth_f32": ([_vp, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_float, ctypes.c_float,
                       ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                       _vp, _vp], ctypes.c_int),
    "ssd_quantize": ([_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _vp],
                     ctypes.c_int),
    "ssd_dequantize": ([_vp, _vp, _vp, _vp], ctypes.c_int),
    "ssd_matvec": ([_vp, _vp, _vp, _vp, _vp], ctypes.c_int),
    "ssd_matvec_independent": ([_vp, _vp, _vp, _vp, _vp], ctypes.c_int),
    "ssd_matvec_residual": ([_vp, _vp, _vp, _vp, _vp, _vp], ctypes.c_int),
    "ssd_fused_rmsnorm_matvec": ([_vp, _vp, _vp, _vp, ctypes.c_float, _vp, _vp], ctypes.c_int),
    "ssd_fused_qkv_rope": ([_vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_float, ctypes.c_int,
                            ctypes.c_int, ctypes.c_float, _vp, _vp, _vp, _vp], ctypes.c_int),
    "ssd_fused_swiglu": ([_vp, _vp, _vp, _vp, _vp, ctypes.c_float, _vp, _vp], ctypes.c_int),
    "ssd_rmsnorm": ([_vp, _vp, _vp, ctypes.c_int, ctypes.c_float, _vp], ctypes.c_int),
    "ssd_fused_post_attn_norm": ([_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_float, _vp, _vp],
                                 ctypes.c_int),
    "ssd_softmax": ([_vp, _vp, ctypes.c_int, _vp], ctypes.c_int),
    "ssd_rope": ([_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                  ctypes.c_float, _vp], ctypes.c_int),
    "ssd_silu": ([_vp, _vp, ctypes.c_int, _vp], ctypes.c_int),
    "ssd_argmax": ([_vp, _vp, ctypes.c_int, _vp, _vp], ctypes.c_int),
    "ssd_kv_create": ([_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_vp)],
                      ctypes.c_int),
    "ssd_kv_free": ([_vp], ctypes.c_int),
    "ssd_kv_pointers": ([_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.POINTER(_vp),
                         ctypes.POINTER(_vp)], ctypes.c_int),
    "ssd_kv_append": ([_vp, _vp, _vp, _vp, ctypes.c_int, _vp], ctypes.c_int),
    "ssd_kv_append_rows": ([_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp], ctypes.c_int),
    "ssd_attention_int8": ([_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp, _vp], ctypes.c_int),
    "ssd_attention_int8_noalloc": ([_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp, _vp],
                                   ctypes.c_int),
    "ssd_prefill_matmul": ([_vp, _vp, _vp, ctypes.c_int, _vp, _vp], ctypes.c_int),
    "ssd_matvec_quantized_host": ([_vp, _vp, ctypes.c_size_t, _vp, _vp, ctypes.c_int,
                                   ctypes.c_int, ctypes.c_int], ctypes.c_int),
    "ssd_model_create": ([_vp, ctypes.POINTER(ModelConfig), ctypes.POINTER(_vp)], ctypes.c_int),
    "ssd_model_free": ([_vp], ctypes.c_int),
    "ssd_shard_range": ([ctypes.POINTER(ModelConfig), ctypes.c_char_p, ctypes.c_int,
                         ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                         ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)],
                        ctypes.c_int),
    "ssd_tp_unique_id": ([ctypes.c_char_p], ctypes.c_int),
    "ssd_model_tp_init": ([_vp, ctypes.c_char_p], ctypes.c_int),
    "ssd_model_synth_weights": ([_vp, ctypes.c_uint64, ctypes.c_float], ctypes.c_int),
    "ssd_model_set_tensor": ([_vp, ctypes.c_char_p, ctypes.c_int, _vp, ctypes.c_size_t],
                             ctypes.c_int),
    "ssd_model_set_tensor_typed": ([_vp, ctypes.c_char_p, ctypes.c_int, _vp, ctypes.c_size_t,
                                    ctypes.c_int], ctypes.c_int),
    "ssd_model_synth_kv": ([_vp, ctypes.c_uint64, ctypes.c_int], ctypes.c_int),
    "ssd_model_set_position": ([_vp, ctypes.c_int], ctypes.c_int),
    "ssd_model_get_position": ([_vp, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "ssd_model_decode_step": ([_vp, ctypes.c_int], ctypes.c_int),
    "ssd_model_decode_token": ([_vp, ctypes.c_int32, ctypes.POINTER(ctypes.c_int32),
                                ctypes.c_int], ctypes.c_int),
    "ssd_model_state": ([_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.POINTER(_vp)],
                        ctypes.c_int),
    "ssd_model_weight": ([_vp, ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(_vp)],
                         ctypes.c_int),
    "ssd_model_norm": ([_vp, ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(_vp)], ctypes.c_int),
    "ssd_model_kv": ([_vp, ctypes.c_int, ctypes.POINTER(_vp)], ctypes.c_int),
    "ssd_model_layer_step": ([_vp, ctypes.c_int], ctypes.c_int),
    "ssd_model_p2p_handle": ([_vp, ctypes.c_char_p], ctypes.c_int),
    "ssd_model_prefill": ([_vp, _vp, ctypes.c_int, ctypes.POINTER(ctypes.c_int32)], ctypes.c_int),
    "ssd_model_p2p_open": ([_vp, ctypes.c_char_p], ctypes.c_int),
    "ssd_model_launches_per_step": ([_vp, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "ssd_attention_prefill": ([_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                               ctypes.c_int, _vp, ctypes.c_int, _vp], ctypes.c_int),
    "ssd_gguf_open": ([ctypes.c_char_p, ctypes.POINTER(_vp)], ctypes.c_int),
    "ssd_gguf_close": ([_vp], ctypes.c_int),
    "ssd_gguf_info": ([_vp, _u32p, _u64p, _u64p, _u64p], ctypes.c_int),
    "ssd_gguf_tensor": ([_vp, ctypes.c_uint64, ctypes.c_char_p, ctypes.c_size_t, _u32p, _u64p,
                         _u32p, _u64p, _u64p], ctypes.c_int),
    "ssd_gguf_find": ([_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64)], ctypes.c_int),
    "ssd_gguf_get_u32": ([_vp, ctypes.c_char_p, _ip, _u32p], ctypes.c_int),
    "ssd_gguf_get_f32": ([_vp, ctypes.c_char_p, _ip, ctypes.POINTER(ctypes.c_float)],
                         ctypes.c_int),
    "ssd_gguf_get_str": ([_vp, ctypes.c_char_p, _ip, ctypes.c_char_p, ctypes.c_size_t],
                         ctypes.c_int),
    "ssd_gguf_array_len": ([_vp, ctypes.c_char_p, _ip, _u64p], ctypes.c_int),
    "ssd_gguf_read": ([_vp, ctypes.c_uint64, _vp, ctypes.c_size_t], ctypes.c_int),
    "ssd_gguf_model_config": ([_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                               ctypes.POINTER(ModelConfig)], ctypes.c_int),
    "ssd_model_load_gguf": ([_vp, _vp, ctypes.c_int], ctypes.c_int),
    "ssd_stream_open": ([_vp, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_int,
                         ctypes.POINTER(_vp)], ctypes.c_int),
    "ssd_stream_pin": ([_vp, ctypes.c_int], ctypes.c_int),
    "ssd_stream_decode_token": ([_vp, ctypes.c_int32, ctypes.POINTER(ctypes.c_int32)],
                                ctypes.c_int),
    "ssd_stream_stats_get": ([_vp, ctypes.POINTER(StreamStats)], ctypes.c_int),
    "ssd_stream_close": ([_vp], ctypes.c_int),
    "ssd_matvec_peer_input": ([_vp, _vp, _vp, _vp, ctypes.c_int, _vp, _vp, ctypes.c_int, _vp,
                               _vp], ctypes.c_int),
    "ssd_batch_create": ([_vp, ctypes.c_int, ctypes.POINTER(_vp)], ctypes.c_int),
    "ssd_batch_free": ([_vp], ctypes.c_int),
    "ssd_batch_slots": ([_vp, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "ssd_batch_step": ([_vp, _vp, _vp, ctypes.c_int], ctypes.c_int),
    "ssd_batch_set_position": ([_vp, ctypes.c_int, ctypes.c_int], ctypes.c_int),
    "ssd_batch_positions": ([_vp, _vp], ctypes.c_int),
    "ssd_batch_synth_kv": ([_vp, ctypes.c_uint64, ctypes.c_int], ctypes.c_int),
    "ssd_batch_kv_pointers": ([_vp, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_vp),
                               ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.POINTER(_vp)],
                              ctypes.c_int),
    "ssd_batch_state": ([_vp, ctypes.POINTER(_vp)], ctypes.c_int),
    "ssd_batch_launches_per_step": ([_vp, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "ssd_matvec_f32_host": ([_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int], ctypes.c_int),
    "ssd_rmsnorm_f32_host": ([_vp, _vp, _vp, ctypes.c_int, ctypes.c_float], ctypes.c_int),
    "ssd_softmax_f32_host": ([_vp, _vp, ctypes.c_int], ctypes.c_int),
    "ssd_flash_attention_f32_host": ([_vp, _vp, _vp, _vp] + [ctypes.c_int] * 6 + [_vp],
                                     ctypes.c_int),
    "ssd_flash_attention_f32": ([_vp, _vp, _vp, _vp] + [ctypes.c_int] * 6 + [_vp, _vp],
                                ctypes.c_int),
    "ssd_fused_qkv_f32_host": ([_vp, _vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int,
                                ctypes.c_int, _vp, _vp, _vp], ctypes.c_int),
    "ssd_fused_qkv_rope_f32_host": ([_vp, _vp, _vp, _vp, _vp] + [ctypes.c_int] * 5 +
                                    [ctypes.c_float, _vp, _vp, _vp], ctypes.c_int),
    "ssd_fused_post_attn_norm_f32_host": ([_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_float,
                                           _vp], ctypes.c_int),
    "ssd_fused_rmsnorm_linear_f32_host": ([_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp],
                                          ctypes.c_int),
    "ssd_feed_forward_f32_host": ([_vp, _vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp],
                                  ctypes.c_int),
}


def lib():
    """Loads libssdllm_cuda.so (raises if it is missing: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} missing: build it with ssd-llm_b200/build.py")
        try:  # torch first, so its libnccl.so.2 is the one both libraries use
            import torch  # noqa: F401
        except ImportError:
            pass
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(status: int):
    if status != 0:
        raise SsdError(status, lib().ssd_last_error().decode(errors="replace"))


def _ptr(t) -> int:
    if t is None:
        return None
    return t.data_ptr()


def _stream():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def row_bytes(wtype: int, cols: int) -> int:
    return int(lib().ssd_row_bytes(wtype, cols))


class Context:
    """A device context (MetalCompute::new / MetalGpu::new)."""

    def __init__(self, device: int = 0, cached: bool = True):
        h = _vp()
        check((lib().ssd_ctx_get if cached else lib().ssd_ctx_create)(device, ctypes.byref(h)))
        self.h = h
        self.device = device
        self.cached = cached

    def sync(self):
        check(lib().ssd_ctx_sync(self.h))

    def device_status(self) -> int:
        st = ctypes.c_int()
        check(lib().ssd_ctx_device_status(self.h, ctypes.byref(st)))
        return st.value

    def set_pdl(self, on: bool):
        check(lib().ssd_ctx_set_pdl(self.h, int(on)))

    def info(self):
        n = ctypes.c_int()
        buf = ctypes.create_string_buffer(256)
        check(lib().ssd_ctx_info(self.h, ctypes.byref(n), buf, 256))
        return n.value, buf.value.decode()

    def close(self):
        if self.h and not self.cached:
            lib().ssd_ctx_destroy(self.h)
        self.h = None


class Weight:
    """HBM-resident quantized tensor (reference block layout in, library layout inside)."""

    def __init__(self, ctx: Context, handle, wtype: int, rows: int, cols: int):
        self.ctx, self.h, self.type, self.rows, self.cols = ctx, handle, wtype, rows, cols

    @classmethod
    def upload(cls, ctx: Context, raw: np.ndarray, wtype: int, rows: int, cols: int):
        raw = np.ascontiguousarray(raw, dtype=np.uint8)
        h = _vp()
        check(lib().ssd_weight_upload(ctx.h, raw.ctypes.data, raw.nbytes, wtype, rows, cols,
                                      ctypes.byref(h)))
        return cls(ctx, h, wtype, rows, cols)

    @classmethod
    def upload_device(cls, ctx: Context, raw_dev, wtype: int, rows: int, cols: int):
        h = _vp()
        check(lib().ssd_weight_upload_device(ctx.h, _ptr(raw_dev), raw_dev.numel(), wtype, rows,
                                             cols, ctypes.byref(h), _stream()))
        return cls(ctx, h, wtype, rows, cols)

    @classmethod
    def synth(cls, ctx: Context, wtype: int, seed: int, tensor_id: int, std: float,
              total_cols: int, row0: int, rows: int, col0: int, cols: int):
        h = _vp()
        check(lib().ssd_weight_synth(ctx.h, wtype, seed, tensor_id, std, total_cols, row0, rows,
                                     col0, cols, ctypes.byref(h), _stream()))
        return cls(ctx, h, wtype, rows, cols)

    def raw_bytes(self) -> int:
        return row_bytes(self.type, self.cols) * self.rows

    def download(self) -> np.ndarray:
        out = np.zeros(self.raw_bytes(), dtype=np.uint8)
        check(lib().ssd_weight_download(self.ctx.h, self.h, out.ctypes.data, out.nbytes))
        return out

    def free(self):
        if self.h and not getattr(self, "borrowed", False):
            lib().ssd_weight_free(self.h)
        self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


# ------------------------------------------------------- device-pointer ops
def matvec(ctx, w: Weight, x, y):
    check(lib().ssd_matvec(ctx.h, w.h, _ptr(x), _ptr(y), _stream()))


def matvec_independent(ctx, w: Weight, x, y):
    """ssd_matvec for matvecs that do not feed each other: x is not written and y is not
    touched by any kernel enqueued before it, so consecutive launches overlap."""
    check(lib().ssd_matvec_independent(ctx.h, w.h, _ptr(x), _ptr(y), _stream()))


def prefill_matmul(ctx, w: Weight, x, y):
    """y[t] = W x[t] for every row t of x (torch [n_tokens][cols] -> [n_tokens][rows])."""
    check(lib().ssd_prefill_matmul(ctx.h, w.h, _ptr(x), x.shape[0], _ptr(y), _stream()))


def matvec_peer_input(ctx, w: Weight, x, partials, n_ranks, flags, epoch, call, y):
    """y = W (x + the n_ranks partial rows), after every rank's flag reaches epoch + call + 1."""
    check(lib().ssd_matvec_peer_input(ctx.h, w.h, _ptr(x), _ptr(partials), n_ranks, _ptr(flags),
                                      _ptr(epoch), call, _ptr(y), _stream()))


def matvec_residual(ctx, w: Weight, x, base, y):
    check(lib().ssd_matvec_residual(ctx.h, w.h, _ptr(x), _ptr(base), _ptr(y), _stream()))


def fused_rmsnorm_matvec(ctx, w: Weight, x, norm_w, eps, y):
    check(lib().ssd_fused_rmsnorm_matvec(ctx.h, w.h, _ptr(x), _ptr(norm_w), eps, _ptr(y),
                                         _stream()))


def fused_qkv_rope(ctx, wq, wk, wv, x, norm_w, eps, head_dim, position, theta, q, k, v):
    check(lib().ssd_fused_qkv_rope(ctx.h, wq.h, wk.h, wv.h, _ptr(x), _ptr(norm_w), eps, head_dim,
                                   position, theta, _ptr(q), _ptr(k), _ptr(v), _stream()))


def fused_swiglu(ctx, wg, wu, x, norm_w, eps, act):
    check(lib().ssd_fused_swiglu(ctx.h, wg.h, wu.h, _ptr(x), _ptr(norm_w), eps, _ptr(act),
                                 _stream()))


def quantize(ctx, x, wtype, raw_out):
    rows, cols = x.shape
    check(lib().ssd_quantize(ctx.h, _ptr(x), rows, cols, wtype, _ptr(raw_out), _stream()))


def dequantize(ctx, w: Weight, out):
    check(lib().ssd_dequantize(ctx.h, w.h, _ptr(out), _stream()))


def synth_f32(ctx, seed, tensor_id, mean, std, total_cols, row0, rows, col0, cols, out):
    check(lib().ssd_synth_f32(ctx.h, seed, tensor_id, mean, std, total_cols, row0, rows, col0,
                              cols, _ptr(out), _stream()))


def rmsnorm(ctx, x, w, eps=1e-5):
    check(lib().ssd_rmsnorm(ctx.h, _ptr(x), _ptr(w), x.numel(), eps, _stream()))


def fused_post_attn_norm(ctx, h, a, w, eps, out):
    check(lib().ssd_fused_post_attn_norm(ctx.h, _ptr(h), _ptr(a), _ptr(w), h.numel(), eps,
                                         _ptr(out), _stream()))


def softmax(ctx, x):
    check(lib().ssd_softmax(ctx.h, _ptr(x), x.numel(), _stream()))


def rope(ctx, x, head_dim, n_heads, position, theta):
    check(lib().ssd_rope(ctx.h, _ptr(x), x.numel(), head_dim, n_heads, position, theta,
                         _stream()))


def silu(ctx, x):
    check(lib().ssd_silu(ctx.h, _ptr(x), x.numel(), _stream()))


def argmax(ctx, v, idx):
    check(lib().ssd_argmax(ctx.h, _ptr(v), v.numel(), _ptr(idx), _stream()))


class KvCache:
    """Device INT8 KV cache of one layer (QuantizedLayerKvCache)."""

    def __init__(self, ctx: Context, capacity: int, n_head_kv: int, head_dim: int):
        h = _vp()
        check(lib().ssd_kv_create(ctx.h, capacity, n_head_kv, head_dim, ctypes.byref(h)))
        self.ctx, self.h = ctx, h
        self.capacity, self.n_head_kv, self.head_dim = capacity, n_head_kv, head_dim

    def pointers(self):
        k, v, ks, vs = _vp(), _vp(), _vp(), _vp()
        check(lib().ssd_kv_pointers(self.h, ctypes.byref(k), ctypes.byref(v), ctypes.byref(ks),
                                    ctypes.byref(vs)))
        return k.value, v.value, ks.value, vs.value

    def append(self, k, v, position: int):
        check(lib().ssd_kv_append(self.ctx.h, self.h, _ptr(k), _ptr(v), position, _stream()))

    def append_rows(self, k, v, position: int):
        check(lib().ssd_kv_append_rows(self.ctx.h, self.h, _ptr(k), _ptr(v), position,
                                       k.shape[0], _stream()))

    def attention(self, q, n_head: int, seq_len: int, out):
        check(lib().ssd_attention_int8(self.ctx.h, self.h, _ptr(q), n_head, seq_len, _ptr(out),
                                       _stream()))

    def attention_prefill(self, q, n_head: int, pos0: int, out):
        """Causal attention of the rows of q (n_q x n_head*head_dim) at positions pos0..
        over this cache (their K/V rows already appended)."""
        n_q = q.shape[0]
        check(lib().ssd_attention_prefill(self.ctx.h, self.h, _ptr(q), n_q, q.shape[1], pos0,
                                          n_head, _ptr(out), out.shape[1], _stream()))

    def attention_noalloc(self, q, n_head: int, seq_len: int, out):
        """ssd_attention_int8 with the partials in the library's fixed device array
        (no device allocation; see include/ssdllm_cuda.h for the limit)."""
        check(lib().ssd_attention_int8_noalloc(self.ctx.h, self.h, _ptr(q), n_head, seq_len,
                                               _ptr(out), _stream()))

    def free(self):
        if self.h:
            lib().ssd_kv_free(self.h)
            self.h = None


class Stream:
    """SSD -> HBM streaming tier over a Model whose layer matrices stay in a GGUF file
    (SsdStreamer + Prefetcher(LookAhead) + LayerCache, src/ssd/streamer.rs:34-80,
    src/ssd/prefetch.rs:24-67, src/model/cache.rs): hbm_budget bytes of layer slots."""

    def __init__(self, model, path: str, hbm_budget: int, lookahead: int = 1):
        self.h = None
        h = _vp()
        check(lib().ssd_stream_open(model.h, os.fsencode(path), hbm_budget, lookahead,
                                    ctypes.byref(h)))
        self.h, self.model = h, model

    def pin(self, layer: int):
        check(lib().ssd_stream_pin(self.h, layer))

    def decode_token(self, token: int) -> int:
        out = ctypes.c_int32()
        check(lib().ssd_stream_decode_token(self.h, token, ctypes.byref(out)))
        return out.value

    def stats(self) -> dict:
        st = StreamStats()
        check(lib().ssd_stream_stats_get(self.h, ctypes.byref(st)))
        return {n: getattr(st, n) for n, _ in StreamStats._fields_}

    def close(self):
        if self.h:
            check(lib().ssd_stream_close(self.h))
            self.h = None


class GgufFile:
    """A parsed GGUF file (GgufFile, src/model/gguf.rs:224-441): header fields, tensor
    infos and metadata lookups, read through the C ABI (host only, no GPU needed)."""

    def __init__(self, path: str):
        self.h = None
        h = _vp()
        check(lib().ssd_gguf_open(os.fsencode(path), ctypes.byref(h)))
        self.h, self.path = h, path
        v, nt, nk, off = ctypes.c_uint32(), ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        check(lib().ssd_gguf_info(h, ctypes.byref(v), ctypes.byref(nt), ctypes.byref(nk),
                                  ctypes.byref(off)))
        self.version, self.n_tensors, self.n_kv = v.value, nt.value, nk.value
        self.data_offset = off.value
        self.tensors = [self._tensor(i) for i in range(self.n_tensors)]

    def _tensor(self, i):
        name = ctypes.create_string_buffer(4096)
        nd, ty = ctypes.c_uint32(), ctypes.c_uint32()
        off, size = ctypes.c_uint64(), ctypes.c_uint64()
        dims = (ctypes.c_uint64 * 8)()
        check(lib().ssd_gguf_tensor(self.h, i, name, 4096, ctypes.byref(nd), dims,
                                    ctypes.byref(ty), ctypes.byref(off), ctypes.byref(size)))
        return {"name": name.value.decode(), "dims": [dims[d] for d in range(nd.value)],
                "type": ty.value, "offset": off.value, "size": size.value}

    def find_tensor(self, name: str):
        idx = ctypes.c_int64()
        check(lib().ssd_gguf_find(self.h, name.encode(), ctypes.byref(idx)))
        return None if idx.value < 0 else self.tensors[idx.value]

    def get_u32(self, key: str):
        f, v = ctypes.c_int(), ctypes.c_uint32()
        check(lib().ssd_gguf_get_u32(self.h, key.encode(), ctypes.byref(f), ctypes.byref(v)))
        return v.value if f.value else None

    def get_f32(self, key: str):
        f, v = ctypes.c_int(), ctypes.c_float()
        check(lib().ssd_gguf_get_f32(self.h, key.encode(), ctypes.byref(f), ctypes.byref(v)))
        return v.value if f.value else None

    def get_str(self, key: str):
        f, buf = ctypes.c_int(), ctypes.create_string_buffer(65536)
        check(lib().ssd_gguf_get_str(self.h, key.encode(), ctypes.byref(f), buf, 65536))
        return buf.value.decode() if f.value else None

    def array_len(self, key: str):
        f, n = ctypes.c_int(), ctypes.c_uint64()
        check(lib().ssd_gguf_array_len(self.h, key.encode(), ctypes.byref(f), ctypes.byref(n)))
        return n.value if f.value else None

    def read(self, name: str) -> np.ndarray:
        """Raw bytes of a tensor in its block format."""
        idx = ctypes.c_int64()
        check(lib().ssd_gguf_find(self.h, name.encode(), ctypes.byref(idx)))
        if idx.value < 0:
            raise KeyError(name)
        out = np.empty(self.tensors[idx.value]["size"], np.uint8)
        check(lib().ssd_gguf_read(self.h, idx.value, out.ctypes.data, out.nbytes))
        return out

    def model_config(self, kv_capacity: int, tp_rank: int = 0, tp_size: int = 1) -> dict:
        c = ModelConfig()
        check(lib().ssd_gguf_model_config(self.h, kv_capacity, tp_rank, tp_size,
                                          ctypes.byref(c)))
        return {n: getattr(c, n) for n, _ in ModelConfig._fields_}

    def close(self):
        if self.h:
            lib().ssd_gguf_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Model:
    """Decode engine (forward_pass / generate's token loop) on HBM-resident weights."""

    def __init__(self, ctx: Context, **cfg):
        c = ModelConfig(**cfg)
        h = _vp()
        check(lib().ssd_model_create(ctx.h, ctypes.byref(c), ctypes.byref(h)))
        self.ctx, self.h, self.cfg = ctx, h, c

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        check(lib().ssd_tp_unique_id(buf))
        return buf.raw

    def tp_init(self, uid: bytes):
        check(lib().ssd_model_tp_init(self.h, uid))

    def p2p_handle(self) -> bytes:
        """This rank's 64-byte CUDA IPC handle of its all-reduce receive buffer."""
        buf = ctypes.create_string_buffer(64)
        check(lib().ssd_model_p2p_handle(self.h, buf))
        return buf.raw

    def p2p_open(self, handles):
        """Maps every rank's buffer (handles in rank order): partial sums then travel
        over peer memory inside the decode kernels instead of ncclAllReduce."""
        check(lib().ssd_model_p2p_open(self.h, b"".join(handles)))

    @classmethod
    def from_gguf(cls, ctx: Context, path: str, kv_capacity: int, tp_rank: int = 0,
                  tp_size: int = 1, uid: bytes = None):
        """The decode engine built from a GGUF file: config from its metadata, every
        tensor streamed into HBM (this rank's shard). TP needs the NCCL id (uid)."""
        g = GgufFile(path)
        try:
            cfg = g.model_config(kv_capacity, tp_rank, tp_size)
            m = cls(ctx, **cfg)
            if tp_size > 1:
                m.tp_init(uid)
            check(lib().ssd_model_load_gguf(m.h, g.h, cfg["n_layers"]))
        finally:
            g.close()
        return m

    def synth_weights(self, seed: int, std: float = 0.02):
        check(lib().ssd_model_synth_weights(self.h, seed, std))

    def set_tensor(self, name: str, layer: int, raw: np.ndarray, wtype: int | None = None):
        """raw: the full tensor in the reference layout; wtype: its own ggml type when it
        differs from the model config's type for that name (files may mix types)."""
        raw = np.ascontiguousarray(raw)
        if wtype is None:
            check(lib().ssd_model_set_tensor(self.h, name.encode(), layer, raw.ctypes.data,
                                             raw.nbytes))
        else:
            check(lib().ssd_model_set_tensor_typed(self.h, name.encode(), layer,
                                                   raw.ctypes.data, raw.nbytes, wtype))

    def synth_kv(self, seed: int, n: int):
        check(lib().ssd_model_synth_kv(self.h, seed, n))

    def set_position(self, pos: int):
        check(lib().ssd_model_set_position(self.h, pos))

    def position(self) -> int:
        p = ctypes.c_int()
        check(lib().ssd_model_get_position(self.h, ctypes.byref(p)))
        return p.value

    def decode_step(self, use_graph: bool = True):
        check(lib().ssd_model_decode_step(self.h, int(use_graph)))

    def decode_token(self, token: int, use_graph: bool = True) -> int:
        out = ctypes.c_int32()
        check(lib().ssd_model_decode_token(self.h, token, ctypes.byref(out), int(use_graph)))
        return out.value

    def prefill(self, tokens) -> int:
        """Batch prefill of the prompt tokens at the current position (batch_prefill_lora
        + the last token's greedy argmax); returns the next token."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = ctypes.c_int32()
        check(lib().ssd_model_prefill(self.h, t.ctypes.data, t.size, ctypes.byref(out)))
        return out.value

    def state_ptrs(self):
        h, lg, t = _vp(), _vp(), _vp()
        check(lib().ssd_model_state(self.h, ctypes.byref(h), ctypes.byref(lg), ctypes.byref(t)))
        return h.value, lg.value, t.value

    def weight(self, name: str, layer: int) -> Weight:
        """Borrowed handle of this rank's shard (owned by the model; do not free)."""
        h = _vp()
        check(lib().ssd_model_weight(self.h, name.encode(), layer, ctypes.byref(h)))
        t, r, c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        check(lib().ssd_weight_info(h, ctypes.byref(t), ctypes.byref(r), ctypes.byref(c), None))
        w = Weight.__new__(Weight)
        w.ctx, w.h, w.type, w.rows, w.cols = self.ctx, h, t.value, r.value, c.value
        w.borrowed = True
        return w

    def norm(self, name: str, layer: int) -> int:
        p = _vp()
        check(lib().ssd_model_norm(self.h, name.encode(), layer, ctypes.byref(p)))
        return p.value

    def kv(self, layer: int):
        h = _vp()
        check(lib().ssd_model_kv(self.h, layer, ctypes.byref(h)))
        k = KvCache.__new__(KvCache)
        k.ctx, k.h = self.ctx, h
        # the cache holds this rank's KV heads (all of them at tp_size 1)
        k.capacity, k.n_head_kv, k.head_dim = (self.cfg.kv_capacity,
                                               self.cfg.n_head_kv // max(self.cfg.tp_size, 1),
                                               self.cfg.head_dim)
        return k

    def layer_step(self, layer: int):
        check(lib().ssd_model_layer_step(self.h, layer))

    def launches_per_step(self) -> int:
        n = ctypes.c_int()
        check(lib().ssd_model_launches_per_step(self.h, ctypes.byref(n)))
        return n.value

    def free(self):
        if self.h:
            lib().ssd_model_free(self.h)
            self.h = None


class Batch:
    """Sixteen decode slots over one model (BatchScheduler's layer-major decode step,
    src/inference/batch_scheduler.rs:149-403): every slot its own INT8 KV cache and
    position; step() advances all of them by one token."""

    def __init__(self, model: Model, capacity: int):
        h = _vp()
        check(lib().ssd_batch_create(model.h, capacity, ctypes.byref(h)))
        n = ctypes.c_int()
        check(lib().ssd_batch_slots(h, ctypes.byref(n)))
        self.model, self.h, self.slots, self.capacity = model, h, n.value, capacity

    def step(self, tokens=None, use_graph: bool = True) -> np.ndarray:
        """tokens: one id per slot (None: each slot continues from its last output).
        Returns the greedy next token of every slot."""
        out = np.zeros(self.slots, np.int32)
        tin = None
        if tokens is not None:
            tin = np.ascontiguousarray(tokens, dtype=np.int32)
            assert tin.size == self.slots
        check(lib().ssd_batch_step(self.h, None if tin is None else tin.ctypes.data,
                                   out.ctypes.data, int(use_graph)))
        return out

    def set_position(self, slot: int, pos: int):
        check(lib().ssd_batch_set_position(self.h, slot, pos))

    def positions(self) -> np.ndarray:
        p = np.zeros(self.slots, np.int32)
        check(lib().ssd_batch_positions(self.h, p.ctypes.data))
        return p

    def synth_kv(self, seed: int, n: int):
        check(lib().ssd_batch_synth_kv(self.h, seed, n))

    def kv_pointers(self, layer: int, slot: int):
        v = [_vp() for _ in range(4)]
        check(lib().ssd_batch_kv_pointers(self.h, layer, slot, *[ctypes.byref(x) for x in v]))
        return tuple(x.value for x in v)

    def hidden_ptr(self) -> int:
        p = _vp()
        check(lib().ssd_batch_state(self.h, ctypes.byref(p)))
        return p.value

    def launches_per_step(self) -> int:
        n = ctypes.c_int()
        check(lib().ssd_batch_launches_per_step(self.h, ctypes.byref(n)))
        return n.value

    def free(self):
        if self.h:
            lib().ssd_batch_free(self.h)
            self.h = None


def shard_range(cfg: ModelConfig, name: str, layer: int):
    """(row0, nrows, col0, ncols) of tensor `name` kept by rank cfg.tp_rank (host only)."""
    v = [ctypes.c_int() for _ in range(4)]
    check(lib().ssd_shard_range(ctypes.byref(cfg), name.encode(), layer,
                                *[ctypes.byref(x) for x in v]))
    return tuple(x.value for x in v)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


class CudaCompute:
    """Host-slice mirror of MetalCompute (src/metal/compute.rs:18-375) and of
    MetalGpu::feed_forward_f32 (src/metal/gpu.rs:789-838).

    Same method names and argument meaning as the reference; numpy arrays stand in for
    Rust slices, and each method is one call of the C entry point a Rust binding would
    make (ssd_*_host: copy in, run the CUDA kernels, copy out, synchronise). In-place
    methods update the given array. `new()` mirrors MetalCompute::new() -> Option<Self>
    but raises instead of returning None when no device is usable (no CPU fallback).
    """

    def __init__(self, device: int = 0):
        self.ctx = Context(device)

    @classmethod
    def new(cls, device: int = 0):
        return cls(device)

    @staticmethod
    def is_available() -> bool:
        """compute.rs:31-45: a usable CUDA device."""
        import torch
        return torch.cuda.is_available()

    def has_gpu(self) -> bool:
        """compute.rs:261-264."""
        return True

    def shader_library_path(self):
        """compute.rs:266-269: no runtime-compiled shader library (sm_100a code in the .so)."""
        return None

    def should_use_gpu(self, elements: int) -> bool:
        """compute.rs:140-143: every call runs on the GPU here (no CPU fallback)."""
        return True

    def matvec_f32(self, w, x, out_dim, in_dim):
        """compute.rs:145-153."""
        w, x = _f32(w), _f32(x)
        y = np.zeros(out_dim, dtype=np.float32)
        check(lib().ssd_matvec_f32_host(self.ctx.h, w.ctypes.data, x.ctypes.data, y.ctypes.data,
                                        out_dim, in_dim))
        return y

    def matvec_quantized(self, w_raw, x, out_dim, in_dim, dtype):
        """compute.rs:157-191"""
        w_raw = np.ascontiguousarray(w_raw, dtype=np.uint8)
        x = _f32(x)
        y = np.zeros(out_dim, dtype=np.float32)
        check(lib().ssd_matvec_quantized_host(self.ctx.h, w_raw.ctypes.data, w_raw.nbytes,
                                              x.ctypes.data, y.ctypes.data, out_dim, in_dim,
                                              dtype))
        return y

    def rmsnorm_f32(self, x: np.ndarray, weight, eps):
        """compute.rs:193-202 (in place on x, a contiguous float32 array)."""
        assert x.dtype == np.float32 and x.flags.c_contiguous
        w = _f32(weight)
        check(lib().ssd_rmsnorm_f32_host(self.ctx.h, x.ctypes.data, w.ctypes.data, x.size, eps))

    def softmax_f32(self, x: np.ndarray):
        """compute.rs:204-215 (in place on x, a contiguous float32 array)."""
        assert x.dtype == np.float32 and x.flags.c_contiguous
        check(lib().ssd_softmax_f32_host(self.ctx.h, x.ctypes.data, x.size))

    def flash_attention_f32(self, q_heads, k_cache, v_cache, n_head, n_head_kv, head_dim,
                            seq_len, window_start, window_end):
        """compute.rs:217-259 (f32 K/V rows [seq][n_head_kv * head_dim])."""
        q, k, v = _f32(q_heads), _f32(k_cache), _f32(v_cache)
        out = np.zeros(n_head * head_dim, dtype=np.float32)
        check(lib().ssd_flash_attention_f32_host(self.ctx.h, q.ctypes.data, k.ctypes.data,
                                                 v.ctypes.data, n_head, n_head_kv, head_dim,
                                                 seq_len, window_start, window_end,
                                                 out.ctypes.data))
        return out

    def fused_qkv_f32(self, wq, wk, wv, x, q_dim, kv_dim, n_embd):
        """compute.rs:273-292 -> (q, k, v)."""
        wq, wk, wv, x = _f32(wq), _f32(wk), _f32(wv), _f32(x)
        q = np.zeros(q_dim, np.float32)
        k, v = np.zeros(kv_dim, np.float32), np.zeros(kv_dim, np.float32)
        check(lib().ssd_fused_qkv_f32_host(self.ctx.h, wq.ctypes.data, wk.ctypes.data,
                                           wv.ctypes.data, x.ctypes.data, q_dim, kv_dim, n_embd,
                                           q.ctypes.data, k.ctypes.data, v.ctypes.data))
        return q, k, v

    def fused_qkv_rope_f32(self, wq, wk, wv, x, q_dim, kv_dim, n_embd, head_dim, position,
                           theta_base):
        """compute.rs:296-323 -> (q_rope, k_rope, v)."""
        wq, wk, wv, x = _f32(wq), _f32(wk), _f32(wv), _f32(x)
        q = np.zeros(q_dim, np.float32)
        k, v = np.zeros(kv_dim, np.float32), np.zeros(kv_dim, np.float32)
        check(lib().ssd_fused_qkv_rope_f32_host(self.ctx.h, wq.ctypes.data, wk.ctypes.data,
                                                wv.ctypes.data, x.ctypes.data, q_dim, kv_dim,
                                                n_embd, head_dim, position, theta_base,
                                                q.ctypes.data, k.ctypes.data, v.ctypes.data))
        return q, k, v

    def fused_post_attn_norm_f32(self, hidden: np.ndarray, attn_output, norm_weight, eps):
        """compute.rs:328-343: hidden += attn in place (float32 array); returns
        rmsnorm(hidden) * norm_weight."""
        assert hidden.dtype == np.float32 and hidden.flags.c_contiguous
        a, w = _f32(attn_output), _f32(norm_weight)
        out = np.zeros(hidden.size, np.float32)
        check(lib().ssd_fused_post_attn_norm_f32_host(self.ctx.h, hidden.ctypes.data,
                                                      a.ctypes.data, w.ctypes.data, hidden.size,
                                                      eps, out.ctypes.data))
        return out

    def fused_rmsnorm_linear_f32(self, x, norm_weight, out_weight, vocab_size, n_embd):
        """compute.rs:348-374."""
        x, nw, ow = _f32(x), _f32(norm_weight), _f32(out_weight)
        out = np.zeros(vocab_size, np.float32)
        check(lib().ssd_fused_rmsnorm_linear_f32_host(self.ctx.h, x.ctypes.data, nw.ctypes.data,
                                                      ow.ctypes.data, vocab_size, n_embd,
                                                      out.ctypes.data))
        return out

    def feed_forward_f32(self, x, w_gate, w_up, w_down, n_embd):
        """MetalGpu::feed_forward_f32 (gpu.rs:789-838); n_ff = len(w_gate) / n_embd."""
        x, wg, wu, wd = _f32(x), _f32(w_gate), _f32(w_up), _f32(w_down)
        n_ff = wg.size // n_embd
        out = np.zeros(n_embd, np.float32)
        check(lib().ssd_feed_forward_f32_host(self.ctx.h, x.ctypes.data, wg.ctypes.data,
                                              wu.ctypes.data, wd.ctypes.data, n_embd, n_ff,
                                              out.ctypes.data))
        return out

    def flash_attention_int8(self, q_heads, k_q, k_scale, v_q, v_scale, n_head, n_head_kv,
                             head_dim, seq_len):
        """The same attention over the INT8 cache (quantized_kv_cache.rs:107-130)."""
        import torch
        kv = KvCache(self.ctx, seq_len, n_head_kv, head_dim)
        try:
            kp, vp, ksp, vsp = kv.pointers()
            torch.cuda.synchronize()
            copy_to_device(self.ctx, kp, np.ascontiguousarray(k_q, dtype=np.int8))
            copy_to_device(self.ctx, vp, np.ascontiguousarray(v_q, dtype=np.int8))
            copy_to_device(self.ctx, ksp, _f32(k_scale))
            copy_to_device(self.ctx, vsp, _f32(v_scale))
            qd = torch.from_numpy(_f32(q_heads)).to(torch.device("cuda", self.ctx.device))
            out = torch.empty(n_head * head_dim, device=qd.device)
            kv.attention(qd, n_head, seq_len, out)
            return out.cpu().numpy()
        finally:
            torch.cuda.synchronize()
            kv.free()


def copy_to_device(ctx: Context, dev_ptr: int, host: np.ndarray):
    host = np.ascontiguousarray(host)
    check(lib().ssd_copy_to_device(ctx.h, dev_ptr, host.ctypes.data, host.nbytes))


def copy_to_host(ctx: Context, host: np.ndarray, dev_ptr: int):
    check(lib().ssd_copy_to_host(ctx.h, host.ctypes.data, dev_ptr, host.nbytes))
