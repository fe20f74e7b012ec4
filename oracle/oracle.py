"""ctypes wrapper of the CPU oracle (TEST INFRASTRUCTURE ONLY).

The oracle (oracle.c) restates ssd-llm's CPU compute path function by function
(citations in oracle.h). Only tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / reference arm load this module; the CUDA product path never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

F32, F16, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K, Q8_K, BF16 = 0, 1, 2, 8, 12, 13, 14, 15, 30
Q2_K, Q3_K, IQ2_XXS, IQ2_XS, IQ3_XXS, IQ4_NL, IQ3_S, IQ4_XS = 10, 11, 16, 17, 18, 20, 21, 23
BLOCK = {Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210),
         Q8_K: (256, 292), F16: (1, 2), BF16: (1, 2), F32: (1, 4)}

_fp = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i8p = ctypes.POINTER(ctypes.c_int8)


def build() -> str:
    """Compile oracle.c with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        i64, i32, f32 = ctypes.c_int64, ctypes.c_int, ctypes.c_float
        L.ora_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.ora_f16_to_f32.restype = f32
        L.ora_f32_to_f16.argtypes = [f32]
        L.ora_f32_to_f16.restype = ctypes.c_uint16
        L.ora_row_bytes.argtypes = [i32, i64]
        L.ora_row_bytes.restype = ctypes.c_size_t
        for n in ("ora_quantize_q4_0", "ora_quantize_q8_0", "ora_quantize_q4_k"):
            getattr(L, n).argtypes = [_fp, i64, _u8p]
            getattr(L, n).restype = None
        L.ora_dequantize.argtypes = [_u8p, i32, i64, _fp]
        L.ora_dequantize.restype = i32
        L.ora_matvec_quantized.argtypes = [_u8p, _fp, i32, i32, i32, _fp]
        L.ora_matvec_quantized.restype = i32
        L.ora_matvec_quantized_mt.argtypes = [_u8p, _fp, i32, i32, i32, _fp, i32]
        L.ora_matvec_quantized_mt.restype = i32
        L.ora_matvec_f32.argtypes = [_fp, _fp, i32, i32, _fp]
        L.ora_flash_attention_f32.argtypes = [_fp, _fp, _fp, i32, i32, i32, i32, i32, i32, _fp]
        L.ora_feed_forward_f32.argtypes = [_fp, _fp, _fp, _fp, i32, i32, _fp]
        L.ora_rmsnorm.argtypes = [_fp, _fp, i32, f32]
        L.ora_fused_residual_rmsnorm.argtypes = [_fp, _fp, _fp, i32, f32]
        L.ora_fused_post_attn_norm.argtypes = [_fp, _fp, _fp, i32, f32, _fp]
        L.ora_fused_rmsnorm_linear.argtypes = [_fp, _fp, _fp, i32, i32, _fp]
        L.ora_rope_multi_head.argtypes = [_fp, i32, i32, i32, i32, f32]
        L.ora_softmax.argtypes = [_fp, i32]
        L.ora_silu.argtypes = [_fp, i32]
        L.ora_argmax.argtypes = [_fp, i32]
        L.ora_argmax.restype = i32
        L.ora_kv_quantize.argtypes = [_fp, i32, _i8p, _fp]
        L.ora_kv_dequantize.argtypes = [_i8p, f32, i32, _fp]
        att = [_fp, _i8p, _fp, _i8p, _fp, i32, i32, i32, i32, _fp]
        L.ora_attention_int8.argtypes = att
        L.ora_flash_attention_int8.argtypes = att
        L.ora_layer_step.argtypes = [ctypes.POINTER(OraLayer), _fp, i32, _i8p, _fp, _i8p, _fp,
                                     i32, i32]
        L.ora_layer_step.restype = i32
        _lib = L
    return _lib


class OraLayer(ctypes.Structure):
    _fields_ = [("n_embd", ctypes.c_int), ("n_head", ctypes.c_int), ("n_head_kv", ctypes.c_int),
                ("head_dim", ctypes.c_int), ("n_ff", ctypes.c_int), ("wtype", ctypes.c_int),
                ("wq", _u8p), ("wk", _u8p), ("wv", _u8p), ("wo", _u8p), ("w_gate", _u8p),
                ("w_up", _u8p), ("w_down", _u8p), ("attn_norm", _fp), ("ffn_norm", _fp),
                ("theta", ctypes.c_float), ("eps", ctypes.c_float), ("wtypes", ctypes.c_int * 7)]


def _f(a):
    return a.ctypes.data_as(_fp)


def _u8(a):
    return a.ctypes.data_as(_u8p)


def _i8(a):
    return a.ctypes.data_as(_i8p)


def f32c(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def row_bytes(wtype: int, n_cols: int) -> int:
    return int(lib().ora_row_bytes(wtype, n_cols))


def quantize(w: np.ndarray, wtype: int) -> np.ndarray:
    """Rows of f32 -> packed reference blocks (uint8 [rows, row_bytes])."""
    w = f32c(w)
    rows, cols = w.shape
    out = np.zeros((rows, row_bytes(wtype, cols)), dtype=np.uint8)
    fn = {Q4_0: lib().ora_quantize_q4_0, Q8_0: lib().ora_quantize_q8_0,
          Q4_K: lib().ora_quantize_q4_k}[wtype]
    fn(_f(w), w.size, _u8(out))
    return out


def dequantize(packed: np.ndarray, wtype: int, n: int) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    out = np.zeros(n, dtype=np.float32)
    if lib().ora_dequantize(_u8(packed), wtype, n, _f(out)) != 0:
        raise ValueError("unsupported type")
    return out


def matvec_quantized(packed, x, out_dim, in_dim, wtype, threads=1):
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    x = f32c(x)
    y = np.zeros(out_dim, dtype=np.float32)
    lib().ora_matvec_quantized_mt(_u8(packed), _f(x), out_dim, in_dim, wtype, _f(y), threads)
    return y


def matvec_f32(w, x):
    w, x = f32c(w), f32c(x)
    y = np.zeros(w.shape[0], dtype=np.float32)
    lib().ora_matvec_f32(_f(w), _f(x), w.shape[0], w.shape[1], _f(y))
    return y


def rmsnorm(x, w, eps=1e-5):
    x = f32c(x).copy()
    lib().ora_rmsnorm(_f(x), _f(f32c(w)), x.size, eps)
    return x


def fused_residual_rmsnorm(x, r, w, eps=1e-5):
    x = f32c(x).copy()
    lib().ora_fused_residual_rmsnorm(_f(x), _f(f32c(r)), _f(f32c(w)), x.size, eps)
    return x


def fused_post_attn_norm(h, a, w, eps=1e-5):
    h = f32c(h).copy()
    out = np.zeros_like(h)
    lib().ora_fused_post_attn_norm(_f(h), _f(f32c(a)), _f(f32c(w)), h.size, eps, _f(out))
    return h, out


def fused_rmsnorm_linear(x, nw, ow, vocab, n_embd):
    out = np.zeros(vocab, dtype=np.float32)
    lib().ora_fused_rmsnorm_linear(_f(f32c(x)), _f(f32c(nw)), _f(f32c(ow)), vocab, n_embd,
                                   _f(out))
    return out


def rope_multi_head(x, head_dim, n_heads, position, theta):
    x = f32c(x).copy()
    lib().ora_rope_multi_head(_f(x), x.size, head_dim, n_heads, position, theta)
    return x


def softmax(x):
    x = f32c(x).copy()
    lib().ora_softmax(_f(x), x.size)
    return x


def silu(x):
    x = f32c(x).copy()
    lib().ora_silu(_f(x), x.size)
    return x


def argmax(v):
    v = f32c(v)
    return int(lib().ora_argmax(_f(v), v.size))


def kv_quantize(v):
    v = f32c(v)
    q = np.zeros(v.size, dtype=np.int8)
    s = np.zeros(1, dtype=np.float32)
    lib().ora_kv_quantize(_f(v), v.size, _i8(q), _f(s))
    return q, float(s[0])


def kv_quantize_rows(rows):
    rows = f32c(rows)
    q = np.zeros(rows.shape, dtype=np.int8)
    s = np.zeros(rows.shape[0], dtype=np.float32)
    for i in range(rows.shape[0]):
        qi, si = kv_quantize(rows[i])
        q[i] = qi
        s[i] = si
    return q, s


def attention_int8(q, k, ks, v, vs, seq_len, n_head, n_head_kv, head_dim, flash=False):
    out = np.zeros(n_head * head_dim, dtype=np.float32)
    fn = lib().ora_flash_attention_int8 if flash else lib().ora_attention_int8
    fn(_f(f32c(q)), _i8(np.ascontiguousarray(k, dtype=np.int8)), _f(f32c(ks)),
       _i8(np.ascontiguousarray(v, dtype=np.int8)), _f(f32c(vs)), seq_len, n_head, n_head_kv,
       head_dim, _f(out))
    return out


def flash_attention_f32(q, k, v, n_head, n_head_kv, head_dim, seq_len, window_start,
                        window_end):
    out = np.zeros(n_head * head_dim, dtype=np.float32)
    lib().ora_flash_attention_f32(_f(f32c(q)), _f(f32c(k)), _f(f32c(v)), n_head, n_head_kv,
                                  head_dim, seq_len, window_start, window_end, _f(out))
    return out


def feed_forward_f32(x, w_gate, w_up, w_down, n_embd, n_ff):
    out = np.zeros(n_embd, dtype=np.float32)
    lib().ora_feed_forward_f32(_f(f32c(x)), _f(f32c(w_gate)), _f(f32c(w_up)), _f(f32c(w_down)),
                               n_embd, n_ff, _f(out))
    return out


class Layer:
    """Packed layer weights in reference layout + norms, for ora_layer_step."""

    def __init__(self, n_embd, n_head, n_head_kv, head_dim, n_ff, wtype, wq, wk, wv, wo,
                 w_gate, w_up, w_down, attn_norm, ffn_norm, theta=10000.0, eps=1e-5,
                 wtypes=None):
        """wtypes: per-matrix types (wq, wk, wv, wo, w_gate, w_up, w_down); default wtype."""
        self._keep = [np.ascontiguousarray(a, dtype=np.uint8)
                      for a in (wq, wk, wv, wo, w_gate, w_up, w_down)]
        self._norms = [f32c(attn_norm), f32c(ffn_norm)]
        k = self._keep
        self.s = OraLayer(n_embd, n_head, n_head_kv, head_dim, n_ff, wtype, _u8(k[0]), _u8(k[1]),
                          _u8(k[2]), _u8(k[3]), _u8(k[4]), _u8(k[5]), _u8(k[6]),
                          _f(self._norms[0]), _f(self._norms[1]), theta, eps,
                          (ctypes.c_int * 7)(*(wtypes if wtypes is not None else [-1] * 7)))

    def step(self, hidden, position, k_cache, k_scales, v_cache, v_scales, mode=0, threads=1):
        """Runs one decode step in place on hidden / caches (numpy arrays)."""
        rc = lib().ora_layer_step(ctypes.byref(self.s), _f(hidden), position, _i8(k_cache),
                                  _f(k_scales), _i8(v_cache), _f(v_scales), mode, threads)
        if rc != 0:
            raise ValueError("ora_layer_step failed")
        return hidden
