"""CPU checks of the C-ABI library: it loads, exports every symbol the public
header declares, and its host-only entry points behave (no GPU needed)."""
import ctypes
import os
import re

import pytest

import ssdllm

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ssdllm_cuda.h")


def declared():
    return sorted(set(re.findall(r"\b(ssd_\w+)\s*\(", open(HEADER).read())))


def test_library_exports_every_declared_symbol():
    L = ssdllm.lib()
    names = declared()
    assert len(names) > 40
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    # the binding declares exactly the header's entry points
    assert set(names) == set(ssdllm._SIGS)


def test_every_declaration_cites_the_reference_or_says_why_not():
    """Each entry point's comment block names the reference interface it replaces
    (src/... path) or says it has no reference counterpart."""
    text = open(HEADER).read()
    blocks = re.split(r"\n(?=/\*)", text)
    for b in blocks:
        fns = re.findall(r"\bint (ssd_\w+)\(", b)
        if not fns or "ssd_abi_version" in fns:
            continue
        assert "src/" in b or "No reference counterpart" in b, fns


def test_abi_version_and_status_strings():
    L = ssdllm.lib()
    assert L.ssd_abi_version() == 1
    assert L.ssd_status_str(0) == b"ok"
    assert L.ssd_status_str(2) == b"unsupported ggml type"
    assert L.ssd_status_str(999) == b"unknown status"


@pytest.mark.parametrize("wtype,cols,expect", [(2, 4096, 128 * 18), (8, 4096, 128 * 34),
                                               (12, 4096, 16 * 144), (0, 10, 40),
                                               (12, 100, 0), (99, 64, 0)])
def test_row_bytes(wtype, cols, expect):
    assert ssdllm.row_bytes(wtype, cols) == expect


def test_null_arguments_are_rejected_with_status():
    L = ssdllm.lib()
    assert L.ssd_ctx_create(0, None) == 1  # SSD_ERR_ARG
    assert L.ssd_weight_free(None) == 0
    assert L.ssd_matvec(None, None, None, None, None) == 1
    assert b"null" in L.ssd_last_error()
    assert L.ssd_matvec_independent(None, None, None, None, None) == 1
    # streaming tier: null model / path / handle
    assert L.ssd_stream_open(None, b"x.gguf", 1 << 30, 1, None) == 1
    assert L.ssd_stream_close(None) == 0
    assert L.ssd_stream_pin(None, 0) == 1
    assert L.ssd_stream_decode_token(None, 0, None) == 1
    assert L.ssd_stream_stats_get(None, None) == 1


def test_context_creation_fails_loudly_without_gpu():
    from _util import gpu_available
    if gpu_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    st = ssdllm.lib().ssd_ctx_create(0, ctypes.byref(h))
    assert st != 0 and not h.value
    with pytest.raises(ssdllm.SsdError):
        ssdllm.Context(0)


def test_shard_ranges_cover_each_tensor_exactly():
    """Row and column shards over N ranks tile the global tensor with no overlap."""
    base = dict(n_layers=2, n_embd=8192, n_head=64, n_head_kv=8, head_dim=128, n_ff=28672,
                vocab=128256, wtype=2, out_type=2, embd_type=2, kv_capacity=4096,
                theta=5e5, eps=1e-5)
    for N in (1, 2, 4, 8):
        for name, layer in (("attn_q", 0), ("attn_k", 0), ("attn_v", 1), ("attn_output", 1),
                            ("ffn_gate", 0), ("ffn_up", 0), ("ffn_down", 1),
                            ("output", -1), ("token_embd", -1)):
            rows_cov, cols_cov = [], []
            for r in range(N):
                cfg = ssdllm.ModelConfig(**base, tp_rank=r, tp_size=N)
                r0, nr, c0, nc = ssdllm.shard_range(cfg, name, layer)
                rows_cov.append((r0, nr))
                cols_cov.append((c0, nc))
            rows_split = len(set(rows_cov)) > 1
            cols_split = len(set(cols_cov)) > 1
            assert not (rows_split and cols_split)
            cov = rows_cov if rows_split else cols_cov
            if rows_split or cols_split:
                cov = sorted(cov)
                assert cov[0][0] == 0
                for (a0, an), (b0, _) in zip(cov, cov[1:]):
                    assert a0 + an == b0
    cfg = ssdllm.ModelConfig(**base, tp_rank=0, tp_size=1)
    with pytest.raises(ssdllm.SsdError):
        ssdllm.shard_range(cfg, "no_such_tensor", 0)


# ------------------------------------------------------------- Rust binding
RUST = os.path.join(ROOT, "ssd-llm_b200", "rust", "src", "cuda")


def _c_params():
    """{name: [param kind]} from the header's prototypes; kind = (pointer depth, base)."""
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for m in re.finditer(r"\b(?:int|size_t|const char\*)\s+(ssd_\w+)\s*\(([^;]*?)\);", text, re.S):
        params = [] if m.group(2).strip() == "void" else m.group(2).split(",")
        kinds = []
        for p in params:
            p = " ".join(p.split())
            arr = re.match(r"(?:const\s+)?(\w+)\s+\w+\[\d+\]$", p)
            if arr:
                kinds.append((1, arr.group(1)))
                continue
            t = re.match(r"(?:const\s+)?(unsigned long long|\w+)\s*(\**)\s*\w+$", p)
            assert t, p
            kinds.append((len(t.group(2)), t.group(1)))
        out[m.group(1)] = kinds
    return out


_RUST_BASE = {"c_int": "int", "c_float": "float", "usize": "size_t", "i64": "int64_t",
              "u64": ("uint64_t", "unsigned long long"), "u32": "uint32_t", "i32": "int32_t",
              "u8": "uint8_t", "i8": "int8_t", "c_void": "void", "c_char": "char",
              "SsdCtx": "ssd_ctx", "SsdWeight": "ssd_weight", "SsdKvCache": "ssd_kv_cache",
              "SsdModel": "ssd_model", "SsdGguf": "ssd_gguf", "SsdBatch": "ssd_batch",
              "SsdModelConfig": "ssd_model_config", "SsdStream": "ssd_stream",
              "SsdStreamStats": "ssd_stream_stats"}


def _rust_params():
    text = open(os.path.join(RUST, "ffi.rs")).read()
    block = text[text.index('extern "C" {'):]
    out = {}
    for m in re.finditer(r"pub fn (ssd_\w+)\((.*?)\)\s*->", block, re.S):
        kinds = []
        for p in [p.strip() for p in m.group(2).split(",") if p.strip()]:
            ty = p.split(":", 1)[1].strip()
            depth = ty.count("*")
            base = ty.replace("*mut", "").replace("*const", "").strip()
            kinds.append((depth, base))
        out[m.group(1)] = kinds
    return out


def test_rust_extern_block_matches_the_header():
    """src/cuda/ffi.rs declares exactly the header's entry points, each with the same
    number of parameters, pointer depths and base types."""
    c, r = _c_params(), _rust_params()
    assert set(c) == set(r), (set(c) ^ set(r))
    for name, ck in c.items():
        rk = r[name]
        assert len(ck) == len(rk), name
        for (cd, cb), (rd, rb) in zip(ck, rk):
            want = _RUST_BASE[rb]
            assert cd == rd and (cb == want or cb in want), (name, cb, rb)


# MetalCompute's public methods (src/metal/compute.rs:31-375) and
# MetalGpu::feed_forward_f32 (src/metal/gpu.rs:789).
METAL_COMPUTE_METHODS = [
    "is_available", "new", "should_use_gpu", "matvec_f32", "matvec_quantized", "rmsnorm_f32",
    "softmax_f32", "flash_attention_f32", "has_gpu", "shader_library_path", "fused_qkv_f32",
    "fused_qkv_rope_f32", "fused_post_attn_norm_f32", "fused_rmsnorm_linear_f32",
    "feed_forward_f32"]


def test_rust_wrapper_has_every_metal_compute_method():
    text = open(os.path.join(RUST, "compute.rs")).read()
    impl = text[text.index("impl CudaCompute {"):text.index("pub struct CudaModel")]
    have = set(re.findall(r"pub fn (\w+)", impl))
    assert set(METAL_COMPUTE_METHODS) <= have, set(METAL_COMPUTE_METHODS) - have
    # every ffi call the wrapper makes is a declared entry point
    called = set(re.findall(r"ffi::(ssd_\w+)\(", text))
    assert called <= set(_rust_params()), called - set(_rust_params())


def test_python_binding_mirrors_the_same_methods():
    have = {n for n in dir(ssdllm.CudaCompute) if not n.startswith("_")}
    assert set(METAL_COMPUTE_METHODS) <= have, set(METAL_COMPUTE_METHODS) - have
