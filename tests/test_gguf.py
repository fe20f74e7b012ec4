"""GGUF reader through the C ABI (host code: runs without a GPU).

Follows GgufFile::open and its accessors (src/model/gguf.rs:233-441): header fields,
metadata of every value type, tensor infos with the reference's size rule
(ceil(n_elements / block) * block bytes, gguf.rs:87-135, :284-291), the aligned data
section (general.alignment, default 32), MetadataValue::as_u32 accepting u32 / i32 / u64
only, and the failures the reference reports (bad magic, versions other than 2-3,
strings over 1 MiB, truncated files). The model config derived from llama.* metadata uses
the reference's defaults.
"""
import struct

import numpy as np
import pytest

import ssdllm
from gguf_write import (ARR, BOOL, F32, F64, I8, I16, I32, I64, STR, U8, U16, U32, U64,
                        llama_metadata, write_gguf)

Q4_0, Q8_0, Q4_K, F32T, F16T = 2, 8, 12, 0, 1


def rand_bytes(n, seed):
    return np.random.default_rng(seed).integers(0, 256, n, dtype=np.uint8).tobytes()


ALL_META = [
    ("k.u8", U8, 7), ("k.i8", I8, -5), ("k.u16", U16, 65000), ("k.i16", I16, -300),
    ("k.u32", U32, 4000000000), ("k.i32", I32, 123456), ("k.f32", F32, 1.5), ("k.bool", BOOL, True),
    ("k.str", STR, "hello gguf"), ("k.u64", U64, 1 << 40), ("k.i64", I64, -(1 << 40)),
    ("k.f64", F64, 2.25), ("k.arr_u32", ARR, (U32, [1, 2, 3])),
    ("k.arr_str", ARR, (STR, ["a", "bb", "ccc", ""])),
    ("k.arr_arr", ARR, (ARR, [(U8, [1, 2]), (U8, [])])),
]


def test_header_metadata_tensors_and_bytes(tmp_path):
    tensors = [
        ("blk.0.attn_q.weight", [64, 3], Q4_0, rand_bytes(3 * 2 * 18, 1)),
        ("blk.0.ffn_norm.weight", [64], F32T, rand_bytes(64 * 4, 2)),
        ("output.weight", [256, 2], Q4_K, rand_bytes(2 * 144, 3)),
        ("token_embd.weight", [32, 5], Q8_0, rand_bytes(5 * 34, 4)),
        ("odd.weight", [40], Q4_0, rand_bytes(2 * 18, 5)),  # 40 elements: 2 blocks
    ]
    path = str(tmp_path / "m.gguf")
    data0 = write_gguf(path, ALL_META, tensors)
    g = ssdllm.GgufFile(path)
    assert (g.version, g.n_tensors, g.n_kv) == (3, len(tensors), len(ALL_META))
    assert g.data_offset == data0 and g.data_offset % 32 == 0
    for (name, dims, gt, raw), t in zip(tensors, g.tensors):
        assert t["name"] == name and t["dims"] == dims and t["type"] == gt
        assert t["size"] == len(raw) and t["offset"] % 32 == 0
        assert g.read(name).tobytes() == raw
    assert g.find_tensor("output.weight")["type"] == Q4_K
    assert g.find_tensor("missing.weight") is None
    # MetadataValue::as_u32: UInt32, Int32, UInt64 (truncated) only
    assert g.get_u32("k.u32") == 4000000000
    assert g.get_u32("k.i32") == 123456
    assert g.get_u32("k.u64") == (1 << 40) & 0xFFFFFFFF
    assert g.get_u32("k.u8") is None and g.get_u32("k.str") is None and g.get_u32("nope") is None
    assert g.get_f32("k.f32") == 1.5 and g.get_f32("k.f64") is None
    assert g.get_str("k.str") == "hello gguf" and g.get_str("k.u32") is None
    assert g.array_len("k.arr_str") == 4 and g.array_len("k.arr_arr") == 2
    assert g.array_len("k.u32") is None
    g.close()


def test_custom_alignment(tmp_path):
    path = str(tmp_path / "a.gguf")
    md = [("general.alignment", U32, 64), ("pad", STR, "x" * 13)]
    tensors = [("a", [32], Q4_0, rand_bytes(18, 6)), ("b", [32], Q4_0, rand_bytes(18, 7))]
    data0 = write_gguf(path, md, tensors, alignment=64)
    g = ssdllm.GgufFile(path)
    assert g.data_offset == data0 and g.data_offset % 64 == 0
    assert g.tensors[1]["offset"] == 64
    assert g.read("b").tobytes() == tensors[1][3]


def test_version_2_is_accepted(tmp_path):
    path = str(tmp_path / "v2.gguf")
    write_gguf(path, [("x", U32, 1)], [("t", [32], Q8_0, rand_bytes(34, 8))], version=2)
    assert ssdllm.GgufFile(path).version == 2


@pytest.mark.parametrize("kind", ["magic", "v1", "v4", "truncated", "long_string", "bad_type"])
def test_malformed_files_are_rejected(tmp_path, kind):
    path = str(tmp_path / f"{kind}.gguf")
    tensors = [("t", [32], Q4_0, rand_bytes(18, 9))]
    if kind == "magic":
        write_gguf(path, [], tensors, magic=b"GGML")
    elif kind in ("v1", "v4"):
        write_gguf(path, [], tensors, version=int(kind[1]))
    elif kind == "truncated":
        write_gguf(path, ALL_META, tensors)
        raw = open(path, "rb").read()
        open(path, "wb").write(raw[:100])
    elif kind == "long_string":  # a key claiming 2 MiB (read_gguf_string's limit is 1 MiB)
        body = b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + struct.pack("<Q", 2 * 1024 * 1024)
        open(path, "wb").write(body + b"k" * 64)
    else:  # metadata value type 13 does not exist
        body = b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + struct.pack("<Q", 1) + b"k"
        open(path, "wb").write(body + struct.pack("<I", 13) + b"\0" * 16)
    with pytest.raises(ssdllm.SsdError) as e:
        ssdllm.GgufFile(path)
    assert e.value.status == 1  # SSD_ERR_ARG


def test_missing_file_is_an_error(tmp_path):
    with pytest.raises(ssdllm.SsdError):
        ssdllm.GgufFile(str(tmp_path / "none.gguf"))


def _llama_tensors(L, E, F, kvd, V, wtype, out=True):
    rows = lambda r, c, t: rand_bytes(ssdllm.row_bytes(t, c) * r, r * 7 + c)
    ts = [("token_embd.weight", [E, V], Q8_0, rows(V, E, Q8_0)),
          ("output_norm.weight", [E], F32T, rand_bytes(E * 4, 1))]
    if out:
        ts.append(("output.weight", [E, V], Q4_0, rows(V, E, Q4_0)))
    for l in range(L):
        ts += [(f"blk.{l}.attn_norm.weight", [E], F32T, rand_bytes(E * 4, 2)),
               (f"blk.{l}.attn_q.weight", [E, E], wtype, rows(E, E, wtype)),
               (f"blk.{l}.attn_k.weight", [E, kvd], wtype, rows(kvd, E, wtype)),
               (f"blk.{l}.attn_v.weight", [E, kvd], wtype, rows(kvd, E, wtype)),
               (f"blk.{l}.attn_output.weight", [E, E], wtype, rows(E, E, wtype)),
               (f"blk.{l}.ffn_norm.weight", [E], F32T, rand_bytes(E * 4, 3)),
               (f"blk.{l}.ffn_gate.weight", [E, F], wtype, rows(F, E, wtype)),
               (f"blk.{l}.ffn_up.weight", [E, F], wtype, rows(F, E, wtype)),
               (f"blk.{l}.ffn_down.weight", [F, E], wtype, rows(E, F, wtype))]
    return ts


def test_model_config_from_llama_metadata(tmp_path):
    path = str(tmp_path / "llama.gguf")
    md = llama_metadata(2, 256, 4, 2, 512, 300, theta=5e5, eps=1e-6)
    write_gguf(path, md, _llama_tensors(2, 256, 512, 128, 300, Q4_0))
    c = ssdllm.GgufFile(path).model_config(kv_capacity=64, tp_rank=1, tp_size=2)
    assert (c["n_layers"], c["n_embd"], c["n_head"], c["n_head_kv"], c["head_dim"]) == (2, 256, 4, 2, 64)
    assert (c["n_ff"], c["vocab"], c["wtype"], c["out_type"], c["embd_type"]) == (512, 300, Q4_0, Q4_0, Q8_0)
    assert (c["kv_capacity"], c["tp_rank"], c["tp_size"]) == (64, 1, 2)
    assert c["theta"] == pytest.approx(5e5) and c["eps"] == pytest.approx(1e-6)


def test_model_config_defaults(tmp_path):
    """head_count_kv -> head_count, rope base 10000 (DEFAULT_ROPE_THETA), eps 1e-5,
    vocab from token_embd when the tokenizer array is absent, output -> token_embd."""
    path = str(tmp_path / "d.gguf")
    md = llama_metadata(1, 128, 2, None, 256, None, arch="mistral")
    write_gguf(path, md, _llama_tensors(1, 128, 256, 128, 77, Q8_0, out=False))
    c = ssdllm.GgufFile(path).model_config(kv_capacity=32)
    assert (c["n_head_kv"], c["vocab"], c["wtype"], c["out_type"]) == (2, 77, Q8_0, Q8_0)
    assert c["theta"] == 10000.0 and c["eps"] == pytest.approx(1e-5)
