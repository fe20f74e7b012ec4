"""Minimal GGUF writer for the tests (test infrastructure, not part of the library).

Writes the layout GgufFile::open parses (src/model/gguf.rs:233-315): magic "GGUF",
version, tensor count, metadata count, metadata key/values, tensor infos (name, n_dims,
dims with ne0 = columns first, ggml type, offset), then the data section at the next
multiple of the alignment with each tensor at an aligned offset.
"""
import struct

# metadata value types (gguf.rs:454-483)
U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f",
        BOOL: "<B", U64: "<Q", I64: "<q", F64: "<d"}


def _str(s) -> bytes:
    b = s.encode() if isinstance(s, str) else s
    return struct.pack("<Q", len(b)) + b


def _value(t, v) -> bytes:
    if t == STR:
        return _str(v)
    if t == ARR:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_value(et, x) for x in items)
    if t == BOOL:
        v = 1 if v else 0
    return struct.pack(_FMT[t], v)


def write_gguf(path, metadata, tensors, alignment=32, version=3, magic=b"GGUF"):
    """metadata: [(key, type, value)], arrays as (ARR, (elem_type, [values])).
    tensors: [(name, dims, ggml_type, raw bytes)]."""
    out = bytearray(magic + struct.pack("<IQQ", version, len(tensors), len(metadata)))
    for k, t, v in metadata:
        out += _str(k) + struct.pack("<I", t) + _value(t, v)
    offs, off = [], 0
    for _, _, _, raw in tensors:
        offs.append(off)
        off += len(raw)
        off = (off + alignment - 1) // alignment * alignment
    for (name, dims, gt, _), o in zip(tensors, offs):
        out += _str(name) + struct.pack("<I", len(dims))
        out += b"".join(struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", gt, o)
    pad = (-len(out)) % alignment
    out += b"\0" * pad
    data0 = len(out)
    for (_, _, _, raw), o in zip(tensors, offs):
        out += b"\0" * (data0 + o - len(out))
        out += bytes(raw)
    with open(path, "wb") as f:
        f.write(out)
    return data0


def llama_metadata(n_layers, n_embd, n_head, n_head_kv, n_ff, vocab, theta=None, eps=None,
                   arch="llama", alignment=None):
    md = [("general.architecture", STR, arch),
          (f"{arch}.block_count", U32, n_layers),
          (f"{arch}.embedding_length", U32, n_embd),
          (f"{arch}.feed_forward_length", U32, n_ff),
          (f"{arch}.attention.head_count", U32, n_head)]
    if n_head_kv is not None:
        md.append((f"{arch}.attention.head_count_kv", U32, n_head_kv))
    if theta is not None:
        md.append((f"{arch}.rope.freq_base", F32, theta))
    if eps is not None:
        md.append((f"{arch}.attention.layer_norm_rms_epsilon", F32, eps))
    if vocab is not None:
        md.append(("tokenizer.ggml.tokens", ARR, (STR, [f"t{i}" for i in range(vocab)])))
    if alignment is not None:
        md.append(("general.alignment", U32, alignment))
    return md
