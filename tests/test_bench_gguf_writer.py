"""CPU check of the streaming bench case's GGUF writer (bench._write_gguf_q4_0): the file it
writes parses with the library's reader (GgufFile::open layout, src/model/gguf.rs:233-315),
gives the Llama config it was asked for, and every tensor lies inside the file with the size
its type and shape imply."""
import os

import ssdllm

import bench

Q4_0_BLOCK = 18


def test_writer_output_parses_with_the_library_reader(tmp_path):
    path = str(tmp_path / "tiny_q4_0.gguf")
    bench._write_gguf_q4_0(path, 3, 256, 4, 2, 512, 1000, seed=5)
    g = ssdllm.GgufFile(path)
    cfg = g.model_config(kv_capacity=32)
    assert (cfg["n_layers"], cfg["n_embd"], cfg["n_head"], cfg["n_head_kv"], cfg["head_dim"],
            cfg["n_ff"], cfg["vocab"]) == (3, 256, 4, 2, 64, 512, 1000)
    assert cfg["wtype"] == cfg["out_type"] == cfg["embd_type"] == 2  # Q4_0
    assert g.n_tensors == 3 + 3 * 9
    size = os.path.getsize(path)
    for t in g.tensors:
        n = 1
        for d in t["dims"]:
            n *= d
        want = n * 4 if t["type"] == 0 else n // 32 * Q4_0_BLOCK
        assert t["size"] == want, t
        assert t["offset"] % 32 == 0 and g.data_offset + t["offset"] + t["size"] <= size
    down = g.find_tensor("blk.2.ffn_down.weight")
    assert down["dims"] == [512, 256]  # ne0 = columns first
