"""Tensor-parallel host logic on CPU: two gloo ranks, the library's own shard plan
(ssd_shard_range, host-only C code), oracle partial sums, gloo all-reduce.

Checks that the row/column split the CUDA engine uses reproduces the unsharded
reference matvecs (src/metal/compute.rs:680-704 per shard, summed as the
NCCL all-reduce would), and that the vocab-sharded argmax combine (max over
packed (value, index) keys) keeps the reference's last-index tie rule
(src/inference/sampler.rs:572-578)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

E, F, NH, NKV, HD, V = 256, 512, 8, 4, 32, 96


def cfg_dict():
    return dict(n_layers=1, n_embd=E, n_head=NH, n_head_kv=NKV, head_dim=HD, n_ff=F, vocab=V,
                wtype=2, out_type=2, embd_type=2, kv_capacity=64, theta=1e4, eps=1e-5)


def weights(seed=7):
    from oracle import oracle as ora
    rng = np.random.default_rng(seed)
    w = {n: (rng.standard_normal(s) * 0.05).astype(np.float32)
         for n, s in (("attn_output", (E, E)), ("ffn_gate", (F, E)), ("ffn_down", (E, F)),
                      ("output", (V, E)))}
    x_attn = rng.standard_normal(E).astype(np.float32)
    x_act = rng.standard_normal(F).astype(np.float32)
    return {k: ora.quantize(v, ora.Q4_0) for k, v in w.items()}, w, x_attn, x_act


def amax_key(v: float, idx: int) -> int:
    """Orderable (value, index) key: the same packing the argmax epilogue uses."""
    u = int(np.float32(v).view(np.uint32))
    u = (~u & 0xFFFFFFFF) if (u & 0x80000000) else (u | 0x80000000)
    return (u << 32) | idx


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import ssdllm
        from oracle import oracle as ora
        packed, _, x_attn, x_act = weights()
        cfg = ssdllm.ModelConfig(**cfg_dict(), tp_rank=rank, tp_size=world)
        res = {}
        # column-sharded Wo / down: partial sums, completed by an all-reduce
        for name, x in (("attn_output", x_attn), ("ffn_down", x_act)):
            r0, nr, c0, nc = ssdllm.shard_range(cfg, name, 0)
            rows, cols = packed[name].shape[0], x.size
            rb = ora.row_bytes(ora.Q4_0, cols)
            kb = ora.row_bytes(ora.Q4_0, nc)
            cb = c0 // 32 * 18
            shard = np.ascontiguousarray(packed[name][r0:r0 + nr, cb:cb + kb])
            assert shard.shape == (nr, kb) and packed[name].shape[1] == rb
            part = torch.from_numpy(ora.matvec_quantized(shard, x[c0:c0 + nc], nr, nc, ora.Q4_0))
            dist.all_reduce(part)
            res[name] = part.numpy()
        # row-sharded gate: all-gather of the row blocks
        r0, nr, c0, nc = ssdllm.shard_range(cfg, "ffn_gate", 0)
        g = torch.from_numpy(ora.matvec_quantized(packed["ffn_gate"][r0:r0 + nr], x_attn, nr, E,
                                                  ora.Q4_0))
        parts = [torch.zeros_like(g) for _ in range(world)]
        dist.all_gather(parts, g)
        res["ffn_gate"] = torch.cat(parts).numpy()
        # vocab-sharded logits with a planted cross-shard tie: argmax via max over keys
        r0, nr, _, _ = ssdllm.shard_range(cfg, "output", -1)
        logits = ora.matvec_quantized(packed["output"][r0:r0 + nr], x_attn, nr, E, ora.Q4_0)
        full = ora.matvec_quantized(packed["output"], x_attn, V, E, ora.Q4_0)
        tie = np.float32(full.max() + 1.0)
        for gi in (3, V - 5):  # one index on each shard
            if r0 <= gi < r0 + nr:
                logits[gi - r0] = tie
        best = max(amax_key(v, r0 + i) for i, v in enumerate(logits))
        # gloo has no uint64 max: compare on the host after an all-gather of keys
        keys = [torch.zeros(2, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(keys, torch.tensor([best >> 32, best & 0xFFFFFFFF], dtype=torch.int64))
        gbest = max((int(k[0]) << 32) | int(k[1]) for k in keys)
        res["argmax"] = gbest & 0xFFFFFFFF
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world", [2])
def test_sharded_matvecs_and_argmax_match_unsharded(world):
    from oracle import oracle as ora
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    packed, _, x_attn, x_act = weights()
    ref = {"attn_output": ora.matvec_quantized(packed["attn_output"], x_attn, E, E, ora.Q4_0),
           "ffn_down": ora.matvec_quantized(packed["ffn_down"], x_act, E, F, ora.Q4_0),
           "ffn_gate": ora.matvec_quantized(packed["ffn_gate"], x_attn, F, E, ora.Q4_0)}
    for r in range(world):
        for k, v in ref.items():
            scale = np.max(np.abs(v))
            assert np.max(np.abs(out[r][k] - v)) / scale < 1e-5, k
        # planted tie at indices 3 (rank 0) and V-5 (rank 1): the LAST index wins
        assert out[r]["argmax"] == V - 5
