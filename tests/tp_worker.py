"""One rank of the tensor-parallel decode check in tests/test_gpu_tp.py (not collected by
pytest; launched with torch.distributed.run, one process per GPU).

Builds a small Llama-shaped model (synthetic weights: every rank keeps exact slices of
the same global tensors), exchanges the NCCL id and the peer-buffer IPC handles over a
gloo process group, decodes STEPS greedy tokens, and writes this rank's tokens and its
vocabulary shard of the first step's logits, and its KV heads' cache bytes and row scales
after the decode, to <out>/<mode>_rank<r>.npz.
Usage: tp_worker.py OUT_DIR MODE   (MODE = p2p or nccl)
"""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "ssd-llm_b200"))
import ssdllm  # noqa: E402

CFG = dict(n_layers=3, n_embd=1024, n_head=8, n_head_kv=4, head_dim=128, n_ff=2816,
           vocab=2048, wtype=2, out_type=2, embd_type=2, kv_capacity=64, theta=1e4, eps=1e-5)
STEPS = 8


def read_caches(model, ctx, n):
    """K, V bytes [layer][n][local kv_dim] and their row scales [layer][2][n] (after decode)."""
    kv_loc = (CFG["n_head_kv"] // model.cfg.tp_size) * CFG["head_dim"]
    ks = np.zeros((CFG["n_layers"], 2, n, kv_loc), np.int8)
    sc = np.zeros((CFG["n_layers"], 2, n), np.float32)
    for layer in range(CFG["n_layers"]):
        kp, vp, ksp, vsp = model.kv(layer).pointers()
        for j, (bp, sp) in enumerate(((kp, ksp), (vp, vsp))):
            ssdllm.copy_to_host(ctx, ks[layer, j], bp)
            ssdllm.copy_to_host(ctx, sc[layer, j], sp)
    return ks, sc


def decode(model, ctx):
    """STEPS greedy tokens from token 5 at position 20; first step's logits shard."""
    toks, logits0, t = [], None, 5
    for i in range(STEPS):
        t = model.decode_token(t, use_graph=True)
        toks.append(t)
        if i == 0:
            _, lg, _ = model.state_ptrs()
            n = model.cfg.vocab // model.cfg.tp_size
            logits0 = np.zeros(n, np.float32)
            ssdllm.copy_to_host(ctx, logits0, lg)
    return np.array(toks), logits0


def main():
    out, mode = sys.argv[1], sys.argv[2]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    ctx = ssdllm.Context(rank)
    m = ssdllm.Model(ctx, **CFG, tp_rank=rank, tp_size=world)
    try:
        uid = [ssdllm.Model.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        m.tp_init(uid[0])
        if mode == "p2p":
            hs = [None] * world
            dist.all_gather_object(hs, m.p2p_handle())
            m.p2p_open(hs)
        m.synth_weights(seed=3, std=0.02)
        m.synth_kv(seed=4, n=20)
        toks, logits0 = decode(m, ctx)
        status = ctx.device_status()
        kv, scales = read_caches(m, ctx, 20 + STEPS)
        dist.barrier()  # no rank frees its buffer while a peer may still write to it
    finally:
        m.free()
    np.savez(os.path.join(out, f"{mode}_rank{rank}.npz"), toks=toks, logits0=logits0,
             status=status, kv=kv, scales=scales)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
