"""GPU parity of continuous-batch decode (BatchScheduler::step's layer-major decode phase,
src/inference/batch_scheduler.rs:225-363): sixteen slots advance together through the
batched tensor-core matvecs (matvec_b.cu) and the slot-indexed attention, and every slot's
greedy tokens must equal the oracle's single-request decode loop from the same start
(generate, src/inference/transformer.rs:681-770). A mismatch is accepted only at a step
whose oracle top-2 logit margin is below fp32 reordering noise, and comparison of that
slot stops there."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import ssdllm  # noqa: E402
from oracle import oracle as ora  # noqa: E402

from _models import OracleDecoder, build_model, make_weights  # noqa: E402

NEAR_TIE = 1e-4


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return ssdllm.Context(0)


def toy_cfg(wtype, out_type=ora.Q4_0, capacity=96):
    return dict(n_layers=2, n_embd=256, n_head=4, n_head_kv=2, head_dim=64, n_ff=512, vocab=512,
                wtype=wtype, out_type=out_type, embd_type=ora.Q4_0, kv_capacity=capacity,
                theta=1e4, eps=1e-5, tp_rank=0, tp_size=1)


def compare(gpu_seq, oracle, start_token, what):
    """gpu_seq: the slot's tokens after start_token; oracle: a fresh OracleDecoder."""
    t = start_token
    for i, g in enumerate(gpu_seq):
        t, margin = oracle.step(t)
        if g != t:
            assert margin < NEAR_TIE, (what, i, g, t, margin)
            return i
        t = g
    return len(gpu_seq)


@pytest.mark.parametrize("wtype", [ora.Q4_0, ora.Q8_0, ora.Q4_K])
def test_sixteen_streams_match_single_stream_oracle(ctx, wtype):
    cfg = toy_cfg(wtype)
    rng = np.random.default_rng(77 + int(wtype))
    layers, glob = make_weights(rng, 256, 4, 2, 64, 512, 512, 2, wtype=wtype)
    m = build_model(ssdllm, ctx, cfg, layers, glob)
    b = ssdllm.Batch(m, capacity=cfg["kv_capacity"])
    try:
        assert b.slots == 16
        starts = np.array([(37 * i + 5) % 512 for i in range(16)], np.int32)
        steps = 40
        seqs = np.zeros((16, steps), np.int32)
        cur = b.step(starts)
        seqs[:, 0] = cur
        for s in range(1, steps):
            cur = b.step(None)
            seqs[:, s] = cur
        assert np.all(b.positions() == steps)
    finally:
        b.free()
        m.free()
    for i in range(16):
        n = compare(list(seqs[i]), OracleDecoder(cfg, layers, glob, cfg["kv_capacity"]),
                    int(starts[i]), f"slot {i}")
        assert n >= steps // 2 or n == steps, (i, n)


def test_requests_join_and_leave_between_steps(ctx):
    """Continuous batching: slots 3 and 9 get new requests (position 0, new first token)
    after 12 steps while the others keep decoding; slot 5 feeds a 4-token prompt through
    its inputs. Every stream still equals its own oracle decode."""
    cfg = toy_cfg(ora.Q4_0)
    rng = np.random.default_rng(404)
    layers, glob = make_weights(rng, 256, 4, 2, 64, 512, 512, 2)
    m = build_model(ssdllm, ctx, cfg, layers, glob)
    b = ssdllm.Batch(m, capacity=cfg["kv_capacity"])
    starts = np.array([(11 * i + 3) % 512 for i in range(16)], np.int32)
    prompt5 = [starts[5], 101, 202, 303]
    try:
        hist = {i: [] for i in range(16)}
        tin = starts.copy()
        for s in range(28):
            if s == 12:
                for sl, tok in ((3, 77), (9, 88)):
                    b.set_position(sl, 0)
                    tin[sl] = tok
                    hist[sl] = []
            if 1 <= s < 4:
                tin[5] = prompt5[s]  # the prompt's next token instead of the output
            out = b.step(tin, use_graph=(s % 2 == 0))
            for i in range(16):
                hist[i].append(int(out[i]))
            tin = out.copy()
    finally:
        b.free()
        m.free()
    for i in range(16):
        o = OracleDecoder(cfg, layers, glob, cfg["kv_capacity"])
        if i in (3, 9):
            compare(hist[i], o, 77 if i == 3 else 88, f"slot {i} (rejoined)")
        elif i == 5:
            for tok in prompt5[:3]:
                o.step(int(tok))  # prompt positions 0-2: outputs not used
            compare(hist[5][3:], o, int(prompt5[3]), "slot 5 (prompt)")
        else:
            compare(hist[i], o, int(starts[i]), f"slot {i}")


def test_batch_launch_count(ctx):
    cfg = toy_cfg(ora.Q4_0)
    m = ssdllm.Model(ctx, **cfg)
    m.synth_weights(seed=3, std=0.05)
    b = ssdllm.Batch(m, capacity=64)
    try:
        b.synth_kv(seed=4, n=20)
        assert np.all(b.positions() == 20)
        b.step(np.arange(16, dtype=np.int32))
        # embed; per layer 4 x (B prep + matvec), 2 norm stats, attention (2); logits
        # (stats, B prep, matvec); finalize
        assert b.launches_per_step() == 1 + cfg["n_layers"] * (4 * 2 + 2 + 2) + 3 + 1
    finally:
        b.free()
        m.free()
