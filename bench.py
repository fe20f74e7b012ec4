#!/usr/bin/env python3
"""Benchmark: Llama-70B-shaped Q4_0 decode on N B200s (benchmark config 4).

One step = one generated token (batch 1) through the whole model: token embedding,
80 decoder layers (fused Q4_0 dequant-matvecs, INT8-KV flash-decode attention),
final RMSNorm + vocab matvec + greedy argmax, tensor-parallel over N GPUs with an
all-reduce after o_proj and down_proj (in the kernels over NVLink peer memory; NCCL with
--allreduce nccl). Weights (39 GB) are synthetic
N(0, 0.02), quantized to Q4_0 on the device; the INT8 KV cache is filled with
N(0, 1) rows to ~3968 positions of a 4096 capacity, so decode runs at ~4K context.

Reported on the same JSON line:
  value      device-timed tokens/s (CUDA events, max over ranks; weights >> L2)
  e2e        the same through ssd_model_decode_token: host token in (pinned H2D),
             graph, next token out (D2H), synchronised every step, timed on the host clock
  roofline   the dominant kernel (gate/up dequant-matvec + SwiGLU) timed alone on
             the model's own layer weights, algorithmic bytes / event time
  kernels    benchmark configs 0-2 one kernel at a time: Q4_0 4096x4096, Q8_0 / Q4_K at
             11008x4096 and 4096x11008 (rotating weight copies > 2x L2), the INT8-KV
             attention at the 70B shape, and the Llama-2-7B-shaped layer step (GB/s,
             fraction of the measured HBM peak); `--case NAME` runs one of them alone
  cpu_baseline  the oracle's restatement of the reference layer step on packed Q4_0
             (src/inference/transformer.rs:283-399 with matvec_quantized_cpu), all host
             cores, one layer timed and extrapolated to 80 layers + logits; each of the
             configs 0-2 kernel cases also carries its own cpu_baseline (the restated
             matvec or layer step on its shape, 1 thread and all host threads)
`--impl reference` times that CPU restatement alone (rank 0) and prints its line: each of its
steps is one 70B-shape layer step (a bounded sample), the tokens/s extrapolated to 80 layers.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "ssd-llm_b200"))
sys.path.insert(0, ROOT)

Q4_0 = 2
CFG70B = dict(n_layers=80, n_embd=8192, n_head=64, n_head_kv=8, head_dim=128, n_ff=28672,
              vocab=128256, wtype=Q4_0, out_type=Q4_0, embd_type=Q4_0, kv_capacity=4096,
              theta=5e5, eps=1e-5)
PROMPT = 3968
Q40_BYTES = 18 / 32  # bytes per Q4_0 weight


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback 6.65 TB/s"


# ------------------------------------------------------------------ clocks
class Clocks:
    """nvidia-smi sampling around the timed region (reads settings, changes none). The
    sampler is started during the warm-up (nvidia-smi needs ~0.5 s to take its first sample
    and a timed region of a few hundred ms would otherwise get none); mark() brackets the
    timed region and summary() keeps the samples taken inside it, or, if it was shorter than
    the sampling period, the samples nearest to it (their count and window are reported)."""
    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None
        self.t = [None, None]
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def mark(self, which):
        """which = 0: timed region starts; 1: it ends (wall clock, as nvidia-smi stamps)."""
        self.t[which] = datetime.datetime.now()

    def __enter__(self):
        if not self.gpus:  # ranks other than 0 sample nothing
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=" + self.Q, "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc and self.proc.poll() is None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.proc:
            return None
        self.f.flush()
        rows = []
        for line in open(self.f.name):
            p = [x.strip() for x in line.split(",")]
            if len(p) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(p[0], "%Y/%m/%d %H:%M:%S.%f")
                if int(p[1]) in self.gpus:
                    rows.append((ts, p[1:]))
            except ValueError:
                continue
        if not rows:
            return None
        window = "timed"
        if self.t[0] and self.t[1]:
            inside = [r for r in rows if self.t[0] <= r[0] <= self.t[1]]
            if inside:
                rows = inside
            else:  # region shorter than the sampling period: the nearest samples, per GPU
                window = "nearest"
                mid = self.t[0] + (self.t[1] - self.t[0]) / 2
                best = {}
                for r in rows:
                    g = r[1][0]
                    if g not in best or abs(r[0] - mid) < abs(best[g][0] - mid):
                        best[g] = r
                rows = list(best.values())
        rows = [r[1] for r in rows]
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": reasons, "samples": len(rows), "window": window}


# -------------------------------------------------------------- CPU baseline
def cpu_layer_inputs(cfg, seed=0):
    """One 70B-shaped layer (packed Q4_0, reference layout) + an INT8 cache of PROMPT rows,
    generated on the host (numpy + the oracle's quantizer)."""
    import numpy as np
    from oracle import oracle as ora
    rng = np.random.default_rng(seed)
    E, F, kvd = cfg["n_embd"], cfg["n_ff"], cfg["n_head_kv"] * cfg["head_dim"]
    shapes = (("attn_q", (E, E)), ("attn_k", (kvd, E)), ("attn_v", (kvd, E)),
              ("attn_output", (E, E)), ("ffn_gate", (F, E)), ("ffn_up", (F, E)),
              ("ffn_down", (E, F)))
    W = {}
    for n, s in shapes:
        w = rng.standard_normal(s, dtype=np.float32)
        w *= np.float32(0.02)
        W[n] = ora.quantize(w, ora.Q4_0)
        del w
    norms = [np.ones(E, np.float32), np.ones(E, np.float32)]
    cap = cfg["kv_capacity"]
    caches = []
    for _ in range(2):
        caches.append(rng.integers(-127, 128, (cap, kvd), dtype=np.int8))
        caches.append((rng.random(cap, dtype=np.float32) * 0.03 + 0.01).astype(np.float32))
    layer = ora.Layer(E, cfg["n_head"], cfg["n_head_kv"], cfg["head_dim"], F, ora.Q4_0,
                      *(W[n] for n, _ in shapes), *norms, theta=cfg["theta"], eps=cfg["eps"])
    h = rng.standard_normal(E, dtype=np.float32)
    return layer, caches, h


def cpu_token_time(cfg, layer_samples, threads):
    """Seconds per token of the restated reference CPU path: measured layer steps
    (median) x n_layers + one measured vocab matvec (fused_rmsnorm_linear's matvec)."""
    import numpy as np
    from oracle import oracle as ora
    layer, (kc, ks, vc, vs), h = cpu_layer_inputs(cfg)
    t_layers = []
    for _ in range(layer_samples):
        hh = h.copy()
        t0 = time.perf_counter()
        layer.step(hh, PROMPT, kc, ks, vc, vs, mode=1, threads=threads)
        t_layers.append(time.perf_counter() - t0)
    rng = np.random.default_rng(1)
    vocab_rows = 16032  # 1/8 of the vocab, scaled by 8 (bounded host memory and time)
    wout = ora.quantize(rng.standard_normal((vocab_rows, cfg["n_embd"]), dtype=np.float32)
                        * np.float32(0.02), ora.Q4_0)
    t0 = time.perf_counter()
    ora.matvec_quantized(wout, h, vocab_rows, cfg["n_embd"], ora.Q4_0, threads=threads)
    t_logits = (time.perf_counter() - t0) * (cfg["vocab"] / vocab_rows)
    t_layer = statistics.median(t_layers)
    return cfg["n_layers"] * t_layer + t_logits, t_layers, t_logits


def cpu_case_baselines(threads):
    """CPU baselines of the per-kernel cases (benchmark configs 0-2): the oracle's C
    restatement of the reference CPU paths on this host, 1 thread (the reference's own CPU
    paths are single-threaded) and all threads (its row split). Matvec configs: the
    restated matvec_quantized_cpu (src/metal/compute.rs:680-750, :904-925) on the case's
    shape; the 7B layer: the restated layer step (transformer.rs:283-399) on packed Q4_0 at
    2048 cached positions. Median of 3 timed calls after one untimed."""
    import numpy as np
    from oracle import oracle as ora

    def timed(fn, reps=3):
        fn()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return statistics.median(ts)

    out = {}
    rng = np.random.default_rng(3)
    for name, wtype, rows, cols in (("q4_0_4096x4096", Q4_0, 4096, 4096),
                                    ("q8_0_11008x4096", 8, 11008, 4096),
                                    ("q8_0_4096x11008", 8, 4096, 11008),
                                    ("q4_k_11008x4096", 12, 11008, 4096),
                                    ("q4_k_4096x11008", 12, 4096, 11008)):
        w = rng.standard_normal((rows, cols), dtype=np.float32)
        w *= np.float32(0.02)
        packed = ora.quantize(w, wtype)
        del w
        x = rng.standard_normal(cols, dtype=np.float32)
        t1 = timed(lambda: ora.matvec_quantized(packed, x, rows, cols, wtype, threads=1))
        tn = timed(lambda: ora.matvec_quantized(packed, x, rows, cols, wtype, threads=threads))
        out[name] = {"us_1thread": round(t1 * 1e6, 1), "us_all_threads": round(tn * 1e6, 1),
                     "cores": threads, "kind": "port", "cpu": cpu_model_name(),
                     "sample": "the whole matvec, median of 3 calls"}
    cfg = dict(n_embd=4096, n_head=32, n_head_kv=32, head_dim=128, n_ff=11008,
               kv_capacity=2049, theta=1e4, eps=1e-5)
    layer, (kc, ks, vc, vs), h = cpu_layer_inputs(cfg, seed=5)
    res = {}
    for t in (1, threads):
        res[t] = timed(lambda: layer.step(h.copy(), 2048, kc, ks, vc, vs, mode=1, threads=t))
    out["layer_7b_q4_0"] = {"us_1thread": round(res[1] * 1e6, 1),
                            "us_all_threads": round(res[threads] * 1e6, 1), "cores": threads,
                            "kind": "port", "cpu": cpu_model_name(),
                            "sample": "one 7B-shape layer step (packed Q4_0, INT8 KV at 2048), "
                                      "median of 3"}
    return out


def cpu_model_name():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args):
    """--impl reference: the oracle port of the reference CPU path, rank 0 only.

    A step is a bounded sample of the workload: one 70B-shape decoder layer step (packed
    Q4_0, INT8 KV at PROMPT positions, all host threads), i.e. 1/80 of a token's layers;
    ms_per_step is that step's measured time, so steps x ms_per_step is the timed region.
    value (tokens/s) is extrapolated from it: 80 x the median layer step + one measured
    vocab matvec (16032 rows, scaled to the 128256-row vocab)."""
    rank, world, _ = env_rank()
    if rank != 0:
        return 0
    from oracle import oracle as ora
    ora.build()
    threads = os.cpu_count() or 1
    cfg = dict(CFG70B)
    t0 = time.perf_counter()
    samples = max(1, args.steps)
    _, t_layers, t_logits = cpu_token_time(cfg, max(1, args.warmup) + samples, threads)
    t_layers = t_layers[max(1, args.warmup):]
    t_layer = statistics.median(t_layers)
    t_tok = cfg["n_layers"] * t_layer + t_logits
    value = 1.0 / t_tok
    line = {
        "impl": "reference", "metric": "decode tokens/s (Llama-70B-shape Q4_0, batch 1)",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": len(t_layers),
        "warmup": args.warmup, "ms_per_step": statistics.mean(t_layers) * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "step": "one 70B-shape decoder layer step (1/80 of a token's layers); value = 1 / "
                "(80 x median layer step + vocab matvec), extrapolated",
        "ms_per_token_extrapolated": t_tok * 1e3,
        "config": {"workload": "llama70b_q4_0_decode_b1", "n_layers": 80, "hidden": 8192,
                   "heads": 64, "kv_heads": 8, "ffn": 28672, "vocab": 128256,
                   "context": PROMPT, "kv": "int8"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "cpu": cpu_model_name(),
                         "sample": f"{len(t_layers)} timed 70B-shape layer steps (packed Q4_0, "
                                   f"INT8 KV at {PROMPT}) x 80 layers + vocab matvec; "
                                   "extrapolated"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "wall_s": time.perf_counter() - t0,
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ CUDA arm
def _graph_time(torch, launches, reps):
    """Capture `launches` (closures that each enqueue one kernel on torch's current
    stream) into one CUDA graph and return microseconds per launch over `reps`
    replays, timed with CUDA events on the replay stream after 3 warm-up replays."""
    for f in launches[:2]:
        f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in launches:
            f()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / (reps * len(launches))


L2_BYTES = 126 * 1024 * 1024
TYPE_NAMES = {2: "Q4_0", 8: "Q8_0", 12: "Q4_K"}


def case_matvec(ctx, torch, ssdllm, peak, wtype, rows, cols, reps=20):
    """Dequant-matvec y = W x (benchmark configs 0 and 1) over rotating weight copies
    whose total exceeds 2x L2, so every launch streams its weights from HBM; with and
    without programmatic dependent launch (PDL); the faster is reported. The variant
    `independent` times the same launches when none depends on the one before."""
    wbytes = rows * ssdllm.row_bytes(wtype, cols)
    copies = min(64, max(2, -(-int(2.2 * L2_BYTES) // wbytes)))
    ws = [ssdllm.Weight.synth(ctx, wtype, 0, 900 + i, 0.02, cols, 0, rows, 0, cols)
          for i in range(copies)]
    x = torch.randn(cols, device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    y = torch.zeros(rows, device="cuda")
    n = max(copies, 64 // copies * copies)
    alg = wbytes + cols * 4 + rows * 4
    res = {}
    for pdl in (False, True):
        ctx.set_pdl(pdl)
        us = _graph_time(torch, [lambda w=ws[i % copies]: ssdllm.matvec(ctx, w, x, y)
                                 for i in range(n)], reps)
        res["pdl" if pdl else "plain"] = {"us_per_launch": round(us, 3),
                                          "gbs": round(alg / us / 1e3, 1),
                                          "frac_of_peak": round(alg / us / 1e3 / peak, 4)}
    ctx.set_pdl(False)
    best = max(res.values(), key=lambda r: r["gbs"])
    # independent launches (ssd_matvec_independent: the same x for every launch, each launch
    # its own y): a kernel does not wait for the one before it, so launches overlap. Reported
    # beside the dependent chain above, which is what a decode step sees; not the case's
    # headline.
    ys = [torch.zeros(rows, device="cuda") for _ in range(n)]
    us = _graph_time(torch, [lambda w=ws[i % copies], yy=ys[i]: ssdllm.matvec_independent(
        ctx, w, x, yy) for i in range(n)], reps)
    res["independent"] = {"us_per_launch": round(us, 3), "gbs": round(alg / us / 1e3, 1),
                          "frac_of_peak": round(alg / us / 1e3 / peak, 4)}
    for w in ws:
        w.free()
    return {"type": TYPE_NAMES[wtype], "shape": [rows, cols], "algorithmic_bytes": alg,
            "rotating_copies": copies, **best, "variants": res}


def case_matvec_q6k(ctx, torch, ssdllm, peak, rows=11008, cols=4096, reps=20):
    """Q6_K dequant-matvec at a config-1 shape. No device quantizer exists for Q6_K, so the
    rotating copies are random reference blocks (every bit pattern is a valid block; d
    set in a typical range) uploaded through ssd_weight_upload."""
    import numpy as np
    Q6_K = 14
    nb = cols // 256
    raw_bytes = rows * nb * 210
    copies = min(16, max(2, -(-int(2.2 * L2_BYTES) // raw_bytes)))
    rng = np.random.default_rng(11)
    ws = []
    for _ in range(copies):
        raw = rng.integers(0, 256, (rows, nb * 210), dtype=np.uint8)
        dv = rng.uniform(2e-5, 2e-4, (rows, nb)).astype(np.float16).view(np.uint16)
        raw[:, 208::210] = (dv & 0xFF).astype(np.uint8)
        raw[:, 209::210] = (dv >> 8).astype(np.uint8)
        ws.append(ssdllm.Weight.upload(ctx, raw, Q6_K, rows, cols))
    x = torch.randn(cols, device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    y = torch.zeros(rows, device="cuda")
    n = max(copies, 64 // copies * copies)
    # bytes the kernel streams: 32 B of signed q per 32 weights + a 4-byte scale word
    alg = rows * (cols // 32) * 36 + cols * 4 + rows * 4
    ctx.set_pdl(True)
    us = _graph_time(torch, [lambda w=ws[i % copies]: ssdllm.matvec(ctx, w, x, y)
                             for i in range(n)], reps)
    ctx.set_pdl(False)
    for w in ws:
        w.free()
    return {"type": "Q6_K", "shape": [rows, cols], "algorithmic_bytes": alg,
            "reference_block_bytes": rows * nb * 210, "rotating_copies": copies,
            "us_per_launch": round(us, 3), "gbs": round(alg / us / 1e3, 1),
            "frac_of_peak": round(alg / us / 1e3 / peak, 4)}


def case_matvec_dense16(ctx, torch, ssdllm, peak, wtype=30, rows=11008, cols=4096, reps=20):
    """16-bit dense (BF16 = 30, F16 = 1) matvec at a config-1 shape: random normal rows
    scaled by 0.05, rotating copies > 2x L2 in total, uploaded through ssd_weight_upload."""
    import numpy as np
    raw_bytes = rows * cols * 2
    copies = min(16, max(2, -(-int(2.2 * L2_BYTES) // raw_bytes)))
    rng = np.random.default_rng(12)
    ws = []
    for _ in range(copies):
        f = (rng.standard_normal((rows, cols)) * 0.05).astype(np.float32)
        raw = (f.astype(np.float16).view(np.uint16) if wtype == 1
               else (f.view(np.uint32) >> 16).astype(np.uint16))
        ws.append(ssdllm.Weight.upload(ctx, raw.view(np.uint8), wtype, rows, cols))
    x = torch.randn(cols, device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    y = torch.zeros(rows, device="cuda")
    n = max(copies, 64 // copies * copies)
    alg = rows * cols * 2 + cols * 4 + rows * 4
    ctx.set_pdl(True)
    us = _graph_time(torch, [lambda w=ws[i % copies]: ssdllm.matvec(ctx, w, x, y)
                             for i in range(n)], reps)
    ctx.set_pdl(False)
    for w in ws:
        w.free()
    return {"type": "F16" if wtype == 1 else "BF16", "shape": [rows, cols],
            "algorithmic_bytes": alg, "rotating_copies": copies,
            "us_per_launch": round(us, 3), "gbs": round(alg / us / 1e3, 1),
            "frac_of_peak": round(alg / us / 1e3 / peak, 4)}


def case_attention(ctx, torch, ssdllm, peak, n_head=64, n_head_kv=8, head_dim=128, seq=4096,
                   reps=20):
    """Split-K flash-decode over the INT8 KV cache (70B shape: 64 q / 8 kv heads,
    4096 positions), 8 rotating caches (> 2x L2 of K/V bytes in total)."""
    kvd = n_head_kv * head_dim
    gen = torch.Generator("cuda").manual_seed(3)
    caches = []
    ncache = max(2, -(-int(2.2 * L2_BYTES) // (2 * seq * kvd)))
    for _ in range(ncache):
        kv = ssdllm.KvCache(ctx, seq, n_head_kv, head_dim)
        k = torch.randn(seq, kvd, device="cuda", generator=gen)
        v = torch.randn(seq, kvd, device="cuda", generator=gen)
        kv.append_rows(k, v, 0)
        caches.append(kv)
    q = torch.randn(n_head * head_dim, device="cuda", generator=gen)
    out = torch.zeros_like(q)
    us = _graph_time(torch, [lambda kv=caches[i % ncache]: kv.attention(q, n_head, seq, out)
                             for i in range(max(ncache, 16))], reps)
    for kv in caches:
        kv.free()
    alg = 2 * seq * kvd + 8 * seq + 2 * n_head * head_dim * 4
    return {"shape": {"n_head": n_head, "n_head_kv": n_head_kv, "head_dim": head_dim,
                      "seq": seq}, "algorithmic_bytes": alg, "rotating_caches": ncache,
            "us_per_call": round(us, 3), "kernels_per_call": 2,
            "gbs": round(alg / us / 1e3, 1), "frac_of_peak": round(alg / us / 1e3 / peak, 4)}


def case_layer_7b(ctx, torch, ssdllm, peak, n_layers=8, reps=10):
    """benchmark config 2: Llama-2-7B-shaped decoder layer decode step (Q4_0, INT8 KV at
    2048 positions), timed as a CUDA-graph decode step of an n_layers-deep model with a
    256-token vocab (embed + logits add < 0.1% of the bytes); per layer = step / n_layers."""
    cfg = dict(n_layers=n_layers, n_embd=4096, n_head=32, n_head_kv=32, head_dim=128,
               n_ff=11008, vocab=256, wtype=Q4_0, out_type=Q4_0, embd_type=Q4_0,
               kv_capacity=2048 + 4 * reps + 16, theta=1e4, eps=1e-5, tp_rank=0, tp_size=1)
    m = ssdllm.Model(ctx, **cfg)
    try:
        m.synth_weights(seed=7, std=0.02)
        m.synth_kv(seed=8, n=2048)
        stream = torch.cuda.ExternalStream(ssdllm_stream(ctx, ssdllm))
        m.decode_step(True)
        for _ in range(3):
            m.decode_step(True)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            m.decode_step(True)
        e1.record(stream)
        torch.cuda.synchronize()
        us_layer = e0.elapsed_time(e1) * 1e3 / reps / n_layers
        launches = m.launches_per_step()
    finally:
        m.free()
    E, F = 4096, 11008
    alg = int((4 * E * E + 3 * F * E) * Q40_BYTES) + 2 * 2049 * E + 8 * 2049 + 2 * E * 4
    return {"shape": "llama2-7b layer, Q4_0, INT8 KV 2048", "algorithmic_bytes": alg,
            "us_per_layer": round(us_layer, 3), "gbs": round(alg / us_layer / 1e3, 1),
            "frac_of_peak": round(alg / us_layer / 1e3 / peak, 4),
            "launches_per_layer": 6, "model_layers_timed": n_layers, "launches_per_step": launches}


def case_swiglu_70b(ctx, torch, ssdllm, peak, reps=10):
    """The decode step's dominant kernel alone: fused gate/up Q4_0 dequant-matvec with the
    FFN RMSNorm prologue and SwiGLU epilogue at the Llama-70B shape (2 x 28672 x 8192,
    264 MB per launch), 2 rotating weight sets."""
    E, F = 8192, 28672
    sets = []
    for i in range(2):
        wg = ssdllm.Weight.synth(ctx, Q4_0, 0, 700 + 2 * i, 0.02, E, 0, F, 0, E)
        wu = ssdllm.Weight.synth(ctx, Q4_0, 0, 701 + 2 * i, 0.02, E, 0, F, 0, E)
        sets.append((wg, wu))
    gen = torch.Generator("cuda").manual_seed(5)
    x = torch.randn(E, device="cuda", generator=gen)
    nw = 1 + 0.1 * torch.randn(E, device="cuda", generator=gen)
    act = torch.zeros(F, device="cuda")
    ctx.set_pdl(True)
    us = _graph_time(torch, [lambda s=sets[i % 2]: ssdllm.fused_swiglu(ctx, s[0], s[1], x, nw,
                                                                       1e-5, act)
                             for i in range(8)], reps)
    ctx.set_pdl(False)
    for wg, wu in sets:
        wg.free()
        wu.free()
    alg = int(2 * F * E * Q40_BYTES) + 2 * E * 4 + F * 4
    return {"shape": [2 * F, E], "algorithmic_bytes": alg, "us_per_launch": round(us, 3),
            "gbs": round(alg / us / 1e3, 1), "frac_of_peak": round(alg / us / 1e3 / peak, 4)}


def case_layer_70b(ctx, torch, ssdllm, peak, n_layers=4, reps=10):
    """One Llama-70B-shaped decoder layer at TP1 (Q4_0, INT8 KV at 4096 positions), timed
    as a CUDA-graph decode step of an n_layers-deep model with a 256-token vocab; per
    layer = step / n_layers (481 MB of weights + 8.4 MB of KV per layer)."""
    cfg = dict(CFG70B, n_layers=n_layers, vocab=256, kv_capacity=4096, tp_rank=0, tp_size=1)
    m = ssdllm.Model(ctx, **cfg)
    try:
        m.synth_weights(seed=7, std=0.02)
        m.synth_kv(seed=8, n=4096 - 4 * reps - 16)
        stream = torch.cuda.ExternalStream(ssdllm_stream(ctx, ssdllm))
        for _ in range(4):
            m.decode_step(True)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            m.decode_step(True)
        e1.record(stream)
        torch.cuda.synchronize()
        us_layer = e0.elapsed_time(e1) * 1e3 / reps / n_layers
    finally:
        m.free()
    E, F, kvd = 8192, 28672, 1024
    alg = int((2 * E * E + 2 * kvd * E + 3 * F * E) * Q40_BYTES) + 2 * 4096 * (kvd + 4) + 2 * E * 4
    return {"shape": "llama-70b layer, Q4_0, INT8 KV ~4040, TP1", "algorithmic_bytes": alg,
            "us_per_layer": round(us_layer, 3), "gbs": round(alg / us_layer / 1e3, 1),
            "frac_of_peak": round(alg / us_layer / 1e3 / peak, 4), "model_layers_timed": n_layers}


def case_prefill_l3_8b(ctx, torch, ssdllm, peak, reps=3):
    """benchmark config 3: layer-major batch prefill of 512 tokens through Llama-3-8B-shaped
    layers (hidden 4096, 32 q / 8 kv heads, FFN 14336, Q4_K weights, RoPE theta 5e5, causal
    attention over the INT8 cache), then the vocab matvec (128256) and argmax of the last
    token. Models of 1 and 3 layers are timed (weight splits prepared by an untimed first
    call); per layer = difference / 2. Useful FLOPs per layer = the GEMMs' 2 M N K + the
    causal attention's QK^T and PV; the tensor-core GEMMs execute 3 fp16 passes of each
    product (hi/lo operand splits) for fp32-level accuracy."""
    M, E, F, nh, nkv, hd, V = 512, 4096, 14336, 32, 8, 128, 128256
    toks = torch.randint(0, V, (M,), generator=torch.Generator().manual_seed(9)).numpy()
    times = {}
    for L in (1, 3):
        cfg = dict(n_layers=L, n_embd=E, n_head=nh, n_head_kv=nkv, head_dim=hd, n_ff=F, vocab=V,
                   wtype=12, out_type=12, embd_type=0, kv_capacity=M, theta=5e5, eps=1e-5,
                   tp_rank=0, tp_size=1)
        m = ssdllm.Model(ctx, **cfg)
        try:
            m.synth_weights(seed=21, std=0.02)
            m.set_position(0)
            m.prefill(toks)  # prepares the weight splits
            ts = []
            for _ in range(reps):
                m.set_position(0)
                t0 = time.perf_counter()
                m.prefill(toks)
                ts.append(time.perf_counter() - t0)
            times[L] = min(ts)
        finally:
            m.free()
    per_layer = (times[3] - times[1]) / 2
    gemm_flops = 2 * M * ((nh * hd + 2 * nkv * hd) * E + E * E + 2 * F * E + F * E)
    attn_flops = 2 * 2 * nh * hd * (M * (M + 1) // 2)
    tflops = (gemm_flops + attn_flops) / per_layer / 1e12
    tpk, _ = measured_tensor_peak()
    return {"shape": "llama3-8b layer, Q4_K, 512 tokens", "useful_flops_per_layer":
            gemm_flops + attn_flops, "ms_per_layer": round(per_layer * 1e3, 3),
            "prefill_ms_1_layer_incl_logits": round(times[1] * 1e3, 3),
            "tokens_per_s_per_layer": round(M / per_layer, 1), "tflops": round(tflops, 1),
            "frac_of_bf16_peak": round(tflops / tpk, 4), "mma_passes": 3}


def measure_batch16(ctx, torch, ssdllm, model, cfg, peak, steps=6, warmup=2):
    """benchmark config 5, continuous batch 16: the 16 slots of ssdllm.Batch over the model's
    weights, every slot's INT8 cache filled to PROMPT positions, one graph-captured step =
    one token for each of the 16 slots (layer-major, the weights streamed once per step)."""
    import numpy as np
    b = ssdllm.Batch(model, capacity=cfg["kv_capacity"])
    try:
        b.synth_kv(seed=11, n=PROMPT - steps - warmup - 2)
        stream = torch.cuda.ExternalStream(ssdllm_stream(ctx, ssdllm))
        b.step(np.arange(16, dtype=np.int32) * 997 % cfg["vocab"])
        for _ in range(warmup):
            b.step(None)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            lib_step(ssdllm, b)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        launches = b.launches_per_step()
    finally:
        b.free()
    wbytes = weight_bytes(cfg)
    kv_bytes = 16 * cfg["n_layers"] * PROMPT * (2 * cfg["n_head_kv"] * cfg["head_dim"] + 8)
    return {"workload": "llama70b_q4_0_decode_b16", "slots": 16, "context": PROMPT,
            "ms_per_step": round(ms, 3), "tokens_per_s": round(16 / (ms / 1e3), 1),
            "weight_stream_gbs": round(wbytes / (ms / 1e3) / 1e9, 1),
            "hbm_bytes_per_step": int(wbytes + kv_bytes),
            "frac_of_peak": round((wbytes + kv_bytes) / (ms / 1e3) / 1e9 / peak, 4),
            "launches_per_step": launches}


def lib_step(ssdllm, b):
    """One batch step without the host copy of the output tokens (device-timed region)."""
    ssdllm.check(ssdllm.lib().ssd_batch_step(b.h, None, None, 1))


def case_decode_b16_70b(ctx, torch, ssdllm, peak):
    """The 70B-shape model built for this case alone (39 GB of Q4_0 weights + 10.7 GB of
    slot caches)."""
    cfg = dict(CFG70B, tp_rank=0, tp_size=1)
    m = ssdllm.Model(ctx, **cfg)
    try:
        m.synth_weights(seed=0, std=0.02)
        return measure_batch16(ctx, torch, ssdllm, m, cfg, peak)
    finally:
        m.free()


def case_decode_b16_2l(ctx, torch, ssdllm, peak):
    """Continuous batch 16 on two Llama-70B-shaped layers (1.6 GB of weights): the small case
    that profiler captures of the batched kernels run (same kernels and shapes per layer)."""
    cfg = dict(CFG70B, n_layers=2, tp_rank=0, tp_size=1)
    m = ssdllm.Model(ctx, **cfg)
    try:
        m.synth_weights(seed=0, std=0.02)
        return measure_batch16(ctx, torch, ssdllm, m, cfg, peak)
    finally:
        m.free()


def _write_gguf_q4_0(path, n_layers, E, n_head, n_head_kv, F, vocab, seed=0):
    """A Llama-shaped GGUF file of synthetic Q4_0 blocks (random nibbles, f16 scales in
    [0.001, 0.003)) written tensor by tensor: the layout GgufFile::open reads
    (src/model/gguf.rs:233-315), alignment 32, ne0 = columns first."""
    import struct
    import numpy as np
    rng = np.random.default_rng(seed)
    hd = E // n_head
    kvd = n_head_kv * hd
    mats = [("attn_q", E, E), ("attn_k", kvd, E), ("attn_v", kvd, E), ("attn_output", E, E),
            ("ffn_gate", F, E), ("ffn_up", F, E), ("ffn_down", E, F)]
    tensors = [("token_embd.weight", [E, vocab], Q4_0), ("output_norm.weight", [E], 0),
               ("output.weight", [E, vocab], Q4_0)]
    for l in range(n_layers):
        tensors += [(f"blk.{l}.attn_norm.weight", [E], 0), (f"blk.{l}.ffn_norm.weight", [E], 0)]
        tensors += [(f"blk.{l}.{n}.weight", [c, r], Q4_0) for n, r, c in mats]
    size = lambda dims, t: (dims[0] * 4 if t == 0 else
                            (dims[0] // 32) * 18 * (dims[1] if len(dims) > 1 else 1))
    S = lambda x: struct.pack("<Q", len(x)) + x.encode()
    md = [("general.architecture", 8, "llama"), ("llama.block_count", 4, n_layers),
          ("llama.embedding_length", 4, E), ("llama.feed_forward_length", 4, F),
          ("llama.attention.head_count", 4, n_head),
          ("llama.attention.head_count_kv", 4, n_head_kv)]
    hdr = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(md)))
    for k, t, v in md:
        hdr += S(k) + struct.pack("<I", t) + (S(v) if t == 8 else struct.pack("<I", v))
    off = 0
    for name, dims, t in tensors:
        hdr += S(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        hdr += struct.pack("<IQ", t, off)
        off = (off + size(dims, t) + 31) // 32 * 32
    hdr += b"\0" * ((-len(hdr)) % 32)
    with open(path, "wb") as f:
        f.write(hdr)
        pos = 0
        for name, dims, t in tensors:
            n = size(dims, t)
            if t == 0:
                data = (1 + 0.1 * rng.standard_normal(dims[0])).astype(np.float32).tobytes()
            else:
                blk = rng.integers(0, 256, size=(n // 18, 18), dtype=np.uint8)
                d = rng.uniform(0.001, 0.003, n // 18).astype(np.float16)
                blk[:, :2] = d.view(np.uint8).reshape(-1, 2)
                data = blk.tobytes()
            f.write(data)
            pos += n
            pad = (-pos) % 32
            f.write(b"\0" * pad)
            pos += pad


def case_stream_7b(ctx, torch, ssdllm, peak, slots=8, lookahead=2, tokens=6):
    """SSD -> HBM streaming tier (ssd_stream_*) on a Llama-2-7B-shaped Q4_0 model (32 layers,
    3.6 GB of layer matrices) written as a GGUF file to the local disk, decoded with an HBM
    budget of `slots` layer slots and `lookahead` layers ahead: every layer is read again each
    token (LRU over 32 layers with 8 slots), so tokens/s x layer bytes is the file -> pinned
    host -> HBM rate. The file was just written, so the reads come from the host page cache:
    this times the host-to-HBM path, not a disk. Host clock over `tokens` tokens after one."""
    import tempfile
    d = tempfile.mkdtemp(prefix="ssd_stream_")
    path = os.path.join(d, "llama7b_q4_0.gguf")
    try:
        _write_gguf_q4_0(path, 32, 4096, 32, 32, 11008, 32000)
        cfg = ssdllm.GgufFile(path).model_config(kv_capacity=64)
        m = ssdllm.Model(ctx, **cfg)
        try:
            probe = ssdllm.Stream(m, path, 1 << 40, 0)
            slot_bytes = probe.stats()["slot_bytes"]
            probe.close()
            st = ssdllm.Stream(m, path, slots * slot_bytes, lookahead)
            try:
                m.set_position(0)
                t = st.decode_token(1)
                s0 = st.stats()
                h0 = time.perf_counter()
                for _ in range(tokens):
                    t = st.decode_token(t)
                dt = time.perf_counter() - h0
                s1 = st.stats()
            finally:
                st.close()
        finally:
            m.free()
        moved = s1["bytes_read"] - s0["bytes_read"]
        return {"workload": "llama7b_q4_0_streamed", "layers": 32, "hbm_slots": slots,
                "lookahead": lookahead, "slot_bytes": slot_bytes,
                "layer_bytes_per_token": moved // tokens,
                "tokens_per_s": round(tokens / dt, 3),
                "stream_gbs": round(moved / dt / 1e9, 2),
                "loads_per_token": (s1["loads"] - s0["loads"]) / tokens,
                "prefetch_hits": s1["prefetch_hits"] - s0["prefetch_hits"],
                "source": "host page cache (file just written)"}
    finally:
        if os.path.exists(path):
            os.remove(path)
        os.rmdir(d)


def measured_tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["bf16_tflops"]), "measured bf16_tflops"
    return 1590.0, "fallback 1.59 PFLOP/s"


def case_mv_shapes(ctx, torch, ssdllm, peak, reps=10):
    """Every decode-step matvec of the Llama-70B shape (QKV + RoPE, o_proj + residual,
    gate/up + SwiGLU, down + residual) at the row/column shards of TP = 1, 2, 4, 8, timed
    with each of the library's two matvec kernels: the FMA kernel (the default) and the
    integer tensor-core kernel (SSD_MV_IMPL=tc, where it covers the shape). Weights
    rotate over copies totalling more than 2x L2; launches are graph-captured with PDL."""
    import os
    E, F, HQ, HKV = 8192, 28672, 8192, 1024
    gen = torch.Generator("cuda").manual_seed(9)
    out = {}
    tid = [2000]

    def synth(rows, cols):
        tid[0] += 1
        return ssdllm.Weight.synth(ctx, Q4_0, 0, tid[0], 0.02, cols, 0, rows, 0, cols)

    for tp in (1, 2, 4, 8):
        hq, ff, ecol, fcol = HQ // tp, F // tp, E // tp, F // tp
        hkv = HKV // tp  # K / V sharded by heads
        kinds = {
            "qkv": (hq + 2 * hkv) * E, "o_proj": E * ecol, "gate_up": 2 * ff * E, "down": E * fcol,
        }
        for kind, nw in kinds.items():
            wbytes = nw * Q40_BYTES
            copies = min(16, max(2, -(-int(2.2 * L2_BYTES) // int(wbytes))))
            x = torch.randn(E if kind in ("qkv", "gate_up") else (ecol if kind == "o_proj" else fcol),
                            device="cuda", generator=gen)
            nw_ = 1 + 0.1 * torch.randn(E, device="cuda", generator=gen)
            if kind == "qkv":
                ws = [(synth(hq, E), synth(hkv, E), synth(hkv, E)) for _ in range(copies)]
                q, k, v = (torch.zeros(n, device="cuda") for n in (hq, hkv, hkv))
                mk = lambda w: (lambda: ssdllm.fused_qkv_rope(ctx, *w, x, nw_, 1e-5, 128, 77, 5e5,
                                                              q, k, v))
                alg = wbytes + E * 4 + (hq + 2 * hkv) * 4
            elif kind == "gate_up":
                ws = [(synth(ff, E), synth(ff, E)) for _ in range(copies)]
                act = torch.zeros(ff, device="cuda")
                mk = lambda w: (lambda: ssdllm.fused_swiglu(ctx, w[0], w[1], x, nw_, 1e-5, act))
                alg = wbytes + E * 4 + ff * 4
            else:
                cols = ecol if kind == "o_proj" else fcol
                ws = [(synth(E, cols),) for _ in range(copies)]
                base = torch.randn(E, device="cuda", generator=gen)
                y = torch.zeros(E, device="cuda")
                mk = lambda w: (lambda: ssdllm.matvec_residual(ctx, w[0], x, base, y))
                alg = wbytes + cols * 4 + 2 * E * 4
            res = {}
            ctx.set_pdl(True)
            for impl in ("tc", "fma"):
                os.environ["SSD_MV_IMPL"] = impl
                n = max(copies, 32 // copies * copies)
                us = _graph_time(torch, [mk(ws[i % copies]) for i in range(n)], reps)
                res[impl] = {"us": round(us, 3), "frac_of_peak": round(alg / us / 1e3 / peak, 4)}
            os.environ.pop("SSD_MV_IMPL", None)
            ctx.set_pdl(False)
            for w in ws:
                for t in w:
                    t.free()
            out[f"tp{tp}_{kind}"] = {"bytes": int(alg), **res}
    return out


CASES = {
    "q4_0_4096x4096": lambda c, t, s, p: case_matvec(c, t, s, p, Q4_0, 4096, 4096),
    "q8_0_11008x4096": lambda c, t, s, p: case_matvec(c, t, s, p, 8, 11008, 4096),
    "q8_0_4096x11008": lambda c, t, s, p: case_matvec(c, t, s, p, 8, 4096, 11008),
    "q4_k_11008x4096": lambda c, t, s, p: case_matvec(c, t, s, p, 12, 11008, 4096),
    "q4_k_4096x11008": lambda c, t, s, p: case_matvec(c, t, s, p, 12, 4096, 11008),
    "q6_k_11008x4096": case_matvec_q6k,
    "bf16_11008x4096": case_matvec_dense16,
    "f16_11008x4096": lambda c, t, s, p: case_matvec_dense16(c, t, s, p, wtype=1),
    "swiglu_q4_0_70b": case_swiglu_70b,
    "attn_int8_70b_4096": case_attention,
    # one rank's heads at TP2 / TP8 (K/V sharded by heads)
    "attn_int8_70b_tp2": lambda c, t, s, p: case_attention(c, t, s, p, n_head=32, n_head_kv=4),
    "attn_int8_70b_tp8": lambda c, t, s, p: case_attention(c, t, s, p, n_head=8, n_head_kv=1),
    "layer_7b_q4_0": case_layer_7b,
    "layer_70b_q4_0": case_layer_70b,
    "prefill_l3_8b_q4_k": case_prefill_l3_8b,
    "mv_shapes_70b": case_mv_shapes,
    "decode_b16_70b": case_decode_b16_70b,
    "decode_b16_2l": case_decode_b16_2l,
    "stream_7b_q4_0": case_stream_7b,
}
# measured on every default run (mv_shapes_70b, a kernel-selection study, only by --case;
# decode_b16_70b is measured on the headline run's own model; decode_b16_2l is the profiler's
# small case; stream_7b_q4_0 writes a 3.7 GB file, only by --case)
DEFAULT_CASES = [n for n in CASES if n not in ("mv_shapes_70b", "decode_b16_70b", "decode_b16_2l",
                                                "stream_7b_q4_0")]


def run_cases(names, peak):
    import torch
    import ssdllm
    ctx = ssdllm.Context(torch.cuda.current_device())
    return {n: CASES[n](ctx, torch, ssdllm, peak) for n in names}


def run_case_cli(args):
    """--case NAME[,NAME...]: one kernel configuration alone (parity configs 0-2 and the
    attention kernel), for profiling and the per-kernel table; prints one JSON line."""
    import torch
    torch.cuda.set_device(0)
    peak, src = measured_peaks()
    names = DEFAULT_CASES if args.case == "all" else args.case.split(",")
    res = run_cases(names, peak)
    print(json.dumps({"cases": res, "peak_gbs": peak, "peak_source": src}), flush=True)
    return 0


def time_dominant_kernel(ctx, model, torch, ssdllm, cfg, world):
    """The fused gate/up + SwiGLU dequant-matvec on every layer's own weights, in layer
    order (each launch reads a different 2 x ff_local x 8192 Q4_0 slab, never in L2)."""
    E = cfg["n_embd"]
    ff_local = cfg["n_ff"] // world
    x = torch.randn(E, device="cuda")
    act = torch.zeros(ff_local, device="cuda")
    ws = [(model.weight("ffn_gate", l), model.weight("ffn_up", l), model.norm("ffn_norm", l))
          for l in range(cfg["n_layers"])]

    class _T:  # borrowed device pointer as a tensor-like for the binding
        def __init__(self, p):
            self.p = p

        def data_ptr(self):
            return self.p

    ctx.set_pdl(True)
    for wg, wu, nw in ws[:2]:
        ssdllm.fused_swiglu(ctx, wg, wu, x, _T(nw), cfg["eps"], act)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for wg, wu, nw in ws:
        ssdllm.fused_swiglu(ctx, wg, wu, x, _T(nw), cfg["eps"], act)
    e1.record()
    torch.cuda.synchronize()
    ctx.set_pdl(False)
    us = e0.elapsed_time(e1) * 1e3 / len(ws)
    alg = 2 * ff_local * E * Q40_BYTES + 2 * E * 4 + ff_local * 4
    return us, alg


def run_cuda(args):
    import numpy as np  # noqa: F401
    import torch
    import torch.distributed as dist
    import ssdllm

    rank, world, local = env_rank()
    assert world == args.gpus, f"WORLD_SIZE {world} != --gpus {args.gpus}"
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    peak, peak_src = measured_peaks()
    cfg = dict(CFG70B)
    if args.layers:
        cfg["n_layers"] = args.layers
    ctx = ssdllm.Context(local)
    model = ssdllm.Model(ctx, **cfg, tp_rank=rank, tp_size=world)
    clk = None
    try:
        if world > 1:
            obj = [ssdllm.Model.unique_id() if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0)
            model.tp_init(obj[0])
            if args.allreduce == "p2p":  # partial sums over NVLink peer memory
                hs = [None] * world
                dist.all_gather_object(hs, model.p2p_handle())
                model.p2p_open(hs)
        # clock sampler running from here (it takes ~0.5 s to start sampling); mark() brackets
        # the timed region below
        clk = Clocks(list(range(world)) if rank == 0 else [])
        clk.__enter__()
        t0 = time.perf_counter()
        model.synth_weights(seed=0, std=0.02)
        total = args.warmup + 2 * args.steps + 1
        prompt = min(PROMPT, cfg["kv_capacity"] - total)
        assert prompt > 0, "too many steps for the 4096-position cache"
        model.synth_kv(seed=1, n=prompt)
        setup_s = time.perf_counter() - t0
        stream = torch.cuda.ExternalStream(ssdllm_stream(ctx, ssdllm))
        model.decode_token(1, use_graph=True)  # capture the graph
        for _ in range(args.warmup - 1):
            model.decode_step(True)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        clk.mark(0)
        e0.record(stream)
        for _ in range(args.steps):
            model.decode_step(True)
        e1.record(stream)
        torch.cuda.synchronize()
        clk.mark(1)
        clk.__exit__()
        if world > 1:
            dist.barrier()
        ms = e0.elapsed_time(e1)
        # e2e: host token in, host token out through the public API, every step, timed on
        # the host clock (each call synchronises on its token copy back)
        t = 5
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        h0 = time.perf_counter()
        for _ in range(args.steps):
            t = model.decode_token(t, use_graph=True)
        ms_e2e = (time.perf_counter() - h0) * 1e3
        if world > 1:
            tt = torch.tensor([ms, ms_e2e], device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms, ms_e2e = float(tt[0]), float(tt[1])
        launches = model.launches_per_step()
        dom_us, dom_bytes = time_dominant_kernel(ctx, model, torch, ssdllm, cfg, world)
        if world > 1:
            tt = torch.tensor([dom_us], device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            dom_us = float(tt[0])
        b16 = None
        if world == 1 and not args.no_kernels:  # config 5's continuous batch 16, same model
            b16 = measure_batch16(ctx, torch, ssdllm, model, cfg, peak)
        k0 = run_cases(DEFAULT_CASES, peak) if rank == 0 and not args.no_kernels else None
        clocks = clk.summary() if rank == 0 else None
    finally:
        if clk is not None:
            clk.__exit__()  # stops the sampler on every path (a second call is a no-op)
        model.free()  # releases the graph holding NCCL calls before the process group
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as ora
        ora.build()
        threads = os.cpu_count() or 1
        t_tok, t_layers, _ = cpu_token_time(cfg, 3, threads)
        cpu = {"value": 1.0 / t_tok, "unit": "tokens/s", "cores": threads, "kind": "port",
               "cpu": cpu_model_name(),
               "sample": f"{len(t_layers)} timed 70B-shape layer steps (packed Q4_0, INT8 KV "
                         f"at {PROMPT}) x 80 layers + vocab matvec; extrapolated"}
        if k0:  # the per-kernel cases' own CPU baselines
            for name, v in cpu_case_baselines(threads).items():
                if name in k0:
                    k0[name]["cpu_baseline"] = v
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    tok_s = args.steps / (ms / 1e3)
    dom_gbs = dom_bytes / dom_us / 1e3
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        traffic = json.load(open(tp)).get(f"swiglu_tp{world}")
    line = {
        "metric": "decode tokens/s (Llama-70B-shape Q4_0, batch 1)",
        "value": tok_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "llama70b_q4_0_decode_b1", "n_layers": cfg["n_layers"],
                   "hidden": 8192, "heads": 64, "kv_heads": 8, "ffn": 28672,
                   "vocab": 128256, "context": prompt, "kv": "int8", "tp": world,
                   "allreduce": args.allreduce if world > 1 else None,
                   "l2": "not flushed: 39 GB of weights per token >> 126 MB L2",
                   "weights_gb_per_gpu": round(weight_bytes(cfg) / world / 1e9, 2)},
        "e2e": {"value": args.steps / (ms_e2e / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4},
        "roofline": {"bound": "hbm", "kernel": "fused gate/up Q4_0 matvec + SwiGLU",
                     "achieved": dom_gbs, "peak": peak, "peak_source": peak_src,
                     "unit": "GB/s", "frac": dom_gbs / peak, "traffic": traffic,
                     "us_per_launch": dom_us, "algorithmic_bytes": dom_bytes,
                     "decode_weight_stream_gbs": weight_bytes(cfg) / world / (ms / args.steps)
                     / 1e6},
        "cpu_baseline": cpu,
        "decode_b16": b16,
        "gpu_launches": launches * args.steps,
        "clocks": clocks,
        "kernels": k0,
        "setup_s": setup_s,
    }
    print(json.dumps(line), flush=True)
    return 0


def weight_bytes(cfg):
    E, F, V = cfg["n_embd"], cfg["n_ff"], cfg["vocab"]
    kvd = cfg["n_head_kv"] * cfg["head_dim"]
    per_layer = (2 * E * E + 2 * kvd * E + 3 * F * E) * Q40_BYTES
    return cfg["n_layers"] * per_layer + V * E * Q40_BYTES


def ssdllm_stream(ctx, ssdllm):
    import ctypes
    s = ctypes.c_void_p()
    ssdllm.check(ssdllm.lib().ssd_ctx_stream(ctx.h, ctypes.byref(s)))
    return s.value


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["cuda", "reference"], default="cuda")
    ap.add_argument("--layers", type=int, default=0,
                    help="override n_layers (debug only; the headline uses 80)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--allreduce", choices=["p2p", "nccl"], default="p2p",
                    help="TP partial sums: in-kernel over NVLink peer memory, or ncclAllReduce")
    ap.add_argument("--no-kernels", action="store_true",
                    help="skip the per-kernel table (benchmark configs 0-2)")
    ap.add_argument("--case", default="",
                    help="run only kernel configuration(s) NAME[,NAME] or 'all': " +
                         ", ".join(CASES))
    args = ap.parse_args()
    if args.warmup < 1:
        args.warmup = 1
    if args.impl == "reference":
        return run_reference(args)
    if args.case:
        return run_case_cli(args)
    return run_cuda(args)


if __name__ == "__main__":
    sys.exit(main())
