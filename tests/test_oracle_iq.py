"""CPU pins of the oracle's low-bit formats (Q3_K, Q2_K, IQ4_NL, IQ4_XS, IQ3_XXS, IQ3_S,
IQ2_XXS, IQ2_XS; oracle/oracle_iq.c restating src/metal/compute.rs:793-1075, 1964-2240):

* the reference's own known-answer tests (compute.rs:2384-2977) with their tolerances;
* the lattice tables of iq_grids.h, expanded to the reference's u64 / u32 entries, against
  the SHA-256 of the reference's tables (tests/golden/iq_grids.sha256, written by
  gen_iq_grids.py from the reference source) and the entries its tests name
  (compute.rs:2849-2861, 2912-2917, 2953-2958);
* dequantize against matvec: the oracle's row sums equal an fp64 dot of its dequantized
  weights within fp32 rounding, on random blocks."""
import hashlib
import os
import re

import numpy as np
import pytest

from oracle import oracle as ora

import _lowbit_kats as K

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GRIDS = os.path.join(ROOT, "ssd-llm_b200", "csrc", "iq_grids.h")


def grids():
    text = open(GRIDS).read()
    vals = {n: [int(v) for v in re.search(n + r"\[\d+\] = \{(.*?)\};", text).group(1).split(",")
                if v.strip()] for n in ("kIq2Vals", "kIq3xxsVals", "kIq3sVals")}
    out = {}
    for name, nbytes, alpha, bits in (("kIq2xxsGrid", 8, "kIq2Vals", 2),
                                      ("kIq2xsGrid", 8, "kIq2Vals", 2),
                                      ("kIq3xxsGrid", 4, "kIq3xxsVals", 3),
                                      ("kIq3sGrid", 4, "kIq3sVals", 3)):
        body = re.search(name + r"\[\d+\] = \{(.*?)\};", text, re.S).group(1)
        codes = [int(v, 16) for v in re.findall(r"0x[0-9a-f]+", body)]
        out[name] = ([sum(vals[alpha][(c >> (bits * j)) & ((1 << bits) - 1)] << (8 * j)
                          for j in range(nbytes)) for c in codes], nbytes)
    return out


def test_grids_match_the_reference_tables():
    g = grids()
    h = hashlib.sha256()
    for name in ("kIq2xxsGrid", "kIq2xsGrid", "kIq3xxsGrid", "kIq3sGrid"):
        vals, nbytes = g[name]
        for v in vals:
            h.update(v.to_bytes(nbytes, "little"))
    assert h.hexdigest() == open(os.path.join(ROOT, "tests", "golden", "iq_grids.sha256")).read().strip()
    assert len(g["kIq2xxsGrid"][0]) == 256 and len(g["kIq2xsGrid"][0]) == 512
    assert len(g["kIq3xxsGrid"][0]) == 256 and len(g["kIq3sGrid"][0]) == 512
    # the entries the reference's tests check
    assert g["kIq3xxsGrid"][0][0] == 0x04040404 and g["kIq3xxsGrid"][0][255] == 0x3e341c04
    assert g["kIq3sGrid"][0][0] == 0x01010101 and g["kIq3sGrid"][0][511] == 0x0f0f0101
    assert g["kIq2xxsGrid"][0][0] == 0x0808080808080808
    assert g["kIq2xxsGrid"][0][255] == 0x2b2b2b1908081908
    assert g["kIq2xsGrid"][0][0] == 0x0808080808080808
    assert g["kIq2xsGrid"][0][511] == 0x2b2b2b2b2b2b2b2b


@pytest.mark.parametrize("case", K.cases(), ids=lambda c: c["name"])
def test_reference_kats(case):
    y = ora.matvec_quantized(case["raw"], case["x"], case["rows"], case["cols"], case["type"])
    assert K.check(case, y), (case["name"], y)


@pytest.mark.parametrize("wtype", K.LOWBIT)
def test_row_bytes_and_dequant_against_matvec(wtype):
    rng = np.random.default_rng(wtype)
    bs, bb = K.BLOCK[wtype]
    rows, cols = 5, 2 * 256
    assert ora.row_bytes(wtype, cols) == cols // bs * bb
    raw = K.random_blocks(rng, wtype, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    w = ora.dequantize(raw, wtype, rows * cols).reshape(rows, cols)
    assert np.all(np.isfinite(w)) and np.any(w != 0)
    y = ora.matvec_quantized(raw, x, rows, cols, wtype)
    ref = w.astype(np.float64) @ x
    assert np.max(np.abs(y - ref)) <= 1e-4 * np.max(np.abs(w) @ np.abs(x))
    # threads give the same bits
    assert np.array_equal(ora.matvec_quantized(raw, x, rows, cols, wtype, threads=3), y)
