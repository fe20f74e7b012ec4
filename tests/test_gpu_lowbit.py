"""Low-bit formats on the GPU (Q3_K, Q2_K, IQ4_NL, IQ4_XS, IQ3_XXS, IQ3_S, IQ2_XXS, IQ2_XS in
the reference's block layouts; matvec_*_cpu, src/metal/compute.rs:793-1075, 1964-2240):

* the reference's own known-answer tests (compute.rs:2384-2977) through the host-slice
  entry point (MetalCompute::matvec_quantized, compute.rs:157-191);
* ssd_dequantize bit-exact with the oracle's element values, byte round trip;
* random blocks at model shapes against the oracle at rel. error 1e-3 (fp64 arbiter), plain
  and residual; the fused epilogues refuse these types."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import ssdllm  # noqa: E402
from oracle import oracle as ora  # noqa: E402

import _lowbit_kats as K  # noqa: E402
from _util import parity, rel_err  # noqa: E402

DEV = "cuda:0"


@pytest.fixture(scope="module")
def cc():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return ssdllm.CudaCompute.new(0)


@pytest.mark.parametrize("case", K.cases(), ids=lambda c: c["name"])
def test_reference_kats(cc, case):
    y = cc.matvec_quantized(case["raw"], case["x"], case["rows"], case["cols"], case["type"])
    assert K.check(case, y), (case["name"], y)


@pytest.mark.parametrize("wtype", K.LOWBIT)
def test_dequant_bit_exact_and_round_trip(cc, wtype):
    rng = np.random.default_rng(100 + wtype)
    rows, cols = 37, 3 * 256
    raw = K.random_blocks(rng, wtype, rows, cols)
    w = ssdllm.Weight.upload(cc.ctx, raw, wtype, rows, cols)
    assert np.array_equal(w.download(), raw.ravel())
    out = torch.zeros(rows * cols, device=DEV)
    ssdllm.dequantize(cc.ctx, w, out)
    ref = ora.dequantize(raw, wtype, rows * cols)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("wtype", K.LOWBIT)
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (1000, 11008 // 256 * 256), (3, 256)])
def test_matvec_matches_oracle(cc, wtype, rows, cols):
    rng = np.random.default_rng(rows + cols + wtype)
    raw = K.random_blocks(rng, wtype, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    w = ssdllm.Weight.upload(cc.ctx, raw, wtype, rows, cols)
    xd = torch.from_numpy(x).to(DEV)
    y = torch.zeros(rows, device=DEV)
    ssdllm.matvec(cc.ctx, w, xd, y)
    ref = ora.matvec_quantized(raw, x, rows, cols, wtype, threads=8)
    exact = ora.dequantize(raw, wtype, rows * cols).reshape(rows, cols).astype(np.float64) @ x
    assert parity(y.cpu().numpy(), ref, exact), rel_err(y.cpu().numpy(), ref)
    base = torch.from_numpy(rng.standard_normal(rows).astype(np.float32)).to(DEV)
    ssdllm.matvec_residual(cc.ctx, w, xd, base, y)
    assert rel_err(y.cpu().numpy(), base.cpu().numpy() + exact) <= 1e-3


def test_fused_epilogues_refuse_lowbit(cc):
    rng = np.random.default_rng(1)
    raw = K.random_blocks(rng, K.IQ2_XS, 256, 256)
    w = ssdllm.Weight.upload(cc.ctx, raw, K.IQ2_XS, 256, 256)
    x = torch.zeros(256, device=DEV)
    y = torch.zeros(256, device=DEV)
    nw = torch.ones(256, device=DEV)
    with pytest.raises(ssdllm.SsdError):
        ssdllm.fused_rmsnorm_matvec(cc.ctx, w, x, nw, 1e-5, y)
