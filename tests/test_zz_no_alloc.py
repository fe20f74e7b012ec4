"""GPU test of ssd_attention_int8_noalloc, the attention entry point that allocates
no device memory.

Who needs it: callers that may not call cudaMalloc/cudaFree at the time they run
attention, such as code running while another part of the process captures a CUDA
graph, hosts whose framework owns the device allocator, or loops that must never
block in the driver. The variant keeps its split-K partials in a fixed device array
inside the library instead of the context's growable scratch buffer.

The test calls both entry points through the C ABI on the same INT8 cache and query
and requires the same output within the parity tolerance of the other GPU tests, on
two calls in a row (the second one shorter, so stale partials left in the shared
array by the first call would show). It also checks that a warm call leaves the
device's free memory unchanged and that an oversized call is refused with
SSD_ERR_SHAPE. The file name sorts last so that a run stopping at the first failure
has run every other test already; it also passes on its own in a fresh process.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import ssdllm  # noqa: E402

from _util import rel_err  # noqa: E402

TOL = 1e-3
DEV = "cuda:0"


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return ssdllm.Context(0)


def _filled_cache(ctx, capacity, n_head_kv, head_dim, seed):
    kv = ssdllm.KvCache(ctx, capacity, n_head_kv, head_dim)
    g = torch.Generator(DEV).manual_seed(seed)
    k = torch.randn(capacity, n_head_kv * head_dim, device=DEV, generator=g)
    v = torch.randn(capacity, n_head_kv * head_dim, device=DEV, generator=g)
    kv.append_rows(k, v, 0)
    torch.cuda.synchronize()
    return kv


def test_noalloc_attention_matches_attention_int8_on_two_calls(ctx):
    n_head, n_head_kv, head_dim, capacity = 16, 4, 128, 1200
    kv = _filled_cache(ctx, capacity, n_head_kv, head_dim, seed=11)
    try:
        g = torch.Generator(DEV).manual_seed(12)
        for call, seq_len in enumerate((1100, 257)):
            q = torch.randn(n_head * head_dim, device=DEV, generator=g)
            ref = torch.zeros_like(q)
            got = torch.full_like(q, float("nan"))
            kv.attention(q, n_head, seq_len, ref)
            torch.cuda.synchronize()
            free_before = torch.cuda.mem_get_info()[0]
            kv.attention_noalloc(q, n_head, seq_len, got)
            torch.cuda.synchronize()
            free_after = torch.cuda.mem_get_info()[0]
            r, y = ref.cpu().numpy(), got.cpu().numpy()
            assert np.all(np.isfinite(y)), f"call {call}: non-finite output"
            err = rel_err(y, r)
            assert err <= TOL, f"call {call} (seq {seq_len}): rel err {err}"
            if call == 1:  # warm: the device address lookup is done, nothing may allocate
                assert free_after == free_before, (free_before, free_after)
    finally:
        kv.free()


def test_noalloc_attention_rejects_sizes_beyond_its_buffer(ctx):
    # 64 heads x 16384 positions x (128 + 2) floats > 1,048,576: refused on the host
    kv = ssdllm.KvCache(ctx, 16384, 8, 128)
    try:
        q = torch.zeros(64 * 128, device=DEV)
        out = torch.zeros_like(q)
        with pytest.raises(ssdllm.SsdError) as e:
            kv.attention_noalloc(q, 64, 16384, out)
        assert e.value.status == 3  # SSD_ERR_SHAPE
        kv.attention_noalloc(q, 64, 16128, out)  # the stated maximum still runs
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
    finally:
        kv.free()
