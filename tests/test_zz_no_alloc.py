"""The allocation-free attention entry point, for callers that cannot allocate device memory.

Some hosts cannot let a library call cudaMalloc (their pool already owns the GPU's memory, or the
implied device-wide synchronisation is unacceptable), so satori_grouped_attention_noalloc keeps its
split-K scratch in a fixed array inside the library.  This test calls it through the C ABI, twice in
a row on different inputs, and checks each result against satori_grouped_attention_device (which
uses a context-owned scratch buffer) within the attention tolerance used throughout the suite,
1e-5 relative + 1e-6 absolute.  It also checks that a shape too large for the fixed array is refused.

The file name makes pytest collect it last, so a run that stops at the first failure has already
run every other test; it also passes on its own in a fresh process.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_REL, TOL_ABS = 1e-5, 1e-6


@pytest.fixture(scope="module")
def env():
    from satori_b200 import build
    build.build()
    import torch

    import satori_b200 as sat
    from satori_b200 import _lib
    return sat, _lib, torch


def _inputs(torch, seed, qh, kvh, hd, T):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(qh * hd, generator=g, device="cuda")
    k = torch.randn(T * kvh * hd, generator=g, device="cuda")
    v = torch.randn(T * kvh * hd, generator=g, device="cuda")
    return q, k, v


def test_noalloc_matches_context_entry_point_twice(env):
    sat, _lib, torch = env
    L = _lib.lib()
    ctx = sat.Context(0)
    qh, kvh, hd = 28, 4, 128
    for call, T in enumerate((4096, 777)):
        q, k, v = _inputs(torch, 100 + call, qh, kvh, hd, T)
        out_noalloc = torch.full((qh * hd,), float("nan"), device="cuda")
        out_ref = torch.full((qh * hd,), float("nan"), device="cuda")
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream().cuda_stream
        _lib.check(L.satori_grouped_attention_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), qh, kvh, hd, T,
                                                      out_noalloc.data_ptr(), stream), "noalloc")
        torch.cuda.synchronize()
        _lib.check(L.satori_grouped_attention_device(ctx.handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), qh, kvh,
                                                     hd, T, out_ref.data_ptr()), "device")
        ctx.synchronize()
        a = out_noalloc.cpu().numpy().astype(np.float64)
        b = out_ref.cpu().numpy().astype(np.float64)
        assert np.all(np.isfinite(a)), call
        assert np.all(np.abs(a - b) <= TOL_REL * np.abs(b) + TOL_ABS), (call, float(np.abs(a - b).max()))
    ctx.close()


def test_noalloc_rejects_shapes_beyond_its_fixed_scratch(env):
    sat, _lib, torch = env
    L = _lib.lib()
    q, k, v = (torch.zeros(8, device="cuda") for _ in range(3))
    out = torch.zeros(8, device="cuda")
    # 8192 heads x (256 + 2) floats of partial records = 2.1M floats: more than the fixed 1,048,576.
    # The size check runs before any launch, so the tiny buffers are never touched.
    status = L.satori_grouped_attention_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), 8192, 8192, 256, 1 << 20,
                                                out.data_ptr(), None)
    assert status == _lib.ERR_ARGUMENT
    assert "scratch" in _lib.last_error()
