"""The allocation-free attention entry point, for callers that cannot allocate device memory.

Some hosts cannot let a library call cudaMalloc (their pool already owns the GPU's memory, or the
implied device-wide synchronisation is unacceptable), so satori_grouped_attention_noalloc keeps its
split-K scratch in a fixed array inside the library.  This test calls it through the C ABI, twice in
a row on different inputs for each kernel family (the TMA streaming kernel at head_dim 128 with 7
query heads per KV head, and the plain-load partial kernel at head_dim 64), and checks:

* each result equals satori_grouped_attention_device's bit for bit (same kernels, same split count;
  only the scratch buffer differs);
* the first call of each family is within the attention tolerance used throughout the suite,
  1e-5 relative + 1e-6 absolute, of the oracle's FP64 GroupedAttention;
* warm calls leave the device's free memory unchanged (they allocate nothing);
* a shape too large for the fixed array is refused.

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


@pytest.mark.parametrize("qh,kvh,hd", [(28, 4, 128), (8, 8, 64)])
def test_noalloc_matches_context_entry_point_twice(env, oracle_lib, qh, kvh, hd):
    sat, _lib, torch = env
    L = _lib.lib()
    ctx = sat.Context(0)
    for call, T in enumerate((4096, 777)):
        q, k, v = _inputs(torch, 100 + call + hd, qh, kvh, hd, T)
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
        a = out_noalloc.cpu().numpy()
        b = out_ref.cpu().numpy()
        assert np.all(np.isfinite(a)), call
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (call, float(np.abs(a - b).max()))
        if call == 0:
            ref = oracle_lib.grouped_attention(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), qh, kvh, hd, T,
                                               threads=8).astype(np.float64)
            err = np.abs(a.astype(np.float64) - ref)
            assert np.all(err <= TOL_REL * np.abs(ref) + TOL_ABS), float(err.max())
    ctx.close()


def test_noalloc_allocates_nothing(env):
    sat, _lib, torch = env
    L = _lib.lib()
    qh, kvh, hd, T = 28, 4, 128, 2048
    q, k, v = _inputs(torch, 7, qh, kvh, hd, T)
    out = torch.empty(qh * hd, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(L.satori_grouped_attention_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), qh, kvh, hd, T,
                                                  out.data_ptr(), stream), "noalloc warm-up")
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        _lib.check(L.satori_grouped_attention_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), qh, kvh, hd, T,
                                                      out.data_ptr(), stream), "noalloc")
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before


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


def test_noalloc_on_two_devices_in_one_process(env):
    """The shared-memory opt-in of the attention kernels is held per device: a call on device 1 after one
    on device 0 (one process, one library) still launches, and gives the same bits as device 0."""
    sat, _lib, torch = env
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    L = _lib.lib()
    qh, kvh, hd, T = 28, 4, 128, 1500
    outs = []
    for dev in (0, 1):
        with torch.cuda.device(dev):
            g = torch.Generator(device="cuda").manual_seed(5)
            q = torch.randn(qh * hd, generator=g, device="cuda")
            k = torch.randn(T * kvh * hd, generator=g, device="cuda")
            v = torch.randn(T * kvh * hd, generator=g, device="cuda")
            out = torch.full((qh * hd,), float("nan"), device="cuda")
            torch.cuda.synchronize()
            _lib.check(L.satori_grouped_attention_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), qh, kvh, hd, T,
                                                          out.data_ptr(), torch.cuda.current_stream().cuda_stream),
                       f"noalloc on device {dev}")
            torch.cuda.synchronize()
            outs.append(out.cpu().numpy())
    assert np.all(np.isfinite(outs[1]))
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
