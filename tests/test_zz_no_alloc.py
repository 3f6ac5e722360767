"""The allocation-free Gram accumulation (cdclq_gram_accumulate_device_noalloc) against the allocating one.

Some callers cannot call cudaMalloc where they accumulate a Hessian (a hook inside a framework whose
allocator owns the device memory, a runtime that forbids allocation after start-up).  The allocation-free
entry point keeps its scratch in a fixed array inside the library; this test checks, through the C ABI, that
two consecutive calls give exactly what cdclq_gram_accumulate_device gives (the Gram kernels are
bit-reproducible, so the tolerance is zero), that the shared scratch carries nothing from one call into the
next, and that a width above the scratch's capacity is refused.  The file is named to be collected last.
"""
import ctypes

import pytest

pytestmark = pytest.mark.gpu


def _call(fn_name, x, y, t, n, h, torch):
    import cdclq

    rc = getattr(cdclq.lib(), fn_name)(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()), t, n,
                                       ctypes.c_void_p(h.data_ptr()), ctypes.c_void_p(
                                           torch.cuda.current_stream().cuda_stream))
    cdclq._lib.check(rc)
    torch.cuda.synchronize()


@pytest.mark.parametrize("t,n,sym", [(5000, 1024, True), (3000, 700, False), (2048, 96, True)])
def test_noalloc_gram_matches_allocating_entry_point(gpu, t, n, sym):
    import torch

    g = torch.Generator(device="cuda")
    g.manual_seed(t + n)
    x = torch.randn(t, n, generator=g, device="cuda") * torch.exp(torch.randn(n, generator=g, device="cuda"))
    y = x if sym else torch.randn(t, n, generator=g, device="cuda")
    ref = torch.full((n, n), 0.5, dtype=torch.float64, device="cuda")
    _call("cdclq_gram_accumulate_device", x, y, t, n, ref, torch)
    # two calls in a row through the allocation-free entry point, each on a fresh accumulator
    for _ in range(2):
        out = torch.full((n, n), 0.5, dtype=torch.float64, device="cuda")
        _call("cdclq_gram_accumulate_device_noalloc", x, y, t, n, out, torch)
        assert torch.equal(out, ref)


def test_noalloc_gram_rejects_width_above_capacity(gpu):
    import torch

    import cdclq

    n = 1025
    x = torch.zeros(4, n, device="cuda")
    h = torch.zeros(n, n, dtype=torch.float64, device="cuda")
    rc = cdclq.lib().cdclq_gram_accumulate_device_noalloc(ctypes.c_void_p(x.data_ptr()),
                                                          ctypes.c_void_p(x.data_ptr()), 4, n,
                                                          ctypes.c_void_p(h.data_ptr()), None)
    assert rc == -3
    assert "exceeds the allocation-free scratch" in cdclq.lib().cdclq_last_error().decode()


def test_noalloc_gram_startup_call_with_no_tokens(gpu):
    """A start-up call with t = 0 (what a runtime that forbids later allocation makes once per device, so that the
    module and its scratch are loaded then) succeeds and leaves H untouched."""
    import torch

    n = 64
    x = torch.zeros(1, n, device="cuda")
    h = torch.full((n, n), 3.0, dtype=torch.float64, device="cuda")
    _call("cdclq_gram_accumulate_device_noalloc", x, x, 0, n, h, torch)
    assert bool((h == 3.0).all())
