"""
The allocation-free sum-of-squares entry point (``csrc/noalloc.h``), called through its exported C symbol.

It exists for callers that may not allocate device memory while they run (a frozen memory pool in a latency-critical
loop, a host callback, a plug-in that only receives raw pointers): its scratch is an array built into the library.
This file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from olmo_b200 import ops

    lib = ops.lib()
    lib.ob_sumsq_f32_noalloc.restype = ctypes.c_int
    lib.ob_sumsq_f32_noalloc_max_elements.restype = ctypes.c_longlong
    lib.ob_noalloc_strerror.restype = ctypes.c_char_p
    return lib


def _noalloc(lib, g, out, accumulate):
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib.ob_sumsq_f32_noalloc(
        ctypes.c_void_p(g.data_ptr()), ctypes.c_longlong(g.numel()), ctypes.c_void_p(out.data_ptr()), ctypes.c_int(int(accumulate)), stream
    )


def test_no_alloc_sumsq_matches_allocating_entry_point_twice_in_a_row():
    from olmo_b200.ops import kernels as k

    lib = _lib()
    torch.manual_seed(0)
    # two different sizes back to back: the second call must not be disturbed by partials the first one left behind
    for n in (3_000_001, 70_003):
        g = torch.randn(n, device="cuda")
        want = torch.zeros(1, device="cuda")
        k.sumsq(g, want)  # existing entry point: scratch from the caching allocator
        got = torch.full((1,), 5.0, device="cuda")
        before = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
        rc = _noalloc(lib, g, got, accumulate=False)
        after = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
        assert rc == 0, lib.ob_noalloc_strerror(rc)
        assert after == before  # nothing was requested from torch's allocator either
        torch.cuda.synchronize()
        assert torch.allclose(got, want, rtol=1e-4), (got.item(), want.item())
        exact = g.double().pow(2).sum().item()  # and both against a float64 sum
        assert abs(got.item() - exact) <= 2e-5 * exact, (got.item(), exact)
        rc = _noalloc(lib, g, got, accumulate=True)
        assert rc == 0
        torch.cuda.synchronize()
        assert torch.allclose(got, 2 * want, rtol=1e-4)


def test_no_alloc_sumsq_rejects_oversize_and_misaligned_input():
    lib = _lib()
    limit = lib.ob_sumsq_f32_noalloc_max_elements()
    assert limit == 8192 * (1 << 18)
    g = torch.ones(64, device="cuda")
    out = torch.zeros(1, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.ob_sumsq_f32_noalloc(ctypes.c_void_p(g.data_ptr()), ctypes.c_longlong(limit + 1), ctypes.c_void_p(out.data_ptr()), 0, stream)
    assert rc == -101 and b"exceeds" in lib.ob_noalloc_strerror(rc)  # refused before any launch
    rc = lib.ob_sumsq_f32_noalloc(ctypes.c_void_p(g.data_ptr() + 4), ctypes.c_longlong(8), ctypes.c_void_p(out.data_ptr()), 0, stream)
    assert rc == -102
    # null pointers are refused on the host: launching on them would fault the device
    assert lib.ob_sumsq_f32_noalloc(ctypes.c_void_p(g.data_ptr()), ctypes.c_longlong(8), ctypes.c_void_p(None), 0, stream) == -106
    assert lib.ob_sumsq_f32_noalloc(ctypes.c_void_p(None), ctypes.c_longlong(8), ctypes.c_void_p(out.data_ptr()), 0, stream) == -106
    torch.cuda.synchronize()
    assert out.item() == 0.0
    # exactly the documented maximum passes the size check (it is then refused for the null input, before any launch)
    assert lib.ob_sumsq_f32_noalloc(ctypes.c_void_p(None), ctypes.c_longlong(limit), ctypes.c_void_p(out.data_ptr()), 0, stream) == -106


def test_no_alloc_sumsq_of_nothing_is_zero():
    lib = _lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    out = torch.full((1,), 7.0, device="cuda")
    assert lib.ob_sumsq_f32_noalloc(ctypes.c_void_p(None), ctypes.c_longlong(0), ctypes.c_void_p(out.data_ptr()), 0, stream) == 0
    torch.cuda.synchronize()
    assert out.item() == 0.0
    out.fill_(7.0)
    assert lib.ob_sumsq_f32_noalloc(ctypes.c_void_p(None), ctypes.c_longlong(0), ctypes.c_void_p(out.data_ptr()), 1, stream) == 0
    torch.cuda.synchronize()
    assert out.item() == 7.0
