"""g4m_linear_run_noalloc (static-scratch form of g4m_linear_run) against
g4m_linear_run on the same resident linears: two calls in a row with
different inputs, both tensor-core and SIMT shapes, bit-identical outputs;
calls past the static scratch are rejected without launching.  Collected last
so it also runs after every other GPU test has used the context."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_ELEMS = 1 << 22


def _run(L, fn, h, x, rows, out):
    import torch
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    yd = torch.full((rows, out), float("nan"), dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = getattr(L, fn)(h, ctypes.c_void_p(xd.data_ptr()), rows, ctypes.c_void_p(yd.data_ptr()), ctypes.c_void_p(st))
    torch.cuda.synchronize()
    return rc, yd.cpu().numpy()


@pytest.mark.parametrize("bits,inp,out", [(0, 768, 768), (4, 1024, 1536), (8, 96, 40)])
def test_noalloc_matches_linear_run(ctx, native, syn, oracle, bits, inp, out):
    L = native.lib()
    rng = np.random.default_rng(bits + inp)
    if bits:
        w = syn.pack_codes(rng.integers(0, 1 << bits, (out, inp)), bits)
    else:
        w = rng.integers(-127, 128, (out, inp)).astype(np.int8)
    s = rng.uniform(0.002, 0.02, out).astype(np.float32)
    b = rng.standard_normal(out).astype(np.float32)
    h = ctypes.c_void_p()
    native.check(L.g4m_linear_prepare(ctx.h, 0, native.ptr(w), bits, out, inp, native.ptr(s), 0.0, 0.0,
                                      native.ptr(b), ctypes.byref(h)))
    try:
        for call, rows in enumerate((300, 77)):
            x = rng.standard_normal((rows, inp)).astype(np.float32)
            rc_a, ref = _run(L, "g4m_linear_run", h, x, rows, out)
            rc_b, got = _run(L, "g4m_linear_run_noalloc", h, x, rows, out)
            assert rc_a == 0 and rc_b == 0, native.last_error()
            assert np.isfinite(got).all()
            assert np.array_equal(ref, got), (call, np.abs(ref - got).max())
    finally:
        L.g4m_linear_free(h)


def test_noalloc_rejects_past_scratch(ctx, native, syn):
    L = native.lib()
    inp, out = 1024, 256
    w = np.ones((out, inp), np.int8)
    s = np.full(out, 0.01, np.float32)
    h = ctypes.c_void_p()
    native.check(L.g4m_linear_prepare(ctx.h, 0, native.ptr(w), 0, out, inp, native.ptr(s), 0.0, 0.0, None,
                                      ctypes.byref(h)))
    try:
        import torch
        rows = MAX_ELEMS // inp + 1
        xd = torch.zeros((rows, inp), dtype=torch.float32, device="cuda")
        yd = torch.zeros((rows, out), dtype=torch.float32, device="cuda")
        rc = L.g4m_linear_run_noalloc(h, ctypes.c_void_p(xd.data_ptr()), rows, ctypes.c_void_p(yd.data_ptr()), None)
        assert rc == 2 and "static scratch" in native.last_error()
        rows = MAX_ELEMS // inp
        x = np.ones((rows, inp), np.float32)
        rc, y = _run(L, "g4m_linear_run_noalloc", h, x, rows, out)
        assert rc == 0 and np.allclose(y, inp * 0.01)
    finally:
        L.g4m_linear_free(h)


def test_noalloc_allocates_nothing(ctx, native):
    """The point of the entry point: a call takes no device memory.  Free
    device memory is read before and after two calls at the largest row count
    on a freshly prepared linear (after one warm-up call, which looks up the
    scratch address).  The same measurement around a first g4m_linear_run on
    another fresh linear shows the drop that an allocating call causes."""
    import torch
    L = native.lib()
    inp, out = 1024, 256
    rows = MAX_ELEMS // inp
    rng = np.random.default_rng(11)
    w = rng.integers(-127, 128, (out, inp)).astype(np.int8)
    s = np.full(out, 0.01, np.float32)
    xd = torch.from_numpy(rng.standard_normal((rows, inp)).astype(np.float32)).cuda()
    yd = torch.empty((rows, out), dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    handles = []
    try:
        for _ in range(2):
            h = ctypes.c_void_p()
            native.check(L.g4m_linear_prepare(ctx.h, 0, native.ptr(w), 0, out, inp, native.ptr(s), 0.0, 0.0, None,
                                              ctypes.byref(h)))
            handles.append(h)
        call = lambda fn, h: getattr(L, fn)(h, ctypes.c_void_p(xd.data_ptr()), rows, ctypes.c_void_p(yd.data_ptr()),
                                            ctypes.c_void_p(st))
        assert call("g4m_linear_run_noalloc", handles[0]) == 0, native.last_error()
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        for _ in range(2):
            assert call("g4m_linear_run_noalloc", handles[0]) == 0, native.last_error()
        torch.cuda.synchronize()
        free1 = torch.cuda.mem_get_info()[0]
        assert free1 == free0, f"noalloc calls changed free device memory by {free0 - free1} bytes"
        assert call("g4m_linear_run", handles[1]) == 0, native.last_error()
        torch.cuda.synchronize()
        free2 = torch.cuda.mem_get_info()[0]
        assert free1 - free2 >= 2 * rows * inp * 2, "the free-memory probe did not see an allocating call"
    finally:
        for h in handles:
            L.g4m_linear_free(h)
