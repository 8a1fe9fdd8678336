"""GPU test of the allocation-free LayerNorm backward C entry point.

The entry point ``kb_layernorm_backward_noalloc`` is called through its
exported C symbol (ctypes), not through the Python bindings, and its results
are compared against the regular ``norm_backward`` binding on two calls in a
row (the second call reuses the shared static scratch left by the first).
Around the second call the test also checks that PyTorch's allocator served
no allocation: the entry point takes its scratch from its own static array.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from koochak_b200 import _native_build
    from koochak_b200.ops import _ext

    _ext.native()  # loads the extension (and libtorch's dependencies) first
    lib = ctypes.CDLL(_native_build.SO_PATH)
    fn = lib.kb_layernorm_backward_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 8 + [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return fn


def _call(fn, dy, x, w, mean, rstd, dx, dw, db, M, C):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), mean.data_ptr(), rstd.data_ptr(), dx.data_ptr(),
              dw.data_ptr(), db.data_ptr(), M, C, stream)


@pytest.mark.parametrize("M,C", [(4096, 768), (333, 1024), (2048, 4096)])
def test_noalloc_layernorm_backward_matches(M, C):
    from koochak_b200.ops import functional as kf

    fn = _lib()
    torch.manual_seed(0)
    dev = torch.device("cuda", 0)
    w = torch.randn(C, device=dev) * 0.5 + 1.0
    b = torch.randn(C, device=dev) * 0.1
    for trial in range(2):
        x = torch.randn(M, C, device=dev) * (1.0 + trial)
        dy = torch.randn(M, C, device=dev).to(torch.bfloat16)
        _, mean, rstd = kf.norm_forward(x, w, b, 1e-5, rms=False, out_dtype=torch.bfloat16)
        dx_ref, dw_ref, db_ref = kf.norm_backward(dy, x, w, mean, rstd, rms=False)
        dx = torch.full_like(x, float("nan"))
        dw = torch.full((C,), float("nan"), device=dev)
        db = torch.full((C,), float("nan"), device=dev)
        torch.cuda.synchronize()
        before = torch.cuda.memory_stats(dev).get("allocation.all.allocated", 0)
        rc = _call(fn, dy, x, w, mean, rstd, dx, dw, db, M, C)
        torch.cuda.synchronize()
        after = torch.cuda.memory_stats(dev).get("allocation.all.allocated", 0)
        assert rc == 0, f"entry point returned {rc}"
        assert after == before, f"the call allocated through PyTorch ({after - before} allocations)"
        torch.testing.assert_close(dx, dx_ref, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(dw, dw_ref, rtol=1e-4, atol=1e-3)
        torch.testing.assert_close(db, db_ref, rtol=1e-4, atol=1e-3)


def test_noalloc_rejects_oversize_rows():
    fn = _lib()
    dev = torch.device("cuda", 0)
    M, C = 8, 8192
    t = torch.zeros(M, C, device=dev)
    v = torch.zeros(C, device=dev)
    r = torch.zeros(M, device=dev)
    dy = torch.zeros(M, C, device=dev, dtype=torch.bfloat16)
    assert _call(fn, dy, t, v, r, r, t, v, v, M, C) == -2
    assert _call(fn, dy, t, v, r, r, t, v, v, M, 6) == -1
