"""The allocation-free RMSNorm-backward C entry point against the regular one.

Callers that cannot allocate device memory (memory pools they do not own, runtimes
without an allocator hook, applications that forbid cudaMalloc after start-up) use
``sv4_rmsnorm_bwd_noalloc``.  This test calls it through its exported C symbol and
checks dx and dw against the torch-facing ``rmsnorm_bwd`` entry point and against the
fp32 formula on two calls in a row (the second call reuses the shared scratch array the
first one left behind), and that repeating a call reproduces dw bit for bit.
It lives in its own file, collected last, so a failure here never hides other tests.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from saint_llm_b200 import _C

    lib = ctypes.CDLL(_C.__file__)
    fn = lib.sv4_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    err = lib.sv4_noalloc_error_string
    err.restype = ctypes.c_char_p
    err.argtypes = [ctypes.c_int]
    return fn, err


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def test_rmsnorm_bwd_noalloc_matches_regular_entry_point(cuda):
    from saint_llm_b200.ops import backend

    ext = backend.ext()
    fn, err = _lib()
    stream = torch.cuda.current_stream().cuda_stream
    for call, (rows, dim) in enumerate([(1000, 2048), (333, 512)]):
        torch.manual_seed(call)
        x = torch.randn(rows, dim, device=cuda, dtype=torch.bfloat16)
        dy = torch.randn(rows, dim, device=cuda, dtype=torch.bfloat16)
        w = torch.rand(dim, device=cuda) + 0.5
        y = torch.empty_like(x)
        rstd = torch.empty(rows, device=cuda)
        ext.rmsnorm_fwd(x, w, y, rstd, 1e-6)
        dx_ref = torch.empty_like(x)
        dw_ref = ext.rmsnorm_bwd(dy, x, w, rstd, dx_ref)
        dx = torch.empty_like(x)
        dw = torch.full((dim,), float("nan"), device=cuda)
        rc = fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(),
                rows, dim, stream)
        torch.cuda.synchronize()
        assert rc == 0, err(rc).decode()
        assert _rel(dx, dx_ref) < 1e-2
        assert _rel(dw, dw_ref) < 1e-3
        # fp32 formula: dx = r (w dy - x r^2 mean(w dy x)), dw = sum_rows dy x r
        xf, gf, r = x.float(), dy.float(), rstd[:, None]
        dot = (w * gf * xf).mean(-1, keepdim=True)
        assert _rel(dx, r * (w * gf - xf * r * r * dot)) < 1e-2
        assert _rel(dw, (gf * xf * r).sum(0)) < 1e-4
        dw2 = torch.full_like(dw, float("nan"))
        rc = fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dw2.data_ptr(),
                rows, dim, stream)
        torch.cuda.synchronize()
        assert rc == 0 and torch.equal(dw, dw2), "dw is not reproducible"


def test_rmsnorm_bwd_noalloc_rejects_oversized_dim(cuda):
    fn, err = _lib()
    t = torch.zeros(16, device=cuda)
    rc = fn(t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), 1, 16384,
            torch.cuda.current_stream().cuda_stream)
    assert rc != 0 and b"8192" in err(rc)
