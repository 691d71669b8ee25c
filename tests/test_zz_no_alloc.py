"""The entry point that allocates no device memory (brain_norm_bwd_noalloc, csrc/no_alloc.h).

Some callers of this library cannot allocate device memory while they run (a C/C++ host linking
libbrain_kernels.so without PyTorch, or a server that reserved the whole GPU under a fixed
budget); they call brain_norm_bwd_noalloc, whose partial sums live in a fixed array inside the
library. This test calls that exported C symbol directly through ctypes and checks it against
the workspace-taking entry point brain_norm_bwd on two calls in a row (the second call reuses
the array left over from the first), for RMSNorm and LayerNorm, and checks the size limit.
The file name sorts last so a run that stops at the first failure has run everything else.
"""
import ctypes

import pytest
import torch

from brain_b200 import _native


def _sym(name):
    lib = _native.load("brain_kernels")
    f = getattr(lib, name)
    f.restype = ctypes.c_int
    return f


def _args(kind, dy, x, w, mean, rstd, dx, dw, db, M, D, dres=None, dw_f32=1, accumulate=0):
    p = lambda t: ctypes.c_void_p(t.data_ptr() if t is not None else 0)  # noqa: E731
    i64 = ctypes.c_int64
    return [ctypes.c_int(kind), p(dy), i64(D), p(x), i64(D), p(w), p(mean), p(rstd), p(dx), i64(D),
            p(dres), i64(D if dres is not None else 0), p(dw), p(db), ctypes.c_int(dw_f32), ctypes.c_int(accumulate)]


def _compare(kind, M, D, fused=False):
    """Run both entry points on the same inputs, twice in a row, and compare their outputs. ``fused``
    adds the residual gradient, accumulates into existing dw/db and writes them in bf16."""
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    noalloc = _sym("brain_norm_bwd_noalloc")
    ref_fn = _sym("brain_norm_bwd")
    parts = _sym("brain_norm_bwd_partials")
    wdt = torch.bfloat16 if fused else torch.float32
    for call in range(2):  # two calls in a row share (and reuse) the fixed scratch
        x = torch.randn(M, D, device="cuda", dtype=torch.bfloat16)
        dy = torch.randn(M, D, device="cuda", dtype=torch.bfloat16)
        dres = torch.randn(M, D, device="cuda", dtype=torch.bfloat16) if fused else None
        w = (torch.randn(D, device="cuda") * 0.1 + 1).bfloat16()
        xf = x.float()
        if kind == 1:
            mean = xf.mean(-1).contiguous()
            rstd = torch.rsqrt(((xf - mean[:, None]) ** 2).mean(-1) + 1e-5).contiguous()
        else:
            mean = None
            rstd = torch.rsqrt(xf.pow(2).mean(-1) + 1e-6).contiguous()
        dw_init = torch.randn(D, device="cuda").to(wdt)
        db_init = torch.randn(D, device="cuda").to(wdt)
        outs = []
        for which in ("noalloc", "workspace"):
            dx = torch.empty_like(x)
            dw = dw_init.clone() if fused else torch.empty(D, device="cuda", dtype=wdt)
            db = (db_init.clone() if fused else torch.empty(D, device="cuda", dtype=wdt)) if kind == 1 else None
            a = _args(kind, dy, x, w, mean, rstd, dx, dw, db, M, D, dres=dres, dw_f32=0 if fused else 1,
                      accumulate=1 if fused else 0)
            if which == "noalloc":
                rc = noalloc(*a, ctypes.c_int(M), ctypes.c_int(D), stream)
            else:
                P = parts(M)
                ws = torch.empty(2 * P * D, device="cuda", dtype=torch.float32)
                rc = ref_fn(*a, ctypes.c_void_p(ws.data_ptr()), ctypes.c_int(M), ctypes.c_int(D), stream)
            assert rc == 0, f"{which} returned {rc}"
            outs.append((dx, dw, db))
        torch.cuda.synchronize()
        (dx0, dw0, db0), (dx1, dw1, db1) = outs
        torch.testing.assert_close(dx0.float(), dx1.float(), rtol=2e-2, atol=2e-2)
        wtol = dict(rtol=1e-2, atol=5e-2) if fused else dict(rtol=1e-3, atol=1e-2)
        torch.testing.assert_close(dw0.float(), dw1.float(), **wtol)
        if kind == 1:
            torch.testing.assert_close(db0.float(), db1.float(), **wtol)


@pytest.mark.gpu
@pytest.mark.parametrize("kind", [0, 1])
@pytest.mark.parametrize("M", [1, 37, 300])
@pytest.mark.parametrize("D", [8, 4096, 8192])
def test_noalloc_norm_backward_matches_workspace_version(kind, M, D):
    """M < 64 uses M partial rows (the LayerNorm bias partials then start at scratch + M * D); M = 300
    strides rows over 64 partials; D = 8192 is the largest the scratch holds."""
    torch.manual_seed(0)
    _compare(kind, M, D)


@pytest.mark.gpu
@pytest.mark.parametrize("kind", [0, 1])
def test_noalloc_fused_residual_accumulate_bf16_matches_workspace_version(kind):
    torch.manual_seed(1)
    _compare(kind, 300, 4096, fused=True)


@pytest.mark.gpu
def test_noalloc_rejects_sizes_beyond_the_scratch():
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    f = _sym("brain_norm_bwd_noalloc")
    M = 4
    for D, want in ((8200, -1000), (0, 1), (-8, 1)):  # 1 = cudaErrorInvalidValue
        Dp = max(D, 8)
        t = torch.zeros(M, Dp, device="cuda", dtype=torch.bfloat16)
        v = torch.zeros(Dp, device="cuda", dtype=torch.float32)
        r = torch.ones(M, device="cuda", dtype=torch.float32)
        rc = f(*_args(0, t, t, t[0], None, r, t, v, None, M, D), ctypes.c_int(M), ctypes.c_int(D), st)
        assert rc == want, (D, rc)
    rc = f(*_args(0, t, t, t[0], None, r, t, v, None, M, 8), ctypes.c_int(-1), ctypes.c_int(8), st)
    assert rc == 1
    es = _native.fn("brain_error_string")(-1000).decode()
    assert "8192" in es
