"""mhc_bwd_noalloc: the layer backward for callers that cannot allocate.

Some callers of this library cannot hand it a workspace: a plugin boundary
that gives a kernel only its inputs and outputs (the shape of the
reference's own mx.fast.metal_kernel boundary), or a runtime that forbids
device allocation on this path.  mhc_bwd_noalloc serves them by keeping the
per-block partial sums in a fixed 16 MiB device array inside the library.

This test calls it through the C ABI twice in a row and checks each result
against the workspace-based entry points (mhc_bwd + mhc_bwd_finalize), within
the tolerance the other fp32 tests use (rel 1e-5; the two paths run the same
kernels, so they normally agree bit for bit).  The second call checks that
the array's leftover contents from the first call do not leak into the
result.  The file is named so that pytest collects it last.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import rel_err
from mhc_b200 import _capi as C

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(T, n, Cc, dt, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, n, Cc, generator=g).to(dt).to(DEV)
    d = torch.randn(T, n, Cc, generator=g).to(DEV)
    M = torch.rand(n, n, generator=g).to(DEV)
    hpre = torch.rand(n, generator=g).to(DEV)
    hpost = (2 * torch.rand(n, generator=g)).to(DEV)
    w = (1 + 0.1 * torch.randn(Cc, generator=g)).to(DEV)
    return x, d, M, hpre, hpost, w


def _with_workspace(x, d, M, hpre, hpost, w, eps):
    T, n, Cc = x.shape
    dx = torch.empty_like(x)
    outs = [torch.empty(n, n, device=DEV), torch.empty(n, device=DEV), torch.empty(n, device=DEV),
            torch.empty(Cc, device=DEV)]
    nb = int(C.query("mhc_bwd_workspace_bytes", T, n, Cc))
    ws = torch.empty(nb, dtype=torch.uint8, device=DEV)
    st = C.stream_of(x)
    C.call("mhc_bwd", C.ptr(x), C.dtype_code(x.dtype), C.ptr(d), C.dtype_code(d.dtype), C.ptr(M),
           C.ptr(hpre), C.ptr(hpost), C.ptr(w), C.ptr(dx), C.dtype_code(dx.dtype), T, n, Cc,
           eps, C.ptr(ws), nb, st)
    C.call("mhc_bwd_finalize", C.ptr(ws), n, Cc, *[C.ptr(o) for o in outs], None, None, None,
           None, 0, eps, None, None, None, st)
    return [dx] + outs


def _no_alloc(x, d, M, hpre, hpost, w, eps):
    T, n, Cc = x.shape
    dx = torch.empty_like(x)
    outs = [torch.empty(n, n, device=DEV), torch.empty(n, device=DEV), torch.empty(n, device=DEV),
            torch.empty(Cc, device=DEV)]
    C.call("mhc_bwd_noalloc", C.ptr(x), C.dtype_code(x.dtype), C.ptr(d), C.dtype_code(d.dtype),
           C.ptr(M), C.ptr(hpre), C.ptr(hpost), C.ptr(w), C.ptr(dx), C.dtype_code(dx.dtype),
           *[C.ptr(o) for o in outs], T, n, Cc, eps, C.stream_of(x))
    return [dx] + outs


@pytest.mark.parametrize("T,n,Cc,dt", [(4096, 4, 4096, torch.float32), (777, 4, 1024, torch.bfloat16),
                                       (64, 16, 256, torch.float32), (3, 3, 129, torch.float32)])
def test_no_alloc_matches_workspace_path_twice(T, n, Cc, dt):
    eps = 1e-5
    # two different problems back to back: the second call must not see the
    # first call's leftovers in the shared array
    for seed in (1, 2):
        args = _inputs(T, n, Cc, dt, seed)
        ref = _with_workspace(*args, eps)
        got = _no_alloc(*args, eps)
        torch.cuda.synchronize()
        for name, a, b in zip(("dx", "dM", "dH_pre", "dH_post", "d_w"), got, ref):
            tol = 1e-5 if (name != "dx" or dt == torch.float32) else 1e-2
            assert rel_err(a, b) < tol, (name, seed, rel_err(a, b))


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_no_alloc_matches_fp64_oracle(dt):
    """The no-allocation path against the float64 oracle of the fused layer's
    VJP directly (not only against the workspace path), twice in a row."""
    from oracle import mhc_oracle as O

    T, n, Cc, eps = 300, 4, 512, 1e-5
    for seed in (3, 4):
        x, d, M, hpre, hpost, w = _inputs(T, n, Cc, dt, seed)
        ref = O.fused_grads(x.cpu(), M.cpu(), hpre.cpu(), hpost.cpu(), w.cpu(), d.cpu(), eps,
                            dtype=torch.float64)
        got = _no_alloc(x, d, M, hpre, hpost, w, eps)
        torch.cuda.synchronize()
        for name, a, b in zip(("dx", "dM", "dH_pre", "dH_post", "d_w"), got, ref[1:]):
            tol = 1e-5 if (name != "dx" or dt == torch.float32) else 2e-2
            assert rel_err(a, b) < tol, (name, seed, rel_err(a, b))


def test_no_alloc_rejects_sizes_beyond_the_array():
    """T=4096, n=4, C=32768 needs more partial rows than the 16 MiB array
    holds.  The size check runs on the host before any pointer is used, so
    small placeholder buffers stand in for the tensors."""
    T, n, Cc = 4096, 4, 32768
    assert int(C.query("mhc_bwd_workspace_bytes", T, n, Cc)) > (16 << 20)
    buf = torch.zeros(16, device=DEV)
    outs = [torch.empty(n, n, device=DEV), torch.empty(n, device=DEV), torch.empty(n, device=DEV),
            torch.empty(16, device=DEV)]
    with pytest.raises(C.MHCError, match="scratch"):
        C.call("mhc_bwd_noalloc", C.ptr(buf), C.MHC_BF16, C.ptr(buf), C.MHC_F32, C.ptr(buf),
               C.ptr(buf), C.ptr(buf), C.ptr(buf), C.ptr(buf), C.MHC_BF16,
               *[C.ptr(o) for o in outs], T, n, Cc, 1e-5, C.stream_of(buf))
