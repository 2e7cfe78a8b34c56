"""GPU parity of the fused layer path against the reference's golden vectors and
the CPU oracle.  All calls go through the C ABI (libmhc_b200.so) via the
reference-named Python entry points.

Tolerances (max |diff| / max |ref| unless noted):
  fp32 outputs and gradients: 1e-5 (the reference north star's fp32 bar)
  half outputs: 5e-3 (fp16) / 2e-2 (bf16) absolute, the reference's test
  tolerances (tests/test_correctness.py:178-186)
"""

from __future__ import annotations

import os

import pytest
import torch

import mhc_b200
from conftest import assert_close_to_reference, golden, max_abs, rel_err
from mhc_b200 import metal
from oracle import mhc_oracle as O

pytestmark = pytest.mark.gpu
G = golden()
DEV = "cuda"
F64 = torch.float64


def cu(a, dtype=torch.float32):
    return torch.as_tensor(a).to(DEV, dtype)


def x_of(d):
    return cu(d["x"], getattr(torch, d.get("dtype", "float32")))


# ------------------------------------------------------------- Sinkhorn --
@pytest.mark.parametrize("case", G.names("sinkhorn"))
def test_sinkhorn_matches_reference(case):
    d = G.get(case)
    M = metal.sinkhorn_knopp_metal(cu(d["H"]), iters=d["iters"], eps=d["eps"])
    assert torch.isfinite(M).all()
    assert max_abs(M, d["M"]) < 2e-6, case


def test_sinkhorn_stability_bomb():
    layer = mhc_b200.MHCLayer(n=32, C=64).to(DEV)
    with torch.no_grad():
        layer.H_res_raw.fill_(100.0)
    M = layer.mixing_matrix().detach()
    assert not torch.isnan(M).any()
    assert (M.sum(1) - 1).abs().max() < 1e-3 and (M.sum(0) - 1).abs().max() < 1e-3


def test_sinkhorn_reciprocal_within_one_ulp():
    """The row / column scales use a branch-free reciprocal (hardware
    approximation plus one Newton-Raphson step) instead of an IEEE division;
    against CUDA's 1/x (torch on the GPU) it is within 1 ulp over positive
    normal floats with normal reciprocals, and exact at 0 / inf results."""
    from mhc_b200 import _capi as C

    g = torch.Generator().manual_seed(0)
    wide = torch.pow(10.0, torch.rand(1 << 20, generator=g, dtype=F64) * 74 - 37)
    sums = torch.rand(1 << 20, generator=g, dtype=F64) * 8 + 1e-5  # the range Sinkhorn sees
    special = torch.tensor([1.0, 2.0, 0.5, 3.0, 4.0, 1e-5, float("inf")], dtype=F64)
    x = torch.cat([wide, sums, special]).float().to(DEV)
    y = torch.empty_like(x)
    C.call("mhc_selftest_reciprocal", C.ptr(x), C.ptr(y), x.numel(), C.stream_of(x))
    ref = 1.0 / x
    ulps = (y.view(torch.int32).long() - ref.view(torch.int32).long()).abs()
    assert int(ulps.max()) <= 1, int(ulps.max())
    assert float(y[-1]) == 0.0


@pytest.mark.parametrize("n,iters", [(4, 20), (2, 20), (8, 20), (16, 10), (32, 20), (64, 20),
                                     (3, 7), (4, 0), (1, 5)])
def test_sinkhorn_backward_matches_oracle(n, iters):
    g = torch.Generator().manual_seed(n * 100 + iters)
    H = torch.randn(n, n, generator=g)
    dM = torch.randn(n, n, generator=g)
    _, dH_ref = O.sinkhorn_grads(H, dM, iters, 1e-5, dtype=F64)
    dH = metal.sinkhorn_knopp_backward_metal(cu(H), cu(dM), iters=iters, eps=1e-5)
    assert rel_err(dH, dH_ref) < 1e-5
    H_ = cu(H).requires_grad_(True)
    M = metal.sinkhorn_knopp_metal_autograd(H_, iters=iters, eps=1e-5)
    (dH2,) = torch.autograd.grad(M, [H_], cu(dM))
    assert torch.equal(dH2, dH)


# ------------------------------------------------------------ fused fwd --
@pytest.mark.parametrize("case", G.names("forward"))
def test_fused_forward_matches_reference(case):
    """mhc_forward_fused_metal with the reference's activations."""
    d = G.get(case)
    x = x_of(d)
    pre, post, M = cu(d["H_pre_raw"]), cu(d["H_post_raw"]), cu(d["H_res_raw"])
    hpre, hpost = torch.sigmoid(pre), 2 * torch.sigmoid(post)
    M = metal.sinkhorn_knopp_metal(M, iters=d["iters"], eps=d["eps"])
    out = metal.mhc_forward_fused_metal(x, M, hpre, hpost, cu(d["rms_weight"]), eps=d["eps"])
    assert out.dtype == torch.float32 and out.shape == x.shape
    assert rel_err(out, d["out"]) < 1e-5, case


@pytest.mark.parametrize("case", [c for c in G.names("forward")
                                  if G.cases[c]["dtype"] in ("float16", "bfloat16")])
def test_fused_forward_half_output(case):
    d = G.get(case)
    x = x_of(d)
    hpre, hpost = torch.sigmoid(cu(d["H_pre_raw"])), 2 * torch.sigmoid(cu(d["H_post_raw"]))
    M = metal.sinkhorn_knopp_metal(cu(d["H_res_raw"]), iters=d["iters"], eps=d["eps"])
    out = metal.mhc_forward_fused_metal(x, M, hpre, hpost, cu(d["rms_weight"]), eps=d["eps"],
                                        output_dtype=x.dtype)
    assert out.dtype == x.dtype
    tol = 5e-3 if x.dtype == torch.float16 else 2e-2
    # the output rounding is relative; the reference tolerance is absolute on O(1) data
    assert max_abs(out, d["out"]) < tol * max(1.0, float(abs(d["out"]).max())), case


def test_identity_mapping_n4():
    d = G.get("identity_bf16")
    x = x_of(d)
    layer = mhc_b200.MHCLayer(n=4, C=64).to(DEV)
    out = layer(x)
    assert max_abs(out, x.float()) < 1e-4


# ---------------------------------------------------------------- layer --
@pytest.mark.parametrize("case", G.names("layer"))
def test_layer_forward_matches_reference(case):
    d = G.get(case)
    layer = mhc_b200.MHCLayer(n=d["n"], C=d["C"]).to(DEV)
    with torch.no_grad():
        for k in ("H_pre_raw", "H_post_raw", "H_res_raw", "rms_weight"):
            getattr(layer, k).copy_(cu(d[k]))
    out = layer(x_of(d))
    assert rel_err(out, d["out"]) < 1e-5, case


def test_layer_init_matches_reference():
    d = G.get("layer_init_identity")
    layer = mhc_b200.MHCLayer(n=4, C=8)
    for k in ("H_pre_raw", "H_post_raw", "H_res_raw", "rms_weight"):
        assert torch.equal(getattr(layer, k).detach(), torch.as_tensor(d[k]))


def _layer_grads(x, params, d_out, iters, eps, return_dtype=None):
    n, C = x.shape[1], x.shape[2]
    layer = mhc_b200.MHCLayer(n=n, C=C, sinkhorn_iters=iters, eps=eps).to(DEV)
    with torch.no_grad():
        for k, v in zip(("H_pre_raw", "H_post_raw", "H_res_raw", "rms_weight"), params):
            getattr(layer, k).copy_(v)
    xg = x.detach().clone().requires_grad_(True)
    out = layer(xg, return_dtype=return_dtype)
    out.backward(d_out.to(out.dtype))
    return (out.detach(), xg.grad, layer.H_pre_raw.grad, layer.H_post_raw.grad,
            layer.H_res_raw.grad, layer.rms_weight.grad)


GRAD_SHAPES = [(1, 4, 16, 5), (2, 4, 128, 20), (3, 4, 129, 20), (2, 1, 64, 3), (2, 2, 100, 20),
               (2, 8, 128, 20), (2, 3, 40, 20), (2, 16, 256, 20), (1, 32, 256, 20),
               (1, 64, 96, 20), (5, 4, 4096, 20), (4, 4, 2048, 20), (3, 4, 1024, 20),
               (300, 4, 4096, 20), (2, 8, 4096, 10),
               # cluster-split generic backward: column slices of a token over 2-8 CTAs
               (2, 32, 4096, 20), (3, 16, 2048, 20), (2, 32, 1000, 20), (1, 64, 1024, 10)]


@pytest.mark.parametrize("B,n,C,dt", [(1, 32, 4096, torch.float32), (3, 16, 4096, torch.float32),
                                      (2, 64, 2048, torch.float32), (5, 32, 1000, torch.float32),
                                      (2, 32, 4096, torch.bfloat16)])
def test_cluster_split_forward_matches_oracle(B, n, C, dt):
    """n >= 16 with a row too wide for the register-resident kernel and few
    tokens: the forward splits each token's columns over a thread-block
    cluster (sum of squares reduced through distributed shared memory),
    including a ragged split (C = 1000).  Outputs match the fp64 oracle."""
    g = torch.Generator().manual_seed(n * 7 + C + B)
    x = torch.randn(B, n, C, generator=g).to(dt)
    params = [0.5 * torch.randn(n, generator=g), 0.5 * torch.randn(n, generator=g),
              torch.randn(n, n, generator=g), 1 + 0.1 * torch.randn(C, generator=g)]
    ref = O.mhc_forward_reference(x.to(F64), *[p.to(F64) for p in params], sinkhorn_iters=20,
                                  eps=1e-5, dtype=F64)
    layer = mhc_b200.MHCLayer(n=n, C=C).to(DEV)
    with torch.no_grad():
        for k, v in zip(("H_pre_raw", "H_post_raw", "H_res_raw", "rms_weight"), params):
            getattr(layer, k).copy_(v)
        out = layer(cu(x, dt))
    assert rel_err(out, ref) < 1e-5


@pytest.mark.parametrize("B,n,C,iters", GRAD_SHAPES)
def test_layer_gradients_match_oracle_fp32(B, n, C, iters):
    g = torch.Generator().manual_seed(B * 1000 + n * 10 + C)
    x = torch.randn(B, n, C, generator=g)
    params = [0.5 * torch.randn(n, generator=g), 0.5 * torch.randn(n, generator=g),
              torch.randn(n, n, generator=g), 1 + 0.1 * torch.randn(C, generator=g)]
    d_out = torch.randn(B, n, C, generator=g)
    ref = O.layer_grads(x, *params, d_out, iters, 1e-5, dtype=F64)
    ref32 = O.layer_grads(x, *params, d_out, iters, 1e-5, dtype=torch.float32)
    got = _layer_grads(cu(x), [cu(p) for p in params], cu(d_out), iters, 1e-5)
    names = ("out", "dx", "dH_pre", "dH_post", "dH_res", "d_w")
    for name, a, b, b32 in zip(names, got, ref, ref32):
        assert_close_to_reference(name, a, b, b32)


# the isolated op sweep's exact cells.  x ~ N(0, 1),
# H_res / H_pre / H_post logits ~ N(0, 0.1), rms_weight = 1, d_out ~ N(0, 1);
# bf16 runs bf16 in -> bf16 out (return_dtype), fp32 runs fp32 end to end.
@pytest.mark.parametrize("io", ["f32", "bf16"])
@pytest.mark.parametrize("C", [512, 2048, 4096])
@pytest.mark.parametrize("B", [1, 32])
def test_config2_sweep_cells_match_oracle(io, C, B):
    n = 4
    g = torch.Generator().manual_seed(20_000 + 7 * C + B + (1 if io == "bf16" else 0))
    dt = torch.float32 if io == "f32" else torch.bfloat16
    x = torch.randn(B, n, C, generator=g).to(dt)
    params = [0.1 * torch.randn(n, generator=g), 0.1 * torch.randn(n, generator=g),
              0.1 * torch.randn(n, n, generator=g), torch.ones(C)]
    d_out = torch.randn(B, n, C, generator=g).to(dt)
    ref = O.layer_grads(x, *params, d_out, 20, 1e-5, dtype=F64)
    got = _layer_grads(cu(x, dt), [cu(p) for p in params], cu(d_out, dt), 20, 1e-5,
                       return_dtype=None if io == "f32" else dt)
    names = ("out", "dx", "dH_pre", "dH_post", "dH_res", "d_w")
    if io == "f32":
        ref32 = O.layer_grads(x, *params, d_out, 20, 1e-5, dtype=torch.float32)
        for name, a, b, b32 in zip(names, got, ref, ref32):
            assert_close_to_reference(name, a, b, b32)
    else:
        assert got[0].dtype == dt and got[1].dtype == dt
        for name, a, b in zip(names, got, ref):
            tol = 2e-2 if name in ("out", "dx") else 1e-5
            assert rel_err(a, b) < tol, (name, rel_err(a, b))


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,n,C", [(2, 4, 128), (3, 4, 4096), (2, 16, 64), (2, 4, 129)])
def test_layer_gradients_half_inputs(dt, B, n, C):
    """Half x, fp32 out: the math is fp32 on exactly-representable inputs, so
    out and the parameter grads hold the fp32 bar; dx is rounded to x's dtype."""
    g = torch.Generator().manual_seed(7 + C)
    x = torch.randn(B, n, C, generator=g).to(dt)
    params = [0.5 * torch.randn(n, generator=g), 0.5 * torch.randn(n, generator=g),
              torch.randn(n, n, generator=g), 1 + 0.1 * torch.randn(C, generator=g)]
    d_out = torch.randn(B, n, C, generator=g)
    ref = O.layer_grads(x, *params, d_out, 20, 1e-5, dtype=F64)
    got = _layer_grads(cu(x, dt), [cu(p) for p in params], cu(d_out), 20, 1e-5)
    assert got[1].dtype == dt
    half_tol = 2e-2 if dt == torch.bfloat16 else 5e-3
    for name, a, b in zip(("out", "dx", "dH_pre", "dH_post", "dH_res", "d_w"), got, ref):
        tol = half_tol if name == "dx" else 1e-5
        assert rel_err(a, b) < tol, (name, rel_err(a, b))


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_layer_half_output_gradients(dt):
    """return_dtype = x's half dtype: the kernel writes half out; d_out arrives in half."""
    g = torch.Generator().manual_seed(11)
    B, n, C = 4, 4, 512
    x = torch.randn(B, n, C, generator=g).to(dt)
    params = [0.5 * torch.randn(n, generator=g), 0.5 * torch.randn(n, generator=g),
              torch.randn(n, n, generator=g), 1 + 0.1 * torch.randn(C, generator=g)]
    d_out = torch.randn(B, n, C, generator=g).to(dt)
    ref = O.layer_grads(x, *params, d_out.float(), 20, 1e-5, dtype=F64)
    got = _layer_grads(cu(x, dt), [cu(p) for p in params], cu(d_out, dt), 20, 1e-5,
                       return_dtype=dt)
    assert got[0].dtype == dt
    tol = 2e-2 if dt == torch.bfloat16 else 5e-3
    for name, a, b in zip(("out", "dx"), got[:2], ref[:2]):
        assert rel_err(a, b) < tol, (name, rel_err(a, b))
    for name, a, b in zip(("dH_pre", "dH_post", "dH_res", "d_w"), got[2:], ref[2:]):
        assert rel_err(a, b) < 1e-5, (name, rel_err(a, b))


def test_fused_autograd_matches_oracle():
    """mhc_forward_fused_metal_autograd: grads w.r.t. (x, M, H_pre, H_post, w)."""
    g = torch.Generator().manual_seed(5)
    B, n, C = 3, 4, 256
    x = torch.randn(B, n, C, generator=g)
    M = O.mixing_matrix_from_logits(torch.randn(n, n, generator=g), 20, 1e-5)
    hpre, hpost = torch.rand(n, generator=g), 2 * torch.rand(n, generator=g)
    w = 1 + 0.1 * torch.randn(C, generator=g)
    d_out = torch.randn(B, n, C, generator=g)
    ref = O.fused_grads(x, M, hpre, hpost, w, d_out, 1e-5, dtype=F64)
    leaves = [cu(t).requires_grad_(True) for t in (x, M, hpre, hpost, w)]
    out = metal.mhc_forward_fused_metal_autograd(*leaves, eps=1e-5)
    grads = torch.autograd.grad(out, leaves, cu(d_out))
    assert rel_err(out, ref[0]) < 1e-5
    for k, (a, b) in enumerate(zip(grads, ref[1:])):
        assert rel_err(a, b) < 1e-5, (k, rel_err(a, b))
    dx, dM, dpre, dpost, dw = metal.mhc_backward_fused_metal(*[t.detach() for t in leaves],
                                                             cu(d_out))
    for a, b in zip((dx, dM, dpre, dpost, dw), grads):
        assert torch.equal(a, b)


def test_backward_loss_matches_reference():
    """reference tests/test_correctness.py:295-344: loss = sum(out)."""
    d = G.get("bwd_case_f32")
    x = x_of(d)
    layer = mhc_b200.MHCLayer(n=4, C=16, sinkhorn_iters=5).to(DEV)
    with torch.no_grad():
        for k in ("H_pre_raw", "H_post_raw", "H_res_raw", "rms_weight"):
            getattr(layer, k).copy_(cu(d[k]))
    loss = layer(x).sum()
    assert abs(float(loss) - float(d["out"].sum())) < 1e-4


def test_use_metal_false_raises():
    layer = mhc_b200.MHCLayer(n=4, C=16, use_metal=False).to(DEV)
    with pytest.raises(RuntimeError):
        layer(torch.randn(1, 4, 16, device=DEV))


def test_generic_path_matches_fast_path():
    """MHC_B200_GENERIC=1 forces the any-n kernels; results agree with the
    specialised ones to fp32 rounding."""
    g = torch.Generator().manual_seed(9)
    B, n, C = 6, 4, 1024
    x, d_out = cu(torch.randn(B, n, C, generator=g)), cu(torch.randn(B, n, C, generator=g))
    params = [cu(0.5 * torch.randn(n, generator=g)), cu(0.5 * torch.randn(n, generator=g)),
              cu(torch.randn(n, n, generator=g)), cu(1 + 0.1 * torch.randn(C, generator=g))]
    fast = _layer_grads(x, params, d_out, 20, 1e-5)
    os.environ["MHC_B200_GENERIC"] = "1"
    try:
        gen = _layer_grads(x, params, d_out, 20, 1e-5)
    finally:
        del os.environ["MHC_B200_GENERIC"]
    for a, b in zip(fast, gen):
        assert rel_err(a, b) < 1e-5


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n,C", [(4, 4096), (4, 2048), (4, 1024), (4, 1000), (2, 2048), (1, 512)])
def test_backward_16bit_dout(dt, n, C):
    """16-bit x and d_out (return_dtype = x's dtype) through the fused
    backward, including a C that leaves the last CTA columns partly empty.
    n = 4 with C = 1024 / 2048 / 4096 runs the full-row kernel with the
    tensor-core dM (block sizes 128 / 256 / 512)."""
    g = torch.Generator().manual_seed(n * 7 + C)
    T = 300
    x = torch.randn(T, n, C, generator=g).to(dt)
    params = [0.5 * torch.randn(n, generator=g), 0.5 * torch.randn(n, generator=g),
              torch.randn(n, n, generator=g), 1 + 0.1 * torch.randn(C, generator=g)]
    d_out = torch.randn(T, n, C, generator=g).to(dt)
    ref = O.layer_grads(x, *params, d_out.float(), 20, 1e-5, dtype=F64)
    ref32 = O.layer_grads(x, *params, d_out.float(), 20, 1e-5, dtype=torch.float32)
    got = _layer_grads(cu(x, dt), [cu(p) for p in params], cu(d_out, dt), 20, 1e-5,
                       return_dtype=dt)
    half_tol = 2e-2 if dt == torch.bfloat16 else 5e-3
    for k, name in enumerate(("out", "dx", "dH_pre", "dH_post", "dH_res", "d_w")):
        if name in ("out", "dx"):
            assert rel_err(got[k], ref[k]) < half_tol, (name, rel_err(got[k], ref[k]))
        else:
            assert_close_to_reference(name, got[k], ref[k], ref32[k])


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T,n,C", [(600, 32, 512), (257, 16, 129), (3, 32, 4), (64, 16, 4096),
                                   (40, 32, 1030), (0, 32, 256)])
def test_wide_backward_matches_oracle_and_generic(dt, T, n, C):
    """n = 16 / 32 run the register-tiled backward (8 x 8 dM blocks over
    column slices, 4 x 4(8) dx blocks): many tokens per CTA, ragged tiles and
    odd C (scalar dx stores), a row narrower than one tile, a cluster split
    with a C that is not a multiple of the slice, and T = 0.  x, d_out and dx
    share dtype dt.  Results match the float64 oracle and the any-n kernel."""
    g = torch.Generator().manual_seed(T * 31 + n + C)
    x = torch.randn(T, n, C, generator=g).to(dt)
    params = [0.5 * torch.randn(n, generator=g), 0.5 * torch.randn(n, generator=g),
              torch.randn(n, n, generator=g), 1 + 0.1 * torch.randn(C, generator=g)]
    d_out = torch.randn(T, n, C, generator=g).to(dt)
    rd = None if dt == torch.float32 else dt
    got = _layer_grads(cu(x, dt), [cu(p) for p in params], cu(d_out, dt), 20, 1e-5,
                       return_dtype=rd)
    os.environ["MHC_B200_GENERIC"] = "1"
    try:
        gen = _layer_grads(cu(x, dt), [cu(p) for p in params], cu(d_out, dt), 20, 1e-5,
                           return_dtype=rd)
    finally:
        del os.environ["MHC_B200_GENERIC"]
    names = ("out", "dx", "dH_pre", "dH_post", "dH_res", "d_w")
    if T == 0:
        for name, a in zip(names[2:], got[2:]):
            assert torch.count_nonzero(a) == 0, name
        return
    ref = O.layer_grads(x, *params, d_out.float(), 20, 1e-5, dtype=F64)
    ref32 = O.layer_grads(x, *params, d_out.float(), 20, 1e-5, dtype=torch.float32)
    half_tol = {torch.bfloat16: 2e-2, torch.float16: 5e-3}.get(dt)
    for k, name in enumerate(names):
        if half_tol is not None and name in ("out", "dx"):
            assert rel_err(got[k], ref[k]) < half_tol, (name, rel_err(got[k], ref[k]))
        else:
            assert_close_to_reference(name, got[k], ref[k], ref32[k])
        # the any-n kernel: same math, another summation order
        if half_tol is not None and name in ("out", "dx"):
            assert rel_err(got[k], gen[k]) < half_tol, (name, rel_err(got[k], gen[k]))
        else:
            assert_close_to_reference(name, got[k], gen[k].double(), ref32[k])
