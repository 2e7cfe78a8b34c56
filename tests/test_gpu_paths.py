"""GPU parity of the batched Sinkhorn, the MHCRewire kernels (pre-scale, mix,
fused post-combine), residual_add_agg, edge cases, and size-independent
properties at the benchmark size (T = 65536, n = 4, C = 4096)."""

from __future__ import annotations

import pytest
import torch
from torch import nn

import mhc_b200
from conftest import golden, max_abs, rel_err
from mhc_b200 import metal
from oracle import mhc_oracle as O

pytestmark = pytest.mark.gpu
G = golden()
DEV = "cuda"
F64 = torch.float64


def cu(a, dtype=torch.float32):
    return torch.as_tensor(a).to(DEV, dtype)


# ------------------------------------------------------- batched Sinkhorn --
@pytest.mark.parametrize("n", [1, 2, 4, 8, 16, 32, 3, 5, 64])
def test_batched_sinkhorn_matches_oracle(n):
    g = torch.Generator().manual_seed(n)
    B = 257 if n <= 32 else 9
    H = torch.randn(B, n, n, generator=g)
    dM = torch.randn(B, n, n, generator=g)
    M_ref, dH_ref = O.sinkhorn_grads(H, dM, 20, 1e-5, dtype=F64)
    Hc = cu(H).requires_grad_(True)
    M = metal.sinkhorn_knopp_batched(Hc, 20, 1e-5)
    (dH,) = torch.autograd.grad(M, [Hc], cu(dM))
    assert max_abs(M, M_ref) < 2e-6
    assert rel_err(dH, dH_ref) < 1e-5
    # single-matrix kernel on the same logits gives the same M to rounding
    M1 = metal.sinkhorn_knopp_metal(cu(H[0]), 20, 1e-5)
    assert max_abs(M1, M[0]) < 1e-6


@pytest.mark.parametrize("n", [1, 2, 4])
@pytest.mark.parametrize("iters", [0, 1, 7, 20, 37, 64])
def test_batched_sinkhorn_iteration_counts(n, iters):
    """n <= 4 runs one thread per matrix with checkpointed replay: iteration
    counts that are not a multiple of the checkpoint spacing, counts whose
    checkpoints need more than the default 48 KB of shared memory, and a
    count beyond the checkpoint path's limit (64: lane kernels' full tape)."""
    g = torch.Generator().manual_seed(100 * n + iters)
    B = 300
    H = torch.randn(B, n, n, generator=g)
    dM = torch.randn(B, n, n, generator=g)
    M_ref, dH_ref = O.sinkhorn_grads(H, dM, iters, 1e-5, dtype=F64)
    Hc = cu(H).requires_grad_(True)
    M = metal.sinkhorn_knopp_batched(Hc, iters, 1e-5)
    (dH,) = torch.autograd.grad(M, [Hc], cu(dM))
    assert max_abs(M, M_ref) < 2e-6
    assert rel_err(dH, dH_ref) < 1e-5


@pytest.mark.parametrize("n", [2, 4])
def test_batched_sinkhorn_unaligned_pointers(n):
    """Inputs that start 4 bytes past a 16-byte boundary take the scalar-load
    variant and give the same bits as aligned inputs."""
    g = torch.Generator().manual_seed(7 + n)
    B = 129
    H = torch.randn(B, n, n, generator=g)
    dM = torch.randn(B, n, n, generator=g)
    bh = torch.empty(B * n * n + 1, device=DEV)
    bd = torch.empty(B * n * n + 1, device=DEV)
    Hu = bh[1:].view(B, n, n)
    dMu = bd[1:].view(B, n, n)
    Hu.copy_(cu(H))
    dMu.copy_(cu(dM))
    assert Hu.data_ptr() % 16 != 0 and dMu.data_ptr() % 16 != 0
    from mhc_b200 import _kernels as K
    M_a, M_u = K.sinkhorn_batched_fwd(cu(H), 20, 1e-5), K.sinkhorn_batched_fwd(Hu, 20, 1e-5)
    dH_a = K.sinkhorn_batched_bwd(cu(H), cu(dM), 20, 1e-5)
    dH_u = K.sinkhorn_batched_bwd(Hu, dMu, 20, 1e-5)
    assert torch.equal(M_a, M_u) and torch.equal(dH_a, dH_u)


def test_batched_sinkhorn_config3_sums_and_stability():
    """65,536 4x4 logits ~ N(0,1), 20 iterations.
    Column sums are 1; row/col sums equal the oracle's to 1e-6; the result
    is bit-stable across runs."""
    g = torch.Generator().manual_seed(3)
    H = torch.randn(65536, 4, 4, generator=g)
    M = metal.sinkhorn_knopp_batched(cu(H), 20, 1e-5)
    M2 = metal.sinkhorn_knopp_batched(cu(H), 20, 1e-5)
    assert torch.equal(M, M2)
    M_ref = O.mixing_matrix_from_logits(H.double(), 20, 1e-5, dtype=F64)
    assert (M.sum(-2) - 1).abs().max() < 1e-6
    assert max_abs(M.sum(-1), M_ref.sum(-1)) < 1e-6
    assert max_abs(M.sum(-2), M_ref.sum(-2)) < 1e-6
    dM = torch.randn(65536, 4, 4, generator=g)
    Hc = cu(H).requires_grad_(True)
    (dH,) = torch.autograd.grad(metal.sinkhorn_knopp_batched(Hc, 20, 1e-5), [Hc], cu(dM))
    idx = torch.randint(0, 65536, (256,), generator=g)
    _, dH_ref = O.sinkhorn_grads(H[idx], dM[idx], 20, 1e-5, dtype=F64)
    assert rel_err(dH[idx.to(DEV)], dH_ref) < 1e-5


# ----------------------------------------------------------- stream mix --
@pytest.mark.parametrize("B,n,C", [(2, 4, 64), (3, 32, 64), (2, 8, 129), (1, 16, 256), (2, 3, 40)])
def test_stream_mix_add_matches_oracle(B, n, C):
    g = torch.Generator().manual_seed(B + n + C)
    x, y, d = (torch.randn(B, n, C, generator=g) for _ in range(3))
    M = torch.rand(n, n, generator=g)
    leaves = [t.double().requires_grad_(True) for t in (x, M, y)]
    out_ref = O.stream_mix_add_reference(*leaves, dtype=F64)
    g_ref = torch.autograd.grad(out_ref, leaves, d.double())
    xs = [cu(t).requires_grad_(True) for t in (x, M, y)]
    out = metal.stream_mix_add_metal_autograd(*xs)
    grads = torch.autograd.grad(out, xs, cu(d))
    assert rel_err(out, out_ref) < 1e-5
    for a, b in zip(grads, g_ref):
        assert rel_err(a, b) < 1e-5
    assert rel_err(metal.stream_mix_backward_dx_metal(cu(M), cu(d)), g_ref[0]) < 1e-5
    assert rel_err(metal.mhc_backward_dM_metal(cu(x), cu(d)), g_ref[1]) < 1e-5


@pytest.mark.parametrize("case", G.names("rewire"))
def test_rewire_module_matches_reference(case):
    d = G.get(case)
    dims, n = d["dims"], d["n"]
    lin = nn.Linear(dims, dims).to(DEV)
    with torch.no_grad():
        lin.weight.copy_(cu(d["W"]))
        lin.bias.copy_(cu(d["b"]))
    model = mhc_b200.MHCRewire(lin, dims=dims, n=n).to(DEV)
    with torch.no_grad():
        for k in ("H_pre_raw", "H_post_raw", "H_res_raw"):
            getattr(model.mhc, k).copy_(cu(d[k]))
    out = model(cu(d["x"]))
    assert out.shape == tuple(d["x"].shape) and out.dtype == torch.float32
    assert rel_err(out, d["out"]) < 1e-5


def _rewire_grads(dims, n, rows, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(dims, dims, generator=g) / dims ** 0.5
    b = 0.1 * torch.randn(dims, generator=g)
    x = torch.randn(rows, dims, generator=g).to(dtype)
    pre, post = 0.5 * torch.randn(n, generator=g), 0.5 * torch.randn(n, generator=g)
    res = torch.randn(n, n, generator=g)
    d = torch.randn(rows, dims, generator=g)
    leaves = [t.double().requires_grad_(True) for t in (x, pre, post, res, W)]
    out_ref = O.rewire_reference(lambda v: v @ leaves[4].T + b.double(), leaves[0], n, *leaves[1:4],
                                 20, 1e-5, dtype=F64)
    g_ref = torch.autograd.grad(out_ref, leaves, d.double())
    lin = nn.Linear(dims, dims).to(DEV, dtype)
    with torch.no_grad():
        lin.weight.copy_(W)
        lin.bias.copy_(b)
    model = mhc_b200.MHCRewire(lin, dims=dims, n=n).to(DEV)
    with torch.no_grad():
        model.mhc.H_pre_raw.copy_(pre)
        model.mhc.H_post_raw.copy_(post)
        model.mhc.H_res_raw.copy_(res)
    xg = cu(x, dtype).requires_grad_(True)
    out = model(xg)
    out.backward(cu(d))
    got = (out, xg.grad, model.mhc.H_pre_raw.grad, model.mhc.H_post_raw.grad,
           model.mhc.H_res_raw.grad, lin.weight.grad)
    return got, (out_ref, *g_ref)


@pytest.mark.parametrize("dims,n,rows", [(64, 4, 3), (256, 16, 2), (2048, 32, 1), (512, 8, 5)])
def test_rewire_gradients_match_oracle(dims, n, rows):
    """BASELINE config 1 (dims 2048, n 32, one row) and smaller: all grads."""
    got, ref = _rewire_grads(dims, n, rows, torch.float32, dims + n)
    for name, a, b in zip(("out", "dx", "dH_pre", "dH_post", "dH_res", "dW"), got, ref):
        # torch's fp32 GEMM (TF32 off by default) bounds dx/dW to ~1e-6
        assert rel_err(a, b) < 1e-5, (name, rel_err(a, b))


def test_rewire_quantized_inner_bf16():
    """BASELINE config 4 shape (reduced rows): MHCRewire n=4 around a 4-bit
    QuantizedLinear, bf16 activations; mHC grads only (inner frozen)."""
    g = torch.Generator().manual_seed(4)
    dims, n, rows = 4096, 4, 64
    ql = mhc_b200.QuantizedLinear.random(dims, dims, group_size=64, bits=4, dtype=torch.bfloat16,
                                         generator=g).to(DEV)
    model = mhc_b200.MHCRewire(ql, dims=dims, n=n).to(DEV)
    with torch.no_grad():
        model.mhc.H_pre_raw.copy_(0.5 * torch.randn(n, generator=g))
        model.mhc.H_res_raw.copy_(torch.randn(n, n, generator=g))
    x = torch.randn(rows, dims, generator=g).to(torch.bfloat16)
    d = torch.randn(rows, dims, generator=g)
    xg = cu(x, torch.bfloat16).requires_grad_(True)
    out = model(xg)
    out.backward(cu(d))
    Wd = ql.dequantize(torch.float64).cpu()
    leaves = [t.double().requires_grad_(True) for t in
              (x, model.mhc.H_pre_raw.detach().cpu(), model.mhc.H_post_raw.detach().cpu(),
               model.mhc.H_res_raw.detach().cpu())]
    out_ref = O.rewire_reference(lambda v: (v.to(torch.bfloat16).double() @ Wd.T), leaves[0], n,
                                 *leaves[1:], 20, 1e-5, dtype=F64)
    g_ref = torch.autograd.grad(out_ref, leaves[1:], d.double())
    # the inner GEMM runs in bf16 on the GPU: compare loosely
    assert rel_err(out, out_ref) < 2e-2
    for a, b in zip((model.mhc.H_pre_raw.grad, model.mhc.H_post_raw.grad,
                     model.mhc.H_res_raw.grad), g_ref):
        assert rel_err(a, b) < 5e-2
    assert len([p for p in model.parameters() if p.requires_grad]) == 4


# --------------------------------------------- quantized linear (in-kernel) --
def _random_qlinear(in_d, out_d, sdt, seed, bias=False):
    g = torch.Generator().manual_seed(seed)
    ql = mhc_b200.QuantizedLinear.random(in_d, out_d, group_size=64, bits=4, dtype=sdt,
                                         generator=g)
    ql = ql.to(DEV)
    if bias:  # random() makes no bias buffer: attach one on the device
        ql.bias = (0.1 * torch.randn(out_d, generator=g)).to(DEV, sdt)
    return ql


@pytest.mark.parametrize("M,N,Kd,xdt,sdt", [
    (8192, 4096, 4096, torch.bfloat16, torch.float16),   # BASELINE config 4, full rows
    (300, 4096, 4096, torch.bfloat16, torch.bfloat16),   # ragged rows, bf16 scales
    (1, 384, 1024, torch.float16, torch.float16),        # one row, 128-wide tiles
    (129, 1024, 2048, torch.bfloat16, torch.float16)])
def test_qlinear_kernels_match_dequantized_gemm(M, N, Kd, xdt, sdt):
    """mhc_qlinear_fwd / mhc_qlinear_bwd_dx (weight dequantised inside the
    tensor-core GEMM) against dequantize() + a float64 matmul; the outputs
    are rounded once to x's dtype (2e-2 is the bf16 tolerance of the other
    tests; the observed error is one rounding)."""
    from mhc_b200 import _kernels as K

    ql = _random_qlinear(Kd, N, sdt, M + N + Kd)
    g = torch.Generator().manual_seed(M)
    x = torch.randn(M, Kd, generator=g).to(xdt).to(DEV)
    dy = torch.randn(M, N, generator=g).to(xdt).to(DEV)
    W = ql.dequantize(xdt).double()
    y = K.qlinear_fwd(x, ql.weight, ql.scales, ql.biases, None, 64, 4)
    dx = K.qlinear_bwd_dx(dy, ql.weight, ql.scales, ql.biases, Kd, 64, 4)
    # the same gradient from the transposed layouts (weights in tensor memory)
    wt, _, _ = ql.transposed(xdt)
    assert torch.equal(wt, ql.pack(ql.codes().t().contiguous(), 4))  # device repack = torch
    dx_t = K.qlinear_bwd_dx_t(dy, *ql.transposed(xdt), Kd, 64, 4)
    assert y.dtype == xdt and dx.dtype == xdt and dx_t.dtype == xdt
    assert rel_err(dx_t, dy.double() @ W) < (1e-2 if xdt == torch.bfloat16 else 2e-3)
    y_ref = x.double() @ W.T
    dx_ref = dy.double() @ W
    tol = 1e-2 if xdt == torch.bfloat16 else 2e-3
    assert rel_err(y, y_ref) < tol, rel_err(y, y_ref)
    assert rel_err(dx, dx_ref) < tol, rel_err(dx, dx_ref)
    # and against torch's own GEMM on the materialised weight
    Wt = ql.dequantize(xdt)
    assert rel_err(y, (x @ Wt.T).double()) < tol
    assert rel_err(dx, (dy @ Wt).double()) < tol


def test_qlinear_module_allocates_no_weight_and_matches_torch_path():
    """QuantizedLinear.forward on CUDA bf16 runs the in-kernel dequantisation:
    no [out, in] weight is allocated (peak memory grows by far less than one
    bf16 copy of it), output and input gradient match the torch
    dequantise-and-matmul path, including a bias."""
    out_d, in_d, M = 4096, 4096, 64
    ql = _random_qlinear(in_d, out_d, torch.float16, 7, bias=True)
    x = torch.randn(M, in_d, device=DEV).to(torch.bfloat16).requires_grad_(True)
    assert ql._in_kernel(x)
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    # first step: builds the backward's transposed 4-bit layout once (in*out/2
    # bytes plus the transposed scales), no dequantised weight
    ql(x).backward(torch.ones(M, out_d, device=DEV, dtype=torch.bfloat16))
    torch.cuda.synchronize()
    first = torch.cuda.max_memory_allocated() - base
    assert first < out_d * in_d * 2 // 2, first  # a bf16 weight copy would be 32 MiB
    x.grad = None
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    y = ql(x)
    y.backward(torch.ones_like(y))
    torch.cuda.synchronize()
    grown = torch.cuda.max_memory_allocated() - base
    assert grown < out_d * in_d * 2 // 8, grown  # steady state: activations only
    W = ql.dequantize(torch.bfloat16)
    xr = x.detach().clone().requires_grad_(True)
    yr = xr @ W.T + ql.bias.to(torch.bfloat16)
    yr.backward(torch.ones_like(yr))
    assert rel_err(y, yr) < 1e-2
    assert rel_err(x.grad, xr.grad) < 1e-2


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_rewire_combine_kernel_matches_oracle(dt):
    g = torch.Generator().manual_seed(21)
    B, n, C = 5, 4, 1024
    x = torch.randn(B, n, C, generator=g).to(dt)
    y = torch.randn(B, n, C, generator=g).to(dt)
    M = O.mixing_matrix_from_logits(torch.randn(n, n, generator=g), 20, 1e-5)
    hpre, hpost = torch.rand(n, generator=g), 2 * torch.rand(n, generator=g)
    d = torch.randn(B, n, C, generator=g)

    def f(x_, y_, M_, a_, b_):
        return (y_ + torch.einsum("ij,bjc->bic", M_ * a_[None, :], x_)) * b_[None, :, None]

    leaves = [t.double().requires_grad_(True) for t in (x, y, M, hpre, hpost)]
    ref = f(*leaves)
    g_ref = torch.autograd.grad(ref, leaves, d.double())
    from mhc_b200.layer import _RewireCombineFn
    xs = [cu(x, dt).requires_grad_(True), cu(y, dt).requires_grad_(True)] + \
         [cu(t).requires_grad_(True) for t in (M, hpre, hpost)]
    out = _RewireCombineFn.apply(*xs)
    grads = torch.autograd.grad(out, xs, cu(d))
    assert rel_err(out, ref) < 1e-5
    tol_act = 1e-5 if dt == torch.float32 else 1e-2
    for k, (a, b) in enumerate(zip(grads, g_ref)):
        assert rel_err(a, b) < (tol_act if k < 2 else 1e-5), k


# ------------------------------------------- MHCRewire end-to-end backward --
def _fused_rewire_ref(x, y, M, hpre, hpost, d, p):
    """Gradients of <out, d> + <x * hpre, p> for the post-combine
    out = (y + (M * hpre) x) * hpost: the x-side gradients of MHCRewire when
    p is the inner module's input gradient (reference layer.py:469-492)."""
    leaves = [t.double().requires_grad_(True) for t in (x, M, hpre, hpost)]
    xd, Md, ad, bd = leaves
    out = (y.double() + torch.einsum("ij,bjc->bic", Md * ad[None, :], xd)) * bd[None, :, None]
    loss = (out * d.double()).sum()
    if p is not None:
        loss = loss + (xd * ad[None, :, None] * p.double()).sum()
    return torch.autograd.grad(loss, leaves), hpost.double()[None, :, None] * d.double()


@pytest.mark.parametrize("B,n,C,dt,with_p", [(5, 4, 1024, torch.float32, True),
                                             (5, 4, 1024, torch.bfloat16, True),
                                             (3, 4, 2048, torch.bfloat16, True),
                                             (3, 4, 1024, torch.bfloat16, False),
                                             (7, 2, 64, torch.float32, True),
                                             (4, 4, 129, torch.float32, True),
                                             (3, 3, 40, torch.bfloat16, True),
                                             (2, 16, 256, torch.float32, True),
                                             (2, 8, 64, torch.float32, False),
                                             (1, 32, 64, torch.float32, True)])
def test_rewire_split_backward_kernels_match_oracle(B, n, C, dt, with_p):
    """mhc_rewire_bwd_dy + mhc_rewire_bwd_dx through the C ABI: dy, dx (both
    branches, written once) and dM / dH_pre / dH_post from one reduction,
    against float64 autograd; d_xpre NULL counts as zero.  The shapes reach
    every x-side kernel: the bulk-copy ring (n <= 4, a few tokens fit in
    shared memory), the register kernel (n = 4, C = 2048: a 64 KB token
    leaves room for only three), and the generic tile kernel (other n, C)."""
    from mhc_b200 import _kernels as K

    g = torch.Generator().manual_seed(31 * n + C + B)
    x = torch.randn(B, n, C, generator=g).to(dt)
    y = torch.randn(B, n, C, generator=g).to(dt)
    M = O.mixing_matrix_from_logits(torch.randn(n, n, generator=g), 20, 1e-5)
    hpre, hpost = torch.rand(n, generator=g), 2 * torch.rand(n, generator=g)
    d = torch.randn(B, n, C, generator=g)
    pg = torch.randn(B, n, C, generator=g).to(dt) if with_p else None
    (gx, gM, gpre, gpost), dy_ref = _fused_rewire_ref(x, y, M, hpre, hpost, d, pg)
    dy, state = K.rewire_bwd_dy(cu(y, dt), cu(d), cu(hpost))
    dx, dM, dpre, dpost = K.rewire_bwd_dx(cu(x, dt), None if pg is None else cu(pg, dt), cu(M),
                                          cu(hpre), cu(hpost), state)
    tol_act = 1e-5 if dt == torch.float32 else 1e-2
    assert dy.dtype == dt and dx.dtype == dt
    assert rel_err(dy, dy_ref) < tol_act
    assert rel_err(dx, gx) < tol_act
    for name, a, b in (("dM", dM, gM), ("dH_pre", dpre, gpre), ("dH_post", dpost, gpost)):
        assert rel_err(a, b) < 1e-5, (name, rel_err(a, b))


@pytest.mark.parametrize("T,n,C,dt,iters", [(6, 4, 1024, torch.bfloat16, 20),
                                             (5, 4, 129, torch.float32, 20),
                                             (0, 4, 64, torch.float32, 20),
                                             (3, 1, 64, torch.float16, 20),
                                             (3, 2, 64, torch.float32, 7),
                                             (3, 8, 128, torch.bfloat16, 20),
                                             (2, 3, 40, torch.float32, 20),
                                             (2, 16, 64, torch.float32, 20),
                                             (2, 32, 64, torch.bfloat16, 20),
                                             (2, 4, 64, torch.float32, 0)])
def test_rewire_in_fwd_matches_parameter_and_prescale_kernels(T, n, C, dt, iters):
    """mhc_rewire_in_fwd (one launch for n <= 8: the parameter chain in one
    block beside the pre-scale) writes the same bits as mhc_params_fwd then
    mhc_prescale_fwd; for n <= 4 its Jacobian row u equals the parameter
    backward of the unit cotangent dM = e_u."""
    from mhc_b200 import _kernels as K

    g = torch.Generator().manual_seed(97 * n + T + iters)
    x = cu(torch.randn(T, n, C, generator=g).to(dt), dt)
    pre, post = cu(torch.randn(n, generator=g)), cu(torch.randn(n, generator=g))
    res = cu(3 * torch.randn(n, n, generator=g))
    xp, hpre, hpost, M, raw = K.rewire_in_fwd(x, pre, post, res, iters, 1e-5)
    hpre2, hpost2, M2, tape2 = K.params_fwd(pre, post, res, iters, 1e-5, want_tape=True)
    xp2 = K.prescale_fwd(x, hpre2)
    assert torch.equal(hpre, hpre2) and torch.equal(hpost, hpost2) and torch.equal(M, M2)
    assert torch.equal(xp, xp2) and xp.dtype == dt
    tape, jac = raw[3], raw[4]
    if iters:
        assert torch.equal(tape, tape2)
    if n not in (1, 2, 4):
        assert jac is None
        return
    assert jac is not None and jac.numel() == n ** 4
    eye = torch.eye(n * n, device=DEV)
    for u in range(n * n):
        _, _, gres = K.params_bwd(pre, post, res, tape2, iters, 1e-5, torch.zeros_like(hpre),
                                  torch.zeros_like(hpost), eye[u].view(n, n))
        assert torch.allclose(jac.view(n * n, n * n)[u], gres.flatten(), rtol=1e-6, atol=1e-7), u


@pytest.mark.parametrize("T,n,C,dt", [(5, 4, 1024, torch.bfloat16), (4, 4, 129, torch.float32),
                                      (3, 4, 2048, torch.bfloat16),
                                      (3, 1, 64, torch.float32), (3, 2, 64, torch.float32),
                                      (3, 8, 64, torch.float32), (2, 3, 40, torch.float32),
                                      (2, 16, 64, torch.float32), (2, 32, 64, torch.float32),
                                      (0, 4, 64, torch.float32)])
def test_rewire_bwd_dx_raw_gradients_match_parameter_kernel(T, n, C, dt):
    """mhc_rewire_bwd_dx with the raw parameters: the finalize carries the
    chain rule on to dH_pre_raw / dH_post_raw / dH_res_raw (the Jacobian's
    dot products for n <= 4, the reverse sweep in the finalize for n != 16,
    the parameter kernel after it for n = 16) and matches mhc_params_bwd on
    the activation gradients of the same call; dx is unchanged."""
    from mhc_b200 import _kernels as K

    g = torch.Generator().manual_seed(13 * n + C + T)
    x = cu(torch.randn(T, n, C, generator=g).to(dt), dt)
    y = cu(torch.randn(T, n, C, generator=g).to(dt), dt)
    d = cu(torch.randn(T, n, C, generator=g))
    p = cu(torch.randn(T, n, C, generator=g).to(dt), dt)
    pre, post = cu(torch.randn(n, generator=g)), cu(torch.randn(n, generator=g))
    res = cu(3 * torch.randn(n, n, generator=g))
    _, hpre, hpost, M, raw = K.rewire_in_fwd(x, pre, post, res, 20, 1e-5)
    _, state = K.rewire_bwd_dy(y, d, hpost)
    dx, dM, dpre, dpost = K.rewire_bwd_dx(x, p, M, hpre, hpost, state)
    _, state = K.rewire_bwd_dy(y, d, hpost)
    dx2, gpre, gpost, gres = K.rewire_bwd_dx(x, p, M, hpre, hpost, state, raw=raw)
    assert torch.equal(dx, dx2)
    rpre, rpost, rres = K.params_bwd(pre, post, res, raw[3], 20, 1e-5, dpre, dpost, dM)
    assert torch.equal(gpre, rpre) and torch.equal(gpost, rpost)
    assert gres.shape == (n, n)
    assert torch.allclose(gres, rres, rtol=1e-5, atol=1e-6 * float(rres.abs().max()) + 1e-30)
    if T == 0:
        assert torch.all(gres == 0) and torch.all(gpre == 0) and torch.all(gpost == 0)
    # run to run the same bits (fixed-order reductions whichever CTA finishes
    # last), also when one dy workspace is finalized twice
    again = K.rewire_bwd_dx(x, p, M, hpre, hpost, state, raw=raw)
    for a, b in zip((dx2, gpre, gpost, gres), again):
        assert torch.equal(a, b)


def test_rewire_backward_runs_no_torch_elementwise_kernel():
    """MHCRewire's backward around a frozen bias-free Linear (BASELINE config 4
    layout, bf16): the GPU kernels it launches are this library's and the
    inner GEMM only; dx is written once, so no torch add / copy kernel runs
    on [T, n, C]."""
    from torch.profiler import ProfilerActivity, profile

    T, dims, n = 512, 4096, 4
    lin = nn.Linear(dims, dims, bias=False).to(DEV, torch.bfloat16).requires_grad_(False)
    model = mhc_b200.MHCRewire(lin, dims=dims, n=n).to(DEV)
    x = torch.randn(T, dims, device=DEV).to(torch.bfloat16).requires_grad_(True)
    d = torch.randn(T, dims, device=DEV)
    for _ in range(2):
        model(x).backward(d)
    out = model(x)
    x.grad = None  # no gradient accumulation into an existing .grad in the profiled backward
    for p_ in model.parameters():
        p_.grad = None
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        out.backward(d)
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    kernels = [k for k in names if not k.startswith(("Memcpy", "Memset"))]
    ours = [k for k in kernels if "mhc::" in k]
    assert any("k_rewire_bwd_x" in k for k in ours), kernels
    assert not any("k_combine_bwd" in k for k in ours), ours  # the unsplit backward did not run
    stray = [k for k in kernels if "mhc::" not in k and "elementwise" in k.lower()]
    assert not stray, stray


def test_rewire_backward_without_a_path_to_the_prescale():
    """When the backward does not reach the pre-scale (an inner module that
    ignores its input, or gradients asked only for the inner weights), the
    post-combine's backward returns every gradient itself."""
    g = torch.Generator().manual_seed(5)
    dims, n, rows = 64, 4, 3
    x = torch.randn(rows, dims, generator=g)
    d = torch.randn(rows, dims, generator=g)

    class Const(nn.Module):
        def __init__(self):
            super().__init__()
            self.c = nn.Parameter(torch.randn(dims, generator=g))

        def forward(self, v):
            return self.c.expand_as(v)

    inner = Const().to(DEV)
    model = mhc_b200.MHCRewire(inner, dims=dims, n=n).to(DEV)
    with torch.no_grad():
        model.mhc.H_pre_raw.copy_(0.5 * torch.randn(n, generator=g))
        model.mhc.H_res_raw.copy_(torch.randn(n, n, generator=g))
    xg = cu(x).requires_grad_(True)
    model(xg).backward(cu(d))
    leaves = [t.double().requires_grad_(True) for t in
              (x, model.mhc.H_pre_raw.detach().cpu(), model.mhc.H_post_raw.detach().cpu(),
               model.mhc.H_res_raw.detach().cpu())]
    c = inner.c.detach().cpu().double()
    out_ref = O.rewire_reference(lambda v: c.expand_as(v), leaves[0], n, *leaves[1:], 20, 1e-5,
                                 dtype=F64)
    g_ref = torch.autograd.grad(out_ref, leaves, d.double())
    for a, b in zip((xg.grad, model.mhc.H_pre_raw.grad, model.mhc.H_post_raw.grad,
                     model.mhc.H_res_raw.grad), g_ref):
        assert rel_err(a, b) < 1e-5
    # gradients of the inner weights only: the pre-scale is not on the path
    lin = nn.Linear(dims, dims).to(DEV)
    model2 = mhc_b200.MHCRewire(lin, dims=dims, n=n).to(DEV)
    out = model2(cu(x).requires_grad_(True))
    (gw,) = torch.autograd.grad(out, [lin.weight], cu(d))
    pre = torch.sigmoid(model2.mhc.H_pre_raw.detach())
    post = 2 * torch.sigmoid(model2.mhc.H_post_raw.detach())
    dy = (cu(d).view(rows, n, -1) * post[None, :, None]).view(rows, dims)
    xp = (cu(x).view(rows, n, -1) * pre[None, :, None]).view(rows, dims)
    assert rel_err(gw, dy.T @ xp) < 1e-5


# --------------------------------------------------------- residual agg --
@pytest.mark.parametrize("B,n,C,dt", [(2, 4, 128, torch.float32), (3, 4, 129, torch.float32),
                                      (2, 16, 64, torch.bfloat16), (2, 5, 32, torch.float16)])
def test_residual_add_agg_matches_oracle(B, n, C, dt):
    g = torch.Generator().manual_seed(C)
    x = torch.randn(B, n, C, generator=g).to(dt)
    r = torch.randn(B, n, C, generator=g).to(dt)
    h = torch.rand(n, generator=g)
    out_ref, y_ref = O.residual_add_agg_reference(x, r, h, dtype=F64)
    out, y = mhc_b200.residual_add_agg(cu(x, dt), cu(r, dt), cu(h))
    assert out.dtype == torch.float32 and y.shape == (B, C)
    assert rel_err(out, out_ref) < 1e-6 and rel_err(y, y_ref) < 1e-5
    out_h, _ = metal.residual_add_agg_metal(cu(x, dt), cu(r, dt), cu(h), output_dtype=torch.bfloat16)
    assert out_h.dtype == torch.bfloat16 and rel_err(out_h, out_ref) < 1e-2


# ----------------------------------------------------------------- edges --
def test_empty_batch():
    layer = mhc_b200.MHCLayer(n=4, C=64).to(DEV)
    x = torch.zeros(0, 4, 64, device=DEV, requires_grad=True)
    out = layer(x)
    assert out.shape == (0, 4, 64)
    out.sum().backward()
    assert layer.H_res_raw.grad is not None and torch.all(layer.H_res_raw.grad == 0)
    assert torch.all(layer.rms_weight.grad == 0)


def test_unaligned_and_noncontiguous_inputs():
    g = torch.Generator().manual_seed(1)
    B, n, C = 3, 4, 256
    base = torch.randn(B * n * C + 1, generator=g)
    x_un = cu(base)[1:].view(B, n, C)  # 4-byte offset: scalar-load path
    x_nc = cu(torch.randn(B, C, n, generator=g)).transpose(1, 2)  # non-contiguous
    M = metal.sinkhorn_knopp_metal(cu(torch.randn(n, n, generator=g)))
    hp, hq, w = cu(torch.rand(n, generator=g)), cu(torch.rand(n, generator=g)), cu(torch.ones(C))
    for x in (x_un, x_nc):
        out = metal.mhc_forward_fused_metal(x, M, hp, hq, w)
        ref = O.mhc_forward_fused_reference(x.cpu(), M.cpu(), hp.cpu(), hq.cpu(), w.cpu(),
                                            dtype=F64)
        assert rel_err(out, ref) < 1e-5


def test_validation_errors_match_reference():
    x = torch.randn(2, 4, 16, device=DEV)
    M = torch.eye(4, device=DEV)
    h = torch.ones(4, device=DEV)
    w = torch.ones(16, device=DEV)
    with pytest.raises(ValueError):
        metal.mhc_forward_fused_metal(x, torch.eye(3, device=DEV), h, h, w)
    with pytest.raises(ValueError):
        metal.mhc_forward_fused_metal(x, M, h, h, torch.ones(8, device=DEV))
    with pytest.raises(ValueError):
        metal.mhc_forward_fused_metal(x, M, h, h, w, threads_per_group=2048)
    with pytest.raises(ValueError):
        metal.mhc_forward_fused_metal(x, M, h, h, w, output_dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        metal.sinkhorn_knopp_metal(torch.randn(65, 65, device=DEV))
    with pytest.raises(ValueError):
        mhc_b200.MHCRewire(nn.Linear(512, 256), dims=512, n=32).to(DEV)(
            torch.randn(1, 512, device=DEV))


def test_determinism_bitwise():
    g = torch.Generator().manual_seed(2)
    B, n, C = 1000, 4, 1024
    x, d = cu(torch.randn(B, n, C, generator=g)), cu(torch.randn(B, n, C, generator=g))
    layer = mhc_b200.MHCLayer(n=n, C=C, identity_init=False).to(DEV)
    res = []
    for _ in range(2):
        layer.zero_grad()
        xg = x.clone().requires_grad_(True)
        out = layer(xg)
        out.backward(d)
        res.append([out, xg.grad] + [p.grad.clone() for p in layer.parameters()])
    for a, b in zip(*res):
        assert torch.equal(a, b)


# -------------------------------------------- benchmark-size properties --
def _oracle_in_chunks(x, d, params, out, dx, chunk=1024):
    """The float64 oracle over the whole batch, run on the GPU in token
    chunks.  out and dx are per token, so each chunk is compared with the
    matching rows of the kernel's out / dx (max |diff| and max |ref| are
    accumulated over chunks); the raw-parameter gradients are sums over
    tokens of a chain that is linear in the upstream gradient, so the
    chunks' gradients add up to the whole batch's."""
    p64 = [p.to(DEV, F64) for p in params]
    err = {"out": 0.0, "dx": 0.0}
    scale = {"out": 0.0, "dx": 0.0}
    sums = None
    for s in range(0, x.shape[0], chunk):
        r = O.layer_grads(x[s:s + chunk], *p64, d[s:s + chunk], 20, 1e-5, dtype=F64)
        for name, got, ref in (("out", out[s:s + chunk], r[0]), ("dx", dx[s:s + chunk], r[1])):
            err[name] = max(err[name], float((got.double() - ref).abs().max()))
            scale[name] = max(scale[name], float(ref.abs().max()))
        sums = list(r[2:]) if sums is None else [a + b for a, b in zip(sums, r[2:])]
        del r
    return {k: err[k] / scale[k] for k in err}, sums


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_full_size_properties(dt):
    """T = 65536, n = 4, C = 4096 (BASELINE target).  Every output, dx and the
    four parameter gradients are compared with the float64 oracle over the
    whole batch (run on the GPU in 1024-token chunks, the parameter gradients
    summed over chunks): rel 1e-5, dx of bf16 inputs 2e-2.  Parameter
    gradients are also additive over tokens: grads(all) equals
    grads(first half) + grads(second half)."""
    T, n, C = 65536, 4, 4096
    g = torch.Generator(device=DEV).manual_seed(17)
    x = torch.randn(T, n, C, device=DEV, generator=g).to(dt)
    d = torch.randn(T, n, C, device=DEV, generator=g)
    gc = torch.Generator().manual_seed(18)
    params = [0.5 * torch.randn(n, generator=gc), 0.5 * torch.randn(n, generator=gc),
              torch.randn(n, n, generator=gc), 1 + 0.1 * torch.randn(C, generator=gc)]
    layer = mhc_b200.MHCLayer(n=n, C=C).to(DEV)

    def run(xs, ds):
        layer.zero_grad()
        with torch.no_grad():
            for k, v in zip(("H_pre_raw", "H_post_raw", "H_res_raw", "rms_weight"), params):
                getattr(layer, k).copy_(v)
        xg = xs.detach().requires_grad_(True)
        out = layer(xg)
        out.backward(ds)
        return out.detach(), xg.grad, [p.grad.clone() for p in layer.parameters()]

    out, dx, pg = run(x, d)
    rel, ref_grads = _oracle_in_chunks(x, d, params, out, dx)
    assert rel["out"] < 1e-5, rel
    assert rel["dx"] < (1e-5 if dt == torch.float32 else 2e-2), rel
    for name, a, b in zip(("dH_pre", "dH_post", "dH_res", "d_w"), pg, ref_grads):
        assert rel_err(a, b) < 1e-5, (name, rel_err(a, b))
    del out, dx
    h = T // 2
    _, _, pa = run(x[:h], d[:h])
    _, _, pb = run(x[h:], d[h:])
    for full, a, b in zip(pg, pa, pb):
        assert rel_err(full, a + b) < 1e-5
        assert torch.isfinite(full).all()


@pytest.mark.parametrize("B,n,C,dt", [(3, 4, 256, torch.float32), (2, 4, 129, torch.float32),
                                      (4, 4, 1024, torch.bfloat16), (2, 32, 64, torch.float32),
                                      (2, 3, 40, torch.float32)])
def test_residual_add_agg_backward_matches_oracle(B, n, C, dt):
    """The VJP this build adds to residual_add_agg (the reference has none)."""
    g = torch.Generator().manual_seed(B * C + n)
    x = torch.randn(B, n, C, generator=g).to(dt)
    r = torch.randn(B, n, C, generator=g).to(dt)
    h = torch.rand(n, generator=g)
    d_out, d_y = torch.randn(B, n, C, generator=g), torch.randn(B, C, generator=g)
    leaves = [t.double().requires_grad_(True) for t in (x, r, h)]
    o_ref, y_ref = O.residual_add_agg_reference(*leaves, dtype=F64)
    g_ref = torch.autograd.grad((o_ref * d_out.double()).sum() + (y_ref * d_y.double()).sum(),
                                leaves)
    xs = [cu(x, dt).requires_grad_(True), cu(r, dt).requires_grad_(True), cu(h).requires_grad_(True)]
    o, y = mhc_b200.residual_add_agg(*xs)
    torch.autograd.backward([o, y], [cu(d_out), cu(d_y)])
    tol = 1e-5 if dt == torch.float32 else 1e-2
    assert rel_err(xs[0].grad, g_ref[0]) < tol and rel_err(xs[1].grad, g_ref[1]) < tol
    assert rel_err(xs[2].grad, g_ref[2]) < 1e-5
    # only one of the two outputs used
    xs2 = [cu(x, dt).requires_grad_(True), cu(r, dt), cu(h).requires_grad_(True)]
    _, y2 = mhc_b200.residual_add_agg(*xs2)
    (y2 * cu(d_y)).sum().backward()
    g2 = torch.autograd.grad((O.residual_add_agg_reference(*leaves, dtype=F64)[1]
                              * d_y.double()).sum(), [leaves[0], leaves[2]])
    assert rel_err(xs2[0].grad, g2[0]) < tol and rel_err(xs2[2].grad, g2[1]) < 1e-5
