"""Pin the CPU oracle (oracle/mhc_oracle.py) against the reference's own
outputs (golden vectors from tests/golden/make_golden.py) and its gradients
against finite differences.  CPU only."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden, max_abs, rel_err
from oracle import mhc_oracle as O

G = golden()
T = torch.as_tensor


def _x(d):
    x = T(d["x"])
    dt = d.get("dtype", "float32")
    return x.to(getattr(torch, dt)) if dt != "float32" else x


@pytest.mark.parametrize("case", G.names("sinkhorn"))
def test_oracle_sinkhorn_matches_reference(case):
    d = G.get(case)
    M = O.mixing_matrix_from_logits(T(d["H"]), iters=d["iters"], eps=d["eps"])
    assert torch.isfinite(M).all()
    assert max_abs(M, d["M"]) < 1e-6, case


@pytest.mark.parametrize("case", G.names("forward"))
def test_oracle_forward_matches_reference(case):
    d = G.get(case)
    out = O.mhc_forward_reference(_x(d), T(d["H_pre_raw"]), T(d["H_post_raw"]), T(d["H_res_raw"]),
                                  T(d["rms_weight"]), sinkhorn_iters=d["iters"], eps=d["eps"])
    assert rel_err(out, d["out"]) < 2e-6, case


@pytest.mark.parametrize("case", G.names("layer"))
def test_oracle_layer_matches_reference(case):
    d = G.get(case)
    out = O.mhc_forward_reference(_x(d), T(d["H_pre_raw"]), T(d["H_post_raw"]), T(d["H_res_raw"]),
                                  T(d["rms_weight"]), sinkhorn_iters=d["iters"], eps=d["eps"])
    assert rel_err(out, d["out"]) < 2e-6, case


@pytest.mark.parametrize("case", G.names("rewire"))
def test_oracle_rewire_matches_reference(case):
    d = G.get(case)
    W, b = T(d["W"]), T(d["b"])
    out = O.rewire_reference(lambda v: v @ W.T + b, T(d["x"]), d["n"], T(d["H_pre_raw"]),
                             T(d["H_post_raw"]), T(d["H_res_raw"]), d["iters"], d["eps"])
    assert rel_err(out, d["out"]) < 2e-6, case


def test_identity_mapping_property():
    """Identity init maps x to itself (reference test_correctness.py:182-220)."""
    d = G.get("identity_bf16")
    x = _x(d)
    out = O.mhc_forward_reference(x, T(d["H_pre_raw"]), T(d["H_post_raw"]), T(d["H_res_raw"]),
                                  T(d["rms_weight"]), 20, 1e-5)
    assert max_abs(out, x.float()) < 1e-4
    assert max_abs(d["out"], x.float()) < 1e-4


def test_stability_doubly_stochastic():
    """H_res = 100: finite, rows and columns sum to 1 within 1e-3
    (reference tests/test_stability.py)."""
    M = O.mixing_matrix_from_logits(torch.full((32, 32), 100.0), 20, 1e-5)
    assert torch.isfinite(M).all()
    assert (M.sum(1) - 1).abs().max() < 1e-3 and (M.sum(0) - 1).abs().max() < 1e-3


def test_batched_sinkhorn_equals_per_matrix():
    g = torch.Generator().manual_seed(0)
    H = torch.randn(17, 4, 4, generator=g)
    Mb = O.mixing_matrix_from_logits(H, 20, 1e-5)
    for k in range(17):
        assert torch.equal(Mb[k], O.mixing_matrix_from_logits(H[k], 20, 1e-5))


def _fd_check(f, inputs, idx, eps=1e-6, samples=6, seed=0):
    """Central differences in float64 on a few coordinates of inputs[idx]."""
    g = torch.Generator().manual_seed(seed)
    leaves = [t.detach().double().clone().requires_grad_(True) for t in inputs]
    y = f(*leaves)
    w = torch.randn(y.shape, generator=g, dtype=torch.float64)
    (grad,) = torch.autograd.grad((y * w).sum(), [leaves[idx]])
    flat = leaves[idx].detach().reshape(-1)
    picks = torch.randint(0, flat.numel(), (samples,), generator=g)
    for p in picks.tolist():
        vals = []
        for s in (+1, -1):
            pert = [t.detach().clone() for t in leaves]
            pert[idx].reshape(-1)[p] += s * eps
            vals.append(float((f(*pert) * w).sum()))
        fd = (vals[0] - vals[1]) / (2 * eps)
        an = float(grad.reshape(-1)[p])
        assert abs(fd - an) <= 1e-6 * max(1.0, abs(an)), (p, fd, an)


@pytest.mark.parametrize("idx", [0, 1, 2, 3, 4])
def test_oracle_layer_gradients_finite_difference(idx):
    g = torch.Generator().manual_seed(3)
    B, n, C = 2, 4, 16
    ins = [torch.randn(B, n, C, generator=g), torch.randn(n, generator=g),
           torch.randn(n, generator=g), torch.randn(n, n, generator=g),
           1 + 0.1 * torch.randn(C, generator=g)]
    f = lambda *a: O.mhc_forward_reference(*a, sinkhorn_iters=5, eps=1e-5, dtype=torch.float64)
    _fd_check(f, ins, idx)


def test_oracle_rewire_gradients_finite_difference():
    g = torch.Generator().manual_seed(4)
    n, dims = 4, 32
    W = torch.randn(dims, dims, generator=g, dtype=torch.float64) / dims ** 0.5
    ins = [torch.randn(3, dims, generator=g), torch.randn(n, generator=g),
           torch.randn(n, generator=g), torch.randn(n, n, generator=g)]
    f = lambda x, a, b, c: O.rewire_reference(lambda v: v @ W.T, x, n, a, b, c, 20, 1e-5,
                                              dtype=torch.float64)
    for idx in range(4):
        _fd_check(f, ins, idx)
