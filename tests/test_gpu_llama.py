"""BASELINE config 5 end to end at a small size: the mHC-patched Llama mock's
loss and mHC gradients on the GPU match a float64 CPU copy in which every
MHCRewire runs the oracle restatement of the reference's MHCRewire."""

from __future__ import annotations

import copy
import sys
from pathlib import Path

import pytest
import torch
import torch.nn.functional as F

from conftest import rel_err
from mhc_b200 import MHCRewire
from mhc_b200.dist import mhc_parameters
from oracle import mhc_oracle as O

sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "mhc-mlx_b200" / "examples"))
import llama_mock  # noqa: E402

pytestmark = pytest.mark.gpu


def _oracle_copy(model):
    ref = copy.deepcopy(model).cpu().double()
    for m in ref.modules():
        if isinstance(m, MHCRewire):
            def fwd(x, m=m):
                return O.rewire_reference(m.inner, x, m.n, m.mhc.H_pre_raw, m.mhc.H_post_raw,
                                          m.mhc.H_res_raw, m.mhc.sinkhorn_iters, m.mhc.eps,
                                          dtype=torch.float64)
            m.forward = fwd
    return ref


def test_llama_mock_matches_oracle_rewire():
    model = llama_mock.build(layers=2, dims=128, num_heads=4, mlp_dims=344, vocab=97,
                             n_streams=4, dtype=torch.float32, device="cuda")
    ref = _oracle_copy(model)
    g = torch.Generator().manual_seed(3)
    tokens = torch.randint(0, 97, (2, 16), generator=g)
    targets = torch.randint(0, 97, (2, 16), generator=g)

    def loss_of(m, dev, dt):
        logits = m(tokens.to(dev))
        return F.cross_entropy(logits.to(dt).flatten(0, 1), targets.to(dev).flatten())

    loss = loss_of(model, "cuda", torch.float32)
    loss.backward()
    loss_ref = loss_of(ref, "cpu", torch.float64)
    loss_ref.backward()
    assert abs(float(loss) - float(loss_ref)) < 1e-5 * max(1.0, abs(float(loss_ref)))
    got = [p.grad for p in mhc_parameters(model) if p.grad is not None]
    want = [p.grad for p in mhc_parameters(ref) if p.grad is not None]
    assert len(got) == len(want) == 2 * 4 * 3
    for a, b in zip(got, want):
        assert rel_err(a, b) < 1e-4, rel_err(a, b)


def test_llama_mock_train_step_bf16():
    """The bf16 training step runs, returns a finite loss and updates the mHC
    parameters; MHCRewire keeps the activations in bf16."""
    model = llama_mock.build(layers=2, dims=256, num_heads=4, mlp_dims=688, vocab=512,
                             n_streams=4, dtype=torch.bfloat16, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(1)
    tokens = torch.randint(0, 512, (2, 64), device="cuda", generator=g)
    targets = torch.randint(0, 512, (2, 64), device="cuda", generator=g)
    before = [p.detach().clone() for p in mhc_parameters(model)]
    with torch.no_grad():
        h = model.layers[0].attention.wq(torch.randn(1, 4, 256, device="cuda",
                                                     dtype=torch.bfloat16))
    assert h.dtype == torch.bfloat16
    loss = llama_mock.train_step(model, tokens, targets, tokens.numel())
    assert torch.isfinite(loss)
    changed = [not torch.equal(a, p.detach()) for a, p in zip(before, mhc_parameters(model))]
    assert sum(changed) >= 2 * 4 * 3
