"""GPU ports of the reference's API-level tests (tests/test_rewire.py,
test_vision.py, test_quantized.py, test_folding.py, test_concurrency.py) plus
CUDA-graph capture and multi-stream use of the layer."""

from __future__ import annotations

import multiprocessing as mp
import sys
import threading
from pathlib import Path

import pytest
import torch
from torch import nn

import mhc_b200
from conftest import rel_err
from mhc_b200 import MHCLayer, MHCRewire, QuantizedLinear

pytestmark = pytest.mark.gpu
DEV = "cuda"
ROOT = Path(__file__).resolve().parent.parent


def test_rewire_linear_and_block_shapes():
    """reference tests/test_rewire.py:5-46"""
    model = MHCRewire(nn.Linear(512, 512), dims=512, n=16).to(DEV)
    y = model(torch.randn(2, 512, device=DEV))
    assert y.shape == (2, 512) and model.mhc.n == 16 and model.mhc.C == 32

    class Block(nn.Module):
        def __init__(self, d):
            super().__init__()
            self.ln = nn.RMSNorm(d)
            self.lin = nn.Linear(d, d)

        def forward(self, x):
            return self.lin(self.ln(x))

    model = MHCRewire(Block(1024), dims=1024, n=32).to(DEV)
    assert model(torch.randn(1, 16, 1024, device=DEV)).shape == (1, 16, 1024)


def test_vision_wrappers():
    """reference tests/test_vision.py: a channels-last Conv2d and a ViT block."""
    class ConvNHWC(nn.Module):  # MLX convolutions are channels-last
        def __init__(self, c):
            super().__init__()
            self.conv = nn.Conv2d(c, c, 3, padding=1)

        def forward(self, x):
            return self.conv(x.permute(0, 3, 1, 2)).permute(0, 2, 3, 1)

    inner = ConvNHWC(64).to(DEV)
    model = MHCRewire(inner, dims=64, n=16).to(DEV)
    x = torch.randn(2, 32, 32, 64, device=DEV)
    y = model(x)
    assert y.shape == (2, 32, 32, 64) and not torch.equal(y, inner(x))

    class ViT(nn.Module):
        def __init__(self, d):
            super().__init__()
            self.norm = nn.LayerNorm(d)
            self.linear = nn.Linear(d, d)

        def forward(self, x):
            return self.linear(self.norm(x))

    model = MHCRewire(ViT(256), dims=256, n=32).to(DEV)
    assert model(torch.randn(2, 196, 256, device=DEV)).shape == (2, 196, 256)


def test_quantized_linear_rewire():
    """reference tests/test_quantized.py: wrap a 4-bit QuantizedLinear (group
    64), freeze it, only the mHC parameters train and get gradients."""
    q = QuantizedLinear.from_linear(nn.Linear(512, 512), group_size=64, bits=4).to(DEV)
    model = MHCRewire(q, dims=512, n=16).to(DEV)
    model.inner.freeze()
    y = model(torch.randn(1, 512, device=DEV, dtype=torch.float16))
    assert y.shape == (1, 512)
    trainable = {n for n, p in model.named_parameters() if p.requires_grad}
    assert trainable and all(n.startswith("mhc.") for n in trainable)
    y.sum().backward()
    assert model.mhc.H_pre_raw.grad is not None and torch.isfinite(model.mhc.H_pre_raw.grad).all()


def test_folding_gradient_flow():
    """reference tests/test_folding.py:41-62: grads reach H_pre_raw and the inner weight."""
    torch.manual_seed(0)
    model = MHCRewire(nn.Linear(64, 64), dims=64, n=4).to(DEV)
    model(torch.randn(1, 64, device=DEV)).sum().backward()
    assert float(model.mhc.H_pre_raw.grad.abs().sum()) > 0
    assert float(model.inner.weight.grad.abs().sum()) > 0


def test_cuda_graph_capture_matches_eager():
    """The layer step (4 kernels) is capture-safe: replaying a captured
    fwd+bwd gives the eager results bit for bit."""
    torch.manual_seed(3)
    layer = MHCLayer(4, 1024, identity_init=False).to(DEV)
    with torch.no_grad():
        for p in (layer.H_pre_raw, layer.H_post_raw, layer.H_res_raw):
            p.normal_(0, 0.5)
    x = torch.randn(64, 4, 1024, device=DEV, requires_grad=True)
    d = torch.randn(64, 4, 1024, device=DEV)

    def step():
        x.grad = None
        for p in layer.parameters():
            p.grad = None
        out = layer(x)
        out.backward(d)
        return out

    eager = step().detach().clone()
    eager_grads = [x.grad.clone()] + [p.grad.clone() for p in layer.parameters()]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            step()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = step()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    for a, b in zip([x.grad] + [p.grad for p in layer.parameters()], eager_grads):
        assert torch.equal(a, b)


def test_concurrent_streams_and_threads():
    """Several host threads, each on its own stream and layer, give the same
    results as a serial run (the library keeps no shared mutable state
    besides a thread-local error string)."""
    torch.manual_seed(1)
    layers = [MHCLayer(4, 512, identity_init=False).to(DEV) for _ in range(4)]
    xs = [torch.randn(32, 4, 512, device=DEV) for _ in range(4)]
    serial = [l(x).detach() for l, x in zip(layers, xs)]
    results = [None] * 4

    def work(k):
        st = torch.cuda.Stream()
        with torch.cuda.stream(st):
            for _ in range(20):
                out = layers[k](xs[k])
            st.synchronize()
            results[k] = out.detach()

    threads = [threading.Thread(target=work, args=(k,)) for k in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    for a, b in zip(results, serial):
        assert torch.equal(a, b)


def _proc(k, q):
    try:
        sys.path.insert(0, str(ROOT / "mhc-mlx_b200"))
        import torch as T

        from mhc_b200 import MHCLayer as L

        layer = L(n=32, C=512).cuda()
        for _ in range(50):
            x = T.randn(2, 32, 512, device="cuda")
            layer(x).sum().backward()
        T.cuda.synchronize()
        q.put((k, "ok"))
    except Exception as e:  # report to the parent
        q.put((k, repr(e)))


def test_multiprocess_stress():
    """reference tests/test_concurrency.py: 4 processes x 50 fwd+bwd iterations."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_proc, args=(k, q)) for k in range(4)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in ps]
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(r[1] == "ok" for r in res), res


def test_workspace_too_small_is_reported():
    from mhc_b200 import _capi as C

    x = torch.randn(8, 4, 64, device=DEV)
    h = torch.ones(4, device=DEV)
    ws = torch.empty(16, dtype=torch.uint8, device=DEV)
    with pytest.raises(C.MHCError, match="workspace"):
        C.call("mhc_bwd", C.ptr(x), 0, C.ptr(x), 0, C.ptr(torch.eye(4, device=DEV)), C.ptr(h),
               C.ptr(h), C.ptr(torch.ones(64, device=DEV)), C.ptr(torch.empty_like(x)), 0, 8, 4,
               64, 1e-5, C.ptr(ws), 16, C.stream_of(x))


def test_grad_bucket_backward_writes_into_the_bucket():
    """With a GradBucket bound, the layer backward's finalize writes the four
    parameter gradients into the bucket's views (they become .grad, same
    values as an unbound layer's), a second backward without zeroing
    accumulates, and allreduce() on one process leaves them unchanged."""
    from mhc_b200.dist import GradBucket

    g = torch.Generator().manual_seed(3)
    n, C, T = 4, 256, 33
    params = [0.5 * torch.randn(n, generator=g), 0.5 * torch.randn(n, generator=g),
              torch.randn(n, n, generator=g), 1 + 0.1 * torch.randn(C, generator=g)]
    x = torch.randn(T, n, C, generator=g).to(DEV)
    d = torch.randn(T, n, C, generator=g).to(DEV)

    def make():
        layer = mhc_b200.MHCLayer(n=n, C=C).to(DEV)
        with torch.no_grad():
            for p, v in zip(layer.parameters(), params):
                p.copy_(v)
        return layer

    plain, bound = make(), make()
    bucket = GradBucket(bound)
    plain(x).backward(d)
    bound(x).backward(d)
    for p, q, v in zip(plain.parameters(), bound.parameters(), bucket.views):
        assert q.grad.data_ptr() == v.data_ptr()
        assert torch.equal(p.grad, q.grad)
    bound(x).backward(d)  # accumulates into the views
    for p, q in zip(plain.parameters(), bound.parameters()):
        assert torch.allclose(q.grad, 2 * p.grad, rtol=1e-6, atol=1e-6)
    for q in bound.parameters():
        q.grad = None
    bound(x).backward(d)
    bucket.allreduce()
    for p, q in zip(plain.parameters(), bound.parameters()):
        assert torch.equal(p.grad, q.grad)
