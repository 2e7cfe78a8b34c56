"""Multi-rank host logic on CPU with gloo (world size 2): token sharding plus
the one bucketed all-reduce of mHC parameter gradients reproduces the
single-process full-batch gradients; a rank that dies before the collective
makes the survivor fail with an error instead of hanging.  Gradients per
shard come from the CPU oracle -- this checks the distributed plumbing, not
the kernels (those are covered by the GPU tests)."""

from __future__ import annotations

import datetime
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(rank, world, port, timeout_s=30):
    for p in (str(ROOT), str(ROOT / "mhc-mlx_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _problem(T=10, n=4, C=32):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(T, n, C, generator=g)
    d = torch.randn(T, n, C, generator=g)
    params = [0.5 * torch.randn(n, generator=g), 0.5 * torch.randn(n, generator=g),
              torch.randn(n, n, generator=g), 1 + 0.1 * torch.randn(C, generator=g)]
    return x, d, params


def _worker_equivalence(rank, world, port, q):
    try:
        _setup(rank, world, port)
        from mhc_b200 import MHCLayer
        from mhc_b200.dist import allreduce_grads, mhc_parameters, shard_tokens
        from oracle import mhc_oracle as O

        x, d, params = _problem()
        layer = MHCLayer(n=4, C=32)
        with torch.no_grad():
            for p, v in zip(mhc_parameters(layer), params):
                p.copy_(v)
        xs, ds = shard_tokens(x, rank, world), shard_tokens(d, rank, world)
        grads = O.layer_grads(xs, *params, ds, 20, 1e-5, dtype=torch.float64)[2:]
        for p, gr in zip(mhc_parameters(layer), grads):
            p.grad = gr.float()
        allreduce_grads(mhc_parameters(layer))
        q.put((rank, xs.shape[0], [p.grad.tolist() for p in mhc_parameters(layer)]))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, -1, repr(e)))


def test_sharded_allreduce_matches_full_batch():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_equivalence, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(r[1] > 0 for r in res), res
    assert sum(r[1] for r in res) == 10  # ragged: 5 + 5
    sys.path.insert(0, str(ROOT))
    from oracle import mhc_oracle as O

    x, d, params = _problem()
    full = O.layer_grads(x, *params, d, 20, 1e-5, dtype=torch.float64)[2:]
    for r in res:
        for a, b in zip(r[2], full):
            assert torch.allclose(torch.tensor(a).double(), b, rtol=1e-5, atol=1e-6)


def _worker_bucket(rank, world, port, q):
    try:
        _setup(rank, world, port)
        from mhc_b200 import MHCLayer
        from mhc_b200.dist import GradBucket, allreduce_grads, mhc_parameters

        torch.manual_seed(rank)
        model = torch.nn.Sequential(MHCLayer(n=4, C=32), MHCLayer(n=2, C=8))
        ps = mhc_parameters(model)
        grads = [torch.randn(p.shape) * (k + 1) for k, p in enumerate(ps)]
        # reference: the gather/scatter all-reduce
        for p, g in zip(ps, grads):
            p.grad = g.clone()
        allreduce_grads(ps)
        want = [p.grad.clone() for p in ps]
        # bucket: gradients arriving as plain tensors, one parameter without a
        # gradient (zeros), one already holding its bucket view
        bucket = GradBucket(model)
        for p, g in zip(ps, grads):
            p.grad = g.clone()
        ps[3].grad = None
        bucket.views[5].copy_(grads[5])
        ps[5].grad = bucket.views[5]
        bucket.allreduce()
        want[3] = torch.zeros_like(want[3])
        got = [p.grad.clone() for p in ps]
        views_ok = all(p.grad.data_ptr() == v.data_ptr() for p, v in zip(ps, bucket.views))
        # plain lists: a worker's tensors would be shared by file descriptor and
        # the worker may exit before the parent reads them
        q.put((rank, views_ok, [g.tolist() for g in got], [w.tolist() for w in want]))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, False, repr(e), None))


def test_grad_bucket_allreduce_matches_gather_scatter():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_bucket, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, views_ok, got, want in res:
        assert views_ok, got
        # parameter 3 has no gradient on either rank in the bucket run: zeros
        for k, (a, b) in enumerate(zip(got, want)):
            assert torch.allclose(torch.tensor(a), torch.tensor(b)), k


def _worker_dead_peer(rank, world, port, q):
    _setup(rank, world, port, timeout_s=10)
    from mhc_b200.dist import allreduce_grads

    if rank == 1:
        os._exit(3)  # leaves between steps, before its collective
    p = torch.nn.Parameter(torch.zeros(4))
    p.grad = torch.ones(4)
    try:
        allreduce_grads([p])
        q.put("no error")
    except Exception as e:
        q.put("error: " + type(e).__name__)


def test_dead_rank_fails_survivor_with_error():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_dead_peer, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    msg = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert msg.startswith("error"), msg


def test_shard_tokens_ragged():
    sys.path.insert(0, str(ROOT / "mhc-mlx_b200"))
    from mhc_b200.dist import shard_tokens

    x = torch.arange(11)
    parts = [shard_tokens(x, r, 3) for r in range(3)]
    assert [len(p) for p in parts] == [4, 4, 3]
    assert torch.equal(torch.cat(parts), x)
