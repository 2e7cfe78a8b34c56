"""Data-parallel plumbing for the mHC path: shard tokens across ranks, then
one all-reduce of the (small) mHC parameter gradients per step.

The mHC layer is per-token, so ranks exchange nothing in the forward; the
only collective is the sum of dH_pre_raw, dH_post_raw, dH_res_raw and
d_rms_weight (n + n + n^2 + C floats per layer), bucketed into a single
flat buffer so one NCCL call covers every layer.  The reference has no
distributed code; this is the B200 build's scaling path.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_tokens(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Contiguous slice of the leading (token) axis owned by `rank`.  Ragged
    token counts give the first T % world ranks one extra token."""
    T = x.shape[0]
    base, extra = divmod(T, world)
    start = rank * base + min(rank, extra)
    return x[start:start + base + (1 if rank < extra else 0)]


def mhc_parameters(module: torch.nn.Module) -> list[torch.nn.Parameter]:
    """The mHC parameters (H_pre_raw, H_post_raw, H_res_raw, rms_weight) of
    every MHCLayer inside `module`, in a fixed order."""
    from .layer import MHCLayer

    out = []
    for m in module.modules():
        if isinstance(m, MHCLayer):
            out += [m.H_pre_raw, m.H_post_raw, m.H_res_raw, m.rms_weight]
    return out


def allreduce_grads(params, group=None, average: bool = False) -> None:
    """Sum (or average) .grad of `params` across the process group with one
    all-reduce on a flat bucket.  Parameters without a gradient contribute
    zeros, so every rank issues the same collective."""
    params = list(params)
    if not params or not dist.is_available() or not dist.is_initialized():
        return
    world = dist.get_world_size(group)
    if world == 1:
        return
    grads = [p.grad if p.grad is not None else torch.zeros_like(p) for p in params]
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    if average:
        flat.div_(world)
    off = 0
    for p, g in zip(params, grads):
        k = g.numel()
        v = flat[off:off + k].view_as(g)
        if p.grad is None:
            p.grad = v.clone()
        else:
            p.grad.copy_(v)
        off += k


class _Binding:
    """The parameters of one MHCLayer and their views in a GradBucket."""

    __slots__ = ("params", "views")

    def __init__(self, params, views):
        self.params, self.views = params, views


class GradBucket:
    """One flat fp32 buffer for the gradients of every MHCLayer parameter in
    `module`, so that a data-parallel step all-reduces them with a single
    NCCL call and no gather / scatter kernels.

    Each MHCLayer is bound to its views of the buffer: when its backward runs
    while none of its four parameters holds a gradient (the usual
    ``p.grad = None`` / ``zero_grad()`` before a step), the backward's
    finalize kernel writes the raw-parameter gradients directly into the
    views and makes them the parameters' ``.grad``.  Gradients that arrived
    any other way (accumulation over several backward passes, MHCRewire's
    parameter chain, unused parameters) are copied or zeroed into the buffer
    by ``allreduce`` before the collective, so the result is the same as
    ``allreduce_grads`` in every case."""

    def __init__(self, module: torch.nn.Module):
        from .layer import MHCLayer

        layers = [m for m in module.modules() if isinstance(m, MHCLayer)]
        self.params = []
        for m in layers:
            self.params += [m.H_pre_raw, m.H_post_raw, m.H_res_raw, m.rms_weight]
        if not self.params:
            raise ValueError("module holds no MHCLayer")
        dev = self.params[0].device
        self.flat = torch.zeros(sum(p.numel() for p in self.params), dtype=torch.float32,
                                device=dev)
        self.views = []
        off = 0
        for p in self.params:
            if p.dtype != torch.float32 or p.device != dev:
                raise ValueError("GradBucket expects fp32 mHC parameters on one device")
            self.views.append(self.flat[off:off + p.numel()].view_as(p))
            off += p.numel()
        for k, m in enumerate(layers):
            m._grad_binding = _Binding(self.params[4 * k:4 * k + 4],
                                       tuple(self.views[4 * k:4 * k + 4]))

    def allreduce(self, group=None, average: bool = False) -> None:
        """Sum (or average) the gradients across the process group: one
        all-reduce on the flat buffer; afterwards every parameter's .grad is
        its view of the reduced buffer."""
        for p, v in zip(self.params, self.views):
            g = p.grad
            if g is None:
                v.zero_()
                p.grad = v
            elif g.data_ptr() != v.data_ptr():
                v.copy_(g)
                p.grad = v
        if not dist.is_available() or not dist.is_initialized():
            return
        world = dist.get_world_size(group)
        if world == 1:
            return
        dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=group)
        if average:
            self.flat.div_(world)
