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
