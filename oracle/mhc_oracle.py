"""CPU oracle for the mHC hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in PyTorch on the CPU, the reference's pure-MLX source of
truth (svdrecbd/mhc-mlx, mhc_mlx/reference.py) operation for operation, and
the reference branches of mhc_mlx/layer.py that the CUDA path replaces.
Gradients come from torch autograd over these same functions, standing in for
MLX autodiff of reference.py (the reference's backward parity target).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import it, and only as the checker / the timed CPU baseline.  The product
package (mhc-mlx_b200/mhc_b200) never imports it and has no CPU path.

Pinning: the forward functions are checked against golden vectors produced
by executing the reference's own reference.py and layer.py (reference
branch) through a numpy-backed stand-in for mlx.core
(tests/golden/make_golden.py); the autograd gradients are checked against
central finite differences in float64 (tests/test_oracle.py).

Every function takes a `dtype` (float32 to mirror the reference, float64 to
measure the oracle's own rounding noise).
"""

from __future__ import annotations

import torch

F32 = torch.float32


# ------------------------------------------------------- reference.py:20-48 --
def sinkhorn_knopp(H: torch.Tensor, iters: int = 20, eps: float = 1e-5,
                   dtype: torch.dtype = F32) -> torch.Tensor:
    """Row step: scale 1/row_sum where row_sum > eps else 1; column step:
    1/col_sum where col_sum > eps else 0 (reference.py:37-46).  Works on
    [..., n, n] (batched over leading axes)."""
    P = H.to(dtype)
    for _ in range(iters):
        row_sum = P.sum(dim=-1)
        row_scale = torch.where(row_sum > eps, 1.0 / row_sum, torch.ones_like(row_sum))
        P = P * row_scale[..., :, None]
        col_sum = P.sum(dim=-2)
        col_scale = torch.where(col_sum > eps, 1.0 / col_sum, torch.zeros_like(col_sum))
        P = P * col_scale[..., None, :]
    return P


# ------------------------------------------------------- reference.py:51-55 --
def activate_pre_post(H_pre_raw, H_post_raw, dtype: torch.dtype = F32):
    return torch.sigmoid(H_pre_raw.to(dtype)), 2.0 * torch.sigmoid(H_post_raw.to(dtype))


# ------------------------------------------------------- reference.py:58-69 --
def mixing_matrix_from_logits(H_res_raw, iters: int = 20, eps: float = 1e-5,
                              dtype: torch.dtype = F32):
    """exp(H - rowmax) then Sinkhorn.  amax's gradient splits evenly over ties,
    as MLX's max VJP does."""
    if H_res_raw.ndim < 2 or H_res_raw.shape[-1] != H_res_raw.shape[-2]:
        raise ValueError(f"H_res_raw must be square [n, n], got shape {tuple(H_res_raw.shape)}")
    H = H_res_raw.to(dtype)
    H_shifted = H - torch.amax(H, dim=-1, keepdim=True)
    return sinkhorn_knopp(torch.exp(H_shifted), iters=iters, eps=eps, dtype=dtype)


# ------------------------------------------------------ reference.py:72-145 --
def stream_aggregate(x, H_pre, dtype: torch.dtype = F32):
    """y_agg[b, c] = sum_i H_pre[i] x[b, i, c]   (reference.py:72-86)"""
    return (x.to(dtype) * H_pre.to(dtype)[None, :, None]).sum(dim=1)


def rms_norm(x, weight, eps: float = 1e-5, dtype: torch.dtype = F32):
    """(x * 1/sqrt(mean(x^2) + eps)) * w   (reference.py:89-105)"""
    x_f = x.to(dtype)
    mean_sq = (x_f * x_f).mean(dim=-1, keepdim=True)
    inv_rms = 1.0 / torch.sqrt(mean_sq + eps)
    return (x_f * inv_rms) * weight.to(dtype)[None, :]


def stream_distribute(y_norm, H_post, dtype: torch.dtype = F32):
    """y_dist[b, i, c] = H_post[i] y_norm[b, c]   (reference.py:108-122)"""
    return y_norm.to(dtype)[:, None, :] * H_post.to(dtype)[None, :, None]


def stream_mix_ref(x, M, dtype: torch.dtype = F32):
    """x_mixed[b, i, c] = sum_j M[i, j] x[b, j, c]   (reference.py:125-145)"""
    return (M.to(dtype)[None, :, :, None] * x.to(dtype)[:, None, :, :]).sum(dim=2)


# ----------------------------------------------------- reference.py:148-184 --
def mhc_forward_fused_reference(x, M, H_pre_act, H_post_act, rms_weight, eps: float = 1e-5,
                                dtype: torch.dtype = F32):
    y_agg = stream_aggregate(x, H_pre_act, dtype)
    y_norm = rms_norm(y_agg, rms_weight, eps=eps, dtype=dtype)
    y_dist = stream_distribute(y_norm, H_post_act, dtype)
    return stream_mix_ref(x, M, dtype) + y_dist


def mhc_forward_reference(x, H_pre_raw, H_post_raw, H_res_raw, rms_weight,
                          sinkhorn_iters: int = 20, eps: float = 1e-5, dtype: torch.dtype = F32):
    H_pre_act, H_post_act = activate_pre_post(H_pre_raw, H_post_raw, dtype)
    M = mixing_matrix_from_logits(H_res_raw, iters=sinkhorn_iters, eps=eps, dtype=dtype)
    return mhc_forward_fused_reference(x, M, H_pre_act, H_post_act, rms_weight, eps, dtype)


# ------------------------------------------------ layer.py reference branches --
def post_combine_reference(x3, y3, H_pre_raw, H_post_raw, H_res_raw, iters: int = 20,
                           eps: float = 1e-5, dtype: torch.dtype = F32):
    """(y_inner + (M * H_pre) x) * H_post   (reference layer.py:332-337)"""
    H_pre_act, H_post_act = activate_pre_post(H_pre_raw, H_post_raw, dtype)
    M = mixing_matrix_from_logits(H_res_raw, iters=iters, eps=eps, dtype=dtype)
    M_final = M * H_pre_act.reshape(1, -1)
    x_mixed = torch.einsum("ij,...jd->...id", M_final, x3.to(dtype))
    n = x3.shape[1]
    return (y3.to(dtype) + x_mixed) * H_post_act.reshape(1, n, 1)


def rewire_reference(inner, x, n: int, H_pre_raw, H_post_raw, H_res_raw, iters: int = 20,
                     eps: float = 1e-5, dtype: torch.dtype = F32):
    """MHCRewire.__call__ (reference layer.py:469-492) with its reference
    post-combine.  `inner` is any callable on the flat layout."""
    dims = x.shape[-1]
    C = dims // n
    H_pre_act, _ = activate_pre_post(H_pre_raw, H_post_raw, dtype)
    x3 = x.reshape(-1, n, C)
    x_pre = (x3.to(dtype) * H_pre_act.reshape(1, n, 1)).reshape(x.shape)
    y_inner = inner(x_pre)
    out = post_combine_reference(x3, y_inner.reshape(-1, n, C), H_pre_raw, H_post_raw, H_res_raw,
                                 iters, eps, dtype)
    return out.reshape(x.shape)


def stream_mix_add_reference(x, M, y_dist, dtype: torch.dtype = F32):
    """out = stream_mix(x, M) + y_dist   (stream_mix_add.metal contract)"""
    return stream_mix_ref(x, M, dtype) + y_dist.to(dtype)


def residual_add_agg_reference(x, res, H_pre, dtype: torch.dtype = F32):
    """out = x + res; y_agg = sum_i H_pre[i] out_i  (reference utils.py:4-24,
    residual_add_agg.metal: fp32 add, aggregate of the fp32 sums)."""
    out = x.to(dtype) + res.to(dtype)
    return out, (out * H_pre.to(dtype)[None, :, None]).sum(dim=1)


# ----------------------------------------------------------------- grads --
def layer_grads(x, H_pre_raw, H_post_raw, H_res_raw, rms_weight, d_out, iters: int = 20,
                eps: float = 1e-5, dtype: torch.dtype = F32):
    """Forward + autograd backward of mhc_forward_reference with upstream
    gradient d_out.  Returns (out, dx, dH_pre_raw, dH_post_raw, dH_res_raw,
    d_rms_weight), all in `dtype`."""
    leaves = [t.detach().to(dtype).clone().requires_grad_(True)
              for t in (x, H_pre_raw, H_post_raw, H_res_raw, rms_weight)]
    out = mhc_forward_reference(*leaves, sinkhorn_iters=iters, eps=eps, dtype=dtype)
    grads = torch.autograd.grad(out, leaves, d_out.to(dtype))
    return (out.detach(), *grads)


def fused_grads(x, M, H_pre_act, H_post_act, rms_weight, d_out, eps: float = 1e-5,
                dtype: torch.dtype = F32):
    """Gradients of mhc_forward_fused_reference w.r.t. (x, M, H_pre_act,
    H_post_act, rms_weight) -- the VJP contract of metal.py:2787-2857."""
    leaves = [t.detach().to(dtype).clone().requires_grad_(True)
              for t in (x, M, H_pre_act, H_post_act, rms_weight)]
    out = mhc_forward_fused_reference(*leaves, eps=eps, dtype=dtype)
    grads = torch.autograd.grad(out, leaves, d_out.to(dtype))
    return (out.detach(), *grads)


def sinkhorn_grads(H_res_raw, dM, iters: int = 20, eps: float = 1e-5, dtype: torch.dtype = F32):
    """(M, dH_res_raw) for M = mixing_matrix_from_logits(H_res_raw); batched
    over leading axes."""
    H = H_res_raw.detach().to(dtype).clone().requires_grad_(True)
    M = mixing_matrix_from_logits(H, iters=iters, eps=eps, dtype=dtype)
    (dH,) = torch.autograd.grad(M, [H], dM.to(dtype))
    return M.detach(), dH
