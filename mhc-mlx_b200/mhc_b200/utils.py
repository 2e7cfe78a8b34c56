"""Fused residual add + stream aggregate (reference mhc_mlx/utils.py:4-24)."""

from __future__ import annotations

import torch

from .metal import residual_add_agg_metal


def residual_add_agg(x: torch.Tensor, res: torch.Tensor, H_pre: torch.Tensor):
    """out = x + res;  y_agg = sum_i H_pre[i] * out[:, i, :].

    x, res: [B, n, C]; H_pre: [n] (used as given).  Returns (out [B, n, C]
    float32, y_agg [B, C] float32), reading each input once."""
    return residual_add_agg_metal(x, res, H_pre)
