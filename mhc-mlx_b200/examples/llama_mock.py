"""Llama-style decoder mock patched with mHC.

The reference's example (examples/patch_llama_mock.py) builds a mock Llama
block -- attention with wq/wk/wv/wo and no RoPE, mask or head split
(softmax((x Wq / sqrt(d)) (x Wk)^T) x Wv Wo), a SwiGLU MLP (w1, w2, w3) and
two RMSNorm pre-norm residuals -- and rewires every square Linear with
MHCRewire.  This module scales that to a full decoder: token embedding,
`layers` such blocks, a final RMSNorm and an LM head, random-initialised in
bf16.  The reference's patch rule wraps only square projections, so each
block gets four MHCRewire (wq, wk, wv, wo), n = 4 streams of C = dims / 4.

Training step (`train_step`): fine-tuning of the mHC parameters only (the
wrapped weights are frozen, as in the reference's quantized example); the
activation gradients still flow through every GEMM.  Sequences are sharded
over ranks; each rank runs its sequences one at a time (gradient
accumulation) and one bucketed NCCL all-reduce sums the mHC gradients.
The GEMMs and attention are library calls outside the mHC hot path.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from mhc_b200 import AutoPatcher
from mhc_b200.dist import allreduce_grads, mhc_parameters


class MockAttention(nn.Module):
    def __init__(self, dims: int, num_heads: int, **kw):
        super().__init__()
        self.num_heads = num_heads  # kept for parity with the reference; the mock uses one head
        self.wq = nn.Linear(dims, dims, bias=False, **kw)
        self.wk = nn.Linear(dims, dims, bias=False, **kw)
        self.wv = nn.Linear(dims, dims, bias=False, **kw)
        self.wo = nn.Linear(dims, dims, bias=False, **kw)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        # one head of width `dims`: two plain GEMMs and a softmax (fp32); the
        # fused SDPA kernels are not built for a 4096-wide head
        q, k, v = self.wq(x), self.wk(x), self.wv(x)
        scale = 1.0 / math.sqrt(x.shape[-1])
        scores = torch.matmul(q * scale, k.transpose(-1, -2))
        attn = torch.softmax(scores.float(), dim=-1).to(v.dtype)
        return self.wo(torch.matmul(attn, v))


class MockMLP(nn.Module):
    def __init__(self, dims: int, mlp_dims: int, **kw):
        super().__init__()
        self.w1 = nn.Linear(dims, mlp_dims, bias=False, **kw)
        self.w2 = nn.Linear(mlp_dims, dims, bias=False, **kw)
        self.w3 = nn.Linear(dims, mlp_dims, bias=False, **kw)

    def forward(self, x):
        return self.w2(F.silu(self.w1(x)) * self.w3(x))


class MockBlock(nn.Module):
    def __init__(self, dims: int, num_heads: int, mlp_dims: int, **kw):
        super().__init__()
        self.attention_norm = nn.RMSNorm(dims, **kw)
        self.attention = MockAttention(dims, num_heads, **kw)
        self.ffn_norm = nn.RMSNorm(dims, **kw)
        self.feed_forward = MockMLP(dims, mlp_dims, **kw)

    def forward(self, x):
        h = x + self.attention(self.attention_norm(x))
        return h + self.feed_forward(self.ffn_norm(h))


class LlamaMock(nn.Module):
    def __init__(self, layers: int = 32, dims: int = 4096, num_heads: int = 32,
                 mlp_dims: int = 11008, vocab: int = 32000, **kw):
        super().__init__()
        self.embed = nn.Embedding(vocab, dims, **kw)
        self.layers = nn.ModuleList(MockBlock(dims, num_heads, mlp_dims, **kw)
                                    for _ in range(layers))
        self.norm = nn.RMSNorm(dims, **kw)
        self.head = nn.Linear(dims, vocab, bias=False, **kw)

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        h = self.embed(tokens)
        for blk in self.layers:
            h = blk(h)
        return self.head(self.norm(h))


def build(layers=32, dims=4096, num_heads=32, mlp_dims=11008, vocab=32000, n_streams=4,
          dtype=torch.bfloat16, device="cuda", seed=0, mhc_seed=1) -> LlamaMock:
    """Random-initialised mock, patched with MHCRewire(n_streams) around every
    square projection, wrapped weights frozen, mHC logits ~ N(0, 0.1)."""
    torch.manual_seed(seed)
    model = LlamaMock(layers, dims, num_heads, mlp_dims, vocab, device=device, dtype=dtype)
    for p in model.parameters():
        p.requires_grad_(False)
    AutoPatcher.patch(model, n_streams=n_streams, verbose=False,
                      output_dtype="input" if dtype in (torch.bfloat16, torch.float16) else None)
    g = torch.Generator().manual_seed(mhc_seed)
    with torch.no_grad():
        for p in mhc_parameters(model):
            if p.ndim == 2 or p.shape[0] == n_streams:  # logits; rms_weight stays 1
                p.copy_(0.1 * torch.randn(p.shape, generator=g))
    return model


def train_step(model: LlamaMock, tokens: torch.Tensor, targets: torch.Tensor,
               global_tokens: int, lr: float = 1e-3) -> float:
    """One step over this rank's sequences [b, S]: mean cross-entropy over the
    global batch, mHC gradients accumulated per sequence, summed over ranks,
    SGD update.  Returns this rank's share of the loss."""
    params = mhc_parameters(model)
    for p in params:
        p.grad = None
    total = torch.zeros((), device=tokens.device, dtype=torch.float32)
    for b in range(tokens.shape[0]):
        logits = model(tokens[b:b + 1])
        loss = F.cross_entropy(logits.float().flatten(0, 1), targets[b:b + 1].flatten(),
                               reduction="sum") / global_tokens
        loss.backward()
        total += loss.detach()
    allreduce_grads(params)
    live = [p for p in params if p.grad is not None]  # MHCRewire leaves rms_weight unused
    with torch.no_grad():
        torch._foreach_add_(live, [p.grad for p in live], alpha=-lr)
    return total
