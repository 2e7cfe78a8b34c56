"""QuantizedLinear: an affine, group-wise 4/8-bit linear layer for torch.

Stand-in for the MLX layer the reference wraps (``nn.QuantizedLinear`` with
``from_linear(linear, group_size, bits)``, used by tests/test_quantized.py:15
and examples/patch_llama_mock.py:90, recognised by patching.py:74-80).
Quantisation follows the published affine scheme: per row and per group of
``group_size`` input columns, w ~= scale * q + bias with q in [0, 2^bits - 1],
scale = (max - min) / (2^bits - 1), bias = min.  Codes are packed
little-endian into uint32 words (32 // bits codes per word); scales and
biases are stored in the weight's float dtype.

On CUDA with bf16 / fp16 activations, 4-bit codes and groups of 64 (the
configuration the reference uses), forward and input-gradient are one
tensor-core GEMM each with the weight dequantised tile by tile inside the
kernel (mhc_qlinear_fwd / mhc_qlinear_bwd_dx): the [out, in] weight is never
materialised.  Other configurations (2 / 8 bits, other group sizes, fp32 or
CPU activations) dequantise with torch ops and run torch.matmul; the wrapped
layer is outside the mHC hot path either way.  Its weights are buffers, so
the layer is frozen by construction; ``freeze()`` exists for API parity.
"""

from __future__ import annotations

import torch
from torch import nn

from . import _kernels as K


class _QLinearFn(torch.autograd.Function):
    """y = x W^T (+ bias) with W dequantised inside the GEMM; the backward
    gives the input gradient only (codes, scales and biases are frozen)."""

    @staticmethod
    def forward(ctx, x, weight, scales, biases, bias, group_size, bits, module=None):
        shape = x.shape
        y = K.qlinear_fwd(x.reshape(-1, shape[-1]), weight, scales, biases, bias, group_size,
                          bits)
        ctx.save_for_backward(weight, scales, biases)
        ctx.meta = (shape, x.dtype, group_size, bits)
        ctx.module = module
        return y.reshape(*shape[:-1], y.shape[-1])

    @staticmethod
    def backward(ctx, dy):
        weight, scales, biases = ctx.saved_tensors
        shape, dtype, group_size, bits = ctx.meta
        dx = None
        if ctx.needs_input_grad[0]:
            dy2 = dy.reshape(-1, dy.shape[-1]).to(dtype)
            if ctx.module is not None:
                wt, st, bt = ctx.module.transposed(dtype)
                dx = K.qlinear_bwd_dx_t(dy2, wt, st, bt, shape[-1], group_size, bits)
            else:
                dx = K.qlinear_bwd_dx(dy2, weight, scales, biases, shape[-1], group_size, bits)
            dx = dx.reshape(shape)
        return dx, None, None, None, None, None, None, None


class QuantizedLinear(nn.Module):
    def __init__(self, input_dims: int, output_dims: int, bias: bool = True,
                 group_size: int = 64, bits: int = 4, dtype=torch.float16, device=None):
        super().__init__()
        if bits not in (2, 4, 8):
            raise ValueError("bits must be one of 2, 4, 8")
        if input_dims % group_size != 0:
            raise ValueError(f"input_dims {input_dims} must be divisible by group_size {group_size}")
        self.input_dims = int(input_dims)
        self.output_dims = int(output_dims)
        self.group_size = int(group_size)
        self.bits = int(bits)
        per_word = 32 // self.bits
        if input_dims % per_word != 0:
            raise ValueError(f"input_dims must be divisible by {per_word} for {bits}-bit packing")
        g = input_dims // group_size
        self.register_buffer("weight", torch.zeros(output_dims, input_dims // per_word,
                                                   dtype=torch.int32, device=device))
        self.register_buffer("scales", torch.ones(output_dims, g, dtype=dtype, device=device))
        self.register_buffer("biases", torch.zeros(output_dims, g, dtype=dtype, device=device))
        if bias:
            self.register_buffer("bias", torch.zeros(output_dims, dtype=dtype, device=device))
        else:
            self.bias = None

    # ---------------------------------------------------------- packing --
    @staticmethod
    def pack(q: torch.Tensor, bits: int) -> torch.Tensor:
        """q: [out, in] integer codes in [0, 2^bits) -> [out, in * bits / 32] int32."""
        per_word = 32 // bits
        q = q.to(torch.int64).reshape(q.shape[0], -1, per_word)
        shifts = torch.arange(per_word, device=q.device, dtype=torch.int64) * bits
        words = (q << shifts).sum(dim=-1)
        words = torch.where(words >= 2**31, words - 2**32, words)
        return words.to(torch.int32)

    def codes(self) -> torch.Tensor:
        per_word = 32 // self.bits
        w = self.weight.to(torch.int64) & 0xFFFFFFFF
        shifts = torch.arange(per_word, device=w.device, dtype=torch.int64) * self.bits
        q = (w.unsqueeze(-1) >> shifts) & ((1 << self.bits) - 1)
        return q.reshape(self.output_dims, self.input_dims)

    def dequantize(self, dtype=None) -> torch.Tensor:
        q = self.codes().to(self.scales.dtype)
        q = q.reshape(self.output_dims, -1, self.group_size)
        w = q * self.scales.unsqueeze(-1) + self.biases.unsqueeze(-1)
        w = w.reshape(self.output_dims, self.input_dims)
        return w if dtype is None else w.to(dtype)

    @classmethod
    def from_linear(cls, linear: nn.Linear, group_size: int = 64, bits: int = 4):
        out_d, in_d = linear.weight.shape
        dtype = linear.weight.dtype if linear.weight.dtype != torch.float32 else torch.float16
        ql = cls(in_d, out_d, bias=linear.bias is not None, group_size=group_size, bits=bits,
                 dtype=dtype, device=linear.weight.device)
        with torch.no_grad():
            w = linear.weight.detach().float().reshape(out_d, -1, group_size)
            wmin = w.amin(dim=-1)
            wmax = w.amax(dim=-1)
            levels = (1 << bits) - 1
            scale = (wmax - wmin) / levels
            scale = torch.where(scale == 0, torch.ones_like(scale), scale)
            q = torch.round((w - wmin.unsqueeze(-1)) / scale.unsqueeze(-1)).clamp_(0, levels)
            ql.weight.copy_(cls.pack(q.reshape(out_d, in_d), bits))
            ql.scales.copy_(scale.to(dtype))
            ql.biases.copy_(wmin.to(dtype))
            if linear.bias is not None:
                ql.bias.copy_(linear.bias.detach().to(dtype))
        return ql

    @classmethod
    def random(cls, input_dims: int, output_dims: int, group_size: int = 64, bits: int = 4,
               dtype=torch.float16, device=None, generator: torch.Generator | None = None,
               scale_std: float = 0.02):
        """Random codes uniform in [0, 2^bits), scales/biases ~ N(0, scale_std)."""
        ql = cls(input_dims, output_dims, bias=False, group_size=group_size, bits=bits,
                 dtype=dtype, device=device)
        g = input_dims // group_size
        q = torch.randint(0, 1 << bits, (output_dims, input_dims), generator=generator)
        ql.weight.copy_(cls.pack(q, bits).to(ql.weight.device))
        ql.scales.copy_((torch.randn(output_dims, g, generator=generator) * scale_std).to(dtype))
        ql.biases.copy_((torch.randn(output_dims, g, generator=generator) * scale_std).to(dtype))
        return ql

    def freeze(self):
        """No trainable parameters: codes, scales and biases are buffers."""
        return self

    def _in_kernel(self, x: torch.Tensor) -> bool:
        return (x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and self.bits == 4
                and self.group_size == 64 and self.input_dims % 128 == 0
                and self.output_dims % 128 == 0
                and self.scales.dtype in (torch.bfloat16, torch.float16))

    def transposed(self, dtype: torch.dtype):
        """Transposed layouts of the frozen weight for the input-gradient GEMM,
        built once per activation dtype and cached (rebuilt if a buffer is
        replaced or modified): the codes of W^T packed like `weight`
        ([in, out/8] words, eight consecutive output rows per word) and the
        scales / biases as [in/group, out] in `dtype`.  4-bit codes take
        in*out/2 bytes: a copy of the packed weight, not a dequantised one."""
        key = (dtype, self.weight.data_ptr(), self.weight._version, self.scales._version,
               self.biases._version)
        cache = getattr(self, "_t_cache", None)
        if cache is not None and cache[0] == key:
            return cache[1]
        with torch.no_grad():
            wt = K.qlinear_transpose_pack(self.weight, self.input_dims)  # [in, out/8]
            st = self.scales.t().contiguous().to(dtype)                   # [in/group, out]
            bt = self.biases.t().contiguous().to(dtype)
        self._t_cache = (key, (wt, st, bt))
        return wt, st, bt

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self._in_kernel(x):
            return _QLinearFn.apply(x, self.weight, self.scales, self.biases, self.bias,
                                    self.group_size, self.bits, self)
        w = self.dequantize(dtype=x.dtype)
        y = torch.matmul(x, w.t())
        if self.bias is not None:
            y = y + self.bias.to(x.dtype)
        return y

    def extra_repr(self) -> str:
        return (f"input_dims={self.input_dims}, output_dims={self.output_dims}, "
                f"group_size={self.group_size}, bits={self.bits}")
