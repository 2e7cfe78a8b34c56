"""Adaptive-dispatch entry points, under the reference's names.

The reference module mhc_mlx/metal.py launches Metal kernels through
mx.fast.metal_kernel.  This module keeps its public function names,
signatures and ValueError conditions, and routes every call to the sm_100a
CUDA kernels of libmhc_b200.so (through ``_kernels``).  Metal-only knobs
(``threads_per_group``, ``mix_kernel``, ``verbose``) are validated as in the
reference and otherwise have no effect on B200: launch shapes are chosen by
the library from n, C, the dtypes and the device's SM count.

Autograd: the ``*_autograd`` functions are torch.autograd.Function wrappers
whose backward runs the fused CUDA backward kernels (reference: the
mx.custom_function VJPs at metal.py:2661-2900).
"""

from __future__ import annotations

import torch

from . import _kernels as K

_MAX_N_ALLOWED = 64  # reference metal.py:71
_MAX_TPG_ALLOWED = 1024  # reference metal.py:72

_HALF = (torch.float16, torch.bfloat16)


# ------------------------------------------------------------- validation --
def _validate_n(n: int) -> int:
    """reference metal.py:826-833"""
    if n <= 0:
        raise ValueError("n must be positive")
    if n > _MAX_N_ALLOWED:
        raise ValueError(
            f"n={n} exceeds MAX_N_ALLOWED={_MAX_N_ALLOWED}. Increase _MAX_N_ALLOWED if needed."
        )
    return int(n)


def _validate_tpg(threads_per_group, what: str = "") -> None:
    if threads_per_group is None:
        return
    if threads_per_group <= 0:
        raise ValueError("threads_per_group must be positive")
    if threads_per_group > _MAX_TPG_ALLOWED:
        raise ValueError(f"threads_per_group must be <= {_MAX_TPG_ALLOWED}{what}")


def _normalize_output_dtype(output_dtype):
    """reference metal.py:855-860"""
    if output_dtype is None:
        return None
    if output_dtype in (torch.float32, torch.float16, torch.bfloat16):
        return output_dtype
    raise ValueError(f"unsupported output_dtype: {output_dtype}")


def _normalize_mix_kernel(mix_kernel: str) -> str:
    """reference metal.py:863-867"""
    key = (mix_kernel or "auto").strip().lower()
    if key in {"auto", "1d", "2d", "col"}:
        return key
    raise ValueError(f"unsupported mix_kernel: {mix_kernel}")


def _out_dtype_for(x: torch.Tensor, output_dtype) -> torch.dtype:
    """fp32 unless a half output_dtype matching x is requested
    (reference metal.py:1610-1616)."""
    output_dtype = _normalize_output_dtype(output_dtype)
    if output_dtype in _HALF:
        if x.dtype != output_dtype:
            raise ValueError(f"x must be {output_dtype} when output_dtype is {output_dtype}")
        return output_dtype
    return torch.float32


def _maybe_print(name: str, verbose: bool) -> None:
    if verbose:
        print(f"--- {name}: sm_100a CUDA kernel in libmhc_b200.so (no runtime source) ---")


def _check_x3(x: torch.Tensor, name: str = "x") -> tuple[int, int, int]:
    if x.ndim != 3:
        raise ValueError(f"{name} must be [B, n, C], got shape {tuple(x.shape)}")
    B, n, C = x.shape
    return int(B), int(n), int(C)


def _check_params(x, M, H_pre, H_post, rms_weight):
    """Shape checks of reference metal.py:1852-1873."""
    _check_x3(x)
    if M.ndim != 2:
        raise ValueError(f"M must be [n, n], got shape {tuple(M.shape)}")
    if H_pre.ndim != 1:
        raise ValueError(f"H_pre must be [n], got shape {tuple(H_pre.shape)}")
    if H_post.ndim != 1:
        raise ValueError(f"H_post must be [n], got shape {tuple(H_post.shape)}")
    if rms_weight.ndim != 1:
        raise ValueError(f"rms_weight must be [C], got shape {tuple(rms_weight.shape)}")
    B, n, C = x.shape
    if tuple(M.shape) != (n, n):
        raise ValueError(f"M must be shape (n,n)=( {n},{n} ), got {tuple(M.shape)}")
    if tuple(H_pre.shape) != (n,):
        raise ValueError(f"H_pre must be shape (n,)=( {n}, ), got {tuple(H_pre.shape)}")
    if tuple(H_post.shape) != (n,):
        raise ValueError(f"H_post must be shape (n,)=( {n}, ), got {tuple(H_post.shape)}")
    if tuple(rms_weight.shape) != (C,):
        raise ValueError(f"rms_weight must be shape (C,)=( {C}, ), got {tuple(rms_weight.shape)}")
    return _validate_n(n)


# --------------------------------------------------- launch-shape helpers --
def suggest_threads_per_group(C: int, max_tpg: int = _MAX_TPG_ALLOWED) -> int:
    """Next power of two >= C, capped (reference metal.py:942-951)."""
    if C <= 0:
        raise ValueError("C must be positive")
    if max_tpg <= 0:
        raise ValueError("max_tpg must be positive")
    tpg = 1 << (int(C) - 1).bit_length()
    return int(min(tpg, int(max_tpg)))


def _tile_tpg_x(n: int, requested: int) -> int:
    if n <= 0:
        raise ValueError("n must be positive")
    if requested <= 0:
        raise ValueError("requested must be positive")
    cap = min(_MAX_TPG_ALLOWED, _MAX_TPG_ALLOWED // int(n))
    if cap <= 0:
        return 1
    target = min(int(requested), int(cap))
    return max(1, 1 << (target.bit_length() - 1))


def mix_add_rms_threadgroup_size(n: int, output_dtype, threads_per_group: int,
                                 mix_kernel: str = "auto") -> int:
    """Threadgroup size the reference's Metal mix/add/RMS kernel would use
    (reference metal.py:915-939); kept for API compatibility.  The CUDA
    kernels size their CTAs from n, C and dtype instead."""
    output_dtype = _normalize_output_dtype(output_dtype)
    mix_kernel = _normalize_mix_kernel(mix_kernel)
    tile_c = None
    if n in (16, 32):
        tile_c = 8 if n == 16 else 4
    if mix_kernel == "2d":
        return int(_tile_tpg_x(n, threads_per_group) * n)
    if mix_kernel == "1d":
        return int(threads_per_group) if tile_c is None else int(n * tile_c)
    if n >= 16 and (output_dtype is None or output_dtype in _HALF):
        return int(_tile_tpg_x(n, threads_per_group) * n)
    return int(threads_per_group) if tile_c is None else int(n * tile_c)


# ---------------------------------------------------------------- Sinkhorn --
def _check_square(H: torch.Tensor) -> int:
    if H.ndim != 2 or H.shape[0] != H.shape[1]:
        raise ValueError(f"H_res_raw must be square [n, n], got shape {tuple(H.shape)}")
    return _validate_n(H.shape[0])


def sinkhorn_knopp_metal(H_res_raw: torch.Tensor, iters: int = 20, eps: float = 1e-5,
                         threads_per_group: int | None = None,
                         verbose: bool = False) -> torch.Tensor:
    """M = sinkhorn_knopp(exp(H_res_raw - rowmax)) (reference metal.py:1525-1577;
    math reference.py:58-69).  Returns [n, n] float32."""
    _check_square(H_res_raw)
    _validate_tpg(threads_per_group)
    _maybe_print("sinkhorn_knopp", verbose)
    _, _, M, _ = K.params_fwd(None, None, H_res_raw, int(iters), float(eps), want_tape=False)
    return M


def sinkhorn_knopp_backward_metal(H_res_raw: torch.Tensor, dM: torch.Tensor, iters: int = 20,
                                  eps: float = 1e-5, threads_per_group: int = 64,
                                  verbose: bool = False) -> torch.Tensor:
    """dH_res for M = sinkhorn_knopp(exp(H_res_raw)) (reference metal.py:1978-2016)."""
    _check_square(H_res_raw)
    if tuple(dM.shape) != tuple(H_res_raw.shape):
        raise ValueError(
            f"dM must match H_res_raw shape, got {tuple(dM.shape)} vs {tuple(H_res_raw.shape)}")
    _validate_tpg(threads_per_group)
    _maybe_print("sinkhorn_knopp_backward", verbose)
    _, _, _, tape = K.params_fwd(None, None, H_res_raw, int(iters), float(eps), want_tape=True)
    _, _, dH = K.params_bwd(None, None, H_res_raw, tape, int(iters), float(eps), None, None, dM)
    return dH


class _SinkhornFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, H_res_raw, iters, eps):
        _, _, M, tape = K.params_fwd(None, None, H_res_raw, iters, eps, want_tape=True)
        ctx.save_for_backward(H_res_raw, tape if tape is not None else M.new_empty(0))
        ctx.iters, ctx.eps, ctx.has_tape = iters, eps, tape is not None
        return M

    @staticmethod
    def backward(ctx, dM):
        H, tape = ctx.saved_tensors
        _, _, dH = K.params_bwd(None, None, H, tape if ctx.has_tape else None, ctx.iters, ctx.eps,
                                None, None, dM)
        return dH, None, None


def sinkhorn_knopp_metal_autograd(H_res_raw: torch.Tensor, iters: int = 20, eps: float = 1e-5,
                                  threads_per_group: int | None = None,
                                  verbose: bool = False) -> torch.Tensor:
    """Sinkhorn with the CUDA backward (reference metal.py:2744-2758)."""
    _check_square(H_res_raw)
    _validate_tpg(threads_per_group)
    _maybe_print("sinkhorn_knopp", verbose)
    return _SinkhornFn.apply(H_res_raw, int(iters), float(eps))


class _BatchedSinkhornFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, H, iters, eps):
        ctx.save_for_backward(H)
        ctx.iters, ctx.eps = iters, eps
        return K.sinkhorn_batched_fwd(H, iters, eps)

    @staticmethod
    def backward(ctx, dM):
        (H,) = ctx.saved_tensors
        return K.sinkhorn_batched_bwd(H, dM, ctx.iters, ctx.eps), None, None


def sinkhorn_knopp_batched(H_res_raw: torch.Tensor, iters: int = 20,
                           eps: float = 1e-5) -> torch.Tensor:
    """Batched Sinkhorn over [batch, n, n] logits (new surface: the reference
    accepts a single 2-D matrix, reference.py:64-65).  Differentiable."""
    if H_res_raw.ndim != 3 or H_res_raw.shape[1] != H_res_raw.shape[2]:
        raise ValueError(f"H_res_raw must be [batch, n, n], got shape {tuple(H_res_raw.shape)}")
    _validate_n(H_res_raw.shape[1])
    return _BatchedSinkhornFn.apply(H_res_raw, int(iters), float(eps))


# ------------------------------------------------------------ fused layer --
def mhc_forward_fused_metal(x: torch.Tensor, M: torch.Tensor, H_pre: torch.Tensor,
                            H_post: torch.Tensor, rms_weight: torch.Tensor, eps: float = 1e-5,
                            threads_per_group: int | None = None, output_dtype=None,
                            mix_kernel: str = "auto", verbose: bool = False) -> torch.Tensor:
    """Aggregate + RMSNorm + mix + residual add in one pass
    (reference metal.py:1823-1975; math reference.py:148-161).

    x: [B, n, C] (fp32 / fp16 / bf16, read in place); M: [n, n]; H_pre, H_post:
    [n] activated; rms_weight: [C].  Returns fp32 unless output_dtype is a
    half dtype equal to x's dtype.
    """
    _check_params(x, M, H_pre, H_post, rms_weight)
    _validate_tpg(threads_per_group, " for the fused kernel")
    _normalize_mix_kernel(mix_kernel)
    out_dtype = _out_dtype_for(x, output_dtype)
    _maybe_print("mhc_fwd", verbose)
    return K.layer_fwd(x, M, H_pre, H_post, rms_weight, float(eps), out_dtype)


def mhc_fully_fused_metal(x, M, H_pre, H_post, rms_weight, eps: float = 1e-5,
                          threads_per_group: int | None = None, output_dtype=None,
                          verbose: bool = False) -> torch.Tensor:
    """Reference metal.py:1580-1643 (one threadgroup per token); on B200 the
    single fused kernel covers every size, so this is the same call."""
    if x.ndim != 3:
        raise ValueError(f"x must be [B, n, C], got shape {tuple(x.shape)}")
    return mhc_forward_fused_metal(x, M, H_pre, H_post, rms_weight, eps=eps,
                                   threads_per_group=threads_per_group,
                                   output_dtype=output_dtype, verbose=verbose)


def mhc_backward_fused_metal(x, M, H_pre, H_post, rms_weight, d_out, eps: float = 1e-5,
                             threads_per_group: int | None = None, verbose: bool = False):
    """Full backward of the fused forward: (dx, dM, dH_pre, dH_post, d_rms_weight).

    Replaces the reference's backward kernel chain (metal.py:2787-2857:
    prep_tile, rms_reduce, dx, dM, dH_pre, dH_post, d_rms_weight) with one
    pass over x and d_out plus a deterministic reduction."""
    _check_params(x, M, H_pre, H_post, rms_weight)
    if tuple(d_out.shape) != tuple(x.shape):
        raise ValueError(f"d_out must match x shape, got {tuple(d_out.shape)} vs {tuple(x.shape)}")
    _validate_tpg(threads_per_group)
    _maybe_print("mhc_bwd", verbose)
    return K.layer_bwd(x, d_out, M, H_pre, H_post, rms_weight, float(eps))


class _FusedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, M, H_pre, H_post, rms_weight, eps, out_dtype):
        ctx.save_for_backward(x, M, H_pre, H_post, rms_weight)
        ctx.eps = eps
        return K.layer_fwd(x, M, H_pre, H_post, rms_weight, eps, out_dtype)

    @staticmethod
    def backward(ctx, dout):
        x, M, H_pre, H_post, w = ctx.saved_tensors
        dx, dM, dpre, dpost, dw = K.layer_bwd(x, dout, M, H_pre, H_post, w, ctx.eps)
        return dx, dM, dpre, dpost, dw, None, None


def mhc_forward_fused_metal_autograd(x: torch.Tensor, M: torch.Tensor, H_pre: torch.Tensor,
                                     H_post: torch.Tensor, rms_weight: torch.Tensor,
                                     eps: float = 1e-5, threads_per_group: int | None = None,
                                     fused_backward: bool = True, output_dtype=None,
                                     mix_kernel: str = "auto",
                                     verbose: bool = False) -> torch.Tensor:
    """Fused forward with the fused CUDA backward (reference metal.py:2862-2900).
    ``fused_backward`` is accepted for compatibility: the CUDA backward is
    always the single-pass kernel + deterministic finalize."""
    _check_params(x, M, H_pre, H_post, rms_weight)
    _validate_tpg(threads_per_group)
    _normalize_mix_kernel(mix_kernel)
    out_dtype = _out_dtype_for(x, output_dtype)
    _maybe_print("mhc_fwd/mhc_bwd", verbose)
    return _FusedFn.apply(x, M, H_pre, H_post, rms_weight, float(eps), out_dtype)


# ------------------------------------------------------------ stream mix --
def _check_mix(x, M, y_dist):
    if x.ndim != 3:
        raise ValueError(f"x must be [B, n, C], got shape {tuple(x.shape)}")
    if M.ndim != 2:
        raise ValueError(f"M must be [n, n], got shape {tuple(M.shape)}")
    if tuple(y_dist.shape) != tuple(x.shape):
        raise ValueError(f"y_dist must match x shape, got {tuple(y_dist.shape)} vs {tuple(x.shape)}")
    n = x.shape[1]
    if tuple(M.shape) != (n, n):
        raise ValueError(f"M must be shape (n,n)=( {n},{n} ), got {tuple(M.shape)}")
    return _validate_n(n)


def stream_mix_add_metal(x: torch.Tensor, M: torch.Tensor, y_dist: torch.Tensor,
                         threads_per_group: int | None = None,
                         verbose: bool = False) -> torch.Tensor:
    """out = stream_mix(x, M) + y_dist, fp32 out (reference metal.py:954-1014)."""
    _check_mix(x, M, y_dist)
    _validate_tpg(threads_per_group)
    _maybe_print("mhc_mix_add_fwd", verbose)
    return K.mix_add_fwd(x, M, y_dist, torch.float32)


def stream_mix_backward_dx_metal(M: torch.Tensor, d_out: torch.Tensor,
                                 threads_per_group: int = 256, verbose: bool = False):
    """dx = M^T d_out (reference metal.py:2599-2640)."""
    if d_out.ndim != 3:
        raise ValueError(f"d_out must be [B, n, C], got shape {tuple(d_out.shape)}")
    if M.ndim != 2:
        raise ValueError(f"M must be [n, n], got shape {tuple(M.shape)}")
    n = d_out.shape[1]
    if tuple(M.shape) != (n, n):
        raise ValueError(f"M must be shape (n,n)=( {n},{n} ), got {tuple(M.shape)}")
    _validate_n(n)
    _validate_tpg(threads_per_group)
    # the fused mix backward also produces dM; x = d_out stands in for x
    dx, _ = K.mix_add_bwd(d_out.float(), M, d_out)
    return dx


def mhc_backward_dM_metal(x: torch.Tensor, d_out: torch.Tensor, threads_per_group: int = 256,
                          verbose: bool = False) -> torch.Tensor:
    """dM[i, j] = sum_{b,c} d_out[b,i,c] x[b,j,c] (reference metal.py:2297-2333)."""
    if x.ndim != 3:
        raise ValueError(f"x must be [B, n, C], got shape {tuple(x.shape)}")
    if tuple(d_out.shape) != tuple(x.shape):
        raise ValueError(f"d_out must match x shape, got {tuple(d_out.shape)} vs {tuple(x.shape)}")
    n = _validate_n(x.shape[1])
    _validate_tpg(threads_per_group)
    eye = torch.eye(n, dtype=torch.float32, device=x.device)
    _, dM = K.mix_add_bwd(x, eye, d_out)
    return dM


class _MixAddFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, M, y_dist):
        ctx.save_for_backward(x, M)
        ctx.y_dtype = y_dist.dtype
        return K.mix_add_fwd(x, M, y_dist, torch.float32)

    @staticmethod
    def backward(ctx, dout):
        x, M = ctx.saved_tensors
        dx, dM = K.mix_add_bwd(x, M, dout)
        return dx, dM, dout.to(ctx.y_dtype)


def stream_mix_add_metal_autograd(x: torch.Tensor, M: torch.Tensor, y_dist: torch.Tensor,
                                  threads_per_group: int | None = None,
                                  verbose: bool = False) -> torch.Tensor:
    """Stream mix + add with the CUDA backward (reference metal.py:2695-2709)."""
    _check_mix(x, M, y_dist)
    _validate_tpg(threads_per_group)
    _maybe_print("mhc_mix_add_fwd/bwd", verbose)
    return _MixAddFn.apply(x, M, y_dist)


# ------------------------------------------------------- residual add agg --
def residual_add_agg_metal(x: torch.Tensor, res: torch.Tensor, H_pre: torch.Tensor,
                           threads_per_group: int | None = None, output_dtype=None,
                           verbose: bool = False):
    """out = x + res; y_agg = sum_i H_pre[i] out[:, i, :]  (reference
    metal.py:1673-1731).  out is fp32 unless output_dtype is given; y_agg fp32.
    Forward only, as in the reference (no VJP registered there)."""
    if x.ndim != 3:
        raise ValueError(f"x must be [B, n, C], got shape {tuple(x.shape)}")
    if tuple(res.shape) != tuple(x.shape):
        raise ValueError(f"res must match x shape, got {tuple(res.shape)} vs {tuple(x.shape)}")
    _validate_n(x.shape[1])
    if threads_per_group is not None and threads_per_group <= 0:
        raise ValueError("threads_per_group must be positive")
    output_dtype = _normalize_output_dtype(output_dtype)
    out_dtype = output_dtype or torch.float32
    if x.dtype != res.dtype:
        x, res = x.float(), res.float()
    _maybe_print("mhc_residual_add_agg", verbose)
    return _ResidualAddAggFn.apply(x, res, H_pre, out_dtype)


class _ResidualAddAggFn(torch.autograd.Function):
    """Adds the VJP the reference lacks: dx = dres = d_out + H_pre (x) d_y,
    dH_pre = sum d_y * out."""

    @staticmethod
    def forward(ctx, x, res, H_pre, out_dtype):
        out, y = K.residual_add_agg(x, res, H_pre, out_dtype)
        ctx.save_for_backward(out, H_pre)
        ctx.dtypes = (x.dtype, res.dtype)
        return out, y

    @staticmethod
    def backward(ctx, d_out, d_y):
        out, H_pre = ctx.saved_tensors
        dx, dpre = K.residual_add_agg_bwd(out, d_out, d_y, H_pre, ctx.dtypes[0])
        dres = dx if ctx.dtypes[1] == ctx.dtypes[0] else dx.to(ctx.dtypes[1])
        return dx, dres, dpre, None
