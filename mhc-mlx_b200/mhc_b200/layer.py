"""MHCLayer and MHCRewire as torch modules over the sm_100a kernels.

Same constructor arguments, parameters, initialisation and call semantics as
the reference (mhc_mlx/layer.py:58-492):

- H_pre_act = sigmoid(H_pre_raw), H_post_act = 2 sigmoid(H_post_raw)
- M = sinkhorn_knopp(exp(H_res_raw - rowmax))
- out = stream_mix(x, M) + H_post_act (x) RMSNorm(sum_i H_pre_act[i] x_i)

Forward + backward of MHCLayer is four kernel launches: the parameter
kernel (sigmoids + Sinkhorn, recording the Sinkhorn tape), the fused
forward, the fused backward, and one finalize launch that reduces the
parameter partials and runs the Sinkhorn / sigmoid chain rule.

Differences from the reference, by design: there is no non-CUDA path, so
``use_metal=False`` or ``MHC_MLX_DISABLE_METAL=1`` raise instead of
silently switching to a slower implementation, and a kernel failure raises
instead of warning and falling back (reference layer.py:408-422).
"""

from __future__ import annotations

import os

import torch
from torch import nn

from . import _kernels as K
from .metal import _HALF, _validate_n

_DISABLE_ENV = "MHC_MLX_DISABLE_METAL"


# ------------------------------------------------------- autograd functions --
class _LayerFn(torch.autograd.Function):
    """x, raw parameters, rms_weight -> out (fused parameter chain)."""

    @staticmethod
    def forward(ctx, x, H_pre_raw, H_post_raw, H_res_raw, rms_weight, iters, eps, out_dtype,
                bound=None):
        hpre, hpost, M, tape = K.params_fwd(H_pre_raw, H_post_raw, H_res_raw, iters, eps,
                                            want_tape=True)
        out = K.layer_fwd(x, M, hpre, hpost, rms_weight, eps, out_dtype)
        empty = M.new_empty(0)
        ctx.save_for_backward(x, H_pre_raw, H_post_raw, H_res_raw, rms_weight, hpre, hpost, M,
                              tape if tape is not None else empty)
        ctx.iters, ctx.eps, ctx.bound = iters, eps, bound
        return out

    @staticmethod
    def backward(ctx, dout):
        x, pre, post, res, w, hpre, hpost, M, tape = ctx.saved_tensors
        raw = (pre, post, res, tape if tape.numel() else None, ctx.iters)
        bound = ctx.bound
        # a gradient bucket (mhc_b200.dist.GradBucket) bound to this layer:
        # when none of the four parameters holds a gradient yet, the finalize
        # writes straight into the bucket's views, which become their .grad
        # (nothing to accumulate into, no copy); otherwise autograd
        # accumulates the returned gradients as usual
        if bound is not None and all(p.grad is None for p in bound.params):
            dx, *_ = K.layer_bwd(x, dout, M, hpre, hpost, w, ctx.eps, raw=raw, out=bound.views)
            for p, v in zip(bound.params, bound.views):
                p.grad = v
            return dx, None, None, None, None, None, None, None, None
        dx, gpre, gpost, gres, dw = K.layer_bwd(x, dout, M, hpre, hpost, w, ctx.eps, raw=raw)
        return dx, gpre, gpost, gres, dw, None, None, None, None


class _ParamsFn(torch.autograd.Function):
    """Raw parameters -> (H_pre_act, H_post_act, M) in one launch."""

    @staticmethod
    def forward(ctx, H_pre_raw, H_post_raw, H_res_raw, iters, eps):
        hpre, hpost, M, tape = K.params_fwd(H_pre_raw, H_post_raw, H_res_raw, iters, eps,
                                            want_tape=True)
        ctx.save_for_backward(H_pre_raw, H_post_raw, H_res_raw,
                              tape if tape is not None else M.new_empty(0))
        ctx.iters, ctx.eps = iters, eps
        return hpre, hpost, M

    @staticmethod
    def backward(ctx, dhpre, dhpost, dM):
        pre, post, res, tape = ctx.saved_tensors
        z = pre.new_zeros
        dhpre = dhpre if dhpre is not None else z(pre.shape)
        dhpost = dhpost if dhpost is not None else z(post.shape)
        dM = dM if dM is not None else z(res.shape)
        gpre, gpost, gres = K.params_bwd(pre, post, res, tape if tape.numel() else None,
                                         ctx.iters, ctx.eps, dhpre, dhpost, dM)
        return gpre, gpost, gres, None, None


class _RewireLink:
    """Hands d_out (and the partial sums of the dy side) from the
    post-combine's backward to the pre-scale's backward within one
    MHCRewire call, so that its backward writes dx once and reduces dH_pre
    once (see _RewireCombineFn.backward)."""

    __slots__ = ("state",)

    def __init__(self):
        self.state = None


class _RewireInputFn(torch.autograd.Function):
    """MHCRewire's input side (reference layer.py:474-480): the wrapped
    MHCLayer's activations from its raw parameters, then
    x_pre[t, i, c] = x[t, i, c] * H_pre_act[i] -- one launch for n <= 8.

    Outputs (x_pre, H_pre_act, H_post_act, M); the last three feed the
    post-combine.  When the post-combine's backward has handed over d_out
    through `link`, this backward is the x side of MHCRewire's end-to-end
    backward and returns the raw-parameter gradients of the whole layer from
    the same finalize launch (the Sinkhorn / sigmoid chain rule folded in).
    Otherwise the post-combine returned its own activation gradients, and
    they are added to the pre-scale's before the parameter backward."""

    @staticmethod
    def forward(ctx, x, H_pre_raw, H_post_raw, H_res_raw, iters, eps, link):
        ctx.set_materialize_grads(False)
        x_pre, hpre, hpost, M, raw = K.rewire_in_fwd(x, H_pre_raw, H_post_raw, H_res_raw,
                                                     iters, eps)
        pre, post, res, tape, jac, _, _ = raw
        z = M.new_empty(0)
        ctx.save_for_backward(x, pre, post, res, hpre, hpost, M,
                              tape if tape is not None else z, jac if jac is not None else z)
        ctx.iters, ctx.eps, ctx.link = iters, eps, link
        return x_pre, hpre, hpost, M

    @staticmethod
    def backward(ctx, d, dhpre, dhpost, dM):
        x, pre, post, res, hpre, hpost, M, tape, jac = ctx.saved_tensors
        tape = tape if tape.numel() else None
        jac = jac if jac.numel() else None
        link = ctx.link
        want_dx = ctx.needs_input_grad[0]
        if link.state is not None:
            state, link.state = link.state, None
            dx, gpre, gpost, gres = K.rewire_bwd_dx(
                x, d, M, hpre, hpost, state, want_dx=want_dx,
                raw=(pre, post, res, tape, jac, ctx.iters, ctx.eps))
            return dx, gpre, gpost, gres, None, None, None
        dx = None
        if d is not None:
            dx, dpre_x = K.prescale_bwd(x, d, hpre)
            dhpre = dpre_x if dhpre is None else dhpre + dpre_x
        if dhpre is None and dhpost is None and dM is None:
            return dx, None, None, None, None, None, None
        z = pre.new_zeros
        gpre, gpost, gres = K.params_bwd(
            pre, post, res, tape, ctx.iters, ctx.eps,
            dhpre if dhpre is not None else z(pre.shape),
            dhpost if dhpost is not None else z(post.shape),
            dM if dM is not None else z(res.shape))
        return dx, gpre, gpost, gres, None, None, None


def _engine_will_run(node) -> bool:
    """Whether the autograd engine runs `node` in the backward pass now in
    progress (torch's own multi-grad hooks ask the same question)."""
    if node is None:
        return False
    try:
        return bool(torch._C._will_engine_execute_node(node))
    except RuntimeError:
        return False


class _RewireCombineFn(torch.autograd.Function):
    """out = H_post (y_inner + M (H_pre x))  (reference layer.py:302-337).

    Inside MHCRewire (link and the pre-scale's autograd node given), the
    backward is split around the inner module's backward when the engine will
    also run the pre-scale's backward: here only dy = H_post * d_out and the
    partial sums of R = sum d_out * y are computed, and the pre-scale's
    backward then writes dx = H_pre (M^T (H_post d_out) + d_xpre) once and
    reduces dM, dH_pre (both branches) and dH_post in one finalize.
    Otherwise (post_combine on its own, or a backward that does not reach the
    pre-scale) this backward returns every gradient itself."""

    @staticmethod
    def forward(ctx, x, y, M, hpre, hpost, out_dtype=torch.float32, link=None, node=None):
        ctx.save_for_backward(x, y, M, hpre, hpost)
        ctx.link, ctx.node = link, node
        return K.rewire_fwd(x, y, M, hpre, hpost, out_dtype)

    @staticmethod
    def backward(ctx, dout):
        x, y, M, hpre, hpost = ctx.saved_tensors
        if ctx.link is not None and _engine_will_run(ctx.node):
            dy, state = K.rewire_bwd_dy(y, dout, hpost)
            ctx.link.state = state
            return None, dy, None, None, None, None, None, None
        dx, dy, dM, dpre, dpost = K.rewire_bwd(x, y, dout, M, hpre, hpost)
        return dx, dy, dM, dpre, dpost, None, None, None


# --------------------------------------------------------------- modules --
class MHCLayer(nn.Module):
    """Manifold-constrained hyper-connection layer over x of shape [B, n, C]."""

    def __init__(
        self,
        n: int,
        C: int,
        sinkhorn_iters: int = 20,
        eps: float = 1e-5,
        use_metal: bool = True,
        threads_per_group: int | None = 256,
        identity_init: bool = True,
        auto_dispatch: bool = True,
        compile_reference: bool | None = None,
        dispatch_policy: str = "auto",
        hybrid_latency: bool = False,
        hybrid_min_C: int = 8192,
        latency_avoid_fused_n32_max_C: int = 2048,
        latency_avoid_fused_B1_min_n: int = 16,
        throughput_allow_fused_n32_min_B: int = 8,
        throughput_allow_fused_n32_min_C: int = 4096,
        throughput_allow_fused_n32_small_C: int = 512,
        fused_backward: bool = False,
        mix_kernel: str = "auto",
        device=None,
    ):
        super().__init__()
        # argument checks of reference layer.py:83-102
        if n <= 0:
            raise ValueError("n must be positive")
        if C <= 0:
            raise ValueError("C must be positive")
        if dispatch_policy not in {"auto", "throughput", "latency"}:
            raise ValueError("dispatch_policy must be one of: auto, throughput, latency")
        if hybrid_min_C <= 0:
            raise ValueError("hybrid_min_C must be positive")
        if latency_avoid_fused_n32_max_C <= 0:
            raise ValueError("latency_avoid_fused_n32_max_C must be positive")
        if latency_avoid_fused_B1_min_n <= 0:
            raise ValueError("latency_avoid_fused_B1_min_n must be positive")
        if throughput_allow_fused_n32_min_B <= 0:
            raise ValueError("throughput_allow_fused_n32_min_B must be positive")
        if throughput_allow_fused_n32_min_C <= 0:
            raise ValueError("throughput_allow_fused_n32_min_C must be positive")
        if throughput_allow_fused_n32_small_C < 0:
            raise ValueError("throughput_allow_fused_n32_small_C must be >= 0")
        if mix_kernel not in {"auto", "1d", "2d"}:
            raise ValueError("mix_kernel must be one of: auto, 1d, 2d")

        self.n = int(n)
        self.C = int(C)
        self.sinkhorn_iters = int(sinkhorn_iters)
        self.eps = float(eps)
        self.use_metal = bool(use_metal) and os.getenv(_DISABLE_ENV, "0") != "1"
        self.threads_per_group = None if threads_per_group is None else int(threads_per_group)
        self.identity_init = bool(identity_init)
        self.auto_dispatch = bool(auto_dispatch)
        self.compile_reference = bool(compile_reference) if compile_reference is not None else False
        self.dispatch_policy = str(dispatch_policy)
        self.hybrid_latency = bool(hybrid_latency)
        self.hybrid_min_C = int(hybrid_min_C)
        self.latency_avoid_fused_n32_max_C = int(latency_avoid_fused_n32_max_C)
        self.latency_avoid_fused_B1_min_n = int(latency_avoid_fused_B1_min_n)
        self.throughput_allow_fused_n32_min_B = int(throughput_allow_fused_n32_min_B)
        self.throughput_allow_fused_n32_min_C = int(throughput_allow_fused_n32_min_C)
        self.throughput_allow_fused_n32_small_C = int(throughput_allow_fused_n32_small_C)
        self.fused_backward = bool(fused_backward)
        self.mix_kernel = str(mix_kernel)

        # identity-friendly init (reference layer.py:139-153)
        f32 = dict(dtype=torch.float32, device=device)
        if self.identity_init:
            off = 12.0
            pre = torch.full((self.n,), -off, **f32)
            post = torch.full((self.n,), -off, **f32)
            res = torch.full((self.n, self.n), -off, **f32) + torch.eye(self.n, **f32) * off
        else:
            pre = torch.zeros(self.n, **f32)
            post = torch.zeros(self.n, **f32)
            res = torch.zeros(self.n, self.n, **f32)
        self.H_pre_raw = nn.Parameter(pre)
        self.H_post_raw = nn.Parameter(post)
        self.H_res_raw = nn.Parameter(res)
        self.rms_weight = nn.Parameter(torch.ones(self.C, **f32))

    # -- dispatch predicates kept for API compatibility (reference layer.py:175-244).
    # On B200 every shape runs the fused CUDA kernels; these report that.
    def _should_use_metal(self, B: int, n: int, C: int) -> bool:
        if os.getenv(_DISABLE_ENV, "0") == "1" or not self.use_metal:
            return False
        return n <= 64

    def _should_use_reference_fallback(self, B: int, n: int, C: int) -> bool:
        return False

    def _should_use_hybrid(self, B: int, n: int, C: int) -> bool:
        return False

    def _should_use_fused_backward(self, B: int, n: int, C: int) -> bool:
        return True

    def _require_cuda_path(self, B: int, n: int, C: int) -> None:
        if not self._should_use_metal(B, n, C):
            raise RuntimeError(
                "mhc_b200 has only the sm_100a CUDA path: use_metal=False or "
                f"{_DISABLE_ENV}=1 requests a non-CUDA path, which this package does not "
                "provide (no silent fallback)."
            )

    def extra_repr(self) -> str:
        return f"n={self.n}, C={self.C}, sinkhorn_iters={self.sinkhorn_iters}, eps={self.eps}"

    def activations(self):
        """(H_pre_act, H_post_act, M) with autograd to the raw parameters."""
        _validate_n(self.n)
        return _ParamsFn.apply(self.H_pre_raw, self.H_post_raw, self.H_res_raw,
                               self.sinkhorn_iters, self.eps)

    def mixing_matrix(self) -> torch.Tensor:
        """Current mixing matrix M (after Sinkhorn), differentiable."""
        return self.activations()[2]

    def post_combine(self, x_reshaped: torch.Tensor, y_inner_reshaped: torch.Tensor) -> torch.Tensor:
        """H_post * (y_inner + (M * H_pre) @ x), H_pre/H_post folded in-kernel
        (reference layer.py:302-337).  Returns float32 like the reference."""
        if x_reshaped.ndim != 3 or x_reshaped.shape[1] != self.n:
            raise ValueError(f"x must be [B, n={self.n}, C], got shape {tuple(x_reshaped.shape)}")
        if tuple(y_inner_reshaped.shape) != tuple(x_reshaped.shape):
            raise ValueError(
                f"inner output shape {tuple(y_inner_reshaped.shape)} does not match the residual "
                f"shape {tuple(x_reshaped.shape)}")
        B, n, C = x_reshaped.shape
        self._require_cuda_path(B, n, C)
        hpre, hpost, M = self.activations()
        return _RewireCombineFn.apply(x_reshaped, y_inner_reshaped, M, hpre, hpost)

    def forward(self, x_expanded: torch.Tensor, *, return_dtype: torch.dtype | None = None):
        """out: [B, n, C]; float32 unless return_dtype is a half dtype equal to
        x's dtype, in which case the kernel writes that dtype directly
        (reference layer.py:339-435)."""
        if x_expanded.ndim != 3:
            raise ValueError(f"x_expanded must be [B, n, C], got shape {tuple(x_expanded.shape)}")
        B, n, C = x_expanded.shape
        if n != self.n:
            raise ValueError(f"x_expanded n={n} does not match layer n={self.n}")
        if C != self.C:
            raise ValueError(f"x_expanded C={C} does not match layer C={self.C}")
        _validate_n(n)
        self._require_cuda_path(B, n, C)
        out_dtype = torch.float32
        if return_dtype is not None and return_dtype == x_expanded.dtype and return_dtype in _HALF:
            out_dtype = return_dtype
        out = _LayerFn.apply(x_expanded, self.H_pre_raw, self.H_post_raw, self.H_res_raw,
                             self.rms_weight, self.sinkhorn_iters, self.eps, out_dtype,
                             getattr(self, "_grad_binding", None))
        if return_dtype is not None and out.dtype != return_dtype:
            out = out.to(return_dtype)
        return out


class MHCRewire(nn.Module):
    """Wrap any module F whose output has its input's shape:

        y = H_post * (F(H_pre * x) + M * H_pre * x)

    over the last axis split into n streams of C = dims // n channels
    (reference layer.py:438-492)."""

    def __init__(self, inner: nn.Module, dims: int, n: int = 32, output_dtype=None,
                 **mhc_kwargs):
        """output_dtype: None returns float32 as the reference does; "input"
        returns x's dtype (the kernel writes it directly, e.g. bf16 models)."""
        super().__init__()
        self.inner = inner
        self.n = n
        self.dims = dims
        if dims % n != 0:
            raise ValueError(f"dims {dims} must be divisible by n={n}")
        if output_dtype not in (None, "input", torch.float32):
            raise ValueError('output_dtype must be None, torch.float32 or "input"')
        self.output_dtype = output_dtype
        self.mhc = MHCLayer(n=n, C=dims // n, **mhc_kwargs)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dims = x.shape[-1]
        if dims % self.n != 0:
            raise ValueError(f"input last dim {dims} must be divisible by n={self.n}")
        C = dims // self.n
        B = x.numel() // dims if dims else 0
        self.mhc._require_cuda_path(B, self.n, C)
        _validate_n(self.n)
        x3 = x.reshape(-1, self.n, C)
        link = _RewireLink()
        mh = self.mhc
        x_pre3, hpre, hpost, M = _RewireInputFn.apply(
            x3, mh.H_pre_raw, mh.H_post_raw, mh.H_res_raw, mh.sinkhorn_iters, mh.eps, link)
        y_inner = self.inner(x_pre3.reshape(x.shape))
        if tuple(y_inner.shape) != tuple(x.shape):
            raise ValueError(
                f"inner module output shape {tuple(y_inner.shape)} must equal its input shape "
                f"{tuple(x.shape)} (mHC needs a residual-compatible module)")
        odt = torch.float32
        if self.output_dtype == "input" and x.dtype in _HALF:
            odt = x.dtype
        out = _RewireCombineFn.apply(x3, y_inner.reshape(-1, self.n, C), M, hpre, hpost, odt,
                                     link, x_pre3.grad_fn)
        return out.reshape(x.shape)
