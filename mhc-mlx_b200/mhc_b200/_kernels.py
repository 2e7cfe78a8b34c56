"""Tensor-level wrappers over the C ABI.

Each function takes CUDA tensors, allocates outputs and workspaces through
torch's caching allocator, and enqueues one or two kernels on the current
stream.  Shapes are assumed validated by the caller (metal.py / layer.py);
only contiguity, dtype and device are normalised here.
"""

from __future__ import annotations

import contextlib
import functools

import torch

from . import _capi as C

F32 = torch.float32

# Optional per-launch timing: when set to a dict, each timed C-ABI launch
# appends a (start, end) pair of CUDA events recorded on the launching
# stream under the entry point's name.  Off (None) in normal use.
TIMING: dict | None = None


@contextlib.contextmanager
def _timed(name: str, ref: torch.Tensor):
    if TIMING is None:
        yield
        return
    st = torch.cuda.current_stream(ref.device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    yield
    b.record(st)
    TIMING.setdefault(name, []).append((a, b))


def _call(name: str, ref: torch.Tensor, *args) -> None:
    """C.call with optional per-launch event timing (see TIMING)."""
    with _timed(name, ref):
        C.call(name, *args)


def _c(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


def _f32(t: torch.Tensor) -> torch.Tensor:
    return _c(t if t.dtype == F32 else t.float())


def _io(t: torch.Tensor) -> torch.Tensor:
    """Activation tensors stay in fp32/fp16/bf16; anything else becomes fp32."""
    if t.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        t = t.float()
    return _c(t)


_NULL = contextlib.nullcontext()


def _on(dev: torch.device):
    """Make `dev` current around a C-ABI call (kernels launch on the current
    device); a no-op context when it already is."""
    if dev.index is None or dev.index == torch.cuda.current_device():
        return _NULL
    return torch.cuda.device(dev)


def _ws(nbytes: int, dev: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=dev)


# ------------------------------------------------------------ parameters --
@functools.lru_cache(maxsize=256)
def tape_floats(n: int, iters: int) -> int:
    return int(C.query("mhc_sinkhorn_tape_floats", n, iters))


@functools.lru_cache(maxsize=4096)
def _ws_query(name: str, device_index: int, *args) -> int:
    """Workspace sizes depend on the shape and on the device's SM count (the
    current device, made current by the caller), hence the device key."""
    return int(C.query(name, *args))


def _ws_bytes(name: str, dev: torch.device, *args) -> int:
    return _ws_query(name, dev.index if dev.index is not None else -1, *args)


def params_fwd(H_pre_raw, H_post_raw, H_res_raw, iters: int, eps: float, want_tape: bool):
    """(H_pre_act, H_post_act, M, tape); any raw input may be None."""
    ref = next(t for t in (H_res_raw, H_pre_raw, H_post_raw) if t is not None)
    dev = C.require_cuda(H_pre_raw, H_post_raw, H_res_raw)
    n = ref.shape[0]
    with _on(dev):
        pre = _f32(H_pre_raw) if H_pre_raw is not None else None
        post = _f32(H_post_raw) if H_post_raw is not None else None
        res = _f32(H_res_raw) if H_res_raw is not None else None
        hpre = torch.empty(n, dtype=F32, device=dev) if pre is not None else None
        hpost = torch.empty(n, dtype=F32, device=dev) if post is not None else None
        M = torch.empty(n, n, dtype=F32, device=dev) if res is not None else None
        tape = None
        if want_tape and res is not None and iters > 0:
            tape = torch.empty(tape_floats(n, iters), dtype=F32, device=dev)
        _call("mhc_params_fwd", ref, C.ptr(pre), C.ptr(post), C.ptr(res), n, int(iters),
              float(eps), C.ptr(hpre), C.ptr(hpost), C.ptr(M), C.ptr(tape), C.stream_of(ref))
    return hpre, hpost, M, tape


def params_bwd(H_pre_raw, H_post_raw, H_res_raw, tape, iters: int, eps: float, dhpre, dhpost, dM):
    """Gradients w.r.t. the raw parameters (None where the input was None)."""
    ref = next(t for t in (H_res_raw, H_pre_raw, H_post_raw) if t is not None)
    dev = C.require_cuda(H_pre_raw, H_post_raw, H_res_raw)
    n = ref.shape[0]
    with _on(dev):
        pre = _f32(H_pre_raw) if (H_pre_raw is not None and dhpre is not None) else None
        post = _f32(H_post_raw) if (H_post_raw is not None and dhpost is not None) else None
        res = _f32(H_res_raw) if (H_res_raw is not None and dM is not None) else None
        gpre = torch.empty(n, dtype=F32, device=dev) if pre is not None else None
        gpost = torch.empty(n, dtype=F32, device=dev) if post is not None else None
        gres = torch.empty(n, n, dtype=F32, device=dev) if res is not None else None
        _call("mhc_params_bwd", ref, C.ptr(pre), C.ptr(post), C.ptr(res), C.ptr(tape), n, int(iters),
               float(eps), C.ptr(_f32(dhpre) if pre is not None else None),
               C.ptr(_f32(dhpost) if post is not None else None),
               C.ptr(_f32(dM) if res is not None else None), C.ptr(gpre), C.ptr(gpost),
               C.ptr(gres), C.stream_of(ref))
    return gpre, gpost, gres


def sinkhorn_batched_fwd(H: torch.Tensor, iters: int, eps: float) -> torch.Tensor:
    dev = C.require_cuda(H)
    B, n, _ = H.shape
    with _on(dev):
        Hc = _f32(H)
        M = torch.empty(B, n, n, dtype=F32, device=dev)
        _call("mhc_sinkhorn_batched_fwd", Hc, C.ptr(Hc), B, n, int(iters), float(eps), C.ptr(M),
               C.stream_of(Hc))
    return M


def sinkhorn_batched_bwd(H: torch.Tensor, dM: torch.Tensor, iters: int, eps: float) -> torch.Tensor:
    dev = C.require_cuda(H, dM)
    B, n, _ = H.shape
    with _on(dev):
        Hc, dMc = _f32(H), _f32(dM)
        dH = torch.empty(B, n, n, dtype=F32, device=dev)
        nb = _ws_bytes("mhc_sinkhorn_batched_workspace_bytes", dev, B, n, int(iters))
        ws = _ws(nb, dev) if nb else None
        _call("mhc_sinkhorn_batched_bwd", Hc, C.ptr(Hc), C.ptr(dMc), B, n, int(iters), float(eps),
               C.ptr(dH), C.ptr(ws), nb, C.stream_of(Hc))
    return dH


# ------------------------------------------------------------------ layer --
def layer_fwd(x, M, hpre, hpost, w, eps: float, out_dtype: torch.dtype) -> torch.Tensor:
    dev = C.require_cuda(x, M, hpre, hpost, w)
    T, n, Cc = x.shape
    with _on(dev):
        xc = _io(x)
        out = torch.empty(T, n, Cc, dtype=out_dtype, device=dev)
        args = (C.ptr(xc), C.dtype_code(xc.dtype), C.ptr(_f32(M)), C.ptr(_f32(hpre)),
                C.ptr(_f32(hpost)), C.ptr(_f32(w)), C.ptr(out), C.dtype_code(out_dtype), T, n, Cc,
                float(eps), C.stream_of(xc))
        _call("mhc_fwd", xc, *args)
    return out


def layer_bwd(x, dout, M, hpre, hpost, w, eps: float, raw=None, out=None):
    """dx plus either (dM, dH_pre_act, dH_post_act, d_w) or, with
    raw = (H_pre_raw, H_post_raw, H_res_raw, tape, iters), the raw-parameter
    gradients (dH_pre_raw, dH_post_raw, dH_res_raw, d_w) from the same
    finalize launch.  With raw, `out` may give the four fp32 destination
    tensors (e.g. views of a flat gradient bucket) that the finalize writes."""
    dev = C.require_cuda(x, dout, M, hpre, hpost, w)
    T, n, Cc = x.shape
    with _on(dev):
        xc = _io(x)
        dc = _c(dout) if dout.dtype in (F32, xc.dtype) else dout.float().contiguous()
        dx = torch.empty(T, n, Cc, dtype=xc.dtype, device=dev)
        nb = _ws_bytes("mhc_bwd_workspace_bytes", dev, T, n, Cc)
        ws = _ws(nb, dev)
        st = C.stream_of(xc)
        args = (C.ptr(xc), C.dtype_code(xc.dtype), C.ptr(dc), C.dtype_code(dc.dtype),
                C.ptr(_f32(M)), C.ptr(_f32(hpre)), C.ptr(_f32(hpost)), C.ptr(_f32(w)), C.ptr(dx),
                C.dtype_code(dx.dtype), T, n, Cc, float(eps), C.ptr(ws), nb, st)
        _call("mhc_bwd", xc, *args)
        dw = torch.empty(Cc, dtype=F32, device=dev)
        if raw is None:
            dM = torch.empty(n, n, dtype=F32, device=dev)
            dpre = torch.empty(n, dtype=F32, device=dev)
            dpost = torch.empty(n, dtype=F32, device=dev)
            _call("mhc_bwd_finalize", xc, C.ptr(ws), n, Cc, C.ptr(dM), C.ptr(dpre), C.ptr(dpost),
                   C.ptr(dw), None, None, None, None, 0, float(eps), None, None, None, st)
            return dx, dM, dpre, dpost, dw
        pre_raw, post_raw, res_raw, tape, iters = raw
        if out is not None:
            gpre, gpost, gres, dw = out
        else:
            gpre = torch.empty(n, dtype=F32, device=dev)
            gpost = torch.empty(n, dtype=F32, device=dev)
            gres = torch.empty(n, n, dtype=F32, device=dev)
        args = (C.ptr(ws), n, Cc, None, None, None, C.ptr(dw), C.ptr(_f32(pre_raw)),
                C.ptr(_f32(post_raw)), C.ptr(_f32(res_raw)), C.ptr(tape), int(iters), float(eps),
                C.ptr(gpre), C.ptr(gpost), C.ptr(gres), st)
        _call("mhc_bwd_finalize", xc, *args)
        return dx, gpre, gpost, gres, dw


# -------------------------------------------------------------------- mix --
def mix_add_fwd(x, M, y, out_dtype=F32) -> torch.Tensor:
    dev = C.require_cuda(x, M, y)
    T, n, Cc = x.shape
    with _on(dev):
        xc = _io(x)
        yc = _c(y) if y.dtype in (F32, xc.dtype) else y.float().contiguous()
        out = torch.empty(T, n, Cc, dtype=out_dtype, device=dev)
        _call("mhc_mix_add_fwd", xc, C.ptr(xc), C.dtype_code(xc.dtype), C.ptr(_f32(M)), C.ptr(yc),
               C.dtype_code(yc.dtype), C.ptr(out), C.dtype_code(out_dtype), T, n, Cc,
               C.stream_of(xc))
    return out


def mix_add_bwd(x, M, dout):
    dev = C.require_cuda(x, M, dout)
    T, n, Cc = x.shape
    with _on(dev):
        xc = _io(x)
        dc = _c(dout) if dout.dtype in (F32, xc.dtype) else dout.float().contiguous()
        dx = torch.empty(T, n, Cc, dtype=xc.dtype, device=dev)
        dM = torch.empty(n, n, dtype=F32, device=dev)
        nb = _ws_bytes("mhc_mix_bwd_workspace_bytes", dev, T, n, Cc)
        ws = _ws(nb, dev)
        _call("mhc_mix_add_bwd", xc, C.ptr(xc), C.dtype_code(xc.dtype), C.ptr(_f32(M)), C.ptr(dc),
               C.dtype_code(dc.dtype), C.ptr(dx), C.dtype_code(dx.dtype), C.ptr(dM), T, n, Cc,
               C.ptr(ws), nb, C.stream_of(xc))
    return dx, dM


def rewire_fwd(x, y, M, hpre, hpost, out_dtype=F32) -> torch.Tensor:
    dev = C.require_cuda(x, y, M, hpre, hpost)
    T, n, Cc = x.shape
    with _on(dev):
        xc = _io(x)
        yc = _c(y) if y.dtype in (F32, xc.dtype) else y.float().contiguous()
        out = torch.empty(T, n, Cc, dtype=out_dtype, device=dev)
        _call("mhc_rewire_combine_fwd", xc, C.ptr(xc), C.dtype_code(xc.dtype), C.ptr(yc),
               C.dtype_code(yc.dtype), C.ptr(_f32(M)), C.ptr(_f32(hpre)), C.ptr(_f32(hpost)),
               C.ptr(out), C.dtype_code(out_dtype), T, n, Cc, C.stream_of(xc))
    return out


def rewire_bwd(x, y, dout, M, hpre, hpost):
    dev = C.require_cuda(x, y, dout, M, hpre, hpost)
    T, n, Cc = x.shape
    with _on(dev):
        xc = _io(x)
        yc = _c(y) if y.dtype in (F32, xc.dtype) else y.float().contiguous()
        dc = _c(dout) if dout.dtype in (F32, xc.dtype) else dout.float().contiguous()
        dx = torch.empty(T, n, Cc, dtype=xc.dtype, device=dev)
        dy = torch.empty(T, n, Cc, dtype=yc.dtype, device=dev)
        dM = torch.empty(n, n, dtype=F32, device=dev)
        dpre = torch.empty(n, dtype=F32, device=dev)
        dpost = torch.empty(n, dtype=F32, device=dev)
        nb = _ws_bytes("mhc_rewire_bwd_workspace_bytes", dev, T, n, Cc)
        ws = _ws(nb, dev)
        _call("mhc_rewire_combine_bwd", xc, C.ptr(xc), C.dtype_code(xc.dtype), C.ptr(yc),
               C.dtype_code(yc.dtype), C.ptr(dc), C.dtype_code(dc.dtype), C.ptr(_f32(M)),
               C.ptr(_f32(hpre)), C.ptr(_f32(hpost)), C.ptr(dx), C.dtype_code(dx.dtype), C.ptr(dy),
               C.dtype_code(dy.dtype), C.ptr(dM), C.ptr(dpre), C.ptr(dpost), T, n, Cc, C.ptr(ws),
               nb, C.stream_of(xc))
    return dx, dy, dM, dpre, dpost


def rewire_bwd_dy(y, dout, hpost):
    """First half of MHCRewire's end-to-end backward (before the inner
    module's backward): dy = H_post * d_out and the partial sums of
    R = sum d_out * y, in a workspace that rewire_bwd_dx completes."""
    dev = C.require_cuda(y, dout, hpost)
    T, n, Cc = y.shape
    with _on(dev):
        yc = _io(y)
        dc = _c(dout) if dout.dtype in (F32, yc.dtype) else dout.float().contiguous()
        dy = torch.empty(T, n, Cc, dtype=yc.dtype, device=dev)
        nb = _ws_bytes("mhc_rewire_fused_bwd_workspace_bytes", dev, T, n, Cc)
        ws = _ws(nb, dev)
        _call("mhc_rewire_bwd_dy", yc, C.ptr(yc), C.dtype_code(yc.dtype), C.ptr(dc),
              C.dtype_code(dc.dtype), C.ptr(_f32(hpost)), C.ptr(dy), C.dtype_code(dy.dtype), T, n,
              Cc, C.ptr(ws), nb, C.stream_of(yc))
    return dy, (ws, nb, dc)


def rewire_bwd_dx(x, d_xpre, M, hpre, hpost, state, want_dx: bool = True, raw=None):
    """Second half (after the inner module's backward gave d_xpre, or None):
    dx written once, and dM, dH_pre_act (both branches), dH_post_act from one
    reduction.  `state` is what rewire_bwd_dy returned.

    raw = (H_pre_raw, H_post_raw, H_res_raw, tape, jacobian, iters, eps), as
    rewire_in_fwd returned them: the same launch carries on to the raw
    gradients, and (dx, dH_pre_raw, dH_post_raw, dH_res_raw) is returned
    instead of (dx, dM, dH_pre_act, dH_post_act)."""
    ws, nb, dc = state
    dev = C.require_cuda(x, d_xpre, M, hpre, hpost)
    T, n, Cc = x.shape
    with _on(dev):
        xc = _io(x)
        pc = None
        if d_xpre is not None:
            pc = _c(d_xpre) if d_xpre.dtype in (F32, xc.dtype) else d_xpre.float().contiguous()
        dx = torch.empty(T, n, Cc, dtype=xc.dtype, device=dev) if want_dx else None
        nn = n * n
        # one buffer for the activation gradients [dM | dpre | dpost] and one
        # for the raw gradients [dres | dpre_raw | dpost_raw]
        act = torch.empty(nn + 2 * n, dtype=F32, device=dev)
        dM, dpre, dpost = act[:nn].view(n, n), act[nn:nn + n], act[nn + n:]
        rargs = (None,) * 5 + (0, 0.0) + (None,) * 3
        if raw is not None:
            pre, post, res, tape, jac, iters, eps = raw
            g = torch.empty(nn + 2 * n, dtype=F32, device=dev)
            gres, gpre, gpost = g[:nn].view(n, n), g[nn:nn + n], g[nn + n:]
            rargs = (C.ptr(pre), C.ptr(post), C.ptr(res), C.ptr(tape), C.ptr(jac), int(iters),
                     float(eps), C.ptr(gpre), C.ptr(gpost), C.ptr(gres))
        _call("mhc_rewire_bwd_dx", xc, C.ptr(xc), C.dtype_code(xc.dtype), C.ptr(dc),
              C.dtype_code(dc.dtype), C.ptr(pc), C.dtype_code(pc.dtype if pc is not None else F32),
              C.ptr(_f32(M)), C.ptr(_f32(hpre)), C.ptr(_f32(hpost)), C.ptr(dx),
              C.dtype_code(xc.dtype), C.ptr(dM), C.ptr(dpre), C.ptr(dpost), *rargs, T, n, Cc,
              C.ptr(ws), nb, C.stream_of(xc))
    if raw is not None:
        return dx, gpre, gpost, gres
    return dx, dM, dpre, dpost


@functools.lru_cache(maxsize=64)
def jacobian_floats(n: int) -> int:
    return int(C.query("mhc_rewire_jacobian_floats", n))


def rewire_in_fwd(x, H_pre_raw, H_post_raw, H_res_raw, iters: int, eps: float, out_dtype=None):
    """MHCRewire's input side in one launch for n <= 8: the activations, M,
    the Sinkhorn tape and (n <= 4) the Jacobian of M, and x_pre = x * H_pre_act.
    Returns (x_pre, hpre, hpost, M, raw) with raw the tuple rewire_bwd_dx takes."""
    dev = C.require_cuda(x, H_pre_raw, H_post_raw, H_res_raw)
    T, n, Cc = x.shape
    with _on(dev):
        xc = _io(x)
        odt = out_dtype or xc.dtype
        pre, post, res = _f32(H_pre_raw), _f32(H_post_raw), _f32(H_res_raw)
        nn, tf, jf = n * n, tape_floats(n, iters), jacobian_floats(n)
        # one buffer: [M | hpre | hpost | tape | jacobian]
        buf = torch.empty(nn + 2 * n + tf + jf, dtype=F32, device=dev)
        M, hpre, hpost = buf[:nn].view(n, n), buf[nn:nn + n], buf[nn + n:nn + 2 * n]
        o = nn + 2 * n
        tape = buf[o:o + tf] if tf else None
        jac = buf[o + tf:o + tf + jf] if jf else None
        out = torch.empty(T, n, Cc, dtype=odt, device=dev)
        _call("mhc_rewire_in_fwd", xc, C.ptr(xc), C.dtype_code(xc.dtype), C.ptr(pre), C.ptr(post),
              C.ptr(res), int(iters), float(eps), C.ptr(hpre), C.ptr(hpost), C.ptr(M),
              C.ptr(tape), C.ptr(jac), C.ptr(out), C.dtype_code(odt), T, n, Cc, C.stream_of(xc))
    return out, hpre, hpost, M, (pre, post, res, tape, jac, int(iters), float(eps))


def prescale_fwd(x, hpre, out_dtype=None) -> torch.Tensor:
    dev = C.require_cuda(x, hpre)
    T, n, Cc = x.shape
    with _on(dev):
        xc = _io(x)
        odt = out_dtype or xc.dtype
        out = torch.empty(T, n, Cc, dtype=odt, device=dev)
        _call("mhc_prescale_fwd", xc, C.ptr(xc), C.dtype_code(xc.dtype), C.ptr(_f32(hpre)), C.ptr(out),
               C.dtype_code(odt), T, n, Cc, C.stream_of(xc))
    return out


def prescale_bwd(x, d, hpre):
    dev = C.require_cuda(x, d, hpre)
    T, n, Cc = x.shape
    with _on(dev):
        xc = _io(x)
        dc = _c(d) if d.dtype in (F32, xc.dtype) else d.float().contiguous()
        dx = torch.empty(T, n, Cc, dtype=xc.dtype, device=dev)
        dpre = torch.empty(n, dtype=F32, device=dev)
        nb = _ws_bytes("mhc_mix_bwd_workspace_bytes", dev, T, n, Cc)
        ws = _ws(nb, dev)
        _call("mhc_prescale_bwd", xc, C.ptr(xc), C.dtype_code(xc.dtype), C.ptr(dc),
               C.dtype_code(dc.dtype), C.ptr(_f32(hpre)), C.ptr(dx), C.dtype_code(dx.dtype),
               C.ptr(dpre), T, n, Cc, C.ptr(ws), nb, C.stream_of(xc))
    return dx, dpre


def residual_add_agg(x, res, hpre, out_dtype=F32):
    dev = C.require_cuda(x, res, hpre)
    T, n, Cc = x.shape
    with _on(dev):
        xc = _io(x)
        rc = _c(res.to(xc.dtype))
        out = torch.empty(T, n, Cc, dtype=out_dtype, device=dev)
        yagg = torch.empty(T, Cc, dtype=F32, device=dev)
        _call("mhc_residual_add_agg", xc, C.ptr(xc), C.dtype_code(xc.dtype), C.ptr(rc),
               C.dtype_code(rc.dtype), C.ptr(_f32(hpre)), C.ptr(out), C.dtype_code(out_dtype),
               C.ptr(yagg), T, n, Cc, C.stream_of(xc))
    return out, yagg


def residual_add_agg_bwd(out, d_out, d_y, hpre, dx_dtype):
    """(dx, dH_pre) for out = x + res, y_agg = sum_i hpre_i out_i; d_out or d_y may be None."""
    dev = C.require_cuda(out, d_out, d_y, hpre)
    T, n, Cc = out.shape
    with _on(dev):
        oc = _c(out)
        dc = None if d_out is None else _c(d_out.to(oc.dtype))
        yc = None if d_y is None else _f32(d_y)
        dx = torch.empty(T, n, Cc, dtype=dx_dtype, device=dev)
        dpre = torch.empty(n, dtype=F32, device=dev)
        nb = _ws_bytes("mhc_mix_bwd_workspace_bytes", dev, T, n, Cc)
        ws = _ws(nb, dev)
        _call("mhc_residual_add_agg_bwd", oc, C.ptr(oc), C.dtype_code(oc.dtype), C.ptr(dc),
              C.dtype_code(oc.dtype), C.ptr(yc), C.ptr(_f32(hpre)), C.ptr(dx),
              C.dtype_code(dx_dtype), C.ptr(dpre), T, n, Cc, C.ptr(ws), nb, C.stream_of(oc))
    return dx, dpre


# ------------------------------------------------------- quantized linear --
def qlinear_fwd(x2, w_packed, scales, biases, bias, group_size: int, bits: int):
    """y[M, N] = x2[M, K] W^T (+ bias) with the 4-bit weight dequantised inside
    the GEMM (mhc_qlinear_fwd)."""
    dev = C.require_cuda(x2, w_packed, scales, biases, bias)
    M, Kd = x2.shape
    N = w_packed.shape[0]
    with _on(dev):
        xc = _c(x2)
        b = None if bias is None else _c(bias.to(xc.dtype))
        y = torch.empty(M, N, dtype=xc.dtype, device=dev)
        _call("mhc_qlinear_fwd", xc, C.ptr(xc), C.dtype_code(xc.dtype), C.ptr(_c(w_packed)),
              C.ptr(_c(scales)), C.ptr(_c(biases)), C.dtype_code(scales.dtype), C.ptr(b),
              C.ptr(y), M, N, Kd, int(group_size), int(bits), C.stream_of(xc))
    return y


def qlinear_bwd_dx(dy2, w_packed, scales, biases, in_dims: int, group_size: int, bits: int):
    """dx[M, K] = dy2[M, N] W with the weight dequantised inside the GEMM
    (mhc_qlinear_bwd_dx)."""
    dev = C.require_cuda(dy2, w_packed, scales, biases)
    M, N = dy2.shape
    with _on(dev):
        dc = _c(dy2)
        dx = torch.empty(M, in_dims, dtype=dc.dtype, device=dev)
        _call("mhc_qlinear_bwd_dx", dc, C.ptr(dc), C.dtype_code(dc.dtype), C.ptr(_c(w_packed)),
              C.ptr(_c(scales)), C.ptr(_c(biases)), C.dtype_code(scales.dtype), C.ptr(dx), M, N,
              in_dims, int(group_size), int(bits), C.stream_of(dc))
    return dx


def qlinear_bwd_dx_t(dy2, wt_packed, scales_t, biases_t, in_dims: int, group_size: int,
                     bits: int):
    """dx[M, K] = dy2[M, N] W from the transposed layouts of the weight (codes
    of W^T, scales / biases [K/64][N] in dy's dtype): mhc_qlinear_bwd_dx_t."""
    dev = C.require_cuda(dy2, wt_packed, scales_t, biases_t)
    M, N = dy2.shape
    with _on(dev):
        dc = _c(dy2)
        dx = torch.empty(M, in_dims, dtype=dc.dtype, device=dev)
        _call("mhc_qlinear_bwd_dx_t", dc, C.ptr(dc), C.dtype_code(dc.dtype), C.ptr(_c(wt_packed)),
              C.ptr(_c(scales_t)), C.ptr(_c(biases_t)), C.ptr(dx), M, N, in_dims,
              int(group_size), int(bits), C.stream_of(dc))
    return dx


def qlinear_transpose_pack(w_packed, in_dims: int):
    """Codes of W^T packed eight per word ([in, out/8] int32) from the layer's
    [out, in/8] words, on the device (mhc_qlinear_transpose_pack)."""
    dev = C.require_cuda(w_packed)
    N = w_packed.shape[0]
    with _on(dev):
        wc = _c(w_packed)
        wt = torch.empty(in_dims, N // 8, dtype=torch.int32, device=dev)
        _call("mhc_qlinear_transpose_pack", wc, C.ptr(wc), C.ptr(wt), N, in_dims, C.stream_of(wc))
    return wt
