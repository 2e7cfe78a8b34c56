"""Generate golden vectors by running the reference's own Python code.

The reference (svdrecbd/mhc-mlx) is pure Python on top of MLX, which cannot be
installed here.  Its source of truth, mhc_mlx/reference.py, and the
reference branches of mhc_mlx/layer.py only use a dozen array primitives
(sum / max / mean over an axis, where, exp, sigmoid, sqrt, einsum, full / eye /
zeros / ones, astype).  This script provides those names through a small
numpy-backed stand-in module registered as ``mlx.core`` (plus a bare
``mlx.nn.Module``), imports the reference files unmodified from
REFERENCE_ROOT, runs them on seeded inputs and writes the inputs and
outputs to ``reference_golden.npz`` next to this file.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py --reference /path/to/mhc-mlx

(or set MHC_REFERENCE_DIR instead of passing --reference).

Inputs mirror the reference tests' shapes (tests/test_correctness.py,
test_stability.py, test_stress.py); MLX's RNG cannot be reproduced, so the
random inputs come from numpy's PCG64 with the seeds listed per case.  The
half-precision cases store the exact fp32 values of bf16 / fp16 numbers, as
MLX's ``astype(float32)`` of a half array would see them.
"""

from __future__ import annotations

import argparse
import os
import importlib
import json
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OUT = HERE / "reference_golden.npz"


# --------------------------------------------------------- mlx stand-in --
def install_mlx_standin() -> None:
    core = types.ModuleType("mlx.core")
    core.array = np.ndarray
    core.Dtype = type
    core.float32 = np.float32
    core.float16 = np.float16
    core.bfloat16 = "bfloat16"  # only compared against, never used to cast here
    core.sum = lambda a, axis=None, keepdims=False: np.sum(a, axis=axis, keepdims=keepdims)
    core.max = lambda a, axis=None, keepdims=False: np.max(a, axis=axis, keepdims=keepdims)
    core.mean = lambda a, axis=None, keepdims=False: np.mean(a, axis=axis, keepdims=keepdims)
    core.where = np.where
    core.exp = np.exp
    core.sigmoid = lambda a: (1.0 / (1.0 + np.exp(-a))).astype(a.dtype)  # logistic function
    core.sqrt = np.sqrt
    core.einsum = np.einsum
    core.full = lambda shape, val, dtype=None: np.full(shape, val, dtype=dtype)
    core.eye = lambda n, dtype=None: np.eye(n, dtype=dtype)
    core.zeros = lambda shape, dtype=None: np.zeros(shape, dtype=dtype)
    core.ones = lambda shape, dtype=None: np.ones(shape, dtype=dtype)
    core.fast = types.SimpleNamespace()  # no metal_kernel: the layer takes its reference branch
    core.compile = lambda f: f

    nn = types.ModuleType("mlx.nn")

    class Module:
        def __init__(self):
            pass

    nn.Module = Module
    mlx = types.ModuleType("mlx")
    mlx.core, mlx.nn = core, nn
    sys.modules.update({"mlx": mlx, "mlx.core": core, "mlx.nn": nn})


def import_reference(root: Path):
    """Import mhc_mlx.reference and mhc_mlx.layer from the checkout without
    running the package __init__ (which imports diagnostics/patching)."""
    pkg = types.ModuleType("mhc_mlx")
    pkg.__path__ = [str(root / "mhc_mlx")]
    sys.modules["mhc_mlx"] = pkg
    ref = importlib.import_module("mhc_mlx.reference")
    layer = importlib.import_module("mhc_mlx.layer")
    return ref, layer


# ----------------------------------------------------------------- inputs --
def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bfloat16 (ties to even), back to fp32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def as_dtype(a: np.ndarray, dtype: str) -> np.ndarray:
    a = np.asarray(a, dtype=np.float32)
    if dtype == "bfloat16":
        return bf16_round(a)
    if dtype == "float16":
        return a.astype(np.float16).astype(np.float32)
    return a


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MHC_REFERENCE_DIR"),
                    required="MHC_REFERENCE_DIR" not in os.environ,
                    help="checkout of svdrecbd/mhc-mlx (default: $MHC_REFERENCE_DIR)")
    args = ap.parse_args(argv)
    root = Path(args.reference)
    install_mlx_standin()
    ref, layer_mod = import_reference(root)

    arrays: dict[str, np.ndarray] = {}
    manifest: list[dict] = []

    def put(case: str, meta: dict, **tensors):
        manifest.append({"case": case, **meta})
        for k, v in tensors.items():
            arrays[f"{case}/{k}"] = np.asarray(v, dtype=np.float32)

    def rng(seed):
        return np.random.Generator(np.random.PCG64(seed))

    # 1. Sinkhorn (tests/test_correctness.py:41-58, test_stress.py:19-31)
    for n, iters, eps, seed in [(4, 20, 1e-5, 0), (16, 10, 1e-5, 0), (8, 20, 1e-3, 123),
                                (8, 20, 1e-6, 123), (32, 20, 1e-5, 5), (64, 20, 1e-5, 6),
                                (4, 0, 1e-5, 7), (3, 7, 1e-5, 8)]:
        H = rng(seed).standard_normal((n, n)).astype(np.float32)
        M = ref.mixing_matrix_from_logits(H, iters=iters, eps=eps)
        put(f"sinkhorn_n{n}_it{iters}_eps{eps:g}", dict(kind="sinkhorn", n=n, iters=iters, eps=eps,
                                                        seed=seed), H=H, M=M)

    # stability: H_res = 100 everywhere, n = 32 (tests/test_stability.py:5-47)
    H = np.full((32, 32), 100.0, dtype=np.float32)
    put("sinkhorn_bomb_n32", dict(kind="sinkhorn", n=32, iters=20, eps=1e-5, seed=-1), H=H,
        M=ref.mixing_matrix_from_logits(H, iters=20, eps=1e-5))

    # identity init logits (layer.py:139-148)
    n = 4
    H = (np.full((n, n), -12.0) + np.eye(n) * 12.0).astype(np.float32)
    put("sinkhorn_identity_n4", dict(kind="sinkhorn", n=4, iters=20, eps=1e-5, seed=-1), H=H,
        M=ref.mixing_matrix_from_logits(H, iters=20, eps=1e-5))

    # 2. full forward, reference.mhc_forward_reference (reference.py:164-184)
    fwd_cases = [
        # (name, B, n, C, dtype, iters, seed)           reference test it mirrors
        ("fused_f32", 2, 4, 128, "float32", 10, 1),     # test_correctness.py:61
        ("fused_f16", 2, 4, 128, "float16", 10, 1),
        ("fused_bf16", 2, 4, 128, "bfloat16", 10, 1),
        ("fused_n16_bf16", 2, 16, 64, "bfloat16", 10, 0),  # :100
        ("large_c_f16", 1, 8, 4096, "float16", 10, 321),   # test_stress.py:36
        ("seed1_bf16", 2, 4, 256, "bfloat16", 10, 1),      # test_stress.py:78
        ("seed7_bf16", 2, 4, 256, "bfloat16", 10, 7),
        ("seed13_bf16", 2, 4, 256, "bfloat16", 10, 13),
        ("odd_c_f32", 3, 4, 129, "float32", 20, 2),
        ("n3_f32", 2, 3, 40, "float32", 20, 3),
        ("bwd_case_f32", 1, 4, 16, "float32", 5, 9),       # test_correctness.py:295
    ]
    for name, B, n, C, dt, iters, seed in fwd_cases:
        g = rng(seed)
        x = as_dtype(g.standard_normal((B, n, C)), dt)
        pre = g.standard_normal(n).astype(np.float32)
        post = g.standard_normal(n).astype(np.float32)
        res = g.standard_normal((n, n)).astype(np.float32)
        w = np.ones(C, dtype=np.float32)
        out = ref.mhc_forward_reference(x, pre, post, res, w, sinkhorn_iters=iters, eps=1e-5)
        hpre, hpost = ref.activate_pre_post(pre, post)
        M = ref.mixing_matrix_from_logits(res, iters=iters, eps=1e-5)
        put(name, dict(kind="forward", B=B, n=n, C=C, dtype=dt, iters=iters, eps=1e-5, seed=seed),
            x=x, H_pre_raw=pre, H_post_raw=post, H_res_raw=res, rms_weight=w, out=out,
            H_pre_act=hpre, H_post_act=hpost, M=M)

    # known-answer (RNG-free) inputs of test_correctness.py:146-179
    B, n, C = 2, 4, 129
    pre = (np.arange(n, dtype=np.float32) * 0.1) - 0.2
    post = (np.arange(n, dtype=np.float32) * 0.07) - 0.1
    res = (np.arange(n * n, dtype=np.float32).reshape(n, n) * 0.01) - 0.05
    w = np.ones(C, dtype=np.float32)
    for dt in ("float16", "bfloat16"):
        x = as_dtype(np.arange(B * n * C, dtype=np.float32).reshape(B, n, C) * 0.001, dt)
        out = ref.mhc_forward_reference(x, pre, post, res, w, sinkhorn_iters=10, eps=1e-5)
        put(f"arange_{dt}", dict(kind="forward", B=B, n=n, C=C, dtype=dt, iters=10, eps=1e-5,
                                 seed=-1), x=x, H_pre_raw=pre, H_post_raw=post, H_res_raw=res,
            rms_weight=w, out=out)

    # identity mapping (test_correctness.py:182-220): out ~= x
    g = rng(123)
    n, C = 4, 64
    x = as_dtype(g.standard_normal((2, n, C)), "bfloat16")
    pre = np.full(n, -12.0, dtype=np.float32)
    post = np.full(n, -12.0, dtype=np.float32)
    res = (np.full((n, n), -12.0) + np.eye(n) * 12.0).astype(np.float32)
    w = np.ones(C, dtype=np.float32)
    put("identity_bf16", dict(kind="forward", B=2, n=n, C=C, dtype="bfloat16", iters=20, eps=1e-5,
                              seed=123), x=x, H_pre_raw=pre, H_post_raw=post, H_res_raw=res,
        rms_weight=w, out=ref.mhc_forward_reference(x, pre, post, res, w, 20, 1e-5))

    # 3. MHCLayer.__call__ reference branch (layer.py:339-435), test_correctness.py:224-292
    for B, n, C, seed in [(1, 4, 64, 104), (2, 8, 128, 108), (2, 16, 256, 116), (1, 32, 256, 132),
                          (1, 32, 1024, 7)]:
        g = rng(seed)
        x = as_dtype(g.standard_normal((B, n, C)), "bfloat16")
        L = layer_mod.MHCLayer(n=n, C=C, use_metal=False, compile_reference=False)
        L.H_pre_raw = g.standard_normal(n).astype(np.float32)
        L.H_post_raw = g.standard_normal(n).astype(np.float32)
        L.H_res_raw = g.standard_normal((n, n)).astype(np.float32)
        L.rms_weight = (1.0 + 0.1 * g.standard_normal(C)).astype(np.float32)
        out = L(x)
        put(f"layer_{B}x{n}x{C}", dict(kind="layer", B=B, n=n, C=C, dtype="bfloat16", iters=20,
                                       eps=1e-5, seed=seed), x=x, H_pre_raw=L.H_pre_raw,
            H_post_raw=L.H_post_raw, H_res_raw=L.H_res_raw, rms_weight=L.rms_weight, out=out)

    # identity-initialised layer parameters (layer.py:139-153)
    L = layer_mod.MHCLayer(n=4, C=8, use_metal=False, compile_reference=False)
    put("layer_init_identity", dict(kind="init", n=4, C=8), H_pre_raw=L.H_pre_raw,
        H_post_raw=L.H_post_raw, H_res_raw=L.H_res_raw, rms_weight=L.rms_weight)

    # 4. MHCRewire around a linear inner module (layer.py:438-492)
    class NpLinear:
        def __init__(self, W, b):
            self.W, self.b = W, b

        def __call__(self, v):
            return (v @ self.W.T + self.b).astype(np.float32)

    for dims, n, rows, seed in [(256, 16, 1, 42), (64, 4, 3, 0), (128, 32, 2, 11)]:
        g = rng(seed)
        bound = 1.0 / np.sqrt(dims)
        W = g.uniform(-bound, bound, (dims, dims)).astype(np.float32)
        b = g.uniform(-bound, bound, dims).astype(np.float32)
        R = layer_mod.MHCRewire(NpLinear(W, b), dims=dims, n=n, use_metal=False,
                                compile_reference=False)
        R.mhc.H_pre_raw = (0.5 * g.standard_normal(n)).astype(np.float32)
        R.mhc.H_post_raw = (0.5 * g.standard_normal(n)).astype(np.float32)
        R.mhc.H_res_raw = g.standard_normal((n, n)).astype(np.float32)
        x = g.standard_normal((rows, dims)).astype(np.float32)
        out = R(x)
        put(f"rewire_{dims}_n{n}", dict(kind="rewire", dims=dims, n=n, rows=rows, iters=20,
                                        eps=1e-5, seed=seed), x=x, W=W, b=b,
            H_pre_raw=R.mhc.H_pre_raw, H_post_raw=R.mhc.H_post_raw, H_res_raw=R.mhc.H_res_raw,
            out=out)

    np.savez_compressed(OUT, **arrays)
    (HERE / "reference_golden.json").write_text(json.dumps(
        {"source": "svdrecbd/mhc-mlx mhc_mlx/reference.py + mhc_mlx/layer.py (reference branch), "
                   "run through a numpy stand-in for mlx.core",
         "numpy": np.__version__, "cases": manifest}, indent=1))
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(manifest)} cases)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
