"""CPU tests of the host side: the C-ABI library loads and exports every
symbol include/mhc_b200.h declares (no compute), the reference-compatible
validation errors, module construction, AutoPatcher, QuantizedLinear,
pickling and determinism of initialisation (reference tests/test_rewire.py,
test_patching.py, test_determinism.py, test_packaging.py)."""

from __future__ import annotations

import io
import pickle
import re
from pathlib import Path

import pytest
import torch
from torch import nn

import mhc_b200
from mhc_b200 import AutoPatcher, MHCLayer, MHCRewire, QuantizedLinear, _capi, metal

HEADER = Path(__file__).resolve().parent.parent / "include" / "mhc_b200.h"


def header_symbols() -> list[str]:
    return re.findall(r"^MHC_API\s+[\w\s\*]+?\b(mhc_\w+)\s*\(", HEADER.read_text(), flags=re.M)


def test_library_exports_every_header_symbol():
    declared = header_symbols()
    assert len(declared) >= 20
    lib = _capi.load()
    for name in declared:
        assert hasattr(lib, name), name
    assert sorted(declared) == sorted(_capi.SIGNATURES), "ctypes table out of sync with header"
    assert _capi.query("mhc_version") >= 10000


def test_library_error_reporting_without_gpu():
    # argument validation runs before any CUDA call
    with pytest.raises(ValueError, match="n=65"):
        _capi.call("mhc_fwd", None, 0, None, None, None, None, None, 0, 1, 65, 16, 1e-5, None)
    with pytest.raises(ValueError, match="dtype"):
        _capi.call("mhc_fwd", None, 7, None, None, None, None, None, 0, 1, 4, 16, 1e-5, None)
    assert _capi.query("mhc_sinkhorn_tape_floats", 4, 20) == 20 * (16 + 8)
    assert _capi.query("mhc_sinkhorn_tape_floats", 65, 20) == 0


def test_package_alias_and_version():
    assert mhc_b200.__version__
    assert {"MHCLayer", "MHCRewire", "AutoPatcher", "residual_add_agg"} <= set(mhc_b200.__all__)


def test_suggest_threads_per_group():
    assert metal.suggest_threads_per_group(129) == 256
    assert metal.suggest_threads_per_group(4096) == 1024
    assert metal.suggest_threads_per_group(100, max_tpg=64) == 64
    with pytest.raises(ValueError):
        metal.suggest_threads_per_group(0)


def test_mix_add_rms_threadgroup_size_matches_reference_rules():
    assert metal.mix_add_rms_threadgroup_size(4, None, 256) == 256
    assert metal.mix_add_rms_threadgroup_size(32, None, 256) == 32 * 32
    assert metal.mix_add_rms_threadgroup_size(16, torch.float32, 256) == 16 * 8
    assert metal.mix_add_rms_threadgroup_size(32, None, 256, "1d") == 128
    with pytest.raises(ValueError):
        metal.mix_add_rms_threadgroup_size(4, torch.int32, 256)


def test_validation_precedes_device_check():
    x = torch.randn(2, 4, 16)
    M, h, w = torch.eye(4), torch.ones(4), torch.ones(16)
    with pytest.raises(ValueError, match="M must be shape"):
        metal.mhc_forward_fused_metal(x, torch.eye(3), h, h, w)
    with pytest.raises(ValueError, match="rms_weight"):
        metal.mhc_forward_fused_metal(x, M, h, h, torch.ones(8))
    with pytest.raises(ValueError, match="x must be"):
        metal.mhc_forward_fused_metal(torch.randn(4, 16), M, h, h, w)
    with pytest.raises(ValueError, match="exceeds MAX_N_ALLOWED"):
        metal.sinkhorn_knopp_metal(torch.randn(65, 65))
    with pytest.raises(ValueError, match="square"):
        metal.sinkhorn_knopp_metal(torch.randn(3, 4))
    with pytest.raises(ValueError, match="threads_per_group"):
        metal.stream_mix_add_metal(x, M, x, threads_per_group=0)
    # valid arguments on CPU tensors: no silent CPU path
    with pytest.raises(RuntimeError, match="CUDA"):
        metal.mhc_forward_fused_metal(x, M, h, h, w)


def test_layer_constructor_checks_and_init():
    with pytest.raises(ValueError):
        MHCLayer(0, 16)
    with pytest.raises(ValueError):
        MHCLayer(4, 16, dispatch_policy="fast")
    with pytest.raises(ValueError):
        MHCLayer(4, 16, mix_kernel="3d")
    L = MHCLayer(4, 16)
    assert L.H_res_raw.shape == (4, 4) and L.rms_weight.shape == (16,)
    assert torch.equal(L.H_res_raw.diag(), torch.zeros(4))
    assert float(L.H_res_raw[0, 1]) == -12.0 and float(L.H_pre_raw[0]) == -12.0
    Z = MHCLayer(4, 16, identity_init=False)
    assert torch.count_nonzero(Z.H_res_raw) == 0
    assert all(p.dtype == torch.float32 for p in L.parameters())
    with pytest.raises(ValueError):
        L(torch.randn(1, 3, 16))
    with pytest.raises(ValueError):
        L(torch.randn(1, 4, 8))


def test_use_metal_false_has_no_fallback(monkeypatch):
    L = MHCLayer(4, 16, use_metal=False)
    assert L._should_use_metal(1, 4, 16) is False
    with pytest.raises(RuntimeError, match="no silent fallback"):
        L(torch.randn(1, 4, 16))
    monkeypatch.setenv("MHC_MLX_DISABLE_METAL", "1")
    L2 = MHCLayer(4, 16)
    with pytest.raises(RuntimeError):
        L2(torch.randn(1, 4, 16))


def test_rewire_construction():
    m = MHCRewire(nn.Linear(512, 512), dims=512, n=16)
    assert m.mhc.n == 16 and m.mhc.C == 32
    with pytest.raises(ValueError):
        MHCRewire(nn.Linear(100, 100), dims=100, n=32)


def test_determinism_and_pickling():
    torch.manual_seed(42)
    a = MHCLayer(16, 64)
    torch.manual_seed(42)
    b = MHCLayer(16, 64)
    for (k1, v1), (k2, v2) in zip(a.state_dict().items(), b.state_dict().items()):
        assert k1 == k2 and torch.equal(v1, v2)
    buf = io.BytesIO()
    pickle.dump(a, buf)
    buf.seek(0)
    c = pickle.load(buf)
    for (k1, v1), (k2, v2) in zip(a.state_dict().items(), c.state_dict().items()):
        assert k1 == k2 and torch.equal(v1, v2)


def test_autopatcher_custom_block(capsys):
    dims, n = 64, 4

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.linear1 = nn.Linear(dims, dims)
            self.linear2 = nn.Linear(dims, dims * 2)
            self.linear3 = nn.Linear(dims * 2, dims)
            self.linear4 = nn.Linear(dims, dims)

    model = Block()
    assert AutoPatcher.patch(model, n_streams=n, verbose=True) == 2
    assert isinstance(model.linear1, MHCRewire) and isinstance(model.linear4, MHCRewire)
    assert not isinstance(model.linear2, MHCRewire) and not isinstance(model.linear3, MHCRewire)
    assert "[AutoPatcher] Rewiring linear1 (dims=64, streams=4)" in capsys.readouterr().out


def test_autopatcher_list_and_dict_containers():
    dims, n = 64, 4

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.layers = nn.ModuleList([nn.Linear(dims, dims), nn.Linear(dims, 32)])
            self.seq = nn.Sequential(nn.Linear(dims, dims), nn.ReLU())
            self.heads = nn.ModuleDict({"a": nn.Linear(dims, dims), "b": nn.Linear(dims, 3)})

    model = Model()
    AutoPatcher.patch(model, n_streams=n, verbose=False)
    assert isinstance(model.layers[0], MHCRewire) and not isinstance(model.layers[1], MHCRewire)
    assert isinstance(model.seq[0], MHCRewire)
    assert isinstance(model.heads["a"], MHCRewire) and not isinstance(model.heads["b"], MHCRewire)
    # idempotent on the wrapped tree: inner Linears of wrappers are not re-wrapped
    assert AutoPatcher.patch(model, n_streams=n, verbose=False) == 0


def test_autopatcher_quantized_linear():
    q = QuantizedLinear.from_linear(nn.Linear(512, 512), group_size=64, bits=4)

    class M(nn.Module):
        def __init__(self):
            super().__init__()
            self.q = q

    m = M()
    assert AutoPatcher._get_dims(q) == 512 and AutoPatcher._is_patchable(q, 16)
    AutoPatcher.patch(m, n_streams=16, verbose=False)
    assert isinstance(m.q, MHCRewire)
    assert not any(p.requires_grad for p in m.q.inner.parameters())


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_quantized_linear_roundtrip(bits):
    torch.manual_seed(0)
    lin = nn.Linear(256, 128)
    q = QuantizedLinear.from_linear(lin, group_size=64, bits=bits)
    codes = q.codes()
    assert codes.min() >= 0 and codes.max() < 2 ** bits
    assert torch.equal(QuantizedLinear.pack(codes, bits), q.weight)
    w = q.dequantize(torch.float32)
    step = (lin.weight.detach().reshape(128, -1, 64).amax(-1) -
            lin.weight.detach().reshape(128, -1, 64).amin(-1)) / (2 ** bits - 1)
    err = (w - lin.weight.detach()).abs().reshape(128, -1, 64).amax(-1)
    assert torch.all(err <= 0.5 * step + 2e-3 * step.clamp_min(1e-3) + 1e-3)
    x = torch.randn(3, 256, dtype=torch.float16)
    y = q(x)
    assert y.shape == (3, 128)


def test_reference_import_names():
    """test_packaging.py analogue: the reference's import names resolve."""
    import mhc_mlx
    import mlx_mhc
    from mhc_mlx.metal import mhc_forward_fused_metal, sinkhorn_knopp_metal  # noqa: F401

    assert mlx_mhc.__version__ == mhc_mlx.__version__ == mhc_b200.__version__
    assert mlx_mhc.MHCLayer is MHCLayer and mhc_mlx.metal is metal


def _llama_mock():
    import sys as _sys
    ex = str(Path(__file__).resolve().parent.parent / "mhc-mlx_b200" / "examples")
    if ex not in _sys.path:
        _sys.path.insert(0, ex)
    import llama_mock

    return llama_mock


def test_llama_mock_patch_structure():
    """BASELINE config 5 wiring: the reference's patch rule wraps the square
    projections (wq, wk, wv, wo) of every block; wrapped weights are frozen."""
    lm = _llama_mock()
    model = lm.build(layers=2, dims=64, num_heads=4, mlp_dims=172, vocab=100, n_streams=4,
                     dtype=torch.float32, device="cpu")
    wrapped = [n for n, m in model.named_modules() if isinstance(m, MHCRewire)]
    assert sorted(wrapped) == sorted(f"layers.{b}.attention.{w}" for b in range(2)
                                     for w in ("wq", "wk", "wv", "wo"))
    trainable = [n for n, p in model.named_parameters() if p.requires_grad]
    assert trainable and all(".mhc." in n for n in trainable)
    assert not isinstance(model.layers[0].feed_forward.w1, MHCRewire)


def test_qlinear_validation_without_gpu():
    """The in-kernel-dequantisation GEMM checks its arguments before any CUDA
    call: unsupported bit widths / group sizes / shapes are reported, not run."""
    with pytest.raises(_capi.MHCError, match="bits=4, group_size=64"):
        _capi.call("mhc_qlinear_fwd", None, _capi.MHC_BF16, None, None, None, _capi.MHC_F16, None,
                   None, 8, 256, 256, 64, 8, None)
    with pytest.raises(_capi.MHCError, match="multiples of 128"):
        _capi.call("mhc_qlinear_bwd_dx", None, _capi.MHC_BF16, None, None, None, _capi.MHC_F16,
                   None, 8, 256, 192, 64, 4, None)
    with pytest.raises(_capi.MHCError, match="bf16 or fp16"):
        _capi.call("mhc_qlinear_fwd", None, _capi.MHC_F32, None, None, None, _capi.MHC_F16, None,
                   None, 8, 256, 256, 64, 4, None)
    # M = 0 is a no-op
    _capi.call("mhc_qlinear_fwd", None, _capi.MHC_BF16, None, None, None, _capi.MHC_F16, None,
               None, 0, 256, 256, 64, 4, None)


def test_qlinear_kernel_selection():
    """CUDA bf16/fp16 activations with 4-bit codes in groups of 64 take the
    in-kernel path; other configurations dequantise with torch."""
    q = QuantizedLinear(256, 256, bits=4, group_size=64)
    x16 = torch.zeros(2, 256, dtype=torch.bfloat16)
    assert not q._in_kernel(x16)  # CPU tensor
    assert not QuantizedLinear(256, 256, bits=8, group_size=64)._in_kernel(x16)
    y = q(x16)  # torch path on the CPU
    assert y.shape == (2, 256)
