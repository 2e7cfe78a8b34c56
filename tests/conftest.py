"""Test configuration: import paths, the `gpu` marker and golden fixtures."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "mhc-mlx_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN_DIR = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device")
    config.addinivalue_line("markers", "slow: long-running")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


class Golden:
    """Cases from tests/golden/reference_golden.npz (see make_golden.py)."""

    def __init__(self):
        self.z = np.load(GOLDEN_DIR / "reference_golden.npz")
        meta = json.loads((GOLDEN_DIR / "reference_golden.json").read_text())
        self.cases = {c["case"]: c for c in meta["cases"]}

    def names(self, kind: str) -> list[str]:
        return [k for k, c in self.cases.items() if c["kind"] == kind]

    def get(self, case: str) -> dict:
        prefix = case + "/"
        d = {k[len(prefix):]: self.z[k] for k in self.z.files if k.startswith(prefix)}
        d.update(self.cases[case])
        return d


_GOLDEN = None


def golden() -> Golden:
    global _GOLDEN
    if _GOLDEN is None:
        _GOLDEN = Golden()
    return _GOLDEN


@pytest.fixture(scope="session")
def gold() -> Golden:
    return golden()


def rel_err(a, b) -> float:
    """max |a - b| / max |b|  (the reference's relative metric,
    tests/test_correctness.py:249-251)."""
    import torch

    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    return float((a - b).abs().max() / max(float(b.abs().max()), 1e-30))


def max_abs(a, b) -> float:
    import torch

    return float((torch.as_tensor(a).double().cpu() - torch.as_tensor(b).double().cpu()).abs().max())


def assert_close_to_reference(name, got, ref64, ref32, rel=1e-5, noise_factor=4.0):
    """got must match the float64 oracle within `rel` of max|ref|, or be no
    further from it than `noise_factor` times the reference algorithm's own
    float32 rounding error (|ref32 - ref64|).  The second branch covers
    quantities that are small differences of large terms (e.g. dH_pre at
    n = 1, where RMSNorm cancels the H_pre scale analytically)."""
    e = max_abs(got, ref64)
    scale = max(float(torch_abs_max(ref64)), 1e-30)
    e32 = max_abs(ref32, ref64)
    assert e <= rel * scale or e <= noise_factor * e32 + 1e-12, (
        f"{name}: err {e:.3e}, rel {e / scale:.3e}, fp32-oracle err {e32:.3e}")


def torch_abs_max(t):
    import torch

    return torch.as_tensor(t).double().abs().max()
