"""mhc_b200: the mHC (manifold-constrained hyper-connections) hot path of
svdrecbd/mhc-mlx, rebuilt for NVIDIA B200 (sm_100a).

Public API mirrors mhc_mlx: MHCLayer, MHCRewire, AutoPatcher,
residual_add_agg, diagnostics; the launcher-level entry points live in
mhc_b200.metal under the reference's names.
"""

from .diagnostics import diagnostics
from .layer import MHCLayer, MHCRewire
from .patching import AutoPatcher
from .quantized import QuantizedLinear
from .utils import residual_add_agg

__version__ = "1.0.0"

__all__ = ["MHCLayer", "MHCRewire", "diagnostics", "residual_add_agg", "AutoPatcher",
           "QuantizedLinear", "__version__"]
