"""The reference package's import name (svdrecbd/mhc-mlx: ``mhc_mlx``), backed
by mhc_b200, so code written against the reference imports unchanged:

    from mhc_mlx import MHCLayer, MHCRewire, AutoPatcher, residual_add_agg
    from mhc_mlx.metal import mhc_forward_fused_metal, sinkhorn_knopp_metal

Submodules metal, layer, patching, utils resolve to their mhc_b200
counterparts.  There is no ``mhc_mlx.reference`` here: the pure-array source
of truth is test infrastructure in this repository, not part of the product.
"""

import importlib as _importlib
import sys as _sys

from mhc_b200 import (AutoPatcher, MHCLayer, MHCRewire, QuantizedLinear, __version__,  # noqa: F401
                      diagnostics, residual_add_agg)

for _name in ("metal", "layer", "patching", "utils", "quantized", "dist"):
    _mod = _importlib.import_module(f"mhc_b200.{_name}")
    _sys.modules[f"{__name__}.{_name}"] = _mod
    globals()[_name] = _mod

__all__ = ["MHCLayer", "MHCRewire", "diagnostics", "residual_add_agg", "AutoPatcher",
           "__version__"]
