"""AutoPatcher: wrap residual-compatible projections of a torch model with
MHCRewire (reference mhc_mlx/patching.py:4-126).

A module is patchable when it is an nn.Linear or a QuantizedLinear whose
input and output widths are equal and divisible by the stream count.  The
walk works on nn.Module trees, including nn.ModuleList / nn.Sequential
(numeric child names) and nn.ModuleDict.
"""

from __future__ import annotations

from torch import nn

from .layer import MHCRewire
from .quantized import QuantizedLinear


class AutoPatcher:
    @staticmethod
    def patch(model: nn.Module, n_streams: int = 32, verbose: bool = True, output_dtype=None,
              **mhc_kwargs) -> int:
        """Patch `model` in place; returns the number of wrapped modules.
        output_dtype and mhc_kwargs are passed to every MHCRewire."""
        count = 0
        # snapshot first: the tree is mutated while walking
        modules = list(model.named_modules())
        for name, module in modules:
            if name == "":
                continue
            parent_path, _, child_name = name.rpartition(".")
            parent = model.get_submodule(parent_path) if parent_path else model
            if isinstance(parent, MHCRewire):
                continue  # never re-wrap the inner module of a fresh wrapper
            if not AutoPatcher._is_patchable(module, n_streams):
                continue
            dims = AutoPatcher._get_dims(module)
            if verbose:
                print(f"[AutoPatcher] Rewiring {name} (dims={dims}, streams={n_streams})")
            wrapped = MHCRewire(module, dims=dims, n=n_streams, output_dtype=output_dtype,
                                **mhc_kwargs)
            p = next(module.parameters(), None) if hasattr(module, "parameters") else None
            if p is not None:
                wrapped.mhc.to(p.device)
            setattr(parent, child_name, wrapped)
            count += 1
        if verbose:
            print(f"[AutoPatcher] Patched {count} layers.")
        return count

    @staticmethod
    def _get_dims(module: nn.Module) -> int:
        if isinstance(module, nn.Linear):
            return int(module.weight.shape[1])  # [out, in]
        if isinstance(module, QuantizedLinear):
            return int(module.input_dims)
        return 0

    @staticmethod
    def _is_patchable(module: nn.Module, n: int) -> bool:
        """Linear / QuantizedLinear, in_dims == out_dims, in_dims % n == 0."""
        if isinstance(module, nn.Linear):
            in_dims, out_dims = int(module.weight.shape[1]), int(module.weight.shape[0])
        elif isinstance(module, QuantizedLinear):
            in_dims, out_dims = int(module.input_dims), int(module.output_dims)
        else:
            return False
        if in_dims == 0 or out_dims == 0:
            return False
        if in_dims != out_dims:
            return False
        return in_dims % n == 0
