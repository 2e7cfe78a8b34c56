"""Environment report (reference mhc_mlx/diagnostics.py): versions, CUDA
device, and whether libmhc_b200.so is built and exports the C ABI."""

from __future__ import annotations

import platform


def diagnostics() -> dict:
    import torch

    from . import __version__, _capi

    info = {
        "mhc_b200": __version__,
        "python": platform.python_version(),
        "torch": torch.__version__,
        "cuda_available": torch.cuda.is_available(),
        "library": str(_capi.library_path()),
        "library_built": _capi.library_path().exists(),
    }
    if torch.cuda.is_available():
        p = torch.cuda.get_device_properties(0)
        info.update(device=p.name, sm=f"{p.major}.{p.minor}", sm_count=p.multi_processor_count,
                    memory_gb=round(p.total_memory / 2**30, 1))
    if info["library_built"]:
        info["exported_symbols"] = len(_capi.exported_symbols())
        info["library_version"] = int(_capi.query("mhc_version"))
    return info


def main() -> None:
    for k, v in diagnostics().items():
        print(f"{k}: {v}")


if __name__ == "__main__":
    main()
