"""ctypes binding of libmhc_b200.so (the C ABI declared in include/mhc_b200.h).

The library is loaded lazily on first use so that the pure host-side parts
of the package (module rewiring, argument validation) import on machines
without a GPU.  There is no fallback: if the library is missing or a call
fails, an exception is raised.
"""

from __future__ import annotations

import ctypes
import os
import threading
from ctypes import c_float, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libmhc_b200.so"

MHC_F32, MHC_F16, MHC_BF16 = 0, 1, 2
MHC_OK, MHC_ERR_INVALID, MHC_ERR_CUDA, MHC_ERR_UNSUPPORTED, MHC_ERR_WORKSPACE = 0, 1, 2, 3, 4

_P = c_void_p
# name -> (restype, argtypes); mirrors include/mhc_b200.h
SIGNATURES: dict[str, tuple] = {
    "mhc_last_error": (ctypes.c_char_p, []),
    "mhc_version": (c_int, []),
    "mhc_build_id": (ctypes.c_char_p, []),
    "mhc_selftest_reciprocal": (c_int, [_P, _P, c_int64, _P]),
    "mhc_device_sm_count": (c_int, [ctypes.POINTER(c_int)]),
    "mhc_sinkhorn_tape_floats": (c_size_t, [c_int, c_int]),
    "mhc_params_fwd": (c_int, [_P, _P, _P, c_int, c_int, c_float, _P, _P, _P, _P, _P]),
    "mhc_params_bwd": (c_int, [_P, _P, _P, _P, c_int, c_int, c_float, _P, _P, _P, _P, _P, _P, _P]),
    "mhc_sinkhorn_batched_workspace_bytes": (c_size_t, [c_int64, c_int, c_int]),
    "mhc_sinkhorn_batched_fwd": (c_int, [_P, c_int64, c_int, c_int, c_float, _P, _P]),
    "mhc_sinkhorn_batched_bwd": (c_int, [_P, _P, c_int64, c_int, c_int, c_float, _P, _P, c_size_t, _P]),
    "mhc_fwd": (c_int, [_P, c_int, _P, _P, _P, _P, _P, c_int, c_int64, c_int, c_int, c_float, _P]),
    "mhc_bwd_workspace_bytes": (c_size_t, [c_int64, c_int, c_int]),
    "mhc_bwd": (c_int, [_P, c_int, _P, c_int, _P, _P, _P, _P, _P, c_int, c_int64, c_int, c_int,
                        c_float, _P, c_size_t, _P]),
    "mhc_bwd_finalize": (c_int, [_P, c_int, c_int, _P, _P, _P, _P, _P, _P, _P, _P, c_int, c_float,
                                 _P, _P, _P, _P]),
    "mhc_bwd_noalloc": (c_int, [_P, c_int, _P, c_int, _P, _P, _P, _P, _P, c_int, _P, _P, _P, _P,
                                c_int64, c_int, c_int, c_float, _P]),
    "mhc_mix_add_fwd": (c_int, [_P, c_int, _P, _P, c_int, _P, c_int, c_int64, c_int, c_int, _P]),
    "mhc_mix_bwd_workspace_bytes": (c_size_t, [c_int64, c_int, c_int]),
    "mhc_mix_add_bwd": (c_int, [_P, c_int, _P, _P, c_int, _P, c_int, _P, c_int64, c_int, c_int, _P,
                                c_size_t, _P]),
    "mhc_rewire_combine_fwd": (c_int, [_P, c_int, _P, c_int, _P, _P, _P, _P, c_int, c_int64, c_int,
                                       c_int, _P]),
    "mhc_rewire_bwd_workspace_bytes": (c_size_t, [c_int64, c_int, c_int]),
    "mhc_rewire_combine_bwd": (c_int, [_P, c_int, _P, c_int, _P, c_int, _P, _P, _P, _P, c_int, _P,
                                       c_int, _P, _P, _P, c_int64, c_int, c_int, _P, c_size_t, _P]),
    "mhc_rewire_fused_bwd_workspace_bytes": (c_size_t, [c_int64, c_int, c_int]),
    "mhc_rewire_bwd_dy": (c_int, [_P, c_int, _P, c_int, _P, _P, c_int, c_int64, c_int, c_int, _P,
                                  c_size_t, _P]),
    "mhc_rewire_bwd_dx": (c_int, [_P, c_int, _P, c_int, _P, c_int, _P, _P, _P, _P, c_int, _P, _P,
                                  _P, _P, _P, _P, _P, _P, c_int, c_float, _P, _P, _P, c_int64,
                                  c_int, c_int, _P, c_size_t, _P]),
    "mhc_rewire_jacobian_floats": (c_size_t, [c_int]),
    "mhc_rewire_in_fwd": (c_int, [_P, c_int, _P, _P, _P, c_int, c_float, _P, _P, _P, _P, _P, _P,
                                  c_int, c_int64, c_int, c_int, _P]),
    "mhc_prescale_fwd": (c_int, [_P, c_int, _P, _P, c_int, c_int64, c_int, c_int, _P]),
    "mhc_prescale_bwd": (c_int, [_P, c_int, _P, c_int, _P, _P, c_int, _P, c_int64, c_int, c_int, _P,
                                 c_size_t, _P]),
    "mhc_qlinear_fwd": (c_int, [_P, c_int, _P, _P, _P, c_int, _P, _P, c_int64, c_int, c_int, c_int,
                                c_int, _P]),
    "mhc_qlinear_bwd_dx": (c_int, [_P, c_int, _P, _P, _P, c_int, _P, c_int64, c_int, c_int, c_int,
                                   c_int, _P]),
    "mhc_qlinear_transpose_pack": (c_int, [_P, _P, c_int, c_int, _P]),
    "mhc_qlinear_bwd_dx_t": (c_int, [_P, c_int, _P, _P, _P, _P, c_int64, c_int, c_int, c_int,
                                     c_int, _P]),
    "mhc_residual_add_agg": (c_int, [_P, c_int, _P, c_int, _P, _P, c_int, _P, c_int64, c_int, c_int,
                                     _P]),
    "mhc_residual_add_agg_bwd": (c_int, [_P, c_int, _P, c_int, _P, _P, _P, c_int, _P, c_int64,
                                         c_int, c_int, _P, c_size_t, _P]),
}

_lib = None
_lock = threading.Lock()

# Number of status-returning C-ABI calls made by this process.  Every such
# call enqueues kernels; the benchmark uses the count to report launches.
CALLS = 0


class MHCError(RuntimeError):
    """A libmhc_b200 call returned a nonzero status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed (status {code}): {msg}")
        self.code = code


def library_path() -> Path:
    override = os.environ.get("MHC_B200_LIB")
    return Path(override) if override else LIB_PATH


def load() -> ctypes.CDLL:
    """Load (once) and return the library, with argtypes set from SIGNATURES."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.exists():
            raise RuntimeError(
                f"libmhc_b200.so not found at {path}; build it with "
                "`python -m mhc_b200._build` (needs nvcc).  There is no non-CUDA fallback."
            )
        lib = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _check_build_id(lib, path)
        _lib = lib
    return _lib


def _check_build_id(lib: ctypes.CDLL, path: Path) -> None:
    """Refuse a library built from other sources than the ones beside it
    (the id compiled into the library is the hash of csrc/ and include/ at
    build time).  Skipped for an explicit MHC_B200_LIB override and when the
    sources are not present."""
    if os.environ.get("MHC_B200_LIB"):
        return
    from . import _build

    if not _build.SRC_DIR.is_dir():
        return
    have = (lib.mhc_build_id() or b"").decode()
    want = _build.source_hash()
    if have != want:
        raise RuntimeError(
            f"{path} was built from different sources (build id {have or 'none'}, sources "
            f"{want}); rebuild it with `python -m mhc_b200._build`.")


def exported_symbols() -> list[str]:
    lib = load()
    return [n for n in SIGNATURES if hasattr(lib, n)]


def call(name: str, *args) -> None:
    """Call a status-returning entry point; raise on a nonzero status."""
    global CALLS
    lib = load()
    rc = getattr(lib, name)(*args)
    CALLS += 1
    if rc != MHC_OK:
        msg = (lib.mhc_last_error() or b"").decode(errors="replace")
        if rc == MHC_ERR_INVALID:
            raise ValueError(f"{name}: {msg}")
        raise MHCError(name, rc, msg)


def query(name: str, *args):
    return getattr(load(), name)(*args)


# ----------------------------------------------------------------- helpers --
_DT = {torch.float32: MHC_F32, torch.float16: MHC_F16, torch.bfloat16: MHC_BF16}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}; expected float32, float16 or bfloat16") from None


def ptr(t: torch.Tensor | None):
    """Device address as a plain int (argtypes convert it to void*); None -> NULL."""
    return None if t is None else t.data_ptr()


# The raw current-stream handle without building a torch Stream object (a
# few microseconds per call on the B=1 path); the public API otherwise.
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(t: torch.Tensor) -> int:
    if _raw_stream is not None:
        return _raw_stream(t.device.index)
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*ts: torch.Tensor | None) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                "mhc_b200 runs only on CUDA tensors (sm_100a kernels); got a tensor on "
                f"{t.device}.  There is no CPU fallback."
            )
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    return dev
