"""Build libmhc_b200.so in-tree with nvcc for sm_100a.

Usage:  python -m mhc_b200._build [--force] [-j N]

The library is written next to this file (``_lib/libmhc_b200.so``) so that it
travels with the source tree; nothing is installed into site-packages.  The
CUDA runtime is linked statically, so loading the library needs no GPU and
no driver (symbols can be inspected on a CPU-only machine).

Staleness is decided by content, not by file times: the build hashes every
source and header together with the compiler flags, compiles that hash into
the library (``mhc_build_id()``) and writes it beside the library
(``libmhc_b200.so.id``).  A library whose id differs from the hash of the
sources next to it is rebuilt, and the ctypes loader refuses to load one.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
SRC_DIR = PKG_DIR.parent / "csrc"
REPO_DIR = PKG_DIR.parent.parent
INCLUDE_DIR = REPO_DIR / "include"
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "libmhc_b200.so"
ID_PATH = LIB_DIR / "libmhc_b200.so.id"
OBJ_DIR = LIB_DIR / "obj"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-DMHC_BUILDING_LIB",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libmhc_b200.so")
    return cand


def sources() -> list[Path]:
    return sorted(SRC_DIR.glob("*.cu"))


def _deps() -> list[Path]:
    return sources() + sorted(SRC_DIR.glob("*.cuh")) + sorted(SRC_DIR.glob("*.h")) + [
        INCLUDE_DIR / "mhc_b200.h"
    ]


def source_hash() -> str:
    """sha256 (first 16 hex digits) of every source and header, by name and
    content, and of the compiler flags."""
    h = hashlib.sha256()
    for p in _deps():
        h.update(p.name.encode() + b"\0" + p.read_bytes() + b"\0")
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()[:16]


def built_id() -> str | None:
    try:
        return ID_PATH.read_text().strip()
    except OSError:
        return None


def is_stale() -> bool:
    return not LIB_PATH.exists() or built_id() != source_hash()


def build(force: bool = False, jobs: int | None = None, verbose: bool = True) -> Path:
    """Compile every csrc/*.cu for sm_100a and link libmhc_b200.so."""
    if not force and not is_stale():
        return LIB_PATH
    nvcc = _nvcc()
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    inc = [f"-I{INCLUDE_DIR}", f"-I{SRC_DIR}"]
    bid = source_hash()

    headers = [p for p in _deps() if p.suffix != ".cu"]

    def compile_one(src: Path) -> Path:
        obj = OBJ_DIR / (src.stem + ".o")
        # an object is reused when its source, every header and the flags are
        # byte-identical to the ones it was compiled from (the build id is
        # only compiled into mhc_capi.cu, which is rebuilt whenever it changes)
        h = hashlib.sha256()
        for q in [src, *headers]:
            h.update(q.name.encode() + b"\0" + q.read_bytes() + b"\0")
        h.update(" ".join(NVCC_FLAGS).encode())
        if src.name == "mhc_capi.cu":
            h.update(bid.encode())
        stamp = obj.with_suffix(".o.id")
        if obj.exists() and stamp.exists() and stamp.read_text().strip() == h.hexdigest():
            return obj
        cmd = [nvcc, *NVCC_FLAGS, f"-DMHC_BUILD_ID=\"{bid}\"", *inc, "-c", str(src), "-o", str(obj)]
        if verbose:
            print("[mhc_b200 build]", " ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        stamp.write_text(h.hexdigest() + "\n")
        return obj

    jobs = jobs or min(8, os.cpu_count() or 4)
    with ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", *map(str, objs), "-o", str(tmp)]
    if verbose:
        print("[mhc_b200 build]", " ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    ID_PATH.write_text(bid + "\n")
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    a = ap.parse_args(argv)
    p = build(force=a.force, jobs=a.jobs)
    print(p)
    return 0


if __name__ == "__main__":
    sys.exit(main())
