"""Build the in-tree CUDA library ``mlx_motif/libmotif_b200.so`` for sm_100a.

Every ``csrc/*.cu`` is compiled with nvcc for ``arch=compute_100a,code=sm_100a``
(objects under ``_build/``, in parallel) and linked into one shared library
exporting the C ABI declared in ``include/motif_b200.h``. A stamp of the
sources, header and flags skips the build when nothing changed.

Usage: ``python mlx-motif_b200/build_native.py [--force]``.
"""

from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = REPO_ROOT / "include"
BUILD = PKG_ROOT / "_build"
LIB = PKG_ROOT / "mlx_motif" / "libmotif_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-DMOTIF_BUILD",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put CUDA's bin on PATH)")


def _stamp(sources: list[Path]) -> str:
    h = hashlib.sha256()
    for p in sorted(sources) + sorted(INCLUDE.glob("*.h")) + sorted(CSRC.glob("*.cuh")):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(ARCH + NVCC_FLAGS).encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile (if needed) and return the path of the shared library."""
    sources = sorted(CSRC.glob("*.cu"))
    stamp = _stamp(sources)
    stamp_file = BUILD / "stamp"
    if not force and LIB.exists() and stamp_file.exists() and stamp_file.read_text() == stamp:
        return LIB
    BUILD.mkdir(parents=True, exist_ok=True)
    nvcc = _nvcc()
    include = ["-I", str(INCLUDE), "-I", str(CSRC)]

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, *include, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        return obj

    workers = max(1, min(len(sources), os.cpu_count() or 4))
    with cf.ThreadPoolExecutor(workers) as ex:
        objs = list(ex.map(compile_one, sources))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    stamp_file.write_text(stamp)
    return LIB


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)
