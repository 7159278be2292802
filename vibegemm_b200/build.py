"""Build recipe for the B200 GEMM library and the VibeGEMM driver binary.

Compiles every CUDA source for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``)
with nvcc, in-tree, so the built files travel with the source tree:

* ``vibegemm_b200/libvibegemm_b200.so`` — kernels, C ABI, registry/backends, engine.
* ``vibegemm_b200/bin/VibeGEMM``        — the driver (main.cu) linked with the same objects.

Objects are cached under ``vibegemm_b200/_build/`` and rebuilt when a source or any
header is newer. ``python -m vibegemm_b200.build`` runs it from the command line.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "libvibegemm_b200.so"
BIN = PKG / "bin" / "VibeGEMM"

LIB_SOURCES = ["gemm_b200.cu", "cublas_backends.cu", "gemm_b200_backends.cu", "engine_capi.cu",
               "host_pipeline.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-DHAS_B200", "-Xcompiler", "-fPIC",
         "--expt-relaxed-constexpr", "-I" + str(INCLUDE), "-I" + str(CSRC)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or add /usr/local/cuda/bin to PATH)")


def _headers() -> list[Path]:
    return list(INCLUDE.glob("*.h")) + list(INCLUDE.glob("*.cuh")) + list(CSRC.rglob("*.cuh"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}\n"
                           f"{proc.stdout}\n{proc.stderr}")


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if _stale(obj, [src] + _headers()):
        _run([nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)], verbose)
    return obj


def build(verbose: bool = False, driver: bool = True) -> Path:
    """Compile the library (and the driver binary); returns the library path."""
    BUILD.mkdir(exist_ok=True)
    srcs = [CSRC / s for s in LIB_SOURCES]
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs + ([CSRC / "main.cu"] if driver else [])))
    lib_objs = objs[: len(srcs)]
    if _stale(LIB, lib_objs):
        _run([nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, lib_objs), "-lcublas", "-lcublasLt"], verbose)
    if driver:
        BIN.parent.mkdir(exist_ok=True)
        if _stale(BIN, objs):
            _run([nvcc(), *ARCH, "-o", str(BIN), *map(str, objs), "-lcublas", "-lcublasLt"], verbose)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
