"""Drop the B200 backend family into a VibeGEMM source tree and build it with its own CMake.

    python -m vibegemm_b200.dropin <copy-of-VibeGEMM> [--build]

``install(tree)`` turns a (copy of a) VibeGEMM tree into one that builds the B200 family
next to its A100/H100 families, with the tree's own ``CMakeLists.txt``, ``main.cu``, engine
and headers. It adds new files and makes four small additive edits; nothing of the tree is
removed or rewritten:

* new files: ``csrc/gemm_b200_backends.cu`` (the ``REGISTER_B200_KERNEL`` registrations),
  ``csrc/gemm_b200.cu`` (launcher and C ABI), ``csrc/b200/*.cuh`` (the kernels),
  ``include/vibegemm_b200.h`` (the C ABI header);
* ``include/registry.cuh``: a ``REGISTER_B200_KERNEL`` macro (priority 3) after the
  H100 one, built on the tree's own ``_KREG_IMPL``;
* ``csrc/cublas_backends.cu``: a ``HAS_B200`` arm before the final ``#else`` / ``#error``,
  with row-major C (the ``HAS_A100`` operand order, which the B200 family writes);
* ``main.cu``: devices of compute capability 10.x log to ``results/perf_b200.txt``, and
  B200 backends are skipped on older devices (as the tree skips H100 ones below sm_90);
* ``CMakeLists.txt``: ``-DTARGET_GPU=B200`` builds the ``gemm_b200`` library for sm_100a
  (linked whole-archive like the other families) and defines ``HAS_B200``.

Every edit is anchored on a line the tree must contain; a tree that lacks one raises
``DropinError`` instead of being edited blindly, and a tree that already has the B200
family is left as it is. ``build(tree)`` configures and builds with
``cmake -DTARGET_GPU=B200``; the driver lands in ``<tree>/out/VibeGEMM``.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
HEADER = PKG.parent / "include" / "vibegemm_b200.h"

# (tree-relative destination, source in this repository)
NEW_FILES = [
    ("csrc/gemm_b200_backends.cu", CSRC / "gemm_b200_backends.cu"),
    ("csrc/gemm_b200.cu", CSRC / "gemm_b200.cu"),
    ("csrc/b200/gemm_kernel.cuh", CSRC / "b200" / "gemm_kernel.cuh"),
    ("csrc/b200/ptx.cuh", CSRC / "b200" / "ptx.cuh"),
    ("csrc/b200/schedule.cuh", CSRC / "b200" / "schedule.cuh"),
    ("include/vibegemm_b200.h", HEADER),
]

MARK = "B200 drop-in"  # tags every inserted block, so a second install is a no-op

# (file, anchor line, "after" | "before", inserted lines). The anchor is matched on the
# stripped text of one line of the tree.
EDITS = [
    ("include/registry.cuh",
     "#define REGISTER_H100_KERNEL(dn, BC)  _KREG_IMPL(2, dn, BC, __COUNTER__)", "after",
     [f"// {MARK}: B200 (sm_100a) family, after the H100 one",
      "#define REGISTER_B200_KERNEL(dn, BC)  _KREG_IMPL(3, dn, BC, __COUNTER__)"]),
    ("csrc/cublas_backends.cu",
     '#error "Neither HAS_H100 nor HAS_A100 is defined"', "before-prev",
     [f"#elif defined(HAS_B200) // {MARK}: row-major C, as the B200 family writes it",
      "        CUBLAS_CHECK(cublasGemmEx(handle_, CUBLAS_OP_T, CUBLAS_OP_N, N, M, K, &alpha, B, CUDA_R_16F,",
      "                                  K, A, CUDA_R_16F, K, &beta, C, CUDA_R_16F, N, CUBLAS_COMPUTE_32F,",
      "                                  CUBLAS_GEMM_DEFAULT));"]),
    ("main.cu",
     'std::string log_file = (sm >= 90) ? "results/perf_h100.txt" : "results/perf_a100.txt";', "after",
     [f"    if (sm >= 100) // {MARK}",
      '        log_file = "results/perf_b200.txt";']),
    ("main.cu",
     'if (sm < 90 && name.find("H100") != std::string::npos)', "after-next",
     [f"        if (sm < 100 && name.find(\"B200\") != std::string::npos) // {MARK}",
      "            continue;"]),
    ("CMakeLists.txt",
     'elseif(TARGET_GPU STREQUAL "A100")', "before",
     [f'elseif(TARGET_GPU STREQUAL "B200") # {MARK}: sm_100a family',
      '    add_gemm_library(gemm_b200 "csrc/gemm_b200_backends.cu;csrc/gemm_b200.cu" "100a")',
      "    list(APPEND GEMM_LIBS $<LINK_LIBRARY:WHOLE_ARCHIVE,gemm_b200>)",
      '    list(APPEND GEMM_ARCHS "100a")',
      "    add_compile_definitions(HAS_B200)"]),
]


class DropinError(RuntimeError):
    """The tree does not look like a VibeGEMM tree this installer knows how to edit."""


def _edit(path: Path, anchor: str, where: str, lines: list[str]) -> None:
    text = path.read_text()
    rows = text.split("\n")
    hits = [i for i, r in enumerate(rows) if r.strip() == anchor]
    if len(hits) != 1:
        raise DropinError(f"{path}: expected exactly one line {anchor!r}, found {len(hits)}")
    i = hits[0]
    if where == "after":
        at = i + 1
    elif where == "after-next":  # after the statement's second line (a `continue;`)
        at = i + 2
    elif where == "before":
        at = i
    elif where == "before-prev":  # before the line preceding the anchor (an `#else`)
        if i == 0 or rows[i - 1].strip() != "#else":
            raise DropinError(f"{path}: no #else directly before {anchor!r}")
        at = i - 1
    else:
        raise ValueError(where)
    rows[at:at] = lines
    path.write_text("\n".join(rows))


def install(tree: str | os.PathLike) -> list[str]:
    """Adds the B200 family to `tree`; returns the tree-relative paths it created or edited."""
    root = Path(tree)
    for f in ("CMakeLists.txt", "main.cu", "include/registry.cuh", "include/backend.cuh",
              "include/engine.cuh", "csrc/cublas_backends.cu"):
        if not (root / f).is_file():
            raise DropinError(f"{root} has no {f}: not a VibeGEMM tree")
    touched = []
    for rel, src in NEW_FILES:
        dst = root / rel
        dst.parent.mkdir(parents=True, exist_ok=True)
        shutil.copyfile(src, dst)
        touched.append(rel)
    for rel, anchor, where, lines in EDITS:
        path = root / rel
        if _has_block(path, lines):  # installed before
            continue
        _edit(path, anchor, where, lines)
        if rel not in touched:
            touched.append(rel)
    return touched


def _has_block(path: Path, lines: list[str]) -> bool:
    return "\n".join(lines) in path.read_text()


def build(tree: str | os.PathLike, jobs: int = 8, cmake: str = "cmake", nvcc: str | None = None) -> Path:
    """Configures and builds `tree` with -DTARGET_GPU=B200; returns the driver's path."""
    root = Path(tree)
    bdir = root / "build"
    cfg = [cmake, "-S", str(root), "-B", str(bdir), "-DTARGET_GPU=B200", "-DCMAKE_BUILD_TYPE=Release"]
    nvcc = nvcc or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cfg.append(f"-DCMAKE_CUDA_COMPILER={nvcc}")
    for cmd in (cfg, [cmake, "--build", str(bdir), "-j", str(jobs)]):
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"{' '.join(cmd)} failed ({proc.returncode}):\n{proc.stdout[-4000:]}\n"
                               f"{proc.stderr[-4000:]}")
    exe = root / "out" / "VibeGEMM"
    if not exe.is_file():
        raise RuntimeError(f"build finished without {exe}")
    return exe


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("tree", help="a VibeGEMM source tree (a writable copy)")
    ap.add_argument("--build", action="store_true", help="also configure and build it with CMake")
    ap.add_argument("-j", "--jobs", type=int, default=8)
    args = ap.parse_args()
    for rel in install(args.tree):
        print("installed", rel)
    if args.build:
        print("built", build(args.tree, args.jobs))


if __name__ == "__main__":
    main()
