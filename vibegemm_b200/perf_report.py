"""Performance report of the VibeGEMM driver logs.

The driver (``bin/VibeGEMM``) writes the reference's text log, ``results/perf_<arch>.txt``,
and one JSON line per (backend, shape) to ``results/perf_<arch>.jsonl``. This module reads
both:

* ``parse_perf_file`` follows the reference's log parser (plot_perf.py:9-25 of VibeGEMM):
  the first ``[cuBLAS]`` block's TFLOPS and, in order, every ``[VibeGEMM ... vN]`` block's
  TFLOPS, with the same two patterns, so logs of all three architectures parse alike.
* ``load_jsonl`` / ``markdown_table`` turn the JSON log into a per-shape table (TFLOP/s,
  % of cuBLAS, % of peak, check result).
* ``main`` runs the reference's task list with a ``perf_b200`` task added
  (plot_perf.py:75-90): a PNG per log when matplotlib is importable, else the text table.

    python -m vibegemm_b200.perf_report [results_dir]
"""
from __future__ import annotations

import json
import os
import re
import sys

_CUBLAS = re.compile(r"\[cuBLAS\].*?(\d+\.\d+)\s+TFLOPS", re.DOTALL)
_VERSION = re.compile(r"\[VibeGEMM.*?v(\d+)\].*?(\d+\.\d+)\s+TFLOPS", re.DOTALL)

TASKS = [
    ("perf_a100.txt", "NVIDIA A100", "perf_a100.png"),
    ("perf_h100.txt", "NVIDIA H100", "perf_h100.png"),
    ("perf_b200.txt", "NVIDIA B200", "perf_b200.png"),
]


def parse_perf_text(text: str) -> tuple[float, list[str], list[float]]:
    """(cuBLAS TFLOPS, ["v0", ...], [TFLOPS, ...]) of one driver log."""
    m = _CUBLAS.search(text)
    cublas = float(m.group(1)) if m else 0.0
    versions, tflops = [], []
    for m in _VERSION.finditer(text):
        versions.append(f"v{m.group(1)}")
        tflops.append(float(m.group(2)))
    return cublas, versions, tflops


def parse_perf_file(path: str) -> tuple[float, list[str], list[float]]:
    with open(path, "r") as f:
        return parse_perf_text(f.read())


def load_jsonl(path: str) -> list[dict]:
    rows = []
    with open(path, "r") as f:
        for line in f:
            line = line.strip()
            if line:
                rows.append(json.loads(line))
    return rows


def markdown_table(rows: list[dict]) -> str:
    """One table row per (shape, backend) that ran, in log order."""
    out = ["| shape | inputs | backend | TFLOP/s | % cuBLAS | % peak | check |",
           "|---|---|---|---|---|---|---|"]
    for r in rows:
        if not r.get("ran", True) or r.get("skipped") or "tflops" not in r:
            continue
        shape = f"{r['M']}×{r['N']}×{r['K']}"
        check = "PASS" if r.get("passed") else "FAIL"
        out.append(f"| {shape} | {r.get('inputs', '')} | {r['backend']} | {r['tflops']:.1f} | "
                   f"{r.get('pct_cublas', 0.0):.1f} | {r.get('pct_peak', 0.0):.1f} | {check} |")
    return "\n".join(out)


def _plot(path: str, gpu: str, outpath: str) -> bool:
    try:
        import matplotlib
        matplotlib.use("Agg")
        import matplotlib.pyplot as plt
    except ImportError:
        return False
    cublas, versions, tflops = parse_perf_file(path)
    fig, ax = plt.subplots(figsize=(10, 6))
    x = list(range(len(versions)))
    ax.plot(x, tflops, marker="o", linewidth=2, label="VibeGEMM")
    if cublas > 0:
        ax.axhline(cublas, linestyle="--", label=f"cuBLAS ({cublas:.1f} TFLOPS)")
    ax.set_xticks(x)
    ax.set_xticklabels(versions)
    ax.set_xlabel("VibeGEMM version")
    ax.set_ylabel("TFLOPS")
    ax.set_title(f"{gpu} — FP16 GEMM")
    ax.set_ylim(bottom=0)
    ax.legend(loc="lower right")
    fig.tight_layout()
    fig.savefig(outpath, dpi=150)
    plt.close(fig)
    return True


def main(argv: list[str]) -> int:
    results = argv[1] if len(argv) > 1 else "results"
    found = False
    for log, gpu, png in TASKS:
        path = os.path.join(results, log)
        if not os.path.exists(path):
            print(f"Warning: {path} not found, skipping.")
            continue
        found = True
        if _plot(path, gpu, os.path.join(results, png)):
            print(f"Saved -> {os.path.join(results, png)}")
        cublas, versions, tflops = parse_perf_file(path)
        print(f"{gpu}: cuBLAS {cublas:.2f} TFLOPS; " +
              ", ".join(f"{v} {t:.2f}" for v, t in zip(versions, tflops)))
        jpath = path[:-4] + ".jsonl"
        if os.path.exists(jpath):
            print(markdown_table(load_jsonl(jpath)))
    return 0 if found else 1


if __name__ == "__main__":
    sys.exit(main(sys.argv))
