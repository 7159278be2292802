"""The reference's own VibeGEMM driver with the B200 family dropped in, on a B200.

`vibegemm_b200/bin/VibeGEMM_dropin` is the reference's main.cu, engine, registry and cuBLAS
backend, built by the reference's CMake with -DTARGET_GPU=B200 after vibegemm_b200.dropin
added the B200 family (see tests/test_dropin.py; build() makes it where the reference tree
is present). Run unchanged, it benchmarks its 8192³ problem with every registered backend
and validates each one against cuBLAS with the reference's check_error: every B200 backend
must report (PASS)."""
import re
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

EXE = Path(__file__).resolve().parents[1] / "vibegemm_b200" / "bin" / "VibeGEMM_dropin"


@pytest.mark.skipif(not EXE.is_file(), reason="drop-in driver not built (no reference tree at build time)")
def test_reference_driver_validates_every_b200_backend(tmp_path):
    proc = subprocess.run([str(EXE)], cwd=tmp_path, capture_output=True, text=True, timeout=600)
    out = proc.stdout
    assert proc.returncode == 0, (out[-3000:], proc.stderr[-3000:])
    blocks = re.split(r"\n\[(.+?)\]\n", out)
    results = {}
    for name, body in zip(blocks[1::2], blocks[2::2]):
        tf = re.search(r"avg latency = ([0-9.]+) ms\s+([0-9.]+) TFLOPS", body)
        verdict = re.search(r"max relative error = .*\((PASS|FAIL)\)", body)
        results[name] = (float(tf.group(2)) if tf else None, verdict.group(1) if verdict else None)
    b200 = {k: v for k, v in results.items() if "B200" in k}
    assert "cuBLAS" in results and len(b200) == 14, results
    assert all(v[1] == "PASS" for v in b200.values()), results
    log = (tmp_path / "results" / "perf_b200.txt").read_text()
    assert "VibeGEMM B200 auto" in log
    print({k: v[0] for k, v in results.items()})
