"""Driver-log parsing (text log in the reference's format, JSON lines) on CPU."""
import json

from vibegemm_b200 import perf_report

LOG = """=== Device: NVIDIA B200 (SM: 100) ===

=== GEMM  M=512  N=512  K=512 ===

[cuBLAS]
  avg latency = 0.009 ms   30.12 TFLOPS
  check: max_abs=0.000000e+00 max_rel=0.000000e+00 (PASS)

[VibeGEMM B200 v0]
  avg latency = 0.008 ms   32.50 TFLOPS
  check: max_abs=0.000000e+00 max_rel=0.000000e+00 (PASS)

[VibeGEMM B200 v1]
  avg latency = 0.008 ms   31.75 TFLOPS
  check: max_abs=0.000000e+00 max_rel=0.000000e+00 (PASS)

[VibeGEMM B200 auto]
  avg latency = 0.008 ms   32.40 TFLOPS
  check: max_abs=0.000000e+00 max_rel=0.000000e+00 (PASS)

Done.
"""


def test_text_log_parses_like_the_reference_plotter():
    cublas, versions, tflops = perf_report.parse_perf_text(LOG)
    assert cublas == 30.12
    assert versions == ["v0", "v1"] and tflops == [32.5, 31.75]


def test_jsonl_table(tmp_path):
    rows = [
        {"gpu": "NVIDIA B200", "sm": 100, "ngpu": 1, "backend": "cuBLAS", "M": 512, "N": 512, "K": 512,
         "inputs": "uniform(-1,1)", "avg_ms": 0.009, "tflops": 30.12, "pct_cublas": 100.0,
         "pct_peak": 1.34, "passed": True, "max_abs_err": 0.0, "max_rel_err": None},
        {"gpu": "NVIDIA B200", "sm": 100, "ngpu": 1, "backend": "VibeGEMM B200 v9", "M": 512,
         "N": 512, "K": 512, "inputs": "uniform(-1,1)", "skipped": True, "ran": False},
    ]
    p = tmp_path / "perf_b200.jsonl"
    p.write_text("".join(json.dumps(r) + "\n" for r in rows))
    table = perf_report.markdown_table(perf_report.load_jsonl(str(p)))
    lines = table.splitlines()
    assert len(lines) == 3 and "| 512×512×512 | uniform(-1,1) | cuBLAS | 30.1 | 100.0 | 1.3 | PASS |" in lines


def test_main_reads_results_dir(tmp_path, capsys):
    (tmp_path / "perf_b200.txt").write_text(LOG)
    assert perf_report.main(["x", str(tmp_path)]) == 0
    out = capsys.readouterr().out
    assert "NVIDIA B200: cuBLAS 30.12 TFLOPS; v0 32.50, v1 31.75" in out
    assert perf_report.main(["x", str(tmp_path / "missing")]) == 1
