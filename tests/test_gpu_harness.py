"""The reference's harness flow on the GPU, end to end through the plugin
boundary: the CLI entry points a harness user runs, in fresh processes.

* ``python -m fa_b200.core.runner --backend <b> --case-index <i> --mode check``
  (reference core/runner.py:32-72): discovers the backend directory,
  builds, runs it on the canonical inputs and checks it against the
  reference backend; prints ``CHECK ... PASS``.
* ``python -m fa_b200.core.bench --backends ... --cases ... --iters ...``
  (reference core/bench.py:79-158): compile phase, then per case the check
  and the profiled timing of every backend, and the CSV report.
"""

import csv
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _run(args, timeout=600):
    env = dict(os.environ)
    env["PYTHONPATH"] = str(ROOT) + os.pathsep + env.get("PYTHONPATH", "")
    return subprocess.run([sys.executable, "-m", *args], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=timeout)


@pytest.mark.gpu
@pytest.mark.parametrize("backend", ["b200_fa_fp16", "b200_fa_fp32"])
@pytest.mark.parametrize("case_index", [3, 2], ids=["C1", "C3"])
def test_runner_check_passes(backend, case_index):
    from fa_b200.problem.cases import CASES

    res = _run(["fa_b200.core.runner", "--backend", backend, "--case-index", str(case_index), "--mode", "check"])
    assert res.returncode == 0, res.stdout + res.stderr
    line = [x for x in res.stdout.splitlines() if x.startswith("CHECK ")]
    assert line and f"CHECK {CASES[case_index].name} backend={backend} PASS" in line[-1], res.stdout


@pytest.mark.gpu
def test_bench_checks_times_and_reports(tmp_path):
    res = _run(["fa_b200.core.bench", "--backends", "b200_fa_fp16,b200_fa_fp32,torch_fp32_ref", "--cases", "3",
                "--iters", "3", "--devices", "0", "--logdir", str(tmp_path)])
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    reports = list(tmp_path.glob("bench_*/report.csv"))
    assert len(reports) == 1, res.stdout
    with open(reports[0], newline="") as f:
        rows = {r["Backend"]: r for r in csv.DictReader(f)}
    assert set(rows) == {"b200_fa_fp16", "b200_fa_fp32", "torch_fp32_ref"}
    assert rows["torch_fp32_ref"]["Ref"] == "ref"
    for name in ("b200_fa_fp16", "b200_fa_fp32"):
        r = rows[name]
        assert r["Case"] == "B1_S2048_Q12_KV1_D128"
        assert r["Check"] == "PASS", r
        assert float(r["MaxDiff"]) <= 2e-3 and float(r["MeanDiff"]) <= 2e-4, r
        assert float(r["Avg_us"]) > 0 and float(r["TFLOPS"]) > 0, r


@pytest.mark.gpu
def test_vendor_attention_is_checked_and_timed_beside_the_b200_kernels(tmp_path):
    """cuDNN's fused attention (torch SDPA) through the same harness flow:
    checked against the FP32 reference and timed, like the reference
    harness's vendor operator row."""
    res = _run(["fa_b200.core.runner", "--backend", "torch_sdpa", "--case-index", "3", "--mode", "check"])
    assert res.returncode == 0, res.stdout + res.stderr
    res = _run(["fa_b200.core.bench", "--backends", "b200_fa_fp16,torch_sdpa,torch_fp32_ref", "--cases", "3",
                "--iters", "3", "--devices", "0", "--logdir", str(tmp_path)])
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    with open(next(tmp_path.glob("bench_*/report.csv")), newline="") as f:
        rows = {r["Backend"]: r for r in csv.DictReader(f)}
    r = rows["torch_sdpa"]
    assert r["Check"] == "PASS", r
    assert float(r["Avg_us"]) > 0 and float(r["TFLOPS"]) > 0, r
