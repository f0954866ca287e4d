"""bench.py's library_baseline leg is a reference point only: when the
vendor's fused attention cannot run (here: no GPU), it reports why instead
of failing the bench."""

import importlib.util
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]


def _bench_module():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_library_baseline_reports_unavailable_without_a_gpu():
    if torch.cuda.is_available():
        return  # the GPU path is exercised by bench.py runs themselves
    bench = _bench_module()
    q = torch.zeros(1, 2, 8, 128, dtype=torch.float16)
    k = torch.zeros(1, 1, 8, 128, dtype=torch.float16)
    res = bench.library_baseline(q, k, k, group=2, flops=4 * 2 * 8 * 8 * 128, reps=1)
    assert set(res) == {"unavailable"} and res["unavailable"], res
