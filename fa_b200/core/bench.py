"""Benchmark orchestrator (CUDA mirror of the reference core/bench.py).

Phase A (CPU, parallel)  build every selected backend whose driver asks for a
                         compile step, in subprocesses with no visible GPU.
Phase B (GPU, per card)  in one process per case: prepare every backend,
                         build the canonical inputs, one warm call each,
                         profile all backends, then check each backend
                         against the single reference in the same process
                         (backends initialise their own workspace).
Report                   long-format CSV + console table per (case, backend).

Same CLI as the reference (``--backends --cases --list-cases --devices
--iters --logdir --no-check --no-compile --seed --atol --rtol``) with the
NPU specifics ported (``torch.cuda.synchronize``, ``CUDA_VISIBLE_DEVICES``).
Additions: the acceptance check of this build (max-abs <= 2e-3 and
mean-abs <= 2e-4 against the FP32 reference, ``--max-abs/--mean-abs``) on
top of the legacy ``assert_close``, and TFLOPS / %-of-peak columns.
Multi-GPU runs of one case (query blocks sharded over ranks) are driven by
the repository's bench.py under torchrun.
"""

import argparse
import csv
import functools
import json
import os
import subprocess
import sys
from datetime import datetime

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402

from fa_b200.core import profiler, registry, schedule  # noqa: E402
from fa_b200.core.contract import KernelNameError  # noqa: E402
from fa_b200.problem.cases import CASES  # noqa: E402

NOMINAL_PEAK_TFLOPS = 2250.0


def _runner_cmd(*extra):
    return [sys.executable, "-m", "fa_b200.core.runner", *map(str, extra)]


def peak_tflops():
    """Dense FP16/BF16 peak per GPU: MEASURED_PEAKS.json (burst) when present, else nominal."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return NOMINAL_PEAK_TFLOPS


# --------------------------------------------------------------------------- #
# Phase A: parallel compile on the CPU
# --------------------------------------------------------------------------- #
def _compile_task(packed):
    backend, case_index = packed
    env = os.environ.copy()
    env["CUDA_VISIBLE_DEVICES"] = ""
    cmd = _runner_cmd("--backend", backend, "--case-index", case_index, "--mode", "compile")
    r = subprocess.run(cmd, env=env, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    return backend, case_index, r.returncode, r.stdout


def compile_phase(backend_names, case_indices):
    tasks = [(n, i) for n in backend_names if registry.needs_compile(registry.get(n)) for i in case_indices]
    if not tasks:
        return
    print(f">>> Phase A: compiling {len(tasks)} backend/case pairs on CPU...")
    failed = []
    for backend, ci, rc, out in schedule.parallel_compile(tasks, _compile_task):
        print(f"    {backend} {CASES[ci].name}: {'ok' if rc == 0 else f'FAIL(rc={rc})'}")
        if rc != 0:
            print(out)
            failed.append(f"{backend}/{CASES[ci].name}")
    if failed:
        raise RuntimeError(f"Compilation failed for {', '.join(failed)}")


# --------------------------------------------------------------------------- #
# Phase B: one process per case on one GPU
# --------------------------------------------------------------------------- #
def check_output(out, ref_out, atol, rtol, max_abs, mean_abs):
    """(status, max-abs, mean-abs) of a backend's output against the reference's."""
    d = (out.float() - ref_out.float()).abs()
    mx, mean = float(d.max()), float(d.mean())
    try:
        torch.testing.assert_close(out.float(), ref_out.float(), atol=atol, rtol=rtol)
        legacy = True
    except AssertionError:
        legacy = False
    ok = legacy and mx <= max_abs and mean <= mean_abs
    return ("PASS" if ok else "FAIL"), mx, mean


def process_case(case_index, device, *, session_dir, backend_names, ref_name, iters, do_check, seed,
                 atol, rtol, max_abs=2e-3, mean_abs=2e-4):
    os.environ["CUDA_VISIBLE_DEVICES"] = str(device)
    from fa_b200.problem.canonical import build_canonical

    case = CASES[case_index]
    prepared, skipped = {}, set()
    for n in backend_names:
        try:
            prepared[n] = registry.prepare_call(registry.get(n), case)
        except KernelNameError:
            raise
        except Exception as e:  # a backend that cannot load is skipped, not fatal
            print(f"    [skip] {n}: {e}")
            skipped.add(n)
    canonical = build_canonical(case, seed)

    calls = {}
    for n in backend_names:
        if n in skipped:
            continue
        try:
            call = prepared[n](canonical)
            call()
            torch.cuda.synchronize()
            calls[n] = call
        except KernelNameError:
            raise
        except Exception as e:
            print(f"    [skip] {n}: {e}")
            skipped.add(n)

    op_types = {n: registry.get(n).META.op_type for n in backend_names}
    times = profiler.profile_case_us(calls, backend_names, iters=iters, op_types=op_types)

    checks = {}
    if do_check:
        ref_out = None
        for n in sorted(backend_names, key=lambda m: not registry.get(m).META.is_reference):
            meta = registry.get(n).META
            if n in skipped:
                checks[n] = ("ref", 0.0, 0.0) if meta.is_reference else ("ERR", None, None)
                continue
            out = calls[n]().float()
            torch.cuda.synchronize()
            if meta.is_reference:
                ref_out = out
                checks[n] = ("ref", 0.0, 0.0)
            elif ref_out is not None:
                checks[n] = check_output(out, ref_out, atol, rtol, max_abs, mean_abs)
            else:
                checks[n] = ("ERR", None, None)

    peak = peak_tflops()
    ref_us = times.get(ref_name)
    rows = []
    for n in backend_names:
        meta = registry.get(n).META
        us = times.get(n)
        ratio = f"{(us / ref_us) * 100:.1f}%" if (us and ref_us) else "N/A"
        status, mx, mean = checks.get(n, ("skip", None, None))
        tflops = case.flops / (us * 1e-6) / 1e12 if us else None
        rows.append([case.name, n, "ref" if meta.is_reference else "",
                     f"{us:.2f}" if us else "N/A", ratio, status,
                     f"{mx:.5f}" if mx is not None else "N/A",
                     f"{mean:.2e}" if mean is not None else "N/A",
                     f"{tflops:.1f}" if tflops else "N/A",
                     f"{100 * tflops / peak:.1f}%" if tflops else "N/A", 1])
    print(f"[done] {case.name:<24} dev={device} " +
          " ".join(f"{n}={times[n]:.1f}us" if times.get(n) else f"{n}=N/A" for n in backend_names))
    return rows


# --------------------------------------------------------------------------- #
def _default_devices():
    env = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    if env.strip():
        return [int(x) for x in env.split(",") if x.strip()]
    return list(range(max(1, torch.cuda.device_count())))


def _parse_cases(spec):
    spec = spec.strip()
    if spec == "all":
        return list(range(len(CASES)))
    out = []
    for tok in spec.split(","):
        tok = tok.strip()
        if not tok:
            continue
        try:
            i = int(tok)
        except ValueError:
            raise SystemExit(f"--cases: '{tok}' is not an integer index or 'all'")
        if not 0 <= i < len(CASES):
            raise SystemExit(f"--cases: index {i} out of range 0..{len(CASES) - 1}")
        if i not in out:
            out.append(i)
    if not out:
        raise SystemExit("--cases: no valid case indices given")
    return out


HEADERS = ["Case", "Backend", "Ref", "Avg_us", "vs_ref", "Check", "MaxDiff", "MeanDiff", "TFLOPS",
           "pct_peak", "GPUs"]


def main():
    p = argparse.ArgumentParser(description="attention benchmark orchestrator")
    p.add_argument("--backends", type=str, default=None, help="comma-separated backend names (default: all)")
    p.add_argument("--cases", type=str, default="all", help="'all' or comma-separated case indices")
    p.add_argument("--list-cases", action="store_true")
    p.add_argument("--devices", type=str, default=None)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--logdir", type=str, default=os.path.join(ROOT, "results"))
    p.add_argument("--no-check", action="store_true")
    p.add_argument("--no-compile", action="store_true")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--atol", type=float, default=1e-2)
    p.add_argument("--rtol", type=float, default=1e-2)
    p.add_argument("--max-abs", type=float, default=2e-3)
    p.add_argument("--mean-abs", type=float, default=2e-4)
    args = p.parse_args()

    if args.list_cases:
        for i, c in enumerate(CASES):
            print(f"{i:2d}  {c.name}")
        return

    backend_names = args.backends.split(",") if args.backends else registry.all_names()
    for name in backend_names:
        registry.require_attention(registry.get(name))
    ref_name, _ = registry.get_reference()
    if ref_name not in backend_names:
        backend_names = [ref_name] + backend_names
    case_indices = _parse_cases(args.cases)
    devices = [int(x) for x in args.devices.split(",")] if args.devices else _default_devices()

    stamp = datetime.now().strftime("%Y%m%d_%H%M%S")
    label = "all" if args.cases.strip() == "all" else "sel" + "_".join(map(str, case_indices))
    session_dir = os.path.join(args.logdir, f"bench_{label}_{stamp}")
    os.makedirs(session_dir, exist_ok=True)
    print(f">>> backends={backend_names} ref={ref_name}")
    print(f">>> cases: {len(case_indices)}/{len(CASES)} -> indices {case_indices} on devices {devices}")
    print(f">>> session: {session_dir}")

    if not args.no_compile:
        compile_phase(backend_names, case_indices)

    print(f">>> Phase B: {len(case_indices)} cases on {len(devices)} GPUs...")
    worker = functools.partial(process_case, session_dir=session_dir, backend_names=backend_names,
                               ref_name=ref_name, iters=args.iters, do_check=not args.no_check,
                               seed=args.seed, atol=args.atol, rtol=args.rtol,
                               max_abs=args.max_abs, mean_abs=args.mean_abs)
    per_case_rows = schedule.distribute_over_cards(case_indices, devices, worker)

    rows = [r for case_rows in per_case_rows for r in case_rows]
    csv_path = os.path.join(session_dir, "report.csv")
    with open(csv_path, "w", newline="", encoding="utf-8") as f:
        w = csv.writer(f)
        w.writerow(HEADERS)
        w.writerows(rows)
    print("\n" + "  ".join(HEADERS))
    for r in rows:
        print("  ".join(str(x) for x in r))
    print(f"\n[done] report -> {csv_path}")


if __name__ == "__main__":
    main()
