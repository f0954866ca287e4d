"""Single (backend x case) execution, run as an isolated subprocess.

Mirror of the reference core/runner.py:

  compile : build the backend through its driver; no GPU is touched.
  check   : run the backend and the reference once on the canonical inputs
            and compare (legacy ``assert_close(atol, rtol)`` plus this
            build's max-abs/mean-abs bar).  A fresh process gives a clean
            device.

Prints ``COMPILE <backend> <case> done`` or
``CHECK <case> backend=<b> PASS|FAIL max_abs_diff=... mean_abs_diff=...``.
"""

import argparse
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def _parse_args(argv=None):
    p = argparse.ArgumentParser(description="single runner")
    p.add_argument("--backend", required=True)
    p.add_argument("--case-index", type=int, required=True)
    p.add_argument("--mode", choices=("compile", "check"), default="check")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--atol", type=float, default=1e-2)
    p.add_argument("--rtol", type=float, default=1e-2)
    p.add_argument("--max-abs", type=float, default=2e-3)
    p.add_argument("--mean-abs", type=float, default=2e-4)
    return p.parse_args(argv)


def main(argv=None):
    args = _parse_args(argv)

    from fa_b200.core import registry
    from fa_b200.problem.cases import CASES

    case = CASES[args.case_index]
    spec = registry.get(args.backend)
    registry.require_attention(spec)
    meta = spec.META
    driver = registry.driver_for(meta)

    if args.mode == "compile":
        driver.compile(spec, case)
        print(f"COMPILE {args.backend} {case.name} done")
        return 0

    import torch

    from fa_b200.core.bench import check_output
    from fa_b200.problem.canonical import build_canonical

    bind = registry.prepare_call(spec, case)
    if not meta.is_reference:
        _, ref_spec = registry.get_reference()
        ref_bind = registry.prepare_call(ref_spec, case)
    canonical = build_canonical(case, args.seed)
    out = bind(canonical)().float()

    if meta.is_reference:
        print(f"CHECK {case.name} backend={args.backend} PASS max_abs_diff=0.00000 (self)")
        return 0

    ref_out = ref_bind(canonical)().float()
    torch.cuda.synchronize()
    status, mx, mean = check_output(out, ref_out, args.atol, args.rtol, args.max_abs, args.mean_abs)
    print(f"CHECK {case.name} backend={args.backend} {status} max_abs_diff={mx:.5f} "
          f"mean_abs_diff={mean:.2e} (atol={args.atol}, rtol={args.rtol}, "
          f"max_abs<={args.max_abs}, mean_abs<={args.mean_abs})")
    return 0 if status == "PASS" else 1


if __name__ == "__main__":
    sys.exit(main())
