"""Generate the golden vectors that pin the oracle to the reference's own code.

Run where a checkout of the reference (platelett/fa) is readable, giving
its root directory (or setting $FA_REFERENCE):

    python tests/golden/make_golden.py <reference checkout>

It executes three pieces of the reference and records their results:

1. ``ref_flash_attn`` (backends/expert_v2/impl_tl.py:701-717), the reference's
   FP32 formula of the operator.  Its module imports the Ascend TileLang
   toolchain at top level, which does not import here, so the function's
   definition is lifted out of the source file with ``ast`` and executed on
   its own with ``torch`` as its only global.  Its outputs (FP16 O) for
   seeded small inputs go to ``attention_vectors.npz``.
2. ``Case`` and ``CASES`` (problem/cases.py:13-39): names, scale and group
   size of the reference's cases plus the added benchmark configurations go to
   ``cases.json``.
3. ``build_canonical`` (problem/canonical.py:18-28), run with the NPU device
   redirected to the CPU, on small cases: a checksum of its q/k/v goes to
   ``cases.json`` so the mirror's canonical inputs are pinned to the same
   seed/shape/order semantics.

Nothing here is read at run time on the GPU host; the tests read only the
files this script writes.
"""

from __future__ import annotations

import ast
import importlib.util
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REF = None  # the reference checkout; set by main() from argv[1] or $FA_REFERENCE

# (B, Hq, Hkv, Nq, Nk, seed, input scale): small cases covering GQA groupings,
# MHA, query/key tails (N % 128 != 0), Nq != Nk, a single key block and
# large-magnitude inputs.
VECTOR_CASES = [
    (1, 2, 1, 256, 256, 0, 1.0),
    (1, 4, 2, 128, 384, 1, 1.0),
    (2, 1, 1, 200, 200, 2, 1.0),
    (1, 3, 1, 130, 333, 3, 1.0),
    (1, 2, 1, 64, 100, 4, 1.0),
    (1, 1, 1, 256, 512, 5, 4.0),
]


def load_ref_flash_attn():
    src_path = REF / "backends/expert_v2/impl_tl.py"
    tree = ast.parse(src_path.read_text())
    fn = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "ref_flash_attn"]
    if len(fn) != 1:
        raise RuntimeError("ref_flash_attn not found in the reference")
    module = ast.Module(body=fn, type_ignores=[])
    namespace = {"torch": torch}
    exec(compile(module, str(src_path), "exec"), namespace)
    return namespace["ref_flash_attn"], fn[0].lineno, fn[0].end_lineno


def load_module(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def seeded_inputs(B, Hq, Hkv, Nq, Nk, seed, mag):
    """q, k, v drawn like problem/canonical.py (seed, randn FP16, q then k then v)."""
    torch.manual_seed(seed)
    q = torch.randn((B, Hq, Nq, 128), dtype=torch.float16)
    k = torch.randn((B, Hkv, Nk, 128), dtype=torch.float16)
    v = torch.randn((B, Hkv, Nk, 128), dtype=torch.float16)
    if mag != 1.0:
        q = (q.float() * mag).half()
        k = (k.float() * mag).half()
    return q, k, v


def make_vectors():
    ref_fn, lo, hi = load_ref_flash_attn()
    arrays = {}
    meta = []
    for i, (B, Hq, Hkv, Nq, Nk, seed, mag) in enumerate(VECTOR_CASES):
        q, k, v = seeded_inputs(B, Hq, Hkv, Nq, Nk, seed, mag)
        o = ref_fn(q, k, v)
        assert o.dtype == torch.float16 and o.shape == q.shape
        arrays[f"q{i}"] = q.numpy()
        arrays[f"k{i}"] = k.numpy()
        arrays[f"v{i}"] = v.numpy()
        arrays[f"o{i}"] = o.numpy()
        meta.append({"B": B, "Hq": Hq, "Hkv": Hkv, "Nq": Nq, "Nk": Nk, "seed": seed, "input_scale": mag})
    np.savez_compressed(HERE / "attention_vectors.npz", **arrays)
    return meta, f"backends/expert_v2/impl_tl.py:{lo}-{hi}"


def make_cases():
    cases_mod = load_module("ref_problem_cases", REF / "problem/cases.py")
    ref_cases = []
    for c in cases_mod.CASES:
        ref_cases.append({"batch": c.batch, "seq_len": c.seq_len, "heads_q": c.heads_q,
                          "heads_kv": c.heads_kv, "dim": c.dim, "name": c.name,
                          "scale": c.scale, "group_size": c.group_size})
    extra = []
    for dims in [(1, 2048, 12, 1, 128), (4, 8192, 32, 8, 128)]:
        c = cases_mod.Case(*dims)
        extra.append({"batch": c.batch, "seq_len": c.seq_len, "heads_q": c.heads_q,
                      "heads_kv": c.heads_kv, "dim": c.dim, "name": c.name,
                      "scale": c.scale, "group_size": c.group_size})

    # build_canonical with the NPU default device redirected to the CPU.
    canon = load_module("ref_problem_canonical", REF / "problem/canonical.py")
    real_set = torch.set_default_device
    checks = []
    try:
        torch.set_default_device = lambda dev: real_set("cpu")
        for dims, seed in [((1, 256, 2, 1, 128), 0), ((2, 130, 4, 2, 128), 7)]:
            c = cases_mod.Case(*dims)
            t = canon.build_canonical(c, seed)
            checks.append({"case": list(dims), "seed": seed,
                           **{f"{n}_sum": float(t[n].double().sum()) for n in ("q", "k", "v")},
                           **{f"{n}_head": [float(x) for x in t[n].flatten()[:4]] for n in ("q", "k", "v")},
                           **{f"{n}_shape": list(t[n].shape) for n in ("q", "k", "v")}})
    finally:
        real_set("cpu")
        torch.set_default_device = real_set
    return ref_cases, extra, checks


def main(argv=None):
    global REF
    argv = sys.argv[1:] if argv is None else argv
    root = argv[0] if argv else os.environ.get("FA_REFERENCE")
    if not root:
        raise SystemExit("usage: make_golden.py <reference checkout>  (or set FA_REFERENCE)")
    REF = Path(root)
    if not (REF / "problem" / "cases.py").is_file():
        raise SystemExit(f"{REF} is not a checkout of the reference (no problem/cases.py)")
    meta, ref_lines = make_vectors()
    ref_cases, extra, canon_checks = make_cases()
    (HERE / "cases.json").write_text(json.dumps({
        "generator": "tests/golden/make_golden.py",
        "torch": torch.__version__,
        "ref_flash_attn": ref_lines,
        "vectors": meta,
        "reference_cases": ref_cases,
        "baseline_cases": extra,
        "canonical_checks": canon_checks,
    }, indent=1))
    print(f"wrote {len(meta)} vectors and {len(ref_cases) + len(extra)} cases")


if __name__ == "__main__":
    sys.exit(main())
