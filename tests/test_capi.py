"""The C ABI library on the CPU: it loads without a GPU, exports every symbol
include/b200fa.h declares, and its host logic (validation, partition,
work-item plan) behaves as specified.  No compute call is made."""

import ctypes as C
import re
from pathlib import Path

import pytest

from fa_b200 import lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "b200fa.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b200fa_[a-z_0-9]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    so = lib.load()
    names = declared_functions()
    assert len(names) >= 10
    for name in names:
        assert hasattr(so, name), name
        assert name in lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_kernel_names():
    assert lib.load().b200fa_version().decode().startswith("b200fa")
    assert lib.kernel_name(lib.VARIANT_FP16) == "b200_fa_fp16_kernel"
    assert lib.kernel_name(lib.VARIANT_FP32) == "b200_fa_fp32_kernel"
    with pytest.raises(ValueError):
        lib.kernel_name(7)


def _fwd(**kw):
    args = dict(q=16, k=16, v=16, o=16, B=1, Hq=2, Hkv=1, Nq=256, Nk=256, D=128, scale=0.088,
                variant=0, ub=0, ue=4, ws=256, ws_bytes=1 << 20)
    args.update(kw)
    return lib.load().b200fa_fwd(args["q"], args["k"], args["v"], args["o"], args["B"], args["Hq"],
                                 args["Hkv"], args["Nq"], args["Nk"], args["D"], args["scale"],
                                 args["variant"], args["ub"], args["ue"], args["ws"],
                                 args["ws_bytes"], None)


@pytest.mark.parametrize("kw,code", [
    (dict(q=None), -1),
    (dict(D=64), -2),
    (dict(Nq=0), -3),
    (dict(B=-1), -3),
    (dict(Hq=3, Hkv=2), -4),
    (dict(Nk=2 ** 31), -5),
    (dict(ue=5), -6),
    (dict(ub=3, ue=2), -6),
    (dict(q=17), -7),
    (dict(ws=None), -8),
    (dict(ws=260), -8),
    (dict(ws_bytes=255), -8),
    (dict(variant=2), -9),
    (dict(scale=0.0), -10),
    (dict(scale=float("nan")), -10),
])
def test_validation_codes_without_gpu(kw, code):
    # Validation precedes every CUDA call, so these run on a CPU-only host.
    assert _fwd(**kw) == code
    assert lib.last_error() != ""


def test_empty_range_is_a_noop():
    assert _fwd(ub=2, ue=2) == 0


def test_workspace_size_and_num_units():
    assert lib.num_units(2, 12, 131072) == 24576
    assert lib.num_units(1, 3, 130) == 6
    n = lib.workspace_size(1, 2, 1, 256, 256, 128, 0)
    assert n == lib.WS_BYTES == lib.WS_TIMELINE_OFFSET + lib.WS_TIMELINE_BYTES
    with pytest.raises(lib.B200FAError):
        lib.workspace_size(1, 2, 1, 256, 256, 64, 0)


@pytest.mark.parametrize("total,parts", [(24576, 8), (10, 3), (3, 8), (0, 2), (7, 1)])
def test_partition_contiguous(total, parts):
    from fa_b200 import shard

    spans = [lib.partition(total, parts, i) for i in range(parts)]
    assert spans[0][0] == 0 and spans[-1][1] == total
    for (b0, e0), (b1, e1) in zip(spans, spans[1:]):
        assert e0 == b1
    sizes = [e - b for b, e in spans]
    assert max(sizes) - min(sizes) <= 1 and sizes == sorted(sizes, reverse=True)
    assert spans == [shard.partition(total, parts, i) for i in range(parts)]


@pytest.mark.parametrize("B,Hq,Nq", [(1, 2, 300), (2, 3, 128), (1, 1, 64), (2, 12, 2048), (1, 5, 1000)])
def test_work_plan_covers_every_unit_once(B, Hq, Nq):
    nqb = -(-Nq // 128)
    units = B * Hq * nqb
    for ub, ue in [(0, units), (1, units), (0, units - 1), (units // 3, 2 * units // 3 + 1), (2, 3)]:
        if not 0 <= ub <= ue <= units:
            continue
        seen = []
        for bh, qb, cnt in lib.plan_items(B, Hq, Nq, ub, ue):
            assert 1 <= cnt <= 2 and 0 <= qb and qb + cnt <= nqb
            seen.extend(bh * nqb + qb + i for i in range(cnt))
        assert seen == list(range(ub, ue))


def test_plan_rejects_bad_range():
    with pytest.raises(lib.B200FAError):
        lib.plan_items(1, 2, 256, 0, 99)


def test_status_calls_reject_null():
    out = (C.c_uint32 * 4)()
    assert lib.load().b200fa_read_status(None, None, out) == -1
    assert lib.load().b200fa_reset_status(None, None) == -1


def _fwd_ex(flags, capture, capture_bytes):
    opts = lib.Options(C.sizeof(lib.Options), flags, 0, 0, capture, capture_bytes)
    return lib.load().b200fa_fwd_ex(16, 16, 16, 16, 1, 2, 1, 300, 1000, 128, 0.088, 0, 0, 6,
                                    256, 1 << 20, None, C.byref(opts))


def test_capture_size_and_validation_without_gpu():
    # four FP32 planes + the 128-float O plane per (b*Hq+hq, key block, query row)
    need = lib.capture_bytes(1, 2, 300, 1000)
    assert need == 528 * 2 * -(-1000 // lib.BLOCK_KEYS) * 300
    with pytest.raises(lib.B200FAError):
        lib.capture_bytes(0, 2, 300, 1000)
    assert _fwd_ex(lib.FLAG_CAPTURE, None, need) == -11      # no buffer
    assert _fwd_ex(lib.FLAG_CAPTURE, 4096 + 4, need) == -11  # not 16-byte aligned
    assert _fwd_ex(lib.FLAG_CAPTURE, 4096, need - 1) == -11  # too small
    assert "capture" in lib.last_error().lower()
    # the legacy 16-byte options layout (no capture fields) is still accepted
    legacy = lib.Options(16, 0, 0, 0, None, 0)
    assert lib.load().b200fa_fwd_ex(16, 16, 16, 16, 1, 2, 1, 300, 1000, 128, 0.088, 0, 2, 2,
                                    256, 1 << 20, None, C.byref(legacy)) == 0


def test_python_constants_match_the_header():
    """fa_b200/lib.py restates the header's #defines (flags, status codes,
    workspace layout): they must agree, or a Python caller would pass the
    wrong bits."""
    import re
    from pathlib import Path

    text = (Path(__file__).resolve().parents[1] / "include" / "b200fa.h").read_text()
    defs = dict(re.findall(r"#define\s+(B200FA_\w+)\s+([0-9]+)u?\b", text))
    pairs = {
        "B200FA_FLAG_TRACE": lib.FLAG_TRACE,
        "B200FA_FLAG_TEST_WITHHOLD_P": lib.FLAG_TEST_WITHHOLD_P,
        "B200FA_FLAG_TIMELINE": lib.FLAG_TIMELINE,
        "B200FA_FLAG_CAPTURE": lib.FLAG_CAPTURE,
        "B200FA_FLAG_TEST_BOUNDS": lib.FLAG_TEST_BOUNDS,
        "B200FA_FLAG_CAUSAL": lib.FLAG_CAUSAL,
        "B200FA_BLOCK_KEYS": lib.BLOCK_KEYS,
        "B200FA_DEV_OK": lib.DEV_OK,
        "B200FA_DEV_TIMEOUT": lib.DEV_TIMEOUT,
        "B200FA_DEV_BOUNDS": lib.DEV_BOUNDS,
        "B200FA_DEV_PHASE": lib.DEV_PHASE,
        "B200FA_WS_HEADER_BYTES": lib.WS_HEADER_BYTES,
        "B200FA_WS_TRACE_BYTES": lib.WS_TRACE_BYTES,
        "B200FA_MAX_CTAS": lib.MAX_CTAS,
        "B200FA_TIMELINE_BLOCKS": lib.TIMELINE_BLOCKS,
        "B200FA_TIMELINE_ROLES": lib.TIMELINE_ROLES,
        "B200FA_VARIANT_FP16": lib.VARIANT_FP16,
        "B200FA_VARIANT_FP32": lib.VARIANT_FP32,
    }
    for name, value in pairs.items():
        assert int(defs[name]) == value, name
    assert lib.WS_TIMELINE_BYTES == 2 * lib.TIMELINE_ROLES * lib.TIMELINE_BLOCKS * 8 * 8
