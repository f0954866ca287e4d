"""ctypes binding of ``libb200fa.so`` (the C ABI of include/b200fa.h).

This module is the Python equivalent of the reference CCE binding's native
half (backends/cce_fa_*/binding.py:7-31: ``CDLL`` of the operator library,
``argtypes``/``restype`` declarations, nonzero status -> ``RuntimeError``).
No torch types cross the boundary: only integers, pointers and a float.

There is no fallback: if the library cannot be built or loaded the calls
raise.
"""

from __future__ import annotations

import ctypes as C
import threading

from . import build as _build

VARIANT_FP16 = 0
VARIANT_FP32 = 1
VARIANTS = {"fp16": VARIANT_FP16, "fp32": VARIANT_FP32}

FLAG_TRACE = 1
FLAG_TEST_WITHHOLD_P = 2
FLAG_TIMELINE = 4
FLAG_CAPTURE = 8
FLAG_TEST_BOUNDS = 16
FLAG_CAUSAL = 32
BLOCK_KEYS = 128

DEV_OK = 0
DEV_TIMEOUT = 1
DEV_BOUNDS = 2
DEV_PHASE = 3
CHECK_SITE = 0x80  # low byte of the status site of a failed check: 0x80 + check number

WS_HEADER_BYTES = 256
WS_TRACE_BYTES = 32
MAX_CTAS = 1024
TIMELINE_BLOCKS = 48
TIMELINE_ROLES = 10
WS_TIMELINE_OFFSET = WS_HEADER_BYTES + WS_TRACE_BYTES * MAX_CTAS
WS_TIMELINE_BYTES = 2 * TIMELINE_ROLES * TIMELINE_BLOCKS * 8 * 8
WS_BYTES = WS_TIMELINE_OFFSET + WS_TIMELINE_BYTES

# name -> (restype, argtypes); the exported C ABI, one entry per declaration
# of include/b200fa.h.
_i64, _i32, _u32, _u64, _p, _f = C.c_int64, C.c_int32, C.c_uint32, C.c_uint64, C.c_void_p, C.c_float


class Options(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("flags", C.c_uint32),
                ("timeout_us", C.c_uint32), ("max_ctas", C.c_int32),
                ("capture", C.c_void_p), ("capture_bytes", C.c_uint64)]


SIGNATURES = {
    "b200fa_num_units": (_i64, [_i64, _i64, _i64]),
    "b200fa_partition": (C.c_int, [_i64, _i32, _i32, C.POINTER(_i64), C.POINTER(_i64)]),
    "b200fa_workspace_size": (_i64, [_i64, _i64, _i64, _i64, _i64, _i64, _i32]),
    "b200fa_fwd": (C.c_int, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _f, _i32,
                             _i64, _i64, _p, _u64, _p]),
    "b200fa_fwd_ex": (C.c_int, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _f, _i32,
                                _i64, _i64, _p, _u64, _p, C.POINTER(Options)]),
    "b200fa_read_status": (C.c_int, [_p, _p, C.POINTER(_u32)]),
    "b200fa_reset_status": (C.c_int, [_p, _p]),
    "b200fa_kernel_name": (C.c_char_p, [_i32]),
    "b200fa_plan_item": (_i64, [_i64, _i64, _i64, _i64, _i64, _i64,
                                C.POINTER(_i64), C.POINTER(_i64), C.POINTER(_i64)]),
    "b200fa_capture_bytes": (_i64, [_i64, _i64, _i64, _i64]),
    "b200fa_last_error_string": (C.c_char_p, []),
    "b200fa_version": (C.c_char_p, []),
    "b200fa_test_exp2": (C.c_int, [_p, _p, _p, _i64, _p]),
    "b200fa_fwd_noalloc": (C.c_int, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _f, _i32,
                                     _i64, _i64, _p, C.POINTER(Options), C.POINTER(_p)]),
}

_lock = threading.Lock()
_libs: dict[bool, C.CDLL] = {}  # debug -> bound library


class B200FAError(RuntimeError):
    """A nonzero status from libb200fa (negative: validation, positive: CUDA)."""

    def __init__(self, where, status, message):
        super().__init__(f"{where}: status {status}: {message}")
        self.status = status


def load(build_if_needed: bool = True, debug: bool = False) -> C.CDLL:
    """Load (building first if the sources changed) and bind the library;
    ``debug`` selects the checking build libb200fa_debug.so."""
    with _lock:
        lib = _libs.get(debug)
        if lib is not None:
            return lib
        if build_if_needed:
            path = _build.build(debug=debug)
        else:
            path = _build.DEBUG_LIB_PATH if debug else _build.LIB_PATH
            if not path.is_file():
                raise FileNotFoundError(f"{path} is not built; run fa_b200.build.build(debug={debug})")
        lib = C.CDLL(str(path), mode=C.RTLD_LOCAL)
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _libs[debug] = lib
        return lib


def last_error(debug: bool = False) -> str:
    return load(debug=debug).b200fa_last_error_string().decode()


def check(status: int, where: str, debug: bool = False) -> None:
    if status != 0:
        raise B200FAError(where, status, last_error(debug))


def num_units(B: int, Hq: int, Nq: int) -> int:
    n = load().b200fa_num_units(B, Hq, Nq)
    if n < 0:
        check(int(n), "b200fa_num_units")
    return int(n)


def partition(total: int, parts: int, index: int) -> tuple[int, int]:
    b, e = _i64(), _i64()
    check(load().b200fa_partition(total, parts, index, C.byref(b), C.byref(e)), "b200fa_partition")
    return b.value, e.value


def workspace_size(B, Hq, Hkv, Nq, Nk, D, variant) -> int:
    n = load().b200fa_workspace_size(B, Hq, Hkv, Nq, Nk, D, variant)
    if n < 0:
        check(int(n), "b200fa_workspace_size")
    return int(n)


def plan_items(B, Hq, Nq, unit_begin, unit_end) -> list[tuple[int, int, int]]:
    """Host-side work-item plan of a unit range: [(bh, first q-block, count)]."""
    lib = load()
    bh, qb, cnt = _i64(), _i64(), _i64()
    n = lib.b200fa_plan_item(B, Hq, Nq, unit_begin, unit_end, -1, None, None, None)
    if n < 0:
        check(int(n), "b200fa_plan_item")
    out = []
    for i in range(n):
        lib.b200fa_plan_item(B, Hq, Nq, unit_begin, unit_end, i, C.byref(bh), C.byref(qb), C.byref(cnt))
        out.append((bh.value, qb.value, cnt.value))
    return out


def kernel_name(variant: int) -> str:
    name = load().b200fa_kernel_name(variant)
    if name is None:
        raise ValueError(f"unknown variant {variant}")
    return name.decode()


def fwd(q_ptr, k_ptr, v_ptr, o_ptr, B, Hq, Hkv, Nq, Nk, D, scale, variant,
        unit_begin, unit_end, ws_ptr, ws_bytes, stream, *, flags=0, timeout_us=0, max_ctas=0,
        capture_ptr=None, capture_bytes=0, debug=False):
    """Raw pointer call of b200fa_fwd_ex (``debug``: of the checking build);
    raises B200FAError on a nonzero status."""
    opts = Options(C.sizeof(Options), flags, timeout_us, max_ctas, capture_ptr, capture_bytes)
    status = load(debug=debug).b200fa_fwd_ex(q_ptr, k_ptr, v_ptr, o_ptr, B, Hq, Hkv, Nq, Nk, D, scale, variant,
                                             unit_begin, unit_end, ws_ptr, ws_bytes, stream, C.byref(opts))
    check(status, "b200fa_fwd", debug)


def capture_bytes(B, Hq, Nq, Nk) -> int:
    """Size of the B200FA_FLAG_CAPTURE buffer (four FP32 planes)."""
    n = int(load().b200fa_capture_bytes(B, Hq, Nq, Nk))
    check(n if n < 0 else 0, "b200fa_capture_bytes")
    return n


def read_status(ws_ptr, stream) -> tuple[int, int, int, int]:
    out = (_u32 * 4)()
    check(load().b200fa_read_status(ws_ptr, stream, out), "b200fa_read_status")
    return tuple(int(x) for x in out)


def reset_status(ws_ptr, stream) -> None:
    check(load().b200fa_reset_status(ws_ptr, stream), "b200fa_reset_status")
