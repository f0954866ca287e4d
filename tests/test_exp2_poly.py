"""The FMA-pipe exp2 of the softmax (``exp2_poly2`` in fa_kernel.cuh).

2^x = 2^n * p(f) with n = round(x), f = x - n in [-1/2, 1/2] (Cody-Waite
split, n inserted into the exponent field with an integer add) and p the
degree-3 minimax polynomial fitted by fa_b200/csrc/fit_exp2_poly.py (Remez
exchange on the relative error).  x is clamped at -120 first, so masked keys
(x = -inf) give 2^-120, which is 0 in FP16 and negligible in a row sum.

CPU tests: the fit reproduces the constants compiled into the kernel, its
relative error is within the stated 7.5e-5, and a float32 emulation of the
device function's steps meets that bound over [-130, 8] (the range the
softmax feeds it: scores minus a reference maximum that is exceeded by at
most 2^8) including -inf.  GPU test: the device function itself, through
the library's test hook b200fa_test_exp2, against float64 exp2 over the
same range.
"""

import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
KERNEL = ROOT / "fa_b200" / "csrc" / "fa_kernel.cuh"
REL_BOUND = 7.5e-5          # the fit's stated relative error
F32_SLACK = 4 * 2.0 ** -24  # float32 rounding of the Horner steps and the final product
CLAMP = -120.0


def _kernel_constants():
    text = KERNEL.read_text()
    found = dict(re.findall(r"kExp2C(\d) = ([-+0-9.eE]+)f;", text))
    return np.array([float(found[str(i)]) for i in range(4)], dtype=np.float32)


def _inputs():
    x = np.concatenate([np.linspace(-130.0, 8.0, 200001), np.arange(-130, 9, dtype=np.float64),
                        np.arange(-130, 8, dtype=np.float64) + 0.5, [-np.inf, -120.0, -119.5, 0.0, 8.0]])
    return x.astype(np.float32)


def _fma32(a, b, c):
    """float32 fused multiply-add: the product is exact in float64, one rounding of the sum."""
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def emulate_exp2_poly(x: np.ndarray, coef: np.ndarray) -> np.ndarray:
    """The device function's steps in float32 (fa_kernel.cuh exp2_poly2)."""
    x = x.astype(np.float32)
    xc = np.maximum(x, np.float32(CLAMP))
    r = (xc + np.float32(12582912.0)).astype(np.float32)          # 1.5 * 2^23: round to integer
    nf = (r + np.float32(-12582912.0)).astype(np.float32)
    f = _fma32(nf, np.float32(-1.0) * np.ones_like(nf), xc)
    c0, c1, c2, c3 = (np.full_like(f, c) for c in coef)
    q = _fma32(c3, f, c2)
    q = _fma32(q, f, c1)
    q = _fma32(q, f, c0)
    bits = (r.view(np.uint32).astype(np.uint64) * (1 << 23) + q.view(np.uint32).astype(np.uint64)) & 0xFFFFFFFF
    return bits.astype(np.uint32).view(np.float32)


def _check_against_exp2(x, y):
    x64 = x.astype(np.float64)
    exact = np.exp2(np.maximum(x64, CLAMP))  # the clamp is part of the contract
    rel = np.abs(y.astype(np.float64) / exact - 1.0)
    assert np.all(np.isfinite(y))
    assert float(rel.max()) <= REL_BOUND + F32_SLACK, float(rel.max())
    below = x64 <= CLAMP
    assert np.all(y[below] <= np.float32(2.0 ** -120 * (1 + REL_BOUND)))
    return float(rel.max())


def test_fit_reproduces_kernel_constants():
    import importlib.util

    spec = importlib.util.spec_from_file_location("fit_exp2_poly", ROOT / "fa_b200" / "csrc" / "fit_exp2_poly.py")
    fit = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(fit)
    coef, err = fit.remez()
    assert err <= REL_BOUND
    kc = _kernel_constants()
    np.testing.assert_array_equal(coef.astype(np.float32), kc)
    grid = np.linspace(-0.5, 0.5, 100001)
    assert float(np.max(np.abs(fit.rel_error(kc.astype(np.float64), grid)))) <= REL_BOUND


def test_emulated_device_steps_meet_the_bound():
    x = _inputs()
    y = emulate_exp2_poly(x, _kernel_constants())
    worst = _check_against_exp2(x, y)
    assert worst > 1e-5  # the polynomial's error, not a trivially exact path
    assert y[np.isneginf(x)][0] == np.float32(2.0 ** -120 * float(_kernel_constants()[0]))


@pytest.mark.gpu
def test_device_exp2_poly_matches_exp2():
    import torch

    from fa_b200 import lib

    so = lib.load()
    x = _inputs()
    n = x.size
    dev = torch.device("cuda", 0)
    xd = torch.from_numpy(x).to(dev)
    poly = torch.full_like(xd, float("nan"))
    mufu = torch.full_like(xd, float("nan"))
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = so.b200fa_test_exp2(C.c_void_p(xd.data_ptr()), C.c_void_p(poly.data_ptr()), C.c_void_p(mufu.data_ptr()),
                             C.c_int64(n), C.c_void_p(stream))
    assert rc == 0, lib.last_error()
    torch.cuda.synchronize(dev)
    y = poly.cpu().numpy()
    _check_against_exp2(x, y)
    # The device result is the emulated one up to the FMA's single rounding.
    emu = emulate_exp2_poly(x, _kernel_constants())
    assert float(np.max(np.abs(y.astype(np.float64) / emu - 1.0))) <= 2.0 ** -22
    # MUFU ex2.approx over the range where it is not flushed: FP16-grade at worst.
    m = mufu.cpu().numpy().astype(np.float64)
    ok = x >= -126
    assert float(np.max(np.abs(m[ok] / np.exp2(x[ok].astype(np.float64)) - 1.0))) <= 1e-6
    assert m[np.isneginf(x)][0] == 0.0
