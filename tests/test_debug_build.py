"""The checking build libb200fa_debug.so (compiled with -DB200FA_DEBUG).

Its kernels verify, before every copy, that the work item's plan and each
TMA coordinate lie inside the problem (checks 0x80-0x84), that the TMEM
allocation and the aligned shared-memory layout are the expected ones
(0x85), and at exit that every role counted the same key blocks (the
parities of all mbarrier waits derive from those counts).  A violation is
reported in the device status word (B200FA_DEV_BOUNDS / B200FA_DEV_PHASE) and
takes the bounded abort path; no out-of-range access is issued.

CPU: the checking build compiles and exports the whole C ABI.  GPU: it gives
the product build's output bit for bit with a clean status over ragged and
GQA shapes, with and without the causal mask (whose per-item block counts
the exit check then verifies), and the planted out-of-range Q coordinate (B200FA_FLAG_TEST_BOUNDS,
checked but never used for a copy) is caught as B200FA_DEV_BOUNDS at check
0x81 while the product build, which has no checks, ignores the flag.
"""

import ctypes as C

import pytest

from fa_b200 import build, lib


def test_debug_build_exports_the_c_abi():
    path = build.build(debug=True)
    assert path.name == "libb200fa_debug.so" and build.is_current(debug=True)
    so = C.CDLL(str(path), mode=C.RTLD_LOCAL)
    for name in lib.SIGNATURES:
        assert hasattr(so, name), name
    assert "-DB200FA_DEBUG" in (build.BUILD_DIR / "build_debug.json").read_text()
    # Separate artefacts: the product library is not the checking one.
    assert build.build() != path


SHAPES = [(1, 2, 1, 128, 128), (1, 4, 2, 300, 77), (2, 6, 3, 1000, 1029), (1, 12, 1, 4096, 4096)]


@pytest.mark.gpu
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("variant", ["fp16", "fp32"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_debug_build_matches_product_with_clean_status(variant, shape, causal):
    import torch

    from fa_b200.ops import Operator

    B, Hq, Hkv, Nq, Nk = shape
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(11)
    q = torch.randn((B, Hq, Nq, 128), device=dev, generator=g).half()
    k = torch.randn((B, Hkv, Nk, 128), device=dev, generator=g).half()
    v = torch.randn((B, Hkv, Nk, 128), device=dev, generator=g).half()
    prod = Operator(variant)
    dbg = Operator(variant, debug=True)
    a = prod(q, k, v, causal=causal)
    b = dbg(q, k, v, causal=causal)
    torch.cuda.synchronize(dev)
    assert dbg.status(dev)[0] == lib.DEV_OK, dbg.status(dev)
    assert prod.status(dev)[0] == lib.DEV_OK
    assert torch.equal(a, b)


@pytest.mark.gpu
@pytest.mark.parametrize("variant", ["fp16", "fp32"])
def test_planted_bad_coordinate_is_caught_not_issued(variant):
    import torch

    from fa_b200.ops import Operator

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    q = torch.randn((1, 4, 512, 128), device=dev, generator=g).half()
    k = torch.randn((1, 2, 640, 128), device=dev, generator=g).half()
    v = torch.randn((1, 2, 640, 128), device=dev, generator=g).half()
    dbg = Operator(variant, debug=True, timeout_us=200000)
    dbg(q, k, v, flags=lib.FLAG_TEST_BOUNDS)
    torch.cuda.synchronize(dev)
    status, site, cta, _ = dbg.status(dev)
    assert status == lib.DEV_BOUNDS, (status, hex(site))
    assert site & 0xFF == lib.CHECK_SITE + 1 and (site >> 8) & 0xFF == 9, hex(site)  # producer warp, Q check
    # The context stays usable: a clean call after a reset gives the product result.
    dbg.reset_status(dev)
    out = dbg(q, k, v)
    prod = Operator(variant)
    ref = prod(q, k, v, flags=lib.FLAG_TEST_BOUNDS)  # the product build ignores the flag
    torch.cuda.synchronize(dev)
    assert dbg.status(dev)[0] == lib.DEV_OK and prod.status(dev)[0] == lib.DEV_OK
    assert torch.equal(out, ref)


@pytest.mark.gpu
def test_timeline_records_every_role_in_pipeline_order():
    """B200FA_FLAG_TIMELINE (checking build): both CTAs of the first pair
    stamp clock64 at fixed points of their first item's first blocks.  Each
    softmax warp stamps its group's blocks in program order, the issuers,
    the forwarder and the producer theirs; the product build ignores the
    flag and leaves the area untouched."""
    import numpy as np
    import torch

    from fa_b200.ops import Operator

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(9)
    q = torch.randn((1, 12, 8192, 128), device=dev, generator=g).half()
    k = torch.randn((1, 1, 8192, 128), device=dev, generator=g).half()
    v = torch.randn((1, 1, 8192, 128), device=dev, generator=g).half()
    dbg = Operator("fp32", debug=True)
    dbg.workspace(dev).zero_()
    dbg(q, k, v, flags=lib.FLAG_TIMELINE)
    assert dbg.status(dev)[0] == lib.DEV_OK
    t = dbg.timeline(dev).numpy()
    assert t.shape == (2, lib.TIMELINE_ROLES, lib.TIMELINE_BLOCKS, 8)
    n = min(8192 // 128, lib.TIMELINE_BLOCKS)
    order = [0, 7, 1, 2, 3, 4, 5, 6]  # start, scores ready, ref seen, max, published, exps, P stored, P arrived
    for rank in (0, 1):
        for w in range(8):
            for j in range(n):
                e = t[rank, w, j]
                if j % 2 == w // 4:
                    assert np.all(e[order] > 0) and np.all(np.diff(e[order]) >= 0), (rank, w, j, e)
                else:
                    assert np.all(e == 0), (rank, w, j, e)
        tma = t[rank, 9, :n]
        assert np.all(tma[:, :4] > 0) and np.all(np.diff(tma[:, :4], axis=1) >= 0)
    iss = t[0, 8, :n]
    assert np.all(iss[:, 2] <= iss[:, 3]) and np.all(iss[:, 0] <= iss[:, 1])  # S / PV: started before issued
    assert np.all(iss[2:, 4] <= iss[2:, 2])  # S of block j waits for "S free" of block j-2
    assert np.all(iss[:, 5] > 0) and np.all(iss[:, 6] > 0)  # completions watched
    fwd = t[1, 8, :n]
    assert np.all(fwd[:, 5] > 0) and np.all(fwd[:, 5] <= fwd[:, 6])  # K forwarded, then V

    prod = Operator("fp32")
    prod.workspace(dev).zero_()
    prod(q, k, v, flags=lib.FLAG_TIMELINE)
    assert prod.status(dev)[0] == lib.DEV_OK
    assert not prod.timeline(dev).any()
