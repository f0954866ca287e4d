"""Size-independent properties of the GPU path, up to the full benchmark sizes.

* shard consistency: running the unit grid as N contiguous shards (the
  multi-GPU split, emulated on one GPU) gives O bit-identical to one call,
  and rows outside a shard are not written;
* determinism: two calls give bit-identical O;
* convexity: every output row is a convex combination of V rows, so it lies
  within [min V, max V] column-wise;
* sampled rows of the full-size cases against the FP32 oracle;
* golden vectors (the reference's own ref_flash_attn outputs) through the
  CUDA path;
* per-CTA trace records of the persistent grid.
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.attention_ref import attention_rows_fp32, errors

GOLDEN = Path(__file__).resolve().parent / "golden"


def _inputs(B, Hq, Hkv, N, seed=0, dev="cuda"):
    torch.manual_seed(seed)
    q = torch.randn((B, Hq, N, 128), dtype=torch.float16, device=dev)
    k = torch.randn((B, Hkv, N, 128), dtype=torch.float16, device=dev)
    v = torch.randn((B, Hkv, N, 128), dtype=torch.float16, device=dev)
    return q, k, v


@pytest.mark.gpu
@pytest.mark.parametrize("variant", ["fp16", "fp32"])
@pytest.mark.parametrize("shape,world", [((1, 3, 1, 1000), 2), ((2, 12, 1, 2048), 8), ((1, 4, 2, 384), 3)])
def test_shards_equal_whole_and_leave_other_rows(variant, shape, world):
    from fa_b200 import shard
    from fa_b200.ops import Operator

    B, Hq, Hkv, N = shape
    q, k, v = _inputs(*shape)
    op = Operator(variant)
    whole = op(q, k, v)
    sharded = torch.full_like(q, float("nan"))
    for r in range(world):
        (ub, ue), (r0, r1) = shard.shard_rows(B, Hq, N, world, r)
        probe = torch.full_like(q, float("nan"))
        op(q, k, v, out=probe, unit_range=(ub, ue))
        pf = probe.view(-1, 128)
        assert torch.isnan(pf[:r0]).all() and torch.isnan(pf[r1:]).all()
        sharded.view(-1, 128)[r0:r1] = pf[r0:r1]
    assert torch.equal(sharded, whole)


@pytest.mark.gpu
@pytest.mark.parametrize("variant", ["fp16", "fp32"])
def test_deterministic(variant):
    from fa_b200.ops import Operator

    q, k, v = _inputs(1, 12, 1, 4096, seed=1)
    op = Operator(variant)
    a = op(q, k, v).clone()
    b = op(q, k, v)
    assert torch.equal(a, b)


@pytest.mark.gpu
@pytest.mark.parametrize("variant", ["fp16", "fp32"])
@pytest.mark.parametrize("shape", [(4, 32, 8, 8192), (2, 12, 1, 131072)], ids=["C2", "C5"])
def test_full_size_sampled_rows_and_convexity(variant, shape):
    from fa_b200.ops import Operator

    B, Hq, Hkv, N = shape
    q, k, v = _inputs(*shape, seed=0)
    out = Operator(variant)(q, k, v)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    G = Hq // Hkv
    # Convexity, column-wise per head.
    for b in range(B):
        for kvh in range(Hkv):
            vmin = v[b, kvh].amin(0).float()
            vmax = v[b, kvh].amax(0).float()
            o = out[b, kvh * G:(kvh + 1) * G].float()
            assert (o >= vmin - 1e-3).all() and (o <= vmax + 1e-3).all()
    # Sampled rows (first/last rows, block edges, random) against the FP32 oracle.
    gen = torch.Generator().manual_seed(7)
    picks = [[0, 0, 0], [B - 1, Hq - 1, N - 1], [0, Hq // 2, 127], [B - 1, 0, 128], [0, 1, N // 2]]
    for _ in range(11):
        picks.append([int(torch.randint(B, (1,), generator=gen)), int(torch.randint(Hq, (1,), generator=gen)),
                      int(torch.randint(N, (1,), generator=gen))])
    rows = torch.tensor(picks)
    ref = attention_rows_fp32(q, k, v, rows.to(q.device))
    got = torch.stack([out[b, h, r] for b, h, r in picks]).float()
    mx, mean = errors(got, ref)
    assert mx <= 2e-3 and mean <= 2e-4, (mx, mean)


@pytest.mark.gpu
@pytest.mark.parametrize("variant", ["fp16", "fp32"])
def test_golden_vectors_through_cuda(variant):
    from fa_b200.ops import Operator

    meta = json.loads((GOLDEN / "cases.json").read_text())
    vec = np.load(GOLDEN / "attention_vectors.npz")
    op = Operator(variant)
    for i, m in enumerate(meta["vectors"]):
        q, k, v, o = (torch.from_numpy(vec[f"{n}{i}"]).cuda() for n in "qkvo")
        out = op(q, k, v)
        mx, mean = errors(out, o)
        # Golden O is the reference's FP32 result rounded to FP16 (half-ulp
        # <= 5e-4 at |O| < 1): the bar is the acceptance bar plus that rounding.
        lim = 2.5e-3 if m["input_scale"] == 1.0 else 2.5e-3 * max(1.0, float(o.abs().max()))
        assert mx <= lim and mean <= 2.5e-4 * (1 if m["input_scale"] == 1.0 else 4), (i, mx, mean)


@pytest.mark.gpu
def test_trace_records_cover_the_grid():
    from fa_b200 import lib
    from fa_b200.ops import Operator

    q, k, v = _inputs(1, 12, 1, 4096, seed=2)
    op = Operator("fp32", trace=True)
    op.workspace(q.device).zero_()
    op(q, k, v)
    recs = op.trace(q.device)
    n_items = len(lib.plan_items(1, 12, 4096, 0, lib.num_units(1, 12, 4096)))
    sms = torch.cuda.get_device_properties(q.device).multi_processor_count
    pairs = len(recs) // 2
    assert len(recs) == 2 * pairs and 1 <= pairs <= min(n_items, sms // 2)
    assert sorted(r["rank"] for r in recs) == [0] * pairs + [1] * pairs
    assert sum(r["items"] for r in recs if r["rank"] == 0) == n_items  # each item once per pair
    assert sum(r["items"] for r in recs if r["rank"] == 1) == n_items
    assert all(r["t_end_ns"] > r["t_start_ns"] for r in recs)
    assert len({r["smid"] for r in recs}) == len(recs)  # one persistent CTA per SM


@pytest.mark.gpu
@pytest.mark.parametrize("chunks", [1, 3, 8])
@pytest.mark.parametrize("shape,world,rank", [((1, 3, 1, 1000), 1, 0), ((2, 4, 2, 700), 3, 1)])
def test_forward_host_matches_device_path(chunks, shape, world, rank):
    """The pipelined host-buffer path (pieces of the unit range with their
    copies overlapped) gives the device path's O bit for bit, and moves only
    the unit range's rows."""
    from fa_b200 import shard
    from fa_b200.ops import Operator

    B, Hq, Hkv, N = shape
    q, k, v = _inputs(*shape, seed=7)
    op = Operator("fp16")
    (ub, ue), (r0, r1) = shard.shard_rows(B, Hq, N, world, rank)
    ref = op(q, k, v, out=torch.zeros_like(q), unit_range=(ub, ue)).view(-1, 128)[r0:r1]
    q_host = q.view(-1, 128)[r0:r1].cpu().pin_memory()
    k_host, v_host = k.cpu().pin_memory(), v.cpu().pin_memory()
    o_host = torch.full((r1 - r0, 128), float("nan"), dtype=torch.float16).pin_memory()
    q_dev, k_dev, v_dev = torch.zeros_like(q), torch.zeros_like(k), torch.zeros_like(v)
    o_dev = torch.full_like(q, float("nan"))
    h2d, d2h = op.forward_host(q_host, k_host, v_host, o_host, q_dev=q_dev, k_dev=k_dev, v_dev=v_dev,
                               o_dev=o_dev, unit_range=(ub, ue), chunks=chunks)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(o_host, ref.cpu())
    # only the K/V heads of the range's (b, hq) went up (the others stay zero)
    nqb = -(-N // 128)
    heads = sorted({(bh // Hq) * Hkv + (bh % Hq) // (Hq // Hkv) for bh in range(ub // nqb, (ue - 1) // nqb + 1)})
    assert d2h == (r1 - r0) * 256 and h2d == (r1 - r0) * 256 + 2 * len(heads) * N * 256
    kf = k_dev.view(B * Hkv, N, 128)
    for kvh in range(B * Hkv):
        assert bool(kf[kvh].abs().sum() > 0) == (kvh in heads)
    of = o_dev.view(-1, 128)
    assert torch.isnan(of[:r0]).all() and torch.isnan(of[r1:]).all()
    with pytest.raises(ValueError):
        op.forward_host(q_host.clone(), k_host, v_host, o_host, q_dev=q_dev, k_dev=k_dev, v_dev=v_dev,
                        o_dev=o_dev, unit_range=(ub, ue))  # not pinned
