"""The optional causal mask (``Operator(...)(q, k, v, causal=True)``,
``B200FA_FLAG_CAUSAL``): query row i attends keys 0..i (top-left aligned,
torch's ``is_causal`` convention).  An addition to the reference's
non-causal operator: each work item stops at the diagonal block of its last
query block, and the block crossing a row's diagonal is masked per row.

CPU: the oracle's causal mask matches torch's ``is_causal`` SDPA.  GPU: both
variants against the FP32 oracle on shapes with Nq = Nk, Nq < Nk, Nq > Nk,
tails, GQA and several work items per CTA pair, at the parity bar of the
non-causal tests; the causal result differs from the non-causal one; and
a sharded causal run equals the whole-range run bit for bit.  The first
rows of a causal problem attend a few keys only (row 0: key 0, O = V[0]),
so |O| reaches ~4 there: as in the non-causal fuzz test, the FP16
variant's bar (FP16 P summed in FP16) is then the north star's relative to
max(1, max|O|) plus the FP16 rounding of the reference itself.
"""

import pytest
import torch

from oracle.attention_ref import attention_fp32, errors

MAX_ABS = 2e-3
MEAN_ABS = 2e-4

SHAPES = [
    # (B, Hq, Hkv, Nq, Nk)
    (1, 2, 1, 256, 256),
    (1, 4, 2, 300, 300),
    (1, 2, 1, 130, 333),
    (1, 2, 1, 333, 130),
    (2, 8, 2, 1000, 777),
    (1, 16, 1, 4096, 384),
    (1, 12, 1, 2048, 2048),
    (1, 2, 1, 1, 1),
]


def _inputs(B, Hq, Hkv, Nq, Nk, seed, device):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn((B, Hq, Nq, 128), generator=g)
    k = torch.randn((B, Hkv, Nk, 128), generator=g)
    v = torch.randn((B, Hkv, Nk, 128), generator=g)
    return [t.half().to(device) for t in (q, k, v)]


def test_oracle_causal_mask_is_torchs_is_causal():
    q, k, v = _inputs(1, 4, 2, 70, 90, 3, "cpu")
    ref = attention_fp32(q, k, v, causal=True, rows_per_block=32)
    kk, vv = k.repeat_interleave(2, dim=1), v.repeat_interleave(2, dim=1)
    sdpa = torch.nn.functional.scaled_dot_product_attention(q.float(), kk.float(), vv.float(), is_causal=True)
    # Two FP32 implementations (their summation order follows torch's CPU
    # threading): agreement to 1e-5, where a mask off by one key or row
    # differs by ~1e-2.
    assert torch.allclose(ref, sdpa, atol=1e-5, rtol=0), float((ref - sdpa).abs().max())


@pytest.mark.gpu
@pytest.mark.parametrize("variant", ["fp16", "fp32"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_causal_parity_vs_oracle(variant, shape):
    from fa_b200.ops import Operator

    q, k, v = _inputs(*shape, seed=sum(shape) + 1, device="cuda")
    op = Operator(variant)
    out = op(q, k, v, causal=True)
    torch.cuda.synchronize()
    assert op.status(q.device)[0] == 0
    ref = attention_fp32(q, k, v, causal=True)
    mx, mean = errors(out, ref)
    assert torch.isfinite(out).all()
    lim_mx, lim_mean = MAX_ABS, MEAN_ABS
    rel = max(1.0, float(ref.abs().max())) if variant == "fp16" else 1.0
    if rel > 1.0:
        floor_mx, floor_mean = errors(ref.half().float(), ref)
        lim_mx, lim_mean = lim_mx * rel + floor_mx, lim_mean * rel + floor_mean
    assert mx <= lim_mx and mean <= lim_mean, (shape, variant, mx, mean, lim_mx, lim_mean)
    if shape[3] > 1:
        full = op(q, k, v)
        torch.cuda.synchronize()
        assert not torch.equal(full, out)


@pytest.mark.gpu
def test_causal_shards_equal_the_whole_range():
    from fa_b200 import shard
    from fa_b200.ops import Operator

    B, Hq, Hkv, N = 1, 12, 1, 2048
    q, k, v = _inputs(B, Hq, Hkv, N, N, seed=5, device="cuda")
    op = Operator("fp32")
    whole = op(q, k, v, causal=True)
    parts = torch.full_like(q, float("nan"))
    units = shard.num_units(B, Hq, N)
    for rank in range(3):
        ub, ue = shard.partition(units, 3, rank)
        op(q, k, v, causal=True, out=parts, unit_range=(ub, ue))
    torch.cuda.synchronize()
    assert op.status(q.device)[0] == 0
    assert torch.equal(parts, whole)
