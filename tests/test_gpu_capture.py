"""Debug capture (B200FA_FLAG_CAPTURE): the kernel's per-block online-softmax
state against the float64 restatement of the recurrence.

The capture is the counterpart of the reference's ``capture`` attribute
(backends/cce_fa_nqkq_nz_resident_v13_q768_pool_i4_p128/binding.py:39-41,
op_kernel/vector_output.h:94-106): per key block and query row the running
maximum m, the running sum l, the rescale factor alpha, the block sum z and
the running output O.

* small ragged cases, both variants: every record against
  ``online_state_f64``; the kernel's own records obey l_j = alpha_j l_(j-1)
  + z_j; capturing does not change the output (bit-identical);
* a shard: records outside its unit range are not written;
* a 4096-key case: the final (m, l) give each row's log-sum-exp and O/l the
  output.

Rows whose block maximum lies within 1e-3 of the lazy-rescale threshold are
left out of the record comparison (the FP32 scores may decide that move
either way; the result is exact both ways).
"""

import numpy as np
import pytest
import torch

from oracle.attention_ref import online_state_f64

# (rtol of z and l, atol of O/l, atol of z) per variant: the FP32 variant
# computes P = 2^x in FP32 (MUFU or a degree-3 polynomial, <= 1e-4
# relative); the FP16 one rounds x to FP16 and sums FP16 exponentials in
# groups of eight, and exponentials below 2^-14 are FP16 subnormals (spacing
# 2^-24): a block far below the running maximum carries up to 128 * 2^-25
# absolute error in z.
TOL = {"fp32": (2e-4, 2e-3, 1e-7), "fp16": (1e-2, 5e-3, 6e-6)}


def _inputs(B, Hq, Hkv, Nq, Nk, kscale=1.0, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((B, Hq, Nq, 128), generator=g).half()
    k = (torch.randn((B, Hkv, Nk, 128), generator=g) * kscale).half()
    v = torch.randn((B, Hkv, Nk, 128), generator=g).half()
    return q.cuda(), k.cuda(), v.cuda()


@pytest.mark.gpu
@pytest.mark.parametrize("variant", ["fp16", "fp32"])
@pytest.mark.parametrize("shape,kscale", [((1, 4, 2, 300, 1000), 1.0), ((2, 2, 1, 128, 80), 1.0),
                                          ((1, 2, 1, 520, 730), 3.0)])
def test_capture_matches_oracle(variant, shape, kscale):
    from fa_b200.ops import Operator

    q, k, v = _inputs(*shape, kscale=kscale)
    op = Operator(variant)
    plain = op(q, k, v)
    cap = Operator.capture_buffer(q, k)
    out = op(q, k, v, capture=cap)
    torch.cuda.synchronize()
    assert torch.equal(out, plain)

    got = {n: t.cpu().double().numpy() for n, t in Operator.capture_view(cap, q, k).items()}
    from fa_b200 import lib

    ref = online_state_f64(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), block=lib.BLOCK_KEYS)
    for n in ("m", "l", "alpha", "z", "o"):
        assert np.isfinite(got[n]).all(), n
    keep = ref["margin"] > 1e-3  # [B, Hq, Nq]
    assert keep.mean() > 0.9
    rtol, otol, zatol = TOL[variant]

    def rows(a):  # [B, Hq, nb, Nq, ...] -> kept rows
        return np.moveaxis(a, 2, 3)[keep]

    np.testing.assert_allclose(rows(got["m"]), rows(ref["m"]), rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(rows(got["alpha"]), rows(ref["alpha"]), rtol=1e-4, atol=1e-7)
    np.testing.assert_allclose(rows(got["z"]), rows(ref["z"]), rtol=rtol, atol=zatol)
    np.testing.assert_allclose(rows(got["l"]), rows(ref["l"]), rtol=rtol)
    o_got = rows(got["o"]) / rows(got["l"])[..., None]
    o_ref = rows(ref["o"]) / rows(ref["l"])[..., None]
    assert np.abs(o_got - o_ref).max() < otol
    # the kernel's own records: l_j = alpha_j l_(j-1) + z_j (FP32 arithmetic)
    lp = np.concatenate([np.zeros_like(got["l"][:, :, :1]), got["l"][:, :, :-1]], axis=2)
    np.testing.assert_allclose(got["l"], got["alpha"] * lp + got["z"], rtol=1e-6)
    # the last block's O / l is the output before its FP16 cast
    final = got["o"][:, :, -1] / got["l"][:, :, -1, :, None]
    np.testing.assert_allclose(final, out.cpu().double().numpy(), rtol=2.0 ** -10, atol=2e-4)


@pytest.mark.gpu
def test_capture_of_a_shard_leaves_other_records():
    from fa_b200 import shard
    from fa_b200.ops import Operator

    B, Hq, Hkv, Nq, Nk = 1, 3, 1, 400, 500
    q, k, v = _inputs(B, Hq, Hkv, Nq, Nk, seed=3)
    op = Operator("fp32")
    (ub, ue), (r0, r1) = shard.shard_rows(B, Hq, Nq, 3, 1)
    cap = Operator.capture_buffer(q, k)
    op(q, k, v, unit_range=(ub, ue), capture=cap)
    torch.cuda.synchronize()
    view = Operator.capture_view(cap, q, k)
    inside = torch.zeros((B * Hq * Nq,), dtype=torch.bool, device=q.device)
    inside[r0:r1] = True
    inside = inside.view(B, Hq, 1, Nq)
    for n in ("m", "l", "alpha", "z"):
        t = view[n]
        assert torch.isfinite(t[inside.expand_as(t)]).all(), n
        assert torch.isnan(t[~inside.expand_as(t)]).all(), n
    o = view["o"]
    assert torch.isfinite(o[inside.expand(o.shape[:-1])]).all()
    assert torch.isnan(o[~inside.expand(o.shape[:-1])]).all()


@pytest.mark.gpu
@pytest.mark.parametrize("variant", ["fp16", "fp32"])
def test_capture_final_state_gives_logsumexp(variant):
    from fa_b200.ops import Operator

    B, Hq, Hkv, N = 1, 2, 1, 4096
    q, k, v = _inputs(B, Hq, Hkv, N, N, seed=5)
    cap = Operator.capture_buffer(q, k)
    out = Operator(variant)(q, k, v, capture=cap)
    view = Operator.capture_view(cap, q, k)
    m, l = view["m"][:, :, -1].double(), view["l"][:, :, -1].double()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        s = (q.double() @ k.double().transpose(-1, -2)) * (128 ** -0.5)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    lse2 = torch.logsumexp(s, dim=-1) / np.log(2.0)
    rtol = TOL[variant][0]
    assert ((m + torch.log2(l)) - lse2).abs().max().item() < 2 * rtol + 1e-5
    final = view["o"][:, :, -1] / view["l"][:, :, -1, :, None]
    torch.testing.assert_close(final, out.float(), rtol=2.0 ** -10, atol=2e-4)


@pytest.mark.gpu
def test_capture_rejects_short_or_wrong_buffers():
    from fa_b200 import lib
    from fa_b200.ops import Operator

    q, k, v = _inputs(1, 2, 1, 256, 256)
    op = Operator("fp16")
    cap = Operator.capture_buffer(q, k)
    with pytest.raises(lib.B200FAError):
        op(q, k, v, capture=cap[:-1])
    with pytest.raises(ValueError):
        op(q, k, v, capture=cap.half())
    with pytest.raises(ValueError):
        Operator.capture_buffer(torch.empty((1, 12, 8192, 128), device="meta"),
                                torch.empty((1, 1, 8192, 128), device="meta"))
