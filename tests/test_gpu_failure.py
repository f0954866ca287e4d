"""Failure detection on the GPU without a fault.

The test-only flag B200FA_FLAG_TEST_WITHHOLD_P makes the softmax warps of
query tile 1 (both CTAs of the pair) withhold their first P-ready arrival.
The MMA thread's bounded wait then runs out (limit set to 0.2 s here), the
kernel records B200FA_DEV_TIMEOUT in its workspace status word, raises the
abort flag of both CTAs, every role leaves its loop, TMEM is freed and the
kernel returns.  The host reads the status; the context stays usable and
the next call is correct.  No trap, no fault, no unbounded wait.
"""

import pytest
import torch

from oracle.attention_ref import attention_fp32, errors


def _inputs():
    g = torch.Generator().manual_seed(5)
    q = torch.randn((1, 2, 256, 128), generator=g).half()
    k = torch.randn((1, 1, 256, 128), generator=g).half()
    v = torch.randn((1, 1, 256, 128), generator=g).half()
    return q, k, v


@pytest.mark.gpu
def test_bounded_wait_reports_timeout_and_context_survives():
    from fa_b200 import lib
    from fa_b200.ops import Operator

    dev = torch.device("cuda", 0)
    q, k, v = (t.to(dev) for t in _inputs())
    op = Operator("fp32", timeout_us=200_000)
    op.reset_status(dev)
    op(q, k, v, flags=lib.FLAG_TEST_WITHHOLD_P)
    status = op.status(dev)
    assert status[0] == lib.DEV_TIMEOUT, status
    site_rank, site_warp = status[1] >> 16, (status[1] >> 8) & 0xFF
    assert site_rank in (0, 1) and 0 <= site_warp <= 11, status  # the first wait that ran out

    op.reset_status(dev)
    assert op.status(dev)[0] == lib.DEV_OK
    out = op(q, k, v)
    assert op.status(dev)[0] == lib.DEV_OK
    mx, mean = errors(out.cpu(), attention_fp32(*_inputs()))
    assert mx <= 2e-3 and mean <= 2e-4
