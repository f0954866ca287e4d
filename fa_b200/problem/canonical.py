"""Canonical attention inputs -- a pure function of (Case, seed, device).

Mirror of the reference problem/canonical.py:18-28: seed the default
generator, then draw q [B,Hq,S,D], k [B,Hkv,S,D], v [B,Hkv,S,D] in that order
with ``torch.randn(..., dtype=float16)``.  The reference allocates on the NPU
through ``torch.set_default_device("npu")``; here the device is a parameter
(default: the current CUDA device) and the global default device is left
alone.  On the CPU the draws are identical to the reference's; on a GPU they
follow CUDA's generator, so cross-device parity is semantic, not bitwise.
"""

import torch


def build_canonical(case, seed: int = 0, device=None) -> dict:
    """Allocate the canonical q/k/v inputs on ``device``."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu"
    torch.manual_seed(seed)

    def rand(*shape):
        return torch.randn(shape, dtype=torch.float16, device=device)

    return {
        "q": rand(case.batch, case.heads_q, case.seq_len, case.dim),
        "k": rand(case.batch, case.heads_kv, case.seq_len, case.dim),
        "v": rand(case.batch, case.heads_kv, case.seq_len, case.dim),
    }
