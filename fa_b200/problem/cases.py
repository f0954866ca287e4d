"""The attention test matrix -- the problem, independent of any backend.

Mirror of the reference problem/cases.py:13-43: a ``Case`` carries only the
logical workload (B, S, Hq, Hkv, D) of one non-causal GQA forward over full
[B, H, S, D] tensors, with ``scale = D**-0.5``, ``group_size = Hq // Hkv``
and the name ``B{b}_S{s}_Q{hq}_KV{hkv}_D{d}``.

``CASES`` keeps the reference's three cases at indices 0-2 (same meaning as
in the reference) and appends the two additional benchmark configurations:
(B=1, S=2048, Hq=12, Hkv=1) and (B=4, S=8192, Hq=32, Hkv=8).
"""

from dataclasses import dataclass


@dataclass(frozen=True)
class Case:
    batch: int          # B
    seq_len: int        # S, both query and key length (non-causal full attention)
    heads_q: int        # query heads
    heads_kv: int       # KV heads (GQA: heads_q % heads_kv == 0)
    dim: int = 128      # head dim (the kernels require 128)

    @property
    def group_size(self) -> int:
        return self.heads_q // self.heads_kv

    @property
    def scale(self) -> float:
        return self.dim ** -0.5

    @property
    def name(self) -> str:
        return f"B{self.batch}_S{self.seq_len}_Q{self.heads_q}_KV{self.heads_kv}_D{self.dim}"

    @property
    def flops(self) -> int:
        """QK^T + PV FLOPs, 4*B*Hq*Nq*Nk*D (reference README.md:86)."""
        return 4 * self.batch * self.heads_q * self.seq_len * self.seq_len * self.dim


CASES = (
    Case(2, 131072, 12, 1, 128),   # reference index 0 (C5, the headline configuration)
    Case(2, 65536, 12, 1, 128),    # reference index 1 (C4)
    Case(1, 32768, 12, 1, 128),    # reference index 2 (C3)
    Case(1, 2048, 12, 1, 128),     # C1: plumbing case, CPU-checkable in full
    Case(4, 8192, 32, 8, 128),     # C2: 4:1 grouping
)

HEADLINE = CASES[0]


def index_of(case: Case) -> int:
    return CASES.index(case)
