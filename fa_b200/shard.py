"""Multi-GPU sharding of the (b, hq, 128-row query block) unit grid.

A unit is independent of every other unit: it needs one 128-row block of Q
and the whole K/V of its KV head.  N ranks split the linear unit range
contiguously (``partition``, the PartitionContiguous semantics of the
reference's cce_task.h:28-35, implemented in the C ABI) and each rank runs
the kernel on its range with K/V replicated.  No collective sits on the hot
path; ``gather_output`` (an all-gather) exists only to verify a sharded
result against an unsharded one.

Units map to rows of O flattened to [B*Hq*Nq, 128]: unit u = (bh, qb) covers
rows bh*Nq + [qb*128, min(Nq, qb*128+128)), so a contiguous unit range is a
contiguous row range.
"""

from __future__ import annotations

import math

BLOCK_M = 128


def partition(total: int, parts: int, index: int) -> tuple[int, int]:
    """[begin, end) of part ``index``: near-equal split, remainder to the first parts."""
    if total < 0 or parts <= 0 or not 0 <= index < parts:
        raise ValueError(f"bad partition total={total} parts={parts} index={index}")
    base, rem = divmod(total, parts)
    begin = index * base + min(index, rem)
    return begin, begin + base + (1 if index < rem else 0)


def num_units(B: int, Hq: int, Nq: int) -> int:
    return B * Hq * math.ceil(Nq / BLOCK_M)


def unit_row(u: int, Nq: int) -> int:
    """First flattened O row of unit ``u`` (or the end row when u == num_units)."""
    nqb = math.ceil(Nq / BLOCK_M)
    bh, qb = divmod(u, nqb)
    return bh * Nq + min(Nq, qb * BLOCK_M)


def row_range(unit_begin: int, unit_end: int, Nq: int) -> tuple[int, int]:
    return unit_row(unit_begin, Nq), unit_row(unit_end, Nq)


def pieces(unit_begin: int, unit_end: int, chunks: int, item_units: int = 2) -> list[int]:
    """Boundaries of ``chunks`` contiguous pieces of [unit_begin, unit_end)
    on whole work items (``item_units`` units from the range start), the
    first and last pieces quarter-sized when there are three or more: the
    schedule of ``Operator.forward_host``, whose end pieces' copies are the
    ones not hidden behind a kernel.  Returns n+1 increasing boundaries
    from unit_begin to unit_end (n >= 1; pieces may be empty only when the
    range is)."""
    if unit_end < unit_begin or chunks < 1 or item_units < 1:
        raise ValueError(f"bad pieces({unit_begin}, {unit_end}, {chunks})")
    items = -(-(unit_end - unit_begin) // item_units)
    n = max(1, min(int(chunks), items))
    w = [1.0] * n
    if n >= 3:
        w[0] = w[-1] = 0.25
    acc = [0.0]
    for x in w:
        acc.append(acc[-1] + x)
    return [min(unit_end, unit_begin + item_units * int(round(items * a / acc[-1]))) for a in acc]


def shard_rows(B: int, Hq: int, Nq: int, world: int, rank: int) -> tuple[tuple[int, int], tuple[int, int]]:
    """(unit range, flattened row range) of ``rank``."""
    ub, ue = partition(num_units(B, Hq, Nq), world, rank)
    return (ub, ue), row_range(ub, ue, Nq)


def gather_output(out, B: int, Hq: int, Nq: int, world: int, rank: int, group=None):
    """All-gather every rank's rows of O; returns the full [B,Hq,Nq,D] tensor on
    every rank (verification only).  ``out`` is this rank's full-size O whose
    rows outside its shard are ignored."""
    import torch
    import torch.distributed as dist

    D = out.shape[-1]
    flat = out.reshape(-1, D)
    spans = [shard_rows(B, Hq, Nq, world, r)[1] for r in range(world)]
    width = max(e - b for b, e in spans)
    r0, r1 = spans[rank]
    send = torch.zeros((width, D), dtype=out.dtype, device=out.device)
    send[: r1 - r0] = flat[r0:r1]
    recv = [torch.empty_like(send) for _ in range(world)]
    dist.all_gather(recv, send, group=group)
    full = torch.empty_like(flat)
    for (b, e), chunk in zip(spans, recv):
        full[b:e] = chunk[: e - b]
    return full.reshape(out.shape)
