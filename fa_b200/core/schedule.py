"""Execution scheduling primitives (mirror of the reference core/schedule.py).

  * parallel_compile       -- compile tasks on a CPU process pool (no GPU).
  * distribute_over_cards  -- one worker process per GPU at a time; GPUs run
                              in parallel; results come back in item order.

Pools use the ``spawn`` start method so that no worker inherits a CUDA
context from its parent.  Workers must be picklable (top-level functions or
``functools.partial`` of one).
"""

import multiprocessing as mp
import os
from concurrent.futures import ProcessPoolExecutor


def _ctx():
    return mp.get_context("spawn")


def parallel_compile(items, compile_one, workers=None):
    if not items:
        return []
    workers = workers or min(len(items), os.cpu_count() or 1)
    with ProcessPoolExecutor(max_workers=workers, mp_context=_ctx()) as pool:
        return list(pool.map(compile_one, items))


def _card_task(packed):
    worker, item, queue = packed
    device = queue.get()
    try:
        return worker(item, device)
    finally:
        queue.put(device)


def distribute_over_cards(items, devices, worker):
    """Run ``worker(item, device)`` over ``devices``, one process per card."""
    if not items:
        return []
    ctx = _ctx()
    with ctx.Manager() as mgr:
        queue = mgr.Queue()
        for d in devices:
            queue.put(d)
        packed = [(worker, it, queue) for it in items]
        with ProcessPoolExecutor(max_workers=len(devices), mp_context=ctx) as pool:
            return list(pool.map(_card_task, packed))
