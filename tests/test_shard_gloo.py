"""Multi-rank sharding logic on CPU ranks (gloo, world size 2 and 3).

Each rank computes the oracle output of its contiguous share of the
(b, hq, q-block) units only, then ``gather_output`` reassembles O; the
result must equal the unsharded oracle bit for bit.  A second test has one
rank fail before the gather and checks that the other rank's collective
ends with an error (short process-group timeout) instead of hanging.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _inputs(B, Hq, Hkv, N):
    g = torch.Generator().manual_seed(3)
    q = torch.randn((B, Hq, N, 128), generator=g).half()
    k = torch.randn((B, Hkv, N, 128), generator=g).half()
    v = torch.randn((B, Hkv, N, 128), generator=g).half()
    return q, k, v


def _worker(rank, world, port, shape, result_q):
    import datetime

    from fa_b200 import shard
    from oracle.attention_ref import attention_rows_fp32

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        B, Hq, Hkv, N = shape
        q, k, v = _inputs(B, Hq, Hkv, N)
        (ub, ue), (r0, r1) = shard.shard_rows(B, Hq, N, world, rank)
        out = torch.full((B, Hq, N, 128), float("nan"), dtype=torch.float32)
        flat = out.view(-1, 128)
        rows = torch.tensor([[r // (Hq * N), (r // N) % Hq, r % N] for r in range(r0, r1)], dtype=torch.long)
        if len(rows):
            flat[r0:r1] = attention_rows_fp32(q, k, v, rows)
        full = shard.gather_output(out, B, Hq, N, world, rank)
        # A numpy array is pickled by value: a tensor would be shared through a
        # file descriptor that dies with this process if it exits first.
        result_q.put((rank, ub, ue, full.numpy() if rank == 0 else None))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,shape", [(2, (1, 3, 1, 200)), (3, (2, 2, 2, 130))])
def test_sharded_oracle_equals_unsharded(world, shape):
    from oracle.attention_ref import attention_fp32

    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shape, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q_out.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    spans = [(ub, ue) for _, ub, ue, _ in results]
    assert spans[0][0] == 0 and all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    full = torch.from_numpy(results[0][3])
    ref = attention_fp32(*_inputs(*shape))
    assert not torch.isnan(full).any()
    assert torch.allclose(full, ref, atol=1e-6, rtol=0)


def _failing_worker(rank, world, port, result_q):
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=5))
        t = torch.ones(4)
        dist.all_reduce(t)  # step 1: every rank takes part
    except Exception as e:
        result_q.put((rank, f"setup failed: {e}"))
        return
    if rank == 1:
        # Leaves between steps: none of its collectives is in flight.
        result_q.put((rank, "left"))
        result_q.close()
        result_q.join_thread()  # flush before the abrupt exit
        os._exit(0)
    try:
        dist.all_reduce(t)  # step 2: the peer is gone
        result_q.put((rank, "completed"))
    except Exception as e:
        result_q.put((rank, f"error: {type(e).__name__}"))


def test_lost_rank_ends_collective_with_error():
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q_out.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert results[1] == "left"
    assert results[0].startswith("error")


@pytest.mark.parametrize("ub,ue,chunks", [(0, 24576, 4), (0, 24576, 1), (5, 37, 3), (0, 3, 8), (7, 8, 4),
                                          (0, 0, 4), (100, 1000, 6), (1, 9, 2)])
def test_host_path_pieces(ub, ue, chunks):
    """Pieces of forward_host: cover the range in order, cut only on whole
    items from the range start, end pieces no larger than the middle ones."""
    from fa_b200.shard import pieces

    b = pieces(ub, ue, chunks)
    assert b[0] == ub and b[-1] == ue and all(x <= y for x, y in zip(b, b[1:]))
    assert 1 <= len(b) - 1 <= max(1, chunks)
    assert all((x - ub) % 2 == 0 for x in b[:-1])  # work items are two units
    sizes = [y - x for x, y in zip(b, b[1:])]
    if len(sizes) >= 3 and ue - ub >= 16 * chunks:
        assert max(sizes[0], sizes[-1]) <= min(sizes[1:-1])
    with pytest.raises(ValueError):
        pieces(5, 4, 2)
