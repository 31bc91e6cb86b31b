"""Multi-rank host logic on CPU (gloo, world size 2): counter reduction,
max-over-ranks timing, and a rank that fails before the collective making the
other rank's collective end with an error instead of hanging."""
import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "a11-llm-optimizer_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    from a11spec import distributed as D
    try:
        D.init(backend="gloo", timeout_s=5.0)
        if mode == "ok":
            stats = torch.arange(6, dtype=torch.int64) * (rank + 1)
            tot = D.reduce_stats(stats)
            t = D.max_time(10.0 + rank)
            q.put((rank, tot.tolist(), t, stats.tolist()))
        elif mode == "periodic":
            # the bench's counter reduction: every 5 steps, 12 steps -> after steps 5 and 10
            stats = torch.zeros(6, dtype=torch.int64)
            red = D.CounterReducer(stats, every=5)
            seen = []
            for _ in range(12):
                stats += torch.arange(6, dtype=torch.int64) + rank  # this step's counters
                red.step()
                if red.result() is not None:
                    seen.append(red.result()["through_step"])
            red.finish()
            q.put((rank, red.result(), sorted(set(seen)), red.reduces))
        else:
            if rank == 1:
                raise RuntimeError("rank 1 fails before the step's collective")
            try:
                D.reduce_stats(torch.ones(6, dtype=torch.int64))
                q.put((rank, "returned"))
            except Exception as e:  # the collective ends with an error (timeout / peer gone)
                q.put((rank, "error:" + type(e).__name__))
    except RuntimeError as e:
        q.put((rank, "raised:" + str(e)))
    finally:
        import torch.distributed as dist
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run(mode, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = {}
    for _ in range(2):
        item = q.get(timeout=timeout)
        out[item[0]] = item[1:]
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


def test_counters_sum_and_time_max_over_ranks():
    out = _run("ok")
    expect = [sum(i * (r + 1) for r in range(2)) for i in range(6)]
    for r in range(2):
        tot, t, local = out[r]
        assert tot == expect and t == 11.0
        assert local == [i * (r + 1) for i in range(6)]  # reduce_stats leaves its input alone


def test_periodic_counter_reduction():
    """CounterReducer (the bench's multi-GPU counter sum) all-reduces a snapshot
    every 5 steps; both ranks see the same sums, covering steps 1-10 of 12."""
    out = _run("periodic")
    want = [10 * (2 * i + 1) for i in range(6)]  # 10 steps of (i + 0) + (i + 1)
    for r in range(2):
        res, seen, reduces = out[r]
        assert reduces == 2 and seen == [5, 10]
        assert res["through_step"] == 10 and res["ranks"] == 2
        from a11spec._lib import STAT_NAMES
        assert [res[n] for n in STAT_NAMES] == want


def test_failed_rank_ends_peer_collective_with_error():
    out = _run("fail")
    assert out[1][0].startswith("raised:")
    assert out[0][0].startswith("error:"), out
