"""Host-side multi-rank logic on CPU with the gloo backend (world size 2).

The B200 op partitions a layer across ranks by kv-head range and/or query slab
(sta.partition) with no data-path collective; the only collectives are the barrier and the
max-over-ranks reduction of step times.  These tests run that partition + timing protocol on
CPU ranks, including a rank that fails between steps.
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
    p = s.getsockname()[1]
    s.close()
    return p


def partition(Hkv, G, world, rank):
    """kv heads [k0, k1) and q heads [k0*G, k1*G) of rank `rank` (bench.py's head rule)."""
    from sta.partition import kv_head_range
    k0, k1 = kv_head_range(Hkv, world, rank)
    return (k0, k1), (k0 * G, k1 * G)


def _worker(rank, world, port, result_q, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=20))
    try:
        Hkv, G = 8, 4
        (k0, k1), (h0, h1) = partition(Hkv, G, world, rank)
        mine = torch.zeros(Hkv * G, dtype=torch.int64)
        mine[h0:h1] = 1
        dist.all_reduce(mine)                      # every q head covered exactly once
        from sta.partition import plan
        N, T = 131072, 32
        cov = torch.zeros((Hkv, N // T), dtype=torch.int64)
        u = plan(Hkv, N, world, rank, "slabs")     # single-sequence query-slab unit
        cov[u["kv"][0]:u["kv"][1], u["slab"][0] // T:u["slab"][1] // T] = 1
        dist.all_reduce(cov)
        assert int(cov.min()) == 1 and int(cov.max()) == 1
        t = torch.tensor([10.0 + rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)   # max-over-ranks step time
        if rank == fail_rank:
            raise RuntimeError("injected failure between steps")
        dist.barrier()
        result_q.put((rank, mine.tolist(), float(t.item()), "ok"))
    except RuntimeError as e:
        result_q.put((rank, None, None, "error: " + str(e)[:60]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in ps:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
    return sorted(out)


def test_partition_covers_all_heads():
    for world in (1, 2, 4, 8):
        seen = []
        for r in range(world):
            (k0, k1), (h0, h1) = partition(8, 4, world, r)
            seen += list(range(h0, h1))
            assert h1 - h0 == 32 // world
        assert seen == list(range(32))


def test_two_gloo_ranks_partition_and_max_time():
    out = _run(2)
    for rank, cover, tmax, status in out:
        assert status == "ok"
        assert cover == [1] * 32
        assert tmax == 11.0


def test_rank_failure_between_steps_is_seen_by_peer():
    out = _run(2, fail_rank=1)
    status = {r: s for r, _, _, s in out}
    assert status[1].startswith("error: injected")
    # the surviving rank's next collective ends with an error (peer gone / timeout), not a hang
    assert status[0].startswith("error"), status[0]
