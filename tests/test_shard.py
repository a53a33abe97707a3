"""Request sharding across ranks (CPU, Gloo, world size 2): LPT balance, the probability gather
to rank 0, and a rank that fails before the gather (the others get an error from a short
process-group timeout instead of hanging)."""
import datetime
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest
import torch

from fastdecisions_b200.shard import bin_loads, gather_probs, lpt_partition


def test_lpt_balance_and_coverage():
    rng = np.random.default_rng(17)
    costs = list(rng.lognormal(0, 1, size=257))
    for n in (1, 2, 4, 8):
        bins = lpt_partition(costs, n)
        flat = sorted(i for b in bins for i in b)
        assert flat == list(range(len(costs)))
        loads = bin_loads(costs, bins)
        # LPT bound: max load <= mean load + largest item
        assert max(loads) <= sum(costs) / n + max(costs) + 1e-9


def test_lpt_rejects_bad_rank_count():
    with pytest.raises(ValueError):
        lpt_partition([1.0], 0)


def test_gather_without_process_group():
    p = torch.arange(6, dtype=torch.float32).reshape(3, 2)
    out = gather_probs(np.array([2, 0, 1]), p, 3)
    assert torch.equal(out, torch.tensor([[2.0, 3.0], [4.0, 5.0], [0.0, 1.0]]))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, fail_rank, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        costs = [float(x) for x in range(1, 11)]
        bins = lpt_partition(costs, world)
        mine = bins[rank]
        probs = torch.tensor([[float(i), float(i) + 0.5] for i in mine])
        if rank == fail_rank:
            raise RuntimeError("injected failure before the gather")
        out = gather_probs(np.array(mine), probs, len(costs))
        if rank == 0:
            q.put(("ok", out.tolist()))
        else:
            q.put(("ok", None))
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent, never hangs
        q.put(("err", f"{type(exc).__name__}: {exc}"))


def _run(world, fail_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, fail_rank, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def test_gather_two_ranks_gloo():
    res = _run(2, fail_rank=-1)
    assert all(r[0] == "ok" for r in res), res
    out = [r[1] for r in res if r[1] is not None][0]
    assert out == [[float(i), float(i) + 0.5] for i in range(10)]


def test_failed_rank_does_not_hang_the_others():
    res = _run(2, fail_rank=1)
    kinds = sorted(r[0] for r in res)
    assert kinds == ["err", "err"], res   # the failing rank raises; rank 0's gather times out
