"""Multi-process host logic of the sharded rollout on CPU ranks (gloo).

Covers the environment sharding, the all-gather of per-rank logits into the
full action vector, and failure detection: a rank that dies between steps
makes the surviving rank's next collective fail within the process-group
timeout instead of hanging.
"""
import datetime
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


def _init(rank, world, port, timeout_s=20):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _gather_worker(rank, world, port, q):
    from rl_for_mario_b200.rollout import gather_rows, shard_range

    _init(rank, world, port)
    lo, hi = shard_range(8, rank, world)
    local = torch.arange(lo, hi, dtype=torch.float32).view(-1, 1).repeat(1, 7) + 0.5
    full = gather_rows(local)
    q.put((rank, lo, hi, full.argmax(-1).tolist(), full[:, 0].tolist()))
    dist.barrier()
    dist.destroy_process_group()


def _failing_worker(rank, world, port, q):
    from rl_for_mario_b200.rollout import gather_rows

    _init(rank, world, port, timeout_s=5)
    gather_rows(torch.ones(2, 7))          # step 1: both ranks
    if rank == 1:
        os._exit(0)                         # rank 1 leaves between steps
    try:
        gather_rows(torch.ones(2, 7))       # step 2: the peer is gone
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001 - any collective error is the detection
        q.put((rank, "error:" + type(e).__name__))


def _run(fn, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    out = []
    while not q.empty():
        out.append(q.get())
    return out


def test_shard_range_partitions_envs():
    from rl_for_mario_b200.rollout import shard_range

    assert [shard_range(65536, r, 8) for r in (0, 7)] == [(0, 8192), (57344, 65536)]
    with pytest.raises(ValueError):
        shard_range(10, 0, 3)


def test_all_gather_of_logits_over_two_cpu_ranks():
    res = sorted(_run(_gather_worker, 2))
    assert [r[0] for r in res] == [0, 1]
    for rank, lo, hi, argmax, col0 in res:
        assert (lo, hi) == ((0, 4) if rank == 0 else (4, 8))
        assert col0 == [i + 0.5 for i in range(8)]   # every rank sees all rows in rank order


def test_dead_rank_is_detected_not_hung():
    res = dict(_run(_failing_worker, 2))
    assert res.get(0, "").startswith("error:")
