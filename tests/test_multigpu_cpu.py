"""Head-parallel sharding host logic on CPU ``gloo`` ranks (world size 2).

The all-gather that reassembles the layer output, the head partition, and
failure detection when a rank dies before the collective (the survivor's
collective ends with an error after the process-group timeout) -- all without
a GPU.
"""

from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fpv2.shard import gather_heads, head_shard


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_head_shard_partition():
    for world in (1, 2, 4, 8):
        seen_q, seen_kv = [], []
        for r in range(world):
            sh = head_shard(32, 8, world, r)
            seen_kv += list(range(sh.kv_start, sh.kv_end))
            seen_q += list(range(sh.q_start, sh.q_end))
            assert sh.q_end - sh.q_start == 4 * (sh.kv_end - sh.kv_start)
        assert seen_kv == list(range(8)) and seen_q == list(range(32))
    with pytest.raises(ValueError, match="evenly"):
        head_shard(32, 8, 3, 0)


def _worker_gather(rank: int, world: int, port: int, q) -> None:
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
        hq, L, D = 8, 16, 4
        full = torch.arange(hq * L * D, dtype=torch.float32).reshape(1, hq, L, D)
        sh = head_shard(hq, 2, world, rank)
        local = full[:, sh.q_start:sh.q_end].clone()
        out = gather_heads(local)
        q.put((rank, bool(torch.equal(out, full))))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover - reported to the parent
        q.put((rank, traceback.format_exc()))


def test_gather_heads_world2_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_gather, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: True, 1: True}, results


def _worker_fail(rank: int, world: int, port: int, q) -> None:
    from fpv2.shard import RankMonitor

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    monitor = RankMonitor(timeout_s=3.0)
    monitor.check()                      # step 1: everyone alive
    if rank == 1:
        # this rank fails between steps, with nothing of its own in flight
        q.put((rank, "left"))
        q.close()
        q.join_thread()   # flush the message before the hard exit
        os._exit(0)
    try:
        monitor.check()                  # step 2: the survivor learns before launching work
        q.put((rank, "no error"))
    except Exception as exc:
        q.put((rank, f"error: {type(exc).__name__}: {str(exc)[:200]}"))
    q.close()
    q.join_thread()
    os._exit(0)


def test_rank_loss_is_reported_before_the_next_step():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_fail, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():  # pragma: no cover
            p.kill()
    assert results[1] == "left"
    assert results[0].startswith("error"), results
    assert "1" in results[0]             # the failed rank is named
