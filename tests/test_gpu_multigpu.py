"""Head-parallel FPV2 on two GPUs equals the single-GPU layer.

Each rank runs the index stage and the sparse attention on its KV-head shard
(and the matching query heads). The output is reassembled either by the
attention kernel itself (multicast stores into a symmetric-memory buffer, where
the GPUs support NVLink multicast) or by one NCCL all-gather; both must equal
the single-GPU layer on every rank.
Every selection reduction, list and K/V read of the path belongs to one KV
head, so the sharded layer must reproduce the single-GPU layer bit for bit.
Skipped unless at least two GPUs are visible.
"""

from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(length: int, hq: int, hkv: int, d: int):
    from tests.synthetic import topic_qkv

    q, k, v = topic_qkv(length=length, query_heads=hq, kv_heads=hkv, head_dim=d, seed=21,
                        dtype=torch.bfloat16)
    return q[None], k[None], v[None]


def _worker(rank: int, world: int, port: int, length: int, hq: int, hkv: int, d: int, queue) -> None:
    import torch.distributed as dist

    try:
        import fpv2
        from fpv2.shard import head_parallel_sdpa, head_shard, shard_inputs

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=dev)
        q, k, v = _inputs(length, hq, hkv, d)
        sh = head_shard(hq, hkv, world, rank)
        ql, kl, vl = (t.to(dev) for t in shard_inputs(q, k, v, sh))
        from fpv2.shard import _SYMM_BUFFERS

        cfg = fpv2.FPV2Config(alpha=0.1)
        ref = fpv2.fpv2_sdpa(q.to(dev), k.to(dev), v.to(dev), scale=d ** -0.5, config=cfg)
        report = []
        for fused in (False, True, True):   # NCCL, then the fused path twice (buffer reuse)
            out = head_parallel_sdpa(ql, kl, vl, scale=d ** -0.5, config=cfg, fused=fused)
            torch.cuda.synchronize(dev)
            diff = (out.float() - ref.float()).abs().max().item()
            report.append(f"{diff}")
        # a kept output is the caller's own: the next same-shape call (different
        # values) must not overwrite it, while copy=False aliases the shared buffer
        kept = out
        other = head_parallel_sdpa(ql, kl, 2 * vl, scale=d ** -0.5, config=cfg, fused=True,
                                   copy=False)
        torch.cuda.synchronize(dev)
        report.append(f"{(kept.float() - ref.float()).abs().max().item()}")
        aliased = other.data_ptr() != kept.data_ptr()
        multicast = any(e is not None for e in _SYMM_BUFFERS.values())
        queue.put((rank, f"maxdiff {' '.join(report)} multicast {multicast} distinct {aliased}"))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # pragma: no cover - reported to the parent
        queue.put((rank, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("length,hq,hkv,d", [(8192, 32, 8, 128), (4096 + 384, 16, 4, 128),
                                             (4096, 8, 2, 256), (4096, 8, 2, 96),
                                             # dense-tail tiles of 256 blocks: split items, whose
                                             # merged output leaves through the combine kernel
                                             (32768, 16, 4, 128)])
def test_head_parallel_two_gpus_matches_single_gpu(length, hq, hkv, d):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, length, hq, hkv, d, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=300) for _ in procs)
    # No rank is ever killed here (a rank's output buffer may be bound to an
    # NVLink multicast object): one that outlives the join fails the test and
    # leaves on its own through the kernels' bounded waits and the process
    # group's 60 s timeout.
    for p in procs:
        p.join(timeout=120)
    alive = [p.pid for p in procs if p.is_alive()]
    assert not alive, f"ranks still running after 120 s (pids {alive})"
    for rank in (0, 1):
        assert results[rank].startswith("maxdiff 0.0 0.0 0.0 0.0 multicast"), results[rank]
        assert results[rank].endswith("distinct True"), results[rank]
