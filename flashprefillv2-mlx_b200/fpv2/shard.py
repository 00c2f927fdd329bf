"""Head-parallel FlashPrefill V2 across the GPUs of one node (one process per GPU).

Every reduction of the index stage, every block list and every K/V read of the
attention belongs to one KV head (fpv2/selection.py:178-185,
fpv2/kernel.py:212-256 of the reference), so the layer splits over KV heads with
no collective inside the hot path: rank r owns KV heads
``[r*Hkv/P, (r+1)*Hkv/P)`` and their query heads, runs the fused index stage and
the sparse attention on them, and a single all-gather reassembles the output
``[Hq, L, D]`` (NCCL over NVLink/NVSwitch on GPUs; any torch.distributed backend
works for the host logic).
"""

from __future__ import annotations

from dataclasses import dataclass
from datetime import timedelta

import torch
import torch.distributed as dist

from fpv2.patch import fpv2_sdpa
from fpv2.selection import FPV2Config


@dataclass(frozen=True)
class HeadShard:
    """KV-head and query-head ranges owned by one rank."""

    rank: int
    world: int
    kv_start: int
    kv_end: int
    q_start: int
    q_end: int


def head_shard(query_heads: int, kv_heads: int, world: int, rank: int) -> HeadShard:
    """Contiguous KV-head block of ``rank`` (KV heads must divide evenly over ranks)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if not kv_heads or query_heads % kv_heads:
        raise ValueError("query heads must be divisible by KV heads")
    if kv_heads % world:
        raise ValueError(f"{kv_heads} KV heads cannot be split evenly over {world} ranks")
    per = kv_heads // world
    group = query_heads // kv_heads
    kv_start = rank * per
    return HeadShard(rank, world, kv_start, kv_start + per, kv_start * group,
                     (kv_start + per) * group)


def shard_inputs(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, shard: HeadShard):
    """Slice ``[B, H, L, D]`` tensors to this rank's heads (contiguous copies)."""
    return (q[:, shard.q_start:shard.q_end].contiguous(),
            k[:, shard.kv_start:shard.kv_end].contiguous(),
            v[:, shard.kv_start:shard.kv_end].contiguous())


def gather_heads(local: torch.Tensor, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather ``[B, H/P, L, D]`` shards along the head axis into ``[B, H, L, D]``."""
    world = dist.get_world_size(group)
    if world == 1:
        return local
    local = local.contiguous()
    b, h, l, d = local.shape
    if out is None:
        out = torch.empty((world, b, h, l, d), dtype=local.dtype, device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out.view(-1), local.view(-1), group=group)
    else:
        dist.all_gather(list(out.unbind(0)), local, group=group)
    return out.permute(1, 0, 2, 3, 4).reshape(b, world * h, l, d)


_SYMM_BUFFERS: dict = {}


def _multicast_buffer(shape, dtype, device, group):
    """Full-output buffer in torch symmetric memory, bound to an NVLink multicast
    object across the group (cached per shape). Returns (tensor, handle,
    multicast address of the tensor) or None when the GPUs offer no multicast."""
    key = (tuple(shape), dtype, device, id(group))
    if key in _SYMM_BUFFERS:
        return _SYMM_BUFFERS[key]
    import torch.distributed._symmetric_memory as symm_mem

    grp = group if group is not None else dist.group.WORLD
    buf = symm_mem.empty(*shape, dtype=dtype, device=device)
    handle = symm_mem.rendezvous(buf, grp)
    entry = None
    mc_base = int(getattr(handle, "multicast_ptr", 0) or 0)
    if mc_base:
        # the tensor's offset inside the symmetric allocation is the same in the
        # local mapping and in the multicast mapping
        off = buf.data_ptr() - int(handle.buffer_ptrs[handle.rank])
        if 0 <= off and off + buf.numel() * buf.element_size() <= int(handle.buffer_size):
            entry = (buf, handle, mc_base + off)
    _SYMM_BUFFERS[key] = entry
    return entry


def head_parallel_sdpa(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    scale: float,
    config: FPV2Config = FPV2Config(),
    group=None,
    fused: bool | None = None,
    copy: bool = True,
) -> torch.Tensor:
    """FPV2 on this rank's head shard (``[1, Hq/P, L, D]``, ``[1, Hkv/P, L, D]``);
    every rank returns the full ``[1, Hq, L, D]`` output.

    Fused (the default where the GPUs support NVLink multicast): the attention
    kernel writes each finished output tile straight into every rank's copy of
    the full output through the multicast address (torch symmetric memory), so
    the reassembly overlaps the computation. That buffer is cached per shape and
    reused by the next call of the same shape (every layer of a model), so by
    default the result is copied out of it; ``copy=False`` returns the buffer
    itself, valid only until the next call with the same shape (for callers that
    consume the output before the next layer). Otherwise one NCCL all-gather
    follows the kernel and the result is a fresh tensor either way."""
    from fpv2 import _lib
    from fpv2.patch import _effective_config

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    hq, lq, d = q.shape[1], q.shape[2], q.shape[3]
    eff = _effective_config(config, hq, k.shape[1])
    if fused is None:
        fused = (world > 1 and eff is not None and q.is_cuda
                 and dist.get_backend(group) == "nccl"
                 and _lib.fast_path_mask(q.dtype, hq, k.shape[1], d, eff.block_k, eff.tile_q, 1) & 2)
    entry = None
    if fused:
        lq_pad = (lq + eff.tile_q - 1) // eff.tile_q * eff.tile_q
        entry = _multicast_buffer((world * hq, lq_pad, d), q.dtype, q.device, group)
    if entry is None:
        local = fpv2_sdpa(q, k, v, scale=scale, config=config)
        return gather_heads(local, group)
    buf, handle, mc_addr = entry
    rank = dist.get_rank(group)
    handle.barrier(channel=0)   # no rank still reads the previous contents
    fpv2_sdpa(q, k, v, scale=scale, config=config, multicast=(mc_addr, rank * hq, world * hq))
    handle.barrier(channel=0)   # every rank's tiles have landed in every buffer
    out = buf[None, :, :lq, :]
    return out.clone() if copy else out


class RankMonitor:
    """Host-side liveness check between steps (failure detection without a GPU fault).

    Holds a ``gloo`` side group; :meth:`check` runs a monitored barrier that
    raises within ``timeout_s`` naming any rank that has died or stopped
    stepping, so the survivors learn of it before they launch the next step's
    kernels and collectives.
    """

    def __init__(self, timeout_s: float = 30.0):
        self.timeout = timedelta(seconds=timeout_s)
        self.group = dist.new_group(backend="gloo") if dist.get_world_size() > 1 else None

    def check(self) -> None:
        if self.group is not None:
            dist.monitored_barrier(group=self.group, timeout=self.timeout, wait_all_ranks=True)
