"""Host-resident inputs streamed through one GPU (no reference counterpart).

The reference runs on Apple unified memory, where the host and the GPU share
one buffer (fpv2/patch.py:102-174 takes MLX arrays). On a discrete GPU a
caller whose q/k/v live in host memory pays the PCIe copies in and out.
``sdpa_from_host`` hides most of that cost: every selection reduction, list and
K/V read of FPV2 belongs to one KV head (fpv2/selection.py:178-185,
fpv2/kernel.py:212-256), so the layer splits into independent KV-head chunks,
and the host->device copy of chunk c+1, the kernels of chunk c and the
device->host copy of chunk c-1 run at the same time on three CUDA streams.
The result equals ``fpv2_sdpa`` on the whole tensors bit for bit.
"""

from __future__ import annotations

import torch

from fpv2.patch import fpv2_sdpa
from fpv2.selection import FPV2Config


def sdpa_from_host(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    scale: float,
    config: FPV2Config = FPV2Config(),
    out: torch.Tensor | None = None,
    kv_heads_per_chunk: int = 1,
    device: torch.device | None = None,
) -> torch.Tensor:
    """``fpv2_sdpa`` for ``[1, H, L, D]`` tensors in (preferably pinned) host memory.

    Returns ``out`` (a new pinned host tensor unless one is given). The work is
    queued on the current CUDA stream of ``device`` and two side streams; the
    current stream waits for the last copy, so synchronising it (or the device)
    makes ``out`` readable. Copies from or to pageable host memory still work but
    do not overlap.
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.device.type != "cpu":
            raise ValueError(f"{name} must be a host tensor; use fpv2_sdpa for device tensors")
        if t.ndim != 4 or t.shape[0] != 1:
            raise ValueError("q, k, and v must have shape [1, heads, sequence, dim]")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    hq, hkv = q.shape[1], k.shape[1]
    if v.shape[1] != hkv or hq % hkv != 0:
        raise ValueError("query heads must be a multiple of the key/value heads")
    if kv_heads_per_chunk <= 0 or hkv % kv_heads_per_chunk != 0:
        raise ValueError("kv_heads_per_chunk must divide the number of key/value heads")
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    elif out.device.type != "cpu" or out.shape != q.shape or out.dtype != q.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous host tensor shaped and typed like q")
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    g = hq // hkv
    cs = kv_heads_per_chunk
    nchunks = hkv // cs

    compute = torch.cuda.current_stream(device)
    h2d = torch.cuda.Stream(device)
    d2h = torch.cuda.Stream(device)
    # two buffer sets: chunk c uses set c % 2
    bufs = []
    with torch.cuda.device(device):
        for _ in range(min(2, nchunks)):
            qb = torch.empty((1, cs * g) + tuple(q.shape[2:]), dtype=q.dtype, device=device)
            kb = torch.empty((1, cs) + tuple(k.shape[2:]), dtype=k.dtype, device=device)
            vb = torch.empty((1, cs) + tuple(v.shape[2:]), dtype=v.dtype, device=device)
            for t in (qb, kb, vb):
                t.record_stream(h2d)
            bufs.append((qb, kb, vb))
    # The buffers come from the compute stream's pool, which only orders their
    # reuse with the compute stream: blocks still read by kernels queued there
    # (the previous call's lists, scratch, inputs) may be handed out again. The
    # copy stream starts after the compute stream's queued work for that reason.
    ready = torch.cuda.Event()
    ready.record(compute)
    h2d.wait_event(ready)
    inputs_free: list[torch.cuda.Event | None] = [None, None]
    last = None
    for c in range(nchunks):
        b = c % 2
        qb, kb, vb = bufs[b]
        hs = slice(c * cs * g, (c + 1) * cs * g)
        ks = slice(c * cs, (c + 1) * cs)
        with torch.cuda.stream(h2d):
            if inputs_free[b] is not None:
                h2d.wait_event(inputs_free[b])   # chunk c-2's kernels have read this set
            qb.copy_(q[:, hs], non_blocking=True)
            kb.copy_(k[:, ks], non_blocking=True)
            vb.copy_(v[:, ks], non_blocking=True)
            loaded = torch.cuda.Event()
            loaded.record(h2d)
        compute.wait_event(loaded)
        with torch.cuda.stream(compute):
            o = fpv2_sdpa(qb, kb, vb, scale=scale, config=config)
            done = torch.cuda.Event()
            done.record(compute)
        inputs_free[b] = done
        with torch.cuda.stream(d2h):
            d2h.wait_event(done)
            out[:, hs].copy_(o, non_blocking=True)
            last = torch.cuda.Event()
            last.record(d2h)
        o.record_stream(d2h)
    if last is not None:
        compute.wait_event(last)
    return out
