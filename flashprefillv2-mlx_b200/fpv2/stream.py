"""Host-resident inputs streamed through one GPU (no reference counterpart).

The reference runs on Apple unified memory, where the host and the GPU share
one buffer (fpv2/patch.py:102-174 takes MLX arrays). On a discrete GPU a
caller whose q/k/v live in host memory pays the PCIe copies in and out.
``sdpa_from_host`` hides most of that cost: every selection reduction, list and
K/V read of FPV2 belongs to one KV head (fpv2/selection.py:178-185,
fpv2/kernel.py:212-256), so the layer splits into independent KV-head chunks,
and the host->device copy of chunk c+1, the kernels of chunk c and the
device->host copy of chunk c-1 run at the same time on three CUDA streams.
The copies in set the pace, so the last chunk is cut again into query slices
(chunked prefill: slice [s0, s1) attends the keys up to s1, and only the final
slice keeps the dense tail), which leaves only the last slice's kernels and
copy out after the last byte has come in.

The device staging buffers (two sets of one chunk's q, k and v) are kept per
device for the next call of the same shapes, so a call's first copies in only
wait for the previous call's kernels that read the same set, not for its last
kernels and copies out: back-to-back calls (consecutive layers or requests)
overlap one call's tail with the next call's copies in. ``release_staging``
frees them.

The result equals ``fpv2_sdpa`` on the whole tensors bit for bit whenever the
attention kernel splits the same long work items over KV segments in both (a
choice made per launch from the number of work items; where it differs the
outputs differ by rounding only, well inside the output tolerance).
"""

from __future__ import annotations

import threading
from dataclasses import replace

import torch

from fpv2.patch import _effective_config, fpv2_sdpa
from fpv2.selection import FPV2Config


# device -> [key, buffer sets, events after which each set is free]
_STAGING: dict = {}
# Calls from several host threads queue their work one at a time, so each call
# sees the events of the call before it on the same kept buffers.
_STAGING_LOCK = threading.RLock()


def release_staging(device: torch.device | None = None) -> None:
    """Drop the staging buffers kept by ``sdpa_from_host`` (all devices by
    default); the caching allocator takes them back once their queued copies
    and kernels are done."""
    with _STAGING_LOCK:
        if device is None:
            _STAGING.clear()
        else:
            _STAGING.pop(torch.device(device), None)


def _staging(device, key, make):
    entry = _STAGING.get(device)
    if entry is not None and entry[0] == key:
        return entry, False
    entry = [key, make(), [None, None]]
    _STAGING[device] = entry
    return entry, True


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
    tail_slices: int = 4,
) -> torch.Tensor:
    """``fpv2_sdpa`` for ``[1, H, L, D]`` tensors in (preferably pinned) host memory.

    Returns ``out`` (a new pinned host tensor unless one is given). The work is
    queued on the current CUDA stream of ``device`` and two side streams; the
    current stream waits for the last copy, so synchronising it (or the device)
    makes ``out`` readable. Copies from or to pageable host memory still work but
    do not overlap. ``tail_slices`` (1 = off) cuts the last chunk into that many
    query slices, on boundaries that are multiples of the selection tile and of
    128 rows. Calls from several host threads queue their work one at a time.
    """
    with _STAGING_LOCK:
        return _sdpa_from_host(q, k, v, scale=scale, config=config, out=out,
                               kv_heads_per_chunk=kv_heads_per_chunk, device=device,
                               tail_slices=tail_slices)


def _sdpa_from_host(q, k, v, *, scale, config, out, kv_heads_per_chunk, device, tail_slices):
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
    if not isinstance(tail_slices, int) or tail_slices < 1:
        raise ValueError("tail_slices must be a positive integer")
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    elif out.device.type != "cpu" or out.shape != q.shape or out.dtype != q.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous host tensor shaped and typed like q")
    # one key per GPU for the kept buffers, whichever form the caller names it in
    device = torch.device("cuda") if device is None else torch.device(device)
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    g = hq // hkv
    cs = kv_heads_per_chunk
    nchunks = hkv // cs
    lq, lk = q.shape[2], k.shape[2]
    offset = lk - lq
    eff = _effective_config(config, hq, hkv)
    unit = max(128, eff.tile_q * max(1, eff.last_n_blocks)) if eff is not None else lq
    bounds = _slice_bounds(lq, tail_slices, unit) if offset >= 0 else [(0, lq)]

    compute = torch.cuda.current_stream(device)
    h2d = torch.cuda.Stream(device)
    d2h = torch.cuda.Stream(device)
    # two buffer sets: chunk c uses set c % 2
    def make():
        sets = []
        with torch.cuda.device(device):
            for _ in range(min(2, nchunks)):
                sets.append((torch.empty((1, cs * g) + tuple(q.shape[2:]), dtype=q.dtype, device=device),
                             torch.empty((1, cs) + tuple(k.shape[2:]), dtype=k.dtype, device=device),
                             torch.empty((1, cs) + tuple(v.shape[2:]), dtype=v.dtype, device=device)))
        return sets

    key = (cs, g, tuple(q.shape[2:]), tuple(k.shape[2:]), q.dtype, k.dtype, nchunks > 1)
    entry, fresh = _staging(device, key, make)
    bufs, inputs_free = entry[1], entry[2]
    for t in (x for st in bufs for x in st):
        t.record_stream(h2d)   # this call's copy stream writes them
    if fresh:
        # New buffers come from the compute stream's pool, which only orders their
        # reuse with the compute stream: blocks still read by kernels queued there
        # may be handed out again, so the copy stream starts after that queued work.
        # Kept buffers only wait for the previous call's kernels that read them.
        ready = torch.cuda.Event()
        ready.record(compute)
        h2d.wait_event(ready)
    last = None
    for c in range(nchunks):
        b = c % 2
        qb, kb, vb = bufs[b]
        hs = slice(c * cs * g, (c + 1) * cs * g)
        ks = slice(c * cs, (c + 1) * cs)
        if c == nchunks - 1 and len(bounds) > 1:
            last, inputs_free[b] = _stream_sliced(q, k, v, out, qb, kb, vb, hs, ks, bounds, offset,
                                                  scale, config, compute, h2d, d2h, inputs_free[b])
            break
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


def _slice_bounds(lq: int, tail_slices: int, unit: int) -> list[tuple[int, int]]:
    """Query slices [s0, s1) of the last chunk: about ``tail_slices`` equal
    parts, cut on multiples of ``unit`` rounded up to 128 rows (the selection
    tile and the dense tail), the final slice at least one unit long."""
    unit = (unit + 127) // 128 * 128
    cuts = sorted({(i * lq // tail_slices) // unit * unit for i in range(1, tail_slices)} - {0})
    while cuts and lq - cuts[-1] < unit:
        cuts.pop()
    return list(zip([0] + cuts, cuts + [lq]))


def _stream_sliced(q, k, v, out, qb, kb, vb, hs, ks, bounds, offset, scale, config,
                   compute, h2d, d2h, inputs_free):
    """The last chunk in query slices: its K and V come in first, then the query
    rows slice by slice (one copy per head: a slice is strided across heads);
    slice i runs as soon as its rows have arrived and goes out right after.
    Returns the event of the last copy out and that of the last kernels that
    read the buffer set."""
    heads = range(hs.start, hs.stop)
    loaded = []
    with torch.cuda.stream(h2d):
        if inputs_free is not None:
            h2d.wait_event(inputs_free)   # chunk c-2's kernels have read this set
        kb.copy_(k[:, ks], non_blocking=True)
        vb.copy_(v[:, ks], non_blocking=True)
        for s0, s1 in bounds:
            for j, h in enumerate(heads):
                qb[0, j, s0:s1].copy_(q[0, h, s0:s1], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(h2d)
            loaded.append(ev)
    last = None
    for i, (s0, s1) in enumerate(bounds):
        final = i == len(bounds) - 1
        compute.wait_event(loaded[i])
        with torch.cuda.stream(compute):
            # queries [s0, s1) attend the keys before offset + s1; only the final
            # slice holds the layer's last tiles (the dense tail)
            cfg = config if final else replace(config, last_n_blocks=0)
            kend = offset + s1
            o = fpv2_sdpa(qb[:, :, s0:s1], kb[:, :, :kend], vb[:, :, :kend], scale=scale, config=cfg)
            done = torch.cuda.Event()
            done.record(compute)
        with torch.cuda.stream(d2h):
            d2h.wait_event(done)
            for j, h in enumerate(heads):
                out[0, h, s0:s1].copy_(o[0, j], non_blocking=True)
            last = torch.cuda.Event()
            last.record(d2h)
        o.record_stream(d2h)
    return last, done
