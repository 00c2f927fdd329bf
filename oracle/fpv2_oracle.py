"""CPU oracle for the FlashPrefill V2 index and attention stages (NumPy).

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this module.
Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of
``bench.py`` (and its ``--impl reference`` arm) may import or run it, and only
as the checker or the timed CPU baseline, never as the thing measured.

It restates the reference's algorithm for the hot path on plain NumPy arrays:

* ``pool_blocks``              fpv2/selection.py:68-80
* ``block_scores_and_select``  fpv2/selection.py:109-201 (with offset,
  padded query rows and query-tile chunking)
* ``density``                  fpv2/selection.py:204-229
* ``compact_block_indices``    fpv2/kernel.py:141-184
* ``sparse_attention``         fpv2/kernel.py:187-414 and 441-590: list-driven
  online softmax in base 2, ``finite_min`` masking, the ``+log2(block_k)``
  pooled correction, pooled K/V cast to the query dtype (kernel.py:553-554)
  and list clipping (kernel.py:555-558)
* ``fpv2_attention_reference`` fpv2/reference.py:10-90 (dense, fp32)
* ``fpv2_attention_blockwise`` the same math as fpv2/reference.py, evaluated
  per (KV head, query tile) over retained blocks only, so that 16k-64k
  token checks fit in host memory
* ``effective_config``, ``request_config``, ``causal_block_count`` and
  ``fpv2_sdpa``                fpv2/patch.py:41-76 and 102-174

Parity status. The reference needs MLX 0.32.2 on an Apple GPU, which cannot be
installed here, so its own outputs cannot be produced in this container. The
oracle is pinned by the reference's deterministic known-answer tests
(tests/test_selection.py:12-87, tests/test_kernel.py:66-77,
tests/test_patch.py:27-41 and 180-201), transcribed into
``tests/golden/reference_kats.json`` and checked by ``tests/test_oracle.py``.
MLX's own rounding and accumulation order inside ``mx.mean``, ``mx.einsum`` and
``mx.exp`` is not reproducible without MLX and is *parity unpinned*; this
oracle defines it as follows.

* Pooling: exact mean (float64 sum of the block, divided by the block size),
  rounded to float32 and then, when the output dtype is bfloat16 or float16, to
  that dtype with round-to-nearest-even.  The CUDA pooling kernel implements
  the same definition, so pooled values are compared bit for bit.
* Scores and energies: float32 products and sums, as the reference asks for
  (``astype(mx.float32)`` before the einsum, selection.py:154-158).  A float64
  twin (``precision="fp64"``) gives the energies used to classify threshold
  flips: a block whose float64 energy lies within a relative ``1e-5`` of
  ``alpha * max`` may legitimately land on either side.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace
from typing import Any

import numpy as np

FINITE_MIN = np.float32(-np.finfo(np.float32).max)
LOG2E = 1.4426950408889634
SUPPORTED_HEAD_DIMS = (64, 96, 128, 256)


# --------------------------------------------------------------------------
# Rounding helpers (bfloat16 has no NumPy dtype; values are carried in fp32)
# --------------------------------------------------------------------------


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 (nearest-even), returned as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000
    out = rounded.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), np.float32(np.nan), out).astype(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` ("fp32", "bf16", "fp16"), as float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "fp32":
        return x
    if dtype == "bf16":
        return round_to_bf16(x)
    if dtype == "fp16":
        return x.astype(np.float16).astype(np.float32)
    raise ValueError(f"unknown dtype {dtype}")


# --------------------------------------------------------------------------
# Config record (same fields and validation as fpv2/selection.py:30-65)
# --------------------------------------------------------------------------


@dataclass(frozen=True)
class OracleConfig:
    block_k: int = 128
    tile_q: int = 128
    alpha: float = 0.1
    sink_tokens: int = 256
    window_tokens: int = 384
    last_n_blocks: int = 2
    mean_correction: bool = True
    score_chunk_tiles: int | None = None
    pack_gqa: bool = False


def as_config(config: Any) -> OracleConfig:
    """Copy any FPV2Config-like object into an ``OracleConfig``."""
    if config is None:
        return OracleConfig()
    if isinstance(config, OracleConfig):
        return config
    return OracleConfig(
        block_k=int(config.block_k),
        tile_q=int(config.tile_q),
        alpha=float(config.alpha),
        sink_tokens=int(config.sink_tokens),
        window_tokens=int(config.window_tokens),
        last_n_blocks=int(config.last_n_blocks),
        mean_correction=bool(config.mean_correction),
        score_chunk_tiles=config.score_chunk_tiles,
        pack_gqa=bool(config.pack_gqa),
    )


# --------------------------------------------------------------------------
# Index stage
# --------------------------------------------------------------------------


def pool_blocks(x: np.ndarray, block_size: int = 128, out_dtype: str = "fp32") -> np.ndarray:
    """Mean over each ``block_size`` run of the sequence axis.

    Follows fpv2/selection.py:68-80 (error message ``divisible`` included).
    The mean is exact (float64 sum), rounded to float32, then to ``out_dtype``.
    """
    x = np.asarray(x)
    if x.ndim < 2:
        raise ValueError("x must have at least sequence and feature dimensions")
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    length, head_dim = x.shape[-2:]
    if length % block_size:
        raise ValueError(
            f"sequence length {length} must be divisible by block_size {block_size}"
        )
    shape = (*x.shape[:-2], length // block_size, block_size, head_dim)
    mean = x.astype(np.float64).reshape(shape).sum(axis=-2) / block_size
    return round_to(mean.astype(np.float32), out_dtype)


def _validate_select(q, pooled_k, config, offset, query_length):
    """fpv2/selection.py:83-106."""
    if q.ndim != 3 or pooled_k.ndim != 3:
        raise ValueError("q and pooled_k must have shape [heads, sequence, dim]")
    query_heads, padded_length, head_dim = q.shape
    kv_heads, num_blocks, key_dim = pooled_k.shape
    if not kv_heads or query_heads % kv_heads:
        raise ValueError("query heads must be divisible by KV heads")
    if head_dim != key_dim:
        raise ValueError("q and pooled_k head dimensions must match")
    if padded_length % config.tile_q:
        raise ValueError("query length must be padded to a multiple of tile_q")
    if not 0 < query_length <= padded_length:
        raise ValueError("query_length must be in (0, q.shape[-2]]")
    if offset < 0:
        raise ValueError("offset must be non-negative")
    if offset + query_length > num_blocks * config.block_k:
        raise ValueError("queries extend beyond the represented key sequence")
    return query_heads, kv_heads, padded_length, num_blocks


@dataclass
class SelectionResult:
    selected: np.ndarray            # bool [Hkv, Nt, Nb]
    raw_scores: np.ndarray | None   # [Hkv, G, Lq_pad, Nb] (unchunked only)
    energies: np.ndarray            # [Hkv, Nt, Nb] in the working precision
    threshold: np.ndarray           # [Hkv, Nt] alpha * max energy


def block_scores_and_select(
    q: np.ndarray,
    pooled_k: np.ndarray,
    *,
    scale: float,
    config: Any = None,
    offset: int = 0,
    query_length: int | None = None,
    precision: str = "fp32",
    keep_scores: bool | None = None,
    only_tiles=None,
) -> SelectionResult:
    """Selection mask ``[Hkv, Nt, Nb]`` following fpv2/selection.py:109-201.

    ``precision`` is "fp32" (the reference's arithmetic) or "fp64" (used to
    classify threshold flips).  Raw scores are kept only when the query-tile
    chunking is off, as in selection.py:196-201.  ``only_tiles`` (not in the
    reference) evaluates only the listed query tiles, each on its own; every
    tile's selection depends on its own rows alone, so the result rows equal
    the corresponding rows of the full mask, shaped ``[Hkv, len(only_tiles), Nb]``.
    ``q`` may be any float array; it is converted to float32 per tile chunk.
    """
    config = as_config(config)
    q = np.asarray(q)
    if q.dtype not in (np.float32, np.float16, np.float64):
        q = q.astype(np.float32)
    pooled_k = np.asarray(pooled_k, dtype=np.float32)
    valid_length = q.shape[-2] if query_length is None else query_length
    query_heads, kv_heads, padded_length, num_blocks = _validate_select(
        q, pooled_k, config, offset, valid_length
    )
    ftype = np.float64 if precision == "fp64" else np.float32
    group = query_heads // kv_heads
    num_tiles = padded_length // config.tile_q
    grouped_q = q.reshape(kv_heads, group, padded_length, q.shape[-1])
    pk = pooled_k.astype(ftype)
    block_starts = np.arange(num_blocks, dtype=np.int64) * config.block_k
    block_ends = block_starts + config.block_k
    sink = block_starts < config.sink_tokens
    chunk_tiles = config.score_chunk_tiles or num_tiles
    if only_tiles is None:
        groups = [(t, min(t + chunk_tiles, num_tiles)) for t in range(0, num_tiles, chunk_tiles)]
    else:
        groups = [(int(t), int(t) + 1) for t in only_tiles]
        keep_scores = False
    if keep_scores is None:
        keep_scores = config.score_chunk_tiles is None
    selected_chunks, energy_chunks, thr_chunks = [], [], []
    raw_scores = (
        np.empty((kv_heads, group, padded_length, num_blocks), dtype=ftype)
        if keep_scores
        else None
    )
    scale_f = ftype(scale)
    alpha_f = ftype(np.float32(config.alpha))
    for tile_start, tile_end in groups:
        row_start = tile_start * config.tile_q
        row_end = tile_end * config.tile_q
        row_ids = np.arange(row_start, row_end, dtype=np.int64)
        tile_ids = np.arange(tile_start, tile_end, dtype=np.int64)
        tile_first = offset + tile_ids * config.tile_q
        tile_last = np.minimum(tile_first + config.tile_q, offset + valid_length) - 1
        rows_q = grouped_q[:, :, row_start:row_end, :].astype(np.float32).astype(ftype)
        scores = np.matmul(rows_q, pk.transpose(0, 2, 1)[:, None])
        scores = scores * scale_f
        if raw_scores is not None:
            raw_scores[:, :, row_start:row_end, :] = scores
        positions = offset + row_ids
        row_visible = (block_starts[None, :] <= positions[:, None]) & (
            row_ids[:, None] < valid_length
        )
        nt = tile_end - tile_start
        tiles = np.where(row_visible[None, None], scores, -np.inf).reshape(
            kv_heads, group, nt, config.tile_q, num_blocks
        )
        fully_visible = block_ends[None, :] <= tile_last[:, None] + 1
        tiles = np.where(fully_visible[None, None, :, None, :], tiles, -np.inf)
        tile_max = tiles.max(axis=(1, 3, 4), keepdims=True)
        finite = tiles > -np.inf
        with np.errstate(invalid="ignore", over="ignore"):
            expo = np.exp(np.where(finite, tiles - tile_max, -np.inf))
        energies = np.where(finite, expo, 0).astype(ftype).sum(axis=(1, 3))
        threshold = alpha_f * energies.max(axis=-1)
        if ftype is np.float32:
            threshold = threshold.astype(np.float32)
        sel = energies >= threshold[..., None]
        visible = block_starts[None, :] <= tile_last[:, None]
        local = block_ends[None, :] > (tile_first[:, None] - config.window_tokens)
        dense_tail = tile_ids >= max(num_tiles - config.last_n_blocks, 0)
        forced = sink[None, :] | local | dense_tail[:, None]
        selected_chunks.append((sel | forced[None]) & visible[None])
        energy_chunks.append(energies)
        thr_chunks.append(threshold)
    return SelectionResult(
        selected=np.concatenate(selected_chunks, axis=1),
        raw_scores=raw_scores,
        energies=np.concatenate(energy_chunks, axis=1),
        threshold=np.concatenate(thr_chunks, axis=1),
    )


def threshold_band(result64: SelectionResult, rel: float = 1e-5) -> np.ndarray:
    """Blocks whose float64 energy is within ``rel`` of the alpha threshold."""
    thr = result64.threshold[..., None]
    return np.abs(result64.energies - thr) <= rel * np.abs(thr)


def density(selected: np.ndarray, *, config: Any = None, offset: int = 0,
            query_length: int | None = None) -> float:
    """fpv2/selection.py:204-229."""
    config = as_config(config)
    if selected.ndim != 3:
        raise ValueError("selected must have shape [KV heads, tiles, blocks]")
    kv_heads, num_tiles, num_blocks = selected.shape
    if offset < 0:
        raise ValueError("offset must be non-negative")
    valid = num_tiles * config.tile_q if query_length is None else query_length
    if not 0 < valid <= num_tiles * config.tile_q:
        raise ValueError("query_length is inconsistent with selected tiles")
    tile_last = np.minimum(
        offset + (np.arange(num_tiles) + 1) * config.tile_q, offset + valid
    ) - 1
    block_starts = np.arange(num_blocks) * config.block_k
    visible = block_starts[None, :] <= tile_last[:, None]
    denominator = np.float32(visible.sum()) * kv_heads
    return float(np.float32(selected.sum()) / np.float32(denominator))


def compact_block_indices(
    selected: np.ndarray,
    *,
    config: Any = None,
    offset: int = 0,
    query_length: int | None = None,
    key_length: int | None = None,
):
    """Padded selected/pruned lists and counts (fpv2/kernel.py:141-184).

    Order: the selected (or pruned) blocks ascending, then every other block
    ascending.  The reference pins only the ascending prefix
    (tests/test_kernel.py:66-72); this stable order defines the padding.
    """
    config = as_config(config)
    selected = np.asarray(selected)
    if selected.ndim != 3:
        raise ValueError("selected must have shape [KV heads, tiles, blocks]")
    if selected.dtype != np.bool_:
        raise ValueError("selected must have boolean dtype")
    _, num_tiles, num_blocks = selected.shape
    padded_q = num_tiles * config.tile_q
    valid_q = padded_q if query_length is None else query_length
    represented_k = num_blocks * config.block_k
    valid_k = represented_k if key_length is None else key_length
    if offset < 0:
        raise ValueError("offset must be non-negative")
    if not 0 < valid_q <= padded_q:
        raise ValueError("query_length is inconsistent with selected tiles")
    if not 0 < valid_k <= represented_k:
        raise ValueError("key_length is inconsistent with selected blocks")
    if offset + valid_q > valid_k:
        raise ValueError("queries extend beyond key_length")
    sel_ids = np.argsort(~selected, axis=-1, kind="stable").astype(np.int32)
    sel_counts = selected.sum(axis=-1).astype(np.int32)
    tile_first = offset + np.arange(num_tiles) * config.tile_q
    block_ends = np.minimum((np.arange(num_blocks) + 1) * config.block_k, valid_k)
    fully_past = block_ends[None, :] <= tile_first[:, None]
    pruned = (~selected) & fully_past[None]
    pr_ids = np.argsort(~pruned, axis=-1, kind="stable").astype(np.int32)
    pr_counts = pruned.sum(axis=-1).astype(np.int32)
    return sel_ids, sel_counts, pr_ids, pr_counts


def lists_to_mask(ids: np.ndarray, counts: np.ndarray, num_blocks: int) -> np.ndarray:
    """Inverse of compaction for the counted prefix."""
    mask = np.zeros((*counts.shape, num_blocks), dtype=bool)
    for idx in np.ndindex(counts.shape):
        mask[idx][ids[idx][: counts[idx]]] = True
    return mask


# --------------------------------------------------------------------------
# Attention stage
# --------------------------------------------------------------------------


def sparse_attention(
    q, k, v, pooled_k, pooled_v, selected_ids, selected_counts, pruned_ids, pruned_counts,
    *, scale: float, config: Any = None, offset: int = 0,
    query_length: int | None = None, key_length: int | None = None,
    dtype: str = "bf16", tiles: list[tuple[int, int]] | None = None,
    pooled_dtype: str | None = None, p_dtype: str | None = None, out_dtype: str | None = None,
) -> np.ndarray:
    """List-driven FPV2 attention, fpv2/kernel.py:187-414 and 441-590.

    Per query row ``o = (sum_sel 2^(s2-m) v + sum_pruned 2^(s2p + log2 bk - m) vbar) / l``
    with ``s2 = scale*log2(e)*q.k``, masked logits at ``finite_min``, pooled K/V
    rounded to ``dtype`` (kernel.py:553-554) and lists clipped (kernel.py:555-558).
    Inputs are float32 arrays carrying ``dtype`` values; the output is rounded
    to ``dtype`` as the kernel stores it (kernel.py:409).  Rows at or beyond
    ``query_length`` are padding and are returned as zeros.  ``tiles``
    restricts the evaluation to the listed (kv_head, tile) pairs.

    Rounding controls (not in the reference; they decompose the error budget
    of an implementation): ``pooled_dtype`` overrides the cast of the pooled
    K/V ("fp32" keeps them), ``p_dtype`` rounds the probabilities P to a
    16-bit type before the P.V product (the row sums keep the unrounded P),
    ``out_dtype`` overrides the rounding of the stored output ("fp32": none).
    """
    config = as_config(config)
    q = np.asarray(q)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    hq, lq_pad, d = q.shape
    hkv, lk_pad, _ = k.shape
    g = hq // hkv
    nt = lq_pad // config.tile_q
    nb = lk_pad // config.block_k
    valid_q = lq_pad if query_length is None else query_length
    valid_k = lk_pad if key_length is None else key_length
    pk = round_to(np.asarray(pooled_k, np.float32), pooled_dtype or dtype)
    pv = round_to(np.asarray(pooled_v, np.float32), pooled_dtype or dtype)
    sel_ids = np.clip(selected_ids, 0, nb - 1)
    sel_counts = np.clip(selected_counts, 0, nb)
    pr_ids = np.clip(pruned_ids, 0, nb - 1)
    pr_counts = np.clip(pruned_counts, 0, nb)
    c2 = np.float32(scale * LOG2E)
    corr_shift = np.float32(math.log2(config.block_k))
    out = np.zeros((hq, lq_pad, d), dtype=np.float32)
    if tiles is None:
        tiles = [(h, t) for h in range(hkv) for t in range(nt)]
    for h, t in tiles:
        rows = np.arange(t * config.tile_q, (t + 1) * config.tile_q)
        rows = rows[rows < valid_q]
        if rows.size == 0:
            continue
        positions = offset + rows
        qt = q[h * g:(h + 1) * g][:, rows, :].astype(np.float32)   # [g, r, d]
        key_idx = []
        for b in sel_ids[h, t, : sel_counts[h, t]]:
            start = int(b) * config.block_k
            if start > positions[-1]:
                break
            key_idx.append(np.arange(start, start + config.block_k))
        keys = np.concatenate(key_idx) if key_idx else np.zeros(0, np.int64)
        s = np.matmul(qt, k[h, keys].T) * c2 if keys.size else np.zeros((g, rows.size, 0), np.float32)
        mask = (keys[None, :] <= positions[:, None]) & (keys[None, :] < valid_k)
        s = np.where(mask[None], s, FINITE_MIN).astype(np.float32)
        vals = v[h, keys]
        if config.mean_correction and pr_counts[h, t] > 0:
            blocks = pr_ids[h, t, : pr_counts[h, t]]
            sc = np.matmul(qt, pk[h, blocks].T) * c2 + corr_shift
            s = np.concatenate([s, sc.astype(np.float32)], axis=-1)
            vals = np.concatenate([vals, pv[h, blocks]], axis=0)
        m = s.max(axis=-1, keepdims=True) if s.shape[-1] else np.zeros((g, rows.size, 1), np.float32)
        p = np.exp2(s - m)
        pr = p if p_dtype is None else round_to(p.astype(np.float32), p_dtype)
        o = np.matmul(pr, vals) / p.sum(axis=-1, keepdims=True)
        out[h * g:(h + 1) * g, rows, :] = o
    return round_to(out, out_dtype or dtype)


def exact_causal_attention(q, k, v, scale: float, offset: int = 0) -> np.ndarray:
    """Plain causal softmax attention in fp32 (tests/test_reference.py:10-26)."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    hq, lq, d = q.shape
    hkv, lk, _ = k.shape
    g = hq // hkv
    gq = q.reshape(hkv, g, lq, d)
    s = np.matmul(gq, k.transpose(0, 2, 1)[:, None]) * np.float32(scale)
    causal = np.arange(lk)[None, :] <= (offset + np.arange(lq)[:, None])
    s = np.where(causal[None, None], s, -np.inf)
    s = s - s.max(axis=-1, keepdims=True)
    w = np.exp(s)
    w /= w.sum(axis=-1, keepdims=True)
    return np.matmul(w, v[:, None]).reshape(hq, lq, d).astype(np.float32)


def fpv2_attention_reference(q, k, v, *, scale: float, config: Any = None, offset: int = 0):
    """Dense fp32 FPV2 output, fpv2/reference.py:10-90 (memory O(Hq*Lq*Lk))."""
    config = as_config(config)
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    if q.ndim != 3 or k.ndim != 3 or v.ndim != 3:
        raise ValueError("q, k, and v must have shape [heads, sequence, dim]")
    if k.shape != v.shape:
        raise ValueError("k and v must have identical shapes")
    if q.shape[-1] != k.shape[-1]:
        raise ValueError("q, k, and v head dimensions must match")
    if q.shape[0] % k.shape[0]:
        raise ValueError("query heads must be divisible by KV heads")
    if q.shape[1] % config.tile_q or k.shape[1] % config.block_k:
        raise ValueError("q and k/v sequence lengths must be tile/block aligned")
    if offset < 0 or offset + q.shape[1] > k.shape[1]:
        raise ValueError("offset does not align queries within the key sequence")
    hq, lq, d = q.shape
    hkv, lk, _ = k.shape
    g = hq // hkv
    nt = lq // config.tile_q
    nb = lk // config.block_k
    gq = q.reshape(hkv, g, lq, d)
    pk = pool_blocks(k, config.block_k, "fp32")
    pv = pool_blocks(v, config.block_k, "fp32")
    sel = block_scores_and_select(q, pk, scale=scale, config=config, offset=offset)
    selected = sel.selected
    pooled_scores = sel.raw_scores
    if pooled_scores is None:
        pooled_scores = np.matmul(gq, pk.transpose(0, 2, 1)[:, None]) * np.float32(scale)
    token_scores = np.matmul(gq, k.transpose(0, 2, 1)[:, None]) * np.float32(scale)
    qpos = offset + np.arange(lq)
    kpos = np.arange(lk)
    causal = kpos[None, :] <= qpos[:, None]
    sel_tokens = np.repeat(np.repeat(selected, config.tile_q, axis=1), config.block_k, axis=2)[:, :lq, :lk]
    kept = sel_tokens[:, None] & causal[None, None]
    exact = np.where(kept, token_scores, -np.inf)
    if config.mean_correction:
        tile_first = offset + np.arange(nt) * config.tile_q
        block_ends = (np.arange(nb) + 1) * config.block_k
        fully_past = block_ends[None, :] <= tile_first[:, None]
        corrected = (~selected) & fully_past[None]
        rows = np.repeat(corrected, config.tile_q, axis=1)
        corr = np.where(rows[:, None], pooled_scores + np.float32(math.log(config.block_k)), -np.inf)
    else:
        corr = np.full_like(pooled_scores, -np.inf)
    row_max = np.maximum(exact.max(axis=-1, keepdims=True), corr.max(axis=-1, keepdims=True))
    ew = np.exp(exact - row_max)
    cw = np.exp(corr - row_max)
    num = np.matmul(ew, v[:, None]) + np.matmul(cw, pv[:, None])
    den = ew.sum(axis=-1, keepdims=True) + cw.sum(axis=-1, keepdims=True)
    return (num / den).reshape(hq, lq, d).astype(np.float32)


def fpv2_attention_blockwise(
    q, k, v, *, scale: float, config: Any = None, offset: int = 0,
    selected: np.ndarray | None = None, tiles: list[tuple[int, int]] | None = None,
    pooled_dtype: str = "fp32",
) -> np.ndarray:
    """fpv2/reference.py:10-90 evaluated per (KV head, tile) over retained blocks.

    Same result as ``fpv2_attention_reference`` without the O(Lq*Lk) tensors.
    ``selected`` may be supplied (else it is computed on fp32 pooled K, as
    reference.py:45-51 does); ``tiles`` restricts the (kv_head, tile) pairs
    evaluated (the others stay zero).
    """
    config = as_config(config)
    q = np.asarray(q)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    hq, lq, d = q.shape
    hkv, lk, _ = k.shape
    g = hq // hkv
    nt = lq // config.tile_q
    nb = lk // config.block_k
    pk = pool_blocks(k, config.block_k, pooled_dtype)
    pv = pool_blocks(v, config.block_k, pooled_dtype)
    if selected is None:
        cfg = replace(config, score_chunk_tiles=config.score_chunk_tiles or max(1, 8192 // config.tile_q))
        selected = block_scores_and_select(q, pk, scale=scale, config=cfg, offset=offset).selected
    out = np.zeros((hq, lq, d), dtype=np.float32)
    sc = np.float32(scale)
    lnbk = np.float32(math.log(config.block_k))
    if tiles is None:
        tiles = [(h, t) for h in range(hkv) for t in range(nt)]
    block_ends = (np.arange(nb) + 1) * config.block_k
    for h, t in tiles:
        rows = np.arange(t * config.tile_q, (t + 1) * config.tile_q)
        positions = offset + rows
        qt = q[h * g:(h + 1) * g][:, rows, :].astype(np.float32)
        blocks = np.nonzero(selected[h, t])[0]
        keys = (blocks[:, None] * config.block_k + np.arange(config.block_k)[None, :]).reshape(-1)
        s = np.matmul(qt, k[h, keys].T) * sc
        s = np.where((keys[None, :] <= positions[:, None])[None], s, -np.inf)
        vals = v[h, keys]
        if config.mean_correction:
            tile_first = offset + t * config.tile_q
            corr_blocks = np.nonzero((~selected[h, t]) & (block_ends <= tile_first))[0]
            if corr_blocks.size:
                s2 = np.matmul(qt, pk[h, corr_blocks].T) * sc + lnbk
                s = np.concatenate([s, s2], axis=-1)
                vals = np.concatenate([vals, pv[h, corr_blocks]], axis=0)
        m = s.max(axis=-1, keepdims=True)
        w = np.exp(s - m)
        out[h * g:(h + 1) * g, rows, :] = np.matmul(w, vals) / w.sum(axis=-1, keepdims=True)
    return out


# --------------------------------------------------------------------------
# Hook semantics (fpv2/patch.py)
# --------------------------------------------------------------------------

PACKED_TILE_ROWS = 128


def effective_config(config: Any, query_heads: int, kv_heads: int):
    """fpv2/patch.py:41-52: 128 packed rows -> 128/G query positions."""
    config = as_config(config)
    if config.tile_q != PACKED_TILE_ROWS:
        return config
    if not kv_heads or query_heads % kv_heads:
        return None
    group = query_heads // kv_heads
    if PACKED_TILE_ROWS % group:
        return None
    return replace(config, tile_q=PACKED_TILE_ROWS // group)


def request_config(config: Any, key_length: int, total_tokens: int | None):
    """fpv2/patch.py:55-63."""
    config = as_config(config)
    if config.last_n_blocks and (total_tokens is None or key_length < total_tokens):
        return replace(config, last_n_blocks=0)
    return config


def causal_block_count(kv_heads: int, query_length: int, offset: int, config: Any) -> int:
    """fpv2/patch.py:66-76."""
    config = as_config(config)
    count = 0
    for start in range(0, query_length, config.tile_q):
        end = offset + min(start + config.tile_q, query_length)
        count += (end + config.block_k - 1) // config.block_k
    return count * kv_heads


def fpv2_sdpa(q, k, v, *, scale: float, config: Any = None, dtype: str = "bf16",
              out_dtype: str | None = None):
    """fpv2/patch.py:102-174 on ``[1, H, L, D]`` float32 arrays of ``dtype`` values.

    ``out_dtype`` ("fp32": unrounded) overrides the rounding of the output."""
    config = as_config(config)
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    eff = effective_config(config, q.shape[1], k.shape[1])
    if eff is None:
        raise ValueError("GQA group size must divide 128 packed query rows")
    config = eff
    lq = q.shape[-2]
    lk = k.shape[-2]
    if lq > lk:
        raise ValueError("query length cannot exceed key length for causal attention")
    offset = lk - lq
    lq_pad = (lq + config.tile_q - 1) // config.tile_q * config.tile_q
    need_k = max(lk, offset + lq_pad)
    lk_pad = (need_k + config.block_k - 1) // config.block_k * config.block_k
    pq = np.zeros((q.shape[1], lq_pad, q.shape[-1]), np.float32)
    pq[:, :lq] = q[0]
    pk = np.zeros((k.shape[1], lk_pad, k.shape[-1]), np.float32)
    pk[:, :lk] = k[0]
    pv = np.zeros_like(pk)
    pv[:, :lk] = v[0]
    pooled_k = pool_blocks(pk, config.block_k, dtype)
    pooled_v = pool_blocks(pv, config.block_k, dtype)
    sel = block_scores_and_select(
        pq, pooled_k, scale=scale,
        config=replace(config, score_chunk_tiles=config.score_chunk_tiles or max(1, 8192 // config.tile_q)),
        offset=offset, query_length=lq,
    ).selected
    lists = compact_block_indices(sel, config=config, offset=offset, query_length=lq, key_length=lk)
    out = sparse_attention(
        pq, pk, pv, pooled_k, pooled_v, *lists, scale=scale, config=config,
        offset=offset, query_length=lq, key_length=lk, dtype=dtype, out_dtype=out_dtype,
    )
    return out[None, :, :lq, :], sel, lists
