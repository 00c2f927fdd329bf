"""Block-list compaction and block-sparse attention for FlashPrefill V2 on B200.

Same operator surface as the reference's fpv2/kernel.py. The attention follows
an ascending block list with a FlashAttention-2 online softmax in base 2, then
appends pooled representatives of safely pruned blocks to the same softmax
with a ``+log2(block_k)`` logit shift (the mean correction).

On B200 the kernel packs the G query heads of a KV head into one 128-row MMA
tile natively (the reference's PackGQA, without the transposes), keeps fp32
accumulators in TMEM and streams K/V tiles with TMA; see csrc/attn_tc.cu.
``TileConfig`` and ``pack_gqa`` are accepted and validated like the
reference's Metal tiling options; the CUDA kernels choose their own tiles.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from fpv2 import _lib
from fpv2.selection import FPV2Config

SUPPORTED_HEAD_DIMS = (64, 96, 128, 256)


@dataclass(frozen=True)
class TileConfig:
    """Tile dimensions of the reference's Metal kernel (fpv2/kernel.py:30-57).

    Validated for API compatibility; the B200 kernels pick their own tiling.
    """

    bq: int
    bk: int
    wm: int

    @property
    def threads(self) -> int:
        return 32 * self.wm

    def check(self, head_dim: int, *, block_k: int = 128, tile_q: int = 128) -> None:
        if min(self.bq, self.bk, self.wm) <= 0:
            raise ValueError("tile dimensions must be positive")
        if self.bq % (8 * self.wm):
            raise ValueError("bq must contain whole 8-row fragments per simdgroup")
        if block_k % self.bk:
            raise ValueError("bk must divide block_k")
        if tile_q < self.bq or tile_q % self.bq:
            raise ValueError("bq must divide tile_q")
        if (self.bk * head_dim) % self.threads:
            raise ValueError("thread count must divide the correction gather")
        memory = (self.bq * (head_dim + 8) + max(
            head_dim * (self.bk + 8), self.bk * (head_dim + 8)
        )) * 2
        if memory > 32 * 1024:
            raise ValueError("tile exceeds 32 KB of threadgroup memory")


_DEFAULT_TILES = {
    64: TileConfig(32, 32, 4),
    96: TileConfig(32, 32, 4),
    128: TileConfig(64, 32, 8),
    256: TileConfig(32, 16, 4),
}


def default_tile(head_dim: int) -> TileConfig:
    """Reference default tile for a supported head dimension (fpv2/kernel.py:68-73)."""
    try:
        return _DEFAULT_TILES[head_dim]
    except KeyError as error:
        raise ValueError(f"head dimension must be one of {SUPPORTED_HEAD_DIMS}") from error


def _tile_for_config(head_dim: int, config: FPV2Config) -> TileConfig:
    """fpv2/kernel.py:76-88."""
    tile = default_tile(head_dim)
    if (
        config.tile_q >= tile.bq
        and config.tile_q % tile.bq == 0
        and config.block_k % tile.bk == 0
    ):
        return tile
    if config.tile_q % 8 or config.block_k % 8:
        raise ValueError("block_k and tile_q must be multiples of 8 for Steel")
    bq = min(config.tile_q, 32)
    bk = min(config.block_k, 16)
    return TileConfig(bq, bk, bq // 8)


def compact_block_indices(
    selected: torch.Tensor,
    *,
    config: FPV2Config = FPV2Config(),
    offset: int = 0,
    query_length: int | None = None,
    key_length: int | None = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Padded selected/pruned block lists and per-row counts (fpv2/kernel.py:141-184).

    ``selected_ids`` holds the selected blocks ascending, then all other blocks
    ascending; ``pruned_ids`` likewise for blocks that are not selected and end
    (clamped to ``key_length``) at or before the tile's first query position.
    """
    if selected.ndim != 3:
        raise ValueError("selected must have shape [KV heads, tiles, blocks]")
    if selected.dtype != torch.bool:
        raise ValueError("selected must have boolean dtype")
    kv_heads, num_tiles, num_blocks = selected.shape
    padded_query_length = num_tiles * config.tile_q
    valid_query_length = padded_query_length if query_length is None else query_length
    represented_key_length = num_blocks * config.block_k
    valid_key_length = represented_key_length if key_length is None else key_length
    if offset < 0:
        raise ValueError("offset must be non-negative")
    if not 0 < valid_query_length <= padded_query_length:
        raise ValueError("query_length is inconsistent with selected tiles")
    if not 0 < valid_key_length <= represented_key_length:
        raise ValueError("key_length is inconsistent with selected blocks")
    if offset + valid_query_length > valid_key_length:
        raise ValueError("queries extend beyond key_length")
    _lib.require_cuda(selected)
    dev = selected.device
    mask = selected.contiguous().view(torch.uint8)
    sel_ids = torch.empty((kv_heads, num_tiles, num_blocks), dtype=torch.int32, device=dev)
    pr_ids = torch.empty_like(sel_ids)
    sel_counts = torch.empty((kv_heads, num_tiles), dtype=torch.int32, device=dev)
    pr_counts = torch.empty_like(sel_counts)
    _lib.check(_lib.lib().fpv2_compact_block_indices(
        _lib.ptr(mask), kv_heads, num_tiles, num_blocks, config.block_k, config.tile_q, offset,
        valid_query_length, valid_key_length, _lib.ptr(sel_ids), _lib.ptr(sel_counts),
        _lib.ptr(pr_ids), _lib.ptr(pr_counts), _lib.stream_of(selected)))
    return sel_ids, sel_counts, pr_ids, pr_counts


def sparse_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    pooled_k: torch.Tensor,
    pooled_v: torch.Tensor,
    selected_ids: torch.Tensor,
    selected_counts: torch.Tensor,
    pruned_ids: torch.Tensor,
    pruned_counts: torch.Tensor,
    *,
    scale: float,
    config: FPV2Config = FPV2Config(),
    offset: int = 0,
    query_length: int | None = None,
    key_length: int | None = None,
    tile: TileConfig | None = None,
    pack_gqa: bool = False,
    multicast: tuple[int, int, int] | None = None,
) -> torch.Tensor | None:
    """Tiled block-sparse attention with the pooled mean correction.

    Validation and error messages follow fpv2/kernel.py:465-510. Pooled K/V may
    be float32 or the query dtype; they are rounded to the query dtype on load
    (fpv2/kernel.py:553-554). Ids are clipped to the block range
    (fpv2/kernel.py:555-558). Rows at or beyond ``query_length`` are padding and
    their output is unspecified.

    ``multicast=(address, head_offset, heads_total)`` (not in the reference: the
    head-parallel multi-GPU layer) writes the output into every rank's full
    ``[heads_total, padded_q_len, dim]`` buffer behind an NVLink multicast
    address instead of a new tensor, at head ``head_offset + h``, and returns None.
    """
    if q.ndim != 3 or k.ndim != 3 or v.ndim != 3:
        raise ValueError("q, k, and v must have shape [heads, sequence, dim]")
    if k.shape != v.shape:
        raise ValueError("k and v must have identical shapes")
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k, and v must share float16 or bfloat16 dtype")
    query_heads, padded_query_length, head_dim = q.shape
    kv_heads, padded_key_length, key_dim = k.shape
    if head_dim != key_dim or head_dim not in SUPPORTED_HEAD_DIMS:
        raise ValueError(f"head dimension must be one of {SUPPORTED_HEAD_DIMS}")
    if not kv_heads or query_heads % kv_heads:
        raise ValueError("query heads must be divisible by KV heads")
    if padded_query_length % config.tile_q or padded_key_length % config.block_k:
        raise ValueError("q and k/v sequence lengths must be tile/block aligned")
    valid_query_length = padded_query_length if query_length is None else query_length
    valid_key_length = padded_key_length if key_length is None else key_length
    if not 0 < valid_query_length <= padded_query_length:
        raise ValueError("query_length must fit within padded q")
    if not 0 < valid_key_length <= padded_key_length:
        raise ValueError("key_length must fit within padded k/v")
    num_tiles = padded_query_length // config.tile_q
    num_blocks = padded_key_length // config.block_k
    expected_lists = (kv_heads, num_tiles, num_blocks)
    expected_counts = (kv_heads, num_tiles)
    if tuple(selected_ids.shape) != expected_lists or tuple(pruned_ids.shape) != expected_lists:
        raise ValueError(f"block lists must have shape {expected_lists}")
    if (tuple(selected_counts.shape) != expected_counts
            or tuple(pruned_counts.shape) != expected_counts):
        raise ValueError(f"block counts must have shape {expected_counts}")
    lists = (selected_ids, pruned_ids)
    counts = (selected_counts, pruned_counts)
    if any(array.dtype != torch.int32 for array in (*lists, *counts)):
        raise ValueError("block lists and counts must have int32 dtype")
    if (tuple(pooled_k.shape) != (kv_heads, num_blocks, head_dim)
            or tuple(pooled_v.shape) != tuple(pooled_k.shape)):
        raise ValueError("pooled k/v shapes do not match padded k/v")
    if offset < 0 or offset + valid_query_length > valid_key_length:
        raise ValueError("offset does not align queries within the key sequence")
    tile = _tile_for_config(head_dim, config) if tile is None else tile
    tile.check(head_dim, block_k=config.block_k, tile_q=config.tile_q)
    group_size = query_heads // kv_heads
    if pack_gqa and (tile.bq % group_size or (config.tile_q * group_size) % tile.bq):
        raise ValueError("PackGQA tile must align with complete GQA groups")

    _lib.require_cuda(q, k, v, pooled_k, pooled_v, *lists, *counts)
    if pooled_k.dtype not in (q.dtype, torch.float32):
        pooled_k = pooled_k.to(q.dtype)
    if pooled_v.dtype != pooled_k.dtype:
        pooled_v = pooled_v.to(pooled_k.dtype)
    qc, kc, vc = q.contiguous(), k.contiguous(), v.contiguous()
    pkc, pvc = pooled_k.contiguous(), pooled_v.contiguous()
    lc = [x.contiguous() for x in (selected_ids, selected_counts, pruned_ids, pruned_counts)]
    workspace = _lib.attention_workspace(qc, kv_heads, padded_key_length, config.block_k,
                                         config.tile_q, pkc.dtype, config.mean_correction)
    args = (
        _lib.ptr(qc), _lib.ptr(kc), _lib.ptr(vc), _lib.ptr(pkc), _lib.ptr(pvc),
        _lib.dtype_code(pkc.dtype), _lib.ptr(lc[0]), _lib.ptr(lc[1]), _lib.ptr(lc[2]),
        _lib.ptr(lc[3]), _lib.dtype_code(q.dtype), query_heads, kv_heads, padded_query_length,
        padded_key_length, head_dim, offset, valid_query_length, valid_key_length, float(scale),
        config.block_k, config.tile_q, 1 if config.mean_correction else 0,
    )
    if multicast is not None:
        mc_ptr, head_offset, heads_total = multicast
        _lib.check(_lib.lib().fpv2_sparse_attention_multicast(
            *args, mc_ptr, head_offset, heads_total, _lib.ptr(workspace), workspace.numel() * 4,
            _lib.stream_of(q)))
        return None
    out = torch.empty_like(qc)
    _lib.check(_lib.lib().fpv2_sparse_attention(
        *args, _lib.ptr(out), _lib.ptr(workspace), workspace.numel() * 4, _lib.stream_of(q)))
    return out


def index_stage(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    scale: float,
    config: FPV2Config,
    offset: int,
    query_length: int,
    key_length: int,
    pooled_dtype: torch.dtype | None = None,
    return_mask: bool = False,
):
    """Fused pool(K), pool(V) -> select -> compact on padded ``[H, L, D]`` tensors.

    Equivalent to ``pool_blocks`` x2, ``block_scores_and_select`` and
    ``compact_block_indices`` in sequence (fpv2/patch.py:137-153), in one C-ABI
    call without host synchronisation. Pooled tensors are written in
    ``pooled_dtype`` (default: the input dtype, as the reference hook pools).
    Returns ``(pooled_k, pooled_v, (sel_ids, sel_counts, pr_ids, pr_counts), mask)``.
    """
    _lib.require_cuda(q, k, v)
    query_heads, padded_q, head_dim = q.shape
    kv_heads, padded_k, _ = k.shape
    num_tiles = padded_q // config.tile_q
    num_blocks = padded_k // config.block_k
    dev = q.device
    pdt = q.dtype if pooled_dtype is None else pooled_dtype
    pooled_k = torch.empty((kv_heads, num_blocks, head_dim), dtype=pdt, device=dev)
    pooled_v = torch.empty_like(pooled_k)
    sel_ids = torch.empty((kv_heads, num_tiles, num_blocks), dtype=torch.int32, device=dev)
    pr_ids = torch.empty_like(sel_ids)
    sel_counts = torch.empty((kv_heads, num_tiles), dtype=torch.int32, device=dev)
    pr_counts = torch.empty_like(sel_counts)
    mask = (torch.empty((kv_heads, num_tiles, num_blocks), dtype=torch.uint8, device=dev)
            if return_mask else None)
    qc, kc, vc = q.contiguous(), k.contiguous(), v.contiguous()
    ws = _lib.select_workspace(qc, pdt, kv_heads, num_blocks, head_dim)
    _lib.check(_lib.lib().fpv2_index_stage(
        _lib.ptr(qc), _lib.ptr(kc), _lib.ptr(vc), _lib.dtype_code(q.dtype), query_heads,
        kv_heads, padded_q, padded_k, head_dim, offset, query_length, key_length, float(scale),
        config.block_k, config.tile_q, float(config.alpha), config.sink_tokens,
        config.window_tokens, config.last_n_blocks, _lib.dtype_code(pdt), _lib.ptr(pooled_k),
        _lib.ptr(pooled_v), _lib.ptr(sel_ids), _lib.ptr(sel_counts), _lib.ptr(pr_ids),
        _lib.ptr(pr_counts), _lib.ptr(mask), *_lib.workspace_args(ws), _lib.stream_of(q)))
    return (pooled_k, pooled_v, (sel_ids, sel_counts, pr_ids, pr_counts),
            None if mask is None else mask.view(torch.bool))


def correction_shift(block_k: int) -> float:
    """``log2(block_k)``: the logit shift of a pooled entry (fpv2/kernel.py:546-548)."""
    return math.log2(block_k)
