"""Block scoring and selection for FlashPrefill V2 on B200 (torch tensors in, CUDA out).

Same operator surface and semantics as the reference's index stage
(fpv2/selection.py): keys are mean-pooled into blocks; every query row is scored
against the pooled keys, ``s = scale * q . kbar``; per KV head and query tile
the block energy is the sum of ``exp(s - max)`` over the tile's rows and the
query heads sharing that KV head, restricted to visible rows and fully visible
blocks; a block is kept when its energy reaches ``alpha`` times the largest
energy, and sink, local-window (including the diagonal) and dense-tail blocks
are forced, all limited to causally visible blocks. ``offset`` is the absolute
key position of query row zero, so bottom-right chunks select what a single
shot selects.

The arithmetic runs in ``libfpv2_b200.so``: a tcgen05 kernel for bf16/fp16
inputs with head_dim 64, 96, 128 or 256, a CUDA-core kernel otherwise. Query-tile chunking
(``score_chunk_tiles``) never changes the result; it only decides whether the
raw score tensor is returned, as in the reference.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from fpv2 import _lib


@dataclass(frozen=True)
class FPV2Config:
    """Parameters controlling block selection and mean correction (fpv2/selection.py:30-65)."""

    block_k: int = 128
    tile_q: int = 128
    alpha: float = 0.1
    sink_tokens: int = 256
    window_tokens: int = 384
    # This is request-level only when the input contains the complete request.
    last_n_blocks: int = 2
    mean_correction: bool = True
    score_chunk_tiles: int | None = None
    pack_gqa: bool = False

    def __post_init__(self) -> None:
        if self.block_k <= 0 or self.tile_q <= 0:
            raise ValueError("block_k and tile_q must be positive")
        if self.alpha < 0:
            raise ValueError("alpha must be non-negative")
        if self.sink_tokens < 0 or self.window_tokens < 0:
            raise ValueError("sink_tokens and window_tokens must be non-negative")
        if (
            not isinstance(self.last_n_blocks, int)
            or isinstance(self.last_n_blocks, bool)
            or self.last_n_blocks < 0
        ):
            raise ValueError("last_n_blocks must be a non-negative integer")
        if self.score_chunk_tiles is not None and (
            not isinstance(self.score_chunk_tiles, int)
            or isinstance(self.score_chunk_tiles, bool)
            or self.score_chunk_tiles <= 0
        ):
            raise ValueError("score_chunk_tiles must be a positive integer or None")
        if not isinstance(self.pack_gqa, bool):
            raise ValueError("pack_gqa must be a boolean")


def pool_blocks(x: torch.Tensor, block_size: int = 128) -> torch.Tensor:
    """Mean-pool the penultimate (sequence) axis into fixed-size blocks.

    Output dtype is the input dtype (fpv2/selection.py:68-80). The mean is exact
    (float64 sum in the kernel), rounded to float32, then to the output dtype.
    """
    if x.ndim < 2:
        raise ValueError("x must have at least sequence and feature dimensions")
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    length, head_dim = x.shape[-2:]
    if length % block_size:
        raise ValueError(
            f"sequence length {length} must be divisible by block_size {block_size}"
        )
    _lib.require_cuda(x)
    code = _lib.dtype_code(x.dtype)
    xc = x.contiguous()
    heads = xc.numel() // max(1, length * head_dim) if length * head_dim else 0
    out = torch.empty((*x.shape[:-2], length // block_size, head_dim), dtype=x.dtype,
                      device=x.device)
    _lib.check(_lib.lib().fpv2_pool_blocks(
        _lib.ptr(xc), code, heads, length, head_dim, block_size, _lib.ptr(out), code,
        _lib.stream_of(x)))
    return out


def _validate_inputs(
    q: torch.Tensor,
    pooled_k: torch.Tensor,
    config: FPV2Config,
    offset: int,
    query_length: int,
) -> tuple[int, int, int, int]:
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


def block_scores_and_select(
    q: torch.Tensor,
    pooled_k: torch.Tensor,
    *,
    scale: float,
    config: FPV2Config = FPV2Config(),
    offset: int = 0,
    query_length: int | None = None,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Return selection ``[Hkv, Nt, Nb]`` (bool) and optional raw scores.

    ``offset`` is the absolute key position corresponding to query row zero.
    Query input must be tile-padded; ``query_length`` excludes padded rows.
    Raw scores have shape ``[Hkv, G, N, Nb]`` (float32) and are returned only
    when ``score_chunk_tiles`` is ``None``, as in fpv2/selection.py:109-201.
    """
    valid_length = q.shape[-2] if query_length is None else query_length
    query_heads, kv_heads, padded_length, num_blocks = _validate_inputs(
        q, pooled_k, config, offset, valid_length
    )
    _lib.require_cuda(q, pooled_k)
    group = query_heads // kv_heads
    num_tiles = padded_length // config.tile_q
    qc = q.contiguous()
    kc = pooled_k.contiguous()
    mask = torch.empty((kv_heads, num_tiles, num_blocks), dtype=torch.uint8, device=q.device)
    raw = None
    if config.score_chunk_tiles is None:
        raw = torch.empty((kv_heads, group, padded_length, num_blocks), dtype=torch.float32,
                          device=q.device)
    ws = _lib.select_workspace(qc, kc.dtype, kv_heads, num_blocks, q.shape[-1])
    _lib.check(_lib.lib().fpv2_block_select(
        _lib.ptr(qc), _lib.dtype_code(q.dtype), _lib.ptr(kc), _lib.dtype_code(pooled_k.dtype),
        query_heads, kv_heads, padded_length, num_blocks, q.shape[-1], offset, valid_length,
        float(scale), config.block_k, config.tile_q, float(config.alpha), config.sink_tokens,
        config.window_tokens, config.last_n_blocks, _lib.ptr(mask), _lib.ptr(raw),
        *_lib.workspace_args(ws), _lib.stream_of(q)))
    return mask.view(torch.bool), raw


def density(
    selected: torch.Tensor,
    *,
    config: FPV2Config = FPV2Config(),
    offset: int = 0,
    query_length: int | None = None,
) -> torch.Tensor:
    """Retained causal block work as a scalar fraction (fpv2/selection.py:204-229)."""
    if selected.ndim != 3:
        raise ValueError("selected must have shape [KV heads, tiles, blocks]")
    kv_heads, num_tiles, num_blocks = selected.shape
    if offset < 0:
        raise ValueError("offset must be non-negative")
    valid_length = num_tiles * config.tile_q if query_length is None else query_length
    if not 0 < valid_length <= num_tiles * config.tile_q:
        raise ValueError("query_length is inconsistent with selected tiles")
    dev = selected.device
    tile_last = torch.minimum(
        offset + (torch.arange(num_tiles, device=dev, dtype=torch.int64) + 1) * config.tile_q,
        torch.tensor(offset + valid_length, device=dev),
    ) - 1
    block_starts = torch.arange(num_blocks, device=dev, dtype=torch.int64) * config.block_k
    visible = block_starts[None, :] <= tile_last[:, None]
    denominator = visible.to(torch.float32).sum() * kv_heads
    return selected.to(torch.float32).sum() / denominator
