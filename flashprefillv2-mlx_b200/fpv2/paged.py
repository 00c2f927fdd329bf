"""Paged K/V (no reference counterpart: the reference's MLX KV cache is one
contiguous array per layer, fpv2/patch.py:102-174).

Serving engines keep keys and values in page pools ``[num_pages, page_size,
kv_heads, head_dim]`` with a per-sequence block table; logical key position p
is row ``p % page_size`` of page ``block_table[p // page_size]``. The block
lists of the index stage hold logical block indices, so they are consumed
unchanged: ``pool_pages`` computes the pooled K/V of the sequence (the exact
mean of ``pool_blocks``) and ``sparse_attention_paged`` runs the attention of
``sparse_attention`` with its K/V tiles fetched through the block table.
"""

from __future__ import annotations

import torch

from fpv2 import _lib
from fpv2.selection import FPV2Config

_PAGED_DIMS = (64, 96, 128)


def _check_pool(cache: torch.Tensor, name: str) -> tuple[int, int, int, int]:
    if cache.ndim != 4:
        raise ValueError(f"{name} must have shape [pages, page_size, kv_heads, dim]")
    if cache.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"{name} must be float16 or bfloat16")
    return tuple(cache.shape)


def _check_table(block_table: torch.Tensor, page_size: int, length: int) -> None:
    if block_table.ndim != 1 or block_table.dtype != torch.int32:
        raise ValueError("block_table must be a 1-D int32 tensor")
    if block_table.numel() * page_size < length:
        raise ValueError("block_table does not cover the key sequence")


def pool_pages(
    cache: torch.Tensor,
    block_table: torch.Tensor,
    block_size: int,
    length: int,
    *,
    dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """Block means ``[kv_heads, length // block_size, dim]`` of the first ``length``
    keys of a paged sequence (``pool_blocks`` on the gathered sequence,
    fpv2/selection.py:68-80), in ``dtype`` (default: the cache dtype)."""
    num_pages, page_size, kv_heads, dim = _check_pool(cache, "cache")
    if block_size <= 0 or length <= 0 or length % block_size:
        raise ValueError("sequence length must be divisible by block size")
    if dim % 8:
        raise ValueError("head dimension must be a multiple of 8")
    _check_table(block_table, page_size, length)
    _lib.require_cuda(cache, block_table)
    out_dtype = cache.dtype if dtype is None else dtype
    out = torch.empty((kv_heads, length // block_size, dim), dtype=out_dtype, device=cache.device)
    cc, bt = cache.contiguous(), block_table.contiguous()
    _lib.check(_lib.lib().fpv2_pool_pages(
        _lib.ptr(cc), _lib.ptr(bt), bt.numel(), num_pages, page_size, kv_heads, dim, length,
        block_size, _lib.dtype_code(cc.dtype), _lib.ptr(out), _lib.dtype_code(out_dtype),
        _lib.stream_of(cc)))
    return out


def sparse_attention_paged(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_table: torch.Tensor,
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
) -> torch.Tensor:
    """``sparse_attention`` (fpv2/kernel.py:441-590) with K/V in page pools.

    ``q`` is ``[heads, padded_q_len, dim]``; the lists, counts and pooled K/V
    are shaped as for ``sparse_attention`` with ``padded_k_len = num_blocks *
    block_k`` logical keys, which the block table must cover. Runs on the
    tensor-core kernel only (bf16/fp16, head_dim 64/96/128, block_k a multiple of
    128, page_size a multiple of 8 that divides 128 or is a multiple of 128).
    """
    if q.ndim != 3:
        raise ValueError("q must have shape [heads, sequence, dim]")
    kshape = _check_pool(k_cache, "k_cache")
    if tuple(v_cache.shape) != kshape or v_cache.dtype != k_cache.dtype:
        raise ValueError("k_cache and v_cache must have identical shapes and dtypes")
    if q.dtype != k_cache.dtype:
        raise ValueError("q, k, and v must share float16 or bfloat16 dtype")
    num_pages, page_size, kv_heads, dim = kshape
    query_heads, padded_query_length, head_dim = q.shape
    if head_dim != dim or head_dim not in _PAGED_DIMS:
        raise ValueError(f"head dimension must be one of {_PAGED_DIMS} for paged K/V")
    if not kv_heads or query_heads % kv_heads:
        raise ValueError("query heads must be divisible by KV heads")
    if padded_query_length % config.tile_q:
        raise ValueError("q and k/v sequence lengths must be tile/block aligned")
    num_tiles = padded_query_length // config.tile_q
    if selected_ids.ndim != 3:
        raise ValueError("block lists must have shape [kv_heads, tiles, blocks]")
    num_blocks = selected_ids.shape[2]
    padded_key_length = num_blocks * config.block_k
    expected_lists = (kv_heads, num_tiles, num_blocks)
    expected_counts = (kv_heads, num_tiles)
    if tuple(selected_ids.shape) != expected_lists or tuple(pruned_ids.shape) != expected_lists:
        raise ValueError(f"block lists must have shape {expected_lists}")
    if (tuple(selected_counts.shape) != expected_counts
            or tuple(pruned_counts.shape) != expected_counts):
        raise ValueError(f"block counts must have shape {expected_counts}")
    if any(t.dtype != torch.int32 for t in (selected_ids, selected_counts, pruned_ids, pruned_counts)):
        raise ValueError("block lists and counts must have int32 dtype")
    if (tuple(pooled_k.shape) != (kv_heads, num_blocks, head_dim)
            or tuple(pooled_v.shape) != tuple(pooled_k.shape)):
        raise ValueError("pooled k/v shapes do not match padded k/v")
    _check_table(block_table, page_size, padded_key_length)
    valid_query_length = padded_query_length if query_length is None else query_length
    valid_key_length = padded_key_length if key_length is None else key_length
    if not 0 < valid_query_length <= padded_query_length:
        raise ValueError("query_length must fit within padded q")
    if not 0 < valid_key_length <= padded_key_length:
        raise ValueError("key_length must fit within padded k/v")
    if offset < 0 or offset + valid_query_length > valid_key_length:
        raise ValueError("offset does not align queries within the key sequence")
    _lib.require_cuda(q, k_cache, v_cache, block_table, pooled_k, pooled_v, selected_ids,
                      selected_counts, pruned_ids, pruned_counts)
    if pooled_k.dtype not in (q.dtype, torch.float32):
        pooled_k = pooled_k.to(q.dtype)
    if pooled_v.dtype != pooled_k.dtype:
        pooled_v = pooled_v.to(pooled_k.dtype)
    qc, kc, vc, bt = q.contiguous(), k_cache.contiguous(), v_cache.contiguous(), block_table.contiguous()
    pkc, pvc = pooled_k.contiguous(), pooled_v.contiguous()
    lc = [x.contiguous() for x in (selected_ids, selected_counts, pruned_ids, pruned_counts)]
    workspace = _lib.attention_workspace(qc, kv_heads, padded_key_length, config.block_k,
                                         config.tile_q, pkc.dtype, config.mean_correction)
    out = torch.empty_like(qc)
    _lib.check(_lib.lib().fpv2_sparse_attention_paged(
        _lib.ptr(qc), _lib.ptr(kc), _lib.ptr(vc), _lib.ptr(bt), bt.numel(), num_pages, page_size,
        _lib.ptr(pkc), _lib.ptr(pvc), _lib.dtype_code(pkc.dtype), _lib.ptr(lc[0]), _lib.ptr(lc[1]),
        _lib.ptr(lc[2]), _lib.ptr(lc[3]), _lib.dtype_code(q.dtype), query_heads, kv_heads,
        padded_query_length, padded_key_length, head_dim, offset, valid_query_length,
        valid_key_length, float(scale), config.block_k, config.tile_q,
        1 if config.mean_correction else 0, _lib.ptr(out), _lib.ptr(workspace),
        workspace.numel() * 4, _lib.stream_of(q)))
    return out
