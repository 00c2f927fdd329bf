"""Model-independent, conservative hook for PyTorch scaled-dot-product attention.

Mirrors the reference hook (fpv2/patch.py), retargeted from MLX's
``mx.fast.scaled_dot_product_attention`` to
``torch.nn.functional.scaled_dot_product_attention``. ``enable`` replaces the
torch entry point with a wrapper that sends a call to FPV2 only when it is a
batch-one causal prefill on CUDA with matching float16/bfloat16 Q/K/V, a
supported head dimension, grouped-query-compatible head counts, at least one
full query tile and a key length meeting ``min_tokens``. Everything else --
array masks, dropout, decode calls, unsupported layouts, CPU tensors -- goes
to the exact original function unchanged.

Causal alignment: MLX's ``"causal"`` is bottom-right aligned, torch's
``is_causal=True`` is top-left aligned. The two agree only when the query and
key lengths are equal, so the hook claims ``is_causal=True`` calls with
``Lq == Lk`` and calls whose ``attn_mask`` is an explicit lower-right causal
bias (``torch.nn.attention.bias.causal_lower_right``), the chunked-prefill
form. For eligible calls ``offset = Lk - Lq`` locates the query chunk in the
causal key prefix; queries and keys are padded only for tile/block processing
and the output padding is removed. ``disable`` restores the original function.
"""

from __future__ import annotations

from dataclasses import replace
from typing import Any

import torch
import torch.nn.functional as F

from fpv2.kernel import SUPPORTED_HEAD_DIMS, index_stage, sparse_attention
from fpv2.selection import FPV2Config

try:  # torch >= 2.3
    from torch.nn.attention.bias import CausalBias, CausalVariant
except ImportError:  # pragma: no cover - older torch
    CausalBias = None
    CausalVariant = None

_ORIGINAL_SDPA = F.scaled_dot_product_attention
_enabled = False
_collect_stats = False
_selected_counts: list[torch.Tensor] = []
_selected_dense_blocks = 0
_visible_blocks = 0
_HOPPER_PACKED_TILE_ROWS = 128


def _effective_config(
    config: FPV2Config, query_heads: int, kv_heads: int
) -> FPV2Config | None:
    """Resolve the default 128 packed rows into query positions (fpv2/patch.py:41-52)."""
    if config.tile_q != _HOPPER_PACKED_TILE_ROWS:
        return config
    if not kv_heads or query_heads % kv_heads:
        return None
    group_size = query_heads // kv_heads
    if _HOPPER_PACKED_TILE_ROWS % group_size:
        return None
    return replace(config, tile_q=_HOPPER_PACKED_TILE_ROWS // group_size)


def _request_config(
    config: FPV2Config, key_length: int, total_tokens: int | None
) -> FPV2Config:
    """Apply the dense tail only when this call reaches the request boundary (fpv2/patch.py:55-63)."""
    if config.last_n_blocks and (total_tokens is None or key_length < total_tokens):
        return replace(config, last_n_blocks=0)
    return config


def _causal_block_count(
    kv_heads: int,
    query_length: int,
    offset: int,
    config: FPV2Config,
) -> int:
    """Visible (also partially visible) blocks summed over tiles (fpv2/patch.py:66-76)."""
    count = 0
    for start in range(0, query_length, config.tile_q):
        end = offset + min(start + config.tile_q, query_length)
        count += (end + config.block_k - 1) // config.block_k
    return count * kv_heads


def block_sparsity() -> float:
    """Return the fraction of visible causal blocks skipped since ``enable``."""
    if not _visible_blocks:
        return 0.0
    selected = _selected_dense_blocks
    if _selected_counts:
        total = torch.stack([x.sum(dtype=torch.int64).to(_selected_counts[0].device)
                             for x in _selected_counts]).sum()
        selected += int(total.item())
    return 1.0 - selected / _visible_blocks


def _pad_sequence(x: torch.Tensor, length: int) -> torch.Tensor:
    """Zero-pad the sequence axis (fpv2/patch.py:91-99); always returns a contiguous tensor."""
    amount = length - x.shape[-2]
    if amount < 0:
        raise ValueError("target length cannot be shorter than the input")
    if not amount:
        return x.contiguous()
    return F.pad(x, (0, 0, 0, amount)).contiguous()


def fpv2_sdpa(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    scale: float,
    config: FPV2Config = FPV2Config(),
    multicast: tuple[int, int, int] | None = None,
) -> torch.Tensor | None:
    """Apply FPV2 to an eligible batch-one, bottom-right causal attention (fpv2/patch.py:102-174).

    ``multicast`` (not in the reference) is forwarded to ``sparse_attention``: the
    output goes to every rank's buffer behind an NVLink multicast address and
    the call returns None.
    """
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q, k, and v must have shape [batch, heads, sequence, dim]")
    if q.shape[0] != 1 or k.shape[0] != 1 or v.shape[0] != 1:
        raise ValueError("FPV2 currently supports batch size 1")
    effective_config = _effective_config(config, q.shape[1], k.shape[1])
    if effective_config is None:
        raise ValueError("GQA group size must divide 128 packed query rows")
    config = effective_config
    query_length = q.shape[-2]
    key_length = k.shape[-2]
    if query_length > key_length:
        raise ValueError("query length cannot exceed key length for causal attention")
    offset = key_length - query_length

    padded_query_length = (query_length + config.tile_q - 1) // config.tile_q * config.tile_q
    required_key_length = max(key_length, offset + padded_query_length)
    padded_key_length = (
        (required_key_length + config.block_k - 1) // config.block_k * config.block_k
    )
    padded_q = _pad_sequence(q[0], padded_query_length)
    padded_k = _pad_sequence(k[0], padded_key_length)
    padded_v = _pad_sequence(v[0], padded_key_length)
    pooled_k, pooled_v, indices, _ = index_stage(
        padded_q, padded_k, padded_v, scale=scale, config=config, offset=offset,
        query_length=query_length, key_length=key_length,
    )
    if _collect_stats:
        global _visible_blocks
        _selected_counts.append(indices[1])
        _visible_blocks += _causal_block_count(k.shape[1], query_length, offset, config)
    output = sparse_attention(
        padded_q, padded_k, padded_v, pooled_k, pooled_v, *indices, scale=scale,
        config=config, offset=offset, query_length=query_length, key_length=key_length,
        pack_gqa=config.pack_gqa, multicast=multicast,
    )
    if output is None:
        return None
    return output[None, :, :query_length, :]


def _call_original(*args: Any, **kwargs: Any) -> torch.Tensor:
    """Call torch's own SDPA exactly as the caller asked.

    A ``CausalBias`` mask dispatches through ``__torch_function__``, which only
    recognises the call while the module attribute is torch's function, so the
    original is put back for the duration of such a call.
    """
    if CausalBias is not None and isinstance(kwargs.get("attn_mask"), CausalBias):
        current = F.scaled_dot_product_attention
        F.scaled_dot_product_attention = _ORIGINAL_SDPA
        try:
            return _ORIGINAL_SDPA(*args, **kwargs)
        finally:
            F.scaled_dot_product_attention = current
    return _ORIGINAL_SDPA(*args, **kwargs)


def _causal_offset(q: torch.Tensor, k: torch.Tensor, attn_mask: object, is_causal: bool) -> int | None:
    """Offset of a bottom-right causal call, or None when the call is not one."""
    if q.ndim != 4 or k.ndim != 4:
        return None
    lq, lk = q.shape[-2], k.shape[-2]
    if attn_mask is None:
        return 0 if (is_causal and lq == lk) else None
    if (CausalBias is not None and isinstance(attn_mask, CausalBias) and not is_causal
            and attn_mask.variant == CausalVariant.LOWER_RIGHT
            and attn_mask.seq_len_q == lq and attn_mask.seq_len_kv == lk):
        return lk - lq
    return None


def _needs_autograd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> bool:
    """True when the call must record a backward graph (grad mode on and an input
    that requires grad). The FPV2 kernels have no backward, so such a call goes
    to torch's own SDPA, which records one; inference and ``no_grad`` calls do not."""
    return torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad)


def _eligible(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    causal_offset: int | None,
    dropout_p: float,
    enable_gqa: bool,
    kwargs: dict[str, Any],
    config: FPV2Config,
    min_tokens: int,
) -> bool:
    """fpv2/patch.py:177-205 for torch SDPA arguments."""
    if causal_offset is None or dropout_p or kwargs:
        return False
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        return False
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        return False
    if q.shape[0] != 1 or k.shape[0] != 1 or v.shape[0] != 1:
        return False
    if k.shape != v.shape or q.shape[-1] != k.shape[-1]:
        return False
    if q.shape[-2] > k.shape[-2] or q.shape[-2] < config.tile_q:
        return False
    if k.shape[-2] < min_tokens:
        return False
    if q.shape[-1] not in SUPPORTED_HEAD_DIMS:
        return False
    if q.dtype not in (torch.float16, torch.bfloat16):
        return False
    if k.dtype != q.dtype or v.dtype != q.dtype:
        return False
    if q.shape[1] != k.shape[1] and not enable_gqa:
        return False
    return bool(k.shape[1] and q.shape[1] % k.shape[1] == 0)


def enable(
    config: FPV2Config | None = None,
    *,
    min_tokens: int = 4_096,
    collect_stats: bool = False,
    total_tokens: int | None = None,
    **config_fields: Any,
) -> None:
    """Replace torch SDPA with an FPV2-gated, request-aware wrapper (fpv2/patch.py:208-272)."""
    global _collect_stats, _enabled, _selected_dense_blocks, _visible_blocks
    if min_tokens <= 0:
        raise ValueError("min_tokens must be positive")
    if not isinstance(collect_stats, bool):
        raise ValueError("collect_stats must be a boolean")
    if total_tokens is not None and (
        not isinstance(total_tokens, int)
        or isinstance(total_tokens, bool)
        or total_tokens <= 0
    ):
        raise ValueError("total_tokens must be a positive integer or None")
    if config is not None and config_fields:
        config = replace(config, **config_fields)
    elif config is None:
        config = FPV2Config(**config_fields)
    _collect_stats = collect_stats
    _selected_counts.clear()
    _selected_dense_blocks = 0
    _visible_blocks = 0

    def wrapped(
        query: torch.Tensor,
        key: torch.Tensor,
        value: torch.Tensor,
        attn_mask: object = None,
        dropout_p: float = 0.0,
        is_causal: bool = False,
        scale: float | None = None,
        enable_gqa: bool = False,
        **kwargs: Any,
    ) -> torch.Tensor:
        call_config = (
            _effective_config(config, query.shape[1], key.shape[1])
            if query.ndim == 4 and key.ndim == 4
            else None
        )
        if call_config is not None:
            call_config = _request_config(call_config, key.shape[-2], total_tokens)
        offset = _causal_offset(query, key, attn_mask, is_causal)
        if call_config is not None and not _needs_autograd(query, key, value) and _eligible(
            query, key, value, offset, dropout_p, enable_gqa, kwargs, call_config, min_tokens
        ):
            call_scale = query.shape[-1] ** -0.5 if scale is None else scale
            return fpv2_sdpa(query, key, value, scale=call_scale, config=call_config)
        if _collect_stats and call_config is not None and _eligible(
            query, key, value, offset, dropout_p, enable_gqa, kwargs, call_config, 1
        ):
            global _selected_dense_blocks, _visible_blocks
            visible = _causal_block_count(
                key.shape[1], query.shape[-2], key.shape[-2] - query.shape[-2], call_config
            )
            _selected_dense_blocks += visible
            _visible_blocks += visible
        return _call_original(
            query, key, value, attn_mask=attn_mask, dropout_p=dropout_p, is_causal=is_causal,
            scale=scale, enable_gqa=enable_gqa, **kwargs
        )

    F.scaled_dot_product_attention = wrapped
    _enabled = True


def disable() -> None:
    """Restore torch's original scaled dot-product attention function."""
    global _collect_stats, _enabled
    F.scaled_dot_product_attention = _ORIGINAL_SDPA
    _collect_stats = False
    _enabled = False


def is_enabled() -> bool:
    """Return whether the FPV2 SDPA hook is installed."""
    return _enabled
