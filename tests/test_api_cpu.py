"""Host logic and the C-ABI boundary, without a GPU.

Checks the reference's validation messages, the hook's config resolution, that
the library loads and exports every symbol declared in include/fpv2_b200.h, and
that CPU tensors are rejected instead of silently computed elsewhere.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

import fpv2
from fpv2 import _lib
from fpv2.kernel import TileConfig, _tile_for_config
from fpv2.patch import _causal_block_count, _causal_offset, _effective_config, _request_config

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols() -> list[str]:
    header = (ROOT / "include" / "fpv2_b200.h").read_text()
    return re.findall(r"FPV2_API\s+(?:const\s+char\s*\*|int64_t|int)\s+(fpv2_\w+)\s*\(", header)


def test_library_exports_every_declared_symbol():
    names = declared_symbols()
    assert len(names) >= 10
    handle = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in names:
        assert hasattr(handle, name), name
    assert set(names) == set(_lib.EXPORTED_SYMBOLS)
    assert _lib.lib().fpv2_version() >= 100


def test_fast_path_selection_rules_without_gpu():
    assert _lib.fast_path_mask(torch.bfloat16, 32, 8, 128, 128, 32, 512) == 3
    assert _lib.fast_path_mask(torch.float16, 64, 8, 128, 128, 16, 1024) == 3
    assert _lib.fast_path_mask(torch.bfloat16, 8, 2, 128, 128, 128, 16) == 7   # direct tile_q 128: chunk pairs
    assert _lib.fast_path_mask(torch.bfloat16, 8, 2, 64, 128, 64, 16) == 7     # 2 chunks of 2 heads x 64
    assert _lib.fast_path_mask(torch.bfloat16, 2, 2, 128, 128, 256, 16) == 3   # one head: slices differ in position
    assert _lib.fast_path_mask(torch.bfloat16, 8, 2, 96, 128, 32, 16) == 3   # zero-padded 128-wide tiles
    assert _lib.fast_path_mask(torch.bfloat16, 8, 2, 256, 128, 32, 16) == 3
    assert _lib.fast_path_mask(torch.bfloat16, 8, 2, 48, 128, 32, 16) == 0
    assert _lib.fast_path_mask(torch.bfloat16, 4, 2, 64, 16, 16, 4) == 1       # select tc, attn generic
    assert _lib.fast_path_mask(torch.float32, 8, 2, 128, 128, 32, 16) == 0


def test_invalid_arguments_return_status_without_gpu():
    before = _lib.launch_count()
    rc = _lib.lib().fpv2_pool_blocks(None, 1, 2, 7, 4, 4, None, 1, None)
    assert rc == _lib.ERR_INVALID_ARGUMENT
    assert "divisible" in _lib.lib().fpv2_last_error().decode()
    assert _lib.launch_count() == before   # a rejected call launches nothing


def test_cpu_tensors_are_rejected():
    with pytest.raises(ValueError, match="CUDA"):
        fpv2.pool_blocks(torch.zeros(2, 8, 4), 4)
    q = torch.zeros(4, 16, 8)
    with pytest.raises(ValueError, match="CUDA"):
        fpv2.block_scores_and_select(q, torch.zeros(2, 1, 8), scale=1.0,
                                     config=fpv2.FPV2Config(block_k=16, tile_q=16))


def test_pool_blocks_rejects_unaligned_length():
    with pytest.raises(ValueError, match="divisible"):
        fpv2.pool_blocks(torch.zeros((2, 7, 4)), 4)


@pytest.mark.parametrize("value", [0, -1, 1.5, True])
def test_score_chunk_tiles_must_be_a_positive_integer(value):
    with pytest.raises(ValueError, match="score_chunk_tiles"):
        fpv2.FPV2Config(score_chunk_tiles=value)


def test_pack_gqa_must_be_boolean():
    with pytest.raises(ValueError, match="pack_gqa"):
        fpv2.FPV2Config(pack_gqa=1)


@pytest.mark.parametrize("value", [-1, 1.5, True])
def test_last_n_blocks_must_be_a_non_negative_integer(value):
    with pytest.raises(ValueError, match="last_n_blocks"):
        fpv2.FPV2Config(last_n_blocks=value)


def test_hopper_selection_defaults():
    c = fpv2.FPV2Config()
    assert c.window_tokens == 384 and c.last_n_blocks == 2


def test_compaction_rejects_non_boolean_mask():
    with pytest.raises(ValueError, match="boolean"):
        fpv2.compact_block_indices(torch.ones((1, 1, 1), dtype=torch.int32))


def test_default_tile_dispatch():
    assert fpv2.default_tile(64) == TileConfig(32, 32, 4)
    assert fpv2.default_tile(96) == TileConfig(32, 32, 4)
    assert fpv2.default_tile(128) == TileConfig(64, 32, 8)
    assert fpv2.default_tile(256) == TileConfig(32, 16, 4)
    assert _tile_for_config(128, _effective_config(fpv2.FPV2Config(), 32, 8)) == TileConfig(32, 16, 4)


def test_default_tile_uses_128_packed_gqa_rows():
    effective = _effective_config(fpv2.FPV2Config(), query_heads=32, kv_heads=8)
    assert effective is not None and effective.tile_q == 32
    custom = fpv2.FPV2Config(tile_q=64)
    assert _effective_config(custom, query_heads=32, kv_heads=8) is custom
    assert _effective_config(fpv2.FPV2Config(), query_heads=16, kv_heads=8).tile_q == 64
    assert _effective_config(fpv2.FPV2Config(), query_heads=24, kv_heads=8) is None   # G = 3


def test_dense_tail_is_applied_only_at_known_request_end():
    config = fpv2.FPV2Config(last_n_blocks=2)
    assert _request_config(config, 2_048, 8_192).last_n_blocks == 0
    assert _request_config(config, 8_192, 8_192) is config
    assert _request_config(config, 8_192, None).last_n_blocks == 0


def test_causal_block_count():
    c = _effective_config(fpv2.FPV2Config(), 4, 2)   # tile_q 64
    assert _causal_block_count(2, 256, 0, c) == 12
    assert _causal_block_count(2, 128, 0, c) == 4


def test_causal_alignment_rules():
    from torch.nn.attention.bias import causal_lower_right, causal_upper_left

    q = torch.zeros(1, 4, 128, 64)
    k = torch.zeros(1, 2, 256, 64)
    assert _causal_offset(q, q, None, True) == 0
    assert _causal_offset(q, k, None, True) is None          # top-left alignment: not ours
    assert _causal_offset(q, k, causal_lower_right(128, 256), False) == 128
    assert _causal_offset(q, k, causal_upper_left(128, 256), False) is None
    assert _causal_offset(q, k, torch.zeros(128, 256), False) is None


@pytest.mark.parametrize("value", [0, -1, 1.5, True])
def test_total_tokens_must_be_a_positive_integer(value):
    with pytest.raises(ValueError, match="total_tokens"):
        fpv2.enable(total_tokens=value)
    fpv2.disable()


def test_enable_disable_restores_original():
    import torch.nn.functional as F

    from fpv2.patch import _ORIGINAL_SDPA

    fpv2.enable(min_tokens=1)
    assert fpv2.is_enabled() and F.scaled_dot_product_attention is not _ORIGINAL_SDPA
    q = torch.randn(1, 2, 8, 16)
    # CPU tensors fall through to the original function, bit for bit
    out = F.scaled_dot_product_attention(q, q, q, is_causal=True)
    assert torch.equal(out, _ORIGINAL_SDPA(q, q, q, is_causal=True))
    fpv2.disable()
    assert not fpv2.is_enabled() and F.scaled_dot_product_attention is _ORIGINAL_SDPA


def test_causal_bias_fall_through_is_bit_identical_on_cpu():
    """A lower-right CausalBias call the hook does not claim reaches torch unchanged."""
    import torch.nn.functional as F
    from torch.nn.attention.bias import causal_lower_right

    from fpv2.patch import _ORIGINAL_SDPA

    q = torch.randn(1, 4, 8, 16)
    k = torch.randn(1, 4, 24, 16)
    v = torch.randn(1, 4, 24, 16)
    bias = causal_lower_right(8, 24)
    expected = _ORIGINAL_SDPA(q, k, v, attn_mask=bias)
    fpv2.enable(min_tokens=1)
    try:
        actual = F.scaled_dot_product_attention(q, k, v, attn_mask=bias)
    finally:
        fpv2.disable()
    assert torch.equal(actual, expected)


def test_calls_that_need_autograd_are_not_claimed():
    """The kernels have no backward: with grad mode on and an input that requires
    grad the hook leaves the call to torch (which records the graph); inference
    and no_grad calls stay claimable."""
    import torch.nn.functional as F

    from fpv2.patch import _ORIGINAL_SDPA, _needs_autograd

    q = torch.randn(1, 4, 8, 16, requires_grad=True)
    k = torch.randn(1, 4, 8, 16)
    assert _needs_autograd(q, k, k)
    assert not _needs_autograd(q.detach(), k, k)
    with torch.no_grad():
        assert not _needs_autograd(q, k, k)
    with torch.inference_mode():
        assert not _needs_autograd(torch.randn(1, 4, 8, 16), k, k)
    fpv2.enable(min_tokens=1)
    try:
        out = F.scaled_dot_product_attention(q, k, k, is_causal=True)
    finally:
        fpv2.disable()
    assert out.grad_fn is not None
    assert torch.equal(out, _ORIGINAL_SDPA(q, k, k, is_causal=True))
    out.sum().backward()
    assert q.grad is not None


def test_sdpa_from_host_validates_before_touching_the_gpu():
    import fpv2

    q = torch.zeros((1, 8, 64, 128), dtype=torch.bfloat16)
    k = torch.zeros((1, 2, 64, 128), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="host tensor"):
        fpv2.sdpa_from_host(q.to("meta"), k, k, scale=1.0)
    with pytest.raises(ValueError, match="kv_heads_per_chunk"):
        fpv2.sdpa_from_host(q, k, k, scale=1.0, kv_heads_per_chunk=3)
    with pytest.raises(ValueError, match="multiple"):
        fpv2.sdpa_from_host(q[:, :7], k, k, scale=1.0)
    with pytest.raises(ValueError, match="out must be"):
        fpv2.sdpa_from_host(q, k, k, scale=1.0, out=torch.zeros((1, 8, 64, 64), dtype=torch.bfloat16))


def test_paged_api_validates_before_touching_the_gpu():
    import fpv2

    cache = torch.zeros((4, 16, 2, 128), dtype=torch.bfloat16)
    table = torch.zeros(8, dtype=torch.int32)
    with pytest.raises(ValueError, match="divisible by block size"):
        fpv2.pool_pages(cache, table, 128, 100)
    with pytest.raises(ValueError, match="does not cover"):
        fpv2.pool_pages(cache, table, 128, 256)
    with pytest.raises(ValueError, match="int32"):
        fpv2.pool_pages(cache, table.long(), 128, 128)
    q = torch.zeros((8, 128, 128), dtype=torch.bfloat16)
    ids = torch.zeros((2, 4, 1), dtype=torch.int32)
    cnt = torch.zeros((2, 4), dtype=torch.int32)
    pk = torch.zeros((2, 1, 128), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="head dimension"):
        fpv2.sparse_attention_paged(q[..., :32], cache[..., :32], cache[..., :32], table, pk, pk,
                                    ids, cnt, ids, cnt, scale=1.0)
    with pytest.raises(ValueError, match="identical shapes"):
        fpv2.sparse_attention_paged(q, cache, cache[:2], table, pk, pk, ids, cnt, ids, cnt, scale=1.0)


def test_workspace_size_queries_without_gpu():
    """The two workspace queries are pure size arithmetic (no device call)."""
    L = _lib.lib()
    hkv, nb, d = 8, 512, 128
    # selection: three 16-bit parts of float32 pooled keys (+ two ints per KV head)
    parts = 3 * hkv * nb * d * 2
    got = L.fpv2_select_workspace_bytes(_lib.BF16, _lib.F32, hkv, nb, d)
    assert got == (parts + 255) // 256 * 256 + 8 * hkv
    assert L.fpv2_select_workspace_bytes(_lib.F16, _lib.F32, hkv, nb, d) == got
    assert L.fpv2_select_workspace_bytes(_lib.BF16, _lib.BF16, hkv, nb, d) == 0   # 16-bit keys need none
    assert L.fpv2_select_workspace_bytes(_lib.F32, _lib.F32, hkv, nb, d) == 0     # CUDA-core path
    # attention: the fp16 copy of bf16 V (and pooled V) leads the split scratch
    args = (32, hkv, 65536, 65536, d, 128, 32)
    bf16 = L.fpv2_attention_workspace_bytes(_lib.BF16, *args, _lib.BF16, 1)
    f16 = L.fpv2_attention_workspace_bytes(_lib.F16, *args, _lib.F16, 1)
    up = lambda x: (x + 255) // 256 * 256
    conv = up(hkv * 65536 * d * 2) + up(hkv * nb * d * 2) + up(hkv * 8)
    assert bf16 - f16 == conv
    assert f16 >= _lib.ATTN_WORKSPACE_BYTES
    assert L.fpv2_attention_workspace_bytes(_lib.F32, *args, _lib.F32, 1) >= _lib.ATTN_WORKSPACE_BYTES


def test_streaming_staging_buffers_are_kept_per_device_and_shape():
    """sdpa_from_host keeps one entry of staging buffers per device: the same
    key reuses it, another key replaces it, release_staging drops it."""
    from fpv2 import stream

    stream.release_staging()
    made = []

    def make():
        made.append(1)
        return [("q", "k", "v")]

    dev = torch.device("cuda", 0)
    e1, fresh1 = stream._staging(dev, ("a",), make)
    e2, fresh2 = stream._staging(dev, ("a",), make)
    assert fresh1 and not fresh2 and e1 is e2 and len(made) == 1
    assert e1[2] == [None, None]
    e3, fresh3 = stream._staging(dev, ("b",), make)
    assert fresh3 and e3 is not e1 and len(stream._STAGING) == 1
    stream._staging(torch.device("cuda", 1), ("a",), make)
    assert len(stream._STAGING) == 2
    stream.release_staging(dev)
    assert list(stream._STAGING) == [torch.device("cuda", 1)]
    stream.release_staging()
    assert not stream._STAGING


@pytest.mark.parametrize("lq,slices,unit", [(65536, 4, 64), (2048, 4, 64), (1920, 4, 64),
                                            (2048, 3, 300), (200, 4, 64), (65536, 1, 64),
                                            (4096, 16, 256)])
def test_streaming_query_slices_cover_the_rows_on_unit_boundaries(lq, slices, unit):
    from fpv2.stream import _slice_bounds

    b = _slice_bounds(lq, slices, unit)
    u = (unit + 127) // 128 * 128
    assert b[0][0] == 0 and b[-1][1] == lq
    assert all(s1 == t0 for (_, s1), (t0, _) in zip(b, b[1:]))   # contiguous, no overlap
    assert all(s0 % u == 0 and s1 > s0 for s0, s1 in b)
    assert b[-1][1] - b[-1][0] >= min(u, lq)                      # the dense tail stays whole
    assert len(b) <= slices
