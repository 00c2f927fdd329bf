"""The torch SDPA hook on a GPU (reference tests/test_patch.py, retargeted to torch).

Eligible causal prefill calls route to FPV2; ineligible calls must be bit
identical to torch's original function; chunked prefill must equal single-shot.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F
from torch.nn.attention.bias import causal_lower_right

import fpv2
from fpv2 import _lib
from fpv2.patch import _ORIGINAL_SDPA, _effective_config, _request_config
from oracle import fpv2_oracle as O
from tests import parity as P
from tests.synthetic import structured_qkv, topic_qkv, uniform_qkv

pytestmark = pytest.mark.gpu
KATS = json.loads((Path(__file__).parent / "golden" / "reference_kats.json").read_text())
DEV = "cuda:0"


@pytest.fixture(autouse=True)
def restore_sdpa():
    fpv2.disable()
    yield
    fpv2.disable()


def inputs(length: int, query_length: int | None = None, seed: int = 7):
    ql = length if query_length is None else query_length
    q, k, v = uniform_qkv((1, 4, ql, 64), (1, 2, length, 64), seed=seed)
    return q.to(DEV), k.to(DEV), v.to(DEV)


def expand_kv(q, k, v):
    """Repeat KV heads to the query heads (torch's lower-right CausalBias path has no GQA)."""
    g = q.shape[1] // k.shape[1]
    return k.repeat_interleave(g, dim=1), v.repeat_interleave(g, dim=1)


def stock(q, k, v, scale):
    lq, lk = q.shape[-2], k.shape[-2]
    if lq == lk:
        return _ORIGINAL_SDPA(q, k, v, is_causal=True, scale=scale, enable_gqa=True)
    ke, ve = expand_kv(q, k, v)
    return _ORIGINAL_SDPA(q, ke, ve, attn_mask=causal_lower_right(lq, lk), scale=scale)


def hooked(q, k, v, scale):
    """The call a model makes; FPV2 claims it when eligible (GQA heads kept packed)."""
    lq, lk = q.shape[-2], k.shape[-2]
    if lq == lk:
        return F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=scale, enable_gqa=True)
    return F.scaled_dot_product_attention(q, k, v, attn_mask=causal_lower_right(lq, lk),
                                          scale=scale, enable_gqa=True)


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-8)).item()


def test_alpha_zero_padded_call_matches_stock():
    q, k, v = inputs(130)
    scale = 64 ** -0.5
    expected = stock(q, k, v, scale)
    fpv2.enable(fpv2.FPV2Config(alpha=0, sink_tokens=0, window_tokens=0), min_tokens=1)
    assert rel_err(hooked(q, k, v, scale), expected) < 2e-2


def test_alpha_zero_unaligned_chunk_matches_stock():
    q, k, v = inputs(190, 128)
    scale = 64 ** -0.5
    expected = stock(q, k, v, scale)
    fpv2.enable(fpv2.FPV2Config(alpha=0, sink_tokens=0, window_tokens=0), min_tokens=1)
    assert rel_err(hooked(q, k, v, scale), expected) < 2e-2


@pytest.mark.parametrize(
    ("length", "query_length", "causal"),
    [(64, 64, True), (128, 1, True), (128, 32, True), (128, 128, False)],
)
def test_ineligible_calls_are_bit_identical(length, query_length, causal):
    q, k, v = inputs(length, query_length)
    scale = 64 ** -0.5
    if causal and query_length != length:
        # lower-right causal chunk (decode / short chunk): KV heads expanded
        k, v = expand_kv(q, k, v)
        bias = causal_lower_right(query_length, length)
        expected = _ORIGINAL_SDPA(q, k, v, attn_mask=bias, scale=scale)
        fpv2.enable(min_tokens=128)
        actual = F.scaled_dot_product_attention(q, k, v, attn_mask=bias, scale=scale)
    else:
        expected = _ORIGINAL_SDPA(q, k, v, is_causal=causal, scale=scale, enable_gqa=True)
        fpv2.enable(min_tokens=128)
        actual = F.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=scale,
                                                enable_gqa=True)
    assert torch.equal(actual, expected)


def test_array_mask_falls_through_and_disable_restores_original():
    q, k, v = inputs(128)
    mask = torch.zeros((128, 128), dtype=torch.bfloat16, device=DEV)
    expected = _ORIGINAL_SDPA(q, k, v, attn_mask=mask, scale=0.125, enable_gqa=True)
    fpv2.enable(min_tokens=1)
    actual = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, scale=0.125, enable_gqa=True)
    assert torch.equal(actual, expected)
    fpv2.disable()
    assert F.scaled_dot_product_attention is _ORIGINAL_SDPA


def test_large_array_mask_falls_through():
    q, k, v = inputs(4096)
    mask = torch.zeros((4096, 4096), dtype=torch.bfloat16, device=DEV)
    expected = _ORIGINAL_SDPA(q, k, v, attn_mask=mask, scale=0.125, enable_gqa=True)
    fpv2.enable(min_tokens=1)
    actual = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, scale=0.125, enable_gqa=True)
    assert torch.equal(actual, expected)


@pytest.mark.parametrize(
    ("key_length", "query_length"),
    [(4_096, 4_096), (4_100, 4_100), (8_192, 2_048), (4_100, 1_000), (6_000, 128)],
)
def test_real_shape_alpha_zero_matches_stock(key_length, query_length):
    q, k, v = uniform_qkv((1, 8, query_length, 128), (1, 2, key_length, 128), seed=17)
    q, k, v = q.to(DEV), k.to(DEV), v.to(DEV)
    scale = 128 ** -0.5
    expected = stock(q, k, v, scale)
    fpv2.enable(fpv2.FPV2Config(alpha=0, sink_tokens=0, window_tokens=0), min_tokens=1)
    actual = hooked(q, k, v, scale)
    assert rel_err(actual, expected) < 2e-2
    assert _lib.device_status() == 0


def test_hook_matches_oracle_sdpa():
    """Eligible call == oracle restatement of fpv2/patch.py:102-174 (alpha 0.15, correction)."""
    q, k, v = structured_qkv(length=4100, query_heads=8, kv_heads=2, head_dim=128,
                             dtype=torch.bfloat16, seed=19)
    q4, k4, v4 = q[None].to(DEV), k[None].to(DEV), v[None].to(DEV)
    cfg = fpv2.FPV2Config(alpha=0.15, mean_correction=True)
    fpv2.enable(cfg, min_tokens=1, total_tokens=4100)
    actual = hooked(q4, k4, v4, 128 ** -0.5)
    exp, _, _ = O.fpv2_sdpa(P.np32(q)[None], P.np32(k)[None], P.np32(v)[None], scale=128 ** -0.5,
                            config=cfg, dtype="bf16")
    mx, mean = P.attention_errors(actual[0], exp[0])
    assert mx < 2e-2 and mean < 2e-3, (mx, mean)


def test_tile_aligned_chunks_match_single_shot_fpv2():
    """Reference tests/test_patch.py:136-166: 4 x 2048 chunks == one 8192 prefill."""
    q, k, v = structured_qkv(length=8192, query_heads=8, kv_heads=2, head_dim=128,
                             dtype=torch.bfloat16, seed=23)
    q, k, v = q[None].to(DEV), k[None].to(DEV), v[None].to(DEV)
    config = fpv2.FPV2Config(alpha=0.15, mean_correction=True)
    scale = 128 ** -0.5
    expected = fpv2.fpv2_sdpa(q, k, v, scale=scale, config=config)
    chunks = []
    for end in range(2048, 8193, 2048):
        chunk_config = _request_config(config, end, q.shape[-2])
        chunks.append(fpv2.fpv2_sdpa(q[:, :, end - 2048:end], k[:, :, :end], v[:, :, :end],
                                     scale=scale, config=chunk_config))
    actual = torch.cat(chunks, dim=2)
    assert rel_err(actual, expected) < 1e-2


def test_eligible_shape_that_needs_autograd_falls_through():
    """An otherwise eligible call whose inputs require grad goes to torch's SDPA
    (bit-identical, with a backward graph); the same call under no_grad is FPV2."""
    q, k, v = inputs(4096)
    q.requires_grad_(True)
    scale = 64 ** -0.5
    expected = stock(q, k, v, scale)
    fpv2.enable(fpv2.FPV2Config(alpha=1.0), min_tokens=1)   # sparse: only forced blocks and the max
    actual = hooked(q, k, v, scale)
    assert actual.grad_fn is not None and torch.equal(actual, expected)
    actual.float().sum().backward()
    assert q.grad is not None
    with torch.no_grad():
        sparse = hooked(q, k, v, scale)
    assert sparse.grad_fn is None and not torch.equal(sparse, expected)


def test_chunked_prefill_with_total_tokens_matches_oracle():
    """A 16k prompt of the topic-block generator (config 2 shape) prefilled in
    2048-token chunks through the hook, ``total_tokens`` known: the first chunk is
    below ``min_tokens`` and goes to the stock path, the others are FPV2 with
    ``offset = end - 2048`` and the dense tail only at the last chunk
    (fpv2/patch.py:55-63, 197-198). Every chunk is compared with the oracle's
    restatement of that call at float32 output, and block sparsity is well above 0."""
    L, chunk, min_tokens = 16384, 2048, 4096
    q, k, v = topic_qkv(length=L, query_heads=32, kv_heads=8, head_dim=128, seed=5,
                        dtype=torch.bfloat16)
    q4, k4, v4 = q[None].to(DEV), k[None].to(DEV), v[None].to(DEV)
    cfg = fpv2.FPV2Config(alpha=0.1)
    scale = 128 ** -0.5
    fpv2.enable(cfg, min_tokens=min_tokens, collect_stats=True, total_tokens=L)
    outs = [hooked(q4[:, :, end - chunk:end], k4[:, :, :end], v4[:, :, :end], scale)
            for end in range(chunk, L + 1, chunk)]
    sparsity = fpv2.block_sparsity()
    fpv2.disable()
    assert _lib.device_status() == 0
    assert sparsity > 0.3, sparsity
    qf, kf, vf = P.np32(q), P.np32(k), P.np32(v)
    for i, end in enumerate(range(chunk, L + 1, chunk)):
        qc = qf[:, end - chunk:end]
        if end < min_tokens:
            exp = O.exact_causal_attention(qc, kf[:, :end], vf[:, :end], scale, offset=end - chunk)
        else:
            c = O.request_config(cfg, end, L)
            exp = O.fpv2_sdpa(qc[None], kf[None, :, :end], vf[None, :, :end], scale=scale, config=c,
                              dtype="bf16", out_dtype="fp32")[0][0]
        mx, mean = P.attention_errors(outs[i][0], exp)
        assert mx <= P.MAX_ABS_TOL and mean <= P.MEAN_ABS_TOL, (end, mx, mean)


def test_block_sparsity_includes_dense_gated_prefill():
    k = KATS["block_sparsity"]
    q, kk, v = inputs(k["first_length"])
    scale = 64 ** -0.5
    fpv2.enable(fpv2.FPV2Config(**k["config"]), min_tokens=k["min_tokens"], collect_stats=True)
    F.scaled_dot_product_attention(q, kk, v, is_causal=True, scale=scale, enable_gqa=True)
    assert fpv2.block_sparsity() == pytest.approx(k["expected_first"])
    q, kk, v = inputs(k["second_length"])
    F.scaled_dot_product_attention(q, kk, v, is_causal=True, scale=scale, enable_gqa=True)
    assert fpv2.block_sparsity() == pytest.approx(k["expected_second"])


def test_effective_config_matches_oracle():
    for hq, hkv in [(32, 8), (64, 8), (8, 8), (16, 2)]:
        a = _effective_config(fpv2.FPV2Config(), hq, hkv)
        b = O.effective_config(O.OracleConfig(), hq, hkv)
        assert (a is None) == (b is None)
        if a is not None:
            assert a.tile_q == b.tile_q
