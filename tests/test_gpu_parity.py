"""CUDA path vs the CPU oracle: pooling, selection, compaction, attention.

Every test here calls the C-ABI library through the public ``fpv2`` operators on
``cuda:0`` and checks the result against oracle/fpv2_oracle.py on the same
seeded inputs (tolerances in tests/parity.py).
"""

from __future__ import annotations

import json
from dataclasses import replace
from pathlib import Path

import numpy as np
import pytest
import torch

import fpv2
from fpv2 import _lib
from fpv2.patch import _effective_config
from oracle import fpv2_oracle as O
from tests import parity as P
from tests.synthetic import structured_qkv, topic_qkv

pytestmark = pytest.mark.gpu
KATS = json.loads((Path(__file__).parent / "golden" / "reference_kats.json").read_text())
DEV = "cuda:0"


def cuda(*ts):
    return [t.to(DEV) for t in ts]


# ---------------------------------------------------------------------------
# pooling
# ---------------------------------------------------------------------------


def test_pool_kat_on_gpu():
    x = torch.arange(32, dtype=torch.float32).reshape(2, 8, 2).to(DEV)
    out = fpv2.pool_blocks(x, 4)
    assert out.cpu().tolist() == KATS["pool_blocks"]["expected"]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("head_dim", [128, 64, 96, 3])
def test_pool_bit_exact(dtype, head_dim):
    g = torch.Generator().manual_seed(head_dim)
    x = (torch.randn((3, 512, head_dim), generator=g) * 2).to(dtype)
    gpu = fpv2.pool_blocks(x.to(DEV), 128)
    ref = O.pool_blocks(P.np32(x), 128, P.dtname(dtype))
    assert gpu.dtype == dtype
    assert np.array_equal(P.np32(gpu), ref)


# ---------------------------------------------------------------------------
# selection known-answer tests (reference tests/test_selection.py)
# ---------------------------------------------------------------------------


def test_partially_visible_block_kat_on_gpu():
    k = KATS["partially_visible_block"]
    q = torch.tensor(k["q"], device=DEV)
    pk = torch.tensor(k["pooled_k"], device=DEV)
    sel, _ = fpv2.block_scores_and_select(q, pk, scale=k["scale"],
                                          config=fpv2.FPV2Config(**k["config"]), offset=k["offset"])
    assert sel.cpu().tolist() == k["expected"]


def test_last_n_dense_tail_kat_on_gpu():
    k = KATS["last_n_dense_tail"]
    q = torch.full(k["q_shape"], k["q_fill"], device=DEV)
    pk = torch.full(k["pooled_k_shape"], k["pooled_k_fill"], device=DEV)
    sel, _ = fpv2.block_scores_and_select(q, pk, scale=k["scale"],
                                          config=fpv2.FPV2Config(**k["config"]))
    assert sel.cpu().tolist() == k["expected"]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_alpha_zero_lower_triangle_on_gpu(dtype):
    k = KATS["alpha_zero_lower_triangle"]
    c = fpv2.FPV2Config(**k["config"])
    q, kk, _ = structured_qkv(length=256, query_heads=8, kv_heads=2, block_size=32, dtype=dtype)
    q, kk = cuda(q, kk)
    sel, raw = fpv2.block_scores_and_select(q, fpv2.pool_blocks(kk, 32), scale=64 ** -0.5, config=c)
    expected = torch.tril(torch.ones(8, 8, dtype=torch.bool)).expand(2, 8, 8)
    assert torch.equal(sel.cpu(), expected)
    assert raw is not None and raw.shape == (2, 4, 256, 8)
    assert fpv2.density(sel, config=c).item() == pytest.approx(1.0)


# ---------------------------------------------------------------------------
# selection parity (tcgen05 and generic paths)
# ---------------------------------------------------------------------------

SELECT_CASES = [
    # length, Hq, Hkv, D, dtype, alpha, seed[, tile_q (default: 128 packed rows)]
    (2048, 8, 2, 128, torch.bfloat16, 0.1, 0),
    (2048, 8, 2, 128, torch.float16, 0.15, 1),
    (4096, 32, 8, 128, torch.bfloat16, 0.1, 2),
    (2048, 8, 2, 64, torch.bfloat16, 0.1, 3),
    (2048, 16, 2, 128, torch.bfloat16, 0.05, 4),    # G = 8, tile_q = 16
    (2048, 8, 2, 96, torch.bfloat16, 0.1, 5),       # tensor cores on zero-padded 128-wide tiles
    (2048, 8, 2, 256, torch.bfloat16, 0.1, 6),      # 256-wide chunks, single-buffered Q
    (2048, 8, 2, 48, torch.bfloat16, 0.1, 7),       # generic CUDA-core path
    (1024, 8, 2, 128, torch.float32, 0.1, 6),       # generic, fp32
    (2048, 8, 2, 128, torch.bfloat16, 0.1, 8, 256),   # 8 query chunks per tile: two items interleaved
    (4096, 8, 2, 128, torch.float16, 0.15, 9, 128),
    (2048, 8, 2, 64, torch.bfloat16, 0.1, 10, 64),
    (2048, 8, 2, 256, torch.bfloat16, 0.1, 11, 128),  # 256-wide chunks: one item at a time
]


@pytest.mark.parametrize("case", SELECT_CASES,
                         ids=lambda c: f"L{c[0]}-Hq{c[1]}-D{c[3]}-{c[4]}" + (f"-t{c[7]}" if len(c) > 7 else ""))
def test_selection_parity(case):
    length, hq, hkv, d, dtype, alpha, seed = case[:7]
    tile_q = case[7] if len(case) > 7 else None
    q, k, v = topic_qkv(length=length, query_heads=hq, kv_heads=hkv, head_dim=d, seed=seed,
                        dtype=dtype)
    cfg = _effective_config(fpv2.FPV2Config(alpha=alpha, score_chunk_tiles=8), hq, hkv)
    if tile_q is not None:
        cfg = replace(cfg, tile_q=tile_q)
    qg, kg = cuda(q, k)
    pk = fpv2.pool_blocks(kg, 128)
    pk_ref = O.pool_blocks(P.np32(k), 128, P.dtname(dtype))
    assert np.array_equal(P.np32(pk), pk_ref)
    scale = d ** -0.5
    sel, raw = fpv2.block_scores_and_select(qg, pk, scale=scale, config=cfg)
    assert raw is None
    chk = P.check_selection(q, pk_ref, sel.cpu().numpy(), scale=scale, config=cfg)
    assert chk.ok, chk


SELECT_F32_CASES = [
    # length, Hq, Hkv, D, q dtype, alpha, seed[, tile_q]: float32 pooled keys
    (2048, 8, 2, 128, torch.bfloat16, 0.1, 30),
    (2048, 8, 2, 128, torch.float16, 0.15, 31),
    (2048, 16, 2, 128, torch.float16, 0.05, 32),     # G = 8, tile_q = 16
    (2048, 8, 2, 64, torch.bfloat16, 0.1, 33),
    (2048, 8, 2, 256, torch.bfloat16, 0.1, 34),
    (2048, 8, 2, 96, torch.bfloat16, 0.1, 37),       # zero-padded 128-wide tiles
    (2048, 8, 2, 128, torch.bfloat16, 0.1, 35, 256),
]


def _select_f32(qg, pk, scale, cfg, workspace):
    """fpv2_block_select on float32 pooled keys with or without the split workspace
    (without: the CUDA-core kernel)."""
    hkv, nb, d = pk.shape
    mask = torch.empty((hkv, qg.shape[1] // cfg.tile_q, nb), dtype=torch.uint8, device=DEV)
    ws = _lib.select_workspace(qg, pk.dtype, hkv, nb, d) if workspace else None
    assert (ws is not None) == workspace
    _lib.check(_lib.lib().fpv2_block_select(
        _lib.ptr(qg), _lib.dtype_code(qg.dtype), _lib.ptr(pk), _lib.dtype_code(pk.dtype),
        qg.shape[0], hkv, qg.shape[1], nb, d, 0, qg.shape[1], float(scale), cfg.block_k,
        cfg.tile_q, float(cfg.alpha), cfg.sink_tokens, cfg.window_tokens, cfg.last_n_blocks,
        _lib.ptr(mask), None, *_lib.workspace_args(ws), _lib.stream_of(qg)))
    return mask.cpu().numpy().astype(bool)


@pytest.mark.parametrize("case", SELECT_F32_CASES,
                         ids=lambda c: f"L{c[0]}-Hq{c[1]}-D{c[3]}-{c[4]}" + (f"-t{c[7]}" if len(c) > 7 else ""))
def test_selection_parity_float32_pooled_keys(case):
    """16-bit queries on float32 pooled keys (fpv2/reference.py:45-51 semantics):
    the tensor-core kernel scores three 16-bit parts of each key; its selection
    and the CUDA-core kernel's both match the float32 oracle."""
    length, hq, hkv, d, dtype, alpha, seed = case[:7]
    q, k, _ = topic_qkv(length=length, query_heads=hq, kv_heads=hkv, head_dim=d, seed=seed,
                        dtype=dtype)
    cfg = _effective_config(fpv2.FPV2Config(alpha=alpha, score_chunk_tiles=8), hq, hkv)
    if len(case) > 7:
        cfg = replace(cfg, tile_q=case[7])
    pk_ref = O.pool_blocks(P.np32(k), 128, "fp32")
    qg, pk = q.to(DEV), torch.from_numpy(pk_ref).to(DEV)
    scale = d ** -0.5
    sel, _ = fpv2.block_scores_and_select(qg, pk, scale=scale, config=cfg)
    chk = P.check_selection(q, pk_ref, sel.cpu().numpy(), scale=scale, config=cfg)
    assert chk.ok, chk
    tc, cc = _select_f32(qg, pk, scale, cfg, True), _select_f32(qg, pk, scale, cfg, False)
    assert np.array_equal(tc, sel.cpu().numpy())
    chk = P.check_selection(q, pk_ref, cc, scale=scale, config=cfg)
    assert chk.ok, chk
    assert (tc != cc).mean() < 1e-3


def test_selection_float32_pooled_keys_beyond_fp16_range():
    """Pooled keys of 2^20 times ordinary magnitude with fp16 queries: the heads'
    16-bit parts are scaled by 2^-e into range and scored at 2^e, so the selection
    is that of the unscaled keys at scale * 2^-20 (exact in float32)."""
    q, k, _ = topic_qkv(length=2048, query_heads=8, kv_heads=2, seed=36, dtype=torch.float16)
    cfg = _effective_config(fpv2.FPV2Config(alpha=0.1, score_chunk_tiles=8), 8, 2)
    pk_ref = O.pool_blocks(P.np32(k), 128, "fp32")
    big = pk_ref * np.float32(2.0 ** 20)
    assert np.abs(big).max() > 65504
    scale = 128 ** -0.5
    qg = q.to(DEV)
    sel, _ = fpv2.block_scores_and_select(qg, torch.from_numpy(big).to(DEV),
                                          scale=scale * 2.0 ** -20, config=cfg)
    assert _lib.device_status() == 0
    chk = P.check_selection(q, big, sel.cpu().numpy(), scale=scale * 2.0 ** -20, config=cfg)
    assert chk.ok, chk
    ref, _ = fpv2.block_scores_and_select(qg, torch.from_numpy(pk_ref).to(DEV), scale=scale,
                                          config=cfg)
    assert (sel != ref).float().mean().item() < 1e-3


@pytest.mark.parametrize("offset,query_length", [(37, 55), (0, 160), (64, 96)])
def test_selection_offset_and_padding(offset, query_length):
    """Chunk offsets and padded query rows (reference tests/test_selection.py:114-144)."""
    c = fpv2.FPV2Config(block_k=16, tile_q=16, alpha=0.4, sink_tokens=16, window_tokens=16)
    q, k, _ = structured_qkv(length=160, query_heads=4, kv_heads=2, block_size=16, seed=11)
    pad = (query_length + 15) // 16 * 16
    pq = torch.zeros((4, pad, q.shape[-1]))
    pq[:, :query_length] = q[:, offset:offset + query_length]
    pk_ref = O.pool_blocks(P.np32(k), 16)
    sel, _ = fpv2.block_scores_and_select(pq.to(DEV), torch.from_numpy(pk_ref).to(DEV),
                                          scale=q.shape[-1] ** -0.5, config=c, offset=offset,
                                          query_length=query_length)
    chk = P.check_selection(pq, pk_ref, sel.cpu().numpy(), scale=q.shape[-1] ** -0.5, config=c,
                            offset=offset, query_length=query_length)
    assert chk.ok, chk


def test_chunked_scoring_matches_unchunked_on_gpu():
    c = fpv2.FPV2Config(block_k=16, tile_q=16, alpha=0.35, sink_tokens=16, window_tokens=32)
    q, k, _ = structured_qkv(length=160, query_heads=8, kv_heads=2, block_size=16, seed=7)
    q, k = cuda(q, k)
    pk = fpv2.pool_blocks(k, 16)
    a, sa = fpv2.block_scores_and_select(q, pk, scale=64 ** -0.5, config=c)
    b, sb = fpv2.block_scores_and_select(q, pk, scale=64 ** -0.5, config=replace(c, score_chunk_tiles=3))
    assert sa is not None and sb is None
    assert torch.equal(a, b)


def test_raw_scores_match_oracle():
    c = fpv2.FPV2Config(alpha=0.1)
    q, k, _ = topic_qkv(length=512, query_heads=8, kv_heads=2, seed=9, dtype=torch.bfloat16)
    qg, kg = cuda(q, k)
    pk = fpv2.pool_blocks(kg, 128)
    _, raw = fpv2.block_scores_and_select(qg, pk, scale=128 ** -0.5, config=c)
    ref = O.block_scores_and_select(P.np32(q), P.np32(pk), scale=128 ** -0.5, config=c).raw_scores
    assert np.allclose(raw.cpu().numpy(), ref, rtol=1e-5, atol=1e-4)


# ---------------------------------------------------------------------------
# compaction and the fused index stage
# ---------------------------------------------------------------------------


def test_compaction_kat_on_gpu():
    k = KATS["compaction_order"]
    ids, counts, _, _ = fpv2.compact_block_indices(torch.tensor(k["selected"], device=DEV),
                                                   config=fpv2.FPV2Config(**k["config"]))
    assert counts.item() == k["count"]
    assert ids[0, 0, : k["count"]].tolist() == k["prefix"]


@pytest.mark.parametrize("nb,key_length,offset", [(37, 37 * 16, 5), (64, 1000, 0), (130, 130 * 16, 100)])
def test_compaction_random_masks_bit_exact(nb, key_length, offset):
    g = torch.Generator().manual_seed(nb)
    c = fpv2.FPV2Config(block_k=16, tile_q=16)
    nt = 12
    mask = torch.rand((3, nt, nb), generator=g) < 0.4
    ql = min(nt * 16, key_length - offset)
    lists = fpv2.compact_block_indices(mask.to(DEV), config=c, offset=offset, query_length=ql,
                                       key_length=key_length)
    assert P.check_lists_of_mask(mask.numpy(), lists, config=c, offset=offset, query_length=ql,
                                 key_length=key_length)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("offset", [0, 1024])
def test_index_stage_parity(dtype, offset):
    length = 2048
    q, k, v = topic_qkv(length=length, query_heads=8, kv_heads=2, seed=21, dtype=dtype)
    q = q[:, offset:]
    ql = q.shape[1]
    cfg = _effective_config(fpv2.FPV2Config(alpha=0.1), 8, 2)
    qg, kg, vg = cuda(q, k, v)
    pk, pv, lists, mask = fpv2.index_stage(qg, kg, vg, scale=128 ** -0.5, config=cfg, offset=offset,
                                           query_length=ql, key_length=length, return_mask=True)
    pk_ref = O.pool_blocks(P.np32(k), 128, P.dtname(dtype))
    assert np.array_equal(P.np32(pk), pk_ref)
    assert np.array_equal(P.np32(pv), O.pool_blocks(P.np32(v), 128, P.dtname(dtype)))
    m = mask.cpu().numpy()
    chk = P.check_selection(q, pk_ref, m, scale=128 ** -0.5, config=cfg, offset=offset)
    assert chk.ok, chk
    assert P.check_lists_of_mask(m, lists, config=cfg, offset=offset, query_length=ql,
                                 key_length=length)
    # the operator-by-operator path gives the same mask
    sel, _ = fpv2.block_scores_and_select(qg, pk, scale=128 ** -0.5,
                                          config=replace(cfg, score_chunk_tiles=4), offset=offset)
    assert torch.equal(sel, mask)


def test_index_stage_float32_pooling_semantics():
    """pooled_dtype=float32 selects on fp32 pooled keys, as fpv2/reference.py does."""
    q, k, v = topic_qkv(length=2048, query_heads=8, kv_heads=2, seed=22, dtype=torch.bfloat16)
    cfg = _effective_config(fpv2.FPV2Config(alpha=0.1), 8, 2)
    qg, kg, vg = cuda(q, k, v)
    pk, pv, lists, mask = fpv2.index_stage(qg, kg, vg, scale=128 ** -0.5, config=cfg, offset=0,
                                           query_length=2048, key_length=2048,
                                           pooled_dtype=torch.float32, return_mask=True)
    pk_ref = O.pool_blocks(P.np32(k), 128, "fp32")
    assert pk.dtype == torch.float32 and np.array_equal(P.np32(pk), pk_ref)
    chk = P.check_selection(q, pk_ref, mask.cpu().numpy(), scale=128 ** -0.5, config=cfg)
    assert chk.ok, chk


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------


def _attention_case(q, k, v, config, *, offset=0, tile=None, pooled_dtype=None):
    """Run the GPU path twice and return (hook_out, kernel_oracle, ref_out, reference).

    * hook semantics (fpv2/patch.py): keys pooled in the input dtype, operator by
      operator; checked against the list-driven oracle on the GPU's own lists;
    * reference.py semantics (fpv2/reference.py:45-51): selection on float32
      pooled keys through the fused index stage; checked against the float32
      reference math.
    """
    scale = q.shape[-1] ** -0.5
    qg, kg, vg = cuda(q, k, v)
    ql, kl = q.shape[1], k.shape[1]
    pk = fpv2.pool_blocks(kg, config.block_k)
    pv = fpv2.pool_blocks(vg, config.block_k)
    if pooled_dtype is not None:
        pk, pv = pk.to(pooled_dtype), pv.to(pooled_dtype)
    sel, _ = fpv2.block_scores_and_select(qg, pk, scale=scale,
                                          config=replace(config, score_chunk_tiles=4), offset=offset)
    lists = fpv2.compact_block_indices(sel, config=config, offset=offset, query_length=ql,
                                       key_length=kl)
    out = fpv2.sparse_attention(qg, kg, vg, pk, pv, *lists, scale=scale, config=config, offset=offset,
                                tile=tile)
    pk32, pv32, lists32, _ = fpv2.index_stage(qg, kg, vg, scale=scale, config=config, offset=offset,
                                              query_length=ql, key_length=kl,
                                              pooled_dtype=torch.float32)
    out_ref = fpv2.sparse_attention(qg, kg, vg, pk32, pv32, *lists32, scale=scale, config=config,
                                    offset=offset, tile=tile)
    assert _lib.device_status() == 0
    qf, kf, vf = P.np32(q), P.np32(k), P.np32(v)
    np_lists = [x.cpu().numpy() for x in lists]
    kern = O.sparse_attention(qf, kf, vf, P.np32(pk), P.np32(pv), *np_lists, scale=scale,
                              config=config, offset=offset, dtype=P.dtname(q.dtype))
    ref = O.fpv2_attention_blockwise(qf, kf, vf, scale=scale, config=config, offset=offset)
    return out, kern, out_ref, ref


ATTN_CASES = [
    # D, dtype, corr, alpha, tile_q (None = effective 128/G)
    (128, torch.bfloat16, True, 0.15, None),
    (128, torch.bfloat16, False, 0.15, None),
    (128, torch.float16, True, 0.1, None),
    (64, torch.bfloat16, True, 0.15, None),
    (128, torch.bfloat16, True, 0.0, None),
    (128, torch.bfloat16, True, 0.15, 128),   # direct 128-position tiles: 4 chunks per tile (pairs)
    (128, torch.float16, True, 0.1, 128),
    (128, torch.bfloat16, False, 0.0, 128),
    (64, torch.bfloat16, True, 0.15, 128),
    (96, torch.bfloat16, True, 0.15, 128),
    (128, torch.bfloat16, True, 0.15, 64),    # 2 chunks of 2 heads x 64 positions (pair)
    (128, torch.bfloat16, True, 0.15, 256),   # 8 chunks: pairs of heads at each position slice
    (96, torch.bfloat16, True, 0.15, None),   # tensor cores on zero-padded 128-wide tiles
    (96, torch.float16, False, 0.1, None),
    (256, torch.bfloat16, True, 0.15, None),  # attn_wide_kernel
    (256, torch.float16, False, 0.1, None),
]


@pytest.mark.parametrize("case", ATTN_CASES, ids=lambda c: f"D{c[0]}-{c[1]}-corr{c[2]}-a{c[3]}-t{c[4]}")
def test_attention_parity(case):
    d, dtype, corr, alpha, tile_q = case
    q, k, v = structured_qkv(length=2048, query_heads=8, kv_heads=2, head_dim=d, dtype=dtype,
                             seed=31 + d)
    base = fpv2.FPV2Config(alpha=alpha, sink_tokens=128, window_tokens=256, mean_correction=corr)
    cfg = replace(base, tile_q=tile_q) if tile_q else _effective_config(base, 8, 2)
    out, kern, out_ref, ref = _attention_case(q, k, v, cfg)
    mx_k, mean_k = P.kernel_errors(out, kern)
    assert mx_k <= P.KERNEL_MAX_ABS_TOL and mean_k <= P.KERNEL_MEAN_ABS_TOL, (mx_k, mean_k)
    mx_r, mean_r = P.attention_errors(out_ref, ref)
    assert mx_r <= P.MAX_ABS_TOL and mean_r <= P.MEAN_ABS_TOL, (mx_r, mean_r)


GQA8_CASES = [
    # Hq, Hkv, length, dtype, corr: G = 8 packs 16 query positions x 8 heads per
    # 128-row tile (fpv2/patch.py:41-52), the packing of config 5
    (16, 2, 4096, torch.bfloat16, True),
    (16, 2, 4096, torch.float16, False),
    (64, 8, 4096, torch.float16, True),
    (64, 8, 4096, torch.bfloat16, False),
    (64, 8, 8192, torch.bfloat16, True),
]


@pytest.mark.parametrize("case", GQA8_CASES, ids=lambda c: f"Hq{c[0]}-Hkv{c[1]}-L{c[2]}-{c[3]}-corr{c[4]}")
def test_attention_parity_gqa8(case):
    hq, hkv, length, dtype, corr = case
    q, k, v = topic_qkv(length=length, query_heads=hq, kv_heads=hkv, head_dim=128, seed=hq + length,
                        dtype=dtype)
    cfg = _effective_config(fpv2.FPV2Config(alpha=0.1, mean_correction=corr), hq, hkv)
    assert cfg.tile_q == 16
    out, kern, out_ref, ref = _attention_case(q, k, v, cfg)
    mx_k, mean_k = P.kernel_errors(out, kern)
    assert mx_k <= P.KERNEL_MAX_ABS_TOL and mean_k <= P.KERNEL_MEAN_ABS_TOL, (mx_k, mean_k)
    mx_r, mean_r = P.attention_errors(out_ref, ref)
    assert mx_r <= P.MAX_ABS_TOL and mean_r <= P.MEAN_ABS_TOL, (mx_r, mean_r)


@pytest.mark.parametrize("offset,query_length", [(1024, 1024), (1920, 128)])
def test_attention_chunk_offsets(offset, query_length):
    """Reference tests/test_kernel.py:135-160 (chunk offsets)."""
    full_q, k, v = structured_qkv(length=2048, query_heads=8, kv_heads=2, head_dim=128,
                                  dtype=torch.bfloat16, seed=37)
    q = full_q[:, offset:offset + query_length]
    cfg = _effective_config(fpv2.FPV2Config(alpha=0.15, sink_tokens=128, window_tokens=256), 8, 2)
    out, kern, out_ref, ref = _attention_case(q, k, v, cfg, offset=offset)
    mx_r, mean_r = P.attention_errors(out_ref, ref)
    assert mx_r <= P.MAX_ABS_TOL and mean_r <= P.MEAN_ABS_TOL, (mx_r, mean_r)
    mx_k, mean_k = P.kernel_errors(out, kern)
    assert mx_k <= P.KERNEL_MAX_ABS_TOL and mean_k <= P.KERNEL_MEAN_ABS_TOL, (mx_k, mean_k)


@pytest.mark.parametrize("corr", [False, True])
@pytest.mark.parametrize("head_dim", [64, 96, 128, 256])
def test_small_block_kernel_matches_reference(corr, head_dim):
    """Reference tests/test_kernel.py:18-63: block_k = tile_q = 16 (generic path)."""
    c = fpv2.FPV2Config(block_k=16, tile_q=16, alpha=0.15, sink_tokens=16, window_tokens=16,
                        mean_correction=corr)
    q, k, v = structured_qkv(length=64, query_heads=4, kv_heads=2, head_dim=head_dim,
                             block_size=16, dtype=torch.bfloat16)
    out, kern, out_ref, ref = _attention_case(q, k, v, c)
    rel = np.abs(P.np32(out_ref) - ref).max() / max(np.abs(ref).max(), 1e-8)
    assert rel < 2e-2
    mx_k, mean_k = P.kernel_errors(out, kern)
    assert mx_k <= P.KERNEL_MAX_ABS_TOL and mean_k <= P.KERNEL_MEAN_ABS_TOL, (mx_k, mean_k)


def test_attention_float32_pooled_inputs():
    q, k, v = structured_qkv(length=2048, query_heads=8, kv_heads=2, head_dim=128,
                             dtype=torch.bfloat16, seed=41)
    cfg = _effective_config(fpv2.FPV2Config(alpha=0.15, sink_tokens=128, window_tokens=256), 8, 2)
    out, kern, out_ref, ref = _attention_case(q, k, v, cfg, pooled_dtype=torch.float32)
    mx_r, mean_r = P.attention_errors(out, ref)
    assert mx_r <= P.MAX_ABS_TOL and mean_r <= P.MEAN_ABS_TOL
    mx_k, mean_k = P.kernel_errors(out, kern)
    assert mx_k <= P.KERNEL_MAX_ABS_TOL and mean_k <= P.KERNEL_MEAN_ABS_TOL, (mx_k, mean_k)


def test_alpha_zero_equals_dense_causal_attention():
    """alpha = 0, no correction: FPV2 equals exact causal attention."""
    q, k, v = topic_qkv(length=2048, query_heads=8, kv_heads=2, seed=43, dtype=torch.bfloat16)
    cfg = _effective_config(fpv2.FPV2Config(alpha=0.0, sink_tokens=0, window_tokens=0,
                                            mean_correction=False), 8, 2)
    out, _, _, _ = _attention_case(q, k, v, cfg)
    exact = O.exact_causal_attention(P.np32(q), P.np32(k), P.np32(v), 128 ** -0.5)
    mx, mean = P.attention_errors(out, exact)
    assert mx <= P.MAX_ABS_TOL and mean <= P.MEAN_ABS_TOL


def test_fast_path_mask():
    assert _lib.fast_path_mask(torch.bfloat16, 32, 8, 128, 128, 32, 512) == 3
    assert _lib.fast_path_mask(torch.bfloat16, 8, 2, 96, 128, 32, 16) == 3
    assert _lib.fast_path_mask(torch.bfloat16, 8, 2, 256, 128, 32, 16) == 3
    assert _lib.fast_path_mask(torch.bfloat16, 8, 2, 48, 128, 32, 16) == 0


def test_bounded_wait_times_out_and_context_survives():
    """Failure detection: a wait nobody satisfies expires with a status, no hang/fault."""
    stream = torch.cuda.current_stream().cuda_stream
    rc = _lib.lib().fpv2_selftest_wait_timeout(50.0, stream)
    assert rc == _lib.ERR_DEVICE_TIMEOUT
    assert "bounded wait" in _lib.lib().fpv2_last_error().decode()
    x = torch.ones(4, device=DEV)
    assert x.sum().item() == 4.0   # context still usable
    assert _lib.device_status() == 0


# ---------------------------------------------------------------------------
# workspace-dependent paths: fp16 copy of V, KV-segment split of long items
# ---------------------------------------------------------------------------


def _attention_with_workspace(q, k, v, pk, pv, lists, cfg, scale, nbytes):
    """fpv2_sparse_attention through the C ABI with a workspace of ``nbytes``."""
    import ctypes

    out = torch.full_like(q, float("nan"))
    ws = torch.zeros((max(nbytes, 16) + 3) // 4, dtype=torch.int32, device=q.device)
    rc = _lib.lib().fpv2_sparse_attention(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), pk.data_ptr(), pv.data_ptr(),
        _lib.dtype_code(pk.dtype), lists[0].data_ptr(), lists[1].data_ptr(), lists[2].data_ptr(),
        lists[3].data_ptr(), _lib.dtype_code(q.dtype), q.shape[0], k.shape[0], q.shape[1],
        k.shape[1], q.shape[2], 0, q.shape[1], k.shape[1], ctypes.c_float(scale), cfg.block_k,
        cfg.tile_q, 1 if cfg.mean_correction else 0, out.data_ptr(), ws.data_ptr(),
        ws.numel() * 4, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.OK, _lib.lib().fpv2_last_error().decode()
    return out


@pytest.mark.parametrize("head_dim,dtype,pooled", [(128, torch.bfloat16, None), (64, torch.bfloat16, None),
                                                   (96, torch.float16, None),
                                                   (128, torch.bfloat16, torch.float32)])
def test_long_items_split_over_segments(head_dim, dtype, pooled):
    """At 32k the dense-tail tiles walk 256 key blocks: with the full workspace they
    are split into segments whose partial results a combine kernel merges. The
    split layer agrees with the unsplit one (same P.V precision, workspace without
    the split scratch) to within rounding, and with the float32 math. Head dims
    64 and 96 (128-wide tiles) exercise the other partial-slot widths, fp16 the
    path without the V copy, float32 pooled inputs the gathered high/low
    correction items of fpv2/reference.py's semantics."""
    length, hq, hkv, d = 32768, 8, 2, head_dim
    q, k, v = topic_qkv(length=length, query_heads=hq, kv_heads=hkv, head_dim=d, seed=61, dtype=dtype)
    cfg = _effective_config(fpv2.FPV2Config(alpha=0.1), hq, hkv)
    scale = d ** -0.5
    qg, kg, vg = cuda(q, k, v)
    pk, pv, lists, mask = fpv2.index_stage(qg, kg, vg, scale=scale, config=cfg, offset=0,
                                           query_length=length, key_length=length, return_mask=True,
                                           pooled_dtype=pooled)
    code = _lib.dtype_code(dtype)
    full = _lib.lib().fpv2_attention_workspace_bytes(code, hq, hkv, length, length, d, 128,
                                                     cfg.tile_q, _lib.dtype_code(pk.dtype), 1)
    nt = length // cfg.tile_q
    split = _attention_with_workspace(qg, kg, vg, pk, pv, lists, cfg, scale, full)
    default = fpv2.sparse_attention(qg, kg, vg, pk, pv, *lists, scale=scale, config=cfg)
    assert torch.equal(split, default)   # the Python operator sizes its workspace the same way
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    nb = length // 128
    v_copy = 0
    if dtype == torch.bfloat16:
        v_copy = ((hkv * length * d * 2 + 255) // 256 * 256 + (hkv * nb * d * 2 + 255) // 256 * 256
                  + (hkv * 8 + 255) // 256 * 256)
    unsplit = _attention_with_workspace(qg, kg, vg, pk, pv, lists, cfg, scale, v_copy + 4096)
    mx, mean = P.kernel_errors(split, P.np32(unsplit))
    assert mx <= 2 ** -7 and mean <= 1e-5, (mx, mean)
    tiles = [0, nt // 2, nt - 3, nt - 2, nt - 1]
    ref = O.fpv2_attention_blockwise(P.np32(q), P.np32(k), P.np32(v), scale=scale, config=cfg,
                                     selected=mask.cpu().numpy(),
                                     pooled_dtype="fp32" if pooled is not None else P.dtname(dtype),
                                     tiles=[(h, t) for h in range(hkv) for t in tiles])
    pos = P.tile_positions(tiles, cfg.tile_q, length)
    err = np.abs(P.rows_of(split, pos) - ref[:, pos])
    assert err.max() <= P.MAX_ABS_TOL and err.mean() <= P.MEAN_ABS_TOL, (err.max(), err.mean())


def test_v_beyond_fp16_range_is_rescaled():
    """bf16 values beyond the fp16 range: the fp16 copy of V is scaled by a power of
    two per KV head and the output scaled back, so scaling V by 2^17 scales the
    output by 2^17 (exactly, up to the few values that the unscaled copy holds
    as fp16 subnormals)."""
    q, k, v = topic_qkv(length=4096, query_heads=8, kv_heads=2, seed=62, dtype=torch.bfloat16)
    cfg = _effective_config(fpv2.FPV2Config(alpha=0.1), 8, 2)
    scale = 128 ** -0.5
    qg, kg, vg = cuda(q, k, v)
    big = vg * (2.0 ** 17)
    assert big.float().abs().max().item() > 65504.0
    pk, pv, lists, _ = fpv2.index_stage(qg, kg, vg, scale=scale, config=cfg, offset=0,
                                        query_length=4096, key_length=4096)
    pkb, pvb, listsb, _ = fpv2.index_stage(qg, kg, big, scale=scale, config=cfg, offset=0,
                                           query_length=4096, key_length=4096)
    assert all(torch.equal(x, y) for x, y in zip(lists, listsb))
    out = fpv2.sparse_attention(qg, kg, vg, pk, pv, *lists, scale=scale, config=cfg)
    outb = fpv2.sparse_attention(qg, kg, big, pkb, pvb, *listsb, scale=scale, config=cfg)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert torch.isfinite(outb).all()
    mx, mean = P.kernel_errors(outb / (2.0 ** 17), P.np32(out))
    assert mx <= 2 ** -7 and mean <= 1e-6, (mx, mean)


def test_launch_count_counts_the_library_kernels():
    """fpv2_launch_count rises by the kernels each call launches: the index stage
    is one pooling launch (K and V) and one selection launch; the attention is the
    fp16 copy of V and its range check, the attention kernel and, when long work
    items split over segments, the combine kernel."""
    q, k, v = topic_qkv(length=4096, query_heads=8, kv_heads=2, seed=63, dtype=torch.bfloat16)
    cfg = _effective_config(fpv2.FPV2Config(alpha=0.1), 8, 2)
    scale = 128 ** -0.5
    qg, kg, vg = cuda(q, k, v)
    c0 = _lib.launch_count()
    pk, pv, lists, _ = fpv2.index_stage(qg, kg, vg, scale=scale, config=cfg, offset=0,
                                        query_length=4096, key_length=4096)
    c1 = _lib.launch_count()
    fpv2.sparse_attention(qg, kg, vg, pk, pv, *lists, scale=scale, config=cfg)
    c2 = _lib.launch_count()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert c1 - c0 == 2
    assert c2 - c1 in (4, 5)
