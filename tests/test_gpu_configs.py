"""Parity at the configurations the benchmark times (64k and 128k layers).

The full layer runs on ``cuda:0`` through the public operators; the CPU oracle
then re-derives a fixed sample of query tiles of every KV head -- the first,
quartile, middle and last tiles (the last two are the dense tail) and a few
seeded random ones -- and the GPU's results for those tiles must match:

* pooled K/V bit-exact (all blocks);
* selection masks bit-exact outside the fp64 1e-5 threshold band;
* full-width lists equal the oracle's compaction of the GPU mask;
* output max-abs <= 2e-2 and mean-abs <= 2e-3 against the float32 math of
  fpv2/reference.py (``fpv2_attention_blockwise``, unrounded), evaluated on
  the GPU's own selection so that an in-band flip cannot cascade.

Two selection semantics are checked. The hook path (fpv2/patch.py:137-146)
pools K/V in the input dtype, so its float32 reference pools in that dtype too;
``pooled_dtype=float32`` is the semantics of fpv2/reference.py:45-51 (float32
pooled keys for the selection and the correction).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import fpv2
from fpv2 import _lib
from fpv2.patch import _effective_config
from oracle import fpv2_oracle as O
from tests import parity as P
from tests.synthetic import topic_qkv

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _layer_check(q, k, v, cfg, *, pooled_dtype=None, tiles=None, check_selection=True):
    """Run the fused index stage + attention on the whole layer and compare the
    sampled tiles with the oracle. Returns (max_abs, mean_abs, flips, sparsity)."""
    hq, L, D = q.shape
    hkv = k.shape[0]
    scale = D ** -0.5
    nt = L // cfg.tile_q
    tiles = P.sample_tiles(nt) if tiles is None else tiles
    qg, kg, vg = q.to(DEV), k.to(DEV), v.to(DEV)
    pk, pv, lists, mask = fpv2.index_stage(qg, kg, vg, scale=scale, config=cfg, offset=0,
                                           query_length=L, key_length=L,
                                           pooled_dtype=pooled_dtype, return_mask=True)
    out = fpv2.sparse_attention(qg, kg, vg, pk, pv, *lists, scale=scale, config=cfg)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0, "a kernel reported a bounded-wait timeout"
    pdt = "fp32" if pooled_dtype == torch.float32 else P.dtname(q.dtype)
    kf, vf = P.np32(k), P.np32(v)
    pk_ref = O.pool_blocks(kf, cfg.block_k, pdt)
    assert np.array_equal(P.np32(pk), pk_ref), "pooled K differs from the oracle"
    assert np.array_equal(P.np32(pv), O.pool_blocks(vf, cfg.block_k, pdt)), "pooled V differs"
    tsel = torch.as_tensor(tiles, device=DEV)
    rows = mask.index_select(1, tsel).cpu().numpy()
    q_np = q.numpy() if q.dtype == torch.float16 else P.np32(q)
    flips = 0
    if check_selection:
        chk = P.check_selection_tiles(q_np, pk_ref, rows, tiles, scale=scale, config=cfg)
        assert chk.ok, f"selection differs from the oracle outside the threshold band: {chk}"
        flips = chk.flips_in_band
    list_rows = [x.index_select(1, tsel).cpu().numpy() for x in lists]
    assert P.check_lists_tiles(rows, list_rows, tiles, config=cfg, offset=0, query_length=L,
                               key_length=L), "lists differ from the compaction of the mask"
    full_mask = np.zeros((hkv, nt, L // cfg.block_k), dtype=bool)
    full_mask[:, tiles] = rows
    ref = O.fpv2_attention_blockwise(q_np, kf, vf, scale=scale, config=cfg, selected=full_mask,
                                     tiles=[(h, t) for h in range(hkv) for t in tiles],
                                     pooled_dtype=pdt)
    pos = P.tile_positions(tiles, cfg.tile_q, L)
    err = np.abs(P.rows_of(out, pos) - ref[:, pos])
    sparsity = 1.0 - float(lists[1].sum().item()) / float(
        hkv * sum((min((t + 1) * cfg.tile_q, L) - 1) // cfg.block_k + 1 for t in range(nt)))
    del qg, kg, vg, pk, pv, lists, mask, out
    torch.cuda.empty_cache()
    return float(err.max()), float(err.mean()), flips, sparsity


# ---------------------------------------------------------------------------
# config 3: Qwen3-4B-shaped layer at 64k (the benchmark's default workload)
# ---------------------------------------------------------------------------


@pytest.fixture(scope="module")
def c3_inputs():
    return topic_qkv(length=65536, query_heads=32, kv_heads=8, head_dim=128, seed=0,
                     dtype=torch.bfloat16)


@pytest.mark.parametrize("corr", [True, False])
def test_c3_layer_hook_semantics(c3_inputs, corr):
    q, k, v = c3_inputs
    cfg = _effective_config(fpv2.FPV2Config(alpha=0.1, mean_correction=corr), 32, 8)
    mx, mean, flips, sparsity = _layer_check(q, k, v, cfg)
    assert sparsity > 0.5, sparsity
    assert mx <= P.MAX_ABS_TOL and mean <= P.MEAN_ABS_TOL, (mx, mean, flips)


def test_c3_layer_reference_semantics(c3_inputs):
    """float32 pooled keys and values (fpv2/reference.py:45-51) through the selection
    and the correction, against the reference's float32 math."""
    q, k, v = c3_inputs
    cfg = _effective_config(fpv2.FPV2Config(alpha=0.1), 32, 8)
    mx, mean, flips, _ = _layer_check(q, k, v, cfg, pooled_dtype=torch.float32)
    assert mx <= P.MAX_ABS_TOL and mean <= P.MEAN_ABS_TOL, (mx, mean, flips)


# ---------------------------------------------------------------------------
# config 5: GQA 8 (16 positions per selection tile) at 128k in fp16
# ---------------------------------------------------------------------------


@pytest.fixture(scope="module")
def c5_inputs():
    return topic_qkv(length=131072, query_heads=64, kv_heads=8, head_dim=128, seed=0,
                     dtype=torch.float16)


@pytest.mark.parametrize("alpha", [0.05, 0.1, 0.2])
def test_c5_layer_hook_semantics(c5_inputs, alpha):
    q, k, v = c5_inputs
    cfg = _effective_config(fpv2.FPV2Config(alpha=alpha, score_chunk_tiles=8), 64, 8)
    assert cfg.tile_q == 16
    mx, mean, flips, sparsity = _layer_check(q, k, v, cfg)
    assert sparsity > 0.5, sparsity
    assert mx <= P.MAX_ABS_TOL and mean <= P.MEAN_ABS_TOL, (mx, mean, flips)


def test_c5_layer_reference_semantics(c5_inputs):
    q, k, v = c5_inputs
    cfg = _effective_config(fpv2.FPV2Config(alpha=0.1, score_chunk_tiles=8), 64, 8)
    mx, mean, flips, _ = _layer_check(q, k, v, cfg, pooled_dtype=torch.float32)
    assert mx <= P.MAX_ABS_TOL and mean <= P.MEAN_ABS_TOL, (mx, mean, flips)
