"""The bench's parity block on the CPU: oracle lists pass, a flipped block far
from the alpha threshold fails, a flipped block at the threshold is an
in-band flip (north_star: lists bit-exact wherever no block energy lies
within 1e-5 relative of the threshold, flips reported otherwise).

The "GPU" lists here are the oracle's own, with the planted changes.
"""

from __future__ import annotations

from dataclasses import replace

import numpy as np
import torch

import bench
import fpv2
from fpv2.patch import _effective_config
from oracle import fpv2_oracle as O
from tests.synthetic import topic_qkv

L, HQ, HKV, D = 2048, 8, 2, 128
G = HQ // HKV
TILES = 4


def _inputs():
    q, k, v = topic_qkv(length=L, query_heads=HQ, kv_heads=HKV, head_dim=D, seed=7,
                        dtype=torch.bfloat16)
    return q, k, v


def _as_gpu(smp, cfg):
    """Full-layout lists and output holding the sample's oracle results."""
    nt, nb = L // cfg.tile_q, L // cfg.block_k
    h, t0, t1 = smp["head"], smp["tiles"][0], smp["tiles"][-1] + 1
    lists = [torch.zeros((HKV, nt, nb), dtype=torch.int32), torch.zeros((HKV, nt), dtype=torch.int32),
             torch.zeros((HKV, nt, nb), dtype=torch.int32), torch.zeros((HKV, nt), dtype=torch.int32)]
    for x, ref in zip(lists, smp["lists"]):
        x[h:h + 1, t0:t1] = torch.from_numpy(ref.astype(np.int32))
    out = torch.zeros((HQ, L, D), dtype=torch.float32)
    out[h * G:(h + 1) * G, t0 * cfg.tile_q:t1 * cfg.tile_q] = torch.from_numpy(smp["out"])
    return lists, out


def _toggle(lists, smp, cfg, t: int, b: int):
    """Flip block b of tile t in the selection and re-compact that tile."""
    h = smp["head"]
    ids, cnt = lists[0][h, t].numpy(), int(lists[1][h, t])
    mask = np.zeros(L // cfg.block_k, dtype=bool)
    mask[ids[:cnt]] = True
    mask[b] = not mask[b]
    nt = L // cfg.tile_q
    c = replace(O.as_config(cfg), last_n_blocks=1 if t >= nt - cfg.last_n_blocks else 0)
    ref = O.compact_block_indices(mask[None, None], config=c, offset=t * cfg.tile_q,
                                  query_length=cfg.tile_q, key_length=L)
    for x, r in zip(lists, ref):
        x[h:h + 1, t:t + 1] = torch.from_numpy(r.astype(np.int32))


def _energies64(q, smp, cfg, t: int):
    rows = q[:G, t * cfg.tile_q:(t + 1) * cfg.tile_q].float().numpy()
    c = replace(O.as_config(cfg), score_chunk_tiles=None, last_n_blocks=0)
    r = O.block_scores_and_select(rows, smp["pk"], scale=D ** -0.5, config=c, offset=t * cfg.tile_q,
                                  precision="fp64")
    return r.energies[0, 0]


def _sample(q, k, v, cfg):
    *_, smp = bench.cpu_sample(q, k, v, cfg, tiles_per_step=TILES, head=0, want_outputs=True)
    return smp


def _free_block(cfg, t: int, e64: np.ndarray, far: bool) -> int:
    """A block that no forcing rule keeps in tile t (not sink, not local, fully
    visible), the one farthest from or nearest below the largest energy."""
    tile_first = t * cfg.tile_q
    cand = [b for b in range(len(e64))
            if b * cfg.block_k >= cfg.sink_tokens
            and (b + 1) * cfg.block_k <= tile_first - cfg.window_tokens
            and e64[b] < e64.max()]
    assert cand
    return min(cand, key=lambda b: e64[b]) if far else max(cand, key=lambda b: e64[b])


def test_oracle_lists_pass_and_far_flip_fails():
    q, k, v = _inputs()
    cfg = _effective_config(fpv2.FPV2Config(alpha=0.1), HQ, HKV)
    smp = _sample(q, k, v, cfg)
    lists, out = _as_gpu(smp, cfg)
    clean = bench.sample_parity([smp], lists, out, G, q, cfg)
    assert clean["ok"] and clean["tiles_with_list_mismatch"] == 0, clean

    t = smp["tiles"][0]                       # not a dense-tail tile
    b = _free_block(cfg, t, _energies64(q, smp, cfg, t), far=True)
    _toggle(lists, smp, cfg, t, b)
    bad = bench.sample_parity([smp], lists, out, G, q, cfg)
    assert bad["tiles_with_list_mismatch"] == 1 and bad["tiles_out_of_band"] == 1, bad
    assert not bad["ok"], bad


def test_flip_at_the_threshold_is_in_band():
    q, k, v = _inputs()
    cfg0 = _effective_config(fpv2.FPV2Config(alpha=0.1), HQ, HKV)
    nt = L // cfg0.tile_q
    t = nt - TILES                            # first tile of the sample, not in the dense tail
    smp0 = _sample(q, k, v, cfg0)
    e64 = _energies64(q, smp0, cfg0, t)
    b = _free_block(cfg0, t, e64, far=False)
    cfg = replace(cfg0, alpha=float(e64[b] / e64.max()))   # block b sits on the threshold
    smp = _sample(q, k, v, cfg)
    lists, out = _as_gpu(smp, cfg)
    _toggle(lists, smp, cfg, t, b)
    res = bench.sample_parity([smp], lists, out, G, q, cfg)
    assert res["tiles_with_list_mismatch"] == 1 and res["tiles_with_in_band_flip"] == 1, res
    assert res["ok"], res
