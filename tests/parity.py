"""Comparison helpers shared by the GPU parity tests, ``smoke()`` and the benchmark.

All checks compare the CUDA path with the CPU oracle (oracle/fpv2_oracle.py) on
identical inputs:

* pooled K/V: bit-exact;
* selection masks: bit-exact except blocks whose float64 energy lies within a
  relative 1e-5 of the alpha threshold (reported as flips);
* lists: bit-exact compaction of the mask (full padded width) and, when no
  block flipped, bit-exact against the oracle's lists;
* attention output: max-abs <= 2e-2 and mean-abs <= 2e-3 against the float32
  reference math of fpv2/reference.py.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import numpy as np
import torch

from oracle import fpv2_oracle as O

MAX_ABS_TOL = 2e-2
MEAN_ABS_TOL = 2e-3
# GPU output vs the list-driven oracle on the same lists (both rounded to the
# compute dtype): the residual is bf16 rounding of P and of the output, so the
# max is taken on |a - b| / max(1, |b|) (a one-ulp flip at |x| in [4, 8) is 2^-5).
KERNEL_MAX_ABS_TOL = 2e-2
KERNEL_MEAN_ABS_TOL = 5e-4
FLIP_REL_BAND = 1e-5

_DT = {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}


def np32(t: torch.Tensor) -> np.ndarray:
    return t.detach().to("cpu", torch.float32).numpy()


def dtname(dtype: torch.dtype) -> str:
    return _DT[dtype]


@dataclass
class SelectCheck:
    mismatches: int
    flips_in_band: int
    out_of_band: int
    band_blocks: int

    @property
    def ok(self) -> bool:
        return self.out_of_band == 0


def check_selection(q: torch.Tensor, pooled_k_np: np.ndarray, gpu_mask: np.ndarray, *, scale: float,
                    config, offset: int = 0, query_length: int | None = None) -> SelectCheck:
    """GPU mask vs the oracle on the same pooled keys, flips allowed only in the fp64 band."""
    c = O.as_config(config)
    chunk = replace(c, score_chunk_tiles=c.score_chunk_tiles or max(1, 4096 // c.tile_q))
    qf = np32(q)
    r32 = O.block_scores_and_select(qf, pooled_k_np, scale=scale, config=chunk, offset=offset,
                                    query_length=query_length)
    r64 = O.block_scores_and_select(qf, pooled_k_np, scale=scale, config=chunk, offset=offset,
                                    query_length=query_length, precision="fp64")
    band = O.threshold_band(r64, FLIP_REL_BAND)
    diff = gpu_mask != r32.selected
    return SelectCheck(
        mismatches=int(diff.sum()),
        flips_in_band=int((diff & band).sum()),
        out_of_band=int((diff & ~band).sum()),
        band_blocks=int(band.sum()),
    )


def check_lists_of_mask(mask: np.ndarray, lists, *, config, offset: int, query_length: int,
                        key_length: int) -> bool:
    """GPU lists equal the oracle's compaction of the same mask, full padded width."""
    ref = O.compact_block_indices(mask.astype(bool), config=config, offset=offset,
                                  query_length=query_length, key_length=key_length)
    return all(np.array_equal(a.cpu().numpy(), b) for a, b in zip(lists, ref))


def kernel_errors(actual: torch.Tensor, expected: np.ndarray):
    """(max |a-b| / max(1, |b|), mean |a-b|) against the list-driven oracle."""
    a = np32(actual)
    err = np.abs(a - expected)
    return float((err / np.maximum(1.0, np.abs(expected))).max()), float(err.mean())


def reference_rel_max(actual: torch.Tensor, expected: np.ndarray) -> float:
    """max |a - b| / max |b|: the criterion of the reference's own kernel tests
    (tests/test_kernel.py:221-224 of the reference)."""
    a = np32(actual)
    return float(np.abs(a - expected).max() / max(float(np.abs(expected).max()), 1e-8))


def attention_errors(actual: torch.Tensor, expected: np.ndarray, rows: int | None = None):
    a = np32(actual)
    if rows is not None:
        a = a[:, :rows]
        expected = expected[:, :rows]
    err = np.abs(a - expected)
    return float(err.max()), float(err.mean())


# ---------------------------------------------------------------------------
# sampled checks of full-size layers (64k / 128k): a fixed set of query tiles
# ---------------------------------------------------------------------------


def sample_tiles(num_tiles: int, *, extra: int = 4, seed: int = 0) -> list[int]:
    """First, quartile, middle and last tiles (the last two are the dense tail)
    plus ``extra`` seeded random tiles."""
    base = {0, 1, num_tiles // 4, num_tiles // 2, (3 * num_tiles) // 4,
            num_tiles - 3, num_tiles - 2, num_tiles - 1}
    rng = np.random.default_rng(seed)
    base |= {int(x) for x in rng.integers(0, num_tiles, size=extra)}
    return sorted(t for t in base if 0 <= t < num_tiles)


def tile_positions(tiles, tile_q: int, valid_length: int) -> np.ndarray:
    pos = np.concatenate([np.arange(t * tile_q, (t + 1) * tile_q) for t in tiles])
    return pos[pos < valid_length]


def check_selection_tiles(q_np: np.ndarray, pooled_k_np: np.ndarray, gpu_rows: np.ndarray, tiles,
                          *, scale: float, config, offset: int = 0,
                          query_length: int | None = None) -> SelectCheck:
    """GPU mask rows ``[Hkv, len(tiles), Nb]`` vs the oracle evaluated on those tiles
    only, flips allowed only in the fp64 band."""
    c = O.as_config(config)
    kw = dict(scale=scale, config=c, offset=offset, query_length=query_length, only_tiles=tiles)
    r32 = O.block_scores_and_select(q_np, pooled_k_np, **kw)
    r64 = O.block_scores_and_select(q_np, pooled_k_np, precision="fp64", **kw)
    band = O.threshold_band(r64, FLIP_REL_BAND)
    diff = gpu_rows != r32.selected
    return SelectCheck(
        mismatches=int(diff.sum()),
        flips_in_band=int((diff & band).sum()),
        out_of_band=int((diff & ~band).sum()),
        band_blocks=int(band.sum()),
    )


def check_lists_tiles(gpu_rows: np.ndarray, list_rows, tiles, *, config, offset: int,
                      query_length: int, key_length: int) -> bool:
    """Each sampled tile's full-width GPU lists equal the oracle's compaction of the
    GPU mask row (a one-tile compaction whose offset is the tile's first position)."""
    c = O.as_config(config)
    for i, t in enumerate(tiles):
        first = t * c.tile_q
        ql = min(c.tile_q, query_length - first)
        if ql <= 0:
            continue
        ref = O.compact_block_indices(gpu_rows[:, i:i + 1], config=c, offset=offset + first,
                                      query_length=ql, key_length=key_length)
        for got, exp in zip(list_rows, ref):
            if not np.array_equal(got[:, i:i + 1], exp):
                return False
    return True


def rows_of(x: torch.Tensor, positions: np.ndarray) -> np.ndarray:
    """Query rows ``positions`` of a ``[H, L, D]`` tensor as float32 NumPy."""
    idx = torch.as_tensor(positions, device=x.device)
    return x.index_select(1, idx).to("cpu", torch.float32).numpy()
