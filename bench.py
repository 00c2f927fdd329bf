"""FPV2 prefill-layer benchmark on B200 (one process per GPU).

A *step* is one FlashPrefill V2 attention layer at 64k tokens (
Qwen3-4B-shaped, Hq=32, Hkv=8, head_dim 128, bf16, alpha=0.1, correction on,
topic-block synthetic inputs): the fused index stage (pool K/V, score, select,
compact) followed by the tcgen05 sparse attention, through the public
``fpv2.fpv2_sdpa`` call with inputs resident in HBM. With N > 1 GPUs the layer
is split head-parallel (Hkv/N KV heads and their query heads per GPU) and the
attention kernel re-assembles the output on every rank with NVLink multicast
stores (one NCCL all-gather where the GPUs offer no multicast); total work is
fixed (strong scaling) and ``value`` is the whole layer's retained TFLOP/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...

``--impl reference`` times the reference's algorithm on the host cores: the
CPU restatement in oracle/fpv2_oracle.py (the reference itself needs MLX on an
Apple GPU), on a bounded sample of the same layer, in the same unit.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from dataclasses import replace
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "flashprefillv2-mlx_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "sparse prefill-attn ms/layer & TFLOP/s (retained) at 64k; % bf16 peak; selection GB/s"
PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# DRAM bytes per launch of the dominant kernels (dram__bytes_read.sum +
# dram__bytes_write.sum) from one earlier ncu capture of the full-size
# single-GPU workload: a recorded constant, not measured by this run.
NCU_TRAFFIC_BYTES = {
    "c3": {"attention": 2890.32e6 + 501.88e6, "index_stage": 268.45e6 + 1.33e6 + 537.55e6 + 57.75e6},
}

CONFIGS = {
    # name: (length, Hq, Hkv, head_dim, dtype, alpha)
    "c3": (65536, 32, 8, 128, torch.bfloat16, 0.1),
    "c2": (16384, 32, 8, 128, torch.bfloat16, 0.1),
    "c5": (131072, 64, 8, 128, torch.float16, 0.1),
}


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------


def load_peaks() -> tuple[dict, str]:
    if PEAKS_FILE.exists():
        return json.loads(PEAKS_FILE.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def retained_attention_flops(sel_ids, sel_counts, pr_counts, *, G, tile_q, block_k, offset,
                             valid_lq, valid_lk, D, corr) -> float:
    """4*D * sum over (kv head, tile) of causal (q, k) pairs of the selected blocks
    (all G heads) plus, with correction, G * (valid rows) * pruned entries."""
    ids = sel_ids.cpu().numpy()
    cnt = sel_counts.cpu().numpy()
    pcnt = pr_counts.cpu().numpy()
    hkv, nt, nb = ids.shape
    total = 0.0
    for h in range(hkv):
        for t in range(nt):
            row0 = t * tile_q
            rows = np.arange(row0, min(row0 + tile_q, valid_lq))
            if rows.size == 0:
                continue
            pos = offset + rows
            blocks = ids[h, t, : cnt[h, t]]
            starts = blocks.astype(np.int64) * block_k
            ends = np.minimum(starts + block_k, valid_lk)
            # causal keys of each row inside each block
            pairs = np.clip(np.minimum(pos[None, :] + 1, ends[:, None]) - starts[:, None], 0, None)
            total += float(pairs.sum()) * G
            if corr:
                total += float(rows.size) * G * float(pcnt[h, t])
    return 4.0 * D * total


def attention_kernel_name(dtype, Hq: int, Hkv: int, D: int, block_k: int, tile_q: int,
                          num_blocks: int) -> str:
    """The attention kernel the library picks for this shape (fpv2_fast_path_mask)."""
    from fpv2 import _lib

    m = _lib.fast_path_mask(dtype, Hq, Hkv, D, block_k, tile_q, num_blocks)
    if not m & 2:
        return "attn_generic_kernel"
    if D == 256:
        return "attn_wide_kernel"
    return "attn_pair_kernel" if m & 4 else "attn_tc_kernel"


def index_stage_bytes(Hq, Hkv, L, D, Nt, Nb, esize=2) -> int:
    """Algorithmic HBM bytes of the fused index stage: read Q, K, V; write pooled K/V,
    two full-width int32 lists and two count arrays."""
    return (Hq * L * D * esize + 2 * Hkv * L * D * esize + 2 * Hkv * Nb * D * esize
            + 2 * Hkv * Nt * Nb * 4 + 2 * Hkv * Nt * 4)


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="fpv2_clocks_", suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self, load_fraction: float = 0.5) -> dict:
        if self.proc is None or self.path is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, flags in rows for i, f in enumerate(flags)
                          if f.lower() == "active"})
        sm = [r[0] for r in rows]
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU leg: the reference algorithm (oracle port) on a bounded sample
# ---------------------------------------------------------------------------


def cpu_sample(q, k, v, cfg, *, tiles_per_step: int, head: int = 0, seed_tile: int | None = None,
               want_outputs: bool = False):
    """Run the oracle's index stage + list-driven attention for ``tiles_per_step``
    tiles of KV head ``head`` (latest tiles, the heaviest) and return
    (seconds, retained FLOPs, description) -- plus, with ``want_outputs``, the
    oracle's lists and float32 output of those tiles for the parity check."""
    from oracle import fpv2_oracle as O

    hq, L, D = q.shape
    hkv = k.shape[0]
    G = hq // hkv
    nt = L // cfg.tile_q
    last = nt if seed_tile is None else seed_tile
    tiles = list(range(max(0, last - tiles_per_step), last))
    qh = q[head * G:(head + 1) * G].float().numpy()
    kh = k[head:head + 1].float().numpy()
    vh = v[head:head + 1].float().numpy()
    pdt = "fp16" if q.dtype == torch.float16 else "bf16"
    t0 = time.perf_counter()
    pk = O.pool_blocks(kh, cfg.block_k, pdt)
    pv = O.pool_blocks(vh, cfg.block_k, pdt)
    # selection for the sampled tiles only: slice their rows (offset keeps positions)
    row0 = tiles[0] * cfg.tile_q
    rows = slice(row0, (tiles[-1] + 1) * cfg.tile_q)
    c = replace(O.as_config(cfg), score_chunk_tiles=8,
                last_n_blocks=max(0, cfg.last_n_blocks - (nt - 1 - tiles[-1])))
    sel = O.block_scores_and_select(qh[:, rows], pk, scale=D ** -0.5, config=c, offset=row0).selected
    lists = O.compact_block_indices(sel, config=c, offset=row0, query_length=qh[:, rows].shape[1],
                                    key_length=L)
    out = O.sparse_attention(qh[:, rows], kh, vh, pk, pv, *lists, scale=D ** -0.5, config=c,
                             offset=row0, dtype=pdt, out_dtype="fp32")
    dt = time.perf_counter() - t0
    assert np.isfinite(out).all()
    flops = retained_attention_flops(torch.from_numpy(lists[0]), torch.from_numpy(lists[1]),
                                     torch.from_numpy(lists[3]), G=G, tile_q=c.tile_q,
                                     block_k=c.block_k, offset=row0,
                                     valid_lq=qh[:, rows].shape[1], valid_lk=L, D=D,
                                     corr=c.mean_correction)
    desc = (f"KV head {head}, tiles {tiles[0]}..{tiles[-1]} ({len(tiles)} of {nt} per head, "
            f"{len(tiles) * G * cfg.tile_q} query rows): oracle pool + select + compact + "
            f"list-driven attention, numpy float32")
    if not want_outputs:
        return dt, flops, desc
    return dt, flops, desc, dict(head=head, row0=row0, tiles=tiles, lists=lists, out=out, pk=pk,
                                 scale=D ** -0.5)


def _tile_flip(q, smp, t: int, gpu_tile, cfg, nt: int, G: int) -> bool:
    """True when tile ``t``'s GPU lists differ from the oracle's only by blocks whose
    float64 energy lies within 1e-5 relative of the alpha threshold, and are the
    exact compaction of the GPU's own selection (north_star's allowed flips)."""
    from oracle import fpv2_oracle as O

    h, tq = smp["head"], cfg.tile_q
    rows = q[h * G:(h + 1) * G, t * tq:(t + 1) * tq].float().numpy()
    c = replace(O.as_config(cfg), score_chunk_tiles=None,
                last_n_blocks=1 if t >= nt - cfg.last_n_blocks else 0)
    kw = dict(scale=smp["scale"], config=c, offset=t * tq)
    r32 = O.block_scores_and_select(rows, smp["pk"], **kw)
    r64 = O.block_scores_and_select(rows, smp["pk"], precision="fp64", **kw)
    band = O.threshold_band(r64)[0, 0]
    ids, counts = gpu_tile[0][0, 0], int(gpu_tile[1][0, 0])
    gpu_mask = np.zeros_like(r32.selected[0, 0])
    gpu_mask[ids[:counts]] = True
    diff = gpu_mask != r32.selected[0, 0]
    if not diff.any() or (diff & ~band).any():
        return False
    ref = O.compact_block_indices(gpu_mask[None, None], config=c, offset=t * tq,
                                  query_length=tq, key_length=q.shape[1])
    return all(np.array_equal(a, b) for a, b in zip(gpu_tile, ref))


def sample_parity(samples, lists_gpu, out_gpu, G: int, q, cfg) -> dict:
    """GPU lists and output of the CPU sample's tiles vs the oracle's: full-width
    lists bit-exact per tile except threshold flips (blocks whose float64 energy
    lies within 1e-5 relative of alpha * max, reported as in-band flips), and
    the output within max-abs 2e-2 / mean-abs 2e-3 of the float32 list-driven
    math (outside the timed region)."""
    tile_q = cfg.tile_q
    nt = q.shape[1] // tile_q
    tiles_total = mismatched = in_band = 0
    mx, sum_abs, n = 0.0, 0.0, 0
    for smp in samples:
        h, tiles = smp["head"], smp["tiles"]
        t0, t1 = tiles[0], tiles[-1] + 1
        gpu_lists = [x[h:h + 1, t0:t1].cpu().numpy() for x in lists_gpu]
        equal = np.ones(t1 - t0, dtype=bool)
        for got, exp in zip(gpu_lists, smp["lists"]):
            same = (got == exp).reshape(t1 - t0, -1).all(axis=1)
            equal &= same
        tiles_total += t1 - t0
        for i in np.nonzero(~equal)[0]:
            mismatched += 1
            tile = [x[:, i:i + 1] for x in gpu_lists]
            in_band += int(_tile_flip(q, smp, t0 + int(i), tile, cfg, nt, G))
        r0, r1 = t0 * tile_q, t1 * tile_q
        o = out_gpu[h * G:(h + 1) * G, r0:r1].to("cpu", torch.float32).numpy()
        err = np.abs(o - smp["out"][:, :r1 - r0])
        mx = max(mx, float(err.max()))
        sum_abs += float(err.sum())
        n += err.size
    mean = sum_abs / max(n, 1)
    return {"tiles_checked": tiles_total, "tiles_with_list_mismatch": mismatched,
            "tiles_with_in_band_flip": in_band, "tiles_out_of_band": mismatched - in_band,
            "max_abs": round(mx, 6), "mean_abs": round(mean, 7),
            "ok": bool(mismatched == in_band and mx <= 2e-2 and mean <= 2e-3),
            "criterion": "full-width lists bit-exact per tile except in-band threshold flips "
                         "(float64 energy within 1e-5 relative of alpha * max); output max-abs "
                         "<= 2e-2 and mean-abs <= 2e-3 against the oracle's float32 "
                         "list-driven math on the same tiles"}


# ---------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS) + ["c4"], default="c3",
                    help="c4: chunked 64k prefill through a random-init Qwen3-4B-architecture model")
    ap.add_argument("--c4-layers", type=int, default=36, help="decoder layers of the c4 model")
    ap.add_argument("--c4-qk-gain", type=float, default=1.0,
                    help="c4: value of the per-head q/k RMSNorm weights (random init leaves them "
                         "at 1, logits of std ~1, so alpha keeps every block; a gain g scales the "
                         "logits by g^2, giving the peaked attention a trained model has)")
    ap.add_argument("--no-corr", action="store_true", help="mean correction off")
    ap.add_argument("--alpha", type=float, default=None)
    ap.add_argument("--tile-q", type=int, default=None,
                    help="query positions per selection tile (default: 128 packed rows = 128/G positions)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-tiles", type=int, default=2048,
                    help="latest tiles of a KV head per CPU sample (the reference arm uses 1/8)")
    ap.add_argument("--cpu-heads", type=int, default=3, help="KV heads in the CPU baseline sample")
    return ap.parse_args(argv)


def dist_setup(n: int):
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return rank, world, local


# ---------------------------------------------------------------------------
# c4: chunked prefill through a random-init Qwen3-4B-architecture model
# ---------------------------------------------------------------------------


def _qwen3_weights(dev, layers, seed=0, qk_gain=1.0):
    """Random bf16 weights ~ N(0, 0.02) of the Qwen3-4B architecture (hidden 2560,
    32 Q / 8 KV heads of 128, SwiGLU 9728, RMSNorm with per-head q/k norms whose
    weights are ``qk_gain``)."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)

    def w(*shape):
        return (torch.randn(*shape, generator=g, device=dev) * 0.02).to(torch.bfloat16)

    H, I, HQ, HKV, D, V = 2560, 9728, 32, 8, 128, 151936
    ones = lambda n: torch.ones(n, device=dev, dtype=torch.bfloat16)  # noqa: E731
    blocks = [dict(ln1=ones(H), wq=w(HQ * D, H), wk=w(HKV * D, H), wv=w(HKV * D, H),
                   qn=ones(D) * qk_gain, kn=ones(D) * qk_gain, wo=w(H, HQ * D), ln2=ones(H),
                   wg=w(I, H), wu=w(I, H), wd=w(H, I))
              for _ in range(layers)]
    return dict(embed=w(V, H), blocks=blocks, norm=ones(H), lm_head=w(V, H))


def _rope(x, pos, theta=1e6):
    d = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, device=x.device, dtype=torch.float32) / d))
    ang = pos[:, None].float() * inv[None]
    cos, sin = ang.cos(), ang.sin()
    x1, x2 = x[..., : d // 2].float(), x[..., d // 2:].float()
    c, s_ = cos[:, None, :], sin[:, None, :]
    return torch.cat([x1 * c - x2 * s_, x2 * c + x1 * s_], dim=-1).to(x.dtype)


def _qwen3_prefill(weights, ids, chunk, dense_expand_kv):
    """Chunked prefill against a growing KV cache; returns last-token logits.

    Attention is a plain ``torch.nn.functional.scaled_dot_product_attention``
    call: ``is_causal=True`` for the first chunk and a bottom-right
    ``causal_lower_right`` bias once the cache is longer than the chunk (the
    form the FPV2 hook claims). The stock dense path cannot combine that bias
    with ``enable_gqa``, so the dense baseline repeats K/V heads instead."""
    import torch.nn.functional as F
    from torch.nn.attention.bias import causal_lower_right

    dev = ids.device
    L = ids.numel()
    HQ, HKV, D = 32, 8, 128
    layers = len(weights["blocks"])
    kc = [torch.empty((HKV, L, D), device=dev, dtype=torch.bfloat16) for _ in range(layers)]
    vc = [torch.empty((HKV, L, D), device=dev, dtype=torch.bfloat16) for _ in range(layers)]
    x = None
    for off in range(0, L, chunk):
        T = min(chunk, L - off)
        pos = torch.arange(off, off + T, device=dev)
        x = weights["embed"][ids[off:off + T]]
        for li, b in enumerate(weights["blocks"]):
            h = F.rms_norm(x, (x.shape[-1],), b["ln1"], eps=1e-6)
            q = F.rms_norm((h @ b["wq"].T).view(T, HQ, D), (D,), b["qn"], eps=1e-6)
            k = F.rms_norm((h @ b["wk"].T).view(T, HKV, D), (D,), b["kn"], eps=1e-6)
            v = (h @ b["wv"].T).view(T, HKV, D)
            q, k = _rope(q, pos), _rope(k, pos)
            kc[li][:, off:off + T] = k.transpose(0, 1)
            vc[li][:, off:off + T] = v.transpose(0, 1)
            q4 = q.transpose(0, 1)[None]
            k4, v4 = kc[li][None, :, :off + T], vc[li][None, :, :off + T]
            if off == 0:
                o = F.scaled_dot_product_attention(q4, k4, v4, is_causal=True, enable_gqa=True,
                                                   scale=D ** -0.5)
            elif dense_expand_kv:
                o = F.scaled_dot_product_attention(
                    q4, k4.repeat_interleave(HQ // HKV, dim=1), v4.repeat_interleave(HQ // HKV, dim=1),
                    attn_mask=causal_lower_right(T, off + T), scale=D ** -0.5)
            else:
                o = F.scaled_dot_product_attention(q4, k4, v4, attn_mask=causal_lower_right(T, off + T),
                                                   enable_gqa=True, scale=D ** -0.5)
            x = x + o[0].transpose(0, 1).reshape(T, HQ * D) @ b["wo"].T
            h = F.rms_norm(x, (x.shape[-1],), b["ln2"], eps=1e-6)
            x = x + (F.silu(h @ b["wg"].T) * (h @ b["wu"].T)) @ b["wd"].T
    last = F.rms_norm(x[-1:], (x.shape[-1],), weights["norm"], eps=1e-6)
    return (last @ weights["lm_head"].T).float()


def c4_prefill(args) -> int:
    """a 65536-token prompt in 2048-token chunks, total_tokens
    known (dense tail only at the last chunk), FPV2 hook vs the stock dense path."""
    import fpv2

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L, chunk = 65536, 2048
    weights = _qwen3_weights(dev, args.c4_layers, qk_gain=args.c4_qk_gain)
    g = torch.Generator(device=dev)
    g.manual_seed(1)
    ids = torch.randint(0, 151936, (L,), device=dev, generator=g)
    times = {}
    logits = {}
    with torch.no_grad():
        for mode in ("fpv2", "dense"):
            if mode == "fpv2":
                fpv2.enable(fpv2.FPV2Config(alpha=0.1), min_tokens=4096, collect_stats=True,
                            total_tokens=L)
            # warm-up on a short prompt (kernels, cuBLAS handles)
            _qwen3_prefill(weights, ids[:2 * chunk], chunk, mode == "dense")
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(0) as clocks:
                e0.record()
                logits[mode] = _qwen3_prefill(weights, ids, chunk, mode == "dense")
                e1.record()
                torch.cuda.synchronize()
            times[mode] = e0.elapsed_time(e1) / 1000.0
            if mode == "fpv2":
                sparsity = fpv2.block_sparsity()
                fpv2.disable()
    a, b = logits["fpv2"], logits["dense"]
    cos = float(torch.nn.functional.cosine_similarity(a, b).item())
    line = {
        "metric": "chunked 64k prefill tokens/s through a Qwen3-4B-architecture model (FPV2 hook)",
        "value": round(L / times["fpv2"], 1), "unit": "tokens/s", "n_gpus": 1, "steps": 1,
        "warmup": 1, "ms_per_step": round(1000 * times["fpv2"], 2), "higher_is_better": True,
        "scaling": "none", "vs_baseline": None, "dtype": "bf16",
        "data": "random-init weights ~ N(0, 0.02), token ids uniform over the 151936 vocab (seed 1)",
        "config": {"workload": f"c4: {L} tokens in {chunk}-token chunks, total_tokens={L}, "
                               f"{args.c4_layers} layers, alpha=0.1, min_tokens=4096",
                   "qk_norm_gain": args.c4_qk_gain,
                   "dense_prefill_s": round(times["dense"], 3),
                   "fpv2_prefill_s": round(times["fpv2"], 3),
                   "speedup_vs_dense": round(times["dense"] / times["fpv2"], 3),
                   "block_sparsity": round(sparsity, 4),
                   "last_token_logit_cosine_vs_dense": round(cos, 5)},
        "clocks": clocks.summary(),
    }
    emit_json(line)
    return 0


_JSON_FD: int | None = None


def emit_json(line: dict) -> None:
    """Write the result line to the real stdout (everything else the process or its
    libraries print goes to stderr, so stdout carries exactly one JSON line)."""
    data = (json.dumps(line) + "\n").encode()
    if _JSON_FD is None:
        sys.stdout.write(data.decode())
        sys.stdout.flush()
    else:
        os.write(_JSON_FD, data)


def main(argv=None) -> int:
    global _JSON_FD
    args = parse_args(argv)
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)   # library banners (NCCL, symmetric memory) go to stderr
    if args.config == "c4":
        return c4_prefill(args)
    length, Hq, Hkv, D, dtype, alpha = CONFIGS[args.config]
    if args.alpha is not None:
        alpha = args.alpha
    import fpv2
    from fpv2.patch import _effective_config
    from tests.synthetic import topic_qkv

    base_cfg = fpv2.FPV2Config(alpha=alpha, mean_correction=not args.no_corr)
    if args.tile_q is not None:
        base_cfg = replace(base_cfg, tile_q=args.tile_q)
    cfg = _effective_config(base_cfg, Hq, Hkv)
    scale = D ** -0.5

    if args.impl == "reference":
        return reference_arm(args, length, Hq, Hkv, D, dtype, cfg)

    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if Hkv % world:
        raise SystemExit("KV heads must divide evenly over the GPUs")
    hkv_r = Hkv // world
    G = Hq // Hkv
    q, k, v = topic_qkv(length=length, query_heads=Hq, kv_heads=Hkv, head_dim=D, seed=0, dtype=dtype)
    qs = q[rank * hkv_r * G:(rank + 1) * hkv_r * G].contiguous()
    ks = k[rank * hkv_r:(rank + 1) * hkv_r].contiguous()
    vs = v[rank * hkv_r:(rank + 1) * hkv_r].contiguous()
    qd, kd, vd = qs.to(dev)[None], ks.to(dev)[None], vs.to(dev)[None]
    out_full = torch.empty((world, hkv_r * G, length, D), dtype=dtype, device=dev) if world > 1 else None
    # Multi-GPU reassembly: fused into the attention kernel (multicast stores into a
    # symmetric-memory buffer) where the GPUs support NVLink multicast, else NCCL.
    mc = None
    if world > 1 and os.environ.get("FPV2_NO_MULTICAST", "0") != "1":
        import torch.distributed as dist
        from fpv2.shard import _multicast_buffer

        good = 1
        try:
            mc = _multicast_buffer((world * hkv_r * G, length, D), dtype, dev, None)
        except Exception as exc:  # no symmetric memory / multicast on this node
            print(f"multicast reassembly unavailable ({exc}); using NCCL all-gather",
                  file=sys.stderr)
            mc, good = None, 0
        agree = torch.tensor([good], dtype=torch.int32, device=dev)
        dist.all_reduce(agree, op=dist.ReduceOp.MIN)   # every rank takes the same path
        if int(agree.item()) == 0:
            mc = None
    mc_args = (mc[2], rank * hkv_r * G, world * hkv_r * G) if mc else None

    def step():
        if mc is not None:
            from fpv2.shard import head_parallel_sdpa

            return head_parallel_sdpa(qd, kd, vd, scale=scale, config=base_cfg, fused=True,
                                      copy=False)
        out = fpv2.fpv2_sdpa(qd, kd, vd, scale=scale, config=base_cfg)
        if world > 1:
            import torch.distributed as dist

            dist.all_gather_into_tensor(out_full.view(-1), out[0].contiguous().view(-1))
        return out

    # Lists once, for the retained-FLOP count of this rank's shard.
    pk, pv, lists, _ = fpv2.index_stage(qd[0], kd[0], vd[0], scale=scale, config=cfg, offset=0,
                                        query_length=length, key_length=length)
    flops_rank = retained_attention_flops(lists[0], lists[1], lists[3], G=G, tile_q=cfg.tile_q,
                                          block_k=cfg.block_k, offset=0, valid_lq=length,
                                          valid_lk=length, D=D, corr=cfg.mean_correction)
    sel_total = int(lists[1].sum().item())
    nt, nb = length // cfg.tile_q, length // cfg.block_k
    visible = sum((min(t * cfg.tile_q + cfg.tile_q, length) - 1) // cfg.block_k + 1
                  for t in range(nt)) * hkv_r
    del pk, pv, lists
    flops_total = torch.tensor([flops_rank], dtype=torch.float64, device=dev)
    counts = torch.tensor([sel_total, visible], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(flops_total)
        dist.all_reduce(counts)
    flops_layer = float(flops_total.item())
    sparsity = 1.0 - float(counts[0].item()) / float(counts[1].item())

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()

    # ---- timed region: K steps, per-stage CUDA events on the launch stream ----
    stream = torch.cuda.current_stream(dev)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    from fpv2.kernel import index_stage, sparse_attention

    def step_timed(e):
        if mc is not None:
            mc[1].barrier(channel=0)   # no rank still reads the previous output
        e[0].record(stream)
        pk_, pv_, lists_, _ = index_stage(qd[0], kd[0], vd[0], scale=scale, config=cfg, offset=0,
                                          query_length=length, key_length=length)
        e[1].record(stream)
        out = sparse_attention(qd[0], kd[0], vd[0], pk_, pv_, *lists_, scale=scale, config=cfg,
                               offset=0, query_length=length, key_length=length, multicast=mc_args)
        e[2].record(stream)
        if mc is not None:
            mc[1].barrier(channel=0)   # every rank's output tiles have landed everywhere
        elif world > 1:
            import torch.distributed as dist

            dist.all_gather_into_tensor(out_full.view(-1), out.view(-1))
        e[3].record(stream)

    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()
    from fpv2 import _lib as fpv2_lib

    launches0 = fpv2_lib.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for i in range(args.steps):
            step_timed(ev[i])
        end.record(stream)
        torch.cuda.synchronize()
    launches = fpv2_lib.launch_count() - launches0   # this rank's kernels in the timed region
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        lt = torch.tensor([launches], dtype=torch.int64, device=dev)
        dist.all_reduce(lt)   # every rank's launches: the whole job's
        launches = int(lt.item())

    status = fpv2_lib.device_status(dev)
    if status:
        raise SystemExit(f"a kernel reported a bounded-wait timeout (status {status})")
    total_ms = start.elapsed_time(end)
    idx_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    attn_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
    gather_ms = statistics.mean(e[2].elapsed_time(e[3]) for e in ev)
    t = torch.tensor([total_ms, idx_ms, attn_ms, gather_ms], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, idx_ms, attn_ms, gather_ms = [float(x) for x in t.tolist()]
    ms_per_step = total_ms / args.steps

    # ---- end-to-end through the public API with host buffers ----
    e2e = None
    if not args.no_e2e:
        qh = qs[None].pin_memory()
        kh = ks[None].pin_memory()
        vh = vs[None].pin_memory()
        oh = torch.empty((1, hkv_r * G, length, D), dtype=dtype).pin_memory()

        def e2e_step():
            # host inputs streamed KV head by KV head: copy in, kernels and copy out of
            # consecutive heads overlap (fpv2.sdpa_from_host). With N GPUs every rank
            # streams its own KV-head shard and writes its shard of the output to host
            # memory, so the ranks together land the whole layer output on the host
            # with no device-side reassembly.
            fpv2.sdpa_from_host(qh, kh, vh, scale=scale, config=base_cfg, out=oh)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_e2e = max(2, min(args.steps, 5))
        s2.record(stream)
        for _ in range(n_e2e):
            e2e_step()
        e2.record(stream)
        torch.cuda.synchronize()
        te = torch.tensor([s2.elapsed_time(e2) / n_e2e], dtype=torch.float64, device=dev)
        if world > 1:
            import torch.distributed as dist

            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = float(te.item())
        esz = torch.finfo(dtype).bits // 8
        h2d = (qs.numel() + ks.numel() + vs.numel()) * esz * world
        d2h = qs.numel() * esz * world
        e2e = {"value": round(flops_layer / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
               "ms_per_layer": round(e2e_ms, 3), "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h)}

    # ---- CPU baseline (rank 0, N = 1 only), and the parity of its sample ----
    cpu = None
    parity = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # one more (untimed) layer on the device, kept for the parity check
        pk_p, pv_p, lists_p, _ = fpv2.index_stage(qd[0], kd[0], vd[0], scale=scale, config=cfg,
                                                  offset=0, query_length=length, key_length=length)
        out_p = fpv2.sparse_attention(qd[0], kd[0], vd[0], pk_p, pv_p, *lists_p, scale=scale,
                                      config=cfg)
        torch.cuda.synchronize()
        dt, fl, descs, samples = 0.0, 0.0, [], []
        with all_host_threads():
            for head in range(min(args.cpu_heads, Hkv)):   # about 10 s of host work by default
                d_h, f_h, desc_h, smp = cpu_sample(q, k, v, cfg, tiles_per_step=args.cpu_tiles,
                                                   head=head, want_outputs=True)
                dt += d_h
                fl += f_h
                descs.append(desc_h)
                samples.append(smp)
        cpu = {"value": round(fl / dt / 1e12, 6), "unit": "TFLOP/s", "cores": os.cpu_count(),
               "kind": "port", "sample": "; ".join(descs), "seconds": round(dt, 2)}
        parity = sample_parity(samples, lists_p, out_p, G, q, cfg)
        del pk_p, pv_p, lists_p, out_p

    if rank == 0:
        peaks, peak_src = load_peaks()
        nt_all, nb_all = length // cfg.tile_q, length // cfg.block_k
        idx_bytes_rank = index_stage_bytes(hkv_r * G, hkv_r, length, D, nt_all, nb_all)
        attn_tflops = flops_rank / (attn_ms * 1e-3) / 1e12
        idx_gbs = idx_bytes_rank / (idx_ms * 1e-3) / 1e9
        # the timed region is tens of milliseconds, not a seconds-long loop: burst peak
        peak_t = peaks["bf16_tflops"]
        peak_sus = peaks.get("bf16_tflops_sustained", peak_t)
        dense_flops = 4.0 * D * Hq * length * (length + 1) / 2
        value = flops_layer / (ms_per_step * 1e-3) / 1e12
        # (the committed ncu traffic figures are for the default tiles)
        traffic = NCU_TRAFFIC_BYTES.get(args.config, {}) if world == 1 and args.tile_q is None else {}
        line = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(3, args.warmup),
            "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16" if dtype == torch.bfloat16 else "fp16",
            "data": "synthetic topic-block generator (seed 0), inputs resident in HBM",
            "config": {
                "workload": layer_workload(args, length, Hq, Hkv, D, cfg),
                "parallelism": (f"head-parallel x{world}, output reassembled by NVLink multicast "
                                "stores from the attention kernel" if mc is not None else
                                f"head-parallel x{world} (+NCCL all-gather of the output)") if world > 1
                               else "single GPU",
                "l2": "inputs (Q+K+V) larger than the 126 MB L2 at every step",
                "ms_per_layer": round(ms_per_step, 4),
                "index_stage_ms": round(idx_ms, 4),
                "attention_ms": round(attn_ms, 4),
                "allgather_ms": round(gather_ms, 4) if world > 1 else 0.0,
                "reassembly": ("multicast stores in the attention kernel" if mc is not None
                               else "NCCL all-gather") if world > 1 else "none",
                "retained_tflop_per_layer": round(flops_layer / 1e12, 4),
                "dense_causal_tflop_per_layer": round(dense_flops / 1e12, 3),
                "block_sparsity": round(sparsity, 4),
                "selection_gbs": round(idx_gbs, 1),
                "attention_tflops": round(attn_tflops, 1),
                "attention_pct_bf16_peak": round(100 * attn_tflops / peak_t, 2),
                "attention_pct_bf16_sustained": round(100 * attn_tflops / peak_sus, 2),
                "attention_pct_bf16_spec_2250": round(100 * attn_tflops / 2250.0, 2),
                "selection_pct_hbm": round(100 * idx_gbs / peaks["hbm_gbs"], 2),
            },
            "roofline": {
                "bound": "tensor", "kernel": f"{attention_kernel_name(dtype, Hq, Hkv, D, cfg.block_k, cfg.tile_q, length // cfg.block_k)} (sparse attention)",
                "achieved": round(attn_tflops, 1), "peak": peak_t, "unit": "TFLOP/s",
                "frac": round(attn_tflops / peak_t, 4), "traffic": traffic.get("attention"),
                "traffic_unit": "bytes per launch (ncu, DRAM read + write)",
                "traffic_source": "recorded constant from an earlier ncu capture of this workload, "
                                  "not measured in this run",
                "peak_source": f"{peak_src} bf16_tflops (burst)",
            },
            "roofline_index_stage": {
                "bound": "hbm", "kernel": "pool_pipe_kernel + select_tc_kernel",
                "achieved": round(idx_gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(idx_gbs / peaks["hbm_gbs"], 4), "traffic": traffic.get("index_stage"),
                "traffic_unit": "bytes per launch pair (ncu, DRAM read + write)",
                "traffic_source": "recorded constant from an earlier ncu capture of this workload, "
                                  "not measured in this run",
                "algorithmic_bytes": idx_bytes_rank, "peak_source": f"{peak_src} hbm_gbs",
            },
            "cpu_baseline": cpu,
            "parity": parity,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clocks.summary(),
        }
        emit_json(line)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def layer_workload(args, length, Hq, Hkv, D, cfg) -> str:
    """The workload both arms name in ``config``: one FPV2 layer of this shape."""
    return (f"{args.config}: FPV2 layer L={length}, Hq={Hq}, Hkv={Hkv}, head_dim={D}, "
            f"alpha={cfg.alpha}, correction={'on' if cfg.mean_correction else 'off'}, "
            f"sink_tokens={cfg.sink_tokens}, window_tokens={cfg.window_tokens}, "
            f"last_n_blocks={cfg.last_n_blocks}, tile_q={cfg.tile_q} ({(Hq // Hkv) * cfg.tile_q} packed rows)")


def all_host_threads():
    """Every host core for the CPU legs: torch's pool and NumPy's BLAS pool (which
    follows OMP_NUM_THREADS, set to 1 per rank by torch.distributed.run)."""
    from threadpoolctl import threadpool_limits

    torch.set_num_threads(os.cpu_count() or 1)
    return threadpool_limits(limits=os.cpu_count() or 1)


def reference_arm(args, length, Hq, Hkv, D, dtype, cfg) -> int:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from tests.synthetic import topic_qkv

    q, k, v = topic_qkv(length=length, query_heads=Hq, kv_heads=Hkv, head_dim=D, seed=0, dtype=dtype)
    times, flops, desc = [], [], ""
    with all_host_threads():
        for _ in range(max(3, args.warmup)):
            cpu_sample(q, k, v, cfg, tiles_per_step=max(8, args.cpu_tiles // 8))
        for _ in range(args.steps):
            dt, fl, desc = cpu_sample(q, k, v, cfg, tiles_per_step=max(8, args.cpu_tiles // 8))
            times.append(dt)
            flops.append(fl)
    value = sum(flops) / sum(times) / 1e12
    ms = 1e3 * sum(times) / len(times)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16" if dtype == torch.bfloat16 else "fp16",
        "data": "synthetic topic-block generator (seed 0)",
        "config": {"workload": layer_workload(args, length, Hq, Hkv, D, cfg)},
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": os.cpu_count(),
                         "kind": "port",
                         "sample": f"CPU port of the reference algorithm on a bounded sample of this "
                                   f"workload per step: {desc}"},
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    emit_json(line)
    return 0


if __name__ == "__main__":
    sys.exit(main())
