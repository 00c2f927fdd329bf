"""Out-of-range block-list entries: clamped like the reference, reported by debug builds.

The attention kernels clamp every list entry, count and page index into range,
as the reference clips its lists (fpv2/kernel.py:555-558), so a corrupt list
can change the output but never the memory a kernel touches. The debug build
(``build.py --debug-bounds`` -> ``libfpv2_b200_debug.so``, selected with
``FPV2_LIBRARY``) also sets bit 8 of the device status word for every value it
had to clamp; the release build stays silent. Each library runs in its own
child process (the library is loaded once per process).
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
LIB_DIR = ROOT / "flashprefillv2-mlx_b200" / "fpv2" / "_lib"

CHILD = r"""
import json, sys, torch
sys.path[:0] = [sys.argv[1], sys.argv[2]]
import fpv2
from fpv2 import _lib
from fpv2.patch import _effective_config
from tests.synthetic import topic_qkv

dev = torch.device("cuda", 0)
q, k, v = topic_qkv(length=2048, query_heads=8, kv_heads=2, seed=41, dtype=torch.bfloat16)
q, k, v = q.to(dev), k.to(dev), v.to(dev)
cfg = _effective_config(fpv2.FPV2Config(alpha=0.1), 8, 2)
scale = 128 ** -0.5
pk, pv, lists, _ = fpv2.index_stage(q, k, v, scale=scale, config=cfg, offset=0,
                                    query_length=2048, key_length=2048)
nb = pk.shape[1]
def run(ls):
    return fpv2.sparse_attention(q, k, v, pk, pv, *ls, scale=scale, config=cfg, offset=0,
                                 query_length=2048, key_length=2048)
clean = run(lists)
status_clean = _lib.device_status(dev)
sc, pc = lists[1].cpu(), lists[3].cpu()      # a late tile with selected and pruned entries
t = next(t for t in range(sc.shape[1] - 1, 5, -1) if sc[0, t] >= 1 and pc[1, t] >= 1)
bad = [x.clone() for x in lists]
bad[0][0, t, 0] = nb + 7                      # selected block past the end
bad[2][1, t, 0] = -3                          # negative pruned block
bad[1][1, t - 5] = nb + 100                   # count past the list width
out_bad = run(bad)
status_bad = _lib.device_status(dev)
fixed = [x.clone() for x in lists]            # the same entries clamped by hand
fixed[0][0, t, 0] = nb - 1
fixed[2][1, t, 0] = 0
fixed[1][1, t - 5] = nb
out_fixed = run(fixed)
print(json.dumps({"lib": str(_lib.LIB_PATH), "clean": status_clean, "bad": status_bad,
                  "clamped": bool(torch.equal(out_bad, out_fixed)),
                  "finite": bool(torch.isfinite(out_bad.float()).all()),
                  "changed": bool(not torch.equal(out_bad, clean))}))
"""


def _run(lib: Path) -> dict:
    env = dict(os.environ, FPV2_LIBRARY=str(lib))
    res = subprocess.run([sys.executable, "-c", CHILD, str(ROOT / "flashprefillv2-mlx_b200"), str(ROOT)],
                         env=env, capture_output=True, text=True, timeout=300, cwd=str(ROOT))
    assert res.returncode == 0, res.stderr[-2000:]
    return json.loads(res.stdout.strip().splitlines()[-1])


def test_release_build_clamps_silently():
    r = _run(LIB_DIR / "libfpv2_b200.so")
    assert r["clean"] == 0 and r["bad"] == 0, r
    assert r["clamped"] and r["finite"] and r["changed"], r


@pytest.mark.skipif(not (LIB_DIR / "libfpv2_b200_debug.so").exists(),
                    reason="debug library not built (build.py --debug-bounds)")
def test_debug_build_reports_clamped_entries():
    r = _run(LIB_DIR / "libfpv2_b200_debug.so")
    assert r["lib"].endswith("libfpv2_b200_debug.so"), r
    assert r["clean"] == 0, r                          # valid lists: nothing to report
    assert r["bad"] & 8, r                             # STATUS_BAD_LIST
    assert r["clamped"] and r["finite"], r             # same output as the hand-clamped lists
