"""The no-allocation attention entry point, ``fpv2_sparse_attention_noalloc``.

Callers that cannot allocate device memory use it: serving engines that have
reserved nearly all HBM for their own KV-cache pool and allow no allocation
outside it, and pipelines that may not let a cudaMalloc (which can synchronise
the device) run between their asynchronous launches. The entry point keeps the
attention kernel's work-queue counter in a fixed array inside the library
instead of a caller-provided workspace.

The GPU test calls it through the C ABI twice in a row on the same inputs and
checks each output against the regular entry point, ``fpv2_sparse_attention``,
given a caller workspace of the same size as the library's array
(FPV2_NOALLOC_SCRATCH_BYTES: room for the work counter only, so neither runs
the fp16 copy of V nor the split of long work items that a full workspace
enables): the same kernel on the same lists, so the outputs must be
bit-identical (every work item is computed whole by one CTA, whatever order the
CTAs take the items in). The cases reach all three tensor-core attention
kernels that draw work from the counter: the single-chunk kernel (default
tiles), the chunk-pair kernel (128-position tiles, four 128-row chunks per
tile) and the head_dim 256 kernel. This file is collected last on purpose, and
the test passes both alone in a fresh process and after the rest of the suite.
"""

from __future__ import annotations

import ctypes
from dataclasses import replace
from pathlib import Path

import pytest
import torch

import fpv2
from fpv2 import _lib
from fpv2.patch import _effective_config
from tests.synthetic import topic_qkv


def _noalloc(q, k, v, pk, pv, lists, out, cfg, scale, stream):
    return _lib.lib().fpv2_sparse_attention_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), pk.data_ptr(), pv.data_ptr(),
        _lib.dtype_code(pk.dtype), lists[0].data_ptr(), lists[1].data_ptr(),
        lists[2].data_ptr(), lists[3].data_ptr(), _lib.dtype_code(q.dtype), q.shape[0],
        k.shape[0], q.shape[1], k.shape[1], q.shape[2], 0, q.shape[1], k.shape[1],
        ctypes.c_float(scale), cfg.block_k, cfg.tile_q, 1 if cfg.mean_correction else 0,
        out.data_ptr(), stream)


NOALLOC_SCRATCH_BYTES = 256   # FPV2_NOALLOC_SCRATCH_BYTES (include/fpv2_b200.h)


def _workspace_call(q, k, v, pk, pv, lists, out, cfg, scale, ws, stream):
    return _lib.lib().fpv2_sparse_attention(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), pk.data_ptr(), pv.data_ptr(),
        _lib.dtype_code(pk.dtype), lists[0].data_ptr(), lists[1].data_ptr(),
        lists[2].data_ptr(), lists[3].data_ptr(), _lib.dtype_code(q.dtype), q.shape[0],
        k.shape[0], q.shape[1], k.shape[1], q.shape[2], 0, q.shape[1], k.shape[1],
        ctypes.c_float(scale), cfg.block_k, cfg.tile_q, 1 if cfg.mean_correction else 0,
        out.data_ptr(), ws.data_ptr(), ws.numel() * 4, stream)


def test_noalloc_scratch_size_matches_header():
    header = (Path(__file__).resolve().parents[1] / "include" / "fpv2_b200.h").read_text()
    assert f"#define FPV2_NOALLOC_SCRATCH_BYTES {NOALLOC_SCRATCH_BYTES}" in header


def test_noalloc_rejects_problems_beyond_its_scratch():
    """Sizes beyond FPV2_NOALLOC_MAX_WORK_ITEMS are refused before any GPU work."""
    rc = _lib.lib().fpv2_sparse_attention_noalloc(
        None, None, None, None, None, 1, None, None, None, None, 1, 64, 1, 1 << 30, 1 << 30,
        128, 0, 1 << 30, 1 << 30, ctypes.c_float(0.1), 128, 1, 1, None, None)
    assert rc == _lib.ERR_INVALID_ARGUMENT
    assert "no-alloc scratch" in _lib.lib().fpv2_last_error().decode()


@pytest.mark.gpu
@pytest.mark.parametrize("length,hq,hkv,head_dim,tile_q", [
    (2048, 8, 2, 128, None),     # attn_tc_kernel (one 128-row chunk per tile)
    (8192, 32, 8, 128, None),
    (4096, 8, 2, 128, 128),      # attn_pair_kernel (four chunks per tile, paired)
    (2048, 8, 2, 256, None),     # attn_wide_kernel
])
def test_noalloc_matches_workspace_entry_twice(length, hq, hkv, head_dim, tile_q):
    dev = torch.device("cuda:0")
    q, k, v = topic_qkv(length=length, query_heads=hq, kv_heads=hkv, head_dim=head_dim, seed=5,
                        dtype=torch.bfloat16)
    q, k, v = q.to(dev), k.to(dev), v.to(dev)
    base = fpv2.FPV2Config(alpha=0.1)
    cfg = replace(base, tile_q=tile_q) if tile_q else _effective_config(base, hq, hkv)
    scale = head_dim ** -0.5
    pk, pv, lists, _ = fpv2.index_stage(q, k, v, scale=scale, config=cfg, offset=0,
                                        query_length=length, key_length=length)
    stream = torch.cuda.current_stream(dev).cuda_stream
    expected = torch.full_like(q, float("nan"))
    ws = torch.zeros(NOALLOC_SCRATCH_BYTES // 4, dtype=torch.int32, device=dev)
    rc = _workspace_call(q, k, v, pk, pv, lists, expected, cfg, scale, ws, stream)
    assert rc == _lib.OK, _lib.lib().fpv2_last_error().decode()
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        rc = _noalloc(q, k, v, pk, pv, lists, out, cfg, scale, stream)
        assert rc == _lib.OK, _lib.lib().fpv2_last_error().decode()
        torch.cuda.synchronize(dev)
        assert _lib.device_status(dev) == 0
        assert torch.equal(out, expected)
