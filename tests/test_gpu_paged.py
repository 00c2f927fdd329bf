"""Paged K/V equals the contiguous layer bit for bit.

Keys and values are scattered into page pools ``[pages, page_size, kv_heads,
dim]`` under a random block table (with unused pages in between); pooling the
pages must reproduce ``pool_blocks`` exactly and the paged attention must
reproduce ``sparse_attention`` on the contiguous tensors exactly, since the
kernels see the same tiles in the same order.
"""

from __future__ import annotations

from dataclasses import replace

import pytest
import torch

import fpv2
from fpv2 import _lib
from fpv2.patch import _effective_config
from tests.synthetic import topic_qkv

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _pool(x: torch.Tensor, page_size: int, extra: int, seed: int):
    heads, length, dim = x.shape
    n = length // page_size
    gen = torch.Generator().manual_seed(seed)
    table = torch.randperm(n + extra, generator=gen)[:n].to(torch.int32)
    cache = torch.zeros((n + extra, page_size, heads, dim), dtype=x.dtype)
    cache[table.long()] = x.reshape(heads, n, page_size, dim).permute(1, 2, 0, 3)
    return cache, table


@pytest.mark.parametrize("page_size,dtype,dim,offset,tile_q", [
    (16, torch.bfloat16, 128, 0, None),
    (128, torch.bfloat16, 128, 0, None),
    (256, torch.float16, 128, 0, None),
    (32, torch.bfloat16, 96, 0, None),
    (64, torch.bfloat16, 64, 0, None),
    (16, torch.bfloat16, 128, 512, None),
    (16, torch.bfloat16, 128, 0, 256),     # chunk pairs of a tile share K/V tiles
    (64, torch.float16, 128, 512, 64),
])
def test_paged_attention_equals_contiguous(page_size, dtype, dim, offset, tile_q):
    length, hq, hkv = 2048, 8, 2
    q, k, v = topic_qkv(length=length, query_heads=hq, kv_heads=hkv, head_dim=dim, seed=5, dtype=dtype)
    q = q[:, offset:].contiguous()
    ql = length - offset
    cfg = _effective_config(fpv2.FPV2Config(alpha=0.1, sink_tokens=128, window_tokens=256), hq, hkv)
    if tile_q is not None:
        cfg = replace(cfg, tile_q=tile_q)
    scale = dim ** -0.5
    qg, kg, vg = q.to(DEV), k.to(DEV), v.to(DEV)
    pk, pv, lists, _ = fpv2.index_stage(qg, kg, vg, scale=scale, config=cfg, offset=offset,
                                        query_length=ql, key_length=length)
    ref = fpv2.sparse_attention(qg, kg, vg, pk, pv, *lists, scale=scale, config=cfg, offset=offset,
                                query_length=ql, key_length=length)
    kc, table = _pool(k, page_size, extra=5, seed=1)
    vc, _ = _pool(v, page_size, extra=5, seed=1)
    kc, vc, table = kc.to(DEV), vc.to(DEV), table.to(DEV)
    pk2 = fpv2.pool_pages(kc, table, cfg.block_k, length)
    pv2 = fpv2.pool_pages(vc, table, cfg.block_k, length)
    assert torch.equal(pk2, pk) and torch.equal(pv2, pv)
    out = fpv2.sparse_attention_paged(qg, kc, vc, table, pk2, pv2, *lists, scale=scale, config=cfg,
                                      offset=offset, query_length=ql, key_length=length)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert torch.equal(out, ref)


def test_paged_pooling_in_float32_matches_pool_blocks():
    _, k, _ = topic_qkv(length=1024, query_heads=4, kv_heads=2, head_dim=128, seed=8,
                        dtype=torch.bfloat16)
    kc, table = _pool(k, 32, extra=3, seed=2)
    got = fpv2.pool_pages(kc.to(DEV), table.to(DEV), 128, 1024, dtype=torch.float32)
    ref32 = fpv2.pool_blocks(k.float().to(DEV), 128)
    assert torch.equal(got, ref32)
    # the 16-bit output is the float32 mean rounded once
    got16 = fpv2.pool_pages(kc.to(DEV), table.to(DEV), 128, 1024)
    assert torch.equal(got16, ref32.to(torch.bfloat16))
