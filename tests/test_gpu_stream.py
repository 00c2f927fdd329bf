"""Host-resident inputs streamed KV head by KV head equal the one-shot layer.

``sdpa_from_host`` splits the layer into KV-head chunks (each chunk's lists,
K/V reads and outputs belong to its own heads) and overlaps the copies with the
kernels; the output must equal ``fpv2_sdpa`` on device tensors bit for bit.
"""

from __future__ import annotations

import pytest
import torch

import fpv2
from tests.synthetic import topic_qkv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("chunk,query_length,tail_slices",
                         [(1, 2048, 4), (2, 2048, 4), (1, 1920, 4), (1, 2048, 1), (2, 1920, 3)])
def test_sdpa_from_host_equals_device_layer(chunk, query_length, tail_slices):
    dev = torch.device("cuda", 0)
    q, k, v = topic_qkv(length=2048, query_heads=16, kv_heads=4, seed=31, dtype=torch.bfloat16)
    q = q[None, :, 2048 - query_length:].contiguous()
    k, v = k[None], v[None]
    cfg = fpv2.FPV2Config(alpha=0.1)
    ref = fpv2.fpv2_sdpa(q.to(dev), k.to(dev), v.to(dev), scale=128 ** -0.5, config=cfg)
    qh, kh, vh = (t.pin_memory() for t in (q, k, v))
    out = fpv2.sdpa_from_host(qh, kh, vh, scale=128 ** -0.5, config=cfg, kv_heads_per_chunk=chunk,
                              tail_slices=tail_slices)
    torch.cuda.synchronize(dev)
    assert out.is_pinned()
    assert torch.equal(out, ref.cpu())


def test_back_to_back_calls_from_host():
    """Calls queued back to back (no synchronisation between them) at a length
    whose dense-tail tiles split over segments: new staging buffers come from the
    compute stream's pool while the previous call's kernels may still run, so the
    copies must wait for them. Every output equals the device layer."""
    dev = torch.device("cuda", 0)
    q, k, v = topic_qkv(length=32768, query_heads=8, kv_heads=2, seed=33, dtype=torch.bfloat16)
    q, k, v = q[None], k[None], v[None]
    cfg = fpv2.FPV2Config(alpha=0.1)
    ref = fpv2.fpv2_sdpa(q.to(dev), k.to(dev), v.to(dev), scale=128 ** -0.5, config=cfg).cpu()
    qh, kh, vh = (t.pin_memory() for t in (q, k, v))
    outs = [fpv2.sdpa_from_host(qh, kh, vh, scale=128 ** -0.5, config=cfg) for _ in range(4)]
    torch.cuda.synchronize(dev)
    from fpv2 import _lib

    assert _lib.device_status(dev) == 0
    for out in outs:
        assert torch.equal(out, ref)


def test_back_to_back_calls_with_different_inputs_share_staging():
    """Consecutive calls reuse the kept staging buffers, and a call's copies in
    start while the previous call's last kernels and copies out may still run:
    with inputs that differ from call to call, each output must still equal its
    own device layer (a copy that overtook a kernel still reading the set would
    show). A new shape replaces the kept buffers, and release_staging drops them."""
    from fpv2 import _lib, stream

    dev = torch.device("cuda", 0)
    cfg = fpv2.FPV2Config(alpha=0.1)
    sets, refs = [], []
    for seed in (35, 36):
        q, k, v = topic_qkv(length=32768, query_heads=8, kv_heads=2, seed=seed, dtype=torch.bfloat16)
        q, k, v = q[None], k[None], v[None]
        refs.append(fpv2.fpv2_sdpa(q.to(dev), k.to(dev), v.to(dev), scale=128 ** -0.5, config=cfg).cpu())
        sets.append(tuple(t.pin_memory() for t in (q, k, v)))
    stream.release_staging()
    outs = [fpv2.sdpa_from_host(*sets[i % 2], scale=128 ** -0.5, config=cfg) for i in range(6)]
    torch.cuda.synchronize(dev)
    assert _lib.device_status(dev) == 0
    assert len(stream._STAGING) == 1
    for i, out in enumerate(outs):
        assert torch.equal(out, refs[i % 2]), i
    q, k, v = topic_qkv(length=4096, query_heads=8, kv_heads=2, seed=37, dtype=torch.bfloat16)
    q, k, v = q[None], k[None], v[None]
    ref = fpv2.fpv2_sdpa(q.to(dev), k.to(dev), v.to(dev), scale=128 ** -0.5, config=cfg).cpu()
    out = fpv2.sdpa_from_host(q.pin_memory(), k.pin_memory(), v.pin_memory(), scale=128 ** -0.5,
                              config=cfg)
    torch.cuda.synchronize(dev)
    assert torch.equal(out, ref)
    assert len(stream._STAGING) == 1
    stream.release_staging(dev)
    assert not stream._STAGING
