"""Seeded synthetic attention inputs shared by tests and the benchmark.

``topic_qkv`` is the benchmark generator (the Qwen3-4B-shaped layer configs):
K/V tokens are ``0.5 * N(0, 1)`` plus the topic vector of their 128-token
block (one of 64 ``N(0, 1)`` topics per KV head), block 0 of K is scaled by 3
as an attention sink, and every query token is ``0.5 * N(0, 1)`` plus the
topic of a uniformly drawn earlier-or-same block.

``structured_qkv`` restates the reference's clustered fixture
(tests/synthetic.py:8-52 of the reference) with torch's CPU generator: cluster
centres ``1.2 * N(0, 1)``, every key block takes a random cluster plus noise,
queries take a random cluster per run of ``block_size / 8`` positions, values
are ``N(0, 1)``. MLX's RNG cannot be reproduced here, so the draws differ from
the reference's; the distribution is the same.

Both draw in float32 on the CPU from ``torch.Generator().manual_seed(seed)`` and
cast at the end, so the same tensors feed the oracle and the GPU.
"""

from __future__ import annotations

import torch


def topic_qkv(
    *,
    length: int,
    query_heads: int,
    kv_heads: int,
    head_dim: int = 128,
    block_size: int = 128,
    topics: int = 64,
    seed: int = 0,
    dtype: torch.dtype = torch.bfloat16,
    sink_scale: float = 3.0,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Return ``q [Hq, L, D], k, v [Hkv, L, D]`` from the topic-block generator."""
    if query_heads % kv_heads:
        raise ValueError("query_heads must be divisible by kv_heads")
    g = torch.Generator().manual_seed(seed)
    nb = (length + block_size - 1) // block_size
    centres = torch.randn((kv_heads, topics, head_dim), generator=g)
    block_topic = torch.randint(0, topics, (kv_heads, nb), generator=g)
    token_block = torch.arange(length) // block_size
    heads = torch.arange(kv_heads)[:, None]
    topic_tok = block_topic[:, token_block]                               # [Hkv, L]
    k = 0.5 * torch.randn((kv_heads, length, head_dim), generator=g) + centres[heads, topic_tok]
    v = 0.5 * torch.randn((kv_heads, length, head_dim), generator=g) + centres[heads, topic_tok]
    k[:, :block_size] *= sink_scale
    group = query_heads // kv_heads
    # every query token attends to the topic of a uniform earlier-or-same block
    u = torch.rand((query_heads, length), generator=g)
    src_block = torch.floor(u * (token_block[None, :] + 1).to(torch.float32)).long()
    kv_of_q = (torch.arange(query_heads) // group)[:, None]
    q_topic = block_topic[kv_of_q, src_block]                             # [Hq, L]
    q = 0.5 * torch.randn((query_heads, length, head_dim), generator=g) + centres[kv_of_q, q_topic]
    return q.to(dtype), k.to(dtype), v.to(dtype)


def structured_qkv(
    *,
    length: int = 2_048,
    query_heads: int = 8,
    kv_heads: int = 2,
    head_dim: int = 64,
    block_size: int = 128,
    clusters: int = 16,
    noise: float = 0.3,
    dtype: torch.dtype = torch.float32,
    seed: int = 0,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Clustered ``q, k, v`` shaped ``[heads, length, dim]``."""
    if length <= 0 or head_dim <= 0 or block_size <= 0 or clusters <= 0:
        raise ValueError("length, head_dim, block_size, and clusters must be positive")
    if query_heads <= 0 or kv_heads <= 0 or query_heads % kv_heads:
        raise ValueError("query_heads must be divisible by positive kv_heads")
    g = torch.Generator().manual_seed(seed)
    centers = 1.2 * torch.randn((kv_heads, clusters, head_dim), generator=g)
    num_blocks = (length + block_size - 1) // block_size
    kv_block_clusters = torch.randint(0, clusters, (kv_heads, num_blocks), generator=g)
    block_ids = torch.arange(length) // block_size
    kv_cluster_ids = kv_block_clusters[:, block_ids]
    head_ids = torch.arange(kv_heads)[:, None]
    keys = centers[head_ids, kv_cluster_ids]
    keys = keys + noise * torch.randn(keys.shape, generator=g)
    group_size = query_heads // kv_heads
    q_kv_ids = torch.arange(query_heads) // group_size
    query_run = max(1, block_size // 8)
    query_run_ids = torch.arange(length) // query_run
    q_run_clusters = torch.randint(
        0, clusters, (query_heads, (length + query_run - 1) // query_run), generator=g
    )
    q_cluster_ids = q_run_clusters[:, query_run_ids]
    queries = centers[q_kv_ids[:, None], q_cluster_ids]
    queries = queries + noise * torch.randn(queries.shape, generator=g)
    values = torch.randn((kv_heads, length, head_dim), generator=g)
    return queries.to(dtype), keys.to(dtype), values.to(dtype)


def uniform_qkv(shape_q, shape_kv, *, seed: int = 0, dtype=torch.bfloat16):
    """Plain ``N(0, 1)`` tensors (the reference's hook tests use these)."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(shape_q, generator=g)
    k = torch.randn(shape_kv, generator=g)
    v = torch.randn(shape_kv, generator=g)
    return q.to(dtype), k.to(dtype), v.to(dtype)
