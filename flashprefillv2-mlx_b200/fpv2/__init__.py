"""FlashPrefill V2 block-sparse prefill attention for NVIDIA B200 (sm_100a).

Drop-in for the reference package's operator surface (fpv2/__init__.py:3-16)
on PyTorch CUDA tensors; the compute runs in the hand-written CUDA kernels of
``libfpv2_b200.so`` (see include/fpv2_b200.h).
"""

from fpv2.kernel import (
    SUPPORTED_HEAD_DIMS,
    TileConfig,
    compact_block_indices,
    default_tile,
    index_stage,
    sparse_attention,
)
from fpv2.paged import pool_pages, sparse_attention_paged
from fpv2.patch import block_sparsity, disable, enable, fpv2_sdpa, is_enabled
from fpv2.selection import FPV2Config, block_scores_and_select, density, pool_blocks
from fpv2.stream import sdpa_from_host

__all__ = [
    "FPV2Config",
    "SUPPORTED_HEAD_DIMS",
    "TileConfig",
    "block_scores_and_select",
    "block_sparsity",
    "compact_block_indices",
    "default_tile",
    "density",
    "disable",
    "enable",
    "fpv2_sdpa",
    "index_stage",
    "is_enabled",
    "pool_blocks",
    "pool_pages",
    "sdpa_from_host",
    "sparse_attention",
    "sparse_attention_paged",
]
