"""The C++ host mirror of ``vasr-paged-attn`` (module ``_vasr_host``).

Re-exports the types the Rust crate exports (vasr-paged-attn/src/lib.rs:12-27):
``PagedKvCache``, ``PagedInputMetadata``, ``PagedBlockManager``,
``PagedCacheRuntime``, ``PagedCacheStats``, ``bytes_per_paged_block``,
``FlashParams``, ``PAD_SLOT_ID``; plus the cuda_graph.rs helpers
(``cuda_graph_batch_bucket``, ``bucket_block_table_cols``,
``pad_decode_batch_to_max``, ``DecodeGraphRegistry``). Import fails loudly
if the module has not been built.
"""
from __future__ import annotations

import importlib
import sys
from pathlib import Path

_LIB_DIR = Path(__file__).resolve().parent.parent / "lib"
if str(_LIB_DIR) not in sys.path:
    sys.path.insert(0, str(_LIB_DIR))
_h = importlib.import_module("_vasr_host")

PAD_SLOT_ID = _h.PAD_SLOT_ID
VasrHostError = _h.VasrHostError
PagedKvCache = _h.PagedKvCache
PagedInputMetadata = _h.PagedInputMetadata
PagedBlockManager = _h.PagedBlockManager
PagedCacheRuntime = _h.PagedCacheRuntime
PagedCacheStats = _h.PagedCacheStats
FlashParams = _h.FlashParams
DecodeGraphRegistry = _h.DecodeGraphRegistry
bytes_per_paged_block = _h.bytes_per_paged_block
blocks_for_byte_budget = _h.blocks_for_byte_budget
cuda_graph_batch_bucket = _h.cuda_graph_batch_bucket
cuda_graph_batch_buckets = _h.cuda_graph_batch_buckets
cuda_graph_block_bucket = _h.cuda_graph_block_bucket
bucket_block_table_cols = _h.bucket_block_table_cols
cuda_graph_prewarm_batch_limit = _h.cuda_graph_prewarm_batch_limit
pad_decode_batch_to_max = _h.pad_decode_batch_to_max
can_admit_with_projected_kv = _h.can_admit_with_projected_kv
cpp_ops = _h.mistralrs_paged_attn


def metadata_cache(num_blocks: int, num_kv_heads: int, head_dim: int, block_size: int,
                   dtype: str = "bf16") -> "PagedKvCache":
    """A geometry-only PagedKvCache (no pages) for building host metadata of a pool."""
    return PagedKvCache.from_external([0], [0], num_blocks, num_kv_heads, head_dim, block_size, dtype)

