"""Fused pre-attention step: q/k RMSNorm + rotary embedding + KV append (one launch).

Replaces the per-layer chain of vasr-models/src/model/thinker_text.rs:1041-1109
(q_norm, k_norm, mRoPE — 1-D RoPE for equal position streams — and
reshape_and_cache) with ``vasr_pa_fused_qk_norm_rope_append``.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from .mistralrs_paged_attn import _require_cuda, _stream, cache_geometry, dtype_code


def qk_norm_rope_append(qkv: torch.Tensor, q_norm_weight: torch.Tensor, k_norm_weight: torch.Tensor,
                        eps: float, cos_table: torch.Tensor, sin_table: torch.Tensor,
                        positions: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                        slot_mapping: torch.Tensor, num_heads: int,
                        q_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """qkv [T, (Hq + 2 Hkv) * D] -> q [T, Hq, D]; k and v are appended to the pages."""
    dev = _require_cuda(qkv, key_cache, value_cache, positions, slot_mapping, cos_table, sin_table)
    nb, hkv, d, bs = cache_geometry(key_cache, value_cache)
    t = int(qkv.shape[0])
    if qkv.dim() != 2 or qkv.stride(1) != 1 or qkv.shape[1] != (num_heads + 2 * hkv) * d:
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "qkv must be [T, (Hq + 2 Hkv) * D] with unit column stride")
    if cos_table.dtype != torch.float32 or sin_table.shape != cos_table.shape or cos_table.shape[1] != d // 2:
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "cos/sin tables must be f32 [max_position, D / 2]")
    if positions.dtype != torch.int64 or slot_mapping.dtype != torch.int64:
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "positions / slot_mapping must be int64")
    if q_out is None:
        q_out = torch.empty((t, num_heads, d), dtype=qkv.dtype, device=dev)
    st = _lib.lib().vasr_pa_fused_qk_norm_rope_append(
        q_out.data_ptr(), qkv.data_ptr(), qkv.stride(0), q_norm_weight.data_ptr(),
        k_norm_weight.data_ptr(), float(eps), cos_table.contiguous().data_ptr(),
        sin_table.contiguous().data_ptr(), int(cos_table.shape[0]), positions.contiguous().data_ptr(),
        key_cache.data_ptr(), value_cache.data_ptr(), slot_mapping.contiguous().data_ptr(), t,
        num_heads, hkv, d, bs, nb, dtype_code(qkv.dtype), _stream(dev))
    _lib.check(st, "fused_qk_norm_rope_append")
    return q_out
