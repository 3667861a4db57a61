"""Tensor-level entry points with the argument order of ``mistralrs_paged_attn``.

The decoder calls these exactly as vasr-models/src/model/thinker_text.rs does
(``reshape_and_cache`` at :1101-1109 / :1324-1332, ``paged_attention`` at
:1126-1139, ``gather_kv_cache`` at :190-198 / :1344-1352); each one checks the
tensors like the Rust wrapper would and forwards raw device pointers to the
C ABI of ``include/vasr_pa.h`` on the current CUDA stream. There is no CPU or
eager fallback: a CPU tensor, an unsupported dtype or a missing library
raises.

``copy_blocks`` / ``swap_blocks`` follow the vLLM names; the reference has no
call site for them. ``paged_attention_varlen_prefill`` follows the argument
order of the reference's Metal entry point
(vasr-paged-attn/src/metal/varlen_prefill.rs:291-427) with causal masking.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import torch

from . import _lib

_DTYPE_CODE = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}
_INDEX32 = (torch.int32, torch.uint32)


# fp8 (E4M3) pages: one byte per element, per-tensor f32 scales on the device
FP8_CACHE = torch.float8_e4m3fn


def _check_scales(k_scale, v_scale, dev) -> None:
    for sc in (k_scale, v_scale):
        if sc is None or sc.dtype != torch.float32 or sc.numel() != 1 or sc.device != dev:
            raise _lib.VasrPaError(_lib.EINVAL_POINTER,
                                   "fp8 caches need k_scale / v_scale as f32 scalars on the cache device")


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise _lib.VasrPaError(_lib.EINVAL_DTYPE, f"unsupported paged cache dtype {dt}") from None


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    for t in tensors:
        if t.device.type != "cuda":
            raise _lib.VasrPaError(_lib.EINVAL_POINTER, "paged attention tensors must be on a CUDA device")
        if t.device != dev:
            raise _lib.VasrPaError(_lib.EINVAL_POINTER, "paged attention tensors on different devices")
    return dev


def cache_geometry(key_cache: torch.Tensor, value_cache: torch.Tensor):
    """(num_blocks, num_kv_heads, head_dim, block_size) of a vLLM-layout cache pair."""
    if key_cache.dim() != 5 or value_cache.dim() != 4:
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, f"cache dims {tuple(key_cache.shape)} / {tuple(value_cache.shape)}")
    nb, hkv, dx, bs, x = key_cache.shape
    nbv, hkvv, d, bsv = value_cache.shape
    if (nb, hkv, bs) != (nbv, hkvv, bsv) or dx * x != d or x * key_cache.element_size() != 16:
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, f"paged cache shape mismatch: key={tuple(key_cache.shape)} value={tuple(value_cache.shape)}")
    if key_cache.dtype != value_cache.dtype:
        raise _lib.VasrPaError(_lib.EINVAL_DTYPE, "key/value cache dtype mismatch")
    if not (key_cache.is_contiguous() and value_cache.is_contiguous()):
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "paged caches must be contiguous")
    return int(nb), int(hkv), int(d), int(bs)


def reshape_and_cache(key: torch.Tensor, value: torch.Tensor, k_scale: Optional[torch.Tensor],
                      v_scale: Optional[torch.Tensor], key_cache: torch.Tensor,
                      value_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """Scatter key/value ``[T, Hkv, D]`` into the pages at ``slot_mapping`` (int64, -1 = skip)."""
    dev = _require_cuda(key, value, key_cache, value_cache, slot_mapping)
    nb, hkv, d, bs = cache_geometry(key_cache, value_cache)
    if key.dim() != 3 or value.shape != key.shape or tuple(key.shape[1:]) != (hkv, d):
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, f"key/value shape {tuple(key.shape)} vs cache heads={hkv} dim={d}")
    fp8 = key_cache.dtype == FP8_CACHE
    if fp8:
        _check_scales(k_scale, v_scale, dev)
        if value.dtype != key.dtype:
            raise _lib.VasrPaError(_lib.EINVAL_DTYPE, "key/value dtype mismatch")
    elif key.dtype != key_cache.dtype or value.dtype != key_cache.dtype:
        raise _lib.VasrPaError(_lib.EINVAL_DTYPE, "key/value dtype must equal the cache dtype")
    for t in (key, value):
        if t.stride(2) != 1 or t.stride(1) != d:
            raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "key/value need unit dim stride and head stride head_dim")
    if slot_mapping.dtype != torch.int64 or slot_mapping.dim() != 1 or slot_mapping.shape[0] != key.shape[0]:
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "slot_mapping must be int64 [num_tokens]")
    slot_mapping = slot_mapping.contiguous()
    if fp8:
        st = _lib.lib().vasr_pa_reshape_and_cache_fp8(
            key.data_ptr(), value.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
            slot_mapping.data_ptr(), key.shape[0], hkv, d, bs, nb, key.stride(0), value.stride(0),
            dtype_code(key.dtype), k_scale.data_ptr(), v_scale.data_ptr(), _stream(dev))
        _lib.check(st, "reshape_and_cache (fp8 cache)")
        return
    st = _lib.lib().vasr_pa_reshape_and_cache(
        key.data_ptr(), value.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
        slot_mapping.data_ptr(), key.shape[0], hkv, d, bs, nb, key.stride(0), value.stride(0),
        dtype_code(key.dtype),
        k_scale.data_ptr() if k_scale is not None else None,
        v_scale.data_ptr() if v_scale is not None else None, _stream(dev))
    _lib.check(st, "reshape_and_cache")


# ---------------------------------------------------------------- workspace
_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}


def paged_attention_workspace_bytes(num_seqs: int, num_heads: int, num_kv_heads: int,
                                    head_dim: int, block_size: int, max_context_len: int,
                                    dtype: torch.dtype) -> int:
    return int(_lib.lib().vasr_pa_paged_attention_workspace_size(
        num_seqs, num_heads, num_kv_heads, head_dim, block_size, max(1, max_context_len),
        dtype_code(dtype)))


def reserve_paged_attention_workspace(device: torch.device, nbytes: int,
                                      stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """Make sure the (device, stream) workspace holds ``nbytes``; call before CUDA-graph capture.

    The workspace is zero-filled when (re)allocated; the kernel leaves its
    counters at zero after every call, so it never needs clearing again.
    One workspace per stream: two streams must not share one concurrently.
    """
    device = torch.device(device)
    s = stream if stream is not None else torch.cuda.current_stream(device)
    key = (device.index if device.index is not None else torch.cuda.current_device(), s.cuda_stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise _lib.VasrPaError(_lib.EINVAL_WORKSPACE,
                                   "paged attention workspace must be reserved before CUDA graph capture")
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


_PREFILL_SCRATCH: dict[tuple[int, int], torch.Tensor] = {}


def _reserve_prefill_scratch(device: torch.device, nbytes: int) -> torch.Tensor:
    """The (device, stream) scratch of the fp8 prefill (a 16-bit copy of the live pages).

    Separate from the paged-attention workspace, whose counters must stay zero."""
    device = torch.device(device)
    s = torch.cuda.current_stream(device)
    key = (device.index if device.index is not None else torch.cuda.current_device(), s.cuda_stream)
    ws = _PREFILL_SCRATCH.get(key)
    if ws is None or ws.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise _lib.VasrPaError(_lib.EINVAL_WORKSPACE,
                                   "fp8 prefill scratch must be reserved before CUDA graph capture")
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _PREFILL_SCRATCH[key] = ws
    return ws


def paged_attention(q: torch.Tensor, k_scale: Optional[torch.Tensor], v_scale: Optional[torch.Tensor],
                    key_cache: torch.Tensor, value_cache: torch.Tensor, block_tables: torch.Tensor,
                    context_lens: torch.Tensor, alibi: Optional[torch.Tensor], max_context_len: int,
                    softmax_scale: float, softcapping: float = 1.0,
                    sinks: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                    after_append: bool = False) -> torch.Tensor:
    """Single-token decode attention over the pages; returns ``[B, Hq, D]`` in q's dtype.

    ``after_append=True`` (16-bit pages) launches it as a programmatic
    dependent of the kernel just issued on the current stream, which must be
    this step's KV append (``reshape_and_cache`` or the fused q/k norm + RoPE +
    append): the pages before each sequence's last one stream in while the
    append finishes (vasr_pa_paged_attention_after_append)."""
    if alibi is not None or sinks is not None:
        raise _lib.VasrPaError(_lib.ENOT_SUPPORTED, "alibi / attention sinks are not used by Qwen3-ASR")
    dev = _require_cuda(q, key_cache, value_cache, block_tables, context_lens)
    nb, hkv, d, bs = cache_geometry(key_cache, value_cache)
    if q.dim() != 3 or q.shape[2] != d or q.stride(2) != 1 or q.stride(1) != d:
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, f"q must be [B, Hq, {d}] with packed heads, got {tuple(q.shape)}")
    fp8 = key_cache.dtype == FP8_CACHE
    if fp8:
        _check_scales(k_scale, v_scale, dev)
    elif q.dtype != key_cache.dtype:
        raise _lib.VasrPaError(_lib.EINVAL_DTYPE, "q dtype must equal the cache dtype")
    b, hq = int(q.shape[0]), int(q.shape[1])
    if block_tables.dtype not in _INDEX32 or block_tables.dim() != 2 or block_tables.shape[0] != b:
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "block_tables must be u32/i32 [B, cols]")
    if context_lens.dtype not in _INDEX32 or context_lens.shape != (b,):
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "context_lens must be u32/i32 [B]")
    block_tables = block_tables.contiguous()
    context_lens = context_lens.contiguous()
    if out is None:
        out = torch.empty((b, hq, d), dtype=q.dtype, device=dev)
    need = paged_attention_workspace_bytes(b, hq, hkv, d, bs, max_context_len, q.dtype)
    ws = reserve_paged_attention_workspace(dev, need)
    if fp8:
        st = _lib.lib().vasr_pa_paged_attention_fp8(
            out.data_ptr(), q.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
            block_tables.data_ptr(), context_lens.data_ptr(), b, hq, hkv, d, bs, nb,
            int(block_tables.shape[1]), int(max_context_len), float(softmax_scale), float(softcapping),
            q.stride(0), dtype_code(q.dtype), k_scale.data_ptr(), v_scale.data_ptr(), ws.data_ptr(),
            ws.numel(), _stream(dev))
        _lib.check(st, "paged_attention (fp8 cache)")
        return out
    entry = _lib.lib().vasr_pa_paged_attention_after_append if after_append else _lib.lib().vasr_pa_paged_attention
    st = entry(
        out.data_ptr(), q.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
        block_tables.data_ptr(), context_lens.data_ptr(), b, hq, hkv, d, bs, nb,
        int(block_tables.shape[1]), int(max_context_len), float(softmax_scale), float(softcapping),
        q.stride(0), dtype_code(q.dtype), ws.data_ptr(), ws.numel(), _stream(dev))
    _lib.check(st, "paged_attention")
    return out


def gather_kv_cache(key_cache: torch.Tensor, value_cache: torch.Tensor,
                    k_scale: Optional[torch.Tensor], v_scale: Optional[torch.Tensor],
                    block_tables: torch.Tensor, cu_seqlens_kv: torch.Tensor,
                    out_dtype: Optional[torch.dtype] = None,
                    total_tokens: Optional[int] = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Packed ``[sum kv, Hkv, D]`` copies of each sequence's first kv_len tokens.

    fp8 (E4M3) pages need k_scale / v_scale and give ``byte * scale`` in
    out_dtype (bf16 when None); other caches keep their dtype."""
    dev = _require_cuda(key_cache, value_cache, block_tables, cu_seqlens_kv)
    nb, hkv, d, bs = cache_geometry(key_cache, value_cache)
    fp8 = key_cache.dtype == FP8_CACHE
    if fp8:
        _check_scales(k_scale, v_scale, dev)
        out_dtype = torch.bfloat16 if out_dtype is None else out_dtype
    elif out_dtype is not None and out_dtype != key_cache.dtype:
        raise _lib.VasrPaError(_lib.EINVAL_DTYPE, "gather_kv_cache keeps the cache dtype")
    else:
        out_dtype = key_cache.dtype
    if block_tables.dtype not in _INDEX32 or cu_seqlens_kv.dtype not in _INDEX32:
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "block_tables / cu_seqlens_kv must be u32/i32")
    b = int(block_tables.shape[0])
    if cu_seqlens_kv.shape != (b + 1,):
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "cu_seqlens_kv must be [B + 1]")
    if total_tokens is None:
        total_tokens = int(cu_seqlens_kv[-1].item())  # host read, as the Rust wrapper sizes outputs
    k_out = torch.empty((total_tokens, hkv, d), dtype=out_dtype, device=dev)
    v_out = torch.empty_like(k_out)
    bt = block_tables.contiguous()
    cu = cu_seqlens_kv.contiguous()
    if fp8:
        st = _lib.lib().vasr_pa_gather_kv_cache_fp8(
            k_out.data_ptr(), v_out.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
            bt.data_ptr(), cu.data_ptr(), b, int(bt.shape[1]), total_tokens, hkv, d, bs, nb,
            dtype_code(out_dtype), k_scale.data_ptr(), v_scale.data_ptr(), _stream(dev))
    else:
        st = _lib.lib().vasr_pa_gather_kv_cache(
            k_out.data_ptr(), v_out.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
            bt.data_ptr(), cu.data_ptr(), b, int(bt.shape[1]), total_tokens, hkv, d, bs, nb,
            dtype_code(key_cache.dtype), _stream(dev))
    _lib.check(st, "gather_kv_cache")
    return k_out, v_out


def paged_attention_varlen_prefill(q: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                                   block_tables: torch.Tensor, context_lens: torch.Tensor,
                                   cu_seqlens_q: torch.Tensor, k_scale: Optional[torch.Tensor],
                                   v_scale: Optional[torch.Tensor], scale: float,
                                   softcapping: float = 1.0, max_query_len: Optional[int] = None,
                                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Causal chunked prefill: packed q ``[T, Hq, D]`` against each sequence's pages.

    fp8 (E4M3) pages need k_scale / v_scale. 16-token pages at GQA 1 / 2 / 4 are
    read by the tcgen05 kernel directly (bytes converted to f16 in shared
    memory); other page sizes are scaled into a 16-bit scratch pool in the
    stream's workspace first."""
    dev = _require_cuda(q, key_cache, value_cache, block_tables, context_lens, cu_seqlens_q)
    nb, hkv, d, bs = cache_geometry(key_cache, value_cache)
    if q.dim() != 3 or q.shape[2] != d or q.stride(2) != 1 or q.stride(1) != d:
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, f"q must be [T, Hq, {d}] with packed heads")
    fp8 = key_cache.dtype == FP8_CACHE
    if fp8:
        _check_scales(k_scale, v_scale, dev)
    elif q.dtype != key_cache.dtype:
        raise _lib.VasrPaError(_lib.EINVAL_DTYPE, "q dtype must equal the cache dtype")
    b = int(block_tables.shape[0])
    if cu_seqlens_q.shape != (b + 1,) or context_lens.shape != (b,):
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "varlen metadata batch mismatch")
    if max_query_len is None:
        max_query_len = int((cu_seqlens_q[1:] - cu_seqlens_q[:-1]).max().item())
    t, hq = int(q.shape[0]), int(q.shape[1])
    if out is None:
        out = torch.empty((t, hq, d), dtype=q.dtype, device=dev)
    bt = block_tables.contiguous()
    if fp8:
        need = int(_lib.lib().vasr_pa_paged_attention_varlen_prefill_fp8_workspace_size(
            b, hkv, d, bs, int(bt.shape[1])))
        ws = _reserve_prefill_scratch(dev, need)
        st = _lib.lib().vasr_pa_paged_attention_varlen_prefill_fp8(
            out.data_ptr(), q.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), bt.data_ptr(),
            context_lens.contiguous().data_ptr(), cu_seqlens_q.contiguous().data_ptr(), b, t,
            int(max_query_len), hq, hkv, d, bs, nb, int(bt.shape[1]), float(scale),
            float(softcapping), q.stride(0), dtype_code(q.dtype), k_scale.data_ptr(),
            v_scale.data_ptr(), ws.data_ptr(), ws.numel(), _stream(dev))
        _lib.check(st, "paged_attention_varlen_prefill (fp8 pages)")
        return out
    st = _lib.lib().vasr_pa_paged_attention_varlen_prefill(
        out.data_ptr(), q.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), bt.data_ptr(),
        context_lens.contiguous().data_ptr(), cu_seqlens_q.contiguous().data_ptr(), b, t,
        int(max_query_len), hq, hkv, d, bs, nb, int(bt.shape[1]), float(scale), float(softcapping),
        q.stride(0), dtype_code(q.dtype), _stream(dev))
    _lib.check(st, "paged_attention_varlen_prefill")
    return out


def copy_blocks(key_caches: Sequence[torch.Tensor], value_caches: Sequence[torch.Tensor],
                block_mapping: torch.Tensor) -> None:
    """For every layer and (src, dst) pair of ``block_mapping`` (int64 [N, 2]): page dst <- page src."""
    if len(key_caches) != len(value_caches) or not key_caches:
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "copy_blocks needs one K and one V cache per layer")
    dev = _require_cuda(*key_caches, *value_caches, block_mapping)
    nb, hkv, d, bs = cache_geometry(key_caches[0], value_caches[0])
    for k, v in zip(key_caches, value_caches):
        if cache_geometry(k, v) != (nb, hkv, d, bs) or k.dtype != key_caches[0].dtype:
            raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "all layers must share one cache geometry")
    if block_mapping.dtype != torch.int64 or block_mapping.dim() != 2 or block_mapping.shape[1] != 2:
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "block_mapping must be int64 [N, 2]")
    bm = block_mapping.contiguous()
    n = len(key_caches)
    kp = (ctypes.c_void_p * n)(*[k.data_ptr() for k in key_caches])
    vp = (ctypes.c_void_p * n)(*[v.data_ptr() for v in value_caches])
    block_bytes = hkv * d * bs * key_caches[0].element_size()
    st = _lib.lib().vasr_pa_copy_blocks(kp, vp, n, bm.data_ptr(), int(bm.shape[0]), nb, block_bytes,
                                        _stream(dev))
    _lib.check(st, "copy_blocks")


def swap_blocks(src: torch.Tensor, dst: torch.Tensor, block_mapping: torch.Tensor) -> None:
    """dst[pair.dst] = src[pair.src] between two caches of one geometry (device or pinned host).

    ``block_mapping`` is int64 [N, 2] on the device or in pinned host memory.
    """
    if src.dtype != dst.dtype or src.shape[1:] != dst.shape[1:]:
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "swap_blocks caches differ in geometry")
    if not (src.is_contiguous() and dst.is_contiguous()):
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "swap_blocks caches must be contiguous")
    for t in (src, dst, block_mapping):
        if t.device.type == "cpu" and not t.is_pinned():
            raise _lib.VasrPaError(_lib.EINVAL_POINTER, "host side of swap_blocks must be pinned memory")
    if block_mapping.dtype != torch.int64 or block_mapping.dim() != 2 or block_mapping.shape[1] != 2:
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "block_mapping must be int64 [N, 2]")
    cuda_side = dst if dst.device.type == "cuda" else src
    dev = cuda_side.device if cuda_side.device.type == "cuda" else torch.device("cuda", torch.cuda.current_device())
    block_bytes = (src[0].numel() * src.element_size()) if src.shape[0] else 0
    st = _lib.lib().vasr_pa_swap_blocks(dst.data_ptr(), src.data_ptr(), block_mapping.data_ptr(),
                                        int(block_mapping.shape[0]), int(src.shape[0]), int(dst.shape[0]),
                                        block_bytes, _stream(dev))
    _lib.check(st, "swap_blocks")


def device_error(clear: bool = True, device: Optional[torch.device] = None) -> int:
    """Device error bits (VASR_PA_DERR_*) of the current device; synchronises the stream."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    out = ctypes.c_int32(0)
    _lib.check(_lib.lib().vasr_pa_get_device_error(ctypes.byref(out), int(clear), _stream(dev)),
               "get_device_error")
    return int(out.value)
