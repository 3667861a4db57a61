"""Seeded synthetic inputs of the BASELINE configs, shared by tests and smoke().

Everything is numpy on the host so the same case feeds the CPU oracle and
(after an upload) the CUDA kernels. Unused pool slots are filled with a NaN
sentinel so that any stray read shows up in the outputs and any stray write
shows up in a bit-exact pool comparison.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

import paged_ref as ref
from vasr_paged_attn.workloads import config3_rounds, loguniform_lens, uniform_lens  # noqa: F401

F32_SENTINEL = np.uint32(0x7FC0DEAD)  # a quiet NaN
BF16_SENTINEL = np.uint16(0x7FC1)     # a quiet NaN
F16_SENTINEL = np.uint16(0x7E5A)      # a quiet NaN


def sentinel_for(dtype: str):
    return {"f32": F32_SENTINEL, "bf16": BF16_SENTINEL, "f16": F16_SENTINEL}[dtype]


def bits_to_f32(bits: np.ndarray, dtype: str) -> np.ndarray:
    """Raw element bits (u32 for f32, u16 for bf16 / f16) -> f32 values."""
    if dtype == "f32":
        return bits.view(np.float32)
    if dtype == "f16":
        return np.ascontiguousarray(bits).view(np.float16).astype(np.float32)
    return ref.bf16_bits_to_f32(bits)


@dataclass
class PagedCase:
    dtype: str            # "f32", "bf16" or "f16"
    num_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    num_blocks: int
    context_lens: np.ndarray      # u32 [B]  (cached + new tokens)
    block_tables: np.ndarray      # u32 [B, cols]
    key_cache: np.ndarray         # raw bits: u32 (f32) or u16 (bf16)
    value_cache: np.ndarray
    q: np.ndarray                 # raw bits [B, Hq, D]
    k_new: np.ndarray             # raw bits [B, Hkv, D]
    v_new: np.ndarray
    slots: np.ndarray             # i64 [B] slot of the new token

    @property
    def bits_dtype(self):
        return np.uint32 if self.dtype == "f32" else np.uint16

    def as_f32(self, bits: np.ndarray) -> np.ndarray:
        return bits_to_f32(bits, self.dtype)


def _to_bits(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "f32":
        return np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    if dtype == "f16":
        return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)
    return ref.f32_to_bf16_bits(x)


def disjoint_block_tables(rng, lens_blocks, num_blocks, cols=None):
    """Seeded permutation of 1..num_blocks-1 (block 0 is the null block), split per sequence."""
    perm = rng.permutation(np.arange(1, num_blocks, dtype=np.int64))
    need = int(sum(lens_blocks))
    if need > len(perm):
        raise ValueError(f"pool too small: need {need} blocks, have {len(perm)}")
    width = cols if cols is not None else max(lens_blocks)
    tables = np.zeros((len(lens_blocks), width), dtype=np.uint32)
    off = 0
    for i, n in enumerate(lens_blocks):
        tables[i, :n] = perm[off:off + n]
        off += n
    return tables


def make_decode_case(seed: int, cached_lens, dtype="f32", num_heads=16, num_kv_heads=8,
                     head_dim=128, block_size=16, num_blocks=512, cols=None) -> PagedCase:
    """Sequences with ``cached_lens`` tokens in the pool, each appending one new token."""
    rng = np.random.default_rng(seed)
    cached = np.asarray(cached_lens, dtype=np.int64)
    ctx = cached + 1
    b = len(ctx)
    lens_blocks = [int(-(-c // block_size)) for c in ctx]
    tables = disjoint_block_tables(rng, lens_blocks, num_blocks, cols)
    x = 16 // (4 if dtype == "f32" else 2)
    sentinel = sentinel_for(dtype)
    kc = np.full((num_blocks, num_kv_heads, head_dim // x, block_size, x), sentinel)
    vc = np.full((num_blocks, num_kv_heads, head_dim, block_size), sentinel)
    # cached tokens, written with the oracle's scatter
    for i in range(b):
        n = int(cached[i])
        if n == 0:
            continue
        k = _to_bits(rng.standard_normal((n, num_kv_heads, head_dim), dtype=np.float32), dtype)
        v = _to_bits(rng.standard_normal((n, num_kv_heads, head_dim), dtype=np.float32), dtype)
        pos = np.arange(n)
        slots = (tables[i, pos // block_size].astype(np.int64) * block_size + pos % block_size)
        ref.reshape_and_cache(k, v, kc, vc, slots, block_size)
    q = _to_bits(rng.standard_normal((b, num_heads, head_dim), dtype=np.float32), dtype)
    k_new = _to_bits(rng.standard_normal((b, num_kv_heads, head_dim), dtype=np.float32), dtype)
    v_new = _to_bits(rng.standard_normal((b, num_kv_heads, head_dim), dtype=np.float32), dtype)
    slots = np.array([int(tables[i, cached[i] // block_size]) * block_size + int(cached[i] % block_size)
                      for i in range(b)], dtype=np.int64)
    return PagedCase(dtype, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                     ctx.astype(np.uint32), tables, kc, vc, q, k_new, v_new, slots)


def appended(case: PagedCase) -> PagedCase:
    """The same case with its new token already in the pool (for decode-only checks)."""
    kc, vc = case.key_cache.copy(), case.value_cache.copy()
    ref.reshape_and_cache(case.k_new, case.v_new, kc, vc, case.slots, case.block_size)
    return PagedCase(case.dtype, case.num_heads, case.num_kv_heads, case.head_dim, case.block_size,
                     case.num_blocks, case.context_lens, case.block_tables, kc, vc, case.q,
                     case.k_new, case.v_new, case.slots)


def oracle_decode(case: PagedCase, scale=None, softcap=1.0, after_append=True, use_double=True):
    """Oracle output (f32) of append(new token) + paged decode for a case."""
    kc, vc = case.key_cache.copy(), case.value_cache.copy()
    if after_append:
        ref.reshape_and_cache(case.k_new, case.v_new, kc, vc, case.slots, case.block_size)
    kf = np.ascontiguousarray(case.as_f32(kc))
    vf = np.ascontiguousarray(case.as_f32(vc))
    qf = np.ascontiguousarray(case.as_f32(case.q))
    scale = scale if scale is not None else case.head_dim ** -0.5
    return ref.paged_attention(qf, kf, vf, np.ascontiguousarray(case.block_tables),
                               np.ascontiguousarray(case.context_lens), scale, softcap,
                               use_double=use_double), kc, vc


# f32, cached {137, 512, 1023, 2048} + 1, 512-block pool, seed 0.
CONFIG1_CACHED = (137, 512, 1023, 2048)


def config1_case() -> PagedCase:
    return make_decode_case(0, CONFIG1_CACHED, dtype="f32", num_blocks=512)


@dataclass
class PrefillCase:
    dtype: str
    num_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    context_lens: np.ndarray      # u32 [B] = cached + chunk
    cu_q: np.ndarray              # u32 [B + 1]
    block_tables: np.ndarray      # u32 [B, cols]
    key_cache: np.ndarray         # raw bits, every token < context_lens[b] present
    value_cache: np.ndarray
    q: np.ndarray                 # raw bits [sum chunk, Hq, D]

    def as_f32(self, bits):
        return bits_to_f32(bits, self.dtype)


def make_prefill_case(seed, cached, chunk, dtype="bf16", num_heads=16, num_kv_heads=8, head_dim=128,
                      block_size=16, num_blocks=None, cols=None) -> PrefillCase:
    """Sequences with ``cached[b]`` tokens in the pool whose next ``chunk[b]`` tokens (also already
    appended, as the engine does before attention) are the packed queries."""
    rng = np.random.default_rng(seed)
    cached = np.asarray(cached, np.int64)
    chunk = np.asarray(chunk, np.int64)
    ctx = cached + chunk
    lens_blocks = [int(-(-c // block_size)) for c in ctx]
    if num_blocks is None:
        num_blocks = sum(lens_blocks) + 8
    tables = disjoint_block_tables(rng, lens_blocks, num_blocks, cols)
    x = 16 // (4 if dtype == "f32" else 2)
    sentinel = sentinel_for(dtype)
    kc = np.full((num_blocks, num_kv_heads, head_dim // x, block_size, x), sentinel)
    vc = np.full((num_blocks, num_kv_heads, head_dim, block_size), sentinel)
    for i, n in enumerate(ctx):
        n = int(n)
        k = _to_bits(rng.standard_normal((n, num_kv_heads, head_dim), dtype=np.float32), dtype)
        v = _to_bits(rng.standard_normal((n, num_kv_heads, head_dim), dtype=np.float32), dtype)
        pos = np.arange(n)
        slots = tables[i, pos // block_size].astype(np.int64) * block_size + pos % block_size
        ref.reshape_and_cache(k, v, kc, vc, slots, block_size)
    total = int(chunk.sum())
    q = _to_bits(rng.standard_normal((total, num_heads, head_dim), dtype=np.float32), dtype)
    cu = np.concatenate([[0], np.cumsum(chunk)]).astype(np.uint32)
    return PrefillCase(dtype, num_heads, num_kv_heads, head_dim, block_size, ctx.astype(np.uint32), cu,
                       tables, kc, vc, q)


def oracle_prefill(case: PrefillCase, scale=None, softcap=1.0, use_double=True):
    kf = np.ascontiguousarray(case.as_f32(case.key_cache))
    vf = np.ascontiguousarray(case.as_f32(case.value_cache))
    qf = np.ascontiguousarray(case.as_f32(case.q))
    scale = scale if scale is not None else case.head_dim ** -0.5
    return ref.prefill_varlen(qf, kf, vf, np.ascontiguousarray(case.block_tables),
                              np.ascontiguousarray(case.context_lens), case.cu_q, scale, softcap,
                              use_double=use_double)


