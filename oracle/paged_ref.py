"""CPU oracle of the paged KV-cache path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs import this module; the product never does.

Two halves:

1. A pure-Python restatement of the integer host logic of the Rust crate
   ``vasr-paged-attn`` (layout dims, slot math, metadata builders, block
   manager, CUDA-graph buckets and padding). Each function cites the Rust
   function it restates. These are pinned bit-exact against the reference's
   own golden vectors in ``tests/test_oracle_golden.py``.
2. ctypes access to ``oracle/_build/liboracle.so`` (``paged_oracle.c``): the
   f32 / f64 restatement of the reference attention and the byte-exact
   append / gather / copy / swap loops, plus a numpy restatement of
   ``vasr-models/src/model/attention.rs`` used to cross-check the C code.
"""
from __future__ import annotations

import ctypes
import math
import subprocess
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional

import numpy as np

PAD_SLOT_ID = -1  # vasr-paged-attn/src/paged_kv_cache.rs:7
ORACLE_DIR = Path(__file__).resolve().parent
ORACLE_SO = ORACLE_DIR / "_build" / "liboracle.so"


class OracleError(ValueError):
    """Mirrors a candle_core::bail! of the reference."""


# ===================================================== paged_kv_cache.rs
def cumulative_seqlens_from_lengths(lengths):
    """paged_kv_cache.rs:58-72 (u32 cumulative sums with overflow checks)."""
    out, total = [0], 0
    for n in lengths:
        if n > 0xFFFFFFFF:
            raise OracleError(f"sequence length overflows u32: {n}")
        total += n
        if total > 0xFFFFFFFF:
            raise OracleError("cumulative sequence length overflow")
        out.append(total)
    return out


def slot_for_block_table_position(block_tables, block_size, num_blocks, seq, position):
    """paged_kv_cache.rs:74-103."""
    if seq >= len(block_tables):
        raise OracleError(f"missing block table for sequence {seq}")
    table = block_tables[seq]
    block_idx, offset = divmod(position, block_size)
    if block_idx >= len(table):
        raise OracleError("missing block table entry")
    block_id = table[block_idx]
    if block_id >= num_blocks:
        raise OracleError(f"block id exceeds paged cache capacity: block_id={block_id} num_blocks={num_blocks}")
    return block_id * block_size + offset


@dataclass
class FlashParamsRef:
    """vasr-paged-attn/src/flash.rs:20-43."""
    max_q: int
    cumulative_seqlens_q: Optional[list]
    max_k: int
    cumulative_seqlens_k: Optional[list]
    causal: bool


def flash_params_new_prefill(max_q, cu_q, max_k, cu_k, causal):
    if max_q is None or max_k is None or max_q > 0xFFFFFFFF or max_k > 0xFFFFFFFF:
        return None
    return FlashParamsRef(max_q, cu_q, max_k, cu_k, causal)


def build_varlen_metadata(query_lens, kv_lens):
    """paged_kv_cache.rs:105-146."""
    cu_q = cumulative_seqlens_from_lengths(query_lens) if query_lens is not None else None
    cu_kv = cumulative_seqlens_from_lengths(kv_lens) if kv_lens is not None else None
    max_q = max(query_lens, default=0) if query_lens is not None else None
    max_kv = max(kv_lens, default=0) if kv_lens is not None else None
    causal = query_lens is not None and any(n > 1 for n in query_lens)
    return flash_params_new_prefill(max_q, cu_q, max_kv, cu_kv, causal), cu_q, cu_kv, max_q, max_kv


@dataclass
class MetadataRef:
    """paged_kv_cache.rs:22-38 (tensors as host lists)."""
    slot_mapping: list
    block_tables: list  # list of rows
    context_lens: list
    max_context_len: int
    token_attention_mask: Optional[list] = None
    prefill_causal_only: bool = False
    query_lens: Optional[list] = None
    kv_lens: Optional[list] = None
    prefill_flash_params: Optional[FlashParamsRef] = None
    cu_seqlens_q: Optional[list] = None
    cu_seqlens_kv: Optional[list] = None
    max_query_len: Optional[int] = None
    max_kv_len: Optional[int] = None

    def flash_params(self, causal):
        """paged_kv_cache.rs:45-55."""
        if self.prefill_flash_params is not None:
            return self.prefill_flash_params
        return flash_params_new_prefill(self.max_query_len, self.cu_seqlens_q, self.max_kv_len,
                                        self.cu_seqlens_kv, causal)


def _pad_tables(block_tables, width):
    return [list(t) + [0] * (width - len(t)) for t in block_tables]


@dataclass
class PagedKvCacheRef:
    """Restatement of PagedKvCache (paged_kv_cache.rs:9-20, 148-1070), host side only."""
    num_layers: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    num_blocks: int
    num_blocks_per_sequence: int
    batch_size: int
    max_tokens_per_sequence: int
    dtype_bytes: int
    max_tokens: int = field(init=False)

    def __post_init__(self):
        # paged_kv_cache.rs:241-283
        for name in ("num_layers", "num_kv_heads", "head_dim", "block_size", "batch_size",
                     "max_tokens_per_sequence", "num_blocks"):
            if getattr(self, name) == 0:
                raise OracleError(f"paged kv cache requires non-zero {name}")
        if self.dtype_bytes == 0 or 16 % self.dtype_bytes != 0:
            raise OracleError("unsupported paged kv cache dtype")
        if self.head_dim % self.key_pack != 0:
            raise OracleError("head_dim must be divisible by key cache pack size")
        self.max_tokens = self.num_blocks * self.block_size

    @property
    def key_pack(self):
        return 16 // self.dtype_bytes

    @classmethod
    def new(cls, num_layers, num_kv_heads, head_dim, block_size, max_tokens, dtype_bytes=4):
        return cls.new_batched(num_layers, num_kv_heads, head_dim, block_size, 1, max_tokens, dtype_bytes)

    @classmethod
    def new_batched(cls, num_layers, num_kv_heads, head_dim, block_size, batch_size,
                    max_tokens_per_sequence, dtype_bytes=4):
        nbps = -(-max_tokens_per_sequence // block_size)
        return cls(num_layers, num_kv_heads, head_dim, block_size, batch_size * nbps, nbps,
                   batch_size, max_tokens_per_sequence, dtype_bytes)

    @classmethod
    def new_pool(cls, num_layers, num_kv_heads, head_dim, block_size, num_blocks, dtype_bytes=4):
        return cls(num_layers, num_kv_heads, head_dim, block_size, num_blocks, num_blocks, 1,
                   num_blocks * block_size, dtype_bytes)

    # layout (paged_kv_cache.rs:285-294)
    @property
    def key_shape(self):
        x = self.key_pack
        return (self.num_blocks, self.num_kv_heads, self.head_dim // x, self.block_size, x)

    @property
    def value_shape(self):
        return (self.num_blocks, self.num_kv_heads, self.head_dim, self.block_size)

    def estimated_bytes(self):
        return 2 * self.num_layers * math.prod(self.value_shape) * self.dtype_bytes

    def block_table_host(self):
        return list(range(self.num_blocks))

    def slot_for_position(self, position):
        return self.slot_for_sequence_position(0, position)

    def slot_for_sequence_position(self, sequence, position):
        """paged_kv_cache.rs:356-378."""
        if sequence >= self.batch_size:
            raise OracleError("sequence exceeds paged kv cache batch")
        if position >= self.max_tokens_per_sequence:
            raise OracleError("position exceeds paged kv cache capacity")
        return sequence * self.num_blocks_per_sequence * self.block_size + position

    def slot_mapping_for_range(self, start, length):
        """paged_kv_cache.rs:380-399."""
        if start + length > self.max_tokens:
            raise OracleError("slot range exceeds paged kv cache capacity")
        return [self.slot_for_position(p) for p in range(start, start + length)]

    def block_tables_tensor(self):
        return [self.block_table_host()]

    def block_tables_tensor_for_batch(self, batch):
        if batch > self.batch_size:
            raise OracleError("requested block table batch exceeds cache batch")
        n = self.num_blocks_per_sequence
        flat = self.block_table_host()[: batch * n]
        return [flat[i * n:(i + 1) * n] for i in range(batch)]

    def context_lens_tensor(self, context_len):
        if context_len > self.max_tokens:
            raise OracleError("context length exceeds paged kv cache capacity")
        return [context_len]

    def input_metadata_for_range(self, start, length, context_len):
        """paged_kv_cache.rs:439-466."""
        fp, cu_q, cu_kv, mq, mk = build_varlen_metadata([length], [context_len])
        return MetadataRef(self.slot_mapping_for_range(start, length), self.block_tables_tensor(),
                           self.context_lens_tensor(context_len), context_len, None, False,
                           [length], [context_len], fp, cu_q, cu_kv, mq, mk)

    def input_metadata_for_batch_ranges(self, starts, length, context_lens):
        """paged_kv_cache.rs:468-545."""
        batch = len(starts)
        if batch == 0:
            raise OracleError("paged metadata batch must be non-empty")
        if len(context_lens) != batch or batch > self.batch_size:
            raise OracleError("context_lens batch mismatch")
        slots = []
        for seq, start in enumerate(starts):
            if start + length > self.max_tokens_per_sequence:
                raise OracleError("slot range exceeds paged kv cache sequence capacity")
            slots += [self.slot_for_sequence_position(seq, p) for p in range(start, start + length)]
        for c in context_lens:
            if c > self.max_tokens_per_sequence:
                raise OracleError("context length exceeds paged kv cache sequence capacity")
        fp, cu_q, cu_kv, mq, mk = build_varlen_metadata([length] * batch, list(context_lens))
        return MetadataRef(slots, self.block_tables_tensor_for_batch(batch), list(context_lens),
                           max(context_lens), None, False, [length] * batch, list(context_lens),
                           fp, cu_q, cu_kv, mq, mk)

    def input_metadata_from_block_tables(self, block_tables, starts, length, context_lens):
        """paged_kv_cache.rs:547-649."""
        batch = len(block_tables)
        if batch == 0:
            raise OracleError("paged metadata batch must be non-empty")
        if len(starts) != batch or len(context_lens) != batch:
            raise OracleError("paged metadata batch mismatch")
        max_blocks = max((len(t) for t in block_tables), default=0)
        if max_blocks == 0:
            raise OracleError("paged metadata requires at least one block per sequence")
        slots = []
        for seq in range(batch):
            for p in range(starts[seq], starts[seq] + length):
                slots.append(slot_for_block_table_position(block_tables, self.block_size,
                                                           self.num_blocks, seq, p))
        fp, cu_q, cu_kv, mq, mk = build_varlen_metadata([length] * batch, list(context_lens))
        return MetadataRef(slots, _pad_tables(block_tables, max_blocks), list(context_lens),
                           max(context_lens), None, False, [length] * batch, list(context_lens),
                           fp, cu_q, cu_kv, mq, mk)

    def input_metadata_from_attention_masks(self, block_tables, attention_masks):
        """paged_kv_cache.rs:651-773."""
        batch = len(attention_masks)
        if batch == 0:
            raise OracleError("paged metadata batch must be non-empty")
        if len(block_tables) != batch:
            raise OracleError("paged metadata batch mismatch")
        seq_len = len(attention_masks[0])
        if seq_len == 0:
            raise OracleError("attention mask rows must be non-empty")
        max_blocks = max((len(t) for t in block_tables), default=0)
        if max_blocks == 0:
            raise OracleError("paged metadata requires at least one block per sequence")
        slots, qlens = [], []
        for seq, row in enumerate(attention_masks):
            if len(row) != seq_len:
                raise OracleError("attention_mask row len mismatch")
            n = 0
            for p, m in enumerate(row):
                if m == 0:
                    slots.append(PAD_SLOT_ID)
                    continue
                slots.append(slot_for_block_table_position(block_tables, self.block_size,
                                                           self.num_blocks, seq, p))
                n += 1
            qlens.append(n)
        fp, cu_q, cu_kv, mq, mk = build_varlen_metadata(qlens, list(qlens))
        return MetadataRef(slots, _pad_tables(block_tables, max_blocks), list(qlens), max(qlens),
                           [list(r) for r in attention_masks], all(n == seq_len for n in qlens),
                           list(qlens), list(qlens), fp, cu_q, cu_kv, mq, mk)

    def input_metadata_from_query_lens(self, block_tables, query_lens):
        """paged_kv_cache.rs:775-869."""
        batch = len(query_lens)
        if batch == 0:
            raise OracleError("paged metadata batch must be non-empty")
        if len(block_tables) != batch:
            raise OracleError("paged metadata batch mismatch")
        max_blocks = max((len(t) for t in block_tables), default=0)
        if max_blocks == 0:
            raise OracleError("paged metadata requires at least one block per sequence")
        if any(n == 0 for n in query_lens):
            raise OracleError("packed prefill query length must be non-zero")
        slots = []
        for seq, n in enumerate(query_lens):
            for p in range(n):
                slots.append(slot_for_block_table_position(block_tables, self.block_size,
                                                           self.num_blocks, seq, p))
            if len(block_tables[seq]) < -(-n // self.block_size):
                raise OracleError("paged block table too short for packed prefill")
        fp, cu_q, cu_kv, mq, mk = build_varlen_metadata(list(query_lens), list(query_lens))
        return MetadataRef(slots, _pad_tables(block_tables, max_blocks), list(query_lens),
                           max(query_lens), None, True, list(query_lens), list(query_lens), fp,
                           cu_q, cu_kv, mq, mk)

    def decode_metadata_for_steps(self, prompt_len, steps):
        """paged_kv_cache.rs:871-922."""
        if prompt_len + steps > self.max_tokens:
            raise OracleError("decode metadata range exceeds paged kv cache capacity")
        out = []
        for step in range(steps):
            out.append(MetadataRef([self.slot_for_position(prompt_len + step)], self.block_tables_tensor(),
                                   [prompt_len + step + 1], prompt_len + step + 1))
        return out

    def decode_metadata_for_batch_steps(self, block_tables, prompt_lens, steps, cuda_graph=False):
        """paged_kv_cache.rs:924-1044 (``cuda_graph`` = the cuda-graph feature's column bucket)."""
        batch = len(block_tables)
        if batch == 0:
            raise OracleError("paged batch decode metadata requires at least one sequence")
        if len(prompt_lens) != batch:
            raise OracleError("paged batch decode metadata mismatch")
        raw = max((len(t) for t in block_tables), default=0)
        if raw == 0:
            raise OracleError("paged batch decode metadata requires at least one block per sequence")
        width = bucket_block_table_cols(raw, self.block_size) if cuda_graph else raw
        tables = _pad_tables(block_tables, width)
        out = []
        for step in range(steps):
            slots, ctxs = [], []
            for seq in range(batch):
                pos = prompt_lens[seq] + step
                if pos + 1 > self.max_tokens_per_sequence:
                    raise OracleError("batch decode context length exceeds paged kv cache sequence capacity")
                slots.append(slot_for_block_table_position(block_tables, self.block_size,
                                                           self.num_blocks, seq, pos))
                ctxs.append(pos + 1)
            out.append(MetadataRef(slots, tables, ctxs, max(ctxs)))
        return out

    def decode_metadata_for_batch_step(self, block_tables, prompt_lens, step, cuda_graph=False):
        """paged_kv_cache.rs:1046-1059."""
        return self.decode_metadata_for_batch_steps(block_tables, prompt_lens, step + 1, cuda_graph)[step]


# ================================================== paged_cache_runtime.rs
def bytes_per_paged_block(num_layers, num_kv_heads, head_dim, block_size, dtype_bytes):
    """paged_cache_runtime.rs:46-71."""
    if 0 in (num_layers, num_kv_heads, head_dim, block_size):
        raise OracleError("paged block sizing requires non-zero layer/head/block parameters")
    if dtype_bytes == 0 or 16 % dtype_bytes != 0:
        raise OracleError("unsupported paged kv cache dtype")
    return num_layers * num_kv_heads * head_dim * block_size * 2 * dtype_bytes


def blocks_for_byte_budget(byte_budget, bytes_per_block):
    """paged_cache_runtime.rs:74-86 (+1 for the null block)."""
    if bytes_per_block == 0:
        raise OracleError("paged block byte size must be non-zero")
    n = byte_budget // bytes_per_block + 1
    if n <= 1:
        raise OracleError("paged KV byte budget is too small for one block")
    return n


class PagedBlockManagerRef:
    """paged_cache_runtime.rs:217-371: FIFO free list of 1..num_blocks, block 0 reserved."""

    def __init__(self, num_blocks, block_size):
        self.block_size = block_size
        self.free = list(range(1, num_blocks))
        self.request_blocks: dict[int, list[int]] = {}

    def free_blocks(self):
        return len(self.free)

    def blocks_for_request(self, rid):
        return len(self.request_blocks.get(rid, []))

    def slots_available_for(self, rid, num_tokens):
        need = max(0, -(-num_tokens // self.block_size) - self.blocks_for_request(rid))
        return need <= len(self.free)

    def try_allocate_slots(self, rid, num_tokens):
        need = max(0, -(-num_tokens // self.block_size) - self.blocks_for_request(rid))
        if need == 0:
            return True
        if need > len(self.free):
            return False
        ids = self.request_blocks.setdefault(rid, [])
        for _ in range(need):
            ids.append(self.free.pop(0))
        return True

    def allocate_slots(self, rid, num_tokens):
        if not self.try_allocate_slots(rid, num_tokens):
            raise OracleError("paged KV cache exhausted")

    def trim_request_to_num_tokens(self, rid, num_tokens):
        keep = -(-num_tokens // self.block_size)
        ids = self.request_blocks.get(rid)
        if ids is None or keep >= len(ids):
            return
        removed = ids[keep:]
        del ids[keep:]
        for b in reversed(removed):
            if b != 0:
                self.free.append(b)

    def free_request(self, rid):
        ids = self.request_blocks.pop(rid, None)
        if ids is not None:
            for b in reversed(ids):
                if b != 0:
                    self.free.append(b)

    def block_ids(self, rid):
        if rid not in self.request_blocks:
            raise OracleError(f"paged KV request has no allocated blocks: request_id={rid}")
        return list(self.request_blocks[rid])


def can_admit_with_projected_kv(block_size, kv_block_capacity, prompt_len, projected_used_blocks,
                                projected_running):
    """vasr-models/src/inference/batch_scheduler.rs:100-113."""
    return projected_used_blocks + -(-prompt_len // block_size) + max(projected_running, 1) <= kv_block_capacity


# ========================================================= cuda_graph.rs
CUDA_GRAPH_CONTEXT_BUCKET_TOKENS = 256
CUDA_DECODE_GRAPH_MAX_BATCH = 256


def cuda_graph_batch_bucket(actual, max_batch):
    """cuda_graph.rs:28-40."""
    if actual == 0 or max_batch == 0 or actual > max_batch:
        return None
    b = {1: 1, 2: 2, 3: 4, 4: 4}.get(actual)
    if b is None:
        b = 8 if actual <= 8 else -(-actual // 16) * 16
    return min(b, max_batch)


def cuda_graph_prewarm_batch_limit(max_batch):
    return min(max_batch, CUDA_DECODE_GRAPH_MAX_BATCH)


def cuda_graph_batch_buckets(max_batch):
    """cuda_graph.rs:42-62."""
    m = cuda_graph_prewarm_batch_limit(max_batch)
    if m == 0:
        return []
    out = [b for b in (1, 2, 4, 8) if b <= m]
    b = 16
    while b <= m:
        out.append(b)
        b += 16
    if out[-1] != m:
        out.append(m)
    return out


def cuda_graph_block_bucket(block_size):
    return max(1, -(-CUDA_GRAPH_CONTEXT_BUCKET_TOKENS // block_size))


def bucket_block_table_cols(blocks, block_size):
    """cuda_graph.rs:70-76."""
    bb = cuda_graph_block_bucket(block_size)
    if blocks == 0:
        return bb
    return max(1 << (blocks - 1).bit_length(), bb)


def pad_decode_batch_to_max(max_batch, input_ids, slot_mapping, context_lens, block_tables, cols):
    """cuda_graph.rs:373-486 on host lists: zero ids/slots, context 1, zero table rows;
    real rows are widened by repeating their last block id."""
    n = len(input_ids)
    if n == 0 or n > max_batch:
        raise OracleError("actual batch exceeds cuda graph max batch")
    meta_cols = max(len(r) for r in block_tables)
    if meta_cols > cols:
        raise OracleError("cannot pad block tables down")
    tables = [list(r) + [r[-1]] * (cols - len(r)) if r else [0] * cols for r in block_tables]
    pad = max_batch - n
    return (list(input_ids) + [0] * pad, list(slot_mapping) + [0] * pad,
            list(context_lens) + [1] * pad, tables + [[0] * cols for _ in range(pad)])


# =========================================== attention.rs (numpy restatement)
# ================================================ fp8 E4M3 (OCP "e4m3fn") pages
def _fp8_table():
    """Values of the bytes 0x00..0x7E: sign 0, 4-bit exponent (bias 7), 3-bit
    mantissa; exponent 0 is subnormal (m/8 * 2^-6); 0x7F is NaN (no infinities)."""
    vals = []
    for b in range(0x7F):
        e, m = b >> 3, b & 7
        vals.append((m / 8.0) * 2.0 ** -6 if e == 0 else (1 + m / 8.0) * 2.0 ** (e - 7))
    return np.array(vals, np.float64)


_FP8_POS = _fp8_table()


def fp8_e4m3_decode(b) -> np.ndarray:
    """Bytes -> f32 values (NaN for 0x7F / 0xFF)."""
    b = np.asarray(b, np.uint8)
    mag = b & 0x7F
    v = np.where(mag == 0x7F, np.nan, _FP8_POS[np.minimum(mag, 0x7E)])
    return np.where(b & 0x80, -v, v).astype(np.float32)


def fp8_e4m3_encode(x) -> np.ndarray:
    """f32 -> bytes, round to nearest (ties to the even mantissa), magnitudes
    above the largest finite value (448) saturate to it, NaN -> 0x7F."""
    x = np.asarray(x, np.float32)
    a = np.abs(x.astype(np.float64))
    hi = np.clip(np.searchsorted(_FP8_POS, a, side="left"), 0, 0x7E)  # first value >= a
    lo = np.maximum(hi - 1, 0)
    d_hi, d_lo = _FP8_POS[hi] - a, a - _FP8_POS[lo]
    pick_lo = (d_lo < d_hi) | ((d_lo == d_hi) & (lo % 2 == 0))
    code = np.where(pick_lo, lo, hi)
    code = np.where(a >= _FP8_POS[-1], 0x7E, code)
    code = np.where(np.isnan(x), 0x7F, code).astype(np.uint8)
    return np.where(np.signbit(x), code | 0x80, code).astype(np.uint8)


def reshape_and_cache_fp8(key, value, key_cache, value_cache, slots, block_size, k_scale, v_scale):
    """The fp8 append: cache byte = encode(value / scale) in f32 (IEEE division)."""
    kq = fp8_e4m3_encode(np.asarray(key, np.float32) / np.float32(k_scale))
    vq = fp8_e4m3_encode(np.asarray(value, np.float32) / np.float32(v_scale))
    t, hkv, d = kq.shape
    for i in range(t):
        s = int(slots[i])
        if s < 0:
            continue
        blk, off = s // block_size, s % block_size
        key_cache[blk, :, :, off, :] = kq[i].reshape(hkv, d // 16, 16)
        value_cache[blk, :, :, off] = vq[i]


def gather_kv_cache_fp8(key_cache, value_cache, block_tables, cu, num_kv_heads, head_dim,
                        block_size, k_scale, v_scale):
    """gather_kv_cache over fp8 pages: the byte gather, then decode(byte) * scale in f32
    (the caller rounds to its out dtype)."""
    kb, vb = gather_kv_cache(key_cache, value_cache, block_tables, cu, num_kv_heads, head_dim,
                             block_size)
    return (fp8_e4m3_decode(kb) * np.float32(k_scale), fp8_e4m3_decode(vb) * np.float32(v_scale))


# ============================================== device decode loop (host restatement)
def decode_step_prepare(state, eos_ids, block_tables, block_table_lens, block_size, num_blocks):
    """One decode step's token feedback + metadata, as the reference host loop does it.

    Restates paged_batch_engine.rs:634-676 (a row whose fed token is an EOS id
    becomes finished; otherwise the token is recorded), the decode metadata of
    paged_kv_cache.rs:924-1059 (position = prompt_len + step, context =
    position + 1, slot by slot_for_block_table_position :74-103) and, for
    finished rows, the padding rows of cuda_graph.rs:373-486 (token 0,
    position 0, slot 0, context 1). ``state`` holds numpy arrays prompt_lens,
    next_ids, finished (bool), generated, history [B, cols] and the int
    ``step``; it is updated in place. Returns (input_ids, positions,
    slot_mapping, context_lens, slot_errors) where slot_errors counts rows
    whose table was too short (slot -1 there).
    """
    b = len(state["prompt_lens"])
    ids = np.zeros(b, np.int64)
    pos = np.zeros(b, np.int64)
    slots = np.zeros(b, np.int64)
    ctx = np.ones(b, np.uint32)
    errors = 0
    hist = state["history"]
    for i in range(b):
        if not state["finished"][i]:
            tok = int(state["next_ids"][i])
            if tok in set(int(e) for e in eos_ids):
                state["finished"][i] = True
            else:
                g = int(state["generated"][i])
                if hist is not None and g < hist.shape[1]:
                    hist[i, g] = tok
                state["generated"][i] = g + 1
                p = int(state["prompt_lens"][i]) + state["step"]
                n = int(block_table_lens[i]) if block_table_lens is not None else block_tables.shape[1]
                table = [int(x) for x in block_tables[i, :n]]
                try:
                    slots[i] = slot_for_block_table_position([table], block_size, num_blocks, 0, p)
                except OracleError:
                    slots[i] = PAD_SLOT_ID
                    errors += 1
                ids[i], pos[i], ctx[i] = tok, p, p + 1
                continue
        # finished (now or before): padding row
    return ids, pos, slots, ctx, errors


def greedy_argmax(logits, finished=None):
    """argmax_token_ids_from_logits (generation.rs:443-460): first index of the row maximum.

    NaN never wins and a row without a value above -inf gives 0; rows with
    finished set are left out (None in the result).
    """
    out = []
    for i, row in enumerate(np.asarray(logits, np.float64)):
        if finished is not None and finished[i]:
            out.append(None)
            continue
        r = np.where(np.isnan(row), -np.inf, row)
        m = r.max()
        out.append(0 if not m > -np.inf else int(np.argmax(r == m)))
    return out


def repeat_kv(x, n_rep):
    """attention.rs:12-21: (b, kvh, s, d) -> (b, kvh * n_rep, s, d), head h <- kv head h // n_rep."""
    if n_rep == 1:
        return x
    b, kvh, s, d = x.shape
    return np.broadcast_to(x[:, :, None], (b, kvh, n_rep, s, d)).reshape(b, kvh * n_rep, s, d)


def make_causal_mask(batch, seq_len, dtype=np.float32):
    """attention.rs:31-76 without a padding mask: 0 allowed, f32::MIN masked."""
    allowed = np.tril(np.ones((seq_len, seq_len), dtype=bool))
    m = np.where(allowed, 0.0, np.finfo(np.float32).min).astype(dtype)
    return np.broadcast_to(m, (batch, 1, seq_len, seq_len))


def make_causal_mask_cached(batch, cache_len, new_len, dtype=np.float32):
    """attention.rs:86-149: key j visible to new query q iff j <= cache_len + q."""
    total = cache_len + new_len
    kv = np.arange(total)[None, :]
    q = np.arange(cache_len, total)[:, None]
    m = np.where(kv <= q, 0.0, np.finfo(np.float32).min).astype(dtype)
    return np.broadcast_to(m, (batch, 1, new_len, total))


def softmax_last_dim(w):
    m = w.max(axis=-1, keepdims=True)
    e = np.exp(w - m)
    return e / e.sum(axis=-1, keepdims=True)


def run_single_sequence_attention(q, k, v, mask, scale, causal, n_kv_groups, dtype=np.float64):
    """attention.rs:243-286 (eager path): repeat_kv -> q k^T * scale (+mask) -> softmax -> . v."""
    q = q.astype(dtype)
    k = repeat_kv(k, n_kv_groups).astype(dtype)
    v = repeat_kv(v, n_kv_groups).astype(dtype)
    w = (q @ np.swapaxes(k, 2, 3)) * dtype(scale)
    if mask is not None:
        w = w + mask.astype(dtype)
    elif causal and q.shape[2] > 1:
        w = w + make_causal_mask(q.shape[0], q.shape[2], dtype)
    return softmax_last_dim(w) @ v


def packed_varlen_attention(q, k, v, cu_q, cu_k, scale, causal, n_kv_groups, dtype=np.float64):
    """attention.rs:379-536 (per-row branch): q (B, H, S, D) right-padded; k, v (1, KVH, total, D)."""
    batch, heads, seq_len, d = q.shape
    rows = []
    for r in range(batch):
        ql = cu_q[r + 1] - cu_q[r]
        kl = cu_k[r + 1] - cu_k[r]
        o = run_single_sequence_attention(q[r:r + 1, :, :ql], k[:, :, cu_k[r]:cu_k[r] + kl],
                                          v[:, :, cu_k[r]:cu_k[r] + kl], None, scale, causal,
                                          n_kv_groups, dtype)
        pad = np.zeros((1, heads, seq_len - ql, d), dtype=o.dtype)
        rows.append(np.concatenate([o, pad], axis=2))
    return np.concatenate(rows, axis=0)


# ============================================ C oracle (paged_oracle.c)
_SO: Optional[ctypes.CDLL] = None


def build_c_oracle() -> Path:
    if not ORACLE_SO.exists() or ORACLE_SO.stat().st_mtime < (ORACLE_DIR / "paged_oracle.c").stat().st_mtime:
        subprocess.run(["make", "-C", str(ORACLE_DIR)], check=True, capture_output=True)
    return ORACLE_SO


def c_oracle() -> ctypes.CDLL:
    global _SO
    if _SO is None:
        build_c_oracle()
        so = ctypes.CDLL(str(ORACLE_SO))
        vp, i32, i64, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
        so.oracle_reshape_and_cache.argtypes = [vp, vp, vp, vp, vp, i64, i32, i32, i32, i64, i64, i64, i32]
        so.oracle_gather_kv_cache.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32]
        so.oracle_copy_blocks.argtypes = [ctypes.POINTER(vp), ctypes.POINTER(vp), i32, vp, i64, i64]
        so.oracle_swap_blocks.argtypes = [vp, vp, vp, i64, i64]
        so.oracle_paged_attention_f32.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32,
                                                  i32, i32, f32, f32, i32, i32]
        so.oracle_prefill_varlen_f32.argtypes = [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32,
                                                 i32, i32, f32, f32, i32, i32]
        so.oracle_max_threads.restype = i32
        _SO = so
    return _SO


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def reshape_and_cache(key, value, key_cache, value_cache, slots, block_size):
    """In-place scatter on numpy arrays of any 2- or 4-byte dtype (bit-exact)."""
    t, h, d = key.shape
    c_oracle().oracle_reshape_and_cache(_ptr(key), _ptr(value), _ptr(key_cache), _ptr(value_cache),
                                        _ptr(slots), t, h, d, block_size, key_cache.shape[0],
                                        h * d, h * d, key.itemsize)


def gather_kv_cache(key_cache, value_cache, block_tables, cu, num_kv_heads, head_dim, block_size):
    total = int(cu[-1])
    k = np.empty((total, num_kv_heads, head_dim), dtype=key_cache.dtype)
    v = np.empty_like(k)
    c_oracle().oracle_gather_kv_cache(_ptr(k), _ptr(v), _ptr(key_cache), _ptr(value_cache),
                                      _ptr(block_tables), _ptr(cu), block_tables.shape[0],
                                      block_tables.shape[1], num_kv_heads, head_dim, block_size,
                                      key_cache.itemsize)
    return k, v


def copy_blocks(key_caches, value_caches, pairs):
    n = len(key_caches)
    kp = (ctypes.c_void_p * n)(*[c.ctypes.data for c in key_caches])
    vp = (ctypes.c_void_p * n)(*[c.ctypes.data for c in value_caches])
    bb = key_caches[0][0].nbytes
    c_oracle().oracle_copy_blocks(kp, vp, n, _ptr(pairs), pairs.shape[0], bb)


def swap_blocks(dst, src, pairs):
    c_oracle().oracle_swap_blocks(_ptr(dst), _ptr(src), _ptr(pairs), pairs.shape[0], src[0].nbytes)


def paged_attention(q, key_cache, value_cache, block_tables, context_lens, scale, softcap=1.0,
                    use_double=True, threads=0):
    """f32 decode attention over f32 values in a paged layout (key pack = key_cache.shape[4])."""
    b, hq, d = q.shape
    hkv, bs = value_cache.shape[1], value_cache.shape[3]
    out = np.empty((b, hq, d), dtype=np.float32)
    c_oracle().oracle_paged_attention_f32(_ptr(out), _ptr(q), _ptr(key_cache), _ptr(value_cache),
                                          _ptr(block_tables), _ptr(context_lens), b, hq, hkv, d, bs,
                                          key_cache.shape[4], block_tables.shape[1], scale, softcap,
                                          int(use_double), threads)
    return out


def prefill_varlen(q, key_cache, value_cache, block_tables, context_lens, cu_q, scale, softcap=1.0,
                   use_double=True, threads=0):
    t, hq, d = q.shape
    hkv, bs = value_cache.shape[1], value_cache.shape[3]
    out = np.empty((t, hq, d), dtype=np.float32)
    c_oracle().oracle_prefill_varlen_f32(_ptr(out), _ptr(q), _ptr(key_cache), _ptr(value_cache),
                                         _ptr(block_tables), _ptr(context_lens), _ptr(cu_q),
                                         block_tables.shape[0], hq, hkv, d, bs, key_cache.shape[4],
                                         block_tables.shape[1], scale, softcap, int(use_double), threads)
    return out


def max_threads() -> int:
    return int(c_oracle().oracle_max_threads())


# ============================== fused q/k RMSNorm + RoPE (thinker_text.rs:1041-1068)
def qk_norm_rope_ref(qkv_bits, q_w_bits, k_w_bits, eps, cos, sin, positions, num_heads, num_kv_heads,
                     head_dim=128):
    """bf16 restatement of per-head RMSNorm (x * rsqrt(mean(x^2) + eps) * w in f32, rounded)
    followed by rotate-half RoPE in f32 on the rounded values (rounded again).
    Returns (q_bits [T, Hq, D], k_bits [T, Hkv, D], v_bits [T, Hkv, D])."""
    t = qkv_bits.shape[0]
    x = bf16_bits_to_f32(qkv_bits).reshape(t, num_heads + 2 * num_kv_heads, head_dim)
    qk = x[:, :num_heads + num_kv_heads].astype(np.float64)
    w = np.concatenate([np.broadcast_to(bf16_bits_to_f32(q_w_bits), (num_heads, head_dim)),
                        np.broadcast_to(bf16_bits_to_f32(k_w_bits), (num_kv_heads, head_dim))])
    inv = 1.0 / np.sqrt((qk ** 2).mean(-1, keepdims=True) + eps)
    n = bf16_bits_to_f32(f32_to_bf16_bits((qk * inv * w).astype(np.float32))).astype(np.float64)
    half = head_dim // 2
    c = cos[positions][:, None, :].astype(np.float64)
    s = sin[positions][:, None, :].astype(np.float64)
    x1, x2 = n[..., :half], n[..., half:]
    r = np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1).astype(np.float32)
    rb = f32_to_bf16_bits(r)
    v_bits = qkv_bits.reshape(t, num_heads + 2 * num_kv_heads, head_dim)[:, num_heads + num_kv_heads:]
    return rb[:, :num_heads], rb[:, num_heads:], np.ascontiguousarray(v_bits)


# ------------------------------------------------------------ bf16 helpers
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit pattern (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r = np.where(nan, np.uint16(0x7FC0), r)
    return r
