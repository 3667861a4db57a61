"""Parity of the sm_100a kernels against the CPU oracle, called through the C ABI.

Tolerances: append, gather, copy, swap are
bit-exact over the whole pool (unused slots hold a NaN sentinel, so stray
writes are caught); f32 attention <= 1e-4 max abs, bf16 attention <= 2e-2
max abs against the f64 oracle on the same bf16-rounded inputs.
"""
import numpy as np
import pytest
import torch

import paged_ref as ref
from cases import (CONFIG1_CACHED, appended, config1_case, disjoint_block_tables, loguniform_lens,
                   make_decode_case, oracle_decode, uniform_lens)
from vasr_paged_attn import _lib
from vasr_paged_attn import mistralrs_paged_attn as pa

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4
BF16_TOL = 2e-2


def to_dev(bits: np.ndarray, dtype: str, dev) -> torch.Tensor:
    bits = np.ascontiguousarray(bits)
    if dtype == "f32":
        return torch.from_numpy(bits.view(np.float32).copy()).to(dev)
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(dev)


def to_bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.float32:
        return t.contiguous().view(torch.int32).cpu().numpy().view(np.uint32)
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def to_f32(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def upload(case, dev):
    return dict(
        kc=to_dev(case.key_cache, case.dtype, dev),
        vc=to_dev(case.value_cache, case.dtype, dev),
        q=to_dev(case.q, case.dtype, dev),
        k=to_dev(case.k_new, case.dtype, dev),
        v=to_dev(case.v_new, case.dtype, dev),
        slots=torch.from_numpy(case.slots).to(dev),
        bt=torch.from_numpy(case.block_tables.astype(np.int32)).to(dev),
        ctx=torch.from_numpy(case.context_lens.astype(np.int32)).to(dev),
    )


@pytest.fixture(autouse=True)
def _clear_device_error(cuda_device):
    pa.device_error(clear=True)
    yield


# ------------------------------------------------------------------ append
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_append_decode_tokens_bitexact_config1(cuda_device, dtype):
    case = make_decode_case(0, CONFIG1_CACHED, dtype=dtype, num_blocks=512)
    t = upload(case, cuda_device)
    pa.reshape_and_cache(t["k"], t["v"], None, None, t["kc"], t["vc"], t["slots"])
    _, kc_ref, vc_ref = oracle_decode(case)
    assert np.array_equal(to_bits(t["kc"]), kc_ref)
    assert np.array_equal(to_bits(t["vc"]), vc_ref)
    assert pa.device_error() == 0


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("block_size", [8, 16, 32])
def test_append_prefill_chunks_bitexact(cuda_device, dtype, block_size):
    """Config-3 shaped: packed 256-token chunks of several ragged prompts, shuffled pages, pads."""
    rng = np.random.default_rng(7)
    lens = [100, 257, 31, 256, 1]
    nb = 200
    hkv, d = 8, 128
    tables = np.zeros((len(lens), 64), np.uint32)
    perm = rng.permutation(np.arange(1, nb))
    off = 0
    slots = []
    for i, n in enumerate(lens):
        nblk = -(-n // block_size)
        tables[i, :nblk] = perm[off:off + nblk]
        off += nblk
        pos = np.arange(n)
        slots.append(tables[i, pos // block_size].astype(np.int64) * block_size + pos % block_size)
    slots = np.concatenate(slots)
    slots[[3, 50, 400]] = ref.PAD_SLOT_ID  # padded rows are skipped
    total = len(slots)
    x = 4 if dtype == "f32" else 8
    bits_t = np.uint32 if dtype == "f32" else np.uint16
    kc = np.full((nb, hkv, d // x, block_size, x), 0x7FC1, dtype=bits_t)
    vc = np.full((nb, hkv, d, block_size), 0x7FC1, dtype=bits_t)
    k = rng.integers(0, np.iinfo(bits_t).max, size=(total, hkv, d), dtype=bits_t)
    v = rng.integers(0, np.iinfo(bits_t).max, size=(total, hkv, d), dtype=bits_t)
    tk, tv = to_dev(kc, dtype, cuda_device), to_dev(vc, dtype, cuda_device)
    dk, dv = to_dev(k, dtype, cuda_device), to_dev(v, dtype, cuda_device)
    ds = torch.from_numpy(slots).to(cuda_device)
    for c0 in range(0, total, 256):  # 256-token chunks as in config 3
        c1 = min(total, c0 + 256)
        pa.reshape_and_cache(dk[c0:c1], dv[c0:c1], None, None, tk, tv, ds[c0:c1])
    ref.reshape_and_cache(k, v, kc, vc, slots, block_size)
    assert np.array_equal(to_bits(tk), kc)
    assert np.array_equal(to_bits(tv), vc)


def test_append_strided_token_rows(cuda_device):
    """key/value as slices of a fused [T, (Hq + 2 Hkv) * D] projection (token stride > Hkv * D)."""
    rng = np.random.default_rng(9)
    t_, hq, hkv, d, bs, nb = 40, 16, 8, 128, 16, 16
    fused = torch.randn(t_, (hq + 2 * hkv) * d, device=cuda_device).to(torch.bfloat16)
    k = fused[:, hq * d:(hq + hkv) * d].view(t_, hkv, d)
    v = fused[:, (hq + hkv) * d:].view(t_, hkv, d)
    slots = torch.from_numpy(rng.permutation(nb * bs)[:t_].astype(np.int64)).to(cuda_device)
    kc = torch.zeros(nb, hkv, d // 8, bs, 8, dtype=torch.bfloat16, device=cuda_device)
    vc = torch.zeros(nb, hkv, d, bs, dtype=torch.bfloat16, device=cuda_device)
    pa.reshape_and_cache(k, v, None, None, kc, vc, slots)
    kc_r = np.zeros(tuple(kc.shape), np.uint16)
    vc_r = np.zeros(tuple(vc.shape), np.uint16)
    ref.reshape_and_cache(to_bits(k.contiguous()), to_bits(v.contiguous()), kc_r, vc_r,
                          slots.cpu().numpy(), bs)
    assert np.array_equal(to_bits(kc), kc_r) and np.array_equal(to_bits(vc), vc_r)


def test_append_out_of_range_slot_is_skipped_and_flagged(cuda_device):
    kc = torch.zeros(4, 8, 16, 16, 8, dtype=torch.bfloat16, device=cuda_device)
    vc = torch.zeros(4, 8, 128, 16, dtype=torch.bfloat16, device=cuda_device)
    k = torch.ones(2, 8, 128, dtype=torch.bfloat16, device=cuda_device)
    slots = torch.tensor([3, 4 * 16 + 5], dtype=torch.int64, device=cuda_device)
    pa.reshape_and_cache(k, k, None, None, kc, vc, slots)
    assert pa.device_error() & _lib.DERR_SLOT_RANGE
    assert int((kc != 0).sum()) == 8 * 128  # only the in-range token landed


# ------------------------------------------------------------------ decode
def run_decode(case, t, max_context_len=None, softcap=1.0):
    mcl = int(max_context_len if max_context_len is not None else case.context_lens.max())
    return pa.paged_attention(t["q"], None, None, t["kc"], t["vc"], t["bt"], t["ctx"], None, mcl,
                              case.head_dim ** -0.5, softcap, None)


def test_decode_config1_f32(cuda_device):
    case = config1_case()
    t = upload(case, cuda_device)
    pa.reshape_and_cache(t["k"], t["v"], None, None, t["kc"], t["vc"], t["slots"])
    out = run_decode(case, t)
    exp, _, _ = oracle_decode(case)
    err = np.abs(to_f32(out) - exp).max()
    assert err <= F32_TOL, err
    assert pa.device_error() == 0


@pytest.mark.parametrize("block_size", [8, 16, 32])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_decode_ragged_contexts(cuda_device, dtype, block_size):
    # context edges: 1 token, exactly one page, page + 1, split boundaries (64/128/256 tokens)
    cached = [0, block_size - 1, block_size, 63, 64, 127, 255, 256, 511, 700]
    case = make_decode_case(11, cached, dtype=dtype, block_size=block_size,
                            num_blocks=(2048 // block_size) + 8)
    t = upload(case, cuda_device)
    pa.reshape_and_cache(t["k"], t["v"], None, None, t["kc"], t["vc"], t["slots"])
    out = run_decode(case, t)
    exp, _, _ = oracle_decode(case)
    err = np.abs(to_f32(out) - exp).max()
    assert err <= (F32_TOL if dtype == "f32" else BF16_TOL), err


@pytest.mark.parametrize("gqa", [1, 2, 4])
def test_decode_gqa_groups(cuda_device, gqa):
    case = appended(make_decode_case(5, [33, 300, 999], dtype="bf16", num_heads=8 * gqa, num_kv_heads=8,
                            num_blocks=128))
    t = upload(case, cuda_device)
    out = run_decode(case, t)
    exp, _, _ = oracle_decode(case, after_append=False)
    assert np.abs(to_f32(out) - exp).max() <= BF16_TOL


def test_decode_config2_shapes_bf16(cuda_device):
    """Config 2 attention shapes: 64 sequences, context ~U[200, 1500], bf16."""
    lens = uniform_lens(0, 64, 200, 1500) - 1
    case = make_decode_case(0, lens, dtype="bf16", num_blocks=64 * 94 + 8)
    t = upload(case, cuda_device)
    pa.reshape_and_cache(t["k"], t["v"], None, None, t["kc"], t["vc"], t["slots"])
    out = run_decode(case, t)
    exp, _, _ = oracle_decode(case)
    err = np.abs(to_f32(out) - exp).max()
    assert err <= BF16_TOL, err


def test_decode_more_than_1024_sequences(cuda_device):
    """More than 1024 sequences (a wide grid of split CTAs; the merge counters per (sequence, kv head))."""
    lens = uniform_lens(3, 1100, 1, 60) - 1
    case = make_decode_case(3, lens, dtype="bf16", num_blocks=1100 * 4 + 8)
    t = upload(case, cuda_device)
    pa.reshape_and_cache(t["k"], t["v"], None, None, t["kc"], t["vc"], t["slots"])
    out = run_decode(case, t, max_context_len=512)
    exp, _, _ = oracle_decode(case)
    assert np.abs(to_f32(out) - exp).max() <= BF16_TOL


def test_decode_persistent_many_items_per_cta(cuda_device):
    """Long bound with short true contexts: most splits of the bound are empty and exit at once."""
    lens = loguniform_lens(4, 300, 1, 3000) - 1
    case = make_decode_case(4, np.maximum(lens, 0), dtype="bf16",
                            num_blocks=int(np.maximum(lens, 0).sum() // 16 + 320))
    t = upload(case, cuda_device)
    pa.reshape_and_cache(t["k"], t["v"], None, None, t["kc"], t["vc"], t["slots"])
    out = run_decode(case, t, max_context_len=4096)
    exp, _, _ = oracle_decode(case)
    assert np.abs(to_f32(out) - exp).max() <= BF16_TOL


def test_decode_graph_bucket_upper_bound_and_padded_tables(cuda_device):
    """max_context_len is only a bound (cuda_graph.rs:141); tables padded by repeating the last block."""
    case = appended(make_decode_case(6, [150, 20, 900], dtype="bf16", num_blocks=128, cols=128))
    for i, n in enumerate(case.context_lens):
        nblk = -(-int(n) // 16)
        case.block_tables[i, nblk:] = case.block_tables[i, nblk - 1]
    t = upload(case, cuda_device)
    out = run_decode(case, t, max_context_len=128 * 16)
    exp, _, _ = oracle_decode(case, after_append=False)
    assert np.abs(to_f32(out) - exp).max() <= BF16_TOL
    assert pa.device_error() == 0


def test_decode_dummy_rows_use_null_block(cuda_device):
    """Graph padding rows: slot 0, context 1, all-zero table row (cuda_graph.rs:402-408)."""
    case = make_decode_case(8, [40, 70], dtype="bf16", num_blocks=32)
    pad = 3
    case.q = np.concatenate([case.q, case.q[:1].repeat(pad, 0)])
    case.k_new = np.concatenate([case.k_new, case.k_new[:1].repeat(pad, 0)])
    case.v_new = np.concatenate([case.v_new, case.v_new[:1].repeat(pad, 0)])
    case.slots = np.concatenate([case.slots, np.zeros(pad, np.int64)])
    case.context_lens = np.concatenate([case.context_lens, np.ones(pad, np.uint32)])
    case.block_tables = np.concatenate([case.block_tables,
                                        np.zeros((pad, case.block_tables.shape[1]), np.uint32)])
    t = upload(case, cuda_device)
    pa.reshape_and_cache(t["k"], t["v"], None, None, t["kc"], t["vc"], t["slots"])
    out = to_f32(run_decode(case, t))
    exp, _, _ = oracle_decode(case)
    assert np.abs(out - exp).max() <= BF16_TOL
    assert np.isfinite(out).all()


def test_decode_softcap(cuda_device):
    case = appended(make_decode_case(12, [77, 513], dtype="f32", num_blocks=64))
    t = upload(case, cuda_device)
    out = run_decode(case, t, softcap=5.0)
    exp, _, _ = oracle_decode(case, softcap=5.0, after_append=False)
    assert np.abs(to_f32(out) - exp).max() <= F32_TOL


def test_decode_zero_context_rows_are_zero(cuda_device):
    case = appended(make_decode_case(13, [10, 20], dtype="f32", num_blocks=16))
    t = upload(case, cuda_device)
    t["ctx"][1] = 0
    out = to_f32(run_decode(case, t, max_context_len=64))
    assert (out[1] == 0).all()
    assert np.isfinite(out[0]).all()


def test_decode_repeatable_and_workspace_reuse(cuda_device):
    """Split-K counters reset themselves: repeated calls are bit-identical."""
    lens = loguniform_lens(1, 48, 64, 4096) - 1
    case = appended(make_decode_case(1, lens, dtype="bf16", num_blocks=int(sum(lens) // 16 + 64)))
    t = upload(case, cuda_device)
    outs = [to_bits(run_decode(case, t)) for _ in range(3)]
    assert all(np.array_equal(outs[0], o) for o in outs[1:])
    exp, _, _ = oracle_decode(case, after_append=False)
    assert np.abs(ref.bf16_bits_to_f32(outs[0]) - exp).max() <= BF16_TOL


def test_decode_cuda_graph_capture_and_replay(cuda_device):
    """Append + decode captured once, replayed on new device-resident metadata (cuda_graph.rs:342-369)."""
    case = make_decode_case(14, [100, 200, 300, 400], dtype="bf16", num_blocks=128, cols=32)
    t = upload(case, cuda_device)
    # step 1 runs eagerly; the graph then replays step 2
    pa.reshape_and_cache(t["k"], t["v"], None, None, t["kc"], t["vc"], t["slots"])
    kc1, vc1 = case.key_cache.copy(), case.value_cache.copy()
    ref.reshape_and_cache(case.k_new, case.v_new, kc1, vc1, case.slots, 16)
    mcl = 32 * 16
    need = pa.paged_attention_workspace_bytes(4, 16, 8, 128, 16, mcl, torch.bfloat16)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        pa.reserve_paged_attention_workspace(cuda_device, need, s)
        out = torch.empty(4, 16, 128, dtype=torch.bfloat16, device=cuda_device)
        run_decode(case, t, max_context_len=mcl)  # warm-up
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            pa.reshape_and_cache(t["k"], t["v"], None, None, t["kc"], t["vc"], t["slots"])
            pa.paged_attention(t["q"], None, None, t["kc"], t["vc"], t["bt"], t["ctx"], None, mcl,
                               128 ** -0.5, 1.0, None, out=out)
    torch.cuda.current_stream().wait_stream(s)
    # step 2: next position of every sequence (no page boundary is crossed)
    case.key_cache, case.value_cache = kc1, vc1
    case.slots = case.slots + 1
    case.context_lens = case.context_lens + 1
    t["slots"].copy_(torch.from_numpy(case.slots))
    t["ctx"].copy_(torch.from_numpy(case.context_lens.astype(np.int32)))
    g.replay()
    torch.cuda.synchronize()
    exp, _, _ = oracle_decode(case)
    assert np.abs(to_f32(out) - exp).max() <= BF16_TOL
    del g


def test_decode_block_id_out_of_range_is_flagged(cuda_device):
    case = make_decode_case(15, [30], dtype="f32", num_blocks=8)
    t = upload(case, cuda_device)
    t["bt"][0, 0] = 1000
    run_decode(case, t)
    torch.cuda.synchronize()
    assert pa.device_error() & _lib.DERR_BLOCK_RANGE


# ------------------------------------------------------------------ gather
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_gather_kv_cache_bitexact(cuda_device, dtype):
    case = make_decode_case(16, [1, 15, 16, 17, 300], dtype=dtype, num_blocks=64)
    t = upload(case, cuda_device)
    lens = case.context_lens.astype(np.int64) - 1  # cached tokens only
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint32)
    k, v = pa.gather_kv_cache(t["kc"], t["vc"], None, None, t["bt"],
                              torch.from_numpy(cu.astype(np.int32)).to(cuda_device))
    kr, vr = ref.gather_kv_cache(case.key_cache, case.value_cache, case.block_tables, cu, 8, 128, 16)
    assert np.array_equal(to_bits(k), kr) and np.array_equal(to_bits(v), vr)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("bs,d", [(8, 128), (32, 128), (16, 64), (32, 256)])
def test_gather_kv_cache_page_sizes_bitexact(cuda_device, dtype, bs, d):
    """Every page size and head dim the gather serves, with partial last pages."""
    rng = np.random.default_rng(bs * 1000 + d)
    hkv = 4
    lens = np.array([1, bs - 1, bs, bs + 1, 3 * bs + 5], np.int64)
    blocks = [-(-int(n) // bs) for n in lens]
    nb = sum(blocks) + 2
    tables = disjoint_block_tables(rng, blocks, nb)
    word = np.uint32 if dtype == "f32" else np.uint16
    x = 16 // np.dtype(word).itemsize
    kc = rng.integers(0, np.iinfo(word).max, size=(nb, hkv, d // x, bs, x), dtype=word)
    vc = rng.integers(0, np.iinfo(word).max, size=(nb, hkv, d, bs), dtype=word)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint32)
    k, v = pa.gather_kv_cache(to_dev(kc, dtype, cuda_device), to_dev(vc, dtype, cuda_device), None, None,
                              torch.from_numpy(tables.astype(np.int32)).to(cuda_device),
                              torch.from_numpy(cu.astype(np.int32)).to(cuda_device))
    kr, vr = ref.gather_kv_cache(kc, vc, np.ascontiguousarray(tables), cu, hkv, d, bs)
    assert np.array_equal(to_bits(k), kr) and np.array_equal(to_bits(v), vr)


# -------------------------------------------------------------- block ops
def test_copy_blocks_bitexact_multi_layer(cuda_device):
    rng = np.random.default_rng(17)
    layers, nb = 3, 300
    kcs = [rng.integers(0, 2**16, size=(nb, 8, 16, 16, 8), dtype=np.uint16) for _ in range(layers)]
    vcs = [rng.integers(0, 2**16, size=(nb, 8, 128, 16), dtype=np.uint16) for _ in range(layers)]
    perm = rng.permutation(nb)
    pairs = np.stack([perm[:100], perm[100:200]], axis=1).astype(np.int64)  # disjoint src/dst
    dk = [to_dev(k, "bf16", cuda_device) for k in kcs]
    dv = [to_dev(v, "bf16", cuda_device) for v in vcs]
    pa.copy_blocks(dk, dv, torch.from_numpy(pairs).to(cuda_device))
    ref.copy_blocks(kcs, vcs, pairs)
    for l in range(layers):
        assert np.array_equal(to_bits(dk[l]), kcs[l]) and np.array_equal(to_bits(dv[l]), vcs[l])


def test_swap_blocks_device_host_roundtrip(cuda_device):
    rng = np.random.default_rng(18)
    nb_dev, nb_host = 64, 32
    dev_cache = torch.from_numpy(rng.integers(-2**15, 2**15, size=(nb_dev, 8, 128, 16), dtype=np.int16)
                                 ).view(torch.bfloat16).to(cuda_device)
    host_cache = torch.zeros(nb_host, 8, 128, 16, dtype=torch.bfloat16).pin_memory()
    src = rng.permutation(nb_dev)[:20]
    dst = rng.permutation(nb_host)[:20]
    out_map = torch.from_numpy(np.stack([src, dst], 1).astype(np.int64)).pin_memory()
    pa.swap_blocks(dev_cache, host_cache, out_map)  # evict: device -> pinned host
    torch.cuda.synchronize()
    ref_host = np.zeros((nb_host, 8, 128, 16), np.uint16)
    ref.swap_blocks(ref_host, to_bits(dev_cache), out_map.numpy())
    assert np.array_equal(to_bits(host_cache), ref_host)
    back = torch.zeros_like(dev_cache)
    in_map = torch.from_numpy(np.stack([dst, src], 1).astype(np.int64)).to(cuda_device)
    pa.swap_blocks(host_cache, back, in_map)  # restore: pinned host -> device
    torch.cuda.synchronize()
    for s_ in src:
        assert np.array_equal(to_bits(back[int(s_)]), to_bits(dev_cache[int(s_)]))


def test_swap_rejects_pageable_host_memory(cuda_device):
    dev_cache = torch.zeros(4, 8, 128, 16, dtype=torch.bfloat16, device=cuda_device)
    host_cache = torch.zeros(4, 8, 128, 16, dtype=torch.bfloat16)  # not pinned
    with pytest.raises(_lib.VasrPaError):
        pa.swap_blocks(dev_cache, host_cache, torch.zeros(1, 2, dtype=torch.int64).pin_memory())
