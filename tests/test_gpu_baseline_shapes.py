"""Parity at the shapes the benchmark and the design notes quote (4, 5),
plus the f16 instantiations and the reference's exact call forms, through the C ABI.

* Config 3: every chunk round of the 32-prompt / 256-token-chunk prefill, bf16 and fp8 pages,
  against the oracle's cached causal mask (2e-2).
* Config 4: copy_blocks of 4096 disjoint pairs over 200k-block pools and swap_blocks of 1024
  blocks device <-> pinned host, bit-exact over the whole pools.
* Config 5: decode of 512 sequences with contexts ~log-U[64, 4096] and the graph-bucket table
  width, against the f64 oracle (2e-2).
* f16 decode and f16 tensor-core prefill (2e-2).
* thinker_text.rs:1126-1139 passes Some(k_scale) / Some(v_scale) (both 1.0) with a 16-bit cache:
  results are bit-identical to the None form.
* Prefill-sized appends (>= 4096 tokens: 16-token tiles) bit- / byte-exact for f32, bf16, f16 and
  fp8 pages, page sizes 8/16/32, pad slots, unaligned runs and an odd kv-head count.
"""
import numpy as np
import pytest
import torch

import paged_ref as ref
from cases import (bits_to_f32, config3_rounds, disjoint_block_tables, make_decode_case, make_prefill_case,
                   oracle_decode, oracle_prefill, sentinel_for)
from vasr_paged_attn import mistralrs_paged_attn as pa
from vasr_paged_attn.workloads import config5_context_lens

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
TORCH = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}
HQ, HKV, D = 16, 8, 128


def to_dev(bits, dtype, dev):
    bits = np.ascontiguousarray(bits)
    if dtype == "f32":
        return torch.from_numpy(bits.view(np.float32).copy()).to(dev)
    return torch.from_numpy(bits.view(np.int16).copy()).view(TORCH[dtype]).to(dev)


def to_bits(t):
    if t.dtype == torch.float32:
        return t.contiguous().view(torch.int32).cpu().numpy().view(np.uint32)
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def idx(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a).astype(np.int32)).to(dev)


@pytest.fixture(autouse=True)
def _clear(cuda_device):
    pa.device_error(clear=True)
    yield
    assert pa.device_error() == 0


def _prefill(case, dev, fp8=None):
    """Run the varlen prefill over the case's pages (fp8: (k bytes, v bytes, ks, vs))."""
    q = to_dev(case.q, case.dtype, dev)
    if fp8 is None:
        kc, vc, sk, sv = to_dev(case.key_cache, case.dtype, dev), to_dev(case.value_cache, case.dtype, dev), None, None
    else:
        kb, vb, ks, vs = fp8
        kc = torch.from_numpy(kb).to(dev).view(torch.float8_e4m3fn)
        vc = torch.from_numpy(vb).to(dev).view(torch.float8_e4m3fn)
        sk = torch.tensor([ks], dtype=torch.float32, device=dev)
        sv = torch.tensor([vs], dtype=torch.float32, device=dev)
    out = pa.paged_attention_varlen_prefill(q, kc, vc, idx(case.block_tables, dev), idx(case.context_lens, dev),
                                            idx(case.cu_q, dev), sk, sv, case.head_dim ** -0.5, 1.0)
    return out.float().cpu().numpy()


# ------------------------------------------------------------------ config 3
@pytest.mark.parametrize("rnd", [0, 1, 2, 3])
def test_prefill_config3_every_round_bf16(cuda_device, rnd):
    """Config 3 (seed 0): 32 prompts ~U[100, 800] in 256-token chunks; round r attends the r-th
    chunk of every prompt that has one over everything before it (offsets 0 / 256 / 512 / 768)."""
    _, rounds = config3_rounds(0)
    assert len(rounds) == 4
    r = rounds[rnd]
    case = make_prefill_case(40 + rnd, [s for (_, s, _) in r], [n for (_, _, n) in r], dtype="bf16")
    err = np.abs(_prefill(case, cuda_device) - oracle_prefill(case)).max()
    assert err <= BF16_TOL, err


def _fp8_pages_of(case, ks, vs):
    """The case's pages quantised to E4M3 bytes (value / scale), unused slots 0x7F (NaN)."""
    kf = bits_to_f32(case.key_cache, case.dtype)
    vf = bits_to_f32(case.value_cache, case.dtype)
    kb = ref.fp8_e4m3_encode(kf / np.float32(ks))
    vb = ref.fp8_e4m3_encode(vf / np.float32(vs))
    # fp8 pages pack 16 elements per key chunk: [nb, hkv, D/8, bs, 8] -> [nb, hkv, D/16, bs, 16]
    nb, hkv, dx, bs, x = kb.shape
    kb = kb.transpose(0, 1, 3, 2, 4).reshape(nb, hkv, bs, dx * x).reshape(nb, hkv, bs, dx * x // 16, 16)
    kb = np.ascontiguousarray(kb.transpose(0, 1, 3, 2, 4))
    return kb, np.ascontiguousarray(vb)


@pytest.mark.parametrize("rnd", [0, 1, 2, 3])
def test_prefill_config3_every_round_fp8(cuda_device, rnd):
    """The same rounds over fp8 (E4M3) pages: the oracle attends the dequantised pages, rounded to
    bf16 as the kernel's 16-bit scratch pool holds them."""
    _, rounds = config3_rounds(0)
    r = rounds[rnd]
    case = make_prefill_case(50 + rnd, [s for (_, s, _) in r], [n for (_, _, n) in r], dtype="bf16")
    ks, vs = 0.02, 0.015
    kb, vb = _fp8_pages_of(case, ks, vs)
    got = _prefill(case, cuda_device, fp8=(kb, vb, ks, vs))
    # the oracle's pages: bf16(decode(byte) * scale), back in the 8-wide key pack
    kf = torch.from_numpy(ref.fp8_e4m3_decode(kb) * np.float32(ks)).to(torch.bfloat16).float().numpy()
    vf = torch.from_numpy(ref.fp8_e4m3_decode(vb) * np.float32(vs)).to(torch.bfloat16).float().numpy()
    nb, hkv, dx, bs, x = kf.shape
    kf = kf.transpose(0, 1, 3, 2, 4).reshape(nb, hkv, bs, D // 8, 8).transpose(0, 1, 3, 2, 4)
    exp = ref.prefill_varlen(np.ascontiguousarray(bits_to_f32(case.q, "bf16")), np.ascontiguousarray(kf),
                             vf, np.ascontiguousarray(case.block_tables), np.ascontiguousarray(case.context_lens),
                             case.cu_q, D ** -0.5)
    err = np.abs(got - exp).max()
    assert err <= BF16_TOL, err


# --------------------------------------------------------------------- f16
@pytest.mark.parametrize("block_size", [8, 16, 32])
def test_prefill_f16(cuda_device, block_size):
    case = make_prefill_case(61, [0, 0, 256, 13, 100, 511], [1, 77, 256, 40, 130, 70], dtype="f16",
                             block_size=block_size)
    err = np.abs(_prefill(case, cuda_device) - oracle_prefill(case)).max()
    assert err <= BF16_TOL, err


@pytest.mark.parametrize("block_size", [8, 16, 32])
@pytest.mark.parametrize("gqa", [1, 2, 4])
def test_decode_f16(cuda_device, block_size, gqa):
    case = make_decode_case(62, [0, block_size, 63, 255, 256, 700, 1500], dtype="f16", num_heads=8 * gqa,
                            block_size=block_size, num_blocks=4096 // block_size + 16)
    t = {k: to_dev(getattr(case, a), "f16", cuda_device)
         for k, a in (("kc", "key_cache"), ("vc", "value_cache"), ("q", "q"), ("k", "k_new"), ("v", "v_new"))}
    pa.reshape_and_cache(t["k"], t["v"], None, None, t["kc"], t["vc"], torch.from_numpy(case.slots).to(cuda_device))
    out = pa.paged_attention(t["q"], None, None, t["kc"], t["vc"], idx(case.block_tables, cuda_device),
                             idx(case.context_lens, cuda_device), None, int(case.context_lens.max()),
                             D ** -0.5, 1.0, None)
    exp, kc_ref, vc_ref = oracle_decode(case)
    assert np.array_equal(to_bits(t["kc"]), kc_ref) and np.array_equal(to_bits(t["vc"]), vc_ref)
    err = np.abs(out.float().cpu().numpy() - exp).max()
    assert err <= BF16_TOL, err


# ----------------------------------------------- the reference's call form
def test_unit_scales_with_16bit_cache_match_the_none_form(cuda_device):
    """thinker_text.rs:1101-1109 / :1126-1139 pass Some(&k_scale), Some(&v_scale) = 1.0 for a bf16
    cache; the scales are unused there, so append and decode must equal the None call bit for bit."""
    case = make_decode_case(63, [37, 300, 1023, 2047], dtype="bf16", num_blocks=300)
    one = torch.ones(1, dtype=torch.float32, device=cuda_device)
    outs, pools = [], []
    for sk, sv in ((None, None), (one, one)):
        kc, vc = to_dev(case.key_cache, "bf16", cuda_device), to_dev(case.value_cache, "bf16", cuda_device)
        q = to_dev(case.q, "bf16", cuda_device)
        pa.reshape_and_cache(to_dev(case.k_new, "bf16", cuda_device), to_dev(case.v_new, "bf16", cuda_device),
                             sk, sv, kc, vc, torch.from_numpy(case.slots).to(cuda_device))
        out = pa.paged_attention(q, sk, sv, kc, vc, idx(case.block_tables, cuda_device),
                                 idx(case.context_lens, cuda_device), None, 2048, D ** -0.5, 1.0, None)
        outs.append(to_bits(out))
        pools.append((to_bits(kc), to_bits(vc)))
    assert np.array_equal(outs[0], outs[1])
    assert np.array_equal(pools[0][0], pools[1][0]) and np.array_equal(pools[0][1], pools[1][1])
    exp, _, _ = oracle_decode(case)
    assert np.abs(ref.bf16_bits_to_f32(outs[1]) - exp).max() <= BF16_TOL


# ------------------------------------------------------------------ config 5
def test_decode_config5_512_sequences_graph_bucket(cuda_device):
    """Config 5 attention: 512 sequences, ctx ~log-U[64, 4096] (seed 0), block tables at the graph's
    bucketed width (right-padded with the null block 0), max_context_len = width x 16 (an upper
    bound). The pool holds N(0,1) bf16 values; every slot no sequence owns holds a NaN sentinel."""
    rng = np.random.default_rng(64)
    lens = config5_context_lens(0).astype(np.int64)
    bs = 16
    blocks = [-(-int(n) // bs) for n in lens]
    cols = ref.bucket_block_table_cols(max(blocks), bs)
    assert cols >= max(blocks)
    nb = sum(blocks) + 1
    tables = disjoint_block_tables(rng, blocks, nb, cols)
    sent = sentinel_for("bf16")

    def rand_bf16(shape):
        out = np.empty(shape, np.uint16)
        for a in range(0, shape[0], 2048):  # truncated N(0,1) in bf16, built in slices
            b = min(shape[0], a + 2048)
            x = rng.standard_normal((b - a,) + shape[1:], dtype=np.float32)
            out[a:b] = (x.view(np.uint32) >> 16).astype(np.uint16)
        return out

    kc = rand_bf16((nb, HKV, D // 8, bs, 8))
    vc = rand_bf16((nb, HKV, D, bs))
    kc[0] = sent
    vc[0] = sent
    for i, n in enumerate(lens):  # the tail of each sequence's last page is not its data
        off = int(n) % bs
        if off:
            blk = int(tables[i, blocks[i] - 1])
            kc[blk, :, :, off:, :] = sent
            vc[blk, :, :, off:] = sent
    q = rand_bf16((len(lens), HQ, D))
    out = pa.paged_attention(to_dev(q, "bf16", cuda_device), None, None, to_dev(kc, "bf16", cuda_device),
                             to_dev(vc, "bf16", cuda_device), idx(tables, cuda_device), idx(lens, cuda_device),
                             None, cols * bs, D ** -0.5, 1.0, None).float().cpu().numpy()
    exp = ref.paged_attention(np.ascontiguousarray(ref.bf16_bits_to_f32(q)), ref.bf16_bits_to_f32(kc),
                              ref.bf16_bits_to_f32(vc), tables, lens.astype(np.uint32), D ** -0.5)
    assert np.isfinite(out).all()
    err = np.abs(out - exp).max()
    assert err <= BF16_TOL, err


# ------------------------------------------------------------------ config 4
def _layers_that_fit(per_layer_bytes, copies, cap):
    free, _ = torch.cuda.mem_get_info()
    return max(1, min(cap, int(free * 0.7 // (per_layer_bytes * copies))))


def test_copy_blocks_config4_full_pools(cuda_device):
    """Config 4 (seed 0): 4096 src -> dst pairs (src and dst disjoint, dst unique) over 200k-block
    bf16 pools, as many layers as fit next to a pristine copy. The oracle's host loop runs on the
    pages of the first 64 pairs; over the whole pools, page dst must hold the pristine page src and
    every other byte must be unchanged."""
    nb = 200_000
    per_layer = nb * HKV * D * 16 * 2 * 2
    layers = _layers_that_fit(per_layer, 2, 3)
    g = torch.Generator(device=cuda_device).manual_seed(0)
    kcs, vcs = [], []
    for _ in range(layers):
        kcs.append(torch.randint(-2**15, 2**15, (nb, HKV, D // 8, 16, 8), generator=g, dtype=torch.int16,
                                 device=cuda_device).view(torch.bfloat16))
        vcs.append(torch.randint(-2**15, 2**15, (nb, HKV, D, 16), generator=g, dtype=torch.int16,
                                 device=cuda_device).view(torch.bfloat16))
    perm = np.random.default_rng(0).permutation(nb)
    pairs = np.stack([perm[:4096], perm[4096:8192]], axis=1).astype(np.int64)
    src = torch.from_numpy(pairs[:, 0]).to(cuda_device)
    dst = torch.from_numpy(pairs[:, 1]).to(cuda_device)
    pristine = [c.view(torch.int16).clone() for c in kcs + vcs]
    pa.copy_blocks(kcs, vcs, torch.from_numpy(pairs).to(cuda_device))
    torch.cuda.synchronize()
    # the oracle on a sample: pages of the first 64 pairs, remapped to a small pool
    sub = pairs[:64]
    blocks = np.unique(sub.reshape(-1))
    remap = {int(b): i for i, b in enumerate(blocks)}
    mapped = np.array([[remap[int(s_)], remap[int(d_)]] for s_, d_ in sub], np.int64)
    sel = torch.from_numpy(blocks).to(cuda_device)
    pre_k = np.ascontiguousarray(pristine[0][sel].cpu().numpy())
    pre_v = np.ascontiguousarray(pristine[layers][sel].cpu().numpy())
    ref.copy_blocks([pre_k], [pre_v], mapped)
    assert np.array_equal(kcs[0].view(torch.int16)[sel].cpu().numpy(), pre_k)
    assert np.array_equal(vcs[0].view(torch.int16)[sel].cpu().numpy(), pre_v)
    # whole pools: dst pages hold the pristine src pages; restoring them gives back the pristine pool
    for got, orig in zip([c.view(torch.int16) for c in kcs + vcs], pristine):
        assert torch.equal(got[dst], orig[src])
        got[dst] = orig[dst]
        assert torch.equal(got, orig)


def test_swap_blocks_config4_1024_blocks(cuda_device):
    """Config 4 eviction and restore: 1024 blocks of a 200k-block device pool -> pinned host pool,
    then back into other device blocks; bit-exact against the oracle's host loop."""
    rng = np.random.default_rng(4)
    nb_dev, nb_host, n = 200_000, 2048, 1024
    g = torch.Generator(device=cuda_device).manual_seed(4)
    dev_pool = torch.randint(-2**15, 2**15, (nb_dev, HKV, D, 16), generator=g, dtype=torch.int16,
                             device=cuda_device).view(torch.bfloat16)
    host_pool = torch.full((nb_host, HKV, D, 16), 0x5A5A, dtype=torch.int16).pin_memory().view(torch.bfloat16)
    src = rng.permutation(nb_dev)[:n]
    dst = rng.permutation(nb_host)[:n]
    out_map = torch.from_numpy(np.stack([src, dst], 1).astype(np.int64)).to(cuda_device)
    pa.swap_blocks(dev_pool, host_pool, out_map)  # evict
    torch.cuda.synchronize()
    src_pages = dev_pool.view(torch.int16)[torch.from_numpy(src).to(cuda_device)].cpu().numpy()
    exp_host = np.full((nb_host, HKV, D, 16), 0x5A5A, np.int16)
    staged = np.zeros((n, HKV, D, 16), np.int16)
    staged[:] = src_pages
    ref.swap_blocks(exp_host, staged, np.stack([np.arange(n), dst], 1).astype(np.int64))
    assert np.array_equal(host_pool.view(torch.int16).numpy(), exp_host)
    # restore into blocks the eviction did not read
    free = np.setdiff1d(np.arange(nb_dev), src)
    back = rng.permutation(free)[:n]
    in_map = torch.from_numpy(np.stack([dst, back], 1).astype(np.int64)).to(cuda_device)
    before = dev_pool.view(torch.int16).clone()
    pa.swap_blocks(host_pool, dev_pool, in_map)  # restore
    torch.cuda.synchronize()
    before[torch.from_numpy(back).to(cuda_device)] = torch.from_numpy(src_pages).to(cuda_device)
    assert torch.equal(dev_pool.view(torch.int16), before)


# ----------------------------------------------- prefill-sized appends
def _slots_with_runs(rng, t, nb, bs):
    """A long run of consecutive slots starting mid-page, then scattered slots; every 9th a pad."""
    start = bs * 3 + 5
    half = t // 2
    slots = np.empty(t, np.int64)
    slots[:half] = np.arange(start, start + half)
    rest = rng.permutation(np.arange(start + half, nb * bs))[: t - half]
    slots[half:] = rest
    slots[::9] = ref.PAD_SLOT_ID
    return slots


@pytest.mark.parametrize("hkv", [3, 8])
@pytest.mark.parametrize("bs", [8, 16, 32])
@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
def test_append_prefill_sized_bitexact(cuda_device, dtype, bs, hkv):
    """4100 tokens (16-token tiles, a ragged last tile) into 16-bit / f32 pages, bit-exact over
    the whole NaN-filled pool."""
    rng = np.random.default_rng(1000 + bs + hkv)
    t = 4100
    nb = 3 * t // bs + 16
    slots = _slots_with_runs(rng, t, nb, bs)
    word = np.uint32 if dtype == "f32" else np.uint16
    x = 16 // np.dtype(word).itemsize
    kc = np.full((nb, hkv, D // x, bs, x), sentinel_for(dtype), word)
    vc = np.full((nb, hkv, D, bs), sentinel_for(dtype), word)
    k = rng.integers(0, np.iinfo(word).max, size=(t, hkv, D), dtype=word)
    v = rng.integers(0, np.iinfo(word).max, size=(t, hkv, D), dtype=word)
    dk, dv = to_dev(kc, dtype, cuda_device), to_dev(vc, dtype, cuda_device)
    pa.reshape_and_cache(to_dev(k, dtype, cuda_device), to_dev(v, dtype, cuda_device), None, None, dk, dv,
                         torch.from_numpy(slots).to(cuda_device))
    ref.reshape_and_cache(k, v, kc, vc, slots, bs)
    assert np.array_equal(to_bits(dk), kc)
    assert np.array_equal(to_bits(dv), vc)


@pytest.mark.parametrize("hkv", [3, 8])
@pytest.mark.parametrize("bs", [8, 16, 32])
@pytest.mark.parametrize("src", ["f32", "bf16", "f16"])
def test_fp8_append_prefill_sized_byte_exact(cuda_device, src, bs, hkv):
    """4100 tokens into fp8 (E4M3) pages: byte-exact against the oracle's encoder."""
    rng = np.random.default_rng(2000 + bs + hkv)
    t = 4100
    nb = 3 * t // bs + 16
    slots = _slots_with_runs(rng, t, nb, bs)
    kf = (rng.standard_normal((t, hkv, D)) * 3).astype(np.float32)
    vf = (rng.standard_normal((t, hkv, D)) * 3).astype(np.float32)
    kf[0, 0, :5] = [1e4, -1e4, 0.0, -0.0, 1e-12]
    kt, vt = torch.from_numpy(kf).to(TORCH[src]), torch.from_numpy(vf).to(TORCH[src])
    ks, vs = 0.05, 0.02
    kc = torch.full((nb, hkv, D // 16, bs, 16), 0x5A, dtype=torch.uint8, device=cuda_device)
    vc = torch.full((nb, hkv, D, bs), 0x5A, dtype=torch.uint8, device=cuda_device)
    sk = torch.tensor([ks], dtype=torch.float32, device=cuda_device)
    sv = torch.tensor([vs], dtype=torch.float32, device=cuda_device)
    pa.reshape_and_cache(kt.to(cuda_device), vt.to(cuda_device), sk, sv, kc.view(torch.float8_e4m3fn),
                         vc.view(torch.float8_e4m3fn), torch.from_numpy(slots).to(cuda_device))
    ek = np.full((nb, hkv, D // 16, bs, 16), 0x5A, np.uint8)
    ev = np.full((nb, hkv, D, bs), 0x5A, np.uint8)
    ref.reshape_and_cache_fp8(kt.float().numpy(), vt.float().numpy(), ek, ev, slots, bs, ks, vs)
    assert np.array_equal(kc.cpu().numpy(), ek)
    assert np.array_equal(vc.cpu().numpy(), ev)
