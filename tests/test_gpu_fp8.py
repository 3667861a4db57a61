"""fp8 (E4M3) KV cache: the append is byte-exact against the oracle's encoder,
decode attention over fp8 pages is within the bf16 tolerance (2e-2) of the
f64 oracle run on the dequantised pages (stored byte value x scale)."""
import numpy as np
import pytest
import torch

import paged_ref as ref
from cases import disjoint_block_tables
from vasr_paged_attn import _lib
from vasr_paged_attn import mistralrs_paged_attn as pa

pytestmark = pytest.mark.gpu

HKV, HQ, D = 8, 16, 128
SENTINEL = 0x5A


@pytest.fixture(autouse=True)
def _clear(cuda_device):
    pa.device_error(clear=True)
    yield
    assert pa.device_error() == 0


def _u8_cache(nb, bs, dev, fill=SENTINEL):
    kc = torch.full((nb, HKV, D // 16, bs, 16), fill, dtype=torch.uint8, device=dev)
    vc = torch.full((nb, HKV, D, bs), fill, dtype=torch.uint8, device=dev)
    return kc, vc


def _scales(dev, ks, vs):
    return (torch.tensor([ks], dtype=torch.float32, device=dev),
            torch.tensor([vs], dtype=torch.float32, device=dev))


@pytest.mark.parametrize("t", [77, 600])  # a warp per (token, head) / 8-token tiles with V runs
@pytest.mark.parametrize("src", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("bs", [8, 16, 32])
def test_fp8_append_is_byte_exact(cuda_device, src, bs, t):
    rng = np.random.default_rng(bs + t)
    nb = 40 if t < 128 else t // bs + 8
    k = (rng.standard_normal((t, HKV, D)) * 3).astype(np.float32)
    v = (rng.standard_normal((t, HKV, D)) * 3).astype(np.float32)
    k[0, 0, :7] = [1e4, -1e4, 0.0, -0.0, 1e-12, 449 * 0.05, 448 * 0.05]  # saturation, signed zeros
    slots = rng.permutation(nb * bs)[:t].astype(np.int64)
    if t >= 128:  # runs of consecutive slots, some page-aligned, some not
        slots[: t // 2] = np.arange(bs * 3 + 5, bs * 3 + 5 + t // 2)
        slots[t // 2:] = rng.permutation(np.arange(bs * 3 + 5 + t // 2, nb * bs))[: t - t // 2]
    slots[::9] = -1
    kt, vt = torch.from_numpy(k).to(src), torch.from_numpy(v).to(src)
    ks, vs = 0.05, 0.02
    kc, vc = _u8_cache(nb, bs, cuda_device)
    sk, sv = _scales(cuda_device, ks, vs)
    pa.reshape_and_cache(kt.to(cuda_device), vt.to(cuda_device), sk, sv, kc.view(torch.float8_e4m3fn),
                         vc.view(torch.float8_e4m3fn), torch.from_numpy(slots).to(cuda_device))
    ek = np.full((nb, HKV, D // 16, bs, 16), SENTINEL, np.uint8)
    ev = np.full((nb, HKV, D, bs), SENTINEL, np.uint8)
    ref.reshape_and_cache_fp8(kt.float().numpy(), vt.float().numpy(), ek, ev, slots, bs, ks, vs)
    assert np.array_equal(kc.cpu().numpy(), ek)
    assert np.array_equal(vc.cpu().numpy(), ev)


def _fp8_decode_case(rng, ctx, bs, ks, vs):
    blocks = [-(-int(c) // bs) for c in ctx]
    nb = sum(blocks) + 4
    tables = disjoint_block_tables(rng, blocks, nb)
    kc = np.full((nb, HKV, D // 16, bs, 16), 0x7F, np.uint8)  # NaN bytes where nothing was written
    vc = np.full((nb, HKV, D, bs), 0x7F, np.uint8)
    for i, n in enumerate(ctx):
        k = rng.standard_normal((int(n), HKV, D)).astype(np.float32)
        v = rng.standard_normal((int(n), HKV, D)).astype(np.float32)
        pos = np.arange(int(n))
        slots = tables[i, pos // bs].astype(np.int64) * bs + pos % bs
        ref.reshape_and_cache_fp8(k, v, kc, vc, slots, bs, ks, vs)
    return tables, kc, vc


@pytest.mark.parametrize("bs", [16, 32])
def test_fp8_decode_matches_oracle(cuda_device, bs):
    rng = np.random.default_rng(100 + bs)
    ctx = np.array([1, 17, 200, 513, 1024, 1500, 2049], np.int64)
    ks, vs = 0.02, 0.015
    tables, kc, vc = _fp8_decode_case(rng, ctx, bs, ks, vs)
    q = torch.from_numpy(rng.standard_normal((len(ctx), HQ, D)).astype(np.float32)).to(torch.bfloat16)
    sk, sv = _scales(cuda_device, ks, vs)
    out = pa.paged_attention(q.to(cuda_device), sk, sv,
                             torch.from_numpy(kc).to(cuda_device).view(torch.float8_e4m3fn),
                             torch.from_numpy(vc).to(cuda_device).view(torch.float8_e4m3fn),
                             torch.from_numpy(tables.astype(np.int32)).to(cuda_device),
                             torch.from_numpy(ctx.astype(np.int32)).to(cuda_device), None,
                             int(ctx.max()), D ** -0.5, 1.0, None).float().cpu().numpy()
    kf = np.ascontiguousarray(ref.fp8_e4m3_decode(kc) * np.float32(ks))
    vf = np.ascontiguousarray(ref.fp8_e4m3_decode(vc) * np.float32(vs))
    exp = ref.paged_attention(np.ascontiguousarray(q.float().numpy()), kf, vf,
                              np.ascontiguousarray(tables.astype(np.uint32)), ctx.astype(np.uint32),
                              D ** -0.5)
    assert np.abs(out - exp).max() <= 2e-2


@pytest.mark.parametrize("bs", [16, 32])
def test_fp8_decode_multi_wave_grid(cuda_device, bs):
    """A launch of at least two waves at six CTAs per SM (64 sequences, max_context_len 4096 as an
    upper bound: four splits per (sequence, kv head), 2048 CTAs) takes the fp8 decode's wide
    instantiation (query fragments in shared memory); splits past a sequence's end exit."""
    rng = np.random.default_rng(777)
    ctx = rng.integers(20, 700, size=64).astype(np.int64)
    ctx[:3] = [1, 16, 699]
    ks, vs = 0.02, 0.015
    tables, kc, vc = _fp8_decode_case(rng, ctx, bs, ks, vs)
    q = torch.from_numpy(rng.standard_normal((len(ctx), HQ, D)).astype(np.float32)).to(torch.bfloat16)
    sk, sv = _scales(cuda_device, ks, vs)
    out = pa.paged_attention(q.to(cuda_device), sk, sv,
                             torch.from_numpy(kc).to(cuda_device).view(torch.float8_e4m3fn),
                             torch.from_numpy(vc).to(cuda_device).view(torch.float8_e4m3fn),
                             torch.from_numpy(tables.astype(np.int32)).to(cuda_device),
                             torch.from_numpy(ctx.astype(np.int32)).to(cuda_device), None,
                             4096, D ** -0.5, 1.0, None).float().cpu().numpy()
    kf = np.ascontiguousarray(ref.fp8_e4m3_decode(kc) * np.float32(ks))
    vf = np.ascontiguousarray(ref.fp8_e4m3_decode(vc) * np.float32(vs))
    exp = ref.paged_attention(np.ascontiguousarray(q.float().numpy()), kf, vf,
                              np.ascontiguousarray(tables.astype(np.uint32)), ctx.astype(np.uint32),
                              D ** -0.5)
    assert np.abs(out - exp).max() <= 2e-2


def test_fp8_append_then_decode(cuda_device):
    """Append bf16 K/V into fp8 pages on the GPU, then decode; the oracle quantises the same values."""
    rng = np.random.default_rng(9)
    bs, ctx = 16, np.array([300, 45, 1200], np.int64)
    blocks = [-(-int(c) // bs) for c in ctx]
    nb = sum(blocks) + 2
    tables = disjoint_block_tables(rng, blocks, nb)
    kc, vc = _u8_cache(nb, bs, cuda_device, fill=0)
    ks, vs = 0.03, 0.02
    sk, sv = _scales(cuda_device, ks, vs)
    ek = np.zeros((nb, HKV, D // 16, bs, 16), np.uint8)
    ev = np.zeros((nb, HKV, D, bs), np.uint8)
    for i, n in enumerate(ctx):
        k = torch.from_numpy(rng.standard_normal((int(n), HKV, D)).astype(np.float32)).to(torch.bfloat16)
        v = torch.from_numpy(rng.standard_normal((int(n), HKV, D)).astype(np.float32)).to(torch.bfloat16)
        pos = np.arange(int(n))
        slots = tables[i, pos // bs].astype(np.int64) * bs + pos % bs
        pa.reshape_and_cache(k.to(cuda_device), v.to(cuda_device), sk, sv, kc.view(torch.float8_e4m3fn),
                             vc.view(torch.float8_e4m3fn), torch.from_numpy(slots).to(cuda_device))
        ref.reshape_and_cache_fp8(k.float().numpy(), v.float().numpy(), ek, ev, slots, bs, ks, vs)
    q = torch.from_numpy(rng.standard_normal((len(ctx), HQ, D)).astype(np.float32)).to(torch.bfloat16)
    out = pa.paged_attention(q.to(cuda_device), sk, sv, kc.view(torch.float8_e4m3fn),
                             vc.view(torch.float8_e4m3fn),
                             torch.from_numpy(tables.astype(np.int32)).to(cuda_device),
                             torch.from_numpy(ctx.astype(np.int32)).to(cuda_device), None,
                             int(ctx.max()), D ** -0.5, 1.0, None).float().cpu().numpy()
    assert np.array_equal(kc.cpu().numpy(), ek) and np.array_equal(vc.cpu().numpy(), ev)
    exp = ref.paged_attention(np.ascontiguousarray(q.float().numpy()),
                              np.ascontiguousarray(ref.fp8_e4m3_decode(ek) * np.float32(ks)),
                              np.ascontiguousarray(ref.fp8_e4m3_decode(ev) * np.float32(vs)),
                              np.ascontiguousarray(tables.astype(np.uint32)), ctx.astype(np.uint32),
                              D ** -0.5)
    assert np.abs(out - exp).max() <= 2e-2


def test_fp8_rejects_missing_scales_and_bs8_decode(cuda_device):
    kc, vc = _u8_cache(4, 8, cuda_device)
    q = torch.zeros(1, HQ, D, dtype=torch.bfloat16, device=cuda_device)
    t = torch.ones(1, 1, dtype=torch.int32, device=cuda_device)
    c = torch.ones(1, dtype=torch.int32, device=cuda_device)
    with pytest.raises(_lib.VasrPaError):
        pa.paged_attention(q, None, None, kc.view(torch.float8_e4m3fn), vc.view(torch.float8_e4m3fn), t, c,
                           None, 8, 0.1, 1.0, None)
    sk, sv = _scales(cuda_device, 1.0, 1.0)
    with pytest.raises(_lib.VasrPaError) as e:
        pa.paged_attention(q, sk, sv, kc.view(torch.float8_e4m3fn), vc.view(torch.float8_e4m3fn), t, c,
                           None, 8, 0.1, 1.0, None)
    assert e.value.status == _lib.ENOT_SUPPORTED


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("bs", [8, 16, 32])
def test_fp8_gather_is_exact(cuda_device, out_dtype, bs):
    """gather_kv_cache over fp8 pages: byte * scale rounded to out_dtype, bit for bit."""
    rng = np.random.default_rng(300 + bs)
    ctx = np.array([1, bs - 1, bs, bs + 1, 77, 300], np.int64)
    blocks = [-(-int(c) // bs) for c in ctx]
    nb = sum(blocks) + 3
    tables = disjoint_block_tables(rng, blocks, nb)
    kc = rng.integers(0, 256, size=(nb, HKV, D // 16, bs, 16), dtype=np.uint8)
    vc = rng.integers(0, 256, size=(nb, HKV, D, bs), dtype=np.uint8)
    for c in (kc, vc):  # no NaN bytes: NaN payloads need not match
        c[(c & 0x7F) == 0x7F] = 0x11
    ks, vs = 0.037, 1.5
    cu = np.concatenate([[0], np.cumsum(ctx)]).astype(np.uint32)
    sk, sv = _scales(cuda_device, ks, vs)
    k, v = pa.gather_kv_cache(torch.from_numpy(kc).to(cuda_device).view(torch.float8_e4m3fn),
                              torch.from_numpy(vc).to(cuda_device).view(torch.float8_e4m3fn), sk, sv,
                              torch.from_numpy(tables.astype(np.int32)).to(cuda_device),
                              torch.from_numpy(cu.astype(np.int32)).to(cuda_device), out_dtype)
    assert k.dtype == out_dtype and k.shape == (int(cu[-1]), HKV, D)
    kr, vr = ref.gather_kv_cache_fp8(kc, vc, np.ascontiguousarray(tables.astype(np.uint32)), cu, HKV, D,
                                     bs, ks, vs)
    for got, exp in ((k, kr), (v, vr)):
        want = torch.from_numpy(exp).to(out_dtype)
        assert torch.equal(got.cpu().view(torch.int16 if out_dtype != torch.float32 else torch.int32),
                           want.view(torch.int16 if out_dtype != torch.float32 else torch.int32))


def test_fp8_gather_requires_scales(cuda_device):
    kc, vc = _u8_cache(4, 16, cuda_device)
    t = torch.ones(1, 1, dtype=torch.int32, device=cuda_device)
    cu = torch.tensor([0, 5], dtype=torch.int32, device=cuda_device)
    with pytest.raises(_lib.VasrPaError):
        pa.gather_kv_cache(kc.view(torch.float8_e4m3fn), vc.view(torch.float8_e4m3fn), None, None, t, cu)


@pytest.mark.parametrize("bs,hq", [(16, 16), (32, 16), (16, 8), (16, 32)])
def test_fp8_prefill_matches_oracle(cuda_device, bs, hq):
    """Varlen prefill over fp8 pages: the oracle runs the same causal mask on the dequantised pages.
    16-token pages (GQA 1 / 2 / 4) take the tcgen05 kernel, which converts the bytes exactly and
    applies the scales to the scores and the output: the oracle sees byte x scale in f32. Other
    page sizes go through the workspace's 16-bit pool of bf16(byte x scale)."""
    rng = np.random.default_rng(500 + bs + hq)
    cached = np.array([0, 37, 256, 5], np.int64)
    chunk = np.array([90, 64, 100, 1], np.int64)
    ctx = cached + chunk
    ks, vs = 0.02, 0.015
    tables, kc, vc = _fp8_decode_case(rng, ctx, bs, ks, vs)
    cu = np.concatenate([[0], np.cumsum(chunk)]).astype(np.int32)
    q = torch.from_numpy(rng.standard_normal((int(cu[-1]), hq, D)).astype(np.float32)).to(torch.bfloat16)
    sk, sv = _scales(cuda_device, ks, vs)
    out = pa.paged_attention_varlen_prefill(
        q.to(cuda_device), torch.from_numpy(kc).to(cuda_device).view(torch.float8_e4m3fn),
        torch.from_numpy(vc).to(cuda_device).view(torch.float8_e4m3fn),
        torch.from_numpy(tables.astype(np.int32)).to(cuda_device),
        torch.from_numpy(ctx.astype(np.int32)).to(cuda_device), torch.from_numpy(cu).to(cuda_device),
        sk, sv, D ** -0.5).float().cpu().numpy()
    kf = np.ascontiguousarray(ref.fp8_e4m3_decode(kc) * np.float32(ks))
    vf = np.ascontiguousarray(ref.fp8_e4m3_decode(vc) * np.float32(vs))
    if bs != 16:  # the 16-bit pool holds bf16(byte * scale): the oracle sees the same rounded pages
        kf = torch.from_numpy(kf).to(torch.bfloat16).float().numpy()
        vf = torch.from_numpy(vf).to(torch.bfloat16).float().numpy()
    exp = ref.prefill_varlen(np.ascontiguousarray(q.float().numpy()), kf, vf,
                             np.ascontiguousarray(tables.astype(np.uint32)), ctx.astype(np.uint32),
                             cu.astype(np.uint32), D ** -0.5)
    assert np.abs(out - exp).max() <= 2e-2


def test_fp8_prefill_long_context_split(cuda_device):
    """A launch of few items over a long fp8 context: the cluster-split variant of the tcgen05
    kernel (key tiles shared by the CTAs of a cluster, combined in distributed shared memory)."""
    rng = np.random.default_rng(77)
    cached = np.array([1490, 768], np.int64)
    chunk = np.array([12, 7], np.int64)
    ctx = cached + chunk
    ks, vs = 0.03, 0.01
    tables, kc, vc = _fp8_decode_case(rng, ctx, 16, ks, vs)
    cu = np.concatenate([[0], np.cumsum(chunk)]).astype(np.int32)
    q = torch.from_numpy(rng.standard_normal((int(cu[-1]), HQ, D)).astype(np.float32)).to(torch.bfloat16)
    sk, sv = _scales(cuda_device, ks, vs)
    out = pa.paged_attention_varlen_prefill(
        q.to(cuda_device), torch.from_numpy(kc).to(cuda_device).view(torch.float8_e4m3fn),
        torch.from_numpy(vc).to(cuda_device).view(torch.float8_e4m3fn),
        torch.from_numpy(tables.astype(np.int32)).to(cuda_device),
        torch.from_numpy(ctx.astype(np.int32)).to(cuda_device), torch.from_numpy(cu).to(cuda_device),
        sk, sv, D ** -0.5).float().cpu().numpy()
    kf = np.ascontiguousarray(ref.fp8_e4m3_decode(kc) * np.float32(ks))
    vf = np.ascontiguousarray(ref.fp8_e4m3_decode(vc) * np.float32(vs))
    exp = ref.prefill_varlen(np.ascontiguousarray(q.float().numpy()), kf, vf,
                             np.ascontiguousarray(tables.astype(np.uint32)), ctx.astype(np.uint32),
                             cu.astype(np.uint32), D ** -0.5)
    assert np.abs(out - exp).max() <= 2e-2


@pytest.mark.parametrize("t", [64, 4160])  # a warp per (token, head) / 16-token tiles
@pytest.mark.parametrize("src", [torch.bfloat16, torch.float16])
def test_fp8_append_every_16bit_input_is_byte_exact(cuda_device, src, t):
    """Every non-NaN bf16 / f16 bit pattern, for several scales, against the oracle's encoder of
    the IEEE quotient: the append's division-free rounding must not move a single byte."""
    bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    vals = torch.from_numpy(bits.view(np.int16).copy()).view(src).float().numpy()
    bits = np.where(np.isnan(vals), np.uint16(0), bits)  # NaN payloads need not match
    reps = t * HKV * D // (1 << 16)
    flat = np.concatenate([np.roll(bits, 4099 * i) for i in range(reps)])
    x = torch.from_numpy(flat.view(np.int16).copy()).view(src).reshape(t, HKV, D)
    bs, nb = 16, t // 16 + 2
    slots = np.arange(t, dtype=np.int64) + bs  # page-aligned runs from block 1
    for ks in (0.05, 0.02, 1.0, 1.0 / 3.0, 7.3e-3, 3.7, 1e-30, 5e29):
        kc, vc = _u8_cache(nb, bs, cuda_device)
        sk, sv = _scales(cuda_device, ks, ks * 1.37)
        pa.reshape_and_cache(x.to(cuda_device), x.to(cuda_device), sk, sv, kc.view(torch.float8_e4m3fn),
                             vc.view(torch.float8_e4m3fn), torch.from_numpy(slots).to(cuda_device))
        ek = np.full((nb, HKV, D // 16, bs, 16), SENTINEL, np.uint8)
        ev = np.full((nb, HKV, D, bs), SENTINEL, np.uint8)
        xf = x.float().numpy()
        ref.reshape_and_cache_fp8(xf, xf, ek, ev, slots, bs, np.float32(ks), np.float32(ks * 1.37))
        assert np.array_equal(kc.cpu().numpy(), ek), ks
        assert np.array_equal(vc.cpu().numpy(), ev), ks
