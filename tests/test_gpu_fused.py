"""Fused q/k RMSNorm + RoPE + KV append against the bf16 oracle and the unfused torch path.

Tolerance: the kernel uses rsqrtf, the oracle an exact square root, so a
bf16 result may differ by one unit in the last place; everything else (v,
slots, untouched pool entries) is bit-exact.
"""
import numpy as np
import pytest
import torch

import paged_ref as ref
from vasr_paged_attn import fused, mistralrs_paged_attn as pa
from vasr_paged_attn.engine import DecoderConfig, RandomQwen3Decoder, allocate_paged_cache

pytestmark = pytest.mark.gpu


def bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def ulp_close(a_bits, b_bits, min_exact=0.999):
    """At least ``min_exact`` of the elements bit-identical; the rest within one bf16 ulp of
    the output (2^-7 relative) plus 4e-3 absolute. rsqrtf can round a normalised value
    (magnitude ~1, bf16 ulp ~4e-3) across a bf16 boundary; the rotation carries that step
    into outputs that may be near-cancelled and small, so the bound is absolute at the
    scale of the normalised inputs."""
    a = ref.bf16_bits_to_f32(a_bits)
    b = ref.bf16_bits_to_f32(b_bits)
    ok = np.abs(a - b) <= np.maximum(np.abs(a), np.abs(b)) * 2.0 ** -7 + 4e-3
    return bool(ok.all()) and (a_bits == b_bits).mean() >= min_exact


@pytest.mark.parametrize("num_tokens,block_size", [(64, 16), (300, 8), (17, 32)])
def test_fused_matches_oracle(cuda_device, num_tokens, block_size):
    dev = cuda_device
    hq, hkv, d, nb = 16, 8, 128, 64
    g = torch.Generator(device="cpu").manual_seed(num_tokens)
    qkv = (torch.randn(num_tokens, (hq + 2 * hkv) * d, generator=g) * 3).to(torch.bfloat16)
    qw = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    model_cfg = DecoderConfig(num_layers=1, vocab_size=16, max_positions=4096)
    inv = 1.0 / (model_cfg.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    ang = torch.outer(torch.arange(4096, dtype=torch.float64), inv)
    cos, sin = torch.cos(ang).float(), torch.sin(ang).float()
    pos = torch.randint(0, 4096, (num_tokens,), generator=g)
    slots = torch.randperm(nb * block_size, generator=g)[:num_tokens].to(torch.int64)
    slots[::7] = -1  # padded rows are skipped
    kc = torch.zeros(nb, hkv, d // 8, block_size, 8, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros(nb, hkv, d, block_size, dtype=torch.bfloat16, device=dev)
    q = fused.qk_norm_rope_append(qkv.to(dev), qw.to(dev), kw.to(dev), 1e-6, cos.to(dev), sin.to(dev),
                                  pos.to(dev), kc, vc, slots.to(dev), hq)
    q_ref, k_ref, v_ref = ref.qk_norm_rope_ref(bits(qkv), bits(qw), bits(kw), 1e-6, cos.numpy(), sin.numpy(),
                                               pos.numpy(), hq, hkv, d)
    assert ulp_close(bits(q), q_ref)
    kc_ref = np.zeros(tuple(kc.shape), np.uint16)
    vc_ref = np.zeros(tuple(vc.shape), np.uint16)
    ref.reshape_and_cache(np.ascontiguousarray(k_ref), v_ref, kc_ref, vc_ref, slots.numpy(), block_size)
    assert np.array_equal(bits(vc), vc_ref)
    written = kc_ref != 0
    assert ulp_close(bits(kc)[written], kc_ref[written])
    assert np.array_equal(bits(kc)[~written], kc_ref[~written])  # nothing else was touched
    assert pa.device_error() == 0


def test_fused_step_matches_unfused_step(cuda_device):
    """A full decode step with the fused kernel equals the torch-op path (same next ids, close logits)."""
    dev = cuda_device
    cfg = DecoderConfig(num_layers=4, vocab_size=4096, max_positions=8192)
    model = RandomQwen3Decoder(cfg, dev, seed=3)
    b, bs, nb = 8, 16, 1 + 8 * 40
    caches_a = allocate_paged_cache(cfg, nb, bs, dev)
    gen = torch.Generator(device=dev).manual_seed(0)
    for kc, vc in caches_a:
        kc.normal_(generator=gen)
        vc.normal_(generator=gen)
    caches_b = [(kc.clone(), vc.clone()) for kc, vc in caches_a]
    rng = np.random.default_rng(0)
    lens = rng.integers(100, 600, size=b)
    tables = np.zeros((b, 40), np.int32)
    perm = rng.permutation(np.arange(1, nb))
    for i in range(b):
        tables[i] = perm[i * 40:(i + 1) * 40]
    pos = torch.from_numpy(lens).to(dev)
    slots = torch.from_numpy(tables[np.arange(b), lens // bs].astype(np.int64) * bs + lens % bs).to(dev)
    ctx = torch.from_numpy((lens + 1).astype(np.int32)).to(dev)
    bt = torch.from_numpy(tables).to(dev)
    ids = torch.from_numpy(rng.integers(0, cfg.vocab_size, size=b)).to(dev)
    a = model.decode_step(ids, pos, caches_a, slots, bt, ctx, 40 * bs, fused=True)
    bb = model.decode_step(ids, pos, caches_b, slots, bt, ctx, 40 * bs, fused=False)
    torch.cuda.synchronize()
    # a 1-ulp bf16 difference may flip a near-tie argmax; nearly all ids must agree
    assert (a == bb).float().mean().item() >= 7 / 8
    pages = torch.from_numpy(tables[np.arange(b), lens // bs].astype(np.int64)).to(dev)
    offs = torch.from_numpy((lens % bs).astype(np.int64)).to(dev)
    for (ka, va), (kb, vb) in zip(caches_a, caches_b):
        assert torch.equal(va, vb)
        wa = ka[pages, :, :, offs, :]  # the new token's K of every sequence
        wb = kb[pages, :, :, offs, :]
        assert ulp_close(bits(wa), bits(wb))
        assert (ka.view(torch.int16) != kb.view(torch.int16)).sum().item() == \
            (wa.view(torch.int16) != wb.view(torch.int16)).sum().item()


def _after_append_case(dev, layers=4, b=64, bs=16, seed=5):
    hq, hkv, d = 16, 8, 128
    rng = np.random.default_rng(seed)
    lens = rng.integers(200, 1501, size=b)  # tokens already cached; the step appends one more
    blocks = (lens + 1 + bs - 1) // bs
    cols = int(blocks.max())
    nb = int(blocks.sum()) + 1
    perm = rng.permutation(np.arange(1, nb))
    tables = np.zeros((b, cols), np.int32)
    off = 0
    for i, n in enumerate(blocks):
        tables[i, :n] = perm[off:off + n]
        off += n
    slots = tables[np.arange(b), lens // bs].astype(np.int64) * bs + lens % bs
    gen = torch.Generator(device=dev).manual_seed(seed)
    caches = []
    for _ in range(layers):
        kc = torch.randn(nb, hkv, d // 8, bs, 8, generator=gen, device=dev).to(torch.bfloat16)
        vc = torch.randn(nb, hkv, d, bs, generator=gen, device=dev).to(torch.bfloat16)
        # the new token's slot holds stale data far from what the append writes:
        # a decode that read it before the append completed would be far off
        pg = torch.from_numpy(slots // bs).to(dev)
        of = torch.from_numpy(slots % bs).to(dev)
        kc[pg, :, :, of, :] = 40.0
        vc[pg, :, :, of] = -40.0
        caches.append((kc, vc))
    qkv = [torch.randn(b, (hq + 2 * hkv) * d, generator=gen, device=dev).to(torch.bfloat16)
           for _ in range(layers)]
    norm_w = torch.ones(d, dtype=torch.bfloat16, device=dev)
    cfg = DecoderConfig(num_layers=1, vocab_size=16, max_positions=4096)
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    ang = torch.outer(torch.arange(4096, dtype=torch.float64), inv)
    cos, sin = torch.cos(ang).float().to(dev), torch.sin(ang).float().to(dev)
    meta = dict(pos=torch.from_numpy(lens).to(dev), slots=torch.from_numpy(slots).to(dev),
                ctx=torch.from_numpy((lens + 1).astype(np.int32)).to(dev),
                tables=torch.from_numpy(tables).to(dev), mcl=cols * bs, hq=hq)
    return caches, qkv, norm_w, cos, sin, meta


def _append_then_decode(caches, qkv, norm_w, cos, sin, m, after_append):
    outs = []
    for (kc, vc), x in zip(caches, qkv):
        q = fused.qk_norm_rope_append(x, norm_w, norm_w, 1e-6, cos, sin, m["pos"], kc, vc, m["slots"], m["hq"])
        outs.append(pa.paged_attention(q, None, None, kc, vc, m["tables"], m["ctx"], None, m["mcl"],
                                       128 ** -0.5, 1.0, None, after_append=after_append))
    return outs


def test_decode_after_append_equals_plain_decode(cuda_device):
    """The programmatic-dependent decode behind the append gives the plain call's bits,
    eagerly and in a CUDA graph of append -> decode pairs, although the new token's
    slot held stale data until the append wrote it."""
    dev = cuda_device
    caches, qkv, w, cos, sin, m = _after_append_case(dev)
    ref_caches = [(k.clone(), v.clone()) for k, v in caches]
    graph_caches = [(k.clone(), v.clone()) for k, v in caches]
    want = _append_then_decode(ref_caches, qkv, w, cos, sin, m, after_append=False)
    got = _append_then_decode(caches, qkv, w, cos, sin, m, after_append=True)
    torch.cuda.synchronize()
    for a, b in zip(got, want):
        assert torch.equal(a, b)
    for (ka, va), (kb, vb) in zip(caches, ref_caches):
        assert torch.equal(ka, kb) and torch.equal(va, vb)
    # the stale values are gone from the outputs: |out| stays at the N(0,1) V scale
    assert max(float(o.float().abs().max()) for o in got) < 8.0

    s = torch.cuda.Stream(device=dev)
    need = pa.paged_attention_workspace_bytes(64, 16, 8, 128, 16, m["mcl"], torch.bfloat16)
    pa.reserve_paged_attention_workspace(dev, need, s)  # one workspace per stream, before capture
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            outs = _append_then_decode(graph_caches, qkv, w, cos, sin, m, after_append=True)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):  # the append rewrites the same slot with the same values
        g.replay()
    torch.cuda.synchronize()
    for a, b in zip(outs, want):
        assert torch.equal(a, b)
    del g
