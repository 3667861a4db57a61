"""Device decode loop: greedy argmax and step prepare against the oracle's host restatement.

Integer outputs (token ids, positions, slots, context lengths, finished
flags, histories) must match exactly.
"""
import numpy as np
import pytest
import torch

import paged_ref as ref
from vasr_paged_attn import _lib
from vasr_paged_attn import decode_loop as dl
from vasr_paged_attn import mistralrs_paged_attn as pa

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _clear(cuda_device):
    pa.device_error(clear=True)
    yield


def _logits(rng, b, vocab, dtype, dev):
    x = rng.standard_normal((b, vocab)).astype(np.float32)
    # planted ties: the same maximum twice, the lower index must win
    for i in range(0, b, 3):
        j, k = sorted(rng.choice(vocab, 2, replace=False))
        x[i, j] = x[i, k] = 50.0
    if b > 4:
        x[1, :] = np.nan                # all NaN -> 0
        x[2, :] = -np.inf               # no value above -inf -> 0
        x[4, rng.integers(0, vocab, 5)] = np.nan
    t = torch.from_numpy(x).to(dtype)
    return t.to(dev), t.float().numpy()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("vocab", [151936, 1000, 7])
def test_greedy_argmax_matches_first_index(cuda_device, dtype, vocab):
    rng = np.random.default_rng(vocab)
    b = 37
    lg, host = _logits(rng, b, vocab, dtype, cuda_device)
    got = dl.greedy_argmax(lg).cpu().numpy()
    exp = ref.greedy_argmax(host)
    assert got.tolist() == exp
    assert pa.device_error() == 0


def test_greedy_argmax_strided_rows_finished_and_step(cuda_device):
    rng = np.random.default_rng(5)
    b, vocab, stride = 19, 5003, 5011  # odd stride: the scalar (non-vector) path
    base = torch.from_numpy(rng.standard_normal((b, stride)).astype(np.float32)).to(torch.bfloat16)
    lg = base.to(cuda_device)[:, :vocab]
    fin = np.zeros(b, np.uint8)
    fin[[0, 7, 18]] = 1
    out = torch.full((b,), -5, dtype=torch.int32, device=cuda_device)
    step = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ws = torch.zeros(dl.greedy_argmax_workspace_bytes(b, vocab), dtype=torch.uint8, device=cuda_device)
    for call in range(3):  # the workspace counters reset themselves
        dl.greedy_argmax(lg, out=out, finished=torch.from_numpy(fin).to(cuda_device), step=step, workspace=ws)
        exp = ref.greedy_argmax(base[:, :vocab].float().numpy(), fin)
        got = out.cpu().numpy()
        for i, e in enumerate(exp):
            assert got[i] == (-5 if e is None else e)
        assert int(step.item()) == call + 1
    assert int(ws.view(torch.int32)[:b].abs().sum().item()) == 0


def test_greedy_argmax_rejects_bad_arguments(cuda_device):
    lg = torch.zeros(4, 100, device=cuda_device)
    ws = torch.zeros(16, dtype=torch.uint8, device=cuda_device)
    with pytest.raises(_lib.VasrPaError):
        dl.greedy_argmax(lg, workspace=ws)  # workspace too small
    with pytest.raises(_lib.VasrPaError):
        dl.greedy_argmax(lg.to(torch.int32))  # dtype


def _loop_case(rng, b, bs, cols, short_row=None):
    prompt = rng.integers(1, 40, b)
    need = (prompt + 30 + bs - 1) // bs
    nb = int(need.sum()) + 2
    perm = rng.permutation(np.arange(1, nb))
    tables = np.zeros((b, cols), np.int32)
    lens = need.copy()
    o = 0
    for i in range(b):
        n = int(need[i])
        tables[i, :n] = perm[o:o + n]
        o += n
    if short_row is not None:
        lens[short_row] = (prompt[short_row] + 2) // bs + 1  # runs out after a few steps
    return prompt, tables, lens, nb


@pytest.mark.parametrize("bs", [16, 8])
def test_decode_step_prepare_matches_host_loop(cuda_device, bs):
    rng = np.random.default_rng(bs)
    b, cols, steps, vocab = 9, 12, 24, 50
    eos = [3, 17]
    prompt, tables, lens, nb = _loop_case(rng, b, bs, cols)
    first = rng.integers(20, vocab, b)
    st = dl.DecodeLoopState(prompt.tolist(), first.tolist(), eos, torch.from_numpy(tables).to(cuda_device),
                            lens.tolist(), bs, nb, vocab, history_cols=16, device=cuda_device)
    host = {"prompt_lens": prompt, "next_ids": first.copy(), "finished": np.zeros(b, bool),
            "generated": np.zeros(b, np.int64), "history": np.zeros((b, 16), np.int64), "step": 0}
    for step in range(steps):
        st.prepare()
        ids, pos, slots, ctx, errs = ref.decode_step_prepare(host, eos, tables, lens, bs, nb)
        assert errs == 0
        assert st.input_ids.cpu().numpy().tolist() == ids.tolist()
        assert st.positions.cpu().numpy().tolist() == pos.tolist()
        assert st.slot_mapping.cpu().numpy().tolist() == slots.tolist()
        assert st.context_lens.cpu().numpy().astype(np.uint32).tolist() == ctx.tolist()
        assert st.finished.cpu().numpy().astype(bool).tolist() == host["finished"].tolist()
        # next tokens: random, with EOS now and then
        nxt = rng.integers(20, vocab, b)
        nxt[rng.random(b) < 0.08] = eos[step % 2]
        st.next_ids.copy_(torch.from_numpy(nxt.astype(np.int32)))
        host["next_ids"] = nxt
        st.step += 1
        host["step"] += 1
    fin, gen, hist = st.read_back()
    assert fin.numpy().tolist() == host["finished"].tolist()
    assert gen.numpy().tolist() == host["generated"].tolist()
    assert hist.numpy().tolist() == host["history"].tolist()
    assert pa.device_error() == 0


def test_decode_step_prepare_slots_match_reference_metadata(cuda_device):
    """Without EOS the prepared metadata equals decode_metadata_for_batch_step of the host mirror."""
    from vasr_paged_attn import host as vh
    g_tables, g_prompt = [[3, 4], [6, 7]], [4, 5]  # paged_kv_cache.rs:1316-1376 golden case
    cache = vh.PagedKvCache.new_pool(1, 2, 8, 4, 16, "f32")
    t = torch.tensor([r + [0] * 2 for r in g_tables], dtype=torch.int32)
    st = dl.DecodeLoopState(g_prompt, [100, 101], [0], t.to(cuda_device), [2, 2], 4, 16, 200,
                            device=cuda_device)
    for step in range(3):
        st.prepare()
        m = cache.decode_metadata_for_batch_step(g_tables, g_prompt, step, False)
        assert st.slot_mapping.cpu().tolist() == list(m.slot_mapping)
        assert st.context_lens.cpu().tolist() == list(m.context_lens)
        st.step += 1


def test_decode_step_prepare_flags_short_tables(cuda_device):
    rng = np.random.default_rng(2)
    b, bs, cols = 5, 16, 8
    prompt, tables, lens, nb = _loop_case(rng, b, bs, cols, short_row=2)
    st = dl.DecodeLoopState(prompt.tolist(), [40] * b, [1], torch.from_numpy(tables).to(cuda_device),
                            lens.tolist(), bs, nb, 64, device=cuda_device)
    host = {"prompt_lens": prompt, "next_ids": np.full(b, 40), "finished": np.zeros(b, bool),
            "generated": np.zeros(b, np.int64), "history": None, "step": 0}
    total_errs = 0
    for step in range(40):
        st.prepare()
        _, _, slots, _, errs = ref.decode_step_prepare(host, [1], tables, lens, bs, nb)
        total_errs += errs
        assert st.slot_mapping.cpu().numpy().tolist() == slots.tolist()
        st.step += 1
        host["step"] += 1
    assert total_errs > 0
    assert pa.device_error(clear=True) & _lib.DERR_SLOT_RANGE


def test_device_loop_graph_matches_host_driven_decode(cuda_device):
    """K replays of the captured prepare → forward → argmax graph generate the same tokens,
    EOS handling included, as the host-driven loop (host metadata + torch.argmax per step)."""
    from vasr_paged_attn import engine as eng
    cfg = eng.DecoderConfig(num_layers=2, vocab_size=4096)
    model = eng.RandomQwen3Decoder(cfg, cuda_device, torch.bfloat16, seed=3)
    rng = np.random.default_rng(11)
    b, bs, steps = 6, 16, 12
    prompt = rng.integers(5, 60, b)
    blocks = (prompt + steps + bs) // bs
    nb = int(blocks.sum()) + 1
    cols = int(blocks.max())
    perm = rng.permutation(np.arange(1, nb))
    tables = np.zeros((b, cols), np.int32)
    o = 0
    for i, n in enumerate(blocks):
        tables[i, :n] = perm[o:o + n]
        o += n
    first = rng.integers(0, cfg.vocab_size, b)

    def fresh_caches():
        caches = eng.allocate_paged_cache(cfg, nb, bs, cuda_device)
        g = torch.Generator(device=cuda_device).manual_seed(5)
        for kc, vc in caches:
            kc.normal_(generator=g)
            vc.normal_(generator=g)
        return caches

    # host-driven reference run; its step-3 token of row 1 becomes an EOS id
    caches = fresh_caches()
    dt = torch.from_numpy(tables).to(cuda_device)
    ids = torch.from_numpy(first).to(cuda_device)
    host_tokens = []
    for s in range(steps):
        pos = torch.from_numpy(prompt + s).to(cuda_device)
        slots = torch.from_numpy((tables[np.arange(b), (prompt + s) // bs].astype(np.int64) * bs
                                  + (prompt + s) % bs)).to(cuda_device)
        ctx = torch.from_numpy((prompt + s + 1).astype(np.int32)).to(cuda_device)
        ids = model.decode_step(ids, pos, caches, slots, dt, ctx, cols * bs)
        host_tokens.append(ids.cpu().numpy().copy())
    host_tokens = np.stack(host_tokens, 1)  # [B, steps]
    eos = int(host_tokens[1, 3])

    caches = fresh_caches()
    st = dl.DecodeLoopState(prompt.tolist(), first.tolist(), [eos], dt, blocks.tolist(), bs, nb,
                            cfg.vocab_size, history_cols=steps + 1, device=cuda_device)
    loop = eng.DecodeLoopGraph(model, caches, st, bs)
    loop.capture()
    for _ in range(steps):
        loop.replay()
    fin, gen, hist = st.read_back()
    loop.release()
    # history[:, 0] is the first fed token; history[:, s + 1] is the token generated at step s
    for i in range(b):
        fed = [int(first[i])] + [int(t) for t in host_tokens[i]]
        if eos in fed[:steps]:
            cut = fed.index(eos)
            assert bool(fin[i]) and int(gen[i]) == cut
            assert hist[i, :cut].tolist() == fed[:cut]
        else:
            assert not bool(fin[i]) and int(gen[i]) == steps
            assert hist[i, :steps].tolist() == fed[:steps]
