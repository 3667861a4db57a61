"""Pin the host logic against the reference's own known-answer vectors.

The same checks run on two implementations:
  * ``oracle``  — the Python restatement in oracle/paged_ref.py (test infra);
  * ``host``    — the C++ host mirror of vasr-paged-attn (product), through
                  its pybind11 module, once built.
Each test mirrors one Rust #[test] of the reference; the vectors live in
tests/golden/reference_vectors.json with their source file:line.
"""
import json
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest

import paged_ref as ref

GOLD = json.loads((Path(__file__).parent / "golden" / "reference_vectors.json").read_text())
DT_BYTES = {"f32": 4, "bf16": 2, "f16": 2}


def _oracle_api():
    return SimpleNamespace(
        name="oracle",
        new=lambda l, h, d, bs, mt, dt: ref.PagedKvCacheRef.new(l, h, d, bs, mt, DT_BYTES[dt]),
        new_batched=lambda l, h, d, bs, b, mt, dt: ref.PagedKvCacheRef.new_batched(l, h, d, bs, b, mt, DT_BYTES[dt]),
        new_pool=lambda l, h, d, bs, nb, dt: ref.PagedKvCacheRef.new_pool(l, h, d, bs, nb, DT_BYTES[dt]),
        BlockManager=ref.PagedBlockManagerRef,
        bytes_per_paged_block=ref.bytes_per_paged_block,
        blocks_for_byte_budget=ref.blocks_for_byte_budget,
        cuda_graph_batch_bucket=ref.cuda_graph_batch_bucket,
        cuda_graph_batch_buckets=ref.cuda_graph_batch_buckets,
        bucket_block_table_cols=ref.bucket_block_table_cols,
        pad_decode_batch_to_max=ref.pad_decode_batch_to_max,
        can_admit=lambda mgr, cap, plen, used, running: ref.can_admit_with_projected_kv(
            mgr.block_size, cap, plen, used, running),
        allocatable_block_capacity=lambda nb: max(nb - 1, 0),
        graph_key=None,
        Error=ref.OracleError,
    )


def host_golden_api():
    """The C++ host mirror behind the same adapter shape as the oracle's."""
    from vasr_paged_attn import host  # C++ mirror; raises if the module is missing

    return SimpleNamespace(
        name="host",
        new=lambda l, h, d, bs, mt, dt: host.PagedKvCache.new(l, h, d, bs, mt, dt),
        new_batched=lambda l, h, d, bs, b, mt, dt: host.PagedKvCache.new_batched(l, h, d, bs, b, mt, dt),
        new_pool=lambda l, h, d, bs, nb, dt: host.PagedKvCache.new_pool(l, h, d, bs, nb, dt),
        BlockManager=host.PagedBlockManager,
        bytes_per_paged_block=host.bytes_per_paged_block,
        blocks_for_byte_budget=host.blocks_for_byte_budget,
        cuda_graph_batch_bucket=host.cuda_graph_batch_bucket,
        cuda_graph_batch_buckets=host.cuda_graph_batch_buckets,
        bucket_block_table_cols=host.bucket_block_table_cols,
        pad_decode_batch_to_max=host.pad_decode_batch_to_max,
        can_admit=host.can_admit_with_projected_kv,
        allocatable_block_capacity=host.PagedBlockManager.allocatable_block_capacity,
        graph_key=host.DecodeGraphRegistry,
        Error=host.VasrHostError,
    )


def _host_api():
    return host_golden_api()


def _apis():
    out = [pytest.param(_oracle_api, id="oracle")]
    out.append(pytest.param(_host_api, id="host"))
    return out


@pytest.fixture(params=_apis())
def api(request):
    try:
        return request.param()
    except ImportError as e:  # host module not built in this checkout
        pytest.fail(f"host mirror unavailable: {e}")


def test_paged_cache_single_sequence_layout(api):
    g = GOLD["single_sequence_layout"]
    c = api.new(*g["new"])
    assert c.block_size == g["block_size"]
    assert c.num_blocks == g["num_blocks"]
    assert list(c.block_table_host()) == g["block_table_host"]
    for pos, slot in g["slot_for_position"]:
        assert c.slot_for_position(pos) == slot


def test_paged_cache_metadata_tensors(api):
    g = GOLD["metadata_tensors"]
    c = api.new(*g["new"])
    r = g["slot_mapping_for_range"]
    assert list(c.slot_mapping_for_range(r["start"], r["len"])) == r["expect"]
    assert [list(x) for x in c.block_tables_tensor()] == g["block_tables_tensor"]
    assert list(c.context_lens_tensor(g["context_lens_tensor"]["context_len"])) == g["context_lens_tensor"]["expect"]
    assert list(c.key_shape) == g["key_dims"]
    assert list(c.value_shape) == g["value_dims"]


def test_paged_cache_multi_sequence_layout(api):
    g = GOLD["multi_sequence_layout"]
    c = api.new_batched(*g["new_batched"])
    assert c.batch_size == g["batch_size"]
    assert c.max_tokens_per_sequence == g["max_tokens_per_sequence"]
    assert c.num_blocks_per_sequence == g["num_blocks_per_sequence"]
    assert c.num_blocks == g["num_blocks"]
    for seq, pos, slot in g["slot_for_sequence_position"]:
        assert c.slot_for_sequence_position(seq, pos) == slot
    br = g["batch_ranges"]
    m = c.input_metadata_for_batch_ranges(br["starts"], br["len"], br["context_lens"])
    assert list(m.slot_mapping) == br["slot_mapping"]
    assert [list(x) for x in m.block_tables] == br["block_tables"]
    assert list(m.context_lens) == br["context_lens_out"]
    assert m.max_context_len == br["max_context_len"]


def test_paged_cache_metadata_from_physical_block_tables(api):
    g = GOLD["physical_block_tables"]
    c = api.new_pool(*g["new_pool"])
    m = c.input_metadata_from_block_tables(g["block_tables"], g["starts"], g["len"], g["context_lens"])
    assert list(m.slot_mapping) == g["slot_mapping"]
    assert [list(x) for x in m.block_tables] == g["block_tables_out"]
    assert list(m.context_lens) == g["context_lens_out"]
    assert m.max_context_len == g["max_context_len"]


def test_paged_cache_metadata_from_attention_masks_tracks_query_lens(api):
    g = GOLD["attention_masks"]
    c = api.new_pool(*g["new_pool"])
    m = c.input_metadata_from_attention_masks(g["block_tables"], g["masks"])
    assert list(m.slot_mapping) == g["slot_mapping"]
    assert [list(r) for r in m.token_attention_mask] == g["masks"]
    assert list(m.context_lens) == g["context_lens"]
    assert list(m.query_lens) == g["query_lens"]
    assert list(m.kv_lens) == g["kv_lens"]
    assert list(m.cu_seqlens_q) == g["cu_seqlens_q"]
    assert list(m.cu_seqlens_kv) == g["cu_seqlens_kv"]
    assert m.max_query_len == g["max_query_len"]
    assert m.max_kv_len == g["max_kv_len"]
    assert m.max_context_len == g["max_context_len"]
    assert m.prefill_causal_only == g["prefill_causal_only"]
    f = m.flash_params(True)
    fe = g["flash_params_causal"]
    assert (f.max_q, f.max_k, f.causal) == (fe["max_q"], fe["max_k"], fe["causal"])
    assert list(f.cumulative_seqlens_q) == fe["cu_q"]
    assert list(f.cumulative_seqlens_k) == fe["cu_k"]


def test_decode_metadata_for_steps_matches_per_step_builder(api):
    g = GOLD["decode_steps_single"]
    c = api.new_pool(*g["new_pool"])
    pre = c.decode_metadata_for_steps(g["prompt_len"], g["steps"])
    for step in range(g["steps"]):
        exp = c.input_metadata_for_range(g["prompt_len"] + step, 1, g["prompt_len"] + step + 1)
        act = pre[step]
        assert list(act.slot_mapping) == list(exp.slot_mapping)
        assert list(act.context_lens) == list(exp.context_lens)
        assert act.max_context_len == exp.max_context_len
        assert act.cu_seqlens_q is None and act.cu_seqlens_kv is None


def test_paged_cache_metadata_from_query_lens_is_packed(api):
    g = GOLD["query_lens_packed"]
    c = api.new_pool(*g["new_pool"])
    m = c.input_metadata_from_query_lens(g["block_tables"], g["query_lens"])
    assert list(m.slot_mapping) == g["slot_mapping"]
    assert [list(x) for x in m.block_tables] == g["block_tables_out"]
    assert list(m.context_lens) == g["context_lens"]
    assert m.max_context_len == g["max_context_len"]
    assert list(m.query_lens) == g["query_lens"]
    assert list(m.kv_lens) == g["kv_lens"]
    assert m.token_attention_mask is None
    assert m.prefill_causal_only == g["prefill_causal_only"]


@pytest.mark.parametrize("cuda_graph", [False, True])
def test_decode_metadata_for_batch_steps_matches_per_step_builder(api, cuda_graph):
    g = GOLD["decode_batch_steps"]
    c = api.new_pool(*g["new_pool"])
    pre = c.decode_metadata_for_batch_steps(g["block_tables"], g["prompt_lens"], g["steps"], cuda_graph)
    tables = g["block_tables"]
    if cuda_graph:
        cols = api.bucket_block_table_cols(max(len(t) for t in tables), c.block_size)
        tables = [list(t) + [0] * (cols - len(t)) for t in tables]
    for step in range(g["steps"]):
        starts = [p + step for p in g["prompt_lens"]]
        ctx = [p + step + 1 for p in g["prompt_lens"]]
        exp = c.input_metadata_from_block_tables(tables, starts, 1, ctx)
        act = pre[step]
        assert list(act.slot_mapping) == list(exp.slot_mapping)
        assert [list(x) for x in act.block_tables] == [list(x) for x in exp.block_tables]
        assert list(act.context_lens) == list(exp.context_lens)
        assert act.max_context_len == exp.max_context_len
        assert act.cu_seqlens_q is None and act.cu_seqlens_kv is None
        one = c.decode_metadata_for_batch_step(g["block_tables"], g["prompt_lens"], step, cuda_graph)
        assert list(one.slot_mapping) == list(act.slot_mapping)


def test_bytes_per_paged_block_matches_qwen3_asr_defaults(api):
    g = GOLD["bytes_per_paged_block"]
    assert api.bytes_per_paged_block(*g["args"]) == g["expect"]


def test_blocks_for_byte_budget_reserves_null_block(api):
    g = GOLD["blocks_for_byte_budget"]
    bpb = api.bytes_per_paged_block(28, 8, 128, 32, 2)
    assert api.blocks_for_byte_budget(bpb * g["budget_blocks"], bpb) == g["expect"]


@pytest.mark.parametrize("case", ["block_manager_allocate_extend_free", "block_manager_trim",
                                  "block_manager_exhaustion"])
def test_block_manager_scripts(api, case):
    g = GOLD[case]
    m = api.BlockManager(*g["new"])
    for step in g["script"]:
        op = step[0]
        if op == "free":
            assert m.free_blocks() == step[1]
        elif op == "allocate":
            m.allocate_slots(step[1], step[2])
        elif op == "blocks":
            assert len(m.block_ids(step[1])) == step[2]
        elif op == "free_request":
            m.free_request(step[1])
        elif op == "trim":
            m.trim_request_to_num_tokens(step[1], step[2])
        elif op == "try_allocate":
            assert m.try_allocate_slots(step[1], step[2]) == step[3]


def test_block_manager_free_list_order(api):
    # free/trim return blocks in reverse order to the back of the FIFO (paged_cache_runtime.rs:320-357)
    m = api.BlockManager(8, 4)
    m.allocate_slots(1, 12)
    assert list(m.block_ids(1)) == [1, 2, 3]
    m.free_request(1)
    m.allocate_slots(2, 28)
    assert list(m.block_ids(2)) == [4, 5, 6, 7, 3, 2, 1]


def test_cuda_graph_batch_bucket_matches_osc_transformers_schedule(api):
    for actual, mx, exp in GOLD["cuda_graph_batch_bucket"]["cases"]:
        assert api.cuda_graph_batch_bucket(actual, mx) == exp


def test_cuda_graph_batch_buckets_include_configured_max_batch(api):
    for mx, exp in GOLD["cuda_graph_batch_buckets"]["cases"]:
        assert list(api.cuda_graph_batch_buckets(mx)) == exp


def test_block_table_bucket_uses_kernel_friendly_power_of_two_widths(api):
    for blocks, bs, exp in GOLD["bucket_block_table_cols"]["cases"]:
        assert api.bucket_block_table_cols(blocks, bs) == exp


def test_pad_decode_batch_uses_valid_dummy_rows_for_cuda_graph_capture(api):
    g = GOLD["pad_decode_batch"]
    ids, slots, ctx, tables = api.pad_decode_batch_to_max(
        g["max_batch"], g["input_ids"], g["slot_mapping"], g["context_lens"], g["block_tables"], g["cols"])
    assert list(ids) == g["ids_out"]
    assert list(slots) == g["slots_out"]
    assert list(ctx) == g["context_lens_out"]
    assert [list(r) for r in tables] == g["block_tables_out"]


def test_projected_kv_admission_respects_block_capacity(api):
    g = GOLD["projected_kv_admission"]
    m = api.BlockManager(g["num_blocks"], g["block_size"])
    cap = api.allocatable_block_capacity(g["num_blocks"])
    assert cap == g["capacity"]
    for plen, used, running, exp in g["cases"]:
        assert api.can_admit(m, cap, plen, used, running) == exp


def test_cuda_graph_disable_is_scoped_to_the_padded_key(api):
    if api.graph_key is None:
        pytest.skip("graph-key registry lives in the host mirror only")
    g = GOLD["graph_key_scope"]
    reg = api.graph_key(g["block_size"], g["max_batch"])
    assert tuple(reg.key(g["batch"], g["cols"])) == tuple(g["expect_key"])
    assert reg.enabled_for(g["batch"], g["cols"])
    reg.disable_for(g["batch"], g["cols"])
    assert not reg.enabled_for(g["batch"], g["cols"])
    assert reg.enabled_for(g["smaller_batch"], g["cols"])


def test_metadata_errors_mirror_reference_bails(api):
    c = api.new_pool(1, 2, 8, 4, 8, "f32")
    with pytest.raises(api.Error):
        c.input_metadata_from_block_tables([[3, 9]], [4], 1, [5])  # block id >= num_blocks
    with pytest.raises(api.Error):
        c.input_metadata_from_query_lens([[3]], [5])  # table too short
    with pytest.raises(api.Error):
        c.input_metadata_from_query_lens([[3]], [0])  # zero-length query
    with pytest.raises(api.Error):
        api.new_pool(1, 2, 6, 4, 8, "f32")  # head_dim not divisible by x=4


# ------------------------------------------------------------------ attention
def _packed_case():
    g = GOLD["packed_varlen_attention"]
    b, s, d, h, kvh = g["batch"], g["seq_len"], g["head_dim"], g["num_heads"], g["num_kv_heads"]
    q = (np.arange(b * h * s * d, dtype=np.float32) * np.float32(g["q_step"])).reshape(b, h, s, d)
    total = sum(g["kv_lens"])
    packed = (np.arange(total * kvh * d, dtype=np.float32) * np.float32(g["kv_step"]) +
              np.float32(g["kv_offset"])).reshape(total, kvh, d)
    return g, q, packed


def test_packed_varlen_attention_matches_unpacked_reference():
    """attention.rs:950-1041 restated on the numpy oracle (<= 1e-4 in f32)."""
    g, q, packed = _packed_case()
    k = packed[None].transpose(0, 2, 1, 3)
    cu = ref.cumulative_seqlens_from_lengths(g["query_lens"])
    cuk = ref.cumulative_seqlens_from_lengths(g["kv_lens"])
    scale = 1.0 / np.sqrt(g["head_dim"])
    got = ref.packed_varlen_attention(q, k, k, cu, cuk, scale, True, 2, dtype=np.float32)
    rows, start = [], 0
    for r, (ql, kl) in enumerate(zip(g["query_lens"], g["kv_lens"])):
        kr = packed[start:start + kl][None].transpose(0, 2, 1, 3)
        ke = ref.repeat_kv(kr, 2)
        w = (q[r:r + 1, :, :ql] @ ke.transpose(0, 1, 3, 2)) * np.float32(scale)
        w = w + ref.make_causal_mask(1, ql)
        o = ref.softmax_last_dim(w) @ ke
        rows.append(np.concatenate([o, np.zeros((1, g["num_heads"], g["seq_len"] - ql, g["head_dim"]),
                                                np.float32)], axis=2))
        start += kl
    assert np.abs(got - np.concatenate(rows)).max() <= g["tolerance"]


def test_cached_causal_mask_semantics():
    """make_causal_mask_cached (attention.rs:86-149): key j visible to query q iff j <= cache_len + q."""
    m = ref.make_causal_mask_cached(1, 3, 2)[0, 0]
    assert m.shape == (2, 5)
    assert (m[0] == 0).tolist() == [True, True, True, True, False]
    assert (m[1] == 0).tolist() == [True] * 5
    assert m[0, 4] == np.finfo(np.float32).min


def _dense_decode(q, k_tok, v_tok, scale):
    """float64 dense reference: q [Hq, D], k/v [n, Hkv, D]."""
    hq, hkv = q.shape[0], k_tok.shape[1]
    out = np.empty_like(q, dtype=np.float64)
    for h in range(hq):
        kv = h // (hq // hkv)
        w = (k_tok[:, kv].astype(np.float64) @ q[h].astype(np.float64)) * scale
        w = np.exp(w - w.max())
        out[h] = (w / w.sum()) @ v_tok[:, kv].astype(np.float64)
    return out


def test_c_oracle_decode_matches_numpy_restatement():
    from cases import make_decode_case, oracle_decode

    case = make_decode_case(3, (5, 16, 33), dtype="f32", num_blocks=32)
    got32, kc, vc = oracle_decode(case, use_double=False)
    got64, _, _ = oracle_decode(case, use_double=True)
    kf, vf = case.as_f32(kc), case.as_f32(vc)
    qf = case.as_f32(case.q)
    scale = case.head_dim ** -0.5
    for b in range(len(case.context_lens)):
        n = int(case.context_lens[b])
        ktok = np.stack([kf[case.block_tables[b, t // 16], :, :, t % 16, :].reshape(case.num_kv_heads, -1)
                         for t in range(n)])
        vtok = np.stack([vf[case.block_tables[b, t // 16], :, :, t % 16] for t in range(n)])
        exp = _dense_decode(qf[b], ktok, vtok, scale)
        assert np.abs(got64[b] - exp).max() < 1e-6
        assert np.abs(got32[b] - exp).max() < 1e-4
    # no NaN sentinel leaked in from unused slots
    assert np.isfinite(got32).all()


def test_c_oracle_prefill_last_row_equals_decode():
    """A prefill chunk's last query row is a decode over the full context."""
    from cases import make_decode_case

    case = make_decode_case(4, (20, 40), dtype="f32", num_blocks=16)
    kc, vc = case.key_cache.copy(), case.value_cache.copy()
    ref.reshape_and_cache(case.k_new, case.v_new, kc, vc, case.slots, 16)
    kf, vf = np.ascontiguousarray(case.as_f32(kc)), np.ascontiguousarray(case.as_f32(vc))
    qf = np.ascontiguousarray(case.as_f32(case.q))
    dec = ref.paged_attention(qf, kf, vf, case.block_tables, case.context_lens, 128 ** -0.5)
    cu = np.array([0, 1, 2], dtype=np.uint32)
    pre = ref.prefill_varlen(qf, kf, vf, case.block_tables, case.context_lens, cu, 128 ** -0.5)
    assert np.abs(pre - dec).max() < 1e-6


def test_c_oracle_reshape_and_cache_layout():
    """Bit-level check of the scatter against the layout formula of paged_kv_cache.rs:285-294."""
    rng = np.random.default_rng(0)
    nb, h, d, bs = 6, 2, 8, 4
    key = rng.integers(0, 2**32, size=(5, h, d), dtype=np.uint32)
    val = rng.integers(0, 2**32, size=(5, h, d), dtype=np.uint32)
    kc = np.zeros((nb, h, d // 4, bs, 4), np.uint32)
    vc = np.zeros((nb, h, d, bs), np.uint32)
    slots = np.array([0, 7, -1, 13, 23], dtype=np.int64)
    ref.reshape_and_cache(key, val, kc, vc, slots, bs)
    for t, s in enumerate(slots):
        if s < 0:
            continue
        for hh in range(h):
            for dd in range(d):
                assert kc[s // bs, hh, dd // 4, s % bs, dd % 4] == key[t, hh, dd]
                assert vc[s // bs, hh, dd, s % bs] == val[t, hh, dd]
    assert np.count_nonzero(kc) == 4 * h * d


def test_decode_step_prepare_oracle_matches_batch_step_metadata(api):
    """The device loop's host restatement reproduces decode_metadata_for_batch_step
    (paged_kv_cache.rs:1316-1376 golden case) while no row has finished."""
    g = GOLD["decode_batch_steps"]
    c = api.new_pool(*g["new_pool"])
    tables = np.array([t + [0] * 2 for t in g["block_tables"]], np.int64)
    state = {"prompt_lens": np.array(g["prompt_lens"]), "next_ids": np.array([7, 8]),
             "finished": np.zeros(2, bool), "generated": np.zeros(2, np.int64),
             "history": np.zeros((2, 4), np.int64), "step": 0}
    for step in range(g["steps"]):
        ids, pos, slots, ctx, errs = ref.decode_step_prepare(state, [0], tables, [2, 2], c.block_size,
                                                             g["new_pool"][4])
        m = c.decode_metadata_for_batch_step(g["block_tables"], g["prompt_lens"], step, False)
        assert errs == 0
        assert slots.tolist() == list(m.slot_mapping)
        assert ctx.tolist() == list(m.context_lens)
        assert pos.tolist() == [p + step for p in g["prompt_lens"]]
        state["step"] += 1
    assert state["history"][:, :3].tolist() == [[7, 7, 7], [8, 8, 8]]


def test_decode_step_prepare_oracle_finished_rows_are_graph_padding():
    """A row fed an EOS id turns into the padding row of pad_decode_batch_to_max
    (cuda_graph.rs:690-763 golden case: id 0, slot 0, context 1)."""
    g = GOLD["pad_decode_batch"]
    state = {"prompt_lens": np.array([5, 6, 7]), "next_ids": np.array([11, 2, 33]),
             "finished": np.zeros(3, bool), "generated": np.zeros(3, np.int64), "history": None, "step": 0}
    tables = np.array(g["block_tables"], np.int64)
    ids, pos, slots, ctx, _ = ref.decode_step_prepare(state, [2], tables, None, 16, 64)
    assert state["finished"].tolist() == [False, True, False]
    pad_ids = g["ids_out"][len(g["input_ids"]):]
    assert (ids[1], slots[1], ctx[1]) == (pad_ids[0], g["slots_out"][-1], g["context_lens_out"][-1])
    assert pos[1] == 0
