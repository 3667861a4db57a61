"""Parity of the varlen chunked-prefill kernel against the oracle's cached causal mask.

bf16/f16 run the tensor-core kernel (tolerance 2e-2 against the f64 oracle on
the same bf16-rounded inputs); f32 runs the CUDA-core kernel (1e-4).
"""
import numpy as np
import pytest
import torch

from cases import config3_rounds, make_prefill_case, oracle_prefill
from vasr_paged_attn import mistralrs_paged_attn as pa

pytestmark = pytest.mark.gpu

TOL = {"bf16": 2e-2, "f32": 1e-4}


def to_dev(bits, dtype, dev):
    bits = np.ascontiguousarray(bits)
    if dtype == "f32":
        return torch.from_numpy(bits.view(np.float32).copy()).to(dev)
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(dev)


def run_prefill(case, dev, softcap=1.0):
    q = to_dev(case.q, case.dtype, dev)
    kc = to_dev(case.key_cache, case.dtype, dev)
    vc = to_dev(case.value_cache, case.dtype, dev)
    bt = torch.from_numpy(case.block_tables.astype(np.int32)).to(dev)
    ctx = torch.from_numpy(case.context_lens.astype(np.int32)).to(dev)
    cu = torch.from_numpy(case.cu_q.astype(np.int32)).to(dev)
    out = pa.paged_attention_varlen_prefill(q, kc, vc, bt, ctx, cu, None, None, case.head_dim ** -0.5,
                                            softcap)
    return out.float().cpu().numpy()


@pytest.fixture(autouse=True)
def _clear(cuda_device):
    pa.device_error(clear=True)
    yield
    assert pa.device_error() == 0


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("block_size", [8, 16, 32])
def test_prefill_ragged_chunks(cuda_device, dtype, block_size):
    # whole prompts (cached 0), chunks behind a cache, single-token chunks, page-straddling offsets
    cached = [0, 0, 256, 13, 100, 0, 511]
    chunk = [1, 77, 256, 40, 1, 129, 70]
    case = make_prefill_case(3, cached, chunk, dtype=dtype, block_size=block_size)
    got = run_prefill(case, cuda_device)
    exp = oracle_prefill(case)
    assert np.abs(got - exp).max() <= TOL[dtype]


@pytest.mark.parametrize("gqa", [1, 2, 4])
def test_prefill_gqa_groups(cuda_device, gqa):
    case = make_prefill_case(4, [0, 30, 200], [90, 64, 33], dtype="bf16", num_heads=8 * gqa)
    assert np.abs(run_prefill(case, cuda_device) - oracle_prefill(case)).max() <= TOL["bf16"]


def test_prefill_softcap(cuda_device):
    case = make_prefill_case(5, [10, 0], [50, 31], dtype="bf16")
    got = run_prefill(case, cuda_device, softcap=8.0)
    assert np.abs(got - oracle_prefill(case, softcap=8.0)).max() <= TOL["bf16"]


def test_prefill_last_row_matches_decode(cuda_device):
    """The last query row of a chunk equals single-token decode over the full context."""
    case = make_prefill_case(6, [300, 45], [64, 20], dtype="bf16")
    got = run_prefill(case, cuda_device)
    q = to_dev(case.q, "bf16", cuda_device)
    last = torch.tensor([int(case.cu_q[1]) - 1, int(case.cu_q[2]) - 1], device=cuda_device)
    dec = pa.paged_attention(q[last].contiguous(), None, None, to_dev(case.key_cache, "bf16", cuda_device),
                             to_dev(case.value_cache, "bf16", cuda_device),
                             torch.from_numpy(case.block_tables.astype(np.int32)).to(cuda_device),
                             torch.from_numpy(case.context_lens.astype(np.int32)).to(cuda_device), None,
                             int(case.context_lens.max()), 128 ** -0.5, 1.0, None).float().cpu().numpy()
    assert np.abs(got[last.cpu().numpy()] - dec).max() <= 2e-2


def test_prefill_config3_first_rounds(cuda_device):
    """Config 3: 32 prompts ~U[100, 800] in 256-token chunks; rounds 0 and 1 (seed 0)."""
    lens, rounds = config3_rounds(0)
    for r in rounds[:2]:
        cached = [start for (_, start, _) in r]
        chunk = [n for (_, _, n) in r]
        case = make_prefill_case(10 + len(r), cached, chunk, dtype="bf16")
        assert np.abs(run_prefill(case, cuda_device) - oracle_prefill(case)).max() <= TOL["bf16"]


def test_prefill_max_query_len_bound(cuda_device):
    """max_query_len 0 means unknown (worst-case schedule); too small a bound is flagged."""
    case = make_prefill_case(7, [0, 40, 7], [150, 3, 64], dtype="bf16")
    exp = oracle_prefill(case)
    args = (to_dev(case.q, "bf16", cuda_device), to_dev(case.key_cache, "bf16", cuda_device),
            to_dev(case.value_cache, "bf16", cuda_device),
            torch.from_numpy(case.block_tables.astype(np.int32)).to(cuda_device),
            torch.from_numpy(case.context_lens.astype(np.int32)).to(cuda_device),
            torch.from_numpy(case.cu_q.astype(np.int32)).to(cuda_device), None, None, 128 ** -0.5, 1.0)
    got = pa.paged_attention_varlen_prefill(*args, 0).float().cpu().numpy()
    assert np.abs(got - exp).max() <= TOL["bf16"]
    assert pa.device_error() == 0
    pa.paged_attention_varlen_prefill(*args, 20)
    assert pa.device_error(clear=True) & 0x20  # VASR_PA_DERR_QLEN_RANGE


@pytest.mark.parametrize("cached,chunk", [([1500, 20], [12, 9]), ([780], [12]), ([900, 600, 64], [3, 40, 1])])
def test_prefill_split_items_long_context(cuda_device, cached, chunk):
    """Few items over long contexts: each item's key tiles are shared by a cluster of CTAs
    (up to 8, combined through distributed shared memory). Short sequences next to a long one
    have fewer key tiles than CTAs in their cluster, so some CTAs hold none."""
    case = make_prefill_case(7, cached, chunk, dtype="bf16")
    got = run_prefill(case, cuda_device)
    assert np.abs(got - oracle_prefill(case)).max() <= TOL["bf16"]
