"""The allocation-free decode entry point, called through the C ABI.

vasr_pa_paged_attention_noalloc exists for callers that cannot allocate
device memory where they run decode attention (a plugin enqueue path, a
fixed-budget host framework, a real-time thread that must not block in the
allocator). Its split-K scratch is a fixed 16 MiB buffer inside the library
instead of a caller workspace. This test checks, on calls in a row whose
(sequence x kv head) footprints grow and then shrink, that its output is
bit-identical to vasr_pa_paged_attention given a regular workspace (the same
kernel with the same split order, so nothing less than equality is right),
that both are within the bf16 tolerance of the other decode tests (2e-2) of
the oracle, and that sizes beyond the fixed buffer are rejected. The file is
named to be collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from cases import appended, make_decode_case, oracle_decode
from vasr_paged_attn import _lib

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2


def _dev_bf16(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy()).view(torch.bfloat16).to(dev)


def _args(case, dev):
    return dict(
        q=_dev_bf16(case.q, dev), kc=_dev_bf16(case.key_cache, dev), vc=_dev_bf16(case.value_cache, dev),
        bt=torch.from_numpy(case.block_tables.astype(np.int32)).to(dev),
        ctx=torch.from_numpy(case.context_lens.astype(np.int32)).to(dev),
    )


def _call(lib, fn_name, out, t, case, mcl, stream, ws=None):
    b, hq, d = case.q.shape
    common = [out.data_ptr(), t["q"].data_ptr(), t["kc"].data_ptr(), t["vc"].data_ptr(),
              t["bt"].data_ptr(), t["ctx"].data_ptr(), b, hq, case.num_kv_heads, d, case.block_size,
              case.num_blocks, case.block_tables.shape[1], mcl, d ** -0.5, 1.0, hq * d, _lib.BF16]
    if fn_name == "vasr_pa_paged_attention":
        return lib.vasr_pa_paged_attention(*common, ws.data_ptr(), ws.numel(), stream)
    return lib.vasr_pa_paged_attention_noalloc(*common, stream)


def test_noalloc_decode_matches_workspace_entry_point(cuda_device):
    lib = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    assert lib.vasr_pa_noalloc_scratch_bytes() == 16 << 20
    # different calls in a row: none may see an earlier call's leftovers in the shared scratch
    for seed, cached in ((21, [40, 300, 1500, 700]), (22, [1023, 5, 257, 64, 2000, 900]),
                         (23, [3000, 17])):
        case = appended(make_decode_case(seed, cached, dtype="bf16", num_blocks=512))
        t = _args(case, cuda_device)
        mcl = int(case.context_lens.max())
        need = lib.vasr_pa_paged_attention_workspace_size(len(cached), 16, 8, 128, 16, mcl, _lib.BF16)
        ws = torch.zeros(need, dtype=torch.uint8, device=cuda_device)
        ref_out = torch.empty(len(cached), 16, 128, dtype=torch.bfloat16, device=cuda_device)
        out = torch.empty_like(ref_out)
        assert _call(lib, "vasr_pa_paged_attention", ref_out, t, case, mcl, stream, ws) == _lib.OK
        assert _call(lib, "vasr_pa_paged_attention_noalloc", out, t, case, mcl, stream) == _lib.OK
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16))
        got = out.float().cpu().numpy()
        oracle, _, _ = oracle_decode(case, after_append=False)
        assert np.abs(got - oracle).max() <= BF16_TOL


def test_noalloc_rejects_sizes_beyond_the_fixed_scratch(cuda_device):
    lib = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    p = ctypes.c_void_p(256)  # never touched: the size check comes first
    big_b, big_ctx = 4096, 65536
    assert lib.vasr_pa_paged_attention_workspace_size(big_b, 16, 8, 128, 16, big_ctx, _lib.BF16) > (16 << 20)
    st = lib.vasr_pa_paged_attention_noalloc(p, p, p, p, p, p, big_b, 16, 8, 128, 16, 100000, 4096,
                                             big_ctx, 0.088, 1.0, 2048, _lib.BF16, stream)
    assert st == _lib.ESCRATCH_LIMIT
    assert "no-alloc" in _lib.status_string(st)
