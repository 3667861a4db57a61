"""The C++ host entry points (``host.cpp_ops``, csrc/host/ops.cpp) on the GPU.

ops.cpp is the C++ side above the C ABI with the argument order of the
reference's ``mistralrs_paged_attn`` calls (thinker_text.rs:1101-1109 and
:1126-1139): it checks tensor views and forwards to vasr_pa_*. Its results
must equal the Python binding's bit for bit (same kernels, same inputs) and
match the oracle.
"""
import numpy as np
import pytest
import torch

from cases import make_decode_case, oracle_decode
from vasr_paged_attn import host
from vasr_paged_attn import mistralrs_paged_attn as pa

pytestmark = pytest.mark.gpu


def _bf16(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy()).view(torch.bfloat16).to(dev)


def test_cpp_ops_append_and_decode_match_the_python_binding(cuda_device):
    case = make_decode_case(70, [37, 300, 1023, 1500], dtype="bf16", num_blocks=256)
    dev = cuda_device
    stream = torch.cuda.current_stream(dev).cuda_stream
    res = []
    for path in ("cpp", "py"):
        kc, vc = _bf16(case.key_cache, dev), _bf16(case.value_cache, dev)
        k, v, q = _bf16(case.k_new, dev), _bf16(case.v_new, dev), _bf16(case.q, dev)
        slots = torch.from_numpy(case.slots).to(dev)
        bt = torch.from_numpy(case.block_tables.astype(np.int32)).to(dev)
        ctx = torch.from_numpy(case.context_lens.astype(np.int32)).to(dev)
        mcl = int(case.context_lens.max())
        out = torch.empty_like(q)
        if path == "cpp":
            ops = host.cpp_ops
            ops.reshape_and_cache(k.data_ptr(), v.data_ptr(), kc.data_ptr(), vc.data_ptr(), slots.data_ptr(),
                                  list(k.shape), list(kc.shape), list(vc.shape), "bf16", dev.index, stream)
            need = pa.paged_attention_workspace_bytes(q.shape[0], 16, 8, 128, 16, mcl, torch.bfloat16)
            ws = torch.zeros(need, dtype=torch.uint8, device=dev)
            ops.paged_attention(out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(),
                                ctx.data_ptr(), list(q.shape), list(kc.shape), list(vc.shape), bt.shape[1], mcl,
                                128 ** -0.5, 1.0, "bf16", dev.index, ws.data_ptr(), ws.numel(), stream)
        else:
            pa.reshape_and_cache(k, v, None, None, kc, vc, slots)
            pa.paged_attention(q, None, None, kc, vc, bt, ctx, None, mcl, 128 ** -0.5, 1.0, None, out=out)
        torch.cuda.synchronize()
        res.append((kc.view(torch.int16).cpu(), vc.view(torch.int16).cpu(), out.view(torch.int16).cpu()))
    for a, b in zip(res[0], res[1]):
        assert torch.equal(a, b)
    exp, kc_ref, _ = oracle_decode(case)
    assert np.array_equal(res[0][0].numpy().view(np.uint16), kc_ref)
    assert np.abs(res[0][2].view(torch.bfloat16).float().numpy() - exp).max() <= 2e-2


def test_cpp_ops_reject_bad_views_before_launching(cuda_device):
    with pytest.raises(host.VasrHostError):
        host.cpp_ops.reshape_and_cache(256, 256, 256, 256, 256, [4, 8, 128], [16, 8, 16, 16, 8],
                                       [16, 8, 64, 16], "bf16", cuda_device.index, 0)
