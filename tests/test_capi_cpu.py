"""C-ABI checks that need no GPU: the library loads, exports every symbol that
include/vasr_pa.h declares, and rejects bad arguments on the host before any
CUDA call (status codes mirror the reference's bail! checks)."""
import ctypes
import re
from pathlib import Path

import pytest

from vasr_paged_attn import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "vasr_pa.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(vasr_pa_[a-z_0-9]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), f"{n} declared in vasr_pa.h but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_abi_version_and_status_strings():
    lib = _lib.lib()
    assert lib.vasr_pa_abi_version() == 1
    assert _lib.status_string(_lib.EINVAL_BLOCKSIZE) == "paged cache block size must be 8, 16, or 32"
    assert _lib.status_string(0) == "ok"


def test_append_rejects_bad_arguments_before_any_cuda_call():
    f = _lib.lib().vasr_pa_reshape_and_cache
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    # bad block size (paged_cache_runtime.rs:406-411)
    assert f(p, p, p, p, p, 4, 8, 128, 12, 10, 1024, 1024, _lib.BF16, None, None, None) == _lib.EINVAL_BLOCKSIZE
    # bad dtype
    assert f(p, p, p, p, p, 4, 8, 128, 16, 10, 1024, 1024, 7, None, None, None) == _lib.EINVAL_DTYPE
    # head_dim not divisible by the key pack x (paged_kv_cache.rs:268-272)
    assert f(p, p, p, p, p, 4, 8, 12, 16, 10, 96, 96, _lib.BF16, None, None, None) == _lib.EINVAL_SHAPE
    # token stride shorter than a token
    assert f(p, p, p, p, p, 4, 8, 128, 16, 10, 512, 1024, _lib.BF16, None, None, None) == _lib.EINVAL_SHAPE
    # unaligned pointer
    q = ctypes.c_void_p(18)
    assert f(q, p, p, p, p, 4, 8, 128, 16, 10, 1024, 1024, _lib.BF16, None, None, None) == _lib.EINVAL_ALIGN
    # zero tokens is a no-op
    assert f(p, p, p, p, p, 0, 8, 128, 16, 10, 1024, 1024, _lib.BF16, None, None, None) == _lib.OK


def test_decode_rejects_bad_arguments_and_sizes_workspace():
    lib = _lib.lib()
    ws = lib.vasr_pa_paged_attention_workspace_size
    assert ws(64, 16, 8, 128, 16, 2048, _lib.BF16) > 0
    assert ws(64, 16, 8, 128, 12, 2048, _lib.BF16) == 0          # bad block size
    assert ws(64, 16, 6, 128, 16, 2048, _lib.BF16) == 0          # Hq % Hkv != 0
    # the workspace grows with the upper bound, not with the true lengths
    assert ws(64, 16, 8, 128, 16, 4096, _lib.BF16) > ws(64, 16, 8, 128, 16, 2048, _lib.BF16)
    f = lib.vasr_pa_paged_attention
    p = ctypes.c_void_p(256)
    args = dict(B=4, Hq=16, Hkv=8, D=128, bs=16, nb=10, cols=4, mcl=64)

    def call(**kw):
        a = {**args, **kw}
        return f(p, p, p, p, p, p, a["B"], a["Hq"], a["Hkv"], a["D"], a["bs"], a["nb"], a["cols"],
                 a["mcl"], 0.088, a.get("softcap", 1.0), a["Hq"] * a["D"], a.get("dt", _lib.BF16),
                 None, 0, None)

    assert call(bs=64) == _lib.EINVAL_BLOCKSIZE
    assert call(Hkv=6) == _lib.EINVAL_SHAPE
    assert call(dt=9) == _lib.EINVAL_DTYPE
    assert call(softcap=0.0) == _lib.EINVAL_SHAPE
    assert call(B=0) == _lib.OK


def _prefill_args(**kw):
    a = dict(B=4, T=64, maxq=16, Hq=16, Hkv=8, D=128, bs=16, nb=40, cols=8, softcap=1.0,
             stride=16 * 128, dt=_lib.BF16)
    a.update(kw)
    return a


def test_prefill_rejects_bad_arguments_before_any_cuda_call():
    f = _lib.lib().vasr_pa_paged_attention_varlen_prefill
    p = ctypes.c_void_p(256)

    def call(**kw):
        a = _prefill_args(**kw)
        ptr = kw.get("ptr", p)
        return f(ptr, p, p, p, p, p, p, a["B"], a["T"], a["maxq"], a["Hq"], a["Hkv"], a["D"],
                 a["bs"], a["nb"], a["cols"], 0.088, a["softcap"], a["stride"], a["dt"], None)

    assert call(bs=12) == _lib.EINVAL_BLOCKSIZE
    assert call(dt=9) == _lib.EINVAL_DTYPE
    assert call(Hkv=6) == _lib.EINVAL_SHAPE            # Hq % Hkv != 0
    assert call(stride=100) == _lib.EINVAL_SHAPE       # token stride shorter than a token
    assert call(softcap=0.0) == _lib.EINVAL_SHAPE
    assert call(ptr=None) == _lib.EINVAL_POINTER
    assert call(ptr=ctypes.c_void_p(258)) == _lib.EINVAL_ALIGN
    assert call(B=0) == _lib.OK and call(T=0) == _lib.OK   # empty batches launch nothing


def test_fp8_prefill_sizes_its_scratch_and_rejects_bad_arguments():
    lib = _lib.lib()
    ws = lib.vasr_pa_paged_attention_varlen_prefill_fp8_workspace_size
    # 16-bit K and V copies of every (sequence, column) page plus the remapped table
    pages = 4 * 8 * 8 * 128 * 16 * 2
    assert ws(4, 8, 128, 16, 8) >= 2 * pages + 4 * 8 * 4
    assert ws(0, 8, 128, 16, 8) == 0 and ws(4, 8, 128, 16, 0) == 0
    f = lib.vasr_pa_paged_attention_varlen_prefill_fp8
    p = ctypes.c_void_p(256)
    need = ws(4, 8, 128, 16, 8)

    def call(scale_ptr=p, ws_ptr=p, ws_bytes=need, **kw):
        a = _prefill_args(**kw)
        return f(p, p, p, p, p, p, p, a["B"], a["T"], a["maxq"], a["Hq"], a["Hkv"], a["D"], a["bs"],
                 a["nb"], a["cols"], 0.088, a["softcap"], a["stride"], a["dt"], scale_ptr, p, ws_ptr,
                 ws_bytes, None)

    assert call(dt=_lib.FP8_E4M3) == _lib.EINVAL_DTYPE   # dtype names the query / output type
    assert call(dt=_lib.F32) == _lib.EINVAL_DTYPE
    assert call(scale_ptr=None) == _lib.EINVAL_POINTER   # fp8 pages need both scales
    assert call(ws_ptr=None) == _lib.EINVAL_WORKSPACE
    assert call(ws_bytes=need - 1) == _lib.EINVAL_WORKSPACE
    assert call(D=64, stride=16 * 64) == _lib.ENOT_SUPPORTED
    assert call(B=0) == _lib.OK


def test_block_ops_reject_bad_arguments():
    lib = _lib.lib()
    arr = (ctypes.c_void_p * 2)(16, 32)
    p = ctypes.c_void_p(64)
    assert lib.vasr_pa_copy_blocks(arr, arr, 0, p, 4, 10, 32768, None) == _lib.EINVAL_SHAPE
    assert lib.vasr_pa_copy_blocks(arr, arr, 2, p, 4, 10, 100, None) == _lib.EINVAL_ALIGN
    assert lib.vasr_pa_copy_blocks(arr, arr, 2, p, 0, 10, 32768, None) == _lib.OK
    assert lib.vasr_pa_swap_blocks(p, p, p, 4, 10, 10, 0, None) == _lib.EINVAL_SHAPE
    assert lib.vasr_pa_swap_blocks(None, p, p, 4, 10, 10, 32768, None) == _lib.EINVAL_POINTER


def test_product_path_has_no_oracle_dependency():
    """The package must not import, load or link the oracle."""
    pkg = Path(__file__).resolve().parent.parent / "qwen3asr.rs_b200"
    for f in list(pkg.rglob("*.py")) + list(pkg.rglob("*.cu")) + list(pkg.rglob("*.cpp")):
        text = f.read_text()
        assert "paged_ref" not in text and "liboracle" not in text, f


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_LIB", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "nope.so")
    with pytest.raises(_lib.VasrPaError):
        _lib.lib()
