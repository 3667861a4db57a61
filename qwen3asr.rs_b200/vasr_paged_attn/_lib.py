"""ctypes binding of the C ABI in ``include/vasr_pa.h``.

This is the Python-side equivalent of the ``extern "C"`` block the Rust crate
declares. Loading fails loudly: there is no fallback implementation, so a
missing or unloadable ``libvasr_pa.so`` raises ``VasrPaError`` at first use.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PKG_ROOT = Path(__file__).resolve().parent.parent
LIB_PATH = Path(os.environ.get("VASR_PA_LIB", _PKG_ROOT / "lib" / "libvasr_pa.so"))

# vasr_pa_dtype
F32, BF16, F16, FP8_E4M3 = 0, 1, 2, 3
# vasr_pa_status
OK = 0
EINVAL_SHAPE = -1
EINVAL_DTYPE = -2
EINVAL_BLOCKSIZE = -3
EINVAL_ALIGN = -4
EINVAL_WORKSPACE = -5
ENOT_SUPPORTED = -6
ELAUNCH = -7
EDEVICE = -8
EINVAL_POINTER = -9
ESCRATCH_LIMIT = -10
# device error bits
DERR_SLOT_RANGE = 0x1
DERR_BLOCK_RANGE = 0x2
DERR_CTX_RANGE = 0x4
DERR_WAIT_TIMEOUT = 0x8
DERR_MAPPING_RANGE = 0x10
DERR_QLEN_RANGE = 0x20

_c_void_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_size = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/vasr_pa.h one to one.
SIGNATURES: dict[str, tuple] = {
    "vasr_pa_abi_version": (_i32, []),
    "vasr_pa_status_string": (ctypes.c_char_p, [_i32]),
    "vasr_pa_reshape_and_cache": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i32, _i32, _i32, _i64,
         _i64, _i64, _i32, _c_void_p, _c_void_p, _c_void_p],
    ),
    "vasr_pa_paged_attention_workspace_size": (_size, [_i32, _i32, _i32, _i32, _i32, _i32, _i32]),
    "vasr_pa_paged_attention": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32,
         _i32, _i32, _i64, _i32, _i32, _f32, _f32, _i64, _i32, _c_void_p, _size, _c_void_p],
    ),
    "vasr_pa_paged_attention_after_append": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32,
         _i32, _i32, _i64, _i32, _i32, _f32, _f32, _i64, _i32, _c_void_p, _size, _c_void_p],
    ),
    "vasr_pa_gather_kv_cache": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i64,
         _i32, _i32, _i32, _i64, _i32, _c_void_p],
    ),
    "vasr_pa_paged_attention_varlen_prefill": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i64,
         _i32, _i32, _i32, _i32, _i32, _i64, _i32, _f32, _f32, _i64, _i32, _c_void_p],
    ),
    "vasr_pa_paged_attention_varlen_prefill_fp8": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i64,
         _i32, _i32, _i32, _i32, _i32, _i64, _i32, _f32, _f32, _i64, _i32, _c_void_p, _c_void_p,
         _c_void_p, _size, _c_void_p],
    ),
    "vasr_pa_paged_attention_varlen_prefill_fp8_workspace_size": (_size, [_i32, _i32, _i32, _i32, _i32]),
    "vasr_pa_copy_blocks": (
        _i32,
        [ctypes.POINTER(_c_void_p), ctypes.POINTER(_c_void_p), _i32, _c_void_p, _i64, _i64, _i64,
         _c_void_p],
    ),
    "vasr_pa_swap_blocks": (
        _i32, [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _c_void_p]
    ),
    "vasr_pa_get_device_error": (_i32, [ctypes.POINTER(_i32), _i32, _c_void_p]),
    "vasr_pa_paged_attention_noalloc": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32,
         _i32, _i32, _i64, _i32, _i32, _f32, _f32, _i64, _i32, _c_void_p],
    ),
    "vasr_pa_noalloc_scratch_bytes": (_size, []),
    "vasr_pa_fused_qk_norm_rope_append": (
        _i32,
        [_c_void_p, _c_void_p, _i64, _c_void_p, _c_void_p, _f32, _c_void_p, _c_void_p, _i64,
         _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i32, _i32, _i32, _i32, _i64, _i32,
         _c_void_p],
    ),
    "vasr_pa_reshape_and_cache_fp8": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i32, _i32, _i32, _i64,
         _i64, _i64, _i32, _c_void_p, _c_void_p, _c_void_p],
    ),
    "vasr_pa_gather_kv_cache_fp8": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i64, _i32,
         _i32, _i32, _i64, _i32, _c_void_p, _c_void_p, _c_void_p],
    ),
    "vasr_pa_paged_attention_fp8": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _i32,
         _i32, _i64, _i32, _i32, _f32, _f32, _i64, _i32, _c_void_p, _c_void_p, _c_void_p, _size,
         _c_void_p],
    ),
    "vasr_pa_decode_step_prepare": (
        _i32,
        [_c_void_p, _c_void_p, _i32, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i64,
         _i32, _c_void_p, _c_void_p, _c_void_p, _i32, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
         _c_void_p],
    ),
    "vasr_pa_greedy_argmax_workspace_size": (_size, [_i32, _i64]),
    "vasr_pa_greedy_argmax": (
        _i32,
        [_c_void_p, _c_void_p, _i32, _i64, _i64, _i32, _c_void_p, _c_void_p, _c_void_p, _size,
         _c_void_p],
    ),
}


class VasrPaError(RuntimeError):
    """A C-ABI call returned a negative vasr_pa_status, or the library is missing."""

    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} (status {status})")


_LIB: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Load ``libvasr_pa.so`` once; raise if it is absent (no CPU fallback exists)."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise VasrPaError(
                EDEVICE,
                f"libvasr_pa.so not found at {LIB_PATH}; run `python build.py` in the package dir",
            )
        dll = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(dll, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = dll
    return _LIB


def status_string(status: int) -> str:
    if _LIB is None and not LIB_PATH.exists():
        return "library not loaded"
    return lib().vasr_pa_status_string(status).decode()


def check(status: int, what: str) -> None:
    if status != OK:
        raise VasrPaError(status, what)
