"""B200 (sm_100a) implementation of the ``vasr-paged-attn`` hot path.

Python face of the crate ``vasr-paged-attn`` (re-exports at
vasr-paged-attn/src/lib.rs:12-27): the tensor entry points of
``mistralrs_paged_attn`` run the hand-written CUDA kernels of
``libvasr_pa.so`` through its C ABI; the cache/metadata/allocator types are
the C++ host mirror compiled as ``_vasr_host`` (see ``host``).
"""
from . import _lib, mistralrs_paged_attn
from ._lib import VasrPaError

PAD_SLOT_ID = -1

__all__ = ["PAD_SLOT_ID", "VasrPaError", "mistralrs_paged_attn", "_lib"]
