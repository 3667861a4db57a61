"""Device-side decode loop: token feedback, EOS state, decode metadata and greedy argmax.

The reference does this on the host every decode step — the token/EOS loop of
``paged_batch_decode_step`` (vasr-models/src/model/paged_batch_engine.rs:634-712),
``decode_metadata_for_batch_step`` (vasr-paged-attn/src/paged_kv_cache.rs:924-1059)
and ``argmax_token_ids_from_logits`` with its device-to-host copy
(vasr-models/src/model/generation.rs:443-460) — which is the dominant decode
cost it documents. ``DecodeLoopState`` keeps all of it in HBM so a captured
decode step (prepare → forward → argmax) replays step after step; the host
only reads the finished flags and tokens back when it wants to.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

from . import _lib
from .mistralrs_paged_attn import _require_cuda, _stream, dtype_code

_U32 = torch.int32  # u32 buffers are held as int32 tensors of the same bits


def greedy_argmax_workspace_bytes(num_seqs: int, vocab: int) -> int:
    return int(_lib.lib().vasr_pa_greedy_argmax_workspace_size(num_seqs, vocab))


def greedy_argmax(logits: torch.Tensor, out: Optional[torch.Tensor] = None,
                  finished: Optional[torch.Tensor] = None, step: Optional[torch.Tensor] = None,
                  workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """next ids (int32 [B]) = row-wise argmax of logits [B, vocab] (lowest index on ties)."""
    dev = _require_cuda(logits)
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "logits must be [B, vocab] with unit column stride")
    b, vocab = int(logits.shape[0]), int(logits.shape[1])
    if out is None:
        out = torch.empty(b, dtype=_U32, device=dev)
    need = greedy_argmax_workspace_bytes(b, vocab)
    if workspace is None:
        workspace = torch.zeros(need, dtype=torch.uint8, device=dev)
    if workspace.numel() < need:
        raise _lib.VasrPaError(_lib.EINVAL_WORKSPACE, "greedy_argmax workspace too small")
    st = _lib.lib().vasr_pa_greedy_argmax(
        out.data_ptr(), logits.data_ptr(), b, vocab, logits.stride(0), dtype_code(logits.dtype),
        finished.data_ptr() if finished is not None else None,
        step.data_ptr() if step is not None else None, workspace.data_ptr(), workspace.numel(),
        _stream(dev))
    _lib.check(st, "greedy_argmax")
    return out


class DecodeLoopState:
    """HBM-resident state of a batch decode (one row per sequence, fixed batch size).

    ``prepare()`` turns last step's tokens into this step's inputs and metadata
    (``input_ids``, ``positions``, ``slot_mapping``, ``context_lens``);
    ``argmax(logits)`` writes the next tokens and advances the step counter.
    Both are capture-safe, so ``prepare → forward → argmax`` can sit in one
    CUDA graph. The host must have allocated, in ``block_tables`` /
    ``block_table_lens``, the blocks for every position the replayed steps reach.
    """

    def __init__(self, prompt_lens: Sequence[int], first_tokens: Sequence[int], eos_ids: Sequence[int],
                 block_tables: torch.Tensor, block_table_lens: Optional[Sequence[int]], block_size: int,
                 num_blocks: int, vocab: int, history_cols: int = 0, device=None):
        dev = torch.device(device) if device is not None else block_tables.device
        b = len(prompt_lens)
        if len(first_tokens) != b or block_tables.dim() != 2 or block_tables.shape[0] != b:
            raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "decode loop batch mismatch")
        if not eos_ids:
            raise _lib.VasrPaError(_lib.EINVAL_SHAPE, "eos_token_ids is empty")
        i32 = lambda xs: torch.tensor(list(xs), dtype=_U32, device=dev)  # noqa: E731
        self.device = dev
        self.num_seqs = b
        self.block_size = int(block_size)
        self.num_blocks = int(num_blocks)
        self.prompt_lens = i32(prompt_lens)
        self.next_ids = i32(first_tokens)
        self.eos_ids = i32(eos_ids)
        self.block_tables = block_tables.to(device=dev, dtype=_U32).contiguous()
        self.block_table_lens = i32(block_table_lens) if block_table_lens is not None else None
        self.step = torch.zeros(1, dtype=_U32, device=dev)
        self.finished = torch.zeros(b, dtype=torch.uint8, device=dev)
        self.generated = torch.zeros(b, dtype=_U32, device=dev)
        self.history_cols = int(history_cols)
        self.history = torch.zeros((b, max(1, self.history_cols)), dtype=_U32, device=dev)
        self.input_ids = torch.zeros(b, dtype=torch.int64, device=dev)
        self.positions = torch.zeros(b, dtype=torch.int64, device=dev)
        self.slot_mapping = torch.zeros(b, dtype=torch.int64, device=dev)
        self.context_lens = torch.ones(b, dtype=_U32, device=dev)
        self.workspace = torch.zeros(greedy_argmax_workspace_bytes(b, vocab), dtype=torch.uint8,
                                     device=dev)

    def prepare(self) -> None:
        h = self.history_cols > 0
        st = _lib.lib().vasr_pa_decode_step_prepare(
            self.next_ids.data_ptr(), self.eos_ids.data_ptr(), int(self.eos_ids.numel()),
            self.prompt_lens.data_ptr(), self.step.data_ptr(), self.block_tables.data_ptr(),
            self.block_table_lens.data_ptr() if self.block_table_lens is not None else None,
            int(self.block_tables.shape[1]), self.block_size, self.num_blocks, self.num_seqs,
            self.finished.data_ptr(), self.generated.data_ptr(),
            self.history.data_ptr() if h else None, self.history_cols if h else 0,
            self.input_ids.data_ptr(), self.positions.data_ptr(), self.slot_mapping.data_ptr(),
            self.context_lens.data_ptr(), _stream(self.device))
        _lib.check(st, "decode_step_prepare")

    def argmax(self, logits: torch.Tensor) -> torch.Tensor:
        return greedy_argmax(logits, out=self.next_ids, finished=self.finished, step=self.step,
                             workspace=self.workspace)

    def read_back(self):
        """(finished bool [B], generated counts [B], history [B, cols]) on the host (synchronises)."""
        return (self.finished.cpu().bool(), self.generated.cpu().long(),
                self.history[:, : self.history_cols].cpu().long())
