"""Batch decode engine over the paged cache — the caller of the hot path.

Mirrors, for the decode step only, what the reference does around
``vasr-paged-attn``:
  * the Qwen3 text-decoder layer of vasr-models/src/model/thinker_text.rs
    (:1026-1251, decode branch): q/k/v projections, per-head q/k RMSNorm,
    rotary embedding, ``reshape_and_cache`` then ``paged_attention`` per
    layer (:1101-1139), o_proj, SiLU-gated MLP, residuals;
  * the 28-layer loop of ThinkerTextModel::forward_with_paged_cache
    (:1702-1734) followed by the final norm, tied lm_head and greedy argmax
    (generation.rs:443, paged_batch_engine.rs:303);
  * DecodeCudaGraph (vasr-paged-attn/src/cuda_graph.rs:119-370): the whole
    step is captured once per (batch, block-table width) and replayed after
    copying the step's metadata into the captured buffers.
Weights are random (the benchmark configs use random init). The linear
layers, norms and RoPE are torch/cuBLAS calls — they are the reference's
Candle/cuBLAS calls, not part of the paged path; the paged-cache work goes
through the sm_100a kernels of ``mistralrs_paged_attn``.

For text and audio tokens the three mRoPE position streams are equal, so the
multimodal rotary embedding reduces to the 1-D rotary embedding used here.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn.functional as F

from . import fused as fused_ops
from . import mistralrs_paged_attn as pa


@dataclass(frozen=True)
class DecoderConfig:
    """Text-decoder shapes (vasr-models/src/config/text_config.rs:84-196)."""
    hidden_size: int = 1024
    num_layers: int = 28
    num_heads: int = 16
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 3072
    vocab_size: int = 151936
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    max_positions: int = 65536

    @staticmethod
    def qwen3_asr_0_6b() -> "DecoderConfig":
        return DecoderConfig()

    @staticmethod
    def qwen3_asr_1_7b() -> "DecoderConfig":
        return DecoderConfig(hidden_size=2048, intermediate_size=6144)

    def param_count(self) -> int:
        h, d = self.hidden_size, self.head_dim
        qkv = h * (self.num_heads + 2 * self.num_kv_heads) * d
        o = self.num_heads * d * h
        mlp = 3 * h * self.intermediate_size
        norms = 2 * h + 2 * d
        return self.num_layers * (qkv + o + mlp + norms) + self.vocab_size * h + h


class RandomQwen3Decoder:
    """Random-init weights of the architecture, bf16, laid out for fused GEMMs."""

    def __init__(self, cfg: DecoderConfig, device, dtype=torch.bfloat16, seed: int = 0):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        g = torch.Generator(device="cpu").manual_seed(seed)
        h, d = cfg.hidden_size, cfg.head_dim
        qkv_out = (cfg.num_heads + 2 * cfg.num_kv_heads) * d

        def w(*shape, std):
            return (torch.randn(*shape, generator=g) * std).to(dtype).to(self.device)

        self.embed = w(cfg.vocab_size, h, std=0.02)  # tied with lm_head
        self.layers = []
        for _ in range(cfg.num_layers):
            self.layers.append(dict(
                in_norm=torch.ones(h, dtype=dtype, device=self.device),
                w_qkv=w(qkv_out, h, std=1.0 / math.sqrt(h)),
                q_norm=torch.ones(d, dtype=dtype, device=self.device),
                k_norm=torch.ones(d, dtype=dtype, device=self.device),
                w_o=w(h, cfg.num_heads * d, std=1.0 / math.sqrt(cfg.num_heads * d)),
                post_norm=torch.ones(h, dtype=dtype, device=self.device),
                w_gate_up=w(2 * cfg.intermediate_size, h, std=1.0 / math.sqrt(h)),
                w_down=w(h, cfg.intermediate_size, std=1.0 / math.sqrt(cfg.intermediate_size)),
            ))
        self.final_norm = torch.ones(h, dtype=dtype, device=self.device)
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
        pos = torch.arange(cfg.max_positions, dtype=torch.float64)
        ang = torch.outer(pos, inv)
        self.rope_cos = torch.cos(ang).to(torch.float32).to(self.device)
        self.rope_sin = torch.sin(ang).to(torch.float32).to(self.device)

    def weight_bytes(self) -> int:
        n = self.embed.numel() + self.final_norm.numel()
        for l in self.layers:
            n += sum(t.numel() for t in l.values())
        return n * self.embed.element_size()

    def _rope(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        # rotate-half RoPE in f32; x [B, H, D]
        xf = x.float()
        half = xf.shape[-1] // 2
        x1, x2 = xf[..., :half], xf[..., half:]
        c, s = cos[:, None, :], sin[:, None, :]
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)

    def decode_step(self, input_ids: torch.Tensor, positions: torch.Tensor, kv_caches,
                    slot_mapping: torch.Tensor, block_tables: torch.Tensor,
                    context_lens: torch.Tensor, max_context_len: int,
                    next_ids_out: Optional[torch.Tensor] = None, fused: bool = True,
                    return_logits: bool = False) -> torch.Tensor:
        """One token per sequence through all layers; returns greedy next ids [B] (int64),
        or the logits [B, vocab] with ``return_logits`` (for the device-side argmax).

        ``fused`` runs q/k RMSNorm + RoPE + KV append as one kernel
        (vasr_pa_fused_qk_norm_rope_append); ``fused=False`` runs the same math
        as separate torch ops followed by reshape_and_cache.
        """
        cfg = self.cfg
        b = input_ids.shape[0]
        hq, hkv, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        x = F.embedding(input_ids, self.embed)
        if not fused:
            cos = self.rope_cos.index_select(0, positions)
            sin = self.rope_sin.index_select(0, positions)
        scale = d ** -0.5
        for l, (kc, vc) in zip(self.layers, kv_caches):
            h = F.rms_norm(x, (cfg.hidden_size,), l["in_norm"], cfg.rms_norm_eps)
            qkv = h @ l["w_qkv"].t()
            if fused:
                q = fused_ops.qk_norm_rope_append(qkv, l["q_norm"], l["k_norm"], cfg.rms_norm_eps,
                                                  self.rope_cos, self.rope_sin, positions, kc, vc,
                                                  slot_mapping, hq)
            else:
                q = qkv[:, : hq * d].view(b, hq, d)
                k = qkv[:, hq * d:(hq + hkv) * d].view(b, hkv, d)
                v = qkv[:, (hq + hkv) * d:].view(b, hkv, d)
                q = F.rms_norm(q, (d,), l["q_norm"], cfg.rms_norm_eps)
                k = F.rms_norm(k, (d,), l["k_norm"], cfg.rms_norm_eps)
                q = self._rope(q, cos, sin)
                k = self._rope(k, cos, sin)
                pa.reshape_and_cache(k, v, None, None, kc, vc, slot_mapping)
            # fused: the append kernel is the one just issued, so the decode
            # starts streaming older pages while it finishes
            attn = pa.paged_attention(q, None, None, kc, vc, block_tables, context_lens, None,
                                      max_context_len, scale, 1.0, None, after_append=fused)
            # residual adds folded into the GEMMs (beta = 1, accumulating into x)
            x.addmm_(attn.view(b, hq * d), l["w_o"].t())
            h = F.rms_norm(x, (cfg.hidden_size,), l["post_norm"], cfg.rms_norm_eps)
            gu = h @ l["w_gate_up"].t()
            gate, up = gu[:, : cfg.intermediate_size], gu[:, cfg.intermediate_size:]
            x.addmm_(F.silu(gate) * up, l["w_down"].t())
        x = F.rms_norm(x, (cfg.hidden_size,), self.final_norm, cfg.rms_norm_eps)
        logits = x @ self.embed.t()
        if return_logits:
            return logits
        nxt = torch.argmax(logits, dim=-1)
        if next_ids_out is not None:
            next_ids_out.copy_(nxt)
            return next_ids_out
        return nxt


def allocate_paged_cache(cfg: DecoderConfig, num_blocks: int, block_size: int, device,
                         dtype=torch.bfloat16, num_layers: Optional[int] = None):
    """Zeroed per-layer K/V pages in the reference layout (paged_kv_cache.rs:285-301)."""
    x = 16 // torch.empty((), dtype=dtype).element_size()
    layers = cfg.num_layers if num_layers is None else num_layers
    out = []
    for _ in range(layers):
        kc = torch.zeros((num_blocks, cfg.num_kv_heads, cfg.head_dim // x, block_size, x), dtype=dtype, device=device)
        vc = torch.zeros((num_blocks, cfg.num_kv_heads, cfg.head_dim, block_size), dtype=dtype, device=device)
        out.append((kc, vc))
    return out


class DecodeGraph:
    """One captured decode step for a fixed (batch, block-table width): cuda_graph.rs:119-370."""

    def __init__(self, model: RandomQwen3Decoder, kv_caches, batch: int, cols: int, block_size: int):
        self.model = model
        self.kv_caches = kv_caches
        dev = model.device
        self.batch, self.cols, self.block_size = batch, cols, block_size
        self.max_context_len = cols * block_size  # upper bound baked into the graph (cuda_graph.rs:141)
        self.input_ids = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.positions = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.slot_mapping = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.context_lens = torch.ones(batch, dtype=torch.int32, device=dev)
        self.block_tables = torch.zeros(batch, cols, dtype=torch.int32, device=dev)
        self.next_ids = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.stream = torch.cuda.Stream(device=dev)

    def _forward(self):
        self.model.decode_step(self.input_ids, self.positions, self.kv_caches, self.slot_mapping,
                               self.block_tables, self.context_lens, self.max_context_len,
                               next_ids_out=self.next_ids)

    def capture(self) -> None:
        cfg = self.model.cfg
        need = pa.paged_attention_workspace_bytes(self.batch, cfg.num_heads, cfg.num_kv_heads,
                                                  cfg.head_dim, self.block_size, self.max_context_len,
                                                  self.model.dtype)
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            pa.reserve_paged_attention_workspace(self.model.device, need, self.stream)
            self._forward()  # eager warm-up (cuda_graph.rs:204-211); writes only block 0 (dummy rows)
            self.stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream):
                self._forward()
        torch.cuda.current_stream().wait_stream(self.stream)
        self.graph = g

    def load(self, input_ids, positions, slot_mapping, context_lens, block_tables) -> None:
        """Copy one step's metadata into the captured buffers (replay_decode, cuda_graph.rs:342-369)."""
        self.input_ids.copy_(input_ids, non_blocking=True)
        self.positions.copy_(positions, non_blocking=True)
        self.slot_mapping.copy_(slot_mapping, non_blocking=True)
        self.context_lens.copy_(context_lens, non_blocking=True)
        self.block_tables.copy_(block_tables, non_blocking=True)

    def replay(self) -> torch.Tensor:
        assert self.graph is not None, "capture() first"
        self.graph.replay()
        return self.next_ids

    def release(self) -> None:
        self.graph = None


class DecodeLoopGraph:
    """A captured decode step whose inputs come from the previous step on the device.

    prepare (token feedback, EOS state, decode metadata) → 28 layers →
    greedy argmax, all in one CUDA graph over a ``DecodeLoopState``: replaying
    it K times decodes K tokens per sequence with no host round trip — the
    device-side version of paged_batch_decode_step's host loop
    (vasr-models/src/model/paged_batch_engine.rs:609-730) and of the per-step
    argmax sync it documents as the dominant decode cost.
    """

    def __init__(self, model: RandomQwen3Decoder, kv_caches, state, block_size: int):
        self.model, self.kv_caches, self.state = model, kv_caches, state
        self.block_size = block_size
        self.max_context_len = int(state.block_tables.shape[1]) * block_size
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.stream = torch.cuda.Stream(device=model.device)

    def _forward(self):
        st = self.state
        st.prepare()
        logits = self.model.decode_step(st.input_ids, st.positions, self.kv_caches, st.slot_mapping,
                                        st.block_tables, st.context_lens, self.max_context_len,
                                        return_logits=True)
        st.argmax(logits)

    def capture(self) -> None:
        cfg = self.model.cfg
        st = self.state
        need = pa.paged_attention_workspace_bytes(st.num_seqs, cfg.num_heads, cfg.num_kv_heads,
                                                  cfg.head_dim, self.block_size, self.max_context_len,
                                                  self.model.dtype)
        saved = {k: getattr(st, k).clone() for k in ("next_ids", "step", "finished", "generated", "history")}
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            pa.reserve_paged_attention_workspace(self.model.device, need, self.stream)
            self._forward()  # eager warm-up; its state changes are undone below
            self.stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream):
                self._forward()
            for k, v in saved.items():
                getattr(st, k).copy_(v)
            self.stream.synchronize()
        torch.cuda.current_stream().wait_stream(self.stream)
        self.graph = g

    def replay(self) -> None:
        assert self.graph is not None, "capture() first"
        self.graph.replay()

    def release(self) -> None:
        self.graph = None
