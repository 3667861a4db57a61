#!/usr/bin/env python
"""Benchmark of the paged KV-cache decode path on B200 (BASELINE.json config 5 by default).

One *step* = one full 28-layer decode step of a random-init bf16 Qwen3-ASR
text decoder: per layer one fused q/k RMSNorm + RoPE + KV append and one
``paged_attention`` through the sm_100a kernels, the rest (GEMMs, norms,
lm_head, argmax) through torch; the step is a captured CUDA graph replayed
per token, as in the reference (vasr-paged-attn/src/cuda_graph.rs).

Default workload = config 5: the 1.7B-shaped decoder (hidden 2048, MLP 6144)
and 512 sequences with contexts ~log-U[64, 4096], split over the ranks by
expected KV bytes (strong scaling: the 512 sequences are the whole job at
every N, one process per GPU, no collective on the hot path).

  value      tokens/s over all ranks, metadata already resident in HBM
             (per step: device-side copy of that step's metadata into the
             graph buffers + replay); device time, max over ranks.
  e2e        tokens/s through the engine's host-facing call: per step the
             host builds the step metadata, copies it from pinned memory,
             replays, and reads the next token ids back (synchronising);
             the host builds step s + 1's metadata (double-buffered pinned
             memory) while the GPU runs step s.
  roofline   the paged decode kernel alone at the workload's shapes (rank 0):
             algorithmic KV bytes per launch / CUDA-event launch time vs the
             measured HBM copy bandwidth.
  ranks      per rank: sequences, context tokens, decode-kernel us and GB/s
             per launch, step ms and the share of the step outside the paged
             decode kernel (the per-replica fixed cost: weights and glue).
  device_loop  tokens/s of the device-side decode loop: step prepare (token
             feedback, EOS state, metadata) + the 28 layers + greedy argmax
             captured as one graph and replayed back to back.
  config2    the same step for config 2 (0.6B decoder, 64 sequences per GPU,
             weak scaling) with its decode-kernel roofline.
  prefill / append / decode_fp8 (config 2) / decode_fp8_config5 / copy_blocks /
  swap_blocks / gather_kv_cache
             (one GPU only) each kernel on its BASELINE config, timed with
             CUDA events over a captured graph of launches whose inputs
             together exceed L2: us, achieved, peak, frac.

``--config 2`` makes config 2 the headline workload instead.
``--kernel NAME`` prints only that kernel microbenchmark.
``--impl reference`` times the reference's CPU attention path (the C
restatement in oracle/, all host threads) on the same contexts.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "qwen3asr.rs_b200"))

METRIC = "decode tok/s & paged-attn KV-read GB/s (% of 8 TB/s) at 1/2/4/8 B200"
BATCH = 64
CTX_LO, CTX_HI = 200, 1500
BLOCK_SIZE = 16
KERNELS = ["decode", "decode5", "decode_fp8", "decode5_fp8", "append", "gather", "prefill", "prefill_fp8",
           "copy", "swap", "config1"]


def parse_args(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None,
                   help="timed steps (default 64 for config 5, 100 for config 2)")
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--cpu-seconds", type=float, default=10.0,
                   help="target CPU time of the bounded cpu_baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extras", action="store_true",
                   help="skip the config-2 step and the per-kernel microbenchmarks of the JSON line")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--config", type=int, choices=[2, 5], default=5,
                   help="decode-step workload: 5 = 1.7B decoder, 512 sequences sharded over the GPUs "
                        "(strong scaling); 2 = 0.6B decoder, 64 sequences per GPU (weak scaling)")
    p.add_argument("--kernel", default=None, choices=KERNELS,
                   help="microbenchmark one kernel on its BASELINE config instead of the decode step")
    p.add_argument("--iters", type=int, default=20, help="timed launches per kernel microbenchmark")
    p.add_argument("--layers", type=int, default=28,
                   help="distinct per-layer caches cycled through by --kernel decode/copy")
    p.add_argument("--pool-blocks", type=int, default=200_000,
                   help="blocks per layer pool of --kernel copy (config 4: 200k; smaller for profiling)")
    args = p.parse_args(argv)
    if args.steps is None:
        args.steps = 64 if args.config == 5 else 100
    return args


# ------------------------------------------------------------------ helpers
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def context_lens(seed: int, rank: int):
    """Config 2: 64 contexts ~U[200, 1500] per rank."""
    import numpy as np

    rng = np.random.default_rng(seed + 1000 * rank)
    return rng.integers(CTX_LO, CTX_HI + 1, size=BATCH).astype(np.int64)


def _peaks_file():
    f = REPO / "MEASURED_PEAKS.json"
    return json.loads(f.read_text()) if f.exists() else None


def load_peaks():
    d = _peaks_file()
    if d:
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_tensor_peak():
    d = _peaks_file()
    if d:
        return float(d["bf16_tflops"]), "measured (burst)"
    return 1590.0, "fallback (burst)"


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples (every 100 ms) kept for the
    timed regions: each sample carries nvidia-smi's timestamp and only those
    inside a region passed to stop() count (all samples if none falls inside)."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def wait_first(self, timeout: float = 5.0):
        """Block until the sampler delivered its first sample (it starts slowly)."""
        t0 = time.time()
        while self.proc is not None and not self.lines and time.time() - t0 < timeout:
            time.sleep(0.02)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu_index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self, windows=()):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        rows = []
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(parts[2]), float(parts[3]),
                             {n for n, v in zip(names, parts[6:10]) if v.lower().startswith("active")}))
            except ValueError:
                continue
        inside = [r for r in rows if any(a - 0.05 <= r[0] <= b + 0.05 for a, b in windows)]
        use = inside or rows
        sm = [r[1] for r in use]
        reasons = set().union(*[r[3] for r in use]) if use else set()
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(r[2] for r in use) if use else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "samples_in_timed_regions": len(inside)}


# ------------------------------------------------------------ CPU baseline
def cpu_attention_sample(seed: int, target_seconds: float, steps: int | None = None, lens=None):
    """Time the oracle's f32 decode attention (reference CPU path restated in C, all threads).

    A step is 28 layers of decode attention over ``lens`` (default: the
    config-2 context set); one layer's cache is generated and attended 28
    times per step (the cost per layer is identical). GEMMs are excluded, so
    this is an upper bound on the CPU's decode tok/s.
    """
    import numpy as np

    sys.path.insert(0, str(REPO / "oracle"))
    import paged_ref as ref

    lens = context_lens(seed, 0) if lens is None else np.asarray(lens, dtype=np.int64)
    batch = len(lens)
    hq, hkv, d, bs = 16, 8, 128, BLOCK_SIZE
    blocks = [-(-int(n) // bs) for n in lens]
    nb = sum(blocks) + 1
    rng = np.random.default_rng(seed)
    kc = rng.standard_normal((nb, hkv, d // 4, bs, 4), dtype=np.float32)
    vc = rng.standard_normal((nb, hkv, d, bs), dtype=np.float32)
    perm = rng.permutation(np.arange(1, nb))
    tables = np.zeros((batch, max(blocks)), np.uint32)
    off = 0
    for i, n in enumerate(blocks):
        tables[i, :n] = perm[off:off + n]
        off += n
    q = rng.standard_normal((batch, hq, d), dtype=np.float32)
    ctx = lens.astype(np.uint32)
    # all host cores this process may run on (torchrun sets OMP_NUM_THREADS=1 per worker,
    # so the OpenMP default would under-report the CPU path)
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    ref.paged_attention(q, kc, vc, tables, ctx, d ** -0.5, use_double=False, threads=threads)
    t0 = time.perf_counter()
    ref.paged_attention(q, kc, vc, tables, ctx, d ** -0.5, use_double=False, threads=threads)
    t_layer = time.perf_counter() - t0
    n_layers = 28
    if steps is None:
        reps = max(1, int(target_seconds / max(t_layer, 1e-6)))
        t0 = time.perf_counter()
        for _ in range(reps):
            ref.paged_attention(q, kc, vc, tables, ctx, d ** -0.5, use_double=False, threads=threads)
        t_layer = (time.perf_counter() - t0) / reps
        return dict(tok_s=batch / (n_layers * t_layer), t_layer=t_layer, reps=reps, threads=threads)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        for _ in range(n_layers):
            ref.paged_attention(q, kc, vc, tables, ctx, d ** -0.5, use_double=False, threads=threads)
        times.append(time.perf_counter() - t0)
    return dict(step_times=times, threads=threads)


def cpu_info() -> str:
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return  # other ranks exit without work
    k, w = args.steps, args.warmup
    # bounded: the reference arm runs min(steps, 3) timed steps of 28 CPU layers
    ks = max(1, min(k, 3))
    if args.config == 5:
        # 64 of the 512 sequences per step, the step time scaled by the context sum
        from vasr_paged_attn.workloads import config5_context_lens
        lens_all = config5_context_lens(args.seed)
        sub = lens_all[:BATCH]
        r = cpu_attention_sample(args.seed, args.cpu_seconds, steps=ks + min(w, 1), lens=sub)
        factor = float(lens_all.sum()) / float(sub.sum())
        batch = len(lens_all)
        sample = (f"{ks} timed steps x 28 layers of decode attention over {len(sub)} of the {batch} "
                  f"config-5 sequences (ctx log-U[64,4096]), step time scaled by the context sum to all "
                  f"{batch}; f32 C/OpenMP restatement of attention.rs, GEMMs excluded; {cpu_info()}")
        workload = "config5: qwen3-asr-1.7B decode step attention, 512 sequences, ctx log-U[64,4096]"
        scaling = "strong"
    else:
        r = cpu_attention_sample(args.seed, args.cpu_seconds, steps=ks + min(w, 1))
        factor, batch = 1.0, BATCH
        sample = (f"{ks} timed steps x 28 layers of decode attention, {BATCH} seqs, ctx U[{CTX_LO},{CTX_HI}], "
                  f"f32 C/OpenMP restatement of attention.rs, GEMMs excluded; {cpu_info()}")
        workload = "config2: qwen3-asr-0.6B decode step attention, B=64, ctx U[200,1500]"
        scaling = "weak"
    times = r["step_times"][min(w, 1):]
    step_s = statistics.mean(times) * factor
    value = batch / step_s
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": ks, "warmup": min(w, 1), "ms_per_step": step_s * 1e3, "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1))",
        "config": {"workload": workload, "global_batch": batch, "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": r["threads"], "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------- decode-step bench
class Ranks:
    """Barrier and max-over-ranks of the one-process-per-GPU job (identity at N = 1)."""

    def __init__(self, world, dev):
        self.world, self.dev = world, dev

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max(self, x: float) -> float:
        if self.world == 1:
            return x
        import torch
        import torch.distributed as dist
        t = torch.tensor([x], dtype=torch.float64, device=self.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def gather(self, row):
        """Every rank's row of floats (all ranks call this at the same point)."""
        if self.world == 1:
            return [list(row)]
        import torch
        import torch.distributed as dist
        t = torch.tensor(row, dtype=torch.float64, device=self.dev)
        out = [torch.zeros_like(t) for _ in range(self.world)]
        dist.all_gather(out, t)
        return [o.cpu().tolist() for o in out]


def decode_step_bench(which: int, args, dev, rank: int, world: int, ranks: Ranks, windows: list,
                      steps: int, full: bool = True):
    """Time the captured 28-layer decode step of config ``which`` (2 or 5) on this rank's
    sequences. Every rank runs the same collective calls in the same order.

    Returns a dict of whole-job rates (device-resident ``value``; with ``full``
    also ``e2e`` and ``device_loop``), the decode kernel's launch time at this
    rank's shapes and every rank's row of per-rank figures."""
    import numpy as np
    import torch

    from vasr_paged_attn import engine as eng
    from vasr_paged_attn import host
    from vasr_paged_attn import mistralrs_paged_attn as pa

    if which == 5:
        from vasr_paged_attn.sharding import lpt_shard
        from vasr_paged_attn.workloads import config5_context_lens
        cfg = eng.DecoderConfig.qwen3_asr_1_7b()
        all_lens = config5_context_lens(args.seed)
        lens0 = np.asarray(all_lens[sorted(lpt_shard(all_lens.tolist(), world)[rank])], dtype=np.int64)
        global_batch = len(all_lens)
    else:
        cfg = eng.DecoderConfig.qwen3_asr_0_6b()
        lens0 = context_lens(args.seed, rank)
        global_batch = BATCH * world
    batch = len(lens0)
    model = eng.RandomQwen3Decoder(cfg, dev, torch.bfloat16, seed=args.seed)
    k_steps, w_steps = steps, max(3, args.warmup)
    # the device-resident, e2e and device-loop runs each replay steps 0 .. W + K - 1
    # (same positions, same contexts), so their rates compare like for like
    total_steps = w_steps + k_steps + 2
    need_tok = lens0 + total_steps
    blocks = np.array([-(-int(n) // BLOCK_SIZE) for n in need_tok])
    nb = int(blocks.sum()) + 1
    rng = np.random.default_rng(args.seed + 7 + rank)
    perm = rng.permutation(np.arange(1, nb))
    raw_cols = int(blocks.max())
    cols = host.bucket_block_table_cols(raw_cols, BLOCK_SIZE)
    tables = np.zeros((batch, cols), np.int32)
    off = 0
    for i, n in enumerate(blocks):
        tables[i, :n] = perm[off:off + n]
        off += n
    caches = eng.allocate_paged_cache(cfg, nb, BLOCK_SIZE, dev)
    gen = torch.Generator(device=dev).manual_seed(args.seed + rank)
    for kc, vc in caches:  # prefilled synthetic cache contents
        kc.normal_(generator=gen)
        vc.normal_(generator=gen)

    graph = eng.DecodeGraph(model, caches, batch, cols, BLOCK_SIZE)
    graph.capture()

    # per-step metadata, device resident: positions advance by one per step
    steps_all = np.arange(total_steps)[:, None]
    pos = lens0[None, :] + steps_all                                    # [S, B]
    slots = tables[np.arange(batch)[None, :], pos // BLOCK_SIZE].astype(np.int64) * BLOCK_SIZE + pos % BLOCK_SIZE
    ctx = (pos + 1).astype(np.int32)
    d_pos = torch.from_numpy(pos.astype(np.int64)).to(dev)
    d_slots = torch.from_numpy(slots).to(dev)
    d_ctx = torch.from_numpy(ctx).to(dev)
    d_tables = torch.from_numpy(tables).to(dev)
    d_ids = torch.zeros(batch, dtype=torch.int64, device=dev)

    def device_step(s):
        graph.input_ids.copy_(graph.next_ids if s > 0 else d_ids)
        graph.positions.copy_(d_pos[s])
        graph.slot_mapping.copy_(d_slots[s])
        graph.context_lens.copy_(d_ctx[s])
        if s == 0:
            graph.block_tables.copy_(d_tables)
        graph.replay()

    s_idx = 0
    for _ in range(w_steps):
        device_step(s_idx)
        s_idx += 1
    torch.cuda.synchronize()
    ranks.barrier()
    torch.cuda.synchronize()
    ranks.barrier()
    w0 = time.time()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed_steps")  # lets ncu --nvtx-include select the timed launches
    e0.record()
    for _ in range(k_steps):
        device_step(s_idx)
        s_idx += 1
    e1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ranks.barrier()
    local_ms = e0.elapsed_time(e1)
    dev_ms = ranks.max(local_ms)
    windows.append((w0, time.time()))
    res = {"cfg": cfg, "model": model, "lens": lens0, "cols": cols, "global_batch": global_batch,
           "batch": batch, "k_steps": k_steps, "w_steps": w_steps, "dev_ms": dev_ms,
           "value": global_batch * k_steps / (dev_ms / 1e3)}

    if full:
        # ---- e2e: host-built metadata, pinned H2D, replay, D2H of next ids. The
        # pinned metadata is double-buffered so that the host builds step s + 1
        # while the GPU runs step s; every step still copies its inputs H2D, reads
        # its next ids D2H and synchronises before the next step starts.
        meta_cache = host.metadata_cache(nb, cfg.num_kv_heads, cfg.head_dim, BLOCK_SIZE, "bf16")

        def pinned_set():
            return {"ids": torch.zeros(batch, dtype=torch.int64).pin_memory(),
                    "pos": torch.zeros(batch, dtype=torch.int64).pin_memory(),
                    "slots": torch.zeros(batch, dtype=torch.int64).pin_memory(),
                    "ctx": torch.zeros(batch, dtype=torch.int32).pin_memory(),
                    "tables": torch.zeros(batch, cols, dtype=torch.int32).pin_memory()}

        sets = [pinned_set(), pinned_set()]
        h_next = torch.zeros(batch, dtype=torch.int64).pin_memory()
        prompt_lens = [int(x) for x in lens0]
        table_rows = [list(map(int, r[:n])) for r, n in zip(tables, blocks)]
        stream = torch.cuda.current_stream()

        def build(s, st):
            # host metadata through the C++ mirror of decode_metadata_for_batch_step
            meta = meta_cache.decode_metadata_for_batch_step(table_rows, prompt_lens, s, True)
            st["slots"].numpy()[:] = meta.slot_mapping
            st["ctx"].numpy()[:] = meta.context_lens
            st["pos"].numpy()[:] = np.asarray(meta.context_lens, dtype=np.int64) - 1
            st["tables"].numpy().reshape(-1)[:] = meta.block_tables_flat

        def e2e_step(s):
            st = sets[s % 2]
            st["ids"].copy_(h_next)  # the previous step's tokens, read back by the host
            graph.input_ids.copy_(st["ids"], non_blocking=True)
            graph.positions.copy_(st["pos"], non_blocking=True)
            graph.slot_mapping.copy_(st["slots"], non_blocking=True)
            graph.context_lens.copy_(st["ctx"], non_blocking=True)
            graph.block_tables.copy_(st["tables"], non_blocking=True)
            graph.replay()
            h_next.copy_(graph.next_ids, non_blocking=True)
            build(s + 1, sets[(s + 1) % 2])  # overlaps the GPU step
            stream.synchronize()

        s_idx = 0
        build(s_idx, sets[s_idx % 2])
        for _ in range(w_steps):
            e2e_step(s_idx)
            s_idx += 1
        torch.cuda.synchronize()
        ranks.barrier()
        t0 = time.perf_counter()
        w0 = time.time()
        for _ in range(k_steps):
            e2e_step(s_idx)
            s_idx += 1
        torch.cuda.synchronize()
        windows.append((w0, time.time()))
        e2e_s = ranks.max(time.perf_counter() - t0)
        ranks.barrier()
        res["e2e"] = {"value": global_batch * k_steps / e2e_s, "unit": "tok/s",
                      "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in sets[0].values()),
                      "d2h_bytes_per_step": h_next.numel() * 8}

        # ---- device decode loop: prepare -> forward -> argmax replayed with no host round trip
        from vasr_paged_attn import decode_loop as dloop
        loop_state = dloop.DecodeLoopState(
            [int(x) for x in lens0], [0] * batch, [cfg.vocab_size],  # EOS id outside the vocab:
            torch.from_numpy(tables).to(dev), blocks.tolist(), BLOCK_SIZE, nb,  # every row stays active
            cfg.vocab_size, device=dev)
        loop = eng.DecodeLoopGraph(model, caches, loop_state, BLOCK_SIZE)
        loop.capture()
        for _ in range(w_steps):
            loop.replay()
        torch.cuda.synchronize()
        ranks.barrier()
        l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0 = time.time()
        l0.record()
        for _ in range(k_steps):
            loop.replay()
        l1.record()
        torch.cuda.synchronize()
        windows.append((w0, time.time()))
        loop_ms = ranks.max(l0.elapsed_time(l1))
        ranks.barrier()
        fin, gen_counts, _ = loop_state.read_back()
        loop.release()
        res["device_loop"] = {
            "value": global_batch * k_steps / (loop_ms / 1e3), "unit": "tok/s", "ms_per_step": loop_ms / k_steps,
            "note": "decode_step_prepare + 28 layers + greedy_argmax captured as one graph and replayed "
                    "back to back: next ids, EOS state and metadata stay on the device (no per-step host "
                    "round trip)",
            "rows_active_at_end": int((~fin).sum()), "tokens_generated": int(gen_counts.sum())}

    # ---- the paged decode kernel alone: one launch per layer, events on its stream
    last = min(w_steps + k_steps - 1, total_steps - 1)  # contexts of the last timed step
    ctx_last = torch.from_numpy(ctx[last]).to(dev)
    q = torch.randn(batch, cfg.num_heads, cfg.head_dim, device=dev, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    mcl = cols * BLOCK_SIZE

    def decode_layer(i):
        kc, vc = caches[i % len(caches)]
        pa.paged_attention(q, None, None, kc, vc, d_tables, ctx_last, None, mcl, cfg.head_dim ** -0.5,
                           1.0, None, out=out)

    # back-to-back launches over the 28 layer caches (as inside the step), one graph replay
    launch_ms = _events_time(decode_layer, 3 * len(caches))
    ctx_sum = int(ctx[last].astype(np.int64).sum())
    kv_bytes = ctx_sum * cfg.num_kv_heads * cfg.head_dim * 2 * 2
    qo_bytes = batch * cfg.num_heads * cfg.head_dim * 2 * 2
    alg_bytes = kv_bytes + qo_bytes
    step_us = local_ms / k_steps * 1e3
    res.update(launch_ms=launch_ms, alg_bytes=alg_bytes)
    rows = ranks.gather([rank, batch, ctx_sum, launch_ms * 1e3, alg_bytes / (launch_ms / 1e3) / 1e9,
                         step_us / 1e3, 1.0 - cfg.num_layers * launch_ms * 1e3 / step_us])
    res["ranks"] = [{"rank": int(r[0]), "seqs": int(r[1]), "ctx_tokens": int(r[2]),
                     "decode_us_per_launch": round(r[3], 2), "decode_GBps": round(r[4], 1),
                     "step_ms": round(r[5], 4), "non_paged_share_of_step": round(r[6], 4)} for r in rows]
    res["kv_step_gb"] = float(lens0.sum()) * cfg.num_kv_heads * cfg.head_dim * 2 * 2 * cfg.num_layers / 1e9
    graph.release()
    del graph, caches
    return res


def _roofline(res, peak, peak_kind):
    achieved = res["alg_bytes"] / (res["launch_ms"] / 1e3) / 1e9
    traffic = None
    tf = REPO / "profiles" / "paged_decode_traffic.json"
    if tf.exists():
        ratio = json.loads(tf.read_text()).get("dram_bytes_per_algorithmic_byte")
        if ratio:
            traffic = ratio * res["alg_bytes"]
    return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "traffic": traffic, "kernel": "paged_decode_mma_kernel", "peak_source": peak_kind,
            "launch_us": res["launch_ms"] * 1e3, "algorithmic_bytes_per_launch": res["alg_bytes"]}


def run_ours(args):
    import numpy as np  # noqa: F401
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device for --impl ours")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        # NCCL's own init lines stay in the log; rank 0 adds a one-line summary
        # of the communicator (the only NCCL traffic: barriers and the
        # max-over-ranks reductions of the timings, outside the timed regions)
        os.environ.setdefault("NCCL_DEBUG", "INFO")
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
        dist.barrier()
        if rank == 0:
            ver = torch.cuda.nccl.version()
            print(json.dumps({"nccl": {"version": ".".join(map(str, ver)) if isinstance(ver, tuple) else ver,
                                       "backend": dist.get_backend(), "world_size": world,
                                       "collectives": "barrier + all-reduce(max) of timings, outside timed regions"}}),
                  file=sys.stderr, flush=True)
    ranks = Ranks(world, dev)
    peak, peak_kind = load_peaks()

    clocks = ClockSampler(local)
    clocks.start()
    clocks.wait_first()
    windows = []  # host wall-clock spans of the timed regions, for the clock samples
    main = decode_step_bench(args.config, args, dev, rank, world, ranks, windows, args.steps, full=True)
    cfg, lens0 = main["cfg"], main["lens"]
    weight_gb = main.pop("model").weight_bytes() / 1e9
    torch.cuda.empty_cache()

    extras = {}
    if args.config == 5 and not args.no_extras:
        c2 = decode_step_bench(2, args, dev, rank, world, ranks, windows, 100, full=False)
        extras["config2"] = {
            "value": c2["value"], "unit": "tok/s", "ms_per_step": c2["dev_ms"] / c2["k_steps"],
            "scaling": "weak", "global_batch": c2["global_batch"],
            "workload": "config2: qwen3-asr-0.6B decode step, 28 layers, B=64 per GPU, ctx U[200,1500]",
            "roofline": _roofline(c2, peak, peak_kind), "ranks": c2["ranks"]}
        del c2
        torch.cuda.empty_cache()
    clk = clocks.stop(windows)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        if args.config == 5:
            # bounded: 64 of the 512 sequences, their layer time scaled by the context sum
            sub = lens0[:BATCH]
            r = cpu_attention_sample(args.seed, args.cpu_seconds, lens=sub)
            t_full = r["t_layer"] * float(lens0.sum()) / float(sub.sum())
            cpu = {"value": len(lens0) / (cfg.num_layers * t_full), "unit": "tok/s", "cores": r["threads"],
                   "kind": "port",
                   "sample": (f"{r['reps']} x one decode-attention layer over {len(sub)} of the {len(lens0)} "
                              f"config-5 sequences (f32 C/OpenMP oracle), layer time scaled by the context "
                              f"sum to all {len(lens0)} and to 28 layers per token step; GEMMs excluded; "
                              f"{cpu_info()}")}
        else:
            r = cpu_attention_sample(args.seed, args.cpu_seconds)
            cpu = {"value": r["tok_s"], "unit": "tok/s", "cores": r["threads"], "kind": "port",
                   "sample": (f"{r['reps']} x one decode-attention layer ({len(lens0)} seqs, "
                              f"ctx U[{CTX_LO},{CTX_HI}], f32 C/OpenMP oracle), scaled to 28 layers per "
                              f"token step; GEMMs excluded; {cpu_info()}")}

    if world == 1 and not args.no_extras:
        # each kernel on its own BASELINE config (one GPU; inputs cycled beyond L2)
        for name, kern in (("prefill", "prefill"), ("append", "append"), ("decode_fp8", "decode_fp8"),
                           ("decode_fp8_config5", "decode5_fp8"), ("copy_blocks", "copy"),
                           ("swap_blocks", "swap"), ("gather_kv_cache", "gather")):
            lines = KERNEL_BENCH[kern](args, torch.device("cuda", local))
            extras[name] = lines[0] if len(lines) == 1 else {ln["config"]: ln for ln in lines}
            torch.cuda.empty_cache()

    if args.config == 5:
        workload = ("config5: qwen3-asr-1.7B decode step, 28 layers, 512 sequences sharded over "
                    f"{world} GPU(s) by KV bytes ({len(lens0)} on rank 0), ctx log-U[64,4096], block_size 16")
        model_name = "Qwen3-ASR-1.7B text decoder (random init)"
    else:
        workload = "config2: qwen3-asr-0.6B decode step, 28 layers, B=64 per GPU, ctx U[200,1500], block_size 16"
        model_name = "Qwen3-ASR-0.6B text decoder (random init)"
    if rank == 0:
        k_steps = main["k_steps"]
        line = {
            "metric": METRIC, "value": main["value"], "unit": "tok/s", "n_gpus": world, "steps": k_steps,
            "warmup": main["w_steps"], "ms_per_step": main["dev_ms"] / k_steps, "higher_is_better": True,
            "scaling": "strong" if args.config == 5 else "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded contexts, random-init weights, N(0,1) cache)",
            "config": {"workload": workload, "model": model_name, "global_batch": main["global_batch"],
                       "seq_len": int(lens0.mean()), "parallelism": f"dp{world} (request-sharded)",
                       "graph_cols": main["cols"],
                       "l2": (f"inputs larger than L2 (per step {main['kv_step_gb']:.1f} GB KV + "
                              f"{weight_gb:.1f} GB weights on rank 0)")},
            "roofline": _roofline(main, peak, peak_kind),
            "cpu_baseline": cpu,
            "e2e": main["e2e"],
            "gpu_launches": 2 * cfg.num_layers * k_steps,
            "ranks": main["ranks"],
            "device_loop": main["device_loop"],
            "clocks": clk,
        }
        line.update(extras)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# -------------------------------------------------- kernel microbenchmarks
def _events_time(fn, iters):
    """Mean device ms per call of fn(i): the calls are captured once into a CUDA graph
    and the replay is timed with CUDA events on its stream, so host launch overhead
    is not counted (3 eager warm-ups and one warm replay first)."""
    import torch

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(3):
            fn(i)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(iters):
                fn(i)
        g.replay()
        s.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s)
        g.replay()
        b.record(s)
        s.synchronize()
    torch.cuda.current_stream().wait_stream(s)
    ms = a.elapsed_time(b) / iters
    del g
    return ms


HQ, HKV, D = 16, 8, 128
L2_BYTES = 126 * 2**20


def _sets_for(bytes_per_set, cap=16):
    """Independent input sets the timed launches cycle through: together at least
    4x the 126 MB L2, so no launch finds the previous launches' data in L2."""
    return max(1, min(cap, -(-4 * L2_BYTES // max(1, int(bytes_per_set)))))


def _pool(dev, nb, layers, dtype):
    import torch

    x = 16 // torch.empty((), dtype=dtype).element_size()
    return [(torch.randn(nb, HKV, D // x, BLOCK_SIZE, x, device=dev).to(dtype),
             torch.randn(nb, HKV, D, BLOCK_SIZE, device=dev).to(dtype)) for _ in range(layers)]


def _tables(rng, lens, nb, cols=None):
    import numpy as np

    blocks = [-(-int(n) // BLOCK_SIZE) for n in lens]
    perm = rng.permutation(np.arange(1, nb))
    t = np.zeros((len(lens), cols or max(blocks)), np.int32)
    off = 0
    for i, n in enumerate(blocks):
        t[i, :n] = perm[off:off + n]
        off += n
    return t


def _hbm_line(kernel, config, ms, alg, **extra):
    peak, kind = load_peaks()
    gbs = alg / ms / 1e6
    d = {"kernel": kernel, "config": config, "us": ms * 1e3, "bytes": alg, "achieved": gbs, "unit": "GB/s",
         "peak": peak, "frac": gbs / peak, "peak_source": kind}
    d.update(extra)
    return d


def kb_decode(args, dev, which="decode"):
    import numpy as np
    import torch

    from vasr_paged_attn import mistralrs_paged_attn as pa

    rng = np.random.default_rng(args.seed)
    dtype = torch.float32 if which == "config1" else torch.bfloat16
    if which == "config1":
        lens = np.array([138, 513, 1024, 2049])
        nb, layers = 512, 1
    elif which == "decode5":  # config 5 attention shapes: 512 sequences, ctx ~log-U[64, 4096]
        from vasr_paged_attn.workloads import config5_context_lens

        lens = config5_context_lens(args.seed)
        nb = sum(-(-int(n) // BLOCK_SIZE) for n in lens) + 1
        layers = min(args.layers, 4)  # 4 x 2 GB pools: well above L2
    else:
        lens = context_lens(args.seed, 0)
        nb = sum(-(-int(n) // BLOCK_SIZE) for n in lens) + 1
        layers = args.layers
    caches = _pool(dev, nb, layers, dtype)
    t = torch.from_numpy(_tables(rng, lens, nb)).to(dev)
    ctx = torch.from_numpy(lens.astype(np.int32)).to(dev)
    q = torch.randn(len(lens), HQ, D, device=dev).to(dtype)
    mcl = int(lens.max())
    out = torch.empty_like(q)
    es = q.element_size()

    def launch(i):
        kc, vc = caches[i % layers]
        pa.paged_attention(q, None, None, kc, vc, t, ctx, None, mcl, D ** -0.5, 1.0, None, out=out)

    ms = _events_time(launch, args.iters)
    alg = int(lens.sum()) * HKV * D * 2 * es + q.numel() * es * 2
    lines = [_hbm_line("paged_decode", {"config1": "config1", "decode5": "config5"}.get(which, "config2"),
                       ms, alg, layers_cycled=layers)]
    if which == "config1":
        kn = torch.randn(4, HKV, D, device=dev)
        sl = torch.from_numpy((t[:, 0].cpu().numpy().astype(np.int64) * BLOCK_SIZE)).to(dev)
        ms = _events_time(lambda i: pa.reshape_and_cache(kn, kn, None, None, caches[0][0], caches[0][1], sl),
                          args.iters)
        lines.append(_hbm_line("kv_append", "config1", ms, 4 * HKV * D * 4 * 2 * 2))
    return lines


def kb_decode_fp8(args, dev, which="config2"):
    """Config 2 (or config 5) shapes over fp8 (E4M3) pages with per-tensor scales (half the KV bytes)."""
    import numpy as np
    import torch

    from vasr_paged_attn import mistralrs_paged_attn as pa

    rng = np.random.default_rng(args.seed)
    if which == "config5":
        from vasr_paged_attn.workloads import config5_context_lens

        lens = config5_context_lens(args.seed)
        layers = min(args.layers, 4)
    else:
        lens = context_lens(args.seed, 0)
        layers = args.layers
    nb = sum(-(-int(n) // BLOCK_SIZE) for n in lens) + 1
    caches = [((torch.randn(nb, HKV, D // 16, BLOCK_SIZE, 16, device=dev) * 8).to(torch.float8_e4m3fn),
               (torch.randn(nb, HKV, D, BLOCK_SIZE, device=dev) * 8).to(torch.float8_e4m3fn))
              for _ in range(layers)]
    sk = torch.tensor([0.125], device=dev)
    sv = torch.tensor([0.125], device=dev)
    t = torch.from_numpy(_tables(rng, lens, nb)).to(dev)
    ctx = torch.from_numpy(lens.astype(np.int32)).to(dev)
    q = torch.randn(len(lens), HQ, D, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)

    def launch(i):
        kc, vc = caches[i % layers]
        pa.paged_attention(q, sk, sv, kc, vc, t, ctx, None, int(lens.max()), D ** -0.5, 1.0, None, out=out)

    ms = _events_time(launch, args.iters)
    alg = int(lens.sum()) * HKV * D * 2 + q.numel() * 2 * 2
    return [_hbm_line("paged_decode_fp8", f"{which} shapes, fp8 E4M3 pages", ms, alg, layers_cycled=layers)]


def kb_append(args, dev):
    import numpy as np
    import torch

    from vasr_paged_attn import mistralrs_paged_attn as pa

    rng = np.random.default_rng(args.seed)
    lines = []
    for name, ntok, per_seq in (("config3_chunk", 32 * 256, 256), ("config2_decode", 64, 1)):
        nb = ntok // per_seq * (-(-per_seq // BLOCK_SIZE)) + 16 + 1
        nset = _sets_for(2 * ntok * HKV * D * 2 + nb * HKV * D * BLOCK_SIZE * 2 * 2)
        pools = _pool(dev, nb, nset, torch.bfloat16)
        ks = [torch.randn(ntok, HKV, D, device=dev).to(torch.bfloat16) for _ in range(nset)]
        vs = [torch.randn(ntok, HKV, D, device=dev).to(torch.bfloat16) for _ in range(nset)]
        nseq = ntok // per_seq
        t = _tables(rng, [per_seq] * nseq, nb)
        pos = np.arange(per_seq)
        slots = np.concatenate([t[i, pos // BLOCK_SIZE].astype(np.int64) * BLOCK_SIZE + pos % BLOCK_SIZE
                                for i in range(nseq)])
        sl = torch.from_numpy(slots).to(dev)
        ms = _events_time(lambda i: pa.reshape_and_cache(ks[i % nset], vs[i % nset], None, None,
                                                         pools[i % nset][0], pools[i % nset][1], sl), args.iters)
        lines.append(_hbm_line("kv_append", name, ms, ntok * HKV * D * 2 * 2 * 2, tokens=ntok,
                               input_sets_cycled=nset))
        # the same tokens into fp8 (E4M3) pages: bf16 read, one byte per element written
        del pools
        p8 = [(torch.zeros(nb, HKV, D // 16, BLOCK_SIZE, 16, dtype=torch.uint8, device=dev).view(torch.float8_e4m3fn),
               torch.zeros(nb, HKV, D, BLOCK_SIZE, dtype=torch.uint8, device=dev).view(torch.float8_e4m3fn))
              for _ in range(nset)]
        sk = torch.tensor([0.05], device=dev)
        ms = _events_time(lambda i: pa.reshape_and_cache(ks[i % nset], vs[i % nset], sk, sk, p8[i % nset][0],
                                                         p8[i % nset][1], sl), args.iters)
        lines.append(_hbm_line("kv_append_fp8", name, ms, ntok * HKV * D * 2 * (2 + 1), tokens=ntok,
                               input_sets_cycled=nset))
        del p8, ks, vs
    for ln in lines:
        ln["config"] = ln["config"] + ("_fp8" if ln["kernel"] == "kv_append_fp8" else "")
    return lines


def kb_gather(args, dev):
    """gather_kv_cache of config 3's full prompts (32 x U[100, 800] tokens) from bf16 and fp8 pages."""
    import numpy as np
    import torch

    from vasr_paged_attn import mistralrs_paged_attn as pa
    from vasr_paged_attn.workloads import config3_rounds

    rng = np.random.default_rng(args.seed)
    lens, _ = config3_rounds(args.seed)
    lens = np.asarray(lens, np.int64)
    nb = sum(-(-int(n) // BLOCK_SIZE) for n in lens) + 1
    t = torch.from_numpy(_tables(rng, lens, nb)).to(dev)
    cu = torch.from_numpy(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)).to(dev)
    total = int(lens.sum())
    nset = _sets_for(nb * HKV * D * BLOCK_SIZE * 2 * 2 + total * HKV * D * 2 * 2)
    pools = _pool(dev, nb, nset, torch.bfloat16)
    ms = _events_time(lambda i: pa.gather_kv_cache(pools[i % nset][0], pools[i % nset][1], None, None, t, cu,
                                                   None, total), args.iters)
    lines = [_hbm_line("gather_kv_cache", "config3 prompts, bf16 pages", ms, total * HKV * D * 2 * 2 * 2,
                       tokens=total, input_sets_cycled=nset)]
    del pools
    nset = _sets_for(nb * HKV * D * BLOCK_SIZE * 2 + total * HKV * D * 2 * 2)
    p8 = [((torch.randn(nb, HKV, D // 16, BLOCK_SIZE, 16, device=dev) * 8).to(torch.float8_e4m3fn),
           (torch.randn(nb, HKV, D, BLOCK_SIZE, device=dev) * 8).to(torch.float8_e4m3fn)) for _ in range(nset)]
    sk = torch.tensor([0.125], device=dev)
    ms = _events_time(lambda i: pa.gather_kv_cache(p8[i % nset][0], p8[i % nset][1], sk, sk, t, cu,
                                                   torch.bfloat16, total), args.iters)
    lines.append(_hbm_line("gather_kv_cache_fp8", "config3 prompts, fp8 pages -> bf16", ms,
                           total * HKV * D * 2 * (1 + 2), tokens=total, input_sets_cycled=nset))
    return lines


def kb_prefill(args, dev, fp8=False):
    import numpy as np
    import torch

    from vasr_paged_attn import mistralrs_paged_attn as pa
    from vasr_paged_attn.workloads import config3_rounds

    rng = np.random.default_rng(args.seed)
    lens, rounds = config3_rounds(args.seed)
    nb = sum(-(-int(n) // BLOCK_SIZE) for n in lens) + 1
    # page pools (one per layer) and query sets cycled so that the launches' inputs exceed L2
    nset = _sets_for(nb * HKV * D * BLOCK_SIZE * 2 * 2 + 2 * 32 * 256 * HQ * D * 2, cap=8)
    sk = sv = None
    if fp8:  # the same pages in E4M3 with per-tensor scales
        pools = [((torch.randn(nb, HKV, D // 16, BLOCK_SIZE, 16, device=dev) * 8).to(torch.float8_e4m3fn),
                  (torch.randn(nb, HKV, D, BLOCK_SIZE, device=dev) * 8).to(torch.float8_e4m3fn))
                 for _ in range(nset)]
        sk = sv = torch.tensor([0.125], device=dev)
    else:
        pools = _pool(dev, nb, nset, torch.bfloat16)
    t_all = _tables(rng, lens, nb)
    total_flops, total_ms = 0.0, 0.0
    rounds_us = []
    for r in rounds:
        idx = [i for (i, _, _) in r]
        chunk = np.array([n for (_, _, n) in r])
        ctx = np.array([s + n for (_, s, n) in r])
        cu = np.concatenate([[0], np.cumsum(chunk)]).astype(np.int32)
        qs = [torch.randn(int(chunk.sum()), HQ, D, device=dev).to(torch.bfloat16) for _ in range(nset)]
        bt = torch.from_numpy(t_all[idx]).to(dev)
        dctx = torch.from_numpy(ctx.astype(np.int32)).to(dev)
        dcu = torch.from_numpy(cu).to(dev)
        mq = int(chunk.max())
        ms = _events_time(lambda i: pa.paged_attention_varlen_prefill(qs[i % nset], pools[i % nset][0],
                                                                      pools[i % nset][1], bt, dctx, dcu, sk, sv,
                                                                      D ** -0.5, 1.0, mq), args.iters)
        vis = sum(sum(int(s) + j + 1 for j in range(int(n))) for (_, s, n) in r)
        total_flops += 4.0 * D * HQ * vis
        total_ms += ms
        rounds_us.append(round(ms * 1e3, 2))
    tflops = total_flops / (total_ms / 1e3) / 1e12
    tpeak, tkind = load_tensor_peak()
    return [{"kernel": "paged_prefill_varlen" + ("_fp8" if fp8 else ""),
             "config": "config3 (one layer, all chunk rounds)", "rounds": len(rounds),
             "us": total_ms * 1e3, "flops": total_flops, "achieved": tflops, "unit": "TFLOP/s",
             "peak": tpeak, "frac": tflops / tpeak, "peak_source": tkind, "input_sets_cycled": nset,
             "rounds_us": rounds_us,
             "tflop_28_layers": total_flops * 28 / 1e12}]


def kb_copy(args, dev):
    """Config 4 copy_blocks: 4096 seeded src -> dst pairs over 200k-block pools, as many layers as fit."""
    import numpy as np
    import torch

    from vasr_paged_attn import mistralrs_paged_attn as pa

    rng = np.random.default_rng(args.seed)
    free, _ = torch.cuda.mem_get_info()
    nb = args.pool_blocks
    per_layer = nb * HKV * D * BLOCK_SIZE * 2 * 2
    layers = max(1, min(args.layers, int(free * 0.8 // per_layer)))
    caches = [(torch.empty(nb, HKV, D // 8, BLOCK_SIZE, 8, dtype=torch.bfloat16, device=dev),
               torch.empty(nb, HKV, D, BLOCK_SIZE, dtype=torch.bfloat16, device=dev)) for _ in range(layers)]
    perm = rng.permutation(nb)
    pairs = torch.from_numpy(np.stack([perm[:4096], perm[4096:8192]], 1).astype(np.int64)).to(dev)
    ms = _events_time(lambda i: pa.copy_blocks([c[0] for c in caches], [c[1] for c in caches], pairs),
                      args.iters)
    alg = 4096 * layers * 2 * (HKV * D * BLOCK_SIZE * 2) * 2
    return [_hbm_line("copy_blocks", "config4" if nb == 200_000 else f"config4 pairs, {nb}-block pools", ms, alg,
                      layers_allocated=layers,
                      ms_28_layers_extrapolated=ms * 28 / layers)]


def kb_swap(args, dev):
    """1024 blocks of one layer cache device <-> pinned host, against pinned cudaMemcpyAsync of the
    same bytes (the host link is the roofline)."""
    import numpy as np
    import torch

    from vasr_paged_attn import mistralrs_paged_attn as pa

    rng = np.random.default_rng(args.seed)
    nb_dev, nb_host = 8192, 2048
    dcache = torch.randn(nb_dev, HKV, D, BLOCK_SIZE, device=dev).to(torch.bfloat16)
    hcache = torch.empty(nb_host, HKV, D, BLOCK_SIZE, dtype=torch.bfloat16).pin_memory()
    src = rng.permutation(nb_dev)[:1024]
    dst = rng.permutation(nb_host)[:1024]
    out_map = torch.from_numpy(np.stack([src, dst], 1).astype(np.int64)).to(dev)
    in_map = torch.from_numpy(np.stack([dst, src], 1).astype(np.int64)).to(dev)
    blk = HKV * D * BLOCK_SIZE * 2
    ms_out = _events_time(lambda i: pa.swap_blocks(dcache, hcache, out_map), args.iters)
    ms_in = _events_time(lambda i: pa.swap_blocks(hcache, dcache, in_map), args.iters)
    big = torch.empty(1024 * blk // 2, dtype=torch.bfloat16, device=dev)
    hbig = torch.empty_like(big, device="cpu").pin_memory()
    ms_d2h = _events_time(lambda i: hbig.copy_(big, non_blocking=True), args.iters)
    ms_h2d = _events_time(lambda i: big.copy_(hbig, non_blocking=True), args.iters)
    n = 1024 * blk
    d2h, h2d = n / ms_out / 1e6, n / ms_in / 1e6
    pd2h, ph2d = n / ms_d2h / 1e6, n / ms_h2d / 1e6
    return [{"kernel": "swap_blocks", "config": "config4 (1024 blocks of one layer cache)", "bytes": n,
             "us_d2h": ms_out * 1e3, "us_h2d": ms_in * 1e3, "achieved": min(d2h, h2d), "unit": "GB/s",
             "peak": min(pd2h, ph2d), "frac": min(d2h / pd2h, h2d / ph2d),
             "peak_source": "pinned cudaMemcpyAsync of the same bytes, measured in this run",
             "d2h_GB/s": d2h, "h2d_GB/s": h2d, "pinned_copy_d2h_GB/s": pd2h, "pinned_copy_h2d_GB/s": ph2d}]


KERNEL_BENCH = {
    "decode": lambda a, d: kb_decode(a, d, "decode"),
    "decode5": lambda a, d: kb_decode(a, d, "decode5"),
    "config1": lambda a, d: kb_decode(a, d, "config1"),
    "decode_fp8": kb_decode_fp8,
    "decode5_fp8": lambda a, d: kb_decode_fp8(a, d, "config5"),
    "append": kb_append,
    "gather": kb_gather,
    "prefill": lambda a, d: kb_prefill(a, d, fp8=False),
    "prefill_fp8": lambda a, d: kb_prefill(a, d, fp8=True),
    "copy": kb_copy,
    "swap": kb_swap,
}


def run_kernel_bench(args):
    """One JSON line per kernel: device time per launch and the roofline fraction."""
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    for ln in KERNEL_BENCH[args.kernel](args, dev):
        print(json.dumps(ln), flush=True)


def main():
    args = parse_args()
    if args.kernel is not None:
        run_kernel_bench(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
