"""Request-level data parallelism for the paged decode path.

The reference runs everything on one device (vasr-runtime/src/device.rs:23,39)
and has no collective; across B200s the paged path shards by request: every
sequence's pages, block table and decode state live on one GPU, so ranks never
exchange KV data. The host decides placement:

* ``lpt_shard``: longest-processing-time-first assignment of a batch by
  expected KV bytes (context length), which balances per-GPU HBM traffic of
  the decode kernel — the dominant per-step cost.
* ``pick_rank_for_admission``: continuous-batching admission sends a new
  request to the rank with the most free blocks
  (PagedCacheStats.free_blocks, vasr-paged-attn/src/paged_cache_runtime.rs:472-476),
  subject to the same projected-KV check as
  vasr-models/src/inference/batch_scheduler.rs:100-113.
* ``gather_counts``: the only cross-rank traffic — an end-of-run host
  gather of small per-rank counters (tokens decoded, steps, errors).
"""
from __future__ import annotations

import heapq
from typing import Optional, Sequence


def lpt_shard(context_lens: Sequence[int], world_size: int) -> list[list[int]]:
    """Indices of ``context_lens`` per rank; heaviest first onto the lightest rank.

    Deterministic: ties break by rank then by index, so every rank computes
    the same plan without communicating.
    """
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    order = sorted(range(len(context_lens)), key=lambda i: (-int(context_lens[i]), i))
    heap = [(0, r) for r in range(world_size)]
    shards: list[list[int]] = [[] for _ in range(world_size)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + int(context_lens[i]), r))
    for s in shards:
        s.sort()
    return shards


def shard_loads(context_lens: Sequence[int], shards: Sequence[Sequence[int]]) -> list[int]:
    return [sum(int(context_lens[i]) for i in s) for s in shards]


def pick_rank_for_admission(free_blocks: Sequence[int], running: Sequence[int], prompt_len: int,
                            block_size: int, capacity: Sequence[int]) -> Optional[int]:
    """Rank with the most free blocks that passes the projected-KV admission check, else None.

    A rank admits when used + prompt blocks + decode headroom (one block per
    running sequence, at least one) fits its allocatable capacity
    (batch_scheduler.rs:100-113).
    """
    best, best_free = None, -1
    prompt_blocks = -(-prompt_len // block_size)
    for r, free in enumerate(free_blocks):
        used = capacity[r] - free
        if used + prompt_blocks + max(running[r], 1) > capacity[r]:
            continue
        if free > best_free:
            best, best_free = r, free
    return best


def gather_counts(counts: Sequence[int], group=None) -> list[list[int]]:
    """All ranks' small integer counters (host tensors over gloo, or NCCL with CUDA tensors)."""
    import torch
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return [list(counts)]
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.tensor(list(counts), dtype=torch.int64, device=dev)
    out = [torch.zeros_like(t) for _ in range(dist.get_world_size(group))]
    dist.all_gather(out, t, group=group)
    return [o.cpu().tolist() for o in out]
