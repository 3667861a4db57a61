"""Multi-rank host logic of the request-sharded decode path, on CPU with gloo.

Each rank computes the same LPT plan without communicating, builds its own
shard's decode metadata with the C++ host mirror over its own page pool, and
the ranks exchange only small counters. A failing rank surfaces on the others
as an error from the short process-group timeout, not as a hang.
"""
import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO / "qwen3asr.rs_b200"))

from vasr_paged_attn import sharding  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_lpt_shard_is_balanced_and_complete():
    import numpy as np

    lens = np.random.default_rng(0).integers(64, 4096, size=512)
    for world in (1, 2, 4, 8):
        shards = sharding.lpt_shard(lens, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(512))
        loads = sharding.shard_loads(lens, shards)
        assert max(loads) - min(loads) <= int(lens.max())  # LPT bound
        assert max(loads) / (sum(loads) / world) < 1.02


def test_admission_prefers_most_free_and_respects_capacity():
    # 64-token prompt = 4 blocks + 3 blocks decode headroom: rank 2 (5 free) cannot take it,
    # rank 1 has the most free blocks among the ranks that can
    r = sharding.pick_rank_for_admission([10, 50, 5], [3, 3, 3], prompt_len=64, block_size=16,
                                         capacity=[100, 100, 100])
    assert r == 1
    assert sharding.pick_rank_for_admission([10, 50, 60], [3, 3, 3], 64, 16, [100, 100, 100]) == 2
    assert sharding.pick_rank_for_admission([1, 2], [1, 1], 64, 16, [10, 10]) is None


def _worker(rank, world, port, result_path, fail_rank):
    import numpy as np
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=15))
    try:
        from vasr_paged_attn import host

        lens = np.random.default_rng(5).integers(200, 1500, size=64)
        shards = sharding.lpt_shard(lens, world)
        mine = shards[rank]
        bs = 16
        blocks = [-(-int(lens[i] + 4) // bs) for i in mine]
        cache = host.metadata_cache(sum(blocks) + 1, 8, 128, bs)
        mgr = host.PagedBlockManager(sum(blocks) + 1, bs)
        for rid, i in enumerate(mine):
            mgr.allocate_slots(rid, int(lens[i]) + 4)
        tables = mgr.block_tables_for(list(range(len(mine))))
        meta = cache.decode_metadata_for_batch_step(tables, [int(lens[i]) for i in mine], 3, True)
        if rank == fail_rank:
            raise RuntimeError("injected host-side failure on this rank")
        ok = int(len(meta.slot_mapping) == len(mine) and
                 list(meta.context_lens) == [int(lens[i]) + 4 for i in mine])
        counts = sharding.gather_counts([len(mine), ok, int(sum(lens[i] for i in mine))])
        if rank == 0:
            Path(result_path).write_text(repr(counts))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run(world, fail_rank, tmp_path):
    port = _free_port()
    out = tmp_path / "counts.txt"
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(out), fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    return codes, out


def test_two_rank_sharded_metadata_and_counter_gather(tmp_path):
    codes, out = _run(2, -1, tmp_path)
    assert codes == [0, 0]
    counts = eval(out.read_text())  # list of [n_seqs, ok, kv_tokens] per rank
    assert sum(c[0] for c in counts) == 64
    assert all(c[1] == 1 for c in counts)
    loads = [c[2] for c in counts]
    assert max(loads) / min(loads) < 1.05


def test_failed_rank_is_reported_not_hung(tmp_path):
    codes, _ = _run(2, 1, tmp_path)
    assert codes[1] != 0          # the failing rank exits with its exception
    assert codes[0] is not None   # the survivor ends (timeout error), it does not hang
