"""The multi-rank plumbing on CPU: two gloo ranks as separate processes.

What runs on N GPUs has two host-side parts that need no GPU: the timing
reduction (every rank's step time, the maximum reported) with the barriers
around it, and the sharding of a batch by `shard_range` (the helper the CNN,
GEMM and FFT workloads slice their batches with) — rank r runs units
[r*B/N, (r+1)*B/N) and the all-gather lays the ranks' logits out in rank
order, so the gathered array is the whole batch's. Here each rank computes its
shard's logits with the oracle's GAP + FC and the shards are gathered over
gloo, in the layout the NCCL all-gather uses.
"""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, errors):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        sys.path.insert(0, str(ROOT))
        import datetime

        import torch
        import torch.distributed as dist

        import bench
        from mantle_cuda.workloads import shard_range
        from oracle import oracle as O

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        try:
            # the step time reported is the slowest rank's
            bench.barrier(world)
            got = bench.max_over_ranks(world, 1.5 + rank)
            assert got == 1.5 + (world - 1), got

            # batch sharding and the rank-ordered gather
            n, hw, c, classes = 12, 9, 64, 10
            rng = np.random.default_rng(21)  # the same inputs on every rank
            act = O.bf16_bits(np.abs(rng.standard_normal((n, hw, 1, c)).astype(np.float32)))
            w = (rng.standard_normal((c, classes)) * np.sqrt(2.0 / c)).astype(np.float32)
            lo, hi = shard_range(n, rank, world)
            mine = torch.from_numpy(O.gap_fc(act[lo:hi], w))
            parts = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(parts, mine)
            gathered = torch.cat(parts).numpy()
            assert np.array_equal(gathered, O.gap_fc(act, w))
            bench.barrier(world)
        finally:
            dist.destroy_process_group()
    except BaseException as e:  # reported to the parent, which fails the test
        errors.put(f"rank {rank}: {type(e).__name__}: {e}")


def test_two_gloo_ranks_time_and_gather():
    world = 2
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, errors)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not alive, "a rank did not finish"
    assert not msgs, "; ".join(msgs)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
