"""Host-side pieces of bench.py and the workload builders that need no GPU:
the batch split every sharded workload uses, and the CPU timing that both the
reference arm and the GPU arm's cpu_baseline legs go through."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
from mantle_cuda.workloads import shard_range  # noqa: E402


@pytest.mark.parametrize("total,world", [(256, 1), (256, 2), (256, 8), (8, 8), (16384, 4)])
def test_shard_range_tiles_the_batch_in_rank_order(total, world):
    got = [shard_range(total, r, world) for r in range(world)]
    assert got[0][0] == 0 and got[-1][1] == total
    assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
    assert len({hi - lo for lo, hi in got}) == 1


def test_shard_range_refuses_uneven_splits_and_bad_ranks():
    with pytest.raises(ValueError):
        shard_range(8, 0, 3)
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


def test_cpu_timed_counts_every_call_and_fills_the_budget():
    calls = []

    def one():
        calls.append(1)
        return 5

    r = bench.cpu_timed(one, steps=4, budget_s=0.05, warm_s=0.01)
    assert r["steps"] == 4 and r["calls"] == 4 * r["reps_per_step"]
    assert r["units_per_s"] == pytest.approx(5 * r["calls"] / r["seconds"])
    assert r["seconds"] >= 0.01


def test_cpu_timed_takes_fewer_steps_when_a_call_is_slow():
    import time

    def slow():
        time.sleep(0.02)
        return 1

    r = bench.cpu_timed(slow, steps=50, budget_s=0.1, warm_s=0.0)
    assert r["steps"] <= 5 and r["reps_per_step"] == 1


def test_both_arms_print_the_same_scatter_config():
    assert bench.scatter_config(1) == bench.scatter_config(1, 1 << 24, 1 << 16, 1 << 20)
