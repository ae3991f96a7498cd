"""The continuous-batching admission process of bench.py's ragged leg (host side, CPU).

Seeded and reproducible; 384-448 live sequences in a padded batch of 448 rows; a slot is
never live in two rows at once and is only reused after its sequence finished; admitted
slots are exactly the rows that change from padding or another slot.
"""
import numpy as np
import pytest

import bench


def test_ragged_schedule_invariants():
    rows, slots, steps = 448, 2048, 700
    initial, sched, admits = bench.ragged_schedule(steps, rows, slots, seed=3000)
    again = bench.ragged_schedule(steps, rows, slots, seed=3000)
    assert np.array_equal(sched, again[1]) and np.array_equal(initial, again[0])
    live = (sched >= 0).sum(axis=1)
    assert live.min() >= 384 and live.max() <= rows
    assert sched.max() < slots and sched.min() >= -1
    assert set(initial.tolist()) == set(sched[0][sched[0] >= 0].tolist())
    finished = set()
    prev = sched[0]
    for k in range(1, steps):
        cur = sched[k]
        ids = cur[cur >= 0]
        assert len(set(ids.tolist())) == ids.size, f"step {k}: a slot sits in two rows"
        changed = (cur != prev) & (cur >= 0)
        assert sorted(cur[changed].tolist()) == sorted(admits[k].tolist()), f"step {k}: admissions"
        gone = set(prev[(prev >= 0) & (cur != prev)].tolist())
        finished |= gone
        for s in admits[k].tolist():
            assert s not in set(prev[prev >= 0].tolist()), f"step {k}: slot {s} admitted while live"
        prev = cur
    assert sum(a.size for a in admits) > 0 and len(finished) > 0


def test_ragged_schedule_rejects_a_pool_no_larger_than_the_batch():
    with pytest.raises(ValueError, match="slots > rows"):
        bench.ragged_schedule(4, 448, 448, seed=0)


def test_ragged_schedule_over_a_sharded_global_slot_space():
    """ws GPUs share one global slot space: rows of part q (the q-th block of 448) only ever
    hold slots of shard q (sharding.slot_range), every part keeps >= 384 live rows, and the
    per-GPU view (local slot = global - first owned) is a valid single-GPU schedule."""
    import torch
    from nested_ssm_b200 import sharding as SH
    ws, rows, slots, steps = 4, 448, 2048, 300
    initial, sched, admits = bench.ragged_schedule(steps, ws * rows, ws * slots, seed=3000, shards=ws)
    for q in range(ws):
        lo, hi = SH.slot_range(ws * slots, q, ws)
        part = sched[:, q * rows:(q + 1) * rows]
        ids = part[part >= 0]
        assert ids.min() >= lo and ids.max() < hi
        assert bool((SH.owner_of(torch.from_numpy(ids), ws * slots, ws) == q).all())
        assert (part >= 0).sum(axis=1).min() >= 384
    for k in range(steps):
        ids = sched[k][sched[k] >= 0]
        assert len(set(ids.tolist())) == ids.size
    assert sum(a.size for a in admits) > 0
