"""Slot sharding over ranks (host logic, CPU, gloo world_size 2).

Each rank owns half the slot pool and runs the state op (the CPU oracle stands in for
the kernel here) on the rows of the global batch whose slots it owns; the gathered
outputs and the per-rank pools must equal one process serving the whole pool."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import oracle as O
from nested_ssm_b200 import sharding as SH

H, P, N, G, PB, C, S, B, STEPS = 8, 16, 32, 2, 8, 2, 10, 7, 5


def test_slot_range_partitions():
    for S_, w in [(10, 2), (11, 4), (3, 4), (4096, 8)]:
        ranges = [SH.slot_range(S_, r, w) for r in range(w)]
        assert ranges[0][0] == 0 and ranges[-1][1] == S_
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        own = SH.owner_of(torch.arange(-1, S_ + 1), S_, w)
        assert own[0] == -1 and own[-1] == -1
        for r, (lo, hi) in enumerate(ranges):
            assert torch.all(own[1 + lo:1 + hi] == r)


def test_local_batch_skips_pad_and_maps_slots():
    slots = torch.tensor([9, -1, 0, 5, 4, -1, 7])
    r0, l0 = SH.local_batch(slots, 0, 2, 10)
    r1, l1 = SH.local_batch(slots, 1, 2, 10)
    assert r0.tolist() == [2, 4] and l0.tolist() == [0, 4]
    assert r1.tolist() == [0, 3, 6] and l1.tolist() == [4, 0, 2]


def _case():
    prm = O.make_params(H, G, N, seed=3)[0]
    xs, dts, Bs, Cs = O.make_inputs(B, H, P, G, N, STEPS, seed=3, io_dtype=torch.float32)
    g = torch.Generator().manual_seed(4)
    state0 = torch.randn(S, H, P, N, generator=g) * 0.3
    batches = [torch.tensor([3, 8, -1, 0, 6, 9, 1]), torch.tensor([8, 3, 6, -1, -1, 0, 5])]
    return prm, xs, dts, Bs, Cs, state0, batches


def _serve(pool, rows_slots, prm, x, dt, Bm, Cm):
    rows, sl = rows_slots
    return O.tiered_step(pool, sl, x[rows], dt[rows], Bm[rows], Cm[rows], prm["A"], prm["D"], prm["dt_bias"])


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        prm, xs, dts, Bs, Cs, state0, batches = _case()
        lo, hi = SH.slot_range(S, rank, world)
        pool = O.TieredPoolRef(hi - lo, H, P, N, G, PB, C, O.FP8, torch.float32)
        O.prefill_split(pool, torch.arange(hi - lo), state0[lo:hi])
        ys = []
        for s in range(STEPS):
            slots = batches[s % 2]
            rows, loc = SH.local_batch(slots, rank, world, S)
            y = _serve(pool, (rows, loc), prm, xs[s], dts[s], Bs[s], Cs[s])
            ys.append(SH.gather_rows(y, rows, B))
        q.put((rank, torch.stack(ys), pool.cold.clone(), pool.hot.clone(), pool.t.clone()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_slot_sharding_matches_single_process():
    prm, xs, dts, Bs, Cs, state0, batches = _case()
    ref = O.TieredPoolRef(S, H, P, N, G, PB, C, O.FP8, torch.float32)
    O.prefill_split(ref, torch.arange(S), state0)
    y_ref = []
    for s in range(STEPS):
        slots = batches[s % 2]
        y_ref.append(O.tiered_step(ref, slots, xs[s], dts[s], Bs[s], Cs[s], prm["A"], prm["D"], prm["dt_bias"]))
    y_ref = torch.stack(y_ref)

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, y, cold, hot, t = q.get(timeout=120)
        res[r] = (y, cold, hot, t)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # the per-rank batches are smaller, so the CPU einsums block differently: equal to
    # fp32 rounding, cold codes within one ulp, bookkeeping exact
    for r in range(2):
        torch.testing.assert_close(res[r][0], y_ref, rtol=1e-5, atol=1e-6)
        lo, hi = SH.slot_range(S, r, 2)
        d = (O.fp8_ordered_codes(res[r][1]) - O.fp8_ordered_codes(ref.cold[lo:hi])).abs()
        assert int(d.max()) <= 1
        torch.testing.assert_close(res[r][2], ref.hot[lo:hi], rtol=1e-5, atol=1e-6)
        assert torch.equal(res[r][3], ref.t[lo:hi])
