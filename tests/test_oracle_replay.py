"""The oracle's rank-c replay against the exact untiered recurrence, on the CPU, for chunk
lengths up to the largest compiled one (c = 64).

With fp32 cold storage nothing is quantised, so on every token the exact state the tiered
pool implies (hot slice + cold slice replayed through the partial ring, `materialize`) must
equal the fresh fp32 state, in particular right after each flush, and the exact-correction
readout (mode "corr") must equal the fresh readout.  Both within fp32 reassociation.  This
pins the replay the GPU kernels are compared with at the chunk lengths the reference's own
fixtures (c = 4) do not reach.
"""
import pytest
import torch

import oracle as O


@pytest.mark.parametrize("c", [1, 2, 4, 16, 64])
def test_replay_equals_fresh_recurrence(c):
    b, H, P, N, G, pb = 3, 8, 16, 32, 2, 8
    steps = 2 * c + 3   # two flushes and part of a third chunk
    prm = O.make_params(H, G, N, seed=c)[0]
    xs, dts, Bs, Cs = O.make_inputs(b, H, P, G, N, steps, seed=c)
    state0 = torch.randn(b, H, P, N, generator=torch.Generator().manual_seed(100 + c)) * 0.1 ** 0.5
    slots = torch.arange(b)
    for mode in ("stale", "corr"):
        pool = O.TieredPoolRef(b, H, P, N, G, pb, c, torch.float32, torch.bfloat16)
        O.prefill_split(pool, slots, state0)
        fresh = state0.clone()
        flushes = 0
        for s in range(steps):
            args = (xs[s], dts[s], Bs[s], Cs[s], prm["A"], prm["D"], prm["dt_bias"], 1e-3)
            y_t = O.tiered_step(pool, slots, *args, mode=mode)
            y_f = O.fresh_step(fresh, slots, *args)
            if mode == "corr":
                torch.testing.assert_close(y_t, y_f, rtol=2e-5, atol=2e-5, msg=lambda m: f"c={c} step {s}: {m}")
            torch.testing.assert_close(O.materialize(pool, slots, prm["A"]), fresh, rtol=2e-5, atol=2e-6,
                                       msg=lambda m: f"{mode} c={c} step {s}: {m}")
            if int(pool.t[0]) % c == 0:
                flushes += 1
                assert float(pool.glog.abs().max()) == 0.0   # re-based at the flush
        assert flushes == steps // c
