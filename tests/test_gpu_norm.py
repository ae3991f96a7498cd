"""nssm_gated_rmsnorm (the mixer's norm(y, gate) after the state op) against the CPU oracle:
within one io ulp (fp32 sums of 1280 squares in another order; expf)."""
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,wdt", [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32),
                                       (torch.bfloat16, torch.float32)])
def test_gated_rmsnorm_matches_oracle(dtype, wdt):
    from nested_ssm_b200 import gated_rmsnorm
    gen = torch.Generator().manual_seed(3)
    b, dim, gs = 37, 10240, 1280
    y = torch.randn(b, 1, dim, generator=gen).to(dtype)
    z = torch.randn(b, 1, dim, generator=gen).to(dtype)
    w = (1.0 + 0.1 * torch.randn(dim, generator=gen)).to(wdt)
    want = O.gated_rmsnorm(y, z, w, 1e-5, gs)
    got = gated_rmsnorm(y.cuda(), z.cuda(), w.cuda(), 1e-5, gs).cpu()
    assert got.shape == want.shape and got.dtype == want.dtype
    ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -20   # one bf16 ulp (two roundings) / fp32 slack
    err = (got.float() - want.float()).abs()
    bound = want.float().abs() * ulp + 1e-6
    assert bool((err <= bound).all()), f"off by {float((err / bound).max()):.2f}x"
    if dtype == torch.bfloat16:   # fp32 outputs differ in the last bits almost everywhere
        assert float((err > 0).float().mean()) <= 5e-2


def _fused_vs_separate(b, S, gate_offset, seed):
    """Two pools from the same state take the same token: one through the step with the fused
    norm, one through the plain step and then gated_rmsnorm.  The pools must end bit-identical
    (the norm changes only what goes to out) and the outputs agree within two bf16 ulps, rarely
    differing at all (the sum of squares is accumulated in another order)."""
    import math
    from nested_ssm_b200 import TieredSlotPool, gated_rmsnorm, prefill_split, tiered_state_update
    H, P, N, G = 128, 80, 128, 8
    prm = O.make_params(H, G, N, seed=seed)[0]
    xs, dts, Bs, Cs = O.make_inputs(b, H, P, G, N, 5, seed=seed)
    gen = torch.Generator().manual_seed(seed)
    slots = torch.randperm(S, generator=gen)[:b].to(torch.int32)
    slots[torch.rand(b, generator=gen) < 0.1] = -1
    pools = [TieredSlotPool(1, S, H, P, N, G, 32, 4, "fp8", torch.bfloat16, "cuda", max_batch=b) for _ in range(2)]
    live = slots >= 0
    gs = torch.Generator(device="cuda").manual_seed(seed)
    for s0 in range(0, S, 64):                           # the same N(0, 0.1) prefill state in both pools
        sl = torch.arange(s0, min(S, s0 + 64), dtype=torch.int32, device="cuda")
        st = torch.randn(sl.numel(), H, P, N, device="cuda", generator=gs) * math.sqrt(0.1)
        for p_ in pools:
            prefill_split(p_, 0, st, sl)
    w = (1.0 + 0.1 * torch.randn(H * P, generator=gen)).to(torch.bfloat16).cuda()
    for s in range(5):                                   # across a flush (c = 4)
        B = O.rot_flat(Bs[s].reshape(b, G * N), prm["R"]).reshape(b, G, N)
        C_ = O.rot_flat(Cs[s].reshape(b, G * N), prm["R"]).reshape(b, G, N)
        gbuf = torch.randn(b, H * P + gate_offset, generator=gen).to(torch.bfloat16).cuda()
        gate = gbuf[:, gate_offset:]                     # offset 0: 16-byte rows (fused); else the fallback
        args = (xs[s].cuda(), dts[s].cuda(), prm["A"].cuda(), B.cuda(), C_.cuda(), prm["D"].cuda(),
                prm["dt_bias"].cuda(), True, slots.cuda(), -1)
        y_f = torch.zeros(b, H, P, dtype=torch.bfloat16, device="cuda")
        tiered_state_update(pools[0], 0, *args, y_f, None, 1e-3, "stale", norm=(gate, w, 1e-5))
        y = torch.zeros(b, H, P, dtype=torch.bfloat16, device="cuda")
        tiered_state_update(pools[1], 0, *args, y, None, 1e-3)
        want = gated_rmsnorm(y.reshape(b, H * P), gate, w, 1e-5, (H // G) * P).reshape(b, H, P)
        torch.cuda.synchronize()
        got, want = y_f.float().cpu(), want.float().cpu()
        # a one-ulp flip of round(h * rstd) (the sums of squares run in another order) is then
        # multiplied by the weight and rounded again: at most two bf16 ulps of the output
        err = (got - want)[live].abs()
        bound = want[live].abs() * 2.0 ** -6 + 1e-6
        assert bool((err <= bound).all()), f"step {s}: fused norm off by {float((err / bound).max()):.2f}x"
        assert float((err > 0).float().mean()) <= 2e-2
        assert bool((got[~live] == 0).all()), "padded rows must be left untouched"
        for name in ("hot", "cold", "scale", "glog", "t", "ring_x", "ring_dt", "ring_b"):
            assert torch.equal(getattr(pools[0], name), getattr(pools[1], name)), name
    for p_ in pools:
        p_.check_status()


@pytest.mark.parametrize("b,S", [(6, 9), (448, 460)])
def test_step_with_fused_norm_matches_step_then_norm(b, S):
    """The gated norm fused into STEP (whole (row, group) units per CTA, the group's sums of
    squares met through an mbarrier) against the step followed by the norm kernel, at a small
    batch and at the benchmarked one."""
    _fused_vs_separate(b, S, gate_offset=0, seed=b)


def test_step_with_norm_falls_back_when_gate_rows_are_unaligned():
    """A gate whose rows are not 16-byte aligned cannot ride in the bulk-copied stage: the step
    writes y and the norm kernel runs after it, with the same result."""
    _fused_vs_separate(6, 9, gate_offset=3, seed=5)
