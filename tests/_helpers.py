"""Shared helpers for the parity tests: matched oracle / GPU pools and comparisons."""
from __future__ import annotations

import torch

import oracle as O

Y_RTOL, Y_ATOL = 2e-3, 1e-3          # y tolerance (fp32 hot state)
COLD = {"fp8": O.FP8, "bf16": torch.bfloat16, "fp32": torch.float32}


def make_case(b, S, H=128, P=80, N=128, G=8, pb=32, c=4, cold="fp8", steps=8, seed=0,
              io_dtype=torch.bfloat16, state_std=0.1 ** 0.5, rotate=True):
    """Seeded synthetic case with the BASELINE distributions."""
    prm = O.make_params(H, G, N, seed=seed)[0]
    xs, dts, Bs, Cs = O.make_inputs(b, H, P, G, N, steps, seed=seed, io_dtype=io_dtype)
    g = torch.Generator().manual_seed(seed + 7)
    state0 = torch.randn(b, H, P, N, generator=g) * state_std
    return dict(prm=prm, xs=xs, dts=dts, Bs=Bs, Cs=Cs, state0=state0, b=b, S=S, H=H, P=P, N=N, G=G,
                pb=pb, c=c, cold=cold, io_dtype=io_dtype, rotate=rotate)


def oracle_pool(case):
    return O.TieredPoolRef(case["S"], case["H"], case["P"], case["N"], case["G"], case["pb"], case["c"],
                           COLD[case["cold"]], case["io_dtype"])


def gpu_pool(case, layers=1, max_batch=None):
    from nested_ssm_b200 import TieredSlotPool
    return TieredSlotPool(layers, case["S"], case["H"], case["P"], case["N"], case["G"], case["pb"],
                          case["c"], case["cold"], case["io_dtype"], "cuda",
                          max_batch=max_batch or max(case["b"], 1))


def rotated(case, step):
    """B, C of a step after the oracle's fp32 rotation (what both sides consume when
    the test isolates the state op from the rotation kernel)."""
    B, C_ = case["Bs"][step], case["Cs"][step]
    if not case["rotate"]:
        return B, C_
    b, G, N = B.shape
    R = case["prm"]["R"]
    Br = O.rot_flat(B.reshape(b, G * N), R, "fp32").reshape(b, G, N)
    Cr = O.rot_flat(C_.reshape(b, G * N), R, "fp32").reshape(b, G, N)
    return Br, Cr


def rotation_close(got, want, x, R, input_ulps=0):
    """A rotated tensor against the oracle's: each value within one ulp of its dtype
    plus the fp32 dot-product rounding bound n * 2^-24 * sum_n |R[m,n]| |x[n]| (two fp32
    sums in different orders can land on either side of a rounding boundary; near zero
    that is more than an ulp of the result).  ``input_ulps``: the rotated inputs themselves
    may differ by that many io ulps (values the GPU computed, e.g. conv outputs), which adds
    input_ulps * ulp * sum_n |R[m,n]| |x[n]|."""
    b = x.shape[0]
    G, N, _ = R.shape
    mag = torch.einsum("tgn,gmn->tgm", x.reshape(b, G, N).float().abs(), R.float().abs()).reshape(got.shape)
    ulp = 2.0 ** -8 if got.dtype == torch.bfloat16 else 2.0 ** -23
    bound = want.float().abs() * ulp + (N * 2.0 ** -24 + input_ulps * ulp) * mag + 1e-30
    err = (got.float() - want.float()).abs()
    assert bool((err <= bound).all()), f"rotation off by {float((err / bound).max()):.2f}x the bound"
    assert float((err > 0).float().mean()) <= 2e-2, "rotation differs too often"


def gpu_rotated(case, step):
    """B, C of a step rotated by the library's rotation kernel (on the GPU), on the CPU."""
    from nested_ssm_b200 import rot_flat
    B, C_ = case["Bs"][step], case["Cs"][step]
    b, G, N = B.shape
    R = case["prm"]["R"].cuda()
    Br = rot_flat(B.reshape(b, G * N).cuda(), R).reshape(b, G, N).cpu()
    Cr = rot_flat(C_.reshape(b, G * N).cuda(), R).reshape(b, G, N).cpu()
    return Br, Cr


def fp8_ulp_dist(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return (O.fp8_ordered_codes(a.cpu()) - O.fp8_ordered_codes(b.cpu())).abs()


def assert_y_close(y_gpu, y_ref, what=""):
    torch.testing.assert_close(y_gpu.float().cpu(), y_ref.float(), rtol=Y_RTOL, atol=Y_ATOL, msg=lambda m: f"{what}: {m}")


def bf16_ulp_dist(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    def codes(t):
        u = t.cpu().contiguous().view(torch.int16).to(torch.int32)
        mag = u & 0x7FFF
        return torch.where(u < 0, -mag, mag)
    return (codes(a) - codes(b)).abs()


def compare_pool(gpool, opool, layer=0, slots=None, cold_kind="fp8", hot_rtol=1e-5, hot_atol=1e-6,
                 max_ulp=1, max_ulp_frac=1.0):
    """Compare a GPU pool layer with the oracle pool (on the given slots); returns the
    fraction of stored cold codes that differ (fp8 / bf16)."""
    sl = slots if slots is not None else torch.arange(opool.num_slots)
    sl = sl[sl >= 0].long()
    torch.testing.assert_close(gpool.hot[layer].cpu()[sl], opool.hot[sl], rtol=hot_rtol, atol=hot_atol)
    assert torch.equal(gpool.t[layer].cpu()[sl], opool.t[sl][:, None].expand(-1, opool.H).to(torch.int32))
    torch.testing.assert_close(gpool.glog[layer].cpu()[sl], opool.glog[sl], rtol=1e-6, atol=1e-6)
    if cold_kind == "fp32_skip":       # hot / t / glog only; cold checked by the caller
        return 0.0
    gc = gpool.cold[layer].cpu()[sl]
    oc = opool.cold[sl]
    if cold_kind in ("fp8", "bf16"):
        d = fp8_ulp_dist(gc, oc) if cold_kind == "fp8" else bf16_ulp_dist(gc, oc)
        frac = float((d > 0).float().mean())
        hist = {int(k): int((d == k).sum()) for k in torch.unique(d)}
        assert int(d.max()) <= max_ulp, f"{cold_kind} cold differs by up to {int(d.max())} ulp; histogram {hist}"
        assert frac <= max_ulp_frac, f"{cold_kind} cold: {frac:.2e} of codes differ; histogram {hist}"
        if cold_kind == "fp8":
            torch.testing.assert_close(gpool.scale[layer].cpu()[sl], opool.scale[sl], rtol=1e-5, atol=0)
        return frac
    torch.testing.assert_close(gc.float(), oc.float(), rtol=1e-5, atol=1e-6)
    return 0.0


def cold_values_close(gpool, opool, layer=0, slots=None, cold_kind="fp8", max_code_frac=1e-3, ulps=1):
    """Bound in value terms: every stored cold value within `ulps` storage ulps of the
    oracle's (relative), or within ulps * 0.2% of its row amax (values that a flush
    cancelled down to near zero); differing codes rare."""
    sl = slots if slots is not None else torch.arange(opool.num_slots)
    sl = sl[sl >= 0].long()
    gq, oq = gpool.cold[layer].cpu()[sl], opool.cold[sl]
    if cold_kind == "fp8":
        gv = O.dequantize_rows(gq, gpool.scale[layer].cpu()[sl])
        ov = O.dequantize_rows(oq, opool.scale[sl])
        d = fp8_ulp_dist(gq, oq)
        rel = 0.13
    else:
        gv, ov = gq.float(), oq.float()
        d = bf16_ulp_dist(gq, oq) if cold_kind == "bf16" else (gv != ov).to(torch.int32)
        rel = 2.0 ** -7 if cold_kind == "bf16" else 1e-5
    amax = ov.abs().amax(dim=-1, keepdim=True)
    bound = ulps * (rel * ov.abs() + 2e-3 * amax) + 1e-7
    err = (gv - ov).abs()
    worst = float((err / bound).max())
    assert worst <= 1.0, f"{cold_kind} cold value off by {worst:.2f}x the {ulps}-ulp bound"
    frac = float((d > 0).float().mean())
    assert frac <= max_code_frac, f"{cold_kind}: {frac:.2e} of codes differ"
    return frac


def cold_error_budget(gpool, opool, budget=None, layer=0, slots=None, cold_kind="fp8", max_code_frac=1e-3):
    """Free-running bound on the stored cold state, for a run whose GPU and oracle
    states are never re-synchronised.  The cold recurrence is contractive
    (v <- v * exp(sum dt*A) + update, exp(...) <= 1, the update computed from the same
    inputs on both sides), so an error made by one requantisation is carried but
    never amplified; what can build up is at most one storage ulp per requantisation.
    ``budget`` accumulates that ulp (relative ulp of the value now, or 0.2% of the row
    amax near zero) step by step; every value must stay within it.  Returns the new
    budget for the next call."""
    sl = slots if slots is not None else torch.arange(opool.num_slots)
    sl = sl[sl >= 0].long()
    gq, oq = gpool.cold[layer].cpu()[sl], opool.cold[sl]
    if cold_kind == "fp8":
        gv = O.dequantize_rows(gq, gpool.scale[layer].cpu()[sl])
        ov = O.dequantize_rows(oq, opool.scale[sl])
        d = fp8_ulp_dist(gq, oq)
        rel = 0.13
    else:
        gv, ov = gq.float(), oq.float()
        d = bf16_ulp_dist(gq, oq)
        rel = 2.0 ** -7
    amax = ov.abs().amax(dim=-1, keepdim=True)
    per = rel * ov.abs() + 2e-3 * amax + 1e-7
    budget = per if budget is None else budget + per
    err = (gv - ov).abs()
    worst = float((err / budget).max())
    assert worst <= 1.0, f"{cold_kind} cold value off by {worst:.2f}x the accumulated one-ulp-per-step budget"
    frac = float((d > 0).float().mean())
    assert frac <= max_code_frac, f"{cold_kind}: {frac:.2e} of codes differ"
    return budget


def assert_y_close_quantized(y_gpu, y_ref, what=""):
    """y of a free-running run with quantised cold: a one-ulp cold code flip moves
    y by C[n]*ulp, so allow rare (<0.1%) excursions up to 1e-2 beyond the y bar."""
    yg, yr = y_gpu.float().cpu(), y_ref.float()
    err = (yg - yr).abs()
    tol = Y_ATOL + Y_RTOL * yr.abs()
    bad = err > tol
    assert float(bad.float().mean()) <= 1e-3, f"{what}: {int(bad.sum())} elements outside the y bar"
    assert float((err - tol).max()) <= 1e-2, f"{what}: excursion {float((err - tol).max()):.3e}"


def sync_oracle_from_gpu(gpool, opool, layer=0):
    """Copy the GPU pool's state into the oracle pool (per-step parity checks)."""
    opool.hot.copy_(gpool.hot[layer].cpu())
    opool.cold.copy_(gpool.cold[layer].cpu())
    if opool.scale is not None:
        opool.scale.copy_(gpool.scale[layer].cpu())
    opool.glog.copy_(gpool.glog[layer].cpu())
    opool.t.copy_(gpool.t[layer].cpu()[:, 0])
    opool.ring_x.copy_(gpool.ring_x[layer].cpu())
    opool.ring_dt.copy_(gpool.ring_dt[layer].cpu()[..., :opool.c])
    opool.ring_b.copy_(gpool.ring_b[layer].cpu())


def step_both(case, gpool, opool, step, slots_cpu, layer=0, mode="stale", use_gpu_rotation=False):
    """Run one token on both sides; returns (y_gpu fp32 cpu, y_oracle fp32)."""
    from nested_ssm_b200 import tiered_state_update
    prm = case["prm"]
    x, dt = case["xs"][step], case["dts"][step]
    if use_gpu_rotation:
        # the GPU rotates B, C itself; the oracle state op gets the GPU's rotated values
        # (fp32 sums in another order may round to a neighbouring io value, checked here
        # separately) so the state-op comparison runs on identical inputs
        Bg, Cg = case["Bs"][step], case["Cs"][step]
        R = prm["R"].cuda()
        Bo, Co = gpu_rotated(case, step)
        Br, Cr = rotated(case, step)
        rotation_close(Bo, Br, case["Bs"][step], prm["R"])
        rotation_close(Co, Cr, case["Cs"][step], prm["R"])
    else:
        Bo, Co = rotated(case, step)
        Bg, Cg = Bo, Co
        R = None
    yo = O.tiered_step(opool, slots_cpu, x, dt, Bo, Co, prm["A"], prm["D"], prm["dt_bias"], 1e-3,
                       mode=mode)
    out = torch.zeros(x.shape[0], case["H"], case["P"], device="cuda")
    tiered_state_update(gpool, layer, x.cuda(), dt.cuda(), prm["A"].cuda(), Bg.cuda(), Cg.cuda(),
                        prm["D"].cuda(), prm["dt_bias"].cuda(), True, slots_cpu.to(torch.int32).cuda(),
                        -1, out, R, 1e-3, mode)
    torch.cuda.synchronize()
    return out.cpu(), yo
