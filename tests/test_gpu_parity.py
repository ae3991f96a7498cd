"""GPU parity of the CUDA path against the CPU oracle (seeded, BASELINE distributions).

Bar: y within rtol 2e-3 / atol 1e-3 (fp32 out), hot state within fp32
reassociation, fp8 cold codes within 1 ulp, slot indexing / t / flush timing
bit-exact, prefill quantisation bit-exact.
"""
import pytest
import torch

import oracle as O
from tests import _helpers as Hh

pytestmark = pytest.mark.gpu


def _split_both(case, gpool, opool, slots):
    from nested_ssm_b200 import prefill_split
    O.prefill_split(opool, slots, case["state0"])
    prefill_split(gpool, 0, case["state0"].cuda(), slots.to(torch.int32).cuda())
    torch.cuda.synchronize()


@pytest.mark.parametrize("cold", ["fp8", "bf16", "fp32"])
@pytest.mark.parametrize("pb", [16, 32, 64])
def test_prefill_split_bitexact(cold, pb):
    case = Hh.make_case(b=5, S=9, pb=pb, cold=cold, steps=1)
    opool, gpool = Hh.oracle_pool(case), Hh.gpu_pool(case)
    slots = torch.tensor([3, 0, 8, 5, 1])
    _split_both(case, gpool, opool, slots)
    sl = slots.long()
    assert torch.equal(gpool.hot[0].cpu()[sl], opool.hot[sl])
    assert torch.equal(gpool.cold[0].cpu()[sl].view(torch.uint8), opool.cold[sl].view(torch.uint8))
    if cold == "fp8":
        assert torch.equal(gpool.scale[0].cpu()[sl], opool.scale[sl])
    assert int(gpool.t[0].cpu()[sl].abs().sum()) == 0


@pytest.mark.parametrize("cold", ["fp8", "bf16", "fp32"])
@pytest.mark.parametrize("pb", [16, 32, 64])
@pytest.mark.parametrize("c", [1, 4])
def test_per_step_parity_from_identical_state(cold, pb, c):
    """Before every step the oracle is re-synced to the GPU's pool, so each step's
    arithmetic is compared on identical state: y within the bar, hot to fp32
    reassociation, stored cold codes within 1 ulp (rarely different at all),
    t / glog / flush timing exact."""
    steps = 2 * c + 3
    case = Hh.make_case(b=6, S=10, pb=pb, c=c, cold=cold, steps=steps, seed=pb + c)
    opool, gpool = Hh.oracle_pool(case), Hh.gpu_pool(case)
    slots = torch.tensor([7, 2, 9, 0, 4, 5])
    _split_both(case, gpool, opool, slots)
    for s in range(steps):
        Hh.sync_oracle_from_gpu(gpool, opool)
        yg, yo = Hh.step_both(case, gpool, opool, s, slots)
        Hh.assert_y_close(yg, yo, f"step {s}")
        if cold == "bf16":
            # bf16 has no row scale: a value a flush cancels towards zero has tiny
            # ulps, so the bar is one ulp of the value or 0.2% of the row amax
            Hh.compare_pool(gpool, opool, 0, slots, "fp32_skip")
            Hh.cold_values_close(gpool, opool, 0, slots, "bf16", max_code_frac=1e-4)
        else:
            Hh.compare_pool(gpool, opool, 0, slots, cold, max_ulp=1, max_ulp_frac=1e-4)


@pytest.mark.parametrize("cold", ["fp8", "bf16", "fp32"])
@pytest.mark.parametrize("pb", [16, 32, 64])
@pytest.mark.parametrize("c", [1, 4])
def test_free_running_matches_oracle(cold, pb, c):
    """Free-running for several flushes.  fp32 cold: the strict bar throughout.
    fp8 / bf16 cold: a code that flips once (exp / log1p differ by an ulp between
    the GPU and the CPU) is carried through later flushes (never amplified: the cold
    recurrence is contractive), so the state bound is one storage ulp per step,
    accumulated, and y may move by a flipped code's C[n] * ulp.  The one-ulp bar is
    the per-step test."""
    steps = 2 * c + 3
    case = Hh.make_case(b=6, S=10, pb=pb, c=c, cold=cold, steps=steps, seed=pb + c)
    opool, gpool = Hh.oracle_pool(case), Hh.gpu_pool(case)
    slots = torch.tensor([7, 2, 9, 0, 4, 5])
    _split_both(case, gpool, opool, slots)
    budget = None
    for s in range(steps):
        yg, yo = Hh.step_both(case, gpool, opool, s, slots)
        if cold == "fp32":
            Hh.assert_y_close(yg, yo, f"step {s}")
            Hh.compare_pool(gpool, opool, 0, slots, "fp32")
        else:
            Hh.assert_y_close_quantized(yg, yo, f"step {s}")
            torch.testing.assert_close(gpool.hot[0].cpu()[slots], opool.hot[slots], rtol=1e-5, atol=1e-6)
            budget = Hh.cold_error_budget(gpool, opool, budget, 0, slots, cold)


def test_large_batch_pipeline_wraps():
    """Enough rows that every persistent CTA streams many items through its
    multi-stage copy ring (and crosses batch-row boundaries mid-range), with padded
    rows and a permuted slot map; per-step parity on identical state."""
    gen = torch.Generator().manual_seed(21)
    b, S = 72, 90
    case = Hh.make_case(b=b, S=S, pb=32, c=4, cold="fp8", steps=9, seed=21)
    opool, gpool = Hh.oracle_pool(case), Hh.gpu_pool(case)
    slots = torch.randperm(S, generator=gen)[:b]
    _split_both(case, gpool, opool, slots)
    for s in range(9):
        sl = slots.clone()
        sl[torch.randperm(b, generator=gen)[:5]] = -1
        Hh.sync_oracle_from_gpu(gpool, opool)
        yg, yo = Hh.step_both(case, gpool, opool, s, sl)
        Hh.assert_y_close(yg, yo, f"step {s}")
        Hh.compare_pool(gpool, opool, 0, slots, "fp8", max_ulp=1, max_ulp_frac=1e-4)


def test_config0_fp32_64_steps_with_rotation():
    """B=8, H=128, P=80, N=128, G=8, pb=32, c=4, hot and cold fp32,
    64 steps, seed 0, rotation on the GPU."""
    case = Hh.make_case(b=8, S=8, pb=32, c=4, cold="fp32", steps=64, seed=0)
    opool, gpool = Hh.oracle_pool(case), Hh.gpu_pool(case)
    slots = torch.arange(8)
    _split_both(case, gpool, opool, slots)
    for s in range(64):
        yg, yo = Hh.step_both(case, gpool, opool, s, slots, use_gpu_rotation=True)
        Hh.assert_y_close(yg, yo, f"step {s}")
    Hh.compare_pool(gpool, opool, 0, slots, "fp32", hot_rtol=1e-4, hot_atol=1e-5)


@pytest.mark.parametrize("c,P", [(2, 80), (8, 80), (16, 80), (64, 80), (4, 64), (8, 64), (16, 64), (64, 64), (4, 48)])
def test_chunk_and_headdim_instances(c, P):
    """The production configuration (fp8 cold, bf16 io) has kernels with c and
    headdim fixed at compile time (c in {4, 8, 16, 64}, headdim in {64, 80}); the others
    read them at run time.  Per-step parity from identical state across two flushes."""
    steps = 2 * c + 1
    case = Hh.make_case(b=6, S=9, P=P, pb=32, c=c, cold="fp8", steps=steps, seed=40 + c + P)
    opool, gpool = Hh.oracle_pool(case), Hh.gpu_pool(case)
    slots = torch.tensor([4, 8, 0, 2, 7, 1])
    _split_both(case, gpool, opool, slots)
    for s in range(steps):
        Hh.sync_oracle_from_gpu(gpool, opool)
        yg, yo = Hh.step_both(case, gpool, opool, s, slots, use_gpu_rotation=(s % 2 == 0))
        Hh.assert_y_close(yg, yo, f"step {s}")
        Hh.compare_pool(gpool, opool, 0, slots, "fp8", max_ulp=1, max_ulp_frac=1e-4)


def test_ragged_pad_and_phase_offsets():
    """Padded rows (slot -1) are skipped and leave out untouched; slots enter at
    different times so each flushes on its own t % c."""
    from nested_ssm_b200 import prefill_split
    case = Hh.make_case(b=6, S=12, pb=32, c=4, cold="fp8", steps=14, seed=11)
    opool, gpool = Hh.oracle_pool(case), Hh.gpu_pool(case)
    all_slots = torch.tensor([11, 3, 6, 0, 8, 2])
    O.prefill_split(opool, all_slots, case["state0"])
    prefill_split(gpool, 0, case["state0"].cuda(), all_slots.to(torch.int32).cuda())
    for s in range(14):
        slots = all_slots.clone()
        # row 1 joins late (reset at step 3), rows 4,5 padded on some steps
        if s < 3:
            slots[1] = -1
        if s == 3:
            O.prefill_split(opool, all_slots[1:2], case["state0"][1:2])
            prefill_split(gpool, 0, case["state0"][1:2].cuda(), all_slots[1:2].to(torch.int32).cuda())
        if s % 3 == 1:
            slots[4] = -1
        if s % 5 == 2:
            slots[5] = -1
        yg, yo = Hh.step_both(case, gpool, opool, s, slots)
        pad = slots < 0
        assert torch.all(yg[pad] == 0), "padded rows must be left untouched"
        Hh.assert_y_close_quantized(yg, yo, f"step {s}")
        Hh.cold_values_close(gpool, opool, 0, all_slots, "fp8", ulps=3)
        assert torch.equal(gpool.t[0].cpu()[all_slots], opool.t[all_slots][:, None].expand(-1, 128))
    assert int(gpool.status.item()) == 0


def test_flush_rows_spread_over_grid():
    """Rows join on different tokens, so on every token a different quarter of the batch
    (interleaved rows) is at a chunk boundary.  FLUSH numbers those rows and splits only
    their items over the whole grid: 16 flushing rows x 128 heads land on hundreds of CTAs
    whose item ranges start and end inside rows."""
    from nested_ssm_b200 import prefill_split
    b, S, c, steps = 64, 80, 4, 10
    case = Hh.make_case(b=b, S=S, pb=32, c=c, cold="fp8", steps=steps, seed=21)
    opool, gpool = Hh.oracle_pool(case), Hh.gpu_pool(case)
    all_slots = torch.randperm(S, generator=torch.Generator().manual_seed(21))[:b]
    join = torch.arange(b) % c   # row r joins on step r % c
    for s in range(steps):
        idx = (join == s).nonzero().flatten()
        if idx.numel():
            O.prefill_split(opool, all_slots[idx], case["state0"][idx])
            prefill_split(gpool, 0, case["state0"][idx].cuda(), all_slots[idx].to(torch.int32).cuda())
        live = join <= s
        slots = torch.where(live, all_slots, torch.full_like(all_slots, -1))
        Hh.sync_oracle_from_gpu(gpool, opool)   # every token from identical state: the per-step bar
        yg, yo = Hh.step_both(case, gpool, opool, s, slots)
        Hh.assert_y_close(yg, yo, f"step {s}")
        Hh.compare_pool(gpool, opool, 0, all_slots, "fp8", max_ulp=1, max_ulp_frac=1e-4)
        if s >= c - 1:   # exactly one quarter of the rows flushed on this token
            assert int((opool.t[all_slots[live]] % c == 0).sum()) == b // c
    assert int(gpool.status.item()) == 0


@pytest.mark.parametrize("mode", ["corr", "coldoff"])
def test_modes(mode):
    case = Hh.make_case(b=4, S=4, pb=32, c=4, cold="fp32", steps=9, seed=5)
    opool, gpool = Hh.oracle_pool(case), Hh.gpu_pool(case)
    slots = torch.arange(4)
    _split_both(case, gpool, opool, slots)
    for s in range(9):
        yg, yo = Hh.step_both(case, gpool, opool, s, slots, mode=mode)
        Hh.assert_y_close(yg, yo, f"{mode} step {s}")
    Hh.compare_pool(gpool, opool, 0, slots, "fp32", hot_rtol=1e-4, hot_atol=1e-5)


def test_corr_fp32_equals_fresh():
    """Exact rank-c correction with fp32 cold reproduces the untiered update
    (the gate of scale/probe_corr_exact.py)."""
    from nested_ssm_b200 import selective_state_update
    case = Hh.make_case(b=4, S=4, pb=32, c=4, cold="fp32", steps=10, seed=8)
    opool, gpool = Hh.oracle_pool(case), Hh.gpu_pool(case)
    slots = torch.arange(4)
    _split_both(case, gpool, opool, slots)
    state = case["state0"].clone().cuda()
    prm = case["prm"]
    for s in range(10):
        yg, _ = Hh.step_both(case, gpool, opool, s, slots, mode="corr")
        B, C_ = Hh.rotated(case, s)
        yf = selective_state_update(state, case["xs"][s].cuda(), case["dts"][s].cuda(), prm["A"].cuda(),
                                    B.cuda(), C_.cuda(), prm["D"].cuda(), None, prm["dt_bias"].cuda(), True,
                                    slots.to(torch.int32).cuda(), -1,
                                    torch.zeros(4, case["H"], case["P"], device="cuda"))
        torch.testing.assert_close(yg, yf.cpu(), rtol=2e-3, atol=1e-3)


def test_fresh_step_matches_oracle():
    from nested_ssm_b200 import selective_state_update
    case = Hh.make_case(b=5, S=7, steps=6, seed=4)
    prm = case["prm"]
    slots = torch.tensor([6, 1, -1, 3, 0])
    st_o = torch.randn(7, 128, 80, 128) * 0.3
    st_g = st_o.clone().cuda()
    for s in range(6):
        B, C_ = Hh.rotated(case, s)
        yo = O.fresh_step(st_o, slots, case["xs"][s], case["dts"][s], B, C_, prm["A"], prm["D"], prm["dt_bias"])
        out = torch.zeros(5, 128, 80, device="cuda")
        selective_state_update(st_g, case["xs"][s].cuda(), case["dts"][s].cuda(), prm["A"].cuda(), B.cuda(),
                               C_.cuda(), prm["D"].cuda(), None, prm["dt_bias"].cuda(), True,
                               slots.to(torch.int32).cuda(), -1, out)
        torch.cuda.synchronize()
        Hh.assert_y_close(out.cpu(), yo, f"fresh step {s}")
    torch.testing.assert_close(st_g.cpu(), st_o, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rot_flat(dtype):
    from nested_ssm_b200 import rot_flat
    prm = O.make_params(128, 8, 128, seed=2)[0]
    x = (torch.randn(37, 8 * 128) / 11.3).to(dtype)
    yo = O.rot_flat(x, prm["R"], "fp32")
    yg = rot_flat(x.cuda(), prm["R"].cuda()).cpu()
    Hh.rotation_close(yg, yo, x, prm["R"])


def test_materialize_matches_oracle_and_native():
    """Materialised full state == oracle materialise; with fp32 cold == the native
    full fresh state (scale/v4_native_decode.py:65-67) to fp32 reassociation."""
    from nested_ssm_b200 import materialize
    case = Hh.make_case(b=3, S=3, pb=32, c=4, cold="fp32", steps=7, seed=9)
    opool, gpool = Hh.oracle_pool(case), Hh.gpu_pool(case)
    npool = O.NativePoolRef(3, 128, 80, 128, 32, 4, torch.float32)
    slots = torch.arange(3)
    _split_both(case, gpool, opool, slots)
    O.prefill_split(npool, slots, case["state0"])
    prm = case["prm"]
    for s in range(7):
        Hh.step_both(case, gpool, opool, s, slots)
        B, C_ = Hh.rotated(case, s)
        O.native_step(npool, slots, case["xs"][s], case["dts"][s], B, C_, prm["A"], prm["D"], prm["dt_bias"])
        mg = materialize(gpool, 0, slots, prm["A"]).cpu()
        mo = O.materialize(opool, slots, prm["A"])
        torch.testing.assert_close(mg, mo, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(mg, npool.state, rtol=1e-4, atol=1e-5)


def test_bad_slot_sets_status_and_skips():
    from nested_ssm_b200 import tiered_state_update
    case = Hh.make_case(b=2, S=4, steps=1, seed=1)
    gpool = Hh.gpu_pool(case)
    prm = case["prm"]
    B, C_ = Hh.rotated(case, 0)
    out = torch.full((2, 128, 80), 7.0, device="cuda")
    tiered_state_update(gpool, 0, case["xs"][0].cuda(), case["dts"][0].cuda(), prm["A"].cuda(), B.cuda(),
                        C_.cuda(), prm["D"].cuda(), prm["dt_bias"].cuda(), True,
                        torch.tensor([1, 9], dtype=torch.int32, device="cuda"), -1, out)
    torch.cuda.synchronize()
    assert int(gpool.status.item()) == 1
    assert bool((out[1] == 7.0).all())
    with pytest.raises(IndexError):
        gpool.check_status()
