"""The self-speculative pieces of the CPU oracle: the hot-only draft pinned to the reference's
own decode (its mode "coldoff" readout, recorded in the golden fixture, is the draft's y: the
same hot update, no cold term), and verify / commit as compositions of decode steps."""
import pytest
import torch

import oracle as O
from tests import _golden as GD
from tests import _helpers as Hh


def test_draft_step_bitexact_vs_reference_coldoff():
    d = GD.load("native_decode_fp32.npz")
    inp = GD.native_inputs("coldoff")
    GD.check_sums(d, inp, "coldoff_")
    cfg = inp["cfg"]
    b, pb = cfg["b"], cfg["pb"]
    draft = inp["s0"][..., :pb].float().clone()
    slots = torch.arange(b)
    for s in range(inp["steps"]):
        Br, Cr = GD.bf16(d["coldoff_Br"][s]), GD.bf16(d["coldoff_Cr"][s])
        y = O.draft_step(draft, slots, inp["xs"][s], inp["dts"][s], Br, Cr, d["A"], d["D"], d["dt_bias"], 1e-3)
        assert torch.equal(y, d["coldoff_y"][s]), f"step {s}"


def _stacked(case, s0, n):
    xs = case["xs"][s0:s0 + n].transpose(0, 1).contiguous()
    dts = case["dts"][s0:s0 + n].transpose(0, 1).contiguous()
    rot = [Hh.rotated(case, s) for s in range(s0, s0 + n)]
    return xs, dts, torch.stack([r[0] for r in rot], 1), torch.stack([r[1] for r in rot], 1)


def test_verify_then_commit_equals_steps():
    case = Hh.make_case(b=4, S=6, H=16, G=2, pb=32, c=4, cold="fp8", steps=9, seed=3)
    prm = case["prm"]
    slots = torch.tensor([5, 1, 3, 0])
    pools = [Hh.oracle_pool(case) for _ in range(2)]
    for p_ in pools:
        O.prefill_split(p_, slots, case["state0"])
    for s in range(2):   # phase 2 of 4
        for p_ in pools:
            Br, Cr = Hh.rotated(case, s)
            O.tiered_step(p_, slots, case["xs"][s], case["dts"][s], Br, Cr, prm["A"], prm["D"], prm["dt_bias"])
    xs, dts, Bs, Cs = _stacked(case, 2, 2)
    y = O.verify_steps(pools[0], slots, xs, dts, Bs, Cs, prm["A"], prm["D"], prm["dt_bias"])
    assert torch.equal(pools[0].t, pools[1].t) and torch.equal(pools[0].hot, pools[1].hot)   # read-only
    accept = torch.tensor([2, 0, 1, 2])
    O.commit_steps(pools[0], slots, accept, xs, dts, Bs, prm["A"], prm["dt_bias"])
    for j in range(2):
        sl = slots.clone()
        sl[accept <= j] = -1
        yj = O.tiered_step(pools[1], sl, xs[:, j], dts[:, j], Bs[:, j], Cs[:, j], prm["A"], prm["D"], prm["dt_bias"])
        keep = accept > j   # the same arithmetic on other batch shapes: einsum may sum in another order
        torch.testing.assert_close(yj[keep], y[keep, j], rtol=1e-5, atol=1e-6)
    for name in ("hot", "cold", "scale", "glog", "t", "ring_x", "ring_dt", "ring_b"):
        assert torch.equal(getattr(pools[0], name), getattr(pools[1], name)), name
    assert pools[0].t.tolist() == [4, 2, 0, 3, 0, 4]   # slots 5 and 0 completed their chunk (flushed)
    assert float(pools[0].glog[0].abs().sum()) == 0.0 and float(pools[0].glog[3].abs().sum()) > 0.0


def test_windows_across_a_chunk_boundary_are_refused():
    case = Hh.make_case(b=2, S=2, H=16, G=2, pb=32, c=4, cold="fp8", steps=4, seed=4)
    prm = case["prm"]
    pool = Hh.oracle_pool(case)
    slots = torch.arange(2)
    O.prefill_split(pool, slots, case["state0"])
    Br, Cr = Hh.rotated(case, 0)
    O.tiered_step(pool, slots, case["xs"][0], case["dts"][0], Br, Cr, prm["A"], prm["D"], prm["dt_bias"])
    xs, dts, Bs, Cs = _stacked(case, 0, 4)
    with pytest.raises(ValueError):
        O.verify_steps(pool, slots, xs, dts, Bs, Cs, prm["A"], prm["D"], prm["dt_bias"])
    with pytest.raises(ValueError):
        O.commit_steps(pool, slots, torch.tensor([4, 3]), xs, dts, Bs, prm["A"], prm["dt_bias"])


def test_draft_equals_coldoff_readout_on_random_cases():
    """The hot-only draft's y and hot evolution are the tiered step's in mode coldoff (the
    readout ignores the cold slice; the hot update never reads it), for every hot width."""
    for pb in (16, 32, 64):
        case = Hh.make_case(b=3, S=5, H=16, G=2, pb=pb, c=4, cold="fp8", steps=6, seed=pb)
        prm = case["prm"]
        slots = torch.tensor([4, 0, 2])
        pool = Hh.oracle_pool(case)
        O.prefill_split(pool, slots, case["state0"])
        draft = pool.hot.clone()
        for s in range(6):
            Br, Cr = Hh.rotated(case, s)
            yd = O.draft_step(draft, slots, case["xs"][s], case["dts"][s], Br, Cr, prm["A"], prm["D"], prm["dt_bias"])
            yc = O.tiered_step(pool, slots, case["xs"][s], case["dts"][s], Br, Cr, prm["A"], prm["D"], prm["dt_bias"],
                               mode="coldoff")
            torch.testing.assert_close(yd, yc, rtol=1e-6, atol=1e-7)
            assert torch.equal(draft[slots], pool.hot[slots])


def test_verify_commit_cover_a_long_chunk():
    """c = 16 from phase 5: verify of the remaining 11 tokens, then a commit that stops short
    of the boundary for some rows and completes the chunk (a flush) for others."""
    case = Hh.make_case(b=3, S=4, H=16, G=2, pb=32, c=16, cold="fp8", steps=16, seed=9)
    prm = case["prm"]
    slots = torch.tensor([3, 1, 0])
    pools = [Hh.oracle_pool(case) for _ in range(2)]
    for p_ in pools:
        O.prefill_split(p_, slots, case["state0"])
        for s in range(5):
            Br, Cr = Hh.rotated(case, s)
            O.tiered_step(p_, slots, case["xs"][s], case["dts"][s], Br, Cr, prm["A"], prm["D"], prm["dt_bias"])
    xs, dts, Bs, Cs = _stacked(case, 5, 11)
    O.verify_steps(pools[0], slots, xs, dts, Bs, Cs, prm["A"], prm["D"], prm["dt_bias"])
    accept = torch.tensor([11, 4, 0])
    O.commit_steps(pools[0], slots, accept, xs, dts, Bs, prm["A"], prm["dt_bias"])
    for j in range(11):
        sl = slots.clone()
        sl[accept <= j] = -1
        O.tiered_step(pools[1], sl, xs[:, j], dts[:, j], Bs[:, j], Cs[:, j], prm["A"], prm["D"], prm["dt_bias"])
    for name in ("hot", "cold", "scale", "glog", "t", "ring_x", "ring_dt", "ring_b"):
        assert torch.equal(getattr(pools[0], name), getattr(pools[1], name)), name
    assert pools[0].t[[3, 1, 0]].tolist() == [16, 9, 5] and float(pools[0].glog[3].abs().sum()) == 0.0
