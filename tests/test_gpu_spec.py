"""Self-speculative decoding on the GPU: the hot-only draft against the oracle's draft (pinned
to the reference's coldoff readout), verify against n sequential oracle steps, and commit
against the decode step itself -- verify(n) + commit(k) must leave every pool buffer bit-identical
to k nssm_tiered_step calls with the same inputs (same kernels' arithmetic, FLUSH included)."""
import pytest
import torch

import oracle as O
from tests import _helpers as Hh

pytestmark = pytest.mark.gpu

POOL_BUFFERS = ("hot", "cold", "scale", "glog", "t", "ring_x", "ring_dt", "ring_b")


def _stacked(case, s0, n):
    xs = case["xs"][s0:s0 + n].transpose(0, 1).contiguous()
    dts = case["dts"][s0:s0 + n].transpose(0, 1).contiguous()
    rot = [Hh.rotated(case, s) for s in range(s0, s0 + n)]
    return xs, dts, torch.stack([r[0] for r in rot], 1).contiguous(), torch.stack([r[1] for r in rot], 1).contiguous()


def _split(case, pools, opool, slots):
    from nested_ssm_b200 import prefill_split
    if opool is not None:
        O.prefill_split(opool, slots, case["state0"])
    for p_ in pools:
        prefill_split(p_, 0, case["state0"].cuda(), slots.to(torch.int32).cuda())


def _gpu_step(case, gpool, s, slots, out=None):
    from nested_ssm_b200 import tiered_state_update
    prm = case["prm"]
    Br, Cr = Hh.rotated(case, s)
    y = out if out is not None else torch.zeros(slots.numel(), case["H"], case["P"], device="cuda")
    tiered_state_update(gpool, 0, case["xs"][s].cuda(), case["dts"][s].cuda(), prm["A"].cuda(), Br.cuda(), Cr.cuda(),
                        prm["D"].cuda(), prm["dt_bias"].cuda(), True, slots.to(torch.int32).cuda(), -1, y, None, 1e-3)
    return y


def _snapshot(gpool):
    return {k: getattr(gpool, k).clone() for k in POOL_BUFFERS if getattr(gpool, k) is not None}


@pytest.mark.parametrize("pb", [16, 32, 64])
def test_draft_matches_oracle_and_leaves_the_pool(pb):
    from nested_ssm_b200 import draft_state_update
    case = Hh.make_case(b=6, S=10, pb=pb, c=4, cold="fp8", steps=4, seed=40 + pb)
    prm = case["prm"]
    opool, gpool = Hh.oracle_pool(case), Hh.gpu_pool(case)
    slots = torch.tensor([7, 2, 9, 0, 4, 5])
    _split(case, [gpool], opool, slots)
    before = _snapshot(gpool)
    odraft = opool.hot.clone()
    gdraft = gpool.new_draft()[0]
    for s in range(4):
        Br, Cr = Hh.rotated(case, s)
        yo = O.draft_step(odraft, slots, case["xs"][s], case["dts"][s], Br, Cr, prm["A"], prm["D"], prm["dt_bias"])
        yg = torch.zeros(6, case["H"], case["P"], device="cuda")
        draft_state_update(gpool, 0, gdraft, case["xs"][s].cuda(), case["dts"][s].cuda(), prm["A"].cuda(), Br.cuda(),
                           Cr.cuda(), prm["D"].cuda(), prm["dt_bias"].cuda(), True, slots.to(torch.int32).cuda(), -1,
                           yg, None, 1e-3, from_pool=(s == 0))
        torch.cuda.synchronize()
        Hh.assert_y_close(yg.cpu(), yo, f"draft step {s}")
        torch.testing.assert_close(gdraft.cpu()[slots], odraft[slots], rtol=1e-5, atol=1e-6)
    for k, v in before.items():
        assert torch.equal(getattr(gpool, k), v), f"the draft wrote the pool's {k}"
    gpool.check_status()


def test_draft_with_rotation_on_the_gpu():
    """R given: B and C are rotated on the GPU first (the decode step's rotation kernel)."""
    from nested_ssm_b200 import draft_state_update
    case = Hh.make_case(b=5, S=5, pb=32, c=4, cold="fp8", steps=2, seed=47)
    prm = case["prm"]
    opool, gpool = Hh.oracle_pool(case), Hh.gpu_pool(case)
    slots = torch.arange(5)
    _split(case, [gpool], opool, slots)
    odraft = opool.hot.clone()
    gdraft = gpool.new_draft()[0]
    for s in range(2):
        Bo, Co = Hh.gpu_rotated(case, s)
        yo = O.draft_step(odraft, slots, case["xs"][s], case["dts"][s], Bo, Co, prm["A"], prm["D"], prm["dt_bias"])
        yg = torch.zeros(5, case["H"], case["P"], device="cuda")   # fp32 out: the bar is an fp32 one
        draft_state_update(gpool, 0, gdraft, case["xs"][s].cuda(), case["dts"][s].cuda(), prm["A"].cuda(),
                           case["Bs"][s].cuda(), case["Cs"][s].cuda(), prm["D"].cuda(), prm["dt_bias"].cuda(),
                           True, slots.to(torch.int32).cuda(), -1, yg, prm["R"].cuda(), 1e-3, from_pool=(s == 0))
        torch.cuda.synchronize()
        Hh.assert_y_close(yg.cpu(), yo, f"draft step {s}")


@pytest.mark.parametrize("cold", ["fp8", "bf16", "fp32"])
@pytest.mark.parametrize("c,phase", [(4, 0), (4, 1), (4, 3), (16, 5)])
@pytest.mark.parametrize("mode", ["stale", "coldoff"])
def test_verify_matches_sequential_oracle(cold, c, phase, mode):
    """Verify of the rest of the chunk (c - phase tokens) against that many oracle steps on
    a copy of the state; the GPU pool is left bit-identical."""
    from nested_ssm_b200 import verify_state_update
    n = c - phase
    case = Hh.make_case(b=6, S=10, pb=32, c=c, cold=cold, steps=phase + n, seed=c + phase)
    prm = case["prm"]
    opool, gpool = Hh.oracle_pool(case), Hh.gpu_pool(case)
    slots = torch.tensor([7, 2, 9, 0, 4, 5])
    _split(case, [gpool], opool, slots)
    for s in range(phase):
        Hh.step_both(case, gpool, opool, s, slots)
    Hh.sync_oracle_from_gpu(gpool, opool)
    before = _snapshot(gpool)
    xs, dts, Bs, Cs = _stacked(case, phase, n)
    yo = O.verify_steps(opool, slots, xs, dts, Bs, Cs, prm["A"], prm["D"], prm["dt_bias"], mode=mode)
    yg = verify_state_update(gpool, 0, xs.cuda(), dts.cuda(), prm["A"].cuda(), Bs.cuda(), Cs.cuda(), prm["D"].cuda(),
                             prm["dt_bias"].cuda(), True, slots.to(torch.int32).cuda(), -1,
                             torch.zeros(6, n, case["H"], case["P"], device="cuda"), None, 1e-3, mode)
    torch.cuda.synchronize()
    for j in range(n):
        Hh.assert_y_close(yg[:, j].cpu(), yo[:, j], f"token {j}")
    for k, v in before.items():
        assert torch.equal(getattr(gpool, k), v), f"verify wrote the pool's {k}"
    gpool.check_status()


def _commit_vs_steps(b, S, c, phase, cold, accept_of, seed, use_rotation=False):
    """Pool A: verify + commit(accept); pool B: the decode step on the rows that keep each
    token.  Every pool buffer must match bit for bit; verify's y must match B's y."""
    import math
    from nested_ssm_b200 import commit_state_update, prefill_split, verify_state_update
    n = c - phase
    H, P, N, G = 128, 80, 128, 8
    prm = O.make_params(H, G, N, seed=seed)[0]
    xs_, dts_, Bs_, Cs_ = O.make_inputs(b, H, P, G, N, phase + n, seed=seed)
    case = dict(prm=prm, xs=xs_, dts=dts_, Bs=Bs_, Cs=Cs_, b=b, S=S, H=H, P=P, N=N, G=G, pb=32, c=c, cold=cold,
                io_dtype=torch.bfloat16, rotate=True)
    gen = torch.Generator().manual_seed(seed)
    slots = torch.randperm(S, generator=gen)[:b]
    slots[torch.rand(b, generator=gen) < 0.05] = -1
    pa, pb_ = Hh.gpu_pool(case, max_batch=b), Hh.gpu_pool(case, max_batch=b)
    gs = torch.Generator(device="cuda").manual_seed(seed)
    for s0 in range(0, S, 64):   # the same N(0, 0.1) prefill state in both pools, made on the GPU
        sl = torch.arange(s0, min(S, s0 + 64), dtype=torch.int32, device="cuda")
        st = torch.randn(sl.numel(), H, P, N, device="cuda", generator=gs) * math.sqrt(0.1)
        for p_ in (pa, pb_):
            prefill_split(p_, 0, st, sl)
    for s in range(phase):
        _gpu_step(case, pa, s, slots)
        _gpu_step(case, pb_, s, slots)
    xs, dts, Bs, Cs = _stacked(case, phase, n)
    R = None
    if use_rotation:   # the raw B / C with R: both sides rotate on the GPU
        Bs = case["Bs"][phase:phase + n].transpose(0, 1).contiguous()
        Cs = case["Cs"][phase:phase + n].transpose(0, 1).contiguous()
        R = prm["R"].cuda()
    accept = accept_of(b, n, gen)
    sl32 = slots.to(torch.int32).cuda()
    yv = verify_state_update(pa, 0, xs.cuda(), dts.cuda(), prm["A"].cuda(), Bs.cuda(), Cs.cuda(), prm["D"].cuda(),
                             prm["dt_bias"].cuda(), True, sl32, -1,
                             torch.zeros(b, n, case["H"], case["P"], device="cuda"), R, 1e-3)
    commit_state_update(pa, 0, accept.to(torch.int32).cuda(), xs.cuda(), dts.cuda(), prm["A"].cuda(), Bs.cuda(),
                        prm["dt_bias"].cuda(), True, sl32, -1, R, 1e-3)
    from nested_ssm_b200 import tiered_state_update
    for j in range(n):
        sl = slots.clone()
        sl[accept <= j] = -1
        y = torch.zeros(b, case["H"], case["P"], device="cuda")
        tiered_state_update(pb_, 0, xs[:, j].cuda(), dts[:, j].cuda(), prm["A"].cuda(), Bs[:, j].cuda(),
                            Cs[:, j].cuda(), prm["D"].cuda(), prm["dt_bias"].cuda(), True, sl.to(torch.int32).cuda(),
                            -1, y, R, 1e-3)
        keep = (accept > j) & (slots >= 0)
        Hh.assert_y_close(yv[:, j].cpu()[keep], y.cpu()[keep], f"token {j}")
    torch.cuda.synchronize()
    for k in POOL_BUFFERS:
        a, b_ = getattr(pa, k), getattr(pb_, k)
        if a is not None:
            assert torch.equal(a, b_), f"{k} differs between commit and the decode steps"
    pa.check_status()
    pb_.check_status()
    return pa, accept


def _random_accept(b, n, gen):
    a = torch.randint(0, n + 1, (b,), generator=gen)
    a[: max(1, b // 3)] = n   # a third accept everything (and complete the chunk)
    return a


@pytest.mark.parametrize("cold", ["fp8", "bf16"])
@pytest.mark.parametrize("c,phase", [(4, 0), (4, 2), (16, 3), (64, 60)])
def test_commit_equals_decode_steps(cold, c, phase):
    _commit_vs_steps(b=12, S=20, c=c, phase=phase, cold=cold, accept_of=_random_accept, seed=c + phase)


def test_commit_with_rotation():
    _commit_vs_steps(b=9, S=9, c=4, phase=1, cold="fp8", accept_of=_random_accept, seed=5, use_rotation=True)


def test_commit_at_the_benchmarked_batch():
    """B = 448 (the tensor-core FLUSH over the rows the commit completes, the persistent STEP
    on the reference side), a full cycle from phase 0."""
    pool, accept = _commit_vs_steps(b=448, S=460, c=4, phase=0, cold="fp8", accept_of=_random_accept, seed=448)
    assert int((accept == 4).sum()) >= 448 // 3


def test_window_and_accept_errors_set_status():
    """A window across a chunk boundary and an accept count above n skip their rows and set
    bit 2 of the status word; the other rows are served."""
    from nested_ssm_b200 import commit_state_update, verify_state_update
    case = Hh.make_case(b=3, S=3, pb=32, c=4, cold="fp8", steps=5, seed=9)
    prm = case["prm"]
    gpool = Hh.gpu_pool(case)
    slots = torch.arange(3)
    _split(case, [gpool], None, slots)
    _gpu_step(case, gpool, 0, torch.tensor([0, -1, -1]))   # row 0 at phase 1, rows 1-2 at phase 0
    xs, dts, Bs, Cs = _stacked(case, 1, 4)
    sl32 = slots.to(torch.int32).cuda()
    y = torch.full((3, 4, case["H"], case["P"]), 7.0, device="cuda")
    verify_state_update(gpool, 0, xs.cuda(), dts.cuda(), prm["A"].cuda(), Bs.cuda(), Cs.cuda(), prm["D"].cuda(),
                        prm["dt_bias"].cuda(), True, sl32, -1, y, None, 1e-3)
    torch.cuda.synchronize()
    assert int(gpool.status.item()) & 4
    assert bool((y[0] == 7.0).all()), "the refused row was written"
    assert not bool((y[1] == 7.0).any())
    gpool.status.zero_()
    t0 = gpool.t.clone()
    commit_state_update(gpool, 0, torch.tensor([0, 5, 2], dtype=torch.int32, device="cuda"), xs.cuda(), dts.cuda(),
                        prm["A"].cuda(), Bs.cuda(), prm["dt_bias"].cuda(), True, sl32, -1, None, 1e-3)
    torch.cuda.synchronize()
    assert int(gpool.status.item()) & 4
    t1 = gpool.t[0].cpu()
    assert int(t1[0, 0]) == int(t0[0, 0, 0]) and int(t1[1, 0]) == int(t0[0, 1, 0]) and int(t1[2, 0]) == int(t0[0, 2, 0]) + 2
    gpool.status.zero_()
