"""nssm_tiered_step_static (static rotation scratch, no caller workspace) against
nssm_tiered_step (caller workspace), both called through the C ABI.

Two pools start from the same prefilled state; each takes the same two tokens
(the second one flushes, c = 2) with the rotation on the GPU, one pool through
each entry point.  Outputs and pool state must agree within the parity bar.
Collected last so it also runs after every other GPU test in one process.
"""
import ctypes as C

import pytest
import torch

from tests import _helpers as Hh

pytestmark = pytest.mark.gpu


def _call(entry, gpool, case, step, slots, out):
    from nested_ssm_b200 import _lib, ops
    prm = case["prm"]
    ws = gpool.workspace if entry == "nssm_tiered_step" else None
    a, out, keep = ops.build_step_args(
        case["xs"][step].cuda(), case["dts"][step].cuda(), prm["A"].cuda(), case["Bs"][step].cuda(),
        case["Cs"][step].cuda(), prm["D"].cuda(), prm["dt_bias"].cuda(), True, slots, -1, out,
        prm["R"].cuda(), 1e-3, "stale", ws, gpool.status, nheads=gpool.H)
    lib = _lib.load()
    rc = getattr(lib, entry)(C.byref(gpool.struct(0)), C.byref(a), torch.cuda.current_stream().cuda_stream)
    return rc, keep


@pytest.mark.parametrize("io_dtype", [torch.bfloat16, torch.float32])
def test_static_scratch_matches_workspace_entry(io_dtype):
    from nested_ssm_b200 import prefill_split
    case = Hh.make_case(b=40, S=48, pb=32, c=2, cold="fp8", steps=2, seed=5, io_dtype=io_dtype)
    slots = torch.randperm(48, generator=torch.Generator().manual_seed(5))[:40].to(torch.int32)
    slots[[3, 17]] = -1
    slots_d = slots.cuda()
    pools = {e: Hh.gpu_pool(case) for e in ("nssm_tiered_step", "nssm_tiered_step_static")}
    for p in pools.values():
        prefill_split(p, 0, case["state0"].cuda(), slots_d)
    for step in range(2):
        ys = {}
        for entry, p in pools.items():
            out = torch.zeros(40, case["H"], case["P"], device="cuda")
            rc, keep = _call(entry, p, case, step, slots_d, out)
            assert rc == 0, f"{entry} returned {rc}"
            ys[entry] = out
        torch.cuda.synchronize()
        ref, got = ys["nssm_tiered_step"], ys["nssm_tiered_step_static"]
        Hh.assert_y_close(got, ref.cpu(), f"step {step}")
        a, b = pools["nssm_tiered_step"], pools["nssm_tiered_step_static"]
        # the same kernels on the same inputs: the hot state is bit-identical
        assert torch.equal(b.hot.cpu(), a.hot.cpu())
        assert int(Hh.fp8_ulp_dist(b.cold, a.cold).max()) <= 1
        torch.testing.assert_close(b.scale.cpu(), a.scale.cpu(), rtol=1e-5, atol=0)
        assert torch.equal(b.t.cpu(), a.t.cpu())
        torch.testing.assert_close(b.glog.cpu(), a.glog.cpu(), rtol=1e-6, atol=1e-6)
        torch.testing.assert_close(b.ring_b.cpu(), a.ring_b.cpu(), rtol=0, atol=0)
    for p in pools.values():
        p.check_status()


def test_static_scratch_rejects_oversized_batch():
    """A batch whose rotated B and C exceed the static scratch is refused before any
    launch (every row is padding, so nothing would be written even if it ran)."""
    from nested_ssm_b200 import _lib
    b = 1025                       # bf16, G=8, N=128: limit is 1024 rows
    case = Hh.make_case(b=b, S=8, H=16, G=8, pb=32, c=4, cold="fp8", steps=1, seed=1)
    gpool = Hh.gpu_pool(case)
    slots = torch.full((b,), -1, dtype=torch.int32, device="cuda")
    out = torch.zeros(b, case["H"], case["P"], device="cuda")
    before = out.clone()
    rc, keep = _call("nssm_tiered_step_static", gpool, case, 0, slots, out)
    assert rc == _lib.NSSM_ERR_INVALID
    msg = _lib.load().nssm_last_error().decode()
    assert "static scratch" in msg and str(4 << 20) in msg
    torch.cuda.synchronize()
    assert torch.equal(out, before)
