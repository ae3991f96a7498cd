"""Failure detection of the persistent decode kernels without a GPU fault: a pipeline wait
that can never complete (the injected stuck copy: CTA 0 announces 16 bytes more than its first
item's copies deliver) runs out after a short poll limit, the call returns with bit 1 of the
status word set, and the CUDA context stays usable (a fresh pool then steps at the parity bar).
Every wait involved is bounded; nothing traps."""
import pytest
import torch

import oracle as O
from tests import _helpers as Hh

pytestmark = pytest.mark.gpu


def _step(case, gpool, s, slots):
    from nested_ssm_b200 import tiered_state_update
    prm = case["prm"]
    B, C_ = Hh.rotated(case, s)
    out = torch.zeros(case["b"], case["H"], case["P"], device="cuda")
    tiered_state_update(gpool, 0, case["xs"][s].cuda(), case["dts"][s].cuda(), prm["A"].cuda(), B.cuda(),
                        C_.cuda(), prm["D"].cuda(), prm["dt_bias"].cuda(), True, slots.cuda(), -1, out, None,
                        1e-3)
    return out


def test_stuck_copy_times_out_with_status_and_context_survives():
    from nested_ssm_b200 import _lib, prefill_split
    lib = _lib.load()
    case = Hh.make_case(b=64, S=64, pb=32, c=4, cold="fp8", steps=2, seed=3)
    slots = torch.arange(64, dtype=torch.int32)
    gpool = Hh.gpu_pool(case)
    prefill_split(gpool, 0, case["state0"].cuda(), slots.cuda())
    old_polls = lib.nssm_set_wait_polls(4096)
    old_inj = lib.nssm_test_inject_stuck_copy(1)
    try:
        _step(case, gpool, 0, slots)
        torch.cuda.synchronize()
        status = int(gpool.status.item())
    finally:
        lib.nssm_test_inject_stuck_copy(old_inj)
        lib.nssm_set_wait_polls(old_polls)
    assert status & 2, f"status {status}: the stuck wait did not report a timeout"
    assert torch.cuda.is_available() and torch.zeros(1, device="cuda").add_(1).item() == 1.0
    # the context is intact: a fresh pool steps at the per-step parity bar
    opool, gpool2 = Hh.oracle_pool(case), Hh.gpu_pool(case)
    O.prefill_split(opool, slots, case["state0"])
    prefill_split(gpool2, 0, case["state0"].cuda(), slots.cuda())
    for s in range(2):
        Hh.sync_oracle_from_gpu(gpool2, opool)
        yg, yo = Hh.step_both(case, gpool2, opool, s, slots)
        Hh.assert_y_close(yg, yo, f"step {s} after the timeout")
        Hh.compare_pool(gpool2, opool, 0, slots, "fp8", max_ulp=1, max_ulp_frac=1e-4)
    assert int(gpool2.status.item()) == 0
