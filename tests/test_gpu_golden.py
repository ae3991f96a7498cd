"""The CUDA path (through the C ABI) against the golden fixtures made by running the
reference's own code (tests/golden/make_golden.py), with no oracle in between.

* ``_v4_decode`` (HF native decode, fp32 hot and cold, c=4), modes stale / corr / coldoff,
  B and C rotated on the GPU: y within the parity bar (rtol 2e-3 / atol 1e-3) at every
  step through three flushes; the final state of two heads within fp32 accumulation.
* ``prefill_snapshot`` with fp8 cold: codes and scales bit-exact.
* ``decode_readout`` with fp8 cold: y within the parity bar, t exact and glog within
  fp32 rounding until the first flush (after it the fp8-only cold master drifts from the
  fp32 master by design; the oracle tests cover the replay).
* rotation: within one ulp plus the fp32 dot-product rounding bound of ``rot_flat`` in fp32.
"""
import pytest
import torch

from tests import _golden as GD
from tests import _helpers as Hh

pytestmark = pytest.mark.gpu


def _pool(S, H, P, N, G, pb, c, cold):
    from nested_ssm_b200 import TieredSlotPool
    return TieredSlotPool(1, S, H, P, N, G, pb, c, cold, torch.bfloat16, "cuda", max_batch=S)


@pytest.mark.parametrize("mode", ["stale", "corr", "coldoff"])
def test_native_decode_golden(mode):
    from nested_ssm_b200 import materialize, prefill_split, tiered_state_update
    d = GD.load("native_decode_fp32.npz")
    inp = GD.native_inputs(mode)
    GD.check_sums(d, inp, f"{mode}_")
    cfg = inp["cfg"]
    b, H, P, N, G, pb, c = (cfg[k] for k in ("b", "H", "P", "N", "G", "pb", "c"))
    pool = _pool(b, H, P, N, G, pb, c, "fp32")
    slots = torch.arange(b, dtype=torch.int32, device="cuda")
    prefill_split(pool, 0, inp["s0"].cuda(), slots)
    A, D, dtb, R = (d[k].cuda() for k in ("A", "D", "dt_bias", "R"))
    for s in range(inp["steps"]):
        out = torch.zeros(b, H, P, device="cuda")
        tiered_state_update(pool, 0, inp["xs"][s].cuda(), inp["dts"][s].cuda(), A, inp["Bs"][s].cuda(),
                            inp["Cs"][s].cuda(), D, dtb, True, slots, -1, out, R, 1e-3, mode)
        Hh.assert_y_close(out, d[f"{mode}_y"][s], f"{mode} step {s}")
    pool.check_status()
    if mode == "stale":
        st = materialize(pool, 0, slots, A).cpu()[:, [0, 9]]
        torch.testing.assert_close(st, d["stale_state_final_h0_h9"], rtol=1e-4, atol=1e-4)


def test_rotation_golden():
    from nested_ssm_b200 import rot_flat
    d = GD.load("rot_flat.npz")
    x, R = GD.bf16(d["x"]).cuda(), d["R"].cuda()
    Hh.rotation_close(rot_flat(x, R).cpu(), d["out_fp32"].to(torch.bfloat16), x.cpu(), R.cpu())
    Hh.rotation_close(rot_flat(x.float(), R).cpu(), d["out_fp32"], x.cpu(), R.cpu())


def test_vllm_fp8_golden():
    from nested_ssm_b200 import prefill_split, tiered_state_update
    d = GD.load("vllm_fp8.npz")
    inp = GD.vllm_inputs()
    GD.check_sums(d, inp)
    cfg = inp["cfg"]
    S, b, H, P, N, G, pb, c = (cfg[k] for k in ("S", "b", "H", "P", "N", "G", "pb", "c"))
    pool = _pool(S, H, P, N, G, pb, c, "fp8")
    slots = inp["slots"].to(torch.int32).cuda()
    prefill_split(pool, 0, inp["s0"].cuda(), slots)
    sl = inp["slots"].long()
    assert torch.equal(pool.cold[0].cpu()[sl].view(torch.uint8), d["pre_codes"])
    assert torch.equal(pool.scale[0].cpu()[sl], d["pre_scale"])
    A, D, dtb = (d[k].cuda() for k in ("A", "D", "dt_bias"))
    for s in range(c):                   # up to and including the first flush token
        out = torch.zeros(b, H, P, device="cuda")
        tiered_state_update(pool, 0, inp["xs"][s].cuda(), inp["dts"][s].cuda(), A, inp["Bs"][s].cuda(),
                            inp["Cs"][s].cuda(), D, dtb, True, slots, -1, out, None, None, "stale")
        Hh.assert_y_close(out, d["y"][s], f"step {s}")
        assert torch.equal(pool.t[0].cpu()[sl], d["t"][s][:, None].expand(-1, H))
        torch.testing.assert_close(pool.glog[0].cpu()[sl], d["glog"][s], rtol=1e-5, atol=1e-6)
    pool.check_status()
