"""The decode-token conv (nssm_conv_step: causal conv1d update + SiLU + split + rotation of
B and C) on the GPU, through the C ABI.

* against the CPU oracle: x, B, C within one io ulp (B, C after the rotation: plus the fp32
  rounding bound and one io ulp of each rotated input), the conv state exactly (it only
  moves stored values), padded rows untouched, a permuted slot map, state lengths K and
  K-1, fp32 and bf16 weights, with and without R;
* against the reference (native_decode_conv.npz): conv + SiLU + rotation + tiered state op,
  fp32, y within the parity bar at every step through two flushes, final conv state exact.
"""
import pytest
import torch

import oracle as O
from tests import _golden as GD
from tests import _helpers as Hh

pytestmark = pytest.mark.gpu

H, P, N, G = 128, 80, 128, 8
I = H * P
D = I + 2 * G * N


def _close_io(got, want, what):
    """Within one io ulp of the oracle's value, or 1e-6 absolute (values near zero)."""
    g, w = got.float().cpu(), want.float()
    ulp = 2.0 ** -8 if got.dtype == torch.bfloat16 else 2.0 ** -23
    bound = w.abs() * ulp + 1e-6
    err = (g - w).abs()
    assert bool((err <= bound).all()), f"{what}: off by {float((err / bound).max()):.2f}x the bound"
    assert float((err > 0).float().mean()) <= 2e-2, f"{what}: differs too often"


@pytest.mark.parametrize("K,L,wdt,rot,last", [(4, 3, torch.bfloat16, True, False), (4, 4, torch.float32, True, False),
                                              (4, 3, torch.float32, False, False), (3, 2, torch.bfloat16, True, False),
                                              (4, 4, torch.bfloat16, True, True), (3, 3, torch.float32, False, True)])
def test_conv_step_matches_oracle(K, L, wdt, rot, last):
    """Width 4 with state length 3 or 4 runs the vectorised kernels, other shapes the
    per-element ones; ``last``: the conv state channels-last, as the HF cache keeps it."""
    from nested_ssm_b200 import conv_step
    gen = torch.Generator().manual_seed(7 + L)
    S, b = 12, 9
    slots = torch.tensor([5, -1, 0, 11, 3, 7, -1, 2, 9])
    state0 = torch.randn(S, D, L, generator=gen).to(torch.bfloat16)
    weight = (torch.rand(D, K, generator=gen) - 0.5).to(wdt)
    bias = (torch.randn(D, generator=gen) * 0.1).to(wdt)
    R = O.make_params(H, G, N, seed=3)[0]["R"] if rot else None
    ostate = state0.clone()
    if last:
        gstate = torch.empty(S, L, D, dtype=torch.bfloat16, device="cuda").transpose(1, 2)
        gstate.copy_(state0)
    else:
        gstate = state0.cuda()
    for step in range(3):
        xbc = torch.randn(b, D, generator=gen).to(torch.bfloat16)
        out = O.conv_step(ostate, slots, xbc, weight, bias, "silu")
        xo, Bo, Co = O.conv_split(out, I, G, N, None, torch.bfloat16)
        Bpre, Cpre = Bo.reshape(b, G * N), Co.reshape(b, G * N)
        if rot:
            Bo = O.rot_flat(Bpre, R, "fp32").reshape(b, G, N)
            Co = O.rot_flat(Cpre, R, "fp32").reshape(b, G, N)
        x0 = torch.full((b, H, P), 7.0, dtype=torch.bfloat16, device="cuda")
        xg, Bg, Cg = conv_step(xbc.cuda(), gstate, weight.cuda(), bias.cuda(), "silu",
                               slots.to(torch.int32).cuda(), -1, None if R is None else R.cuda(),
                               nheads=H, headdim=P, ngroups=G, dstate=N, x_out=x0)
        torch.cuda.synchronize()
        live = slots >= 0
        assert torch.equal(gstate.cpu(), ostate), f"step {step}: conv state differs"
        assert bool((xg.cpu()[~live] == 7.0).all()), "padded rows must be left untouched"
        _close_io(xg.cpu()[live].reshape(-1, I), xo[live], f"step {step} x")
        if rot:
            # the rotated inputs are the GPU's own conv outputs, each within one io ulp
            Hh.rotation_close(Bg.cpu()[live].reshape(-1, G * N), Bo[live].reshape(-1, G * N), Bpre[live], R, 1)
            Hh.rotation_close(Cg.cpu()[live].reshape(-1, G * N), Co[live].reshape(-1, G * N), Cpre[live], R, 1)
        else:
            _close_io(Bg.cpu()[live], Bo[live], f"step {step} B")
            _close_io(Cg.cpu()[live], Co[live], f"step {step} C")


def test_conv_then_tiered_step_vs_reference():
    """native_decode_conv.npz: the reference's _v4_decode with a real conv1d and its
    ActRotMask activation; here nssm_conv_step then nssm_tiered_step, fp32 throughout."""
    from nested_ssm_b200 import TieredSlotPool, conv_step, prefill_split, tiered_state_update
    d = GD.load("native_decode_conv.npz")
    cfg, inp = GD.conv_case()
    b, h, p, n, g, pb, c = (cfg[k] for k in ("b", "H", "P", "N", "G", "pb", "c"))
    pool = TieredSlotPool(1, b, h, p, n, g, pb, c, "fp32", torch.float32, "cuda", max_batch=b)
    slots = torch.arange(b, dtype=torch.int32, device="cuda")
    prefill_split(pool, 0, inp["s0"].cuda(), slots)
    conv_state = inp["state"].cuda().contiguous()
    weight = inp["weight"].reshape(-1, cfg["K"]).cuda().contiguous()
    bias = inp["bias"].cuda()
    R, A, Dh, dtb = (d[k].cuda() for k in ("R", "A", "D", "dt_bias"))
    for s in range(cfg["steps"]):
        x, Bv, Cv = conv_step(inp["xbc"][s].cuda(), conv_state, weight, bias, "silu", slots, -1, R,
                              nheads=h, headdim=p, ngroups=g, dstate=n)
        out = torch.zeros(b, h, p, device="cuda")
        tiered_state_update(pool, 0, x, inp["dts"][s].cuda(), A, Bv, Cv, Dh, dtb, True, slots, -1, out,
                            None, 1e-3)
        Hh.assert_y_close(out, d["y"][s], f"step {s}")
    pool.check_status()
    assert torch.equal(conv_state.cpu(), d["conv_state_final"])
