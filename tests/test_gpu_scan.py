"""The prefill chunked scan (nssm_chunk_scan, tcgen05 tensor cores) through the C ABI.

* against the CPU oracle's restatement of mamba_ssm's chunked algorithm with the same bf16
  operand roundings (oracle/scan.py): y within one bf16 ulp plus the scale of an occasional
  flipped intermediate rounding, the fp32 final state within the accumulation-order scale;
  prompts of one token, one exact chunk, ragged chunks, several chunks; headdim 80 and 64;
  with and without initial states and D; fp32 and bf16 dt; dt clamps; x / B / C / dt as
  strided views of the conv output and in_proj output, as the reference passes them;
* against the reference's prefill (prefill_hf.npz, fp32): within the bf16 rounding of the
  operands that the reference's own lean prefill (mamba_ssm) also rounds.
"""
import math

import pytest
import torch

import oracle as O
from tests import _golden as GD

pytestmark = pytest.mark.gpu


def _inputs(b, T, H, P, G, seed, N=128, strided=True, dt_bf16=True):
    """x / B / C as views of one [b, T, conv_dim] conv output and dt as a view of an in_proj
    output (the reference's _lean_prefill layout), bf16, on the GPU; plus CPU copies."""
    g = torch.Generator().manual_seed(seed)
    I, GN = H * P, G * N
    xbc = torch.cat([torch.randn(b, T, I, generator=g), torch.randn(b, T, 2 * GN, generator=g) / N ** 0.25], -1)
    xbc = xbc.to(torch.bfloat16)
    proj = torch.randn(b, T, 2 * I + H, generator=g)
    proj = proj.to(torch.bfloat16) if dt_bf16 else proj
    prm = O.make_params(H, G, N, seed=seed)[0]
    cpu = dict(x=xbc[..., :I].reshape(b, T, H, P), B=xbc[..., I:I + GN].reshape(b, T, G, N),
               C=xbc[..., I + GN:].reshape(b, T, G, N), dt=proj[..., 2 * I:], A=prm["A"], D=prm["D"],
               dt_bias=prm["dt_bias"], s0=torch.randn(b, H, P, N, generator=g) * 0.3)
    if strided:
        xg, pg = xbc.cuda(), proj.cuda()
        gpu = dict(x=xg[..., :I].view(b, T, H, P), B=xg[..., I:I + GN].view(b, T, G, N),
                   C=xg[..., I + GN:].view(b, T, G, N), dt=pg[..., 2 * I:])
    else:
        gpu = {k: cpu[k].contiguous().cuda() for k in ("x", "B", "C", "dt")}
    for k in ("A", "D", "dt_bias", "s0"):
        gpu[k] = cpu[k].cuda()
    return cpu, gpu


def _abs_scan(cpu, s0, lim, T_chunk=128):
    """Magnitudes for the error bounds: the fp32 scan of |x|, |B|, |C| (and |S0|) without D,
    i.e. sum |M x| + sum |C S| e^cs per y element and sum |B_s x| per state element, each term
    a bound on the corresponding |term| of the real scan."""
    return O.chunk_scan(cpu["x"].abs(), cpu["dt"], cpu["A"], cpu["B"].abs(), cpu["C"].abs(), T_chunk, None,
                        cpu["dt_bias"], None if s0 is None else s0.abs(), True, lim, rounding=False)


def _close_y(got, want, yabs, what):
    """|dy| <= one bf16 ulp of y + one bf16 ulp of every intermediate term (an operand
    rounding that falls the other way: M = bf16(C.B e dt) or bf16(S_prev), whose inputs
    differ in the last fp32 bits through the cumsum order and exp) + fp32 accumulation."""
    g, w = got.float().cpu(), want.float()
    err = (g - w).abs()
    bound = (w.abs() + yabs) * 2.0 ** -7 + yabs * 1e-5 + 1e-6
    assert bool((err <= bound).all()), f"{what}: max err/bound {float((err / bound).max()):.2f}"
    rel = float(err.norm() / w.norm())
    assert rel < 2e-3, f"{what}: relative error norm {rel:.2e}"


def _close_state(got, want, sabs, what):
    """|dS| <= one bf16 ulp of every bf16(B e dt) term times |x| + fp32 accumulation."""
    g, w = got.cpu(), want
    err = (g - w).abs()
    bound = sabs * (2.0 ** -7 + 1e-5) + 1e-7
    assert bool((err <= bound).all()), f"{what}: max err/bound {float((err / bound).max()):.2f}"
    rel = float(err.norm() / w.norm())
    assert rel < 2e-3, f"{what}: relative error norm {rel:.2e}"


@pytest.mark.parametrize("T,P,H,G,init,D,dt_bf16,strided,lim", [
    (300, 80, 8, 2, False, True, True, True, (0.0, math.inf)),
    (128, 80, 8, 2, True, True, True, True, (0.0, math.inf)),
    (1, 80, 8, 2, True, True, False, False, (0.0, math.inf)),
    (77, 80, 4, 1, False, False, True, False, (1e-3, math.inf)),
    (513, 64, 8, 4, True, True, False, True, (1e-3, 0.08)),
    (260, 64, 4, 2, False, True, True, False, (0.0, math.inf)),
])
def test_scan_matches_oracle(T, P, H, G, init, D, dt_bf16, strided, lim):
    from nested_ssm_b200 import mamba_chunk_scan_combined
    b = 2
    cpu, gpu = _inputs(b, T, H, P, G, seed=T + P, strided=strided, dt_bf16=dt_bf16)
    s0 = cpu["s0"] if init else None
    y_ref, S_ref = O.chunk_scan(cpu["x"], cpu["dt"], cpu["A"], cpu["B"], cpu["C"], 128, cpu["D"] if D else None,
                                cpu["dt_bias"], s0, True, lim)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    y, S = mamba_chunk_scan_combined(gpu["x"], gpu["dt"], gpu["A"], gpu["B"], gpu["C"], 128,
                                     D=gpu["D"] if D else None, dt_bias=gpu["dt_bias"],
                                     initial_states=gpu["s0"] if init else None, dt_softplus=True, dt_limit=lim,
                                     return_final_states=True, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    yabs, sabs = _abs_scan(cpu, s0, lim)
    _close_y(y, y_ref, yabs, f"T={T} P={P} y")
    _close_state(S, S_ref, sabs, f"T={T} P={P} final state")


def test_scan_vs_reference_prefill():
    """prefill_hf.npz: the reference's prefill on the same (bf16-representable) inputs, fp32."""
    from nested_ssm_b200 import mamba_chunk_scan_combined
    d = GD.load("prefill_hf.npz")
    cfg = GD.MG.PREFILL
    inp = GD.MG.prefill_inputs(cfg)
    cu = {k: inp[k].to(torch.bfloat16).cuda() for k in ("x", "B", "C")}
    y, S = mamba_chunk_scan_combined(cu["x"], inp["dt"].cuda(), inp["A"].cuda(), cu["B"], cu["C"], cfg["chunk"],
                                     D=inp["D"].cuda(), dt_bias=inp["dt_bias"].cuda(), dt_softplus=True,
                                     dt_limit=(1e-3, math.inf), return_final_states=True)
    torch.cuda.synchronize()
    # the reference computes in fp32; the bf16 operand roundings (as mamba_ssm's) bound the gap
    yr, Sr = d["y"], d["state"]
    err = (y.float().cpu() - yr).abs()
    assert float(err.max()) <= 1e-2 * float(yr.abs().max()), float(err.max())
    assert float((S.cpu() - Sr).abs().max()) <= 1e-2 * float(Sr.abs().max())
    # and against the oracle's restatement of the same roundings: tight
    y_ref, S_ref = O.chunk_scan(inp["x"].bfloat16(), inp["dt"], inp["A"], inp["B"].bfloat16(), inp["C"].bfloat16(),
                                cfg["chunk"], inp["D"], inp["dt_bias"], None, True, (1e-3, math.inf))
    yabs, sabs = _abs_scan(inp, None, (1e-3, math.inf))
    _close_y(y, y_ref, yabs, "golden y")
    _close_state(S, S_ref, sabs, "golden final state")


def test_scan_final_state_splits_into_pool():
    """Prefill as the reference's lean prefill + prefill_snapshot do it: the scan's final state
    split into a tiered fp8 pool equals the split of the same state done separately."""
    from nested_ssm_b200 import TieredSlotPool, mamba_chunk_scan_combined, materialize, prefill_split
    b, T, H, P, G = 3, 200, 8, 80, 2
    cpu, gpu = _inputs(b, T, H, P, G, seed=9)
    y, S = mamba_chunk_scan_combined(gpu["x"], gpu["dt"], gpu["A"], gpu["B"], gpu["C"], 128, D=gpu["D"],
                                     dt_bias=gpu["dt_bias"], dt_softplus=True, return_final_states=True)
    pool = TieredSlotPool(1, 5, H, P, 128, G, 32, 4, "fp8", torch.bfloat16, "cuda", max_batch=b)
    slots = torch.tensor([4, 0, 2], dtype=torch.int32, device="cuda")
    prefill_split(pool, 0, S, slots)
    full = materialize(pool, 0, slots, gpu["A"])
    torch.cuda.synchronize()
    Sc = S.cpu()
    assert torch.equal(full[..., :32].cpu(), Sc[..., :32])
    cold = full[..., 32:].cpu()
    want = O.dequantize_rows(*O.quantize_rows(Sc[..., 32:], torch.float8_e4m3fn))
    assert torch.equal(cold, want)
