"""The prefill-scan oracle (oracle/scan.py) on the CPU.

* against the reference's own prefill (prefill_hf.npz: ``_dispatch`` of
  scale/v4_native_decode.py with ``lean_prefill=0`` on a stub mixer, i.e. transformers'
  NemotronH torch_forward chunked SSD), fp32 operands: y and the final state;
* the chunked form against the token-by-token recurrence on prompts of several chunks
  (ragged last chunk, other chunk sizes, initial states, dt clamps, no D);
* the bf16 operand rounding of mamba_ssm's kernels stays within its own error scale.
"""
import math

import pytest
import torch

import oracle as O
from tests import _golden as GD


def _case(b, T, H, P, G, N=128, seed=0):
    g = torch.Generator().manual_seed(seed)
    prm = O.make_params(H, G, N, seed=seed)[0]
    bf = lambda t: t.to(torch.bfloat16)   # noqa: E731
    return dict(x=bf(torch.randn(b, T, H, P, generator=g)), dt=bf(torch.randn(b, T, H, generator=g)),
                A=prm["A"], B=bf(torch.randn(b, T, G, N, generator=g) / N ** 0.25),
                C=bf(torch.randn(b, T, G, N, generator=g) / N ** 0.25), D=prm["D"], dt_bias=prm["dt_bias"],
                s0=torch.randn(b, H, P, N, generator=g) * 0.3)


def test_chunk_scan_matches_reference_prefill():
    d = GD.load("prefill_hf.npz")
    cfg = GD.MG.PREFILL
    inp = GD.MG.prefill_inputs(cfg)
    for k in ("x", "B", "C", "dt"):
        assert float(d[f"sum_{k}"]) == GD.MG.checksum(inp[k]), f"regenerated input {k} differs from the fixture's"
    y, S = O.chunk_scan(inp["x"], inp["dt"], inp["A"], inp["B"], inp["C"], cfg["chunk"], inp["D"], inp["dt_bias"],
                        None, True, (1e-3, math.inf), rounding=False)
    torch.testing.assert_close(y, d["y"], rtol=1e-5, atol=2e-5)
    torch.testing.assert_close(S, d["state"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("T,Q,init,lim,D", [(300, 128, False, (0.0, math.inf), True), (300, 64, True, (0.0, math.inf), True),
                                            (129, 128, True, (1e-3, 0.05), False), (1, 128, True, (0.0, math.inf), True)])
def test_chunked_equals_recurrence(T, Q, init, lim, D):
    c = _case(2, T, 4, 80, 2, seed=T + Q)
    s0 = c["s0"] if init else None
    Dv = c["D"] if D else None
    y, S = O.chunk_scan(c["x"], c["dt"], c["A"], c["B"], c["C"], Q, Dv, c["dt_bias"], s0, True, lim, rounding=False)
    yr, Sr = O.scan_recurrent(c["x"], c["dt"], c["A"], c["B"], c["C"], Dv, c["dt_bias"], s0, True, lim)
    torch.testing.assert_close(y, yr, rtol=1e-5, atol=1e-5 * float(yr.abs().max()))
    torch.testing.assert_close(S, Sr, rtol=1e-5, atol=1e-5 * float(Sr.abs().max()))


def test_bf16_rounding_stays_small():
    c = _case(2, 300, 4, 80, 2, seed=5)
    yf, Sf = O.chunk_scan(c["x"], c["dt"], c["A"], c["B"], c["C"], 128, c["D"], c["dt_bias"], c["s0"], True,
                          rounding=False)
    yb, Sb = O.chunk_scan(c["x"], c["dt"], c["A"], c["B"], c["C"], 128, c["D"], c["dt_bias"], c["s0"], True)
    assert yb.dtype == torch.bfloat16
    assert float((yb.float() - yf).abs().max()) < 1e-2 * float(yf.abs().max())
    assert float((Sb - Sf).abs().max()) < 1e-2 * float(Sf.abs().max())
