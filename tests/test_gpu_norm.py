"""nssm_gated_rmsnorm (the mixer's norm(y, gate) after the state op) against the CPU oracle:
within one io ulp (fp32 sums of 1280 squares in another order; expf)."""
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,wdt", [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32),
                                       (torch.bfloat16, torch.float32)])
def test_gated_rmsnorm_matches_oracle(dtype, wdt):
    from nested_ssm_b200 import gated_rmsnorm
    gen = torch.Generator().manual_seed(3)
    b, dim, gs = 37, 10240, 1280
    y = torch.randn(b, 1, dim, generator=gen).to(dtype)
    z = torch.randn(b, 1, dim, generator=gen).to(dtype)
    w = (1.0 + 0.1 * torch.randn(dim, generator=gen)).to(wdt)
    want = O.gated_rmsnorm(y, z, w, 1e-5, gs)
    got = gated_rmsnorm(y.cuda(), z.cuda(), w.cuda(), 1e-5, gs).cpu()
    assert got.shape == want.shape and got.dtype == want.dtype
    ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -20   # one bf16 ulp (two roundings) / fp32 slack
    err = (got.float() - want.float()).abs()
    bound = want.float().abs() * ulp + 1e-6
    assert bool((err <= bound).all()), f"off by {float((err / bound).max()):.2f}x"
    if dtype == torch.bfloat16:   # fp32 outputs differ in the last bits almost everywhere
        assert float((err > 0).float().mean()) <= 5e-2
