"""The HF integration (``nested_ssm_b200.hf.install``) against the reference's own
(hf_generate.npz: a small seeded NemotronH, rotated mixers, the reference's ``install`` with
``cold_bf16=0``, greedy generate on the CPU): the same model on the GPU with our install must
produce the same tokens and logits within fp32 rounding of the decode path."""
import pytest
import torch

from tests import _golden as GD

pytestmark = pytest.mark.gpu


class RotAct(torch.nn.Module):
    """SiLU, then the per-group rotation of the B and C slices of the conv output: what the
    reference's ActRotMask does for a full-width (unmasked) rotation
    (scale/nemotron_retrofit.py:18-54).  The decode path reads R and the SiLU from it."""

    def __init__(self, act, inter, ngroups, dstate, R):
        super().__init__()
        self.act = act
        self.inter, self.ng, self.ds = inter, ngroups, dstate
        self.R = torch.nn.Parameter(R.clone())

    def forward(self, x):
        x = self.act(x)
        if x.dim() == 3 and x.shape[-1] == self.inter + 2 * self.ng * self.ds:
            h, B, C = torch.split(x, [self.inter, self.ng * self.ds, self.ng * self.ds], dim=-1)
            b, t, _ = B.shape
            rot = lambda v: torch.einsum("btgn,gmn->btgm", v.view(b, t, self.ng, self.ds),  # noqa: E731
                                         self.R.to(v.dtype)).reshape(b, t, -1)
            x = torch.cat([h, rot(B), rot(C)], dim=-1)
        return x


def test_hf_generate_matches_reference_install():
    from nested_ssm_b200.hf import install
    d = GD.load("hf_generate.npz")
    cfg = GD.MG.HF
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    model = GD.MG.hf_model(cfg["seed"])
    Rs = GD.MG.hf_rotations(model, cfg["seed"])
    mixers = [m for m in model.modules() if type(m).__name__ == "NemotronHMamba2Mixer"]
    for m, R in zip(mixers, Rs):
        m.act = RotAct(m.act, m.intermediate_size, m.n_groups, m.ssm_state_size, R)
    model = model.cuda()
    assert install(model, pb=cfg["pb"], c=cfg["c"], cold_bf16=0) == len(mixers)
    with torch.no_grad():
        out = model.generate(d["ids"].cuda(), max_new_tokens=cfg["new"], do_sample=False, output_logits=True,
                             return_dict_in_generate=True)
    logits = torch.stack(out.logits).float().cpu()
    torch.testing.assert_close(logits, d["logits"], rtol=1e-3, atol=1e-3)
    assert torch.equal(out.sequences.cpu(), d["tokens"])
    for m in mixers:   # the decode went through the tiered pool
        assert m._nssm["pool"] is not None and int(m._nssm["pool"].t[0].max()) == cfg["new"] - 1
