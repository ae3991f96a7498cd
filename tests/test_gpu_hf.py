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

    def __init__(self, act, inter, ngroups, dstate, R, width=None):
        super().__init__()
        self.act = act
        self.inter, self.ng, self.ds = inter, ngroups, dstate
        self.R = torch.nn.Parameter(R.clone())
        self.width = dstate if width is None else width

    def forward(self, x):
        x = self.act(x)
        if x.dim() == 3 and x.shape[-1] == self.inter + 2 * self.ng * self.ds:
            h, B, C = torch.split(x, [self.inter, self.ng * self.ds, self.ng * self.ds], dim=-1)
            b, t, _ = B.shape
            keep = (torch.arange(self.ds, device=x.device) < self.width).to(x.dtype)   # int width
            rot = lambda v: (torch.einsum("btgn,gmn->btgm", v.view(b, t, self.ng, self.ds),  # noqa: E731
                                          self.R.to(v.dtype)) * keep).reshape(b, t, -1)
            x = torch.cat([h, rot(B), rot(C)], dim=-1)
        return x


def _mixer_decode_outputs(mixers):
    outs = [[] for _ in mixers]
    for i, m in enumerate(mixers):
        def hook(mod, args, out, i=i):
            if out.shape[1] == 1:
                outs[i].append(out.detach().float().cpu().clone())
        m.register_forward_hook(hook)
    return outs


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


def test_hf_width_mask_matches_reference():
    """ActRotMask's width (the reference's set_width, scale/nemotron_retrofit.py:112-114) masks
    the rotated B and C to their first 64 coordinates; hf_generate_width.npz holds the
    reference's install + generate with that mask on a model whose mixer output is dominated
    by the state term.  Every mixer's output at every decode step must match it to 2e-3 of its
    magnitude (ignoring the mask moves it by ~95%)."""
    from nested_ssm_b200.hf import install
    d = GD.load("hf_generate_width.npz")
    cfg = GD.MG.HF
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    model = GD.MG.hf_state_dominant(GD.MG.hf_model(cfg["seed"]))
    Rs = GD.MG.hf_rotations(model, cfg["seed"])
    mixers = [m for m in model.modules() if type(m).__name__ == "NemotronHMamba2Mixer"]
    for m, R in zip(mixers, Rs):
        m.act = RotAct(m.act, m.intermediate_size, m.n_groups, m.ssm_state_size, R, width=GD.MG.HF_WIDTH)
    model = model.cuda()
    assert install(model, pb=cfg["pb"], c=cfg["c"], cold_bf16=0) == len(mixers)
    outs = _mixer_decode_outputs(mixers)
    with torch.no_grad():
        out = model.generate(d["ids"].cuda(), max_new_tokens=cfg["new"], do_sample=False, output_logits=True,
                             return_dict_in_generate=True)
    got = torch.stack([torch.stack(o) for o in outs])
    ref = d["mixer_out"]
    assert got.shape == ref.shape
    scale = float(ref.abs().max())
    err = float((got - ref).abs().max())
    assert err <= 2e-3 * scale, f"mixer outputs differ by {err:.3e} (|ref| max {scale:.3e})"
    assert torch.equal(out.sequences.cpu(), d["tokens"])


def _bf16_model(seed: int):
    """A small bf16 NemotronH whose mixers have the compiled chunk-scan shapes (headdim 80,
    d_state 128, chunk 128), with seeded rotations wrapped around the activation."""
    from transformers import NemotronHConfig, NemotronHForCausalLM
    cfg = NemotronHConfig(hidden_size=128, num_hidden_layers=3, mamba_num_heads=8, mamba_head_dim=80,
                          ssm_state_size=128, n_groups=2, vocab_size=100, hybrid_override_pattern="M*M",
                          num_attention_heads=4, num_key_value_heads=2, head_dim=32, chunk_size=128)
    torch.manual_seed(seed)
    model = NemotronHForCausalLM(cfg).to(torch.bfloat16).eval()
    Rs = GD.MG.hf_rotations(model, seed)
    for m, R in zip([m for m in model.modules() if type(m).__name__ == "NemotronHMamba2Mixer"], Rs):
        m.act = RotAct(m.act, m.intermediate_size, m.n_groups, m.ssm_state_size, R)
    return model.cuda()


def test_hf_lean_prefill_matches_torch_prefill():
    """install(lean_prefill=1) runs the chunk scan for the prompt; on a one-chunk prompt (where
    transformers' torch prefill is the exact recurrence) its logits agree with
    install(lean_prefill=0) to the bf16 rounding of the two prefills, and the tiered pool holds
    the scan's final state."""
    from nested_ssm_b200 import materialize
    from nested_ssm_b200.hf import install
    g = torch.Generator().manual_seed(21)
    ids = torch.randint(0, 100, (2, 100), generator=g).cuda()
    outs = {}
    for lean in (1, 0):
        model = _bf16_model(16)
        install(model, pb=32, c=4, cold_bf16=0, lean_prefill=lean)
        with torch.no_grad():
            out = model.generate(ids, max_new_tokens=3, do_sample=False, output_logits=True,
                                 return_dict_in_generate=True, past_key_values=None)
        outs[lean] = torch.stack(out.logits).float().cpu()
        if lean:
            mixers = [m for m in model.modules() if type(m).__name__ == "NemotronHMamba2Mixer"]
            for m in mixers:
                assert m._nssm["pool"] is not None
    a, b = outs[1][0], outs[0][0]   # the logits of the prefill step
    err = float((a - b).abs().max())
    assert err <= 3e-2 * float(b.abs().max()) + 3e-2, f"lean vs torch prefill logits differ by {err}"


def test_hf_lean_prefill_multi_chunk_runs():
    """A 300-token prompt (three chunks) through the lean prefill: finite logits and the pool's
    materialised state equals the fp32 state the scan left in the cache (fp32 cold)."""
    from nested_ssm_b200 import materialize
    from nested_ssm_b200.hf import install
    g = torch.Generator().manual_seed(22)
    ids = torch.randint(0, 100, (2, 300), generator=g).cuda()
    model = _bf16_model(17)
    install(model, pb=32, c=4, cold_bf16=0, lean_prefill=1)
    captured = {}
    mixers = [m for m in model.modules() if type(m).__name__ == "NemotronHMamba2Mixer"]
    for m in mixers:
        def hook(mod, args, kwargs, out, m=m):
            cache = kwargs.get("cache_params", args[1] if len(args) > 1 else None)
            if cache is not None and m._nssm["pool"] is not None and m.layer_idx not in captured:
                captured[m.layer_idx] = cache.layers[m.layer_idx].recurrent_states.float().clone()
        m.register_forward_hook(hook, with_kwargs=True)
    with torch.no_grad():
        out = model(ids, use_cache=True)
    assert torch.isfinite(out.logits.float()).all()
    for m in mixers:
        st = m._nssm
        full = materialize(st["pool"], 0, st["slots"], -torch.exp(m.A_log.float()))
        torch.cuda.synchronize()
        torch.testing.assert_close(full.cpu(), captured[m.layer_idx].cpu(), rtol=0, atol=0)


def test_hf_hot_only_draft_install():
    """install(cold="off"), the reference's hot-only draft model (scale/v4_fused_decode.py:
    140-142): every decode token goes through the draft kernel, and its mixer outputs are those
    of the tiered install in mode coldoff (the same hot evolution and hot-only readout,
    scale/v4_native_decode.py:118-127) to fp32 rounding of the readout."""
    from nested_ssm_b200.hf import install
    d = GD.load("hf_generate.npz")
    cfg = GD.MG.HF
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    outs = []
    for kw in (dict(cold="off"), dict(cold="fp32", coldoff=1)):
        model = GD.MG.hf_model(cfg["seed"])
        Rs = GD.MG.hf_rotations(model, cfg["seed"])
        mixers = [m for m in model.modules() if type(m).__name__ == "NemotronHMamba2Mixer"]
        for m, R in zip(mixers, Rs):
            m.act = RotAct(m.act, m.intermediate_size, m.n_groups, m.ssm_state_size, R)
        model = model.cuda()
        install(model, pb=cfg["pb"], c=cfg["c"], **kw)
        mo = _mixer_decode_outputs(mixers)
        with torch.no_grad():
            out = model.generate(d["ids"].cuda(), max_new_tokens=cfg["new"], do_sample=False)
        outs.append((out.cpu(), mo, mixers))
    (seq_d, mo_d, mix_d), (seq_c, mo_c, _) = outs
    assert torch.equal(seq_d, seq_c)
    for a, b in zip(mo_d, mo_c):
        for ya, yb in zip(a, b):
            torch.testing.assert_close(ya, yb, rtol=1e-3, atol=1e-4)
    for m in mix_d:   # the draft kernel ran and the pool's bookkeeping never moved
        assert m._nssm["draft"] is not None and int(m._nssm["pool"].t[0].max()) == 0
