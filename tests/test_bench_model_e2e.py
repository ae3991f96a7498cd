"""The end-to-end model leg of bench.py (a reduced BASELINE config 4) on the CPU: the 9B
architecture it builds, and its generate-timing harness on a tiny model of the same layout
through the reference's own install and transformers' decode (the tiered arm needs a GPU)."""
import collections
import os
import types

import pytest
import torch

import bench


def test_nemotron_h_9b_architecture():
    m = bench.nemotron_h_9b("meta")
    kinds = collections.Counter(type(layer.mixer).__name__ for layer in m.model.layers)
    assert kinds == {"NemotronHMamba2Mixer": 27, "NemotronHMLP": 25, "NemotronHAttention": 4}
    mx = next(x for x in m.modules() if type(x).__name__ == "NemotronHMamba2Mixer")
    assert (mx.num_heads, mx.head_dim, mx.ssm_state_size, mx.n_groups, mx.conv_kernel_size) == (128, 80, 128, 8, 4)
    mlp = next(x for x in m.modules() if type(x).__name__ == "NemotronHMLP")
    assert mlp.up_proj.weight.shape == (15680, 4480)
    assert abs(sum(p.numel() for p in m.parameters()) / 1e9 - 8.888) < 0.01


def _tiny(device):
    from transformers import NemotronHConfig, NemotronHForCausalLM
    from transformers.models.nemotron_h import modeling_nemotron_h as MH
    kinds = {"M": "mamba", "*": "attention", "-": "moe"}
    cfg = NemotronHConfig(hidden_size=64, layers_block_type=[kinds[c] for c in "M-M*-M"], num_hidden_layers=6,
                          mamba_num_heads=8, mamba_head_dim=16, ssm_state_size=16, n_groups=2, conv_kernel=4,
                          expand=2, intermediate_size=96, mlp_hidden_act="relu2", num_attention_heads=4,
                          num_key_value_heads=2, head_dim=16, vocab_size=40000, chunk_size=8,
                          initializer_range=0.02)
    saved = MH.MIXER_TYPES["moe"]
    MH.MIXER_TYPES["moe"] = lambda config, layer_idx=None: MH.NemotronHMLP(config)
    try:
        with torch.device(device):
            return NemotronHForCausalLM(cfg).float().eval()
    finally:
        MH.MIXER_TYPES["moe"] = saved


@pytest.mark.skipif(not os.path.exists(os.path.join(bench.REF_DIR, "v4_native_decode.py")),
                    reason="baseline/_ref is not installed")
def test_model_e2e_harness_on_cpu():
    args = types.SimpleNamespace(model_batch=3, model_prompt=8, model_gen=3, model_arms="reference,hf")
    out = bench.model_e2e(args, device="cpu", build=_tiny)
    arms = out["arms"]
    assert set(arms) == {"reference", "hf"}
    for a in arms.values():
        assert a["decode_tokens_per_s"] > 0 and a["decode_ms_per_token"] > 0
    # the reference's bf16-cold tiered decode of an fp32 model picks the same greedy tokens here
    assert arms["reference"]["tokens_crc"] == arms["hf"]["tokens_crc"]


def test_vllm_leg_model_dir_and_shadow(tmp_path):
    """The serving-engine leg's pieces on the CPU: the 9B config as vLLM's own NemotronH config
    class reads it, and the shadow vllm package (file symlinks, the two patched sources) that
    the hooked arm imports; the installed package is left untouched."""
    pytest.importorskip("vllm")
    import importlib.util
    from nested_ssm_b200 import vllm_hook as VH
    from vllm.transformers_utils.configs.nemotron_h import NemotronHConfig
    d = bench.vllm_model_dir(str(tmp_path))
    cfg = NemotronHConfig.from_pretrained(d)
    assert cfg.hybrid_override_pattern == bench.NEMOTRON_9B_LAYOUT and cfg.mamba_head_dim == 80
    top = bench.vllm_shadow(str(tmp_path))
    src = os.path.dirname(importlib.util.find_spec("vllm").origin)
    for rel, marks in ((VH.MIXER, 5), (VH.NEMOTRON, 2)):
        path = os.path.join(top, "vllm", rel)
        assert not os.path.islink(path)
        text = open(path).read()
        assert text.count("[nested_ssm]") >= marks
        assert "[nested_ssm]" not in open(os.path.join(src, rel)).read()
    assert os.path.islink(os.path.join(top, "vllm", "__init__.py"))
    assert "_nssm.apply_ckpt(self)  # [nested_ssm] dummy weights" in open(os.path.join(top, "vllm", VH.NEMOTRON)).read()
