"""The vLLM hook's host side on the CPU: the NESTED_SSM_* configuration, the rotation
checkpoint loader, apply_ckpt on a model's MambaMixer2 modules, and the anchored installer run
against copies of the installed vLLM 0.22 sources (the reference's five anchors,
scale/install_vllm_v4.sh:27-107; the installed package itself is never touched)."""
import os
import py_compile
import shutil

import pytest
import torch

from nested_ssm_b200 import vllm_hook as VH


def test_config_from_env_defaults_and_errors():
    assert VH.config_from_env({}) is None
    cfg = VH.config_from_env({"NESTED_SSM_CKPT": "r.pt"})
    assert cfg == dict(ckpt="r.pt", mode="fresh", pb=32, c=4, cold="bf16", readout="stale")   # vllm_v4_patch.py:28-38
    cfg = VH.config_from_env({"NESTED_SSM_CKPT": "r.pt", "NESTED_SSM_MODE": "v4", "NESTED_SSM_PB": "16",
                              "NESTED_SSM_C": "8", "NESTED_SSM_COLD": "fp8", "NESTED_SSM_READOUT": "corr"})
    assert cfg == dict(ckpt="r.pt", mode="v4", pb=16, c=8, cold="fp8", readout="corr")
    for bad in ({"NESTED_SSM_MODE": "v5"}, {"NESTED_SSM_COLD": "fp4"}, {"NESTED_SSM_C": "0"},
                {"NESTED_SSM_READOUT": "exact"}):
        with pytest.raises(ValueError):
            VH.config_from_env({"NESTED_SSM_CKPT": "r.pt", **bad})


def _ckpt(tmp_path, L=3, G=2, N=8, decay=True, extra=None):
    g = torch.Generator().manual_seed(0)
    d = {i: torch.linalg.qr(torch.randn(G, N, N, generator=g))[0] for i in range(L)}
    if decay:
        d["decay"] = {"A_log": [torch.rand(4, generator=g) for _ in range(L)],
                      "dt_bias": [torch.randn(4, generator=g) for _ in range(L)]}
    d.update(extra or {})
    path = os.path.join(str(tmp_path), "rot.pt")
    torch.save(d, path)
    return path, d


def test_load_ckpt_reads_rotations_and_decay(tmp_path):
    path, d = _ckpt(tmp_path)
    Rs, decay = VH.load_ckpt(path, num_mixers=3, ngroups=2, dstate=8)
    assert len(Rs) == 3 and all(torch.equal(Rs[i], d[i].float()) for i in range(3))
    assert torch.equal(decay["A_log"][1], d["decay"]["A_log"][1])
    with pytest.raises(ValueError, match="3 rotations for 4"):
        VH.load_ckpt(path, num_mixers=4)
    with pytest.raises(ValueError, match="needs"):
        VH.load_ckpt(path, ngroups=4)
    path2, _ = _ckpt(tmp_path, decay=False, extra={5: torch.eye(8)[None]})
    with pytest.raises(ValueError, match="0..L-1"):
        VH.load_ckpt(path2)


class MambaMixer2(torch.nn.Module):
    """Stand-in with the attributes apply_ckpt reads (class name as vLLM's)."""

    def __init__(self, H=4, G=2, N=8):
        super().__init__()
        self.A = torch.nn.Parameter(-torch.ones(H))
        self.dt_bias = torch.nn.Parameter(torch.zeros(H))
        self.n_groups, self.ssm_state_size, self.tp_size, self.num_spec = G, N, 1, 0
        self.nssm = None
        self.nssm_R = None


def test_apply_ckpt_sets_rotation_decay_and_mode(tmp_path):
    path, d = _ckpt(tmp_path)
    model = torch.nn.Sequential(MambaMixer2(), torch.nn.Linear(2, 2), MambaMixer2(), MambaMixer2())
    assert VH.apply_ckpt(model, {}) == 0
    assert VH.apply_ckpt(model, {"NESTED_SSM_CKPT": path}) == 3
    mixers = [model[0], model[2], model[3]]
    for i, m in enumerate(mixers):
        assert torch.equal(m.nssm_R, d[i].float())
        torch.testing.assert_close(m.A.data, -torch.exp(d["decay"]["A_log"][i]))
        assert torch.equal(m.dt_bias.data, d["decay"]["dt_bias"][i])
        assert m.nssm is None                                     # fresh mode: R only
    VH.apply_ckpt(model, {"NESTED_SSM_CKPT": path, "NESTED_SSM_MODE": "v4", "NESTED_SSM_COLD": "fp8"})
    st = dict(mixers[1].nssm)
    assert st.pop("slots") > 0
    assert st == dict(pb=32, c=4, cold="fp8", readout="stale", pool=None)


def _vllm_copy(tmp_path):
    vllm = pytest.importorskip("vllm")
    src = os.path.dirname(vllm.__file__)
    dst = os.path.join(str(tmp_path), "vllm")
    for rel in (VH.MIXER, VH.NEMOTRON):
        os.makedirs(os.path.dirname(os.path.join(dst, rel)), exist_ok=True)
        shutil.copy(os.path.join(src, rel), os.path.join(dst, rel))
    return dst


def test_installer_patches_a_copy_of_vllm_idempotently(tmp_path):
    d = _vllm_copy(tmp_path)
    before = {rel: open(os.path.join(d, rel)).read() for rel in (VH.MIXER, VH.NEMOTRON)}
    assert VH.install(d, check_only=True) == []                   # every anchor present, nothing written
    changed = VH.install(d)
    assert len(changed) == 2
    mixer = open(os.path.join(d, VH.MIXER)).read()
    nem = open(os.path.join(d, VH.NEMOTRON)).read()
    for frel, how, anchor, text in VH.PATCHES:
        assert text in (mixer if frel == VH.MIXER else nem)
    assert mixer.count(VH.MARK) >= 5 and nem.count(VH.MARK) == 1
    assert "_nssm.decode(" in mixer and "                selective_state_update(" in mixer   # fallback kept
    for rel in (VH.MIXER, VH.NEMOTRON):
        py_compile.compile(os.path.join(d, rel), doraise=True)
    assert VH.install(d) == []                                    # idempotent
    assert open(os.path.join(d, VH.MIXER)).read() == mixer
    # removing the inserted lines gives the original source back (edits are additive)
    assert len(mixer) > len(before[VH.MIXER])


def test_installer_refuses_a_source_without_the_anchor():
    with pytest.raises(ValueError, match="anchor"):
        VH.patch_source("def f():\n    pass\n", "after", "missing anchor\n", "x = 1\n", "f.py")


def test_slot_map_assigns_reuses_and_reclaims():
    """The hook's block -> pool-slot map on the host: a block keeps its slot, a full map gives
    back the slots of blocks that neither decode nor prefill this step, and more live sequences
    than slots is an error."""
    m = VH.SlotMap(4)
    s1, freed = m.assign([10, 20, 30], [])
    assert len(set(s1)) == 3 and freed == []
    s2, _ = m.assign([20], [10, 30])                      # a block already mapped keeps its slot
    assert s2 == [s1[1]]
    s3, freed = m.assign([40, 50], [10])                  # one free slot, two needed: 20, 30 finished
    assert sorted(freed) == [20, 30] and len(set(s3)) == 2 and s1[0] not in s3
    with pytest.raises(RuntimeError, match="exceed"):
        m.assign([60, 70, 80], [10, 40, 50])


def test_slot_map_under_a_simulated_block_allocator():
    """Requests arrive and finish at random; each takes a free block id from a pool of 8x the
    slots (as vLLM 0.22's shared block pool does), prefills once and then decodes every step.
    Live sequences always hold distinct slots, a sequence's slot never changes while it lives,
    and the map never needs more slots than live sequences + the step's prefills."""
    import random
    rng = random.Random(3)
    cap, nblocks = 16, 128
    m = VH.SlotMap(cap)
    free_blocks = list(range(1, nblocks))          # block 0: vLLM's null block
    live = {}                                       # block -> slot given at its prefill
    for step in range(400):
        for k in [k for k in live if rng.random() < 0.1]:   # finished requests free their block
            del live[k]
            free_blocks.append(k)
        rng.shuffle(free_blocks)
        new = [free_blocks.pop() for _ in range(min(rng.randint(0, 4), cap - len(live)))]
        slots, _ = m.assign(new, list(live))
        for k, s in zip(new, slots):
            live[k] = s
        assert len(set(live.values())) == len(live) <= cap
        for k, s in live.items():
            assert m.of_block[k] == s
