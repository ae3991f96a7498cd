"""The vLLM hook on the GPU: the calls the installed anchors make inside MambaMixer2 (prefill
after vLLM wrote the final states, then decode in place of selective_state_update) on a mixer
stand-in with vLLM's attribute names, against the oracle with vLLM's semantics (no dt clamp,
padded decode rows on NULL_BLOCK_ID = 0), per step from identical state across a flush.
Reference: scale/vllm_v4_patch.py:123-179 (prefill_snapshot / decode_readout)."""
import types

import pytest
import torch

import oracle as O
from tests import _helpers as Hh

pytestmark = pytest.mark.gpu


def test_vllm_hook_prefill_and_decode_match_oracle(monkeypatch):
    """vLLM 0.22 addresses a Mamba layer's state by block id over its whole block pool: the
    hook maps the blocks of live sequences to compact pool slots.  Blocks here are spread over a
    pool of 40 blocks, the tiered pool has 8 slots, block 0 is vLLM's null block."""
    from nested_ssm_b200 import rot_flat
    from nested_ssm_b200 import vllm_hook as VH
    monkeypatch.setenv("NESTED_SSM_SLOTS", "8")
    H, P, N, G, pb, c, NB = 128, 80, 128, 8, 32, 4, 40
    case = Hh.make_case(b=6, S=8, pb=pb, c=c, cold="fp8", steps=2 * c + 1, seed=31)
    prm = case["prm"]
    blocks = torch.tensor([33, 7, 21, 9, 14, 38], dtype=torch.int32)
    mixer = types.SimpleNamespace(num_heads=H, head_dim=P, n_groups=G, ssm_state_size=N,
                                  A=prm["A"].cuda(), D=prm["D"].to(torch.bfloat16).cuda(),
                                  dt_bias=prm["dt_bias"].to(torch.bfloat16).cuda(),
                                  nssm=dict(pb=pb, c=c, cold="fp8", pool=None), nssm_R=prm["R"].cuda())
    ssm_state = torch.zeros(NB, H, P, N, device="cuda")
    ssm_state[blocks.long().cuda()] = case["state0"].cuda()              # vLLM's prefill write
    VH.prefill(mixer, ssm_state, blocks.cuda())
    gpool = mixer.nssm["pool"]
    assert gpool is not None and gpool.S == 8
    slots = mixer.nssm["map"][blocks.long().cuda()].cpu()                # compact pool slots
    assert sorted(slots.tolist()) == list(range(6))
    assert int((mixer.nssm["map"] >= 0).sum()) == 6
    opool = Hh.oracle_pool(case)
    O.prefill_split(opool, slots, case["state0"])
    Hh.compare_pool(gpool, opool, 0, slots, "fp8", max_ulp=0, max_ulp_frac=0.0)   # the split is exact
    # the oracle sees vLLM's parameter dtypes: D and dt_bias as stored (bf16), A fp32
    D32, db32 = mixer.D.float().cpu(), mixer.dt_bias.float().cpu()
    for s in range(case["xs"].shape[0]):
        bl, sl = blocks.clone(), slots.clone()
        if s % 3 == 1:
            bl[2], sl[2] = VH.NULL_BLOCK_ID, -1                          # a padded decode row
        x = case["xs"][s].reshape(6, H * P).cuda()
        dt = case["dts"][s].cuda()
        B = case["Bs"][s].reshape(6, G * N).cuda()
        C_ = case["Cs"][s].reshape(6, G * N).cuda()
        Br = rot_flat(B, mixer.nssm_R).reshape(6, G, N).cpu()            # what the hook's step rotates to
        Cr = rot_flat(C_, mixer.nssm_R).reshape(6, G, N).cpu()
        Hh.sync_oracle_from_gpu(gpool, opool)
        yo = O.tiered_step(opool, sl, case["xs"][s], case["dts"][s], Br, Cr, prm["A"], D32, db32, None)
        out = torch.zeros(6, H, P, device="cuda")
        bl_d = bl.cuda()
        VH.decode(mixer, ssm_state, x, dt, B.view(6, G, N), C_.view(6, G, N), bl_d, bl_d, out)
        torch.cuda.synchronize()
        yg = out.cpu()
        live = sl >= 0
        Hh.assert_y_close(yg[live], yo[live], f"step {s}")
        assert torch.all(yg[~live] == 0)
        Hh.compare_pool(gpool, opool, 0, slots, "fp8", max_ulp=1, max_ulp_frac=1e-4)
    gpool.check_status()
    # three new sequences with the pool full of mapped blocks: the blocks that are neither
    # decoding this step nor prefilling give their slots back
    new_blocks = torch.tensor([3, 5, 11], dtype=torch.int32, device="cuda")
    ssm_state[new_blocks.long()] = case["state0"][:3].cuda()
    VH.prefill(mixer, ssm_state, new_blocks, blocks[:4].cuda())        # blocks 33, 7, 21, 9 still decode
    m = mixer.nssm["map"]
    assert int(m[blocks.long().cuda()[4:]].max()) == -1                  # 14 and 38 finished: unmapped
    assert bool((m[blocks.long().cuda()[:4]] == slots[:4].cuda()).all())
    fresh = m[new_blocks.long()].cpu()
    assert int(fresh.min()) >= 0 and len(set(fresh.tolist()) | set(slots[:4].tolist())) == 7


def test_vllm_hook_refuses_prefix_caching():
    from nested_ssm_b200 import vllm_hook as VH
    mixer = types.SimpleNamespace(num_heads=128, head_dim=80, n_groups=8, ssm_state_size=128,
                                  nssm=dict(pb=32, c=4, cold="fp8", pool=None), nssm_R=None)
    a = torch.zeros(2, dtype=torch.int32, device="cuda")
    b = torch.ones(2, dtype=torch.int32, device="cuda")
    with pytest.raises(NotImplementedError, match="prefix caching"):
        VH.decode(mixer, None, None, None, None, None, a, b, torch.zeros(2, 128, 80, device="cuda"))
