"""Generate the golden fixtures of tests/golden/ by running the REFERENCE's own Python
on the CPU (the fixtures are committed; this script is how they were made).

    python tests/golden/make_golden.py --reference <checkout of omin-Kwon/nested_ssm>

Three fixtures, all from seeded inputs that ``oracle.make_params`` / ``oracle.make_inputs``
regenerate (checksums stored beside the outputs):

* ``native_decode_fp32.npz`` -- ``_v4_decode`` of ``scale/v4_native_decode.py:26-172``
  (the HF NemotronH decode branch with the tiered readout), fp32 hot and cold, pb=32, c=4,
  modes stale / corr / coldoff.  It is driven through a stub mixer whose in_proj, act,
  norm and out_proj are identities and whose conv1d passes the newest column through,
  so its inputs are exactly the (x, rotated B, rotated C, dt_raw) the state op sees and
  its output is the pre-norm y.  Rotation: ``rot_flat`` of ``scale/vllm_v4_patch.py:41-45``
  called on fp32 B, C (the fp32 einsum of ``scale/v4_fused_decode.py:47-48``), cast to bf16.
* ``vllm_fp8.npz`` -- ``prefill_snapshot`` / ``decode_readout`` of
  ``scale/vllm_v4_patch.py:123-179`` with fp8 cold snapshots on a stub mixer; the fresh
  state update that vLLM's selective_state_update performs before the readout is done
  here in torch (softplus without clamp, as vLLM).
* ``rot_flat.npz`` -- ``rot_flat`` on bf16 input (the bf16 einsum of ActRotMask) and on
  fp32 input.
* ``native_decode_conv.npz`` -- ``_v4_decode`` again, now with a real conv1d (weights, bias,
  a conv state advanced by the transformers cache roll) and the reference's own
  ``ActRotMask`` (``scale/nemotron_retrofit.py:18-54``: SiLU, then the rotation of B and C)
  as the activation, so y covers conv + SiLU + split + rotation + tiered state op.
* ``prefill_hf.npz`` -- the reference's prefill dispatch (``_dispatch`` of
  ``scale/v4_native_decode.py:223-244`` with ``lean_prefill=0``, i.e. transformers' NemotronH
  ``torch_forward`` chunked SSD prefill) on a stub mixer whose in_proj, act, norm and
  out_proj are identities and whose conv1d is a causal identity, so its inputs are the seeded
  (x, B, C, dt_raw) of a 100-token prompt (one ragged chunk of the 128-token chunking) and
  its outputs are the pre-norm y and the final recurrent state the tiered pool is split from.
  One chunk only: transformers 5.5's ``torch_forward`` sums its chunk-decay matrix over the
  wrong index, so for prompts longer than a chunk its carried state is not the recurrence's
  (its final state is the last chunk's local state); the reference's default prefill
  (``lean_prefill=1``, mamba_ssm's ``mamba_chunk_scan_combined``) has no such step.
* ``hf_generate.npz`` -- the reference's HF integration end to end: a small random NemotronH
  (two Mamba2 layers and one attention layer, seeded), its mixers' activation wrapped in the
  reference's ``ActRotMask`` with seeded rotations, ``install(model, pb=32, c=4,
  cold_bf16=0)`` (``scale/v4_native_decode.py:247-256``, the HF torch prefill), then greedy
  ``generate``: the tokens and the logits of every step.
* ``hf_generate_width.npz`` -- the same model and prompt with the state term made dominant
  (``hf_state_dominant``) and the rotated B and C masked to their first 64 coordinates
  (``set_width(model, 64)``, ``scale/nemotron_retrofit.py:112-114``; ``ActRotMask._mask``
  zeroes the coordinates at and past the width).  Both HF fixtures also hold every mixer's
  output at every decode step.
"""
from __future__ import annotations

import argparse
import math
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

import oracle as O  # noqa: E402

# fixture shapes (small enough to commit, real headdim / d_state / hot width)
NATIVE = dict(b=2, H=16, P=80, N=128, G=2, pb=32, c=4, seed=11, steps=13, steps_modes=9)
VLLM = dict(b=2, S=4, H=8, P=80, N=128, G=2, pb=32, c=4, seed=12, steps=9, slots=[2, 0])
ROT = dict(T=6, G=2, N=128, seed=13)
CONV = dict(b=2, H=16, P=80, N=128, G=2, pb=32, c=4, seed=14, steps=9, K=4)
HF = dict(b=2, prompt=7, new=9, seed=15, pb=32, c=4)
HF_WIDTH = 64
PREFILL = dict(b=2, T=100, H=4, P=80, N=128, G=2, chunk=128, seed=16)


def hf_model(seed: int):
    """The small NemotronH of hf_generate.npz (fp32, CPU), built from its seed."""
    from transformers import NemotronHConfig, NemotronHForCausalLM
    cfg = NemotronHConfig(hidden_size=64, num_hidden_layers=3, mamba_num_heads=8, mamba_head_dim=32,
                          ssm_state_size=128, n_groups=2, vocab_size=100, hybrid_override_pattern="M*M",
                          num_attention_heads=4, num_key_value_heads=2, head_dim=16)
    torch.manual_seed(seed)
    return NemotronHForCausalLM(cfg).float().eval()


def hf_state_dominant(model):
    """Make the state term dominate the mixers' output (D = 0, dt = softplus(dt_raw + 1)): in
    the randomly initialised model the D x skip and the small initial dt leave the state op's
    share of the mixer output near 1e-5, too little for a fixture to tell masks apart."""
    for m in model.modules():
        if type(m).__name__ == "NemotronHMamba2Mixer":
            m.D.data.zero_()
            m.dt_bias.data.fill_(1.0)
    return model


def hf_rotations(model, seed: int):
    """Seeded per-group orthogonal rotations, one per Mamba2 mixer."""
    g = torch.Generator().manual_seed(seed + 1)
    out = []
    for m in model.modules():
        if type(m).__name__ == "NemotronHMamba2Mixer":
            out.append(torch.linalg.qr(torch.randn(m.n_groups, m.ssm_state_size, m.ssm_state_size, generator=g))[0])
    return out


def state0(b, H, P, N, seed):
    g = torch.Generator().manual_seed(seed + 7)
    return torch.randn(b, H, P, N, generator=g) * math.sqrt(0.1)


def checksum(t: torch.Tensor) -> float:
    return float(t.double().sum())


def _conv_cache(conv_dim, K=4):
    """Stub cache: update_conv_state returns the new column at the newest tap only."""
    cache = types.SimpleNamespace()

    def update_conv_state(hs, idx):          # hs [b, conv_dim, 1]
        b = hs.shape[0]
        st = torch.zeros(b, conv_dim, K, dtype=hs.dtype)
        st[..., -1] = hs[..., -1]
        return st

    def update_recurrent_state(s, idx):
        cache.layers[idx].recurrent_states = s
        return s

    cache.update_conv_state = update_conv_state
    cache.update_recurrent_state = update_recurrent_state
    return cache


def run_native(V, rot_flat, cfg, mode):
    b, H, P, N, G, pb, c, seed = (cfg[k] for k in ("b", "H", "P", "N", "G", "pb", "c", "seed"))
    steps = cfg["steps"] if mode == "stale" else cfg["steps_modes"]
    prm = O.make_params(H, G, N, seed=seed)[0]
    xs, dts, Bs, Cs = O.make_inputs(b, H, P, G, N, steps, seed=seed, io_dtype=torch.bfloat16)
    s0 = state0(b, H, P, N, seed)
    A_log = torch.log(-prm["A"])
    A = -torch.exp(A_log.float())                       # what the mixer computes
    K = 4
    I, conv_dim = H * P, H * P + 2 * G * N
    m = types.SimpleNamespace(
        num_heads=H, head_dim=P, ssm_state_size=N, n_groups=G, intermediate_size=I,
        conv_dim=conv_dim, in_proj=torch.nn.Identity(), act=torch.nn.Identity(),
        use_conv_bias=False, A_log=A_log, D=prm["D"], dt_bias=prm["dt_bias"],
        time_step_min=1e-3, layer_idx=0, out_proj=torch.nn.Identity(),
        norm=lambda y, gate: y,
        v4cfg=dict(pb=pb, c=c, cold_bf16=0, corr=int(mode == "corr"), coldoff=int(mode == "coldoff")))
    w = torch.zeros(conv_dim, 1, K)
    w[:, 0, -1] = 1.0
    m.conv1d = types.SimpleNamespace(weight=w, bias=torch.zeros(conv_dim))
    m._v4state = {"snap": s0[..., pb:].clone(), "glog": torch.zeros(b, H, P), "t": 0,
                  "bufB": [], "bufX": [], "bufG": []}
    cache = _conv_cache(conv_dim, K)
    cache.layers = [types.SimpleNamespace(recurrent_states=s0.clone())]
    ys, Brs, Crs = [], [], []
    for s in range(steps):
        Br = rot_flat(Bs[s].reshape(b, G * N).float(), prm["R"]).to(torch.bfloat16)
        Cr = rot_flat(Cs[s].reshape(b, G * N).float(), prm["R"]).to(torch.bfloat16)
        Brs.append(Br.reshape(b, G, N))
        Crs.append(Cr.reshape(b, G, N))
        gate = torch.zeros(b, I)
        proj = torch.cat([gate, xs[s].float().reshape(b, I), Br.float(), Cr.float(),
                          dts[s].float()], dim=-1)[:, None, :]
        y = V._v4_decode(m, proj, cache, None)
        ys.append(y.reshape(b, H, P).float())
    out = dict(y=torch.stack(ys), Br=torch.stack(Brs), Cr=torch.stack(Crs))   # B', C' bf16 (stored as int16 bits)
    if mode == "stale":
        out["state_final_h0_h9"] = cache.layers[0].recurrent_states[:, [0, 9]].float()
    out["t_final"] = torch.tensor(m._v4state["t"])
    meta = dict(x=checksum(xs), dt=checksum(dts), B=checksum(Bs), C=checksum(Cs), s0=checksum(s0))
    return out, prm, A, meta


def make_native(ref):
    sys.path.insert(0, os.path.join(ref, "scale"))
    import v4_native_decode as V
    import vllm_v4_patch as VP
    arrays = {}
    for mode in ("stale", "corr", "coldoff"):
        out, prm, A, meta = run_native(V, VP.rot_flat, NATIVE, mode)
        for k, v in out.items():
            arrays[f"{mode}_{k}"] = v
        for k, v in meta.items():
            arrays[f"{mode}_sum_{k}"] = torch.tensor(v, dtype=torch.float64)
    arrays["R"] = prm["R"]
    arrays["A"] = A
    arrays["D"] = prm["D"]
    arrays["dt_bias"] = prm["dt_bias"]
    return arrays


def make_vllm(ref):
    sys.path.insert(0, os.path.join(ref, "scale"))
    import vllm_v4_patch as VP
    cfg = VLLM
    b, S, H, P, N, G, pb, c, seed = (cfg[k] for k in ("b", "S", "H", "P", "N", "G", "pb", "c", "seed"))
    steps = cfg["steps"]
    slots = torch.tensor(cfg["slots"])
    prm = O.make_params(H, G, N, seed=seed)[0]
    xs, dts, Bs, Cs = O.make_inputs(b, H, P, G, N, steps, seed=seed, io_dtype=torch.bfloat16)
    s0 = state0(b, H, P, N, seed)
    mixer = types.SimpleNamespace(v4cfg=dict(pb=pb, c=c, cold="fp8"), _v4buf=None, num_heads=H,
                                  D=prm["D"], dt_bias=prm["dt_bias"], A=prm["A"])
    ssm = torch.zeros(S, H, P, N)
    ssm[slots] = s0
    VP.prefill_snapshot(mixer, ssm, slots)
    buf = mixer._v4buf
    arrays = dict(pre_codes=buf["snap"][slots].view(torch.uint8).clone(),
                  pre_scale=buf["scale"][slots][..., 0].clone())
    ys, ts, glogs, flush_codes, flush_scale = [], [], [], [], []
    HG = H // G
    for s in range(steps):
        # the fresh update selective_state_update performs before decode_readout (no dt clamp)
        dt = torch.nn.functional.softplus(dts[s].float() + prm["dt_bias"].view(1, -1))
        dA = dt * prm["A"].view(1, -1)
        Bh = Bs[s].float().repeat_interleave(HG, dim=1)
        x = xs[s].float()
        st = ssm[slots]
        st = st * torch.exp(dA)[:, :, None, None] + (dt[:, :, None, None] * Bh[:, :, None, :]) * x[..., None]
        ssm[slots] = st
        out = torch.zeros(b, H, P)
        VP.decode_readout(mixer, ssm, out, xs[s], dts[s], Cs[s], slots)
        ys.append(out.clone())
        ts.append(buf["t"][slots].clone())
        glogs.append(buf["glog"][slots].clone())
        if (s + 1) % c == 0:
            flush_codes.append(buf["snap"][slots].view(torch.uint8).clone())
            flush_scale.append(buf["scale"][slots][..., 0].clone())
    arrays.update(y=torch.stack(ys), t=torch.stack(ts), glog=torch.stack(glogs),
                  flush_codes=torch.stack(flush_codes), flush_scale=torch.stack(flush_scale),
                  A=prm["A"], D=prm["D"], dt_bias=prm["dt_bias"])
    for k, v in dict(x=xs, dt=dts, B=Bs, C=Cs, s0=s0).items():
        arrays[f"sum_{k}"] = torch.tensor(checksum(v), dtype=torch.float64)
    return arrays


def make_rot(ref):
    sys.path.insert(0, os.path.join(ref, "scale"))
    import vllm_v4_patch as VP
    T, G, N, seed = ROT["T"], ROT["G"], ROT["N"], ROT["seed"]
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(T, G * N, generator=g) / math.sqrt(N)).to(torch.bfloat16)
    R = torch.linalg.qr(torch.randn(G, N, N, generator=g))[0].contiguous().float()
    return dict(x=x.view(torch.int16), R=R, out_bf16=VP.rot_flat(x, R).view(torch.int16),
                out_fp32=VP.rot_flat(x.float(), R))


def conv_inputs(cfg):
    """Seeded conv-step inputs (bf16-representable values held in fp32)."""
    b, H, P, N, G, K, seed, steps = (cfg[k] for k in ("b", "H", "P", "N", "G", "K", "seed", "steps"))
    D = H * P + 2 * G * N
    g = torch.Generator().manual_seed(seed + 100)
    bf = lambda t: t.to(torch.bfloat16).float()   # noqa: E731
    return dict(
        xbc=bf(torch.randn(steps, b, D, generator=g)),
        dts=bf(torch.randn(steps, b, H, generator=g)),
        state=bf(torch.randn(b, D, K, generator=g) * 0.5),
        weight=bf(torch.rand(D, 1, K, generator=g) - 0.5),
        bias=bf(torch.randn(D, generator=g) * 0.1),
        s0=state0(b, H, P, N, seed))


def make_native_conv(ref):
    sys.path.insert(0, os.path.join(ref, "scale"))
    import v4_native_decode as V
    import nemotron_retrofit as NR
    cfg = CONV
    b, H, P, N, G, pb, c, seed, K = (cfg[k] for k in ("b", "H", "P", "N", "G", "pb", "c", "seed", "K"))
    prm = O.make_params(H, G, N, seed=seed)[0]
    inp = conv_inputs(cfg)
    I = H * P
    D = I + 2 * G * N
    A_log = torch.log(-prm["A"])
    act = NR.ActRotMask(torch.nn.SiLU(), I, G, N)
    act.R.data.copy_(prm["R"])
    m = types.SimpleNamespace(
        num_heads=H, head_dim=P, ssm_state_size=N, n_groups=G, intermediate_size=I, conv_dim=D,
        in_proj=torch.nn.Identity(), act=act, use_conv_bias=True, A_log=A_log, D=prm["D"],
        dt_bias=prm["dt_bias"], time_step_min=1e-3, layer_idx=0, out_proj=torch.nn.Identity(),
        norm=lambda y, gate: y, v4cfg=dict(pb=pb, c=c, cold_bf16=0, corr=0, coldoff=0))
    m.conv1d = types.SimpleNamespace(weight=inp["weight"], bias=inp["bias"])
    m._v4state = {"snap": inp["s0"][..., pb:].clone(), "glog": torch.zeros(b, H, P), "t": 0,
                  "bufB": [], "bufX": [], "bufG": []}
    cache = types.SimpleNamespace()
    cache.conv = inp["state"].clone()

    def update_conv_state(hs, idx):   # the transformers cache's decode update: roll, append
        st = cache.conv.roll(shifts=-1, dims=-1)
        st[:, :, -1:] = hs
        cache.conv = st
        return st

    def update_recurrent_state(s_, idx):
        cache.layers[idx].recurrent_states = s_
        return s_

    cache.update_conv_state = update_conv_state
    cache.update_recurrent_state = update_recurrent_state
    cache.layers = [types.SimpleNamespace(recurrent_states=inp["s0"].clone())]
    ys = []
    for s in range(cfg["steps"]):
        proj = torch.cat([torch.zeros(b, I), inp["xbc"][s], inp["dts"][s]], dim=-1)[:, None, :]
        ys.append(V._v4_decode(m, proj, cache, None).reshape(b, H, P).float())
    arrays = dict(y=torch.stack(ys), conv_state_final=cache.conv.clone(),
                  state_final_h0_h9=cache.layers[0].recurrent_states[:, [0, 9]].float(),
                  R=prm["R"], A=-torch.exp(A_log.float()), D=prm["D"], dt_bias=prm["dt_bias"])
    for k in ("xbc", "dts", "state", "weight", "bias", "s0"):
        arrays[f"sum_{k}"] = torch.tensor(checksum(inp[k]), dtype=torch.float64)
    return arrays


def prefill_inputs(cfg):
    """Seeded prefill inputs, bf16-representable values held in fp32: x ~ N(0,1),
    B, C ~ N(0,1) / N**0.25 (so C.B is O(1)), dt_raw ~ N(0,1); A, D, dt_bias of make_params."""
    b, T, H, P, N, G, seed = (cfg[k] for k in ("b", "T", "H", "P", "N", "G", "seed"))
    prm = O.make_params(H, G, N, seed=seed)[0]
    g = torch.Generator().manual_seed(seed + 200)
    bf = lambda t: t.to(torch.bfloat16).float()   # noqa: E731
    return dict(x=bf(torch.randn(b, T, H, P, generator=g)),
                B=bf(torch.randn(b, T, G, N, generator=g) / N ** 0.25),
                C=bf(torch.randn(b, T, G, N, generator=g) / N ** 0.25),
                dt=bf(torch.randn(b, T, H, generator=g)),
                A=-torch.exp(torch.log(-prm["A"]).float()), D=prm["D"], dt_bias=prm["dt_bias"],
                A_log=torch.log(-prm["A"]))


def make_prefill(ref):
    sys.path.insert(0, os.path.join(ref, "scale"))
    import v4_native_decode as V
    cfg = PREFILL
    b, T, H, P, N, G, Q = (cfg[k] for k in ("b", "T", "H", "P", "N", "G", "chunk"))
    inp = prefill_inputs(cfg)
    K = 4
    I, conv_dim = H * P, H * P + 2 * G * N
    conv = torch.nn.Conv1d(conv_dim, conv_dim, K, groups=conv_dim, padding=K - 1, bias=False)
    conv.weight.data.zero_()
    conv.weight.data[:, 0, -1] = 1.0                   # causal identity
    m = types.SimpleNamespace(
        num_heads=H, head_dim=P, ssm_state_size=N, n_groups=G, intermediate_size=I, conv_dim=conv_dim,
        conv_kernel_size=K, chunk_size=Q, in_proj=torch.nn.Identity(), act=torch.nn.Identity(), conv1d=conv,
        use_conv_bias=False, A_log=inp["A_log"], D=inp["D"], dt_bias=inp["dt_bias"], time_step_min=1e-3,
        time_step_limit=(0.0, float("inf")), layer_idx=0, out_proj=torch.nn.Identity(),
        norm=lambda y, gate: y, _v4state=None, v4cfg=dict(pb=32, c=4, cold_bf16=0, lean_prefill=0))
    cache = types.SimpleNamespace(layers=[types.SimpleNamespace(recurrent_states=None)])
    cache.has_previous_state = lambda idx: False
    cache.update_conv_state = lambda st, idx: st

    def update_recurrent_state(s, idx):
        cache.layers[idx].recurrent_states = s
        return s

    cache.update_recurrent_state = update_recurrent_state
    proj = torch.cat([torch.zeros(b, T, I), inp["x"].reshape(b, T, I), inp["B"].reshape(b, T, G * N),
                      inp["C"].reshape(b, T, G * N), inp["dt"]], dim=-1)
    y = V._dispatch(m, proj, cache, None)
    out = dict(y=y.reshape(b, T, H, P).float(), state=cache.layers[0].recurrent_states.float())
    for k in ("x", "B", "C", "dt"):
        out[f"sum_{k}"] = torch.tensor(checksum(inp[k]), dtype=torch.float64)
    return out


def make_hf(ref, width=None):
    sys.path.insert(0, os.path.join(ref, "scale"))
    import v4_native_decode as V
    import nemotron_retrofit as NR
    cfg = HF
    model = hf_model(cfg["seed"])
    if width is not None:
        hf_state_dominant(model)
    Rs = hf_rotations(model, cfg["seed"])
    mixers = [m for m in model.modules() if type(m).__name__ == "NemotronHMamba2Mixer"]
    for m, R in zip(mixers, Rs):
        act = NR.ActRotMask(m.act, m.intermediate_size, m.n_groups, m.ssm_state_size)
        act.R.data.copy_(R)
        m.act = act
    if width is not None:
        NR.set_width(model, width)
    V.install(model, pb=cfg["pb"], c=cfg["c"], cold_bf16=0)
    for m in mixers:
        m.v4cfg["lean_prefill"] = 0          # the HF torch prefill (no fused kernels on CPU)
    g = torch.Generator().manual_seed(cfg["seed"] + 2)
    ids = torch.randint(0, 100, (cfg["b"], cfg["prompt"]), generator=g)
    outs = mixer_decode_outputs(mixers)
    out = model.generate(ids, max_new_tokens=cfg["new"], do_sample=False, output_logits=True,
                         return_dict_in_generate=True)
    return dict(ids=ids, tokens=out.sequences, logits=torch.stack(out.logits).float(),
                mixer_out=torch.stack([torch.stack(o) for o in outs]).float())


def mixer_decode_outputs(mixers):
    """Forward hooks recording every one-token call's output of each mixer (the decode steps):
    the mixer output is far more sensitive to the state op than the logits of a random model."""
    outs = [[] for _ in mixers]
    for i, m in enumerate(mixers):
        def hook(mod, args, out, i=i):
            if out.shape[1] == 1:
                outs[i].append(out.detach().clone())
        m.register_forward_hook(hook)
    return outs


def save(name, arrays):
    np_arrays = {k: (v.view(torch.int16) if v.dtype == torch.bfloat16 else v).numpy() for k, v in arrays.items()}
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **np_arrays)
    print(f"wrote {path} ({os.path.getsize(path) / 1024:.0f} KiB)")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of omin-Kwon/nested_ssm")
    ap.add_argument("--only", nargs="*", default=None, help="fixture file names to (re)make")
    a = ap.parse_args()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    ref = a.reference
    makers = {
        "native_decode_fp32.npz": lambda: make_native(ref),
        "vllm_fp8.npz": lambda: make_vllm(ref),
        "rot_flat.npz": lambda: make_rot(ref),
        "native_decode_conv.npz": lambda: make_native_conv(ref),
        "hf_generate.npz": lambda: make_hf(ref),
        "hf_generate_width.npz": lambda: make_hf(ref, width=HF_WIDTH),
        "prefill_hf.npz": lambda: make_prefill(ref),
    }
    with torch.no_grad():
        for name, make in makers.items():
            if a.only is None or name in a.only:
                save(name, make())


if __name__ == "__main__":
    main()
