"""vLLM integration: the tiered decode state op inside vLLM's ``MambaMixer2`` (vLLM 0.22).

Drop-in for the reference's vLLM hook (``scale/vllm_v4_patch.py``, installed by
``scale/install_vllm_v4.sh:27-107``), with the same configuration surface, so ``vllm serve``
stays stock and the mode is chosen by the environment (``scale/vllm_v4_patch.py:28-38``):

    NESTED_SSM_CKPT=<rotation checkpoint>   enables R (and the tuned decay, if stored)
    NESTED_SSM_MODE=fresh|v4                fresh: R only, vLLM's own state update;
                                            v4: the tiered decode state op (default fresh)
    NESTED_SSM_PB=32  NESTED_SSM_C=4        hot width and flush period
    NESTED_SSM_COLD=fp32|bf16|fp8           cold storage (default bf16)
    NESTED_SSM_READOUT=stale|corr|coldoff   v4 readout (default stale, the reference's; corr is
                                            the exact rank-c correction of
                                            scale/v4_native_decode.py:81-117, coldoff the
                                            hot-only readout; an extension of the reference's
                                            configuration)

Checkpoint (``scale/vllm_v4_patch.py:59-84``): ``torch.save``'d dict ``{i: R_i [G, N, N]}`` with
one rotation per Mamba2 mixer in model order, plus optionally ``"decay": {"A_log": [...],
"dt_bias": [...]}`` per mixer, which replaces the mixers' A (= -exp(A_log)) and dt_bias.

The hooks (``install`` puts calls to them into vLLM's source, at the reference's five anchors):

* ``__init__``: ``self.nssm = None`` (config and pool, set by ``apply_ckpt``), ``self.nssm_R``;
* prefill, after the split of the conv output: B and C rotated by R (fp32 accumulation);
* prefill, after vLLM wrote the final states: ``prefill`` splits them into the tiered pool
  (hot fp32 + cold in its storage dtype, t = 0, glog = 0);
* decode, after the split: the raw dt is kept; in v4 mode ``decode`` REPLACES vLLM's
  ``selective_state_update``: one tiered step (rotation of B and C, hot update, stale cold
  readout, ring write, rank-c flush every c tokens) writes y into vLLM's output buffer;
  in fresh mode B and C are rotated and vLLM's own update runs;
* ``NemotronHForCausalLM.load_weights`` ends with ``apply_ckpt(self)``.

Differences from the reference's hook, by design: the reference keeps vLLM's full fp32
state and only overrides the readout (its docstring calls that port accuracy-grade, "the speed
path lands separately"); here the state op itself is tiered, so vLLM's ``ssm_state`` is only
the prefill's output buffer and the decode reads and writes the tiered pool.  dt is not
clamped on decode (vLLM's form, semantic decision D1), padded decode rows carry vLLM's
``NULL_BLOCK_ID`` (0), prefix caching of Mamba states (``mamba_cache_mode="all"``),
speculative decoding and tensor parallelism > 1 are refused with an error.
"""
from __future__ import annotations

import argparse
import os
import py_compile
import sys

import torch

MARK = "[nested_ssm]"
NULL_BLOCK_ID = 0   # vllm/v1/attention/backends/utils.py:45 (padded decode entries)
_MODES = ("fresh", "v4")
_COLDS = ("fp32", "bf16", "fp8")
_READOUTS = ("stale", "corr", "coldoff")


# --------------------------------------------------------------------------
# configuration and checkpoint
# --------------------------------------------------------------------------
def config_from_env(env=None) -> dict | None:
    """The NESTED_SSM_* configuration (None when NESTED_SSM_CKPT is unset), with the
    reference's defaults (scale/vllm_v4_patch.py:28-38); bad values raise ValueError."""
    env = os.environ if env is None else env
    ck = env.get("NESTED_SSM_CKPT")
    if not ck:
        return None
    cfg = dict(ckpt=ck, mode=env.get("NESTED_SSM_MODE", "fresh"), pb=int(env.get("NESTED_SSM_PB", "32")),
               c=int(env.get("NESTED_SSM_C", "4")), cold=env.get("NESTED_SSM_COLD", "bf16"),
               readout=env.get("NESTED_SSM_READOUT", "stale"))
    if cfg["mode"] not in _MODES:
        raise ValueError(f"NESTED_SSM_MODE={cfg['mode']!r}: expected one of {_MODES}")
    if cfg["cold"] not in _COLDS:
        raise ValueError(f"NESTED_SSM_COLD={cfg['cold']!r}: expected one of {_COLDS}")
    if cfg["readout"] not in _READOUTS:
        raise ValueError(f"NESTED_SSM_READOUT={cfg['readout']!r}: expected one of {_READOUTS}")
    if cfg["c"] < 1 or cfg["pb"] < 1:
        raise ValueError("NESTED_SSM_C and NESTED_SSM_PB must be positive")
    return cfg


def load_ckpt(path: str, num_mixers: int | None = None, ngroups: int | None = None,
              dstate: int | None = None):
    """Read a rotation checkpoint: returns ``(Rs, decay)`` with ``Rs`` a list of fp32
    ``[G, N, N]`` tensors in mixer order and ``decay`` None or ``{"A_log": [...],
    "dt_bias": [...]}`` (fp32 per mixer).  Validates the keys, shapes and finiteness."""
    saved = torch.load(path, map_location="cpu", weights_only=False)
    if not isinstance(saved, dict):
        raise ValueError(f"{path}: expected a dict {{mixer index: R}}, got {type(saved).__name__}")
    idx = sorted(k for k in saved if isinstance(k, int))
    if not idx or idx != list(range(len(idx))):
        raise ValueError(f"{path}: rotation keys must be 0..L-1, got {idx[:8]}")
    if num_mixers is not None and len(idx) != num_mixers:
        raise ValueError(f"{path}: {len(idx)} rotations for {num_mixers} Mamba2 mixers")
    Rs = []
    for i in idx:
        R = torch.as_tensor(saved[i]).float()
        if R.dim() != 3 or R.shape[1] != R.shape[2]:
            raise ValueError(f"{path}: R[{i}] has shape {tuple(R.shape)}, expected [G, N, N]")
        if (ngroups is not None and R.shape[0] != ngroups) or (dstate is not None and R.shape[1] != dstate):
            raise ValueError(f"{path}: R[{i}] is {tuple(R.shape)}, the mixer needs [{ngroups}, {dstate}, {dstate}]")
        if not torch.isfinite(R).all():
            raise ValueError(f"{path}: R[{i}] is not finite")
        Rs.append(R.contiguous())
    decay = None
    if "decay" in saved:
        d = saved["decay"]
        if not isinstance(d, dict) or "A_log" not in d or "dt_bias" not in d:
            raise ValueError(f"{path}: 'decay' must hold 'A_log' and 'dt_bias'")
        if len(d["A_log"]) != len(Rs) or len(d["dt_bias"]) != len(Rs):
            raise ValueError(f"{path}: 'decay' must hold one A_log / dt_bias per mixer")
        decay = {k: [torch.as_tensor(v).float() for v in d[k]] for k in ("A_log", "dt_bias")}
    return Rs, decay


def _mixers(model):
    return [m for m in model.modules() if type(m).__name__ == "MambaMixer2"]


def apply_ckpt(model, env=None) -> int:
    """End of NemotronHForCausalLM.load_weights: rotations (and decay) from NESTED_SSM_CKPT
    into every MambaMixer2, and the tiered state op in v4 mode; returns the mixers
    configured (0 when the environment asks for nothing)."""
    cfg = config_from_env(env)
    if cfg is None:
        return 0
    mixers = _mixers(model)
    if not mixers:
        return 0
    m0 = mixers[0]
    ng = getattr(m0, "n_groups", None)
    tp = getattr(m0, "tp_size", 1)
    if tp != 1:
        raise NotImplementedError("nested_ssm vLLM hook: tensor parallelism > 1 is not supported")
    Rs, decay = load_ckpt(cfg["ckpt"], len(mixers), ng, getattr(m0, "ssm_state_size", None))
    dev = m0.A.device
    for i, m in enumerate(mixers):
        m.nssm_R = Rs[i].to(dev)
        if decay is not None:
            m.A.data.copy_((-torch.exp(decay["A_log"][i])).to(dev, m.A.dtype))
            m.dt_bias.data.copy_(decay["dt_bias"][i].to(dev, m.dt_bias.dtype))
        if cfg["mode"] == "v4":
            if getattr(m, "num_spec", 0):
                raise NotImplementedError("nested_ssm vLLM hook: speculative decoding is not supported")
            m.nssm = dict(pb=cfg["pb"], c=cfg["c"], cold=cfg["cold"], readout=cfg["readout"], pool=None,
                          slots=_pool_slots())
    print(f"{MARK} ckpt {cfg['ckpt']} applied to {len(mixers)} mixers (mode={cfg['mode']} "
          f"pb={cfg['pb']} c={cfg['c']} cold={cfg['cold']} readout={cfg['readout']})", flush=True)
    return len(mixers)


# --------------------------------------------------------------------------
# the hooks called from vLLM's MambaMixer2
# --------------------------------------------------------------------------
def rotate(mixer, B: torch.Tensor, C: torch.Tensor):
    """B, C [T, G*N] (views of the conv output) rotated by the mixer's R: fp32 accumulation,
    rounded to their dtype (scale/vllm_v4_patch.py:41-45 with semantic decision D6)."""
    from .ops import rot_flat
    R = mixer.nssm_R
    if R is None or B.shape[0] == 0:
        return B, C
    return rot_flat(B, R), rot_flat(C, R)


class SlotMap:
    """vLLM block id -> tiered-pool slot.  vLLM 0.22 indexes a Mamba layer's state by block id
    over the whole block pool it shares with the other layer groups (a layer's state tensor has
    num_blocks rows, of which one per live request is used), so the tiered pool is sized by the
    number of concurrent sequences and reached through this map.  A block keeps its slot while
    it is mapped; when a prefill needs slots and none is free, the slots of blocks that are in
    neither this step's decode batch nor its prefill rows (finished requests) are reclaimed."""

    def __init__(self, num_slots: int):
        self.num_slots = num_slots
        self.of_block: dict[int, int] = {}
        self.free = list(range(num_slots - 1, -1, -1))

    def assign(self, blocks: list[int], live: list[int]) -> tuple[list[int], list[int]]:
        """Slots for the prefill rows' ``blocks``; returns (slots, blocks unmapped by a
        reclamation).  ``live``: this step's decode blocks."""
        need = [k for k in dict.fromkeys(blocks) if k not in self.of_block]
        freed = []
        if len(need) > len(self.free):
            keep = set(blocks) | set(live)
            for k in [k for k in self.of_block if k not in keep]:
                self.free.append(self.of_block.pop(k))
                freed.append(k)
            if len(need) > len(self.free):
                raise RuntimeError(f"nested_ssm vLLM hook: {len(self.of_block) + len(need)} live sequences exceed "
                                   f"the tiered pool's {self.num_slots} slots (NESTED_SSM_SLOTS)")
        for k in need:
            self.of_block[k] = self.free.pop()
        return [self.of_block[k] for k in blocks], freed


def _pool_slots() -> int:
    """Tiered-pool slots per layer: NESTED_SSM_SLOTS, else the engine's max_num_seqs + 64 (read
    while the model is built, when vLLM's config is current), else 320."""
    if int(os.environ.get("NESTED_SSM_SLOTS", "0")) > 0:
        return int(os.environ["NESTED_SSM_SLOTS"])
    try:
        from vllm.config import get_current_vllm_config
        return int(get_current_vllm_config().scheduler_config.max_num_seqs) + 64
    except Exception:   # outside a vLLM engine (tests)
        return 320


def _pool(mixer, ssm_state: torch.Tensor):
    """The layer's tiered pool and block map, made for this ssm_state tensor (vLLM's profiling
    run calls the layer before the real cache exists; a new cache makes a new pool)."""
    st = mixer.nssm
    src = (ssm_state.data_ptr(), tuple(ssm_state.shape))
    if st.get("pool") is None or st.get("src") != src:
        from .pool import TieredSlotPool
        nb, H, P, N = ssm_state.shape
        slots = st.get("slots") or _pool_slots()
        st["pool"] = TieredSlotPool(1, slots, H, P, N, mixer.n_groups, st["pb"], st["c"], st["cold"],
                                    torch.bfloat16, ssm_state.device, max_batch=max(slots, 8192))
        st["map"] = torch.full((nb,), -1, dtype=torch.int32, device=ssm_state.device)   # block -> slot
        st["slotmap"] = SlotMap(slots)
        st["src"] = src
    return st["pool"]


def prefill(mixer, ssm_state: torch.Tensor, slots: torch.Tensor, decode_slots: torch.Tensor | None = None) -> None:
    """After vLLM wrote the prefill's final states into ``ssm_state[slots]`` (block ids): give
    the blocks tiered-pool slots and split the states into them (scale/vllm_v4_patch.py:123-137).
    ``decode_slots``: this step's decode blocks (kept when slots are reclaimed).  The block ids
    are read on the host: one synchronisation per prefill step (vLLM never captures batches with
    prefills in CUDA graphs; decode steps, which may be captured, do not synchronise)."""
    if mixer.nssm is None:
        return
    from .ops import prefill_split
    if slots.dim() > 1:
        slots = slots.reshape(-1)
    pool = _pool(mixer, ssm_state)
    st = mixer.nssm
    blocks = slots.tolist()
    live = decode_slots.reshape(-1).tolist() if decode_slots is not None else []
    comp, freed = st["slotmap"].assign(blocks, live)
    dev = ssm_state.device
    if freed:
        st["map"][torch.tensor(freed, dtype=torch.long, device=dev)] = -1
    comp_t = torch.tensor(comp, dtype=torch.int32, device=dev)
    st["map"][slots.long()] = comp_t
    prefill_split(pool, 0, ssm_state[slots].float().contiguous(), comp_t)


def decode(mixer, ssm_state, x, dt_raw, B, C, slots_in, slots_out, out) -> None:
    """The tiered decode step in place of vLLM's selective_state_update (v4 mode).

    x [b, H*P] or [b, H, P], dt_raw [b, H] before dt_bias and softplus, B / C [b, G*N] as
    split from the conv output (rotated here, on the GPU, by R), slots [b] (or vLLM's [b, 1])
    with NULL_BLOCK_ID on padded rows, out [b, H, P] (vLLM's preallocated output).  The state
    lives in the tiered pool, reached through the block map (an unmapped block, the null block of
    padded rows among them, is skipped)."""
    from .ops import tiered_state_update
    if slots_in is not slots_out and slots_in.data_ptr() != slots_out.data_ptr():
        raise NotImplementedError("nested_ssm vLLM hook: prefix caching of Mamba states is not supported")
    st = mixer.nssm
    H, P, G = mixer.num_heads, mixer.head_dim, mixer.n_groups
    b = out.shape[0]
    pool = _pool(mixer, ssm_state)
    if "A" not in st:   # fp32 per-head parameters, made once (no allocation in captured graphs)
        st["A"] = mixer.A.detach().float().reshape(-1).contiguous()
        st["D"] = mixer.D.detach().float().reshape(-1).contiguous()
        st["dt_bias"] = mixer.dt_bias.detach().float().reshape(-1).contiguous()
    comp = st["map"][slots_in.reshape(-1).long()]   # block -> slot, -1 when unmapped
    bf = torch.bfloat16
    x3 = x.reshape(b, H, P)
    if x3.dtype != bf:
        x3 = x3.to(bf)
    tiered_state_update(pool, 0, x3, dt_raw, st["A"], B.reshape(b, G, -1).to(bf), C.reshape(b, G, -1).to(bf),
                        st["D"], st["dt_bias"], True, comp, -1, out, mixer.nssm_R, 0.0,
                        st.get("readout", "stale"))


# --------------------------------------------------------------------------
# the installer: anchors in vLLM 0.22's sources (the reference's five, scale/install_vllm_v4.sh)
# --------------------------------------------------------------------------
MIXER = os.path.join("model_executor", "layers", "mamba", "mamba_mixer2.py")
NEMOTRON = os.path.join("model_executor", "models", "nemotron_h.py")

# (file, anchor, text): text is inserted after the anchor ("after") or replaces it ("replace")
PATCHES = [
    (MIXER, "after",
     "        self.is_blackwell = current_platform.is_device_capability_family(100)\n",
     "\n"
     "        # [nested_ssm] rotation R and the tiered decode state op (set by apply_ckpt)\n"
     "        self.nssm = None\n"
     "        self.nssm_R = None\n"),
    (MIXER, "after",
     "            hidden_states_p, B_p, C_p = self.split_hidden_states_B_C_fn(\n"
     "                hidden_states_B_C_p\n"
     "            )\n",
     "            if self.nssm_R is not None:  # [nested_ssm] rotate B/C per group\n"
     "                from nested_ssm_b200 import vllm_hook as _nssm\n"
     "                B_p, C_p = _nssm.rotate(self, B_p, C_p)\n"),
    (MIXER, "after",
     "                assert state_indices_tensor_p is not None\n"
     "                ssm_state[state_indices_tensor_p] = varlen_states\n",
     "                if self.nssm is not None:  # [nested_ssm] final states -> tiered pool\n"
     "                    from nested_ssm_b200 import vllm_hook as _nssm\n"
     "                    _nssm.prefill(self, ssm_state, state_indices_tensor_p,\n"
     "                                  state_indices_tensor_d if has_decode else None)\n"),
    (MIXER, "after",
     "            hidden_states_d, B_d, C_d = self.split_hidden_states_B_C_fn(\n"
     "                hidden_states_B_C_d\n"
     "            )\n",
     "            _nssm_dt_raw = dt_d  # [nested_ssm] pre-softplus dt (b, H)\n"
     "            if self.nssm_R is not None and self.nssm is None:  # [nested_ssm] fresh mode\n"
     "                from nested_ssm_b200 import vllm_hook as _nssm\n"
     "                B_d, C_d = _nssm.rotate(self, B_d, C_d)\n"),
    (MIXER, "replace",
     "            selective_state_update(\n"
     "                ssm_state,\n"
     "                hidden_states_d,\n"
     "                dt_d,\n"
     "                A_d,\n"
     "                B_d,\n"
     "                C_d,\n"
     "                D_d,\n"
     "                dt_bias,\n"
     "                dt_softplus=True,\n"
     "                state_batch_indices=state_indices_tensor_d_input,\n"
     "                dst_state_batch_indices=state_indices_tensor_d_output,\n"
     "                out=preallocated_ssm_out_d.view(num_decode_tokens, -1, self.head_dim),\n"
     "                num_accepted_tokens=num_accepted_tokens,\n"
     "                cu_seqlens=query_start_loc_d,\n"
     "                is_blackwell=self.is_blackwell,\n"
     "            )\n",
     "            if self.nssm is not None:  # [nested_ssm] tiered decode state op\n"
     "                from nested_ssm_b200 import vllm_hook as _nssm\n"
     "                _nssm.decode(\n"
     "                    self, ssm_state, hidden_states_d, _nssm_dt_raw, B_d, C_d,\n"
     "                    state_indices_tensor_d_input, state_indices_tensor_d_output,\n"
     "                    preallocated_ssm_out_d.view(num_decode_tokens, -1, self.head_dim),\n"
     "                )\n"
     "            else:\n"
     "                selective_state_update(\n"
     "                    ssm_state,\n"
     "                    hidden_states_d,\n"
     "                    dt_d,\n"
     "                    A_d,\n"
     "                    B_d,\n"
     "                    C_d,\n"
     "                    D_d,\n"
     "                    dt_bias,\n"
     "                    dt_softplus=True,\n"
     "                    state_batch_indices=state_indices_tensor_d_input,\n"
     "                    dst_state_batch_indices=state_indices_tensor_d_output,\n"
     "                    out=preallocated_ssm_out_d.view(num_decode_tokens, -1, self.head_dim),\n"
     "                    num_accepted_tokens=num_accepted_tokens,\n"
     "                    cu_seqlens=query_start_loc_d,\n"
     "                    is_blackwell=self.is_blackwell,\n"
     "                )  # [nested_ssm] vLLM's own update otherwise\n"),
    (NEMOTRON, "replace",
     "        loader = AutoWeightsLoader(self, skip_prefixes=[\"mtp\"])\n"
     "        return loader.load_weights(weights, mapper=self.hf_to_vllm_mapper)\n",
     "        loader = AutoWeightsLoader(self, skip_prefixes=[\"mtp\"])\n"
     "        loaded = loader.load_weights(weights, mapper=self.hf_to_vllm_mapper)\n"
     "        from nested_ssm_b200 import vllm_hook as _nssm\n"
     "        _nssm.apply_ckpt(self)  # [nested_ssm] no-op unless NESTED_SSM_CKPT is set\n"
     "        return loaded\n"),
]


def patch_source(src: str, how: str, anchor: str, text: str, name: str = "") -> tuple[str, bool]:
    """Apply one anchored edit; returns (new source, changed).  Already-applied edits are left
    alone (idempotent); a missing anchor raises ValueError."""
    if text in src:
        return src, False
    if src.count(anchor) != 1:
        raise ValueError(f"{name}: anchor found {src.count(anchor)} times (expected once):\n{anchor}")
    return (src.replace(anchor, anchor + text, 1) if how == "after" else src.replace(anchor, text, 1)), True


def install(vllm_dir: str, check_only: bool = False) -> list[str]:
    """Patch vLLM's mamba_mixer2.py and nemotron_h.py under ``vllm_dir`` (the ``vllm`` package
    directory); returns the files changed.  Every edit carries the marker; re-running changes
    nothing.  ``check_only`` verifies that every anchor is present without writing."""
    changed = []
    for rel in (MIXER, NEMOTRON):
        path = os.path.join(vllm_dir, rel)
        with open(path) as f:
            src = f.read()
        new = src
        for frel, how, anchor, text in PATCHES:
            if frel == rel:
                new, _ = patch_source(new, how, anchor, text, rel)
        if new != src and not check_only:
            with open(path, "w") as f:
                f.write(new)
            py_compile.compile(path, doraise=True)
            changed.append(path)
    return changed


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Install the nested_ssm tiered decode into a vLLM 0.22 install")
    ap.add_argument("--vllm", default=None, help="the vllm package directory (default: the importable one)")
    ap.add_argument("--check", action="store_true", help="only verify the anchors")
    a = ap.parse_args(argv)
    d = a.vllm
    if d is None:
        import vllm
        d = os.path.dirname(vllm.__file__)
    done = install(d, check_only=a.check)
    print(f"{MARK} {'anchors present' if a.check else 'patched: ' + (', '.join(done) or 'nothing (already patched)')}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
