"""Drop-in for the reference's HF integration: ``install(model, pb, c, ...)`` puts the tiered
decode state op into a transformers NemotronH model's Mamba2 mixers.

Mirrors ``install`` / ``_dispatch`` / ``_v4_decode`` of scale/v4_native_decode.py:26-256:
prefill (or any call that is not a one-token decode with a cache) runs the model's own
torch forward, after which the final recurrent state of every row is split into a tiered
slot pool; each one-token decode then runs in_proj, ``conv_step`` (conv1d update of the HF
cache's conv state, SiLU, split, rotation by the mixer's ``ActRotMask`` R when it has one),
``tiered_state_update``, ``gated_rmsnorm`` (the mixer's norm) and out_proj.  The decode path runs
on the GPU only; the model's weights and cache must live on a CUDA device.

Cold storage: ``cold="fp32"`` reproduces the reference's ``cold_bf16=0`` to fp32 rounding;
``"bf16"`` / ``"fp8"`` keep the cold slice only in that dtype (dequantise, replay,
requantise every c tokens), where the reference re-snapshots a full fp32 state.
"""
from __future__ import annotations

import torch

from .ops import conv_step, gated_rmsnorm, prefill_split, tiered_state_update
from .pool import TieredSlotPool

_MODES = {(0, 0): "stale", (1, 0): "corr", (0, 1): "coldoff"}


def _is_silu(act) -> bool:
    return isinstance(act, torch.nn.SiLU) or type(act).__name__ in ("SiLU", "SiLUActivation")


def _rotation_and_act(mixer):
    """(R or None) of the mixer's activation: the reference's ActRotMask wraps the SiLU and
    holds R [G, N, N] (scale/nemotron_retrofit.py:18-54)."""
    act = mixer.act
    if hasattr(act, "R") and hasattr(act, "act"):
        if not _is_silu(act.act):
            raise NotImplementedError("the tiered decode supports a SiLU activation only")
        return act.R.detach()
    if not _is_silu(act):
        raise NotImplementedError("the tiered decode supports a SiLU activation only")
    return None


def _decode(self, input_states, cache_params):
    """One decode token: _v4_decode (scale/v4_native_decode.py:29-172) on the GPU kernels."""
    st = self._nssm
    b = input_states.shape[0]
    dtype = input_states.dtype
    H, P, N, G = self.num_heads, self.head_dim, self.ssm_state_size, self.n_groups
    I = self.intermediate_size
    proj = self.in_proj(input_states)
    d_mlp = (proj.shape[-1] - 2 * I - 2 * G * N - H) // 2
    _, _, gate, xbc, dt = proj.split([d_mlp, d_mlp, I, self.conv_dim, H], dim=-1)
    conv_state = cache_params.layers[self.layer_idx].conv_states
    if st["R"] is not None and st["R"].device != conv_state.device:
        st["R"] = st["R"].to(conv_state.device, torch.float32).contiguous()
    x, Bv, Cv = conv_step(xbc[:, 0].contiguous(), conv_state, self.conv1d.weight,
                          self.conv1d.bias if self.use_conv_bias else None, "silu", None, -1, st["R"],
                          nheads=H, headdim=P, ngroups=G, dstate=N)
    A = -torch.exp(self.A_log.float())
    y = torch.empty(b, H, P, dtype=dtype, device=input_states.device)
    tiered_state_update(st["pool"], 0, x, dt[:, 0], A, Bv, Cv, self.D, self.dt_bias, True, st["slots"], -1, y,
                        None, self.time_step_min, st["mode"])
    norm = self.norm
    if all(hasattr(norm, a) for a in ("weight", "variance_epsilon", "group_size")):   # Zamba2RMSNormGated
        scan_output = gated_rmsnorm(y.reshape(b, 1, I), gate, norm.weight, norm.variance_epsilon, norm.group_size)
    else:
        scan_output = norm(y.reshape(b, 1, I), gate)
    return self.out_proj(scan_output.to(dtype))


def _dispatch(self, input_states, cache_params=None, attention_mask=None):
    st = self._nssm
    seq_len = input_states.shape[1]
    if (cache_params is not None and seq_len == 1 and st["pool"] is not None
            and cache_params.has_previous_state(self.layer_idx)):
        return _decode(self, input_states, cache_params)
    out = st["orig"](self, input_states, cache_params, attention_mask)
    if cache_params is not None:   # end of prefill: the tiered pool takes the final states
        ssm = cache_params.layers[self.layer_idx].recurrent_states.float()
        b, H, P, N = ssm.shape
        pool = st["pool"]
        if pool is None or pool.S != b or pool.device != ssm.device:
            pool = TieredSlotPool(1, b, H, P, N, self.n_groups, st["pb"], st["c"], st["cold"],
                                  input_states.dtype, ssm.device, max_batch=b)
            st["pool"] = pool
            st["slots"] = torch.arange(b, dtype=torch.int32, device=ssm.device)
        prefill_split(pool, 0, ssm.contiguous(), st["slots"])
    return out


def install(model, pb: int = 32, c: int = 16, cold: str | None = None, corr: int = 0, coldoff: int = 0,
            cold_bf16: int | None = None) -> int:
    """Put the tiered decode into every NemotronH Mamba2 mixer of ``model``; returns how many.

    Argument names follow scale/v4_native_decode.py:247-256 (``cold_bf16=1`` means
    ``cold="bf16"``, ``0`` means ``"fp32"``); ``cold="fp8"`` is the fp8 storage."""
    if cold is None:
        cold = "fp32" if cold_bf16 == 0 else "bf16"
    mode = _MODES.get((int(bool(corr)), int(bool(coldoff))))
    if mode is None:
        raise ValueError("corr and coldoff are exclusive")
    n = 0
    for m in model.modules():
        if type(m).__name__ == "NemotronHMamba2Mixer":
            orig = type(m).torch_forward
            m._nssm = dict(pb=pb, c=c, cold=cold, mode=mode, pool=None, slots=None, orig=orig,
                           R=_rotation_and_act(m))
            m.torch_forward = _dispatch.__get__(m)
            n += 1
    return n
