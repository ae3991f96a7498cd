"""Drop-in for the reference's HF integration: ``install(model, pb, c, ...)`` puts the tiered
decode state op into a transformers NemotronH model's Mamba2 mixers.

Mirrors ``install`` / ``_dispatch`` / ``_lean_prefill`` / ``_v4_decode`` of
scale/v4_native_decode.py:26-256.  Prefill with a cache runs the lean prefill when
``lean_prefill`` (the reference's default) and the shapes are compiled (bf16, headdim 64 / 80,
d_state 128, chunk 128): in_proj, the model's conv1d + SiLU over the prompt, the rotation of B
and C by the mixer's ``ActRotMask`` R (``rot_flat``), ``mamba_chunk_scan_combined`` (the
tcgen05 chunk scan) with the final states into the cache, ``gated_rmsnorm``, out_proj; other
prefills run the model's own torch forward (the reference's ``lean_prefill=0``).  Either way
the final recurrent state of every row is then split into a tiered slot pool, and each
one-token decode runs in_proj, ``conv_step`` (conv1d update of the HF cache's conv state,
SiLU, split, rotation), ``tiered_state_update``, ``gated_rmsnorm`` and out_proj.  The model's
weights and cache must live on a CUDA device.

Cold storage: ``cold="fp32"`` reproduces the reference's ``cold_bf16=0`` to fp32 rounding;
``"bf16"`` / ``"fp8"`` keep the cold slice only in that dtype (dequantise, replay,
requantise every c tokens), where the reference re-snapshots a full fp32 state.
``cold="off"`` is the hot-only self-speculative draft model (the reference's
``install(..., cold="off")``, scale/v4_fused_decode.py:140-142 and :49-55): after the prefill
split, every decode token runs ``draft_state_update`` on a draft copy of the hot slice, with no
cold read, ring or flush.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .ops import (conv_step, draft_state_update, gated_rmsnorm, mamba_chunk_scan_combined, prefill_split, rot_flat,
                  tiered_state_update)
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


def _width_mask(mixer, rows: int, device) -> torch.Tensor | None:
    """Mask of the rotated B / C coordinates the mixer's ActRotMask keeps, or None when it
    keeps all of them.  ``ActRotMask._mask`` (scale/nemotron_retrofit.py:29-37) zeroes the
    coordinates ``n >= width`` of every group after the rotation; an int width applies to every
    row, a 1-D tensor width holds one width per batch row (it broadcasts against the batch
    axis).  The width is read at every call, so ``set_width`` (nemotron_retrofit.py:112-114)
    takes effect on the next token.  Returns a float mask that broadcasts against
    ``[rows, G, N]``."""
    act = mixer.act
    if not (hasattr(act, "R") and hasattr(act, "width")):
        return None
    N = mixer.ssm_state_size
    w = act.width
    idx = torch.arange(N, device=device)
    if torch.is_tensor(w) and w.dim() > 0:
        w = w.reshape(-1).to(device)
        if w.numel() != rows:
            raise ValueError(f"ActRotMask width holds {w.numel()} per-row widths for a batch of {rows}")
        return (idx[None, :] < w[:, None]).float()[:, None, :]
    w = int(w)
    if w >= N:
        return None
    return (idx < w).float()[None, None, :]


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
    mask = _width_mask(self, b, Bv.device)
    if mask is not None:   # ActRotMask's width mask on the rotated B and C
        Bv = Bv * mask.to(Bv.dtype)
        Cv = Cv * mask.to(Cv.dtype)
    A = -torch.exp(self.A_log.float())
    y = torch.empty(b, H, P, dtype=dtype, device=input_states.device)
    norm = self.norm
    if st["cold"] == "off":   # hot-only draft: the first token after the prefill starts from the pool
        draft_state_update(st["pool"], 0, st["draft"], x, dt[:, 0], A, Bv, Cv, self.D, self.dt_bias, True,
                           st["slots"], -1, y, None, self.time_step_min, from_pool=st["draft_fresh"])
        st["draft_fresh"] = False
        return self.out_proj(_norm(self, y.reshape(b, 1, I), gate).to(dtype))
    if (all(hasattr(norm, a) for a in ("weight", "variance_epsilon", "group_size"))
            and norm.group_size == (H // G) * P):
        # the gated norm fused into the step (its group is one SSM group of a row)
        tiered_state_update(st["pool"], 0, x, dt[:, 0], A, Bv, Cv, self.D, self.dt_bias, True, st["slots"], -1,
                            y, None, self.time_step_min, st["mode"],
                            norm=(gate[:, 0], norm.weight, norm.variance_epsilon))
        scan_output = y.reshape(b, 1, I)
    else:
        tiered_state_update(st["pool"], 0, x, dt[:, 0], A, Bv, Cv, self.D, self.dt_bias, True, st["slots"], -1, y,
                            None, self.time_step_min, st["mode"])
        scan_output = _norm(self, y.reshape(b, 1, I), gate)
    return self.out_proj(scan_output.to(dtype))


def _norm(self, y, gate):
    norm = self.norm
    if all(hasattr(norm, a) for a in ("weight", "variance_epsilon", "group_size")):   # Zamba2RMSNormGated
        return gated_rmsnorm(y, gate, norm.weight, norm.variance_epsilon, norm.group_size)
    return norm(y, gate)


def _lean_ok(self, input_states) -> bool:
    """Shapes the chunk scan is compiled for (else the model's own prefill runs)."""
    return (input_states.is_cuda and input_states.dtype == torch.bfloat16 and self.head_dim in (64, 80)
            and self.ssm_state_size == 128 and getattr(self, "chunk_size", 0) == 128 and _is_silu_like(self))


def _is_silu_like(self) -> bool:
    act = self.act.act if (hasattr(self.act, "R") and hasattr(self.act, "act")) else self.act
    return _is_silu(act)


def _lean_prefill(self, input_states, cache_params, attention_mask):
    """The memory-lean prefill (scale/v4_native_decode.py:175-220) on the GPU kernels: conv1d +
    SiLU over the prompt (the model's own conv, activation in fp32), B and C rotated by R,
    the chunk scan with its final states into the cache, the gated norm, out_proj."""
    st = self._nssm
    b, T, _ = input_states.shape
    dtype = input_states.dtype
    if attention_mask is not None and not torch.all(attention_mask == 1):
        input_states = (input_states * attention_mask[:, :, None]).to(dtype)
    H, P, N, G = self.num_heads, self.head_dim, self.ssm_state_size, self.n_groups
    I, GN = self.intermediate_size, G * N
    proj = self.in_proj(input_states)
    d_mlp = (proj.shape[-1] - 2 * I - 2 * GN - H) // 2
    _, _, gate, xbc, dt = proj.split([d_mlp, d_mlp, I, self.conv_dim, H], dim=-1)
    xbc_t = xbc.transpose(1, 2)
    if cache_params is not None:
        cache_params.update_conv_state(F.pad(xbc_t, (self.conv_kernel_size - xbc_t.shape[-1], 0)), self.layer_idx)
    # conv + bias + SiLU in fp32, rounded once to the activation dtype (causal_conv1d_fn's
    # rounding, scale/v4_native_decode.py:198-200)
    K = self.conv_kernel_size
    w = self.conv1d.weight.float()
    bias = self.conv1d.bias.float() if self.conv1d.bias is not None else None
    conv = F.conv1d(xbc_t.float(), w, bias, padding=K - 1, groups=w.shape[0])[..., :T]
    conv = F.silu(conv).to(dtype).transpose(1, 2).contiguous()   # [b, T, conv_dim]
    x = conv[..., :I].view(b, T, H, P)
    Bm, Cm = conv[..., I:I + GN], conv[..., I + GN:]
    if st["R"] is not None:
        if st["R"].device != conv.device:
            st["R"] = st["R"].to(conv.device, torch.float32).contiguous()
        Bm = rot_flat(Bm.reshape(b * T, GN), st["R"])
        Cm = rot_flat(Cm.reshape(b * T, GN), st["R"])
    mask = _width_mask(self, b, conv.device)
    if mask is not None:   # ActRotMask's width mask, per row over every prompt token
        Bm = (Bm.reshape(b, T, G, N) * mask[:, None].to(Bm.dtype)).reshape(b * T, GN)
        Cm = (Cm.reshape(b, T, G, N) * mask[:, None].to(Cm.dtype)).reshape(b * T, GN)
    A = -torch.exp(self.A_log.float())
    lim = getattr(self, "time_step_limit", None)
    lim = (0.0, math.inf) if lim is None else (float(lim[0]), float(lim[1]))
    y, ssm = mamba_chunk_scan_combined(x, dt, A, Bm.reshape(b, T, G, N), Cm.reshape(b, T, G, N), self.chunk_size,
                                       D=self.D, dt_bias=self.dt_bias, dt_softplus=True, dt_limit=lim,
                                       return_final_states=True)
    if cache_params is not None:
        cache_params.update_recurrent_state(ssm, self.layer_idx)
    scan_output = _norm(self, y.view(b, T, I), gate)
    return self.out_proj(scan_output.to(self.out_proj.weight.dtype))


def _dispatch(self, input_states, cache_params=None, attention_mask=None):
    st = self._nssm
    seq_len = input_states.shape[1]
    if (cache_params is not None and seq_len == 1 and st["pool"] is not None
            and cache_params.has_previous_state(self.layer_idx)):
        return _decode(self, input_states, cache_params)
    if (seq_len > 1 and cache_params is not None and not cache_params.has_previous_state(self.layer_idx)
            and st["lean_prefill"] and _lean_ok(self, input_states)):
        out = _lean_prefill(self, input_states, cache_params, attention_mask)
    else:
        out = st["orig"](self, input_states, cache_params, attention_mask)
    if cache_params is not None:   # end of prefill: the tiered pool takes the final states
        ssm = cache_params.layers[self.layer_idx].recurrent_states.float()
        b, H, P, N = ssm.shape
        pool = st["pool"]
        if pool is None or pool.S != b or pool.device != ssm.device:
            off = st["cold"] == "off"   # the draft never reads the cold slice, ring or chunk (the
            storage, chunk = ("fp8", 4) if off else (st["cold"], st["c"])   # reference passes c = 1 << 20)
            pool = TieredSlotPool(1, b, H, P, N, self.n_groups, st["pb"], chunk, storage,
                                  input_states.dtype, ssm.device, max_batch=b)
            st["pool"] = pool
            st["slots"] = torch.arange(b, dtype=torch.int32, device=ssm.device)
            st["draft"] = pool.new_draft()[0] if st["cold"] == "off" else None
        prefill_split(pool, 0, ssm.contiguous(), st["slots"])
        st["draft_fresh"] = True
    return out


def install(model, pb: int = 32, c: int = 16, cold: str | None = None, corr: int = 0, coldoff: int = 0,
            cold_bf16: int | None = None, lean_prefill: int = 1) -> int:
    """Put the tiered decode into every NemotronH Mamba2 mixer of ``model``; returns how many.

    Argument names follow scale/v4_native_decode.py:247-256 (``cold_bf16=1`` means
    ``cold="bf16"``, ``0`` means ``"fp32"``); ``cold="fp8"`` is the fp8 storage;
    ``lean_prefill`` (default 1, as the reference's ``v4cfg.get("lean_prefill", 1)``) selects
    the chunk-scan prefill; ``cold="off"`` installs the hot-only draft model
    (scale/v4_fused_decode.py:140-142)."""
    if cold is None:
        cold = "fp32" if cold_bf16 == 0 else "bf16"
    mode = _MODES.get((int(bool(corr)), int(bool(coldoff))))
    if mode is None:
        raise ValueError("corr and coldoff are exclusive")
    n = 0
    for m in model.modules():
        if type(m).__name__ == "NemotronHMamba2Mixer":
            orig = type(m).torch_forward
            m._nssm = dict(pb=pb, c=c, cold=cold, mode=mode, pool=None, slots=None, orig=orig, draft=None,
                           draft_fresh=True,
                           R=_rotation_and_act(m), lean_prefill=int(bool(lean_prefill)))
            m.torch_forward = _dispatch.__get__(m)
            n += 1
    return n
