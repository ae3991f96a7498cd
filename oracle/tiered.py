"""TEST INFRASTRUCTURE ONLY -- CPU oracle for the tiered Mamba2 decode state op.

Restates, in torch eager on the CPU, the per-layer decode state op of
nested_ssm ("v4" tiering).  Citations are ``path:line`` inside the reference
project (omin-Kwon/nested_ssm):

* rotation of B and C by a per-group orthogonal R:
  ``scale/nemotron_retrofit.py:24-27`` (ActRotMask._rot),
  ``scale/vllm_v4_patch.py:41-45`` (rot_flat), ``scale/v4_fused_decode.py:45-48``
  (fp32 einsum, cast back);
* dt discretisation: ``scale/v4_native_decode.py:50-55`` (softplus, clamp at
  ``time_step_min``), ``scale/vllm_v4_patch.py:176-177`` (fp32 softplus);
* hot-slice update ``h <- exp(dt*A) h + (dt*B) x``: ``scale/v4_native_decode.py:56-67``;
* tiered readout ``y = C_hot.h + exp(glog) C_cold.snap + D x``:
  ``scale/v4_native_decode.py:145-158,168-169``, ``scale/vllm_v4_patch.py:161-167``;
* fp8 cold storage, one scale per (slot, head, headdim row):
  ``scale/vllm_v4_patch.py:106-120``;
* per-slot bookkeeping (t, flush every c tokens, glog lag of one token):
  ``scale/vllm_v4_patch.py:170-179``, ``scale/v4_native_decode.py:159-167``;
* ring of the last c tokens and the rank-c flush replay with suffix decays:
  ``scale/v4_fused_decode.py:71-92``;
* prefill split of a full state into hot / quantised cold: ``scale/vllm_v4_patch.py:123-137``;
* exact rank-c correction variant: ``scale/v4_native_decode.py:81-117``.

Two semantics are provided:

``replay`` (what the CUDA kernels implement): the cold slice lives ONLY in its
storage dtype (fp8 + scale, bf16 or fp32).  Between flushes it is read stale
with the lagged decay correction; every c tokens it is dequantised, replayed
with the ring (``cold <- exp(sum dA) cold + sum_j exp(suf_j) (dt_j x_j) B_j``)
and requantised.

``native`` (what the reference's HF/vLLM paths do): a full fp32 state is kept
fresh and the cold snapshot is re-taken from it every c tokens.  With fp32 cold
storage both semantics agree to fp32 reassociation; with fp8/bf16 storage the
replay requantises the accumulated cold each flush, and the difference is
reported as drift, not asserted.

All arithmetic is fp32 (the reference's fused and vLLM paths compute dt, the
update and the readout in fp32).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

__all__ = [
    "FP8", "FP8_MAX", "SCALE_EPS", "rot_flat", "dt_softplus", "quantize_rows",
    "dequantize_rows", "TieredPoolRef", "NativePoolRef", "prefill_split",
    "tiered_step", "native_step", "fresh_step", "materialize", "make_inputs",
    "make_params", "fp8_ordered_codes", "conv_step", "conv_split", "gated_rmsnorm",
    "draft_step", "verify_steps", "commit_steps",
]

FP8 = torch.float8_e4m3fn
FP8_MAX = 448.0
SCALE_EPS = 1e-12


# --------------------------------------------------------------------------
# elementary pieces
# --------------------------------------------------------------------------
def rot_flat(x: torch.Tensor, R: torch.Tensor, mode: str = "fp32") -> torch.Tensor:
    """Rotate flat B or C ``[T, G*N]`` by ``R [G, N, N]``: ``x'[g,m] = sum_n R[g,m,n] x[g,n]``.

    ``mode="fp32"``: fp32 einsum, cast back to ``x.dtype`` (scale/v4_fused_decode.py:47-48).
    ``mode="native"``: einsum in ``x.dtype`` with ``R.to(x.dtype)``
    (scale/vllm_v4_patch.py:41-45, scale/nemotron_retrofit.py:24-27).
    """
    T = x.shape[0]
    G, N, _ = R.shape
    if mode == "fp32":
        out = torch.einsum("tgn,gmn->tgm", x.reshape(T, G, N).float(), R.float())
        return out.reshape(T, G * N).to(x.dtype)
    if mode == "native":
        return torch.einsum("tgn,gmn->tgm", x.reshape(T, G, N), R.to(x.dtype)).reshape(T, G * N)
    raise ValueError(f"unknown rotation mode {mode!r}")


def dt_softplus(dt_raw: torch.Tensor, dt_bias: torch.Tensor, clamp_min: float | None) -> torch.Tensor:
    """``dt = clamp(softplus(dt_raw + dt_bias), time_step_min)`` in fp32, ``[b, H]``.

    softplus: scale/vllm_v4_patch.py:176 (fp32); clamp: scale/v4_native_decode.py:55.
    """
    dt = F.softplus(dt_raw.float() + dt_bias.float().view(1, -1))
    if clamp_min is not None:
        dt = torch.clamp(dt, min=clamp_min)
    return dt


def quantize_rows(v: torch.Tensor, cold_dtype: torch.dtype):
    """Store an fp32 cold slice ``[..., P, Nc]`` in its storage dtype.

    fp8: ``scale = amax_n |v| / 448 + 1e-12`` per (.., p) row, ``q = (v / scale) -> e4m3fn``
    (scale/vllm_v4_patch.py:106-114).  Returns ``(q, scale[..., P] or None)``.
    """
    if cold_dtype == FP8:
        sc = v.abs().amax(dim=-1, keepdim=True) / FP8_MAX + SCALE_EPS
        return (v / sc).to(FP8), sc.squeeze(-1)
    return v.to(cold_dtype), None


def dequantize_rows(q: torch.Tensor, scale: torch.Tensor | None) -> torch.Tensor:
    """fp32 view of a stored cold slice (scale/vllm_v4_patch.py:116-120)."""
    s = q.float()
    if scale is not None:
        s = s * scale[..., None]
    return s


def fp8_ordered_codes(q: torch.Tensor) -> torch.Tensor:
    """Map e4m3fn bytes to integers that are monotone in value (for ulp distances)."""
    u = q.view(torch.uint8).to(torch.int32)
    mag = u & 0x7F
    return torch.where(u >= 0x80, -mag, mag)


# --------------------------------------------------------------------------
# decode-token conv ahead of the state op
# --------------------------------------------------------------------------
def conv_step(conv_state: torch.Tensor, slots, xbc: torch.Tensor, weight: torch.Tensor,
              bias: torch.Tensor | None, act: str | None = "silu", pad_slot_id: int = -1) -> torch.Tensor:
    """Causal conv1d update of one decode token; mutates ``conv_state [S, D, L]`` and returns
    the activated conv output ``[b, D]`` in fp32 (padded rows zero).

    HF decode branch: the cache rolls the state left and appends the new column
    (transformers ``update_conv_state``), then ``sum(conv_states * weight) + bias`` and the
    activation (scale/v4_native_decode.py:36-49); the fused path's ``causal_conv1d_update``
    (scale/v4_fused_decode.py:39-41) keeps L >= K-1 columns: window = last K of
    ``[state, x]``, new state = last L.  Taps accumulate in k order with one rounding per
    tap (a fused multiply-add), the activation is ``v / (1 + exp(-v))``."""
    rows, s = _valid_rows(slots, pad_slot_id)
    b, D = xbc.shape
    K = weight.shape[-1]
    L = conv_state.shape[-1]
    out = torch.zeros(b, D)
    if rows.numel() == 0:
        return out
    full = torch.cat([conv_state[s].float(), xbc[rows].float()[..., None]], dim=-1)   # [r, D, L+1]
    win = full[..., L + 1 - K:]
    w = weight.reshape(D, K).double()
    acc = torch.zeros(rows.numel(), D)
    for k in range(K):   # fma: exact product + accumulator, rounded once
        acc = (w[:, k] * win[..., k].double() + acc.double()).float()
    if bias is not None:
        acc = acc + bias.float()
    if act == "silu":
        acc = acc / (1.0 + torch.exp(-acc))
    conv_state[s] = full[..., 1:].to(conv_state.dtype)
    out[rows] = acc
    return out


def conv_split(out: torch.Tensor, I: int, G: int, N: int, R: torch.Tensor | None, io_dtype):
    """Split a conv output ``[b, I + 2 G N]`` into x ``[b, I]``, B, C ``[b, G, N]`` in the io
    dtype, B and C rounded to it first and then rotated by ``R`` in fp32 (the post-conv
    rotation of scale/v4_fused_decode.py:45-48)."""
    b = out.shape[0]
    x = out[:, :I].to(io_dtype)
    Bv = out[:, I:I + G * N].to(io_dtype)
    Cv = out[:, I + G * N:].to(io_dtype)
    if R is not None:
        Bv, Cv = rot_flat(Bv, R, "fp32"), rot_flat(Cv, R, "fp32")
    return x, Bv.reshape(b, G, N), Cv.reshape(b, G, N)


def gated_rmsnorm(y: torch.Tensor, gate: torch.Tensor, weight: torch.Tensor, eps: float,
                  group_size: int) -> torch.Tensor:
    """The mixer's ``norm(y, gate)`` after the state op (scale/v4_native_decode.py:171):
    transformers' Zamba2RMSNormGated, restated by the reference as
    ``rmsnorm_fn(norm_before_gate=False)`` (scale/nemotron_retrofit.py:146-161):
    ``h = y * silu(gate)`` in fp32, per group ``h * rsqrt(mean(h^2) + eps)``, cast to y's
    dtype, times ``weight``."""
    dt = y.dtype
    h = y.float() * F.silu(gate.float())
    s = h.shape
    hg = h.view(*s[:-1], s[-1] // group_size, group_size)
    hg = hg * torch.rsqrt(hg.pow(2).mean(-1, keepdim=True) + eps)
    return (weight * hg.view(s).to(dt)).to(dt)


# --------------------------------------------------------------------------
# pools
# --------------------------------------------------------------------------
@dataclass
class TieredPoolRef:
    """One layer's tiered slot pool (replay semantics)."""
    num_slots: int
    H: int
    P: int
    N: int
    G: int
    pb: int
    c: int
    cold_dtype: torch.dtype = FP8
    io_dtype: torch.dtype = torch.bfloat16
    hot: torch.Tensor = field(init=False)
    cold: torch.Tensor = field(init=False)
    scale: torch.Tensor | None = field(init=False)
    glog: torch.Tensor = field(init=False)
    t: torch.Tensor = field(init=False)
    ring_x: torch.Tensor = field(init=False)
    ring_dt: torch.Tensor = field(init=False)
    ring_b: torch.Tensor = field(init=False)

    def __post_init__(self):
        S, H, P, N, G, pb, c = self.num_slots, self.H, self.P, self.N, self.G, self.pb, self.c
        Nc = N - pb
        self.hot = torch.zeros(S, H, P, pb)
        self.cold = torch.zeros(S, H, P, Nc).to(self.cold_dtype)
        self.scale = torch.ones(S, H, P) if self.cold_dtype == FP8 else None
        self.glog = torch.zeros(S, H)
        self.t = torch.zeros(S, dtype=torch.int32)
        self.ring_x = torch.zeros(S, H, c, P, dtype=self.io_dtype)
        self.ring_dt = torch.zeros(S, H, c)
        self.ring_b = torch.zeros(S, G, c, Nc, dtype=self.io_dtype)

    @property
    def Nc(self) -> int:
        return self.N - self.pb


@dataclass
class NativePoolRef:
    """One layer's pool in the reference's native semantics: full fp32 state kept
    fresh, cold snapshot re-taken every c tokens (scale/v4_native_decode.py:159-167,
    scale/vllm_v4_patch.py:90-103)."""
    num_slots: int
    H: int
    P: int
    N: int
    pb: int
    c: int
    cold_dtype: torch.dtype = torch.float32
    state: torch.Tensor = field(init=False)
    snap: torch.Tensor = field(init=False)
    scale: torch.Tensor | None = field(init=False)
    glog: torch.Tensor = field(init=False)
    t: torch.Tensor = field(init=False)

    def __post_init__(self):
        S, H, P, N, pb = self.num_slots, self.H, self.P, self.N, self.pb
        self.state = torch.zeros(S, H, P, N)
        self.snap = torch.zeros(S, H, P, N - pb).to(self.cold_dtype)
        self.scale = torch.ones(S, H, P) if self.cold_dtype == FP8 else None
        self.glog = torch.zeros(S, H)
        self.t = torch.zeros(S, dtype=torch.int32)


# --------------------------------------------------------------------------
# the state op
# --------------------------------------------------------------------------
def _valid_rows(slots: torch.Tensor, pad_slot_id: int):
    slots = slots.reshape(-1).long()
    rows = torch.nonzero(slots != pad_slot_id).reshape(-1)
    return rows, slots[rows]


def prefill_split(pool, slots: torch.Tensor, state: torch.Tensor, pad_slot_id: int = -1):
    """Split prefill final states ``state [b, H, P, N]`` (row i -> ``slots[i]``) into the pool.

    hot <- state[..., :pb]; cold <- quant(state[..., pb:]); glog <- 0; t <- 0
    (scale/vllm_v4_patch.py:123-137, scale/v4_native_decode.py:234-243).
    """
    rows, s = _valid_rows(slots, pad_slot_id)
    st = state[rows].float()
    pb = pool.pb
    if isinstance(pool, TieredPoolRef):
        pool.hot[s] = st[..., :pb]
        q, sc = quantize_rows(st[..., pb:], pool.cold_dtype)
        pool.cold[s] = q
        if sc is not None:
            pool.scale[s] = sc
    else:
        pool.state[s] = st
        q, sc = quantize_rows(st[..., pb:], pool.cold_dtype)
        pool.snap[s] = q
        if sc is not None:
            pool.scale[s] = sc
    pool.glog[s] = 0.0
    pool.t[s] = 0


def _expand_groups(v: torch.Tensor, H: int) -> torch.Tensor:
    """``[b, G, N]`` -> ``[b, H, N]`` (head h uses group h // (H/G); scale/v4_native_decode.py:59-61)."""
    G = v.shape[1]
    return v.float().repeat_interleave(H // G, dim=1)


def tiered_step(pool: TieredPoolRef, slots, x, dt_raw, B, C, A, D, dt_bias,
                clamp_min: float | None = 1e-3, pad_slot_id: int = -1,
                mode: str = "stale") -> torch.Tensor:
    """One decode token of one layer, replay semantics.  Mutates ``pool``.

    x ``[b, H, P]``, dt_raw ``[b, H]``, B/C ``[b, G, N]`` (already rotated),
    A/D/dt_bias ``[H]`` fp32, slots ``[b]``.  Returns fp32 ``y [b, H, P]``; rows
    whose slot is ``pad_slot_id`` are returned as zeros and touch nothing.

    mode ``"stale"``: the default tiered read (glog excludes this token's dA;
    scale/v4_native_decode.py:145-167).  ``"corr"``: the exact rank-c correction
    (glog inclusive, ring terms added; scale/v4_native_decode.py:81-117).
    ``"coldoff"``: hot-only readout, cold still maintained
    (scale/v4_native_decode.py:118-127).
    """
    H, P, pb, c, G = pool.H, pool.P, pool.pb, pool.c, pool.G
    HG = H // G
    out = torch.zeros(x.shape[0], H, P)
    rows, s = _valid_rows(slots, pad_slot_id)
    if rows.numel() == 0:
        return out
    A = A.float()
    xf = x[rows].float()                                         # [b,H,P]
    dt = dt_softplus(dt_raw[rows], dt_bias, clamp_min)           # [b,H]
    dA = dt * A.view(1, -1)                                      # [b,H]
    Bh = _expand_groups(B[rows], H)                              # [b,H,N]
    Ch = _expand_groups(C[rows], H)
    # ---- hot update (scale/v4_native_decode.py:56-67 on the first pb columns)
    hot = pool.hot[s]
    dB = dt[:, :, None, None] * Bh[:, :, None, :pb]
    hot = hot * torch.exp(dA)[:, :, None, None] + dB * xf[..., None]
    pool.hot[s] = hot
    y = torch.einsum("bhpn,bhn->bhp", hot, Ch[..., :pb])
    # ---- bookkeeping (scale/vllm_v4_patch.py:170-172)
    t_new = pool.t[s] + 1
    pool.t[s] = t_new
    flush = (t_new % c) == 0
    pos = ((t_new - 1) % c).long()
    cold_old = dequantize_rows(pool.cold[s], None if pool.scale is None else pool.scale[s])
    glog = pool.glog[s]
    if mode == "corr":
        glog_read = glog + dA                                    # G_t inclusive
    else:
        glog_read = glog
    if mode != "coldoff":
        y_cold = torch.einsum("bhpn,bhn->bhp", cold_old, Ch[..., pb:])
        y = y + y_cold * torch.exp(glog_read)[..., None]
    # ring gather for this row: entries 0..pos-1 are this chunk's earlier tokens
    rx = pool.ring_x[s].float()                                  # [b,H,c,P]
    rdt = pool.ring_dt[s]                                        # [b,H,c]
    rb = pool.ring_b[s].float()                                  # [b,G,c,Nc]
    if mode == "corr":
        # y_cold += sum_{j<=t} exp(G_t - G_j) (C_cold . B_j) (dt_j x_j)   (j = this chunk)
        for i in range(rows.numel()):
            p_i = int(pos[i])
            dts = torch.cat([rdt[i, :, :p_i], dt[i, :, None]], dim=1)        # [H,J]
            xs = torch.cat([rx[i, :, :p_i], xf[i, :, None]], dim=1)          # [H,J,P]
            bs = torch.cat([rb[i, :, :p_i], B[rows[i]].float()[:, None, pb:]], dim=1)  # [G,J,Nc]
            dAs = dts * A.view(-1, 1)
            J = dts.shape[1]
            suf = torch.zeros_like(dAs)
            for j in range(J - 2, -1, -1):
                suf[:, j] = suf[:, j + 1] + dAs[:, j + 1]
            bsh = bs.repeat_interleave(HG, dim=0)                            # [H,J,Nc]
            sj = torch.einsum("hjn,hn->hj", bsh, Ch[i, :, pb:])
            w = torch.exp(suf) * sj
            y[i] = y[i] + torch.einsum("hj,hjp->hp", w, dts[..., None] * xs)
    y = y + xf * D.float().view(1, H, 1)
    out[rows] = y
    # ---- non-flushing rows: ring write at pos, glog += dA (scale/v4_fused_decode.py:71-75,93)
    nf = torch.nonzero(~flush).reshape(-1)
    if nf.numel():
        sn, pn = s[nf], pos[nf]
        pool.ring_x[sn, :, pn] = x[rows[nf]].to(pool.io_dtype)
        pool.ring_dt[sn, :, pn] = dt[nf]
        pool.ring_b[sn, :, pn] = B[rows[nf]][..., pb:].to(pool.io_dtype)
        pool.glog[sn] = glog[nf] + dA[nf]
    # ---- flushing rows: rank-c replay + requant (scale/v4_fused_decode.py:76-92)
    fl = torch.nonzero(flush).reshape(-1)
    if fl.numel():
        sf = s[fl]
        dts = torch.cat([rdt[fl, :, : c - 1], dt[fl, :, None]], dim=2)            # [f,H,c]
        xs = torch.cat([rx[fl, :, : c - 1], xf[fl, :, None]], dim=2)              # [f,H,c,P]
        bs = torch.cat([rb[fl, :, : c - 1], B[rows[fl]].float()[:, :, None, pb:]], dim=2)  # [f,G,c,Nc]
        dAs = dts * A.view(1, -1, 1)
        tot = torch.zeros_like(dAs[..., 0])
        for j in range(c):
            tot = tot + dAs[..., j]
        suf = torch.zeros_like(dAs)
        for j in range(c - 2, -1, -1):
            suf[..., j] = suf[..., j + 1] + dAs[..., j + 1]
        W = torch.exp(suf)[..., None] * (dts[..., None] * xs)                     # [f,H,c,P]
        bsh = bs.repeat_interleave(HG, dim=1)                                     # [f,H,c,Nc]
        upd = torch.zeros_like(cold_old[fl])
        for j in range(c):
            upd = upd + W[:, :, j, :, None] * bsh[:, :, j, None, :]
        v = cold_old[fl] * torch.exp(tot)[..., None, None] + upd
        q, sc = quantize_rows(v, pool.cold_dtype)
        pool.cold[sf] = q
        if sc is not None:
            pool.scale[sf] = sc
        pool.glog[sf] = 0.0
    return out


def native_step(pool: NativePoolRef, slots, x, dt_raw, B, C, A, D, dt_bias,
                clamp_min: float | None = 1e-3, pad_slot_id: int = -1) -> torch.Tensor:
    """One decode token in the reference's native semantics (full fp32 state fresh,
    stale snapshot readout): scale/v4_native_decode.py:56-67,145-169 with the
    per-slot bookkeeping of scale/vllm_v4_patch.py:170-179."""
    H, P, pb, c = pool.H, pool.P, pool.pb, pool.c
    out = torch.zeros(x.shape[0], H, P)
    rows, s = _valid_rows(slots, pad_slot_id)
    if rows.numel() == 0:
        return out
    xf = x[rows].float()
    dt = dt_softplus(dt_raw[rows], dt_bias, clamp_min)
    dA = dt * A.float().view(1, -1)
    Bh = _expand_groups(B[rows], H)
    Ch = _expand_groups(C[rows], H)
    S = pool.state[s]
    S = S * torch.exp(dA)[:, :, None, None] + (dt[:, :, None, None] * Bh[:, :, None, :]) * xf[..., None]
    pool.state[s] = S
    snap = dequantize_rows(pool.snap[s], None if pool.scale is None else pool.scale[s])
    y = torch.einsum("bhpn,bhn->bhp", S[..., :pb], Ch[..., :pb]) \
        + torch.einsum("bhpn,bhn->bhp", snap, Ch[..., pb:]) * torch.exp(pool.glog[s])[..., None]
    y = y + xf * D.float().view(1, H, 1)
    out[rows] = y
    t_new = pool.t[s] + 1
    pool.t[s] = t_new
    flush = (t_new % c) == 0
    fl = torch.nonzero(flush).reshape(-1)
    if fl.numel():
        q, sc = quantize_rows(S[fl][..., pb:], pool.cold_dtype)
        pool.snap[s[fl]] = q
        if sc is not None:
            pool.scale[s[fl]] = sc
    pool.glog[s] = torch.where(flush[:, None], torch.zeros_like(dA), pool.glog[s] + dA)
    return out


def fresh_step(state: torch.Tensor, slots, x, dt_raw, B, C, A, D, dt_bias,
               clamp_min: float | None = 1e-3, pad_slot_id: int = -1) -> torch.Tensor:
    """Untiered fp32 selective state update + readout (the fresh control; the
    HF decode branch ``modeling_nemotron_h.py`` torch_forward, pb = N)."""
    H = state.shape[1]
    out = torch.zeros(x.shape[0], H, state.shape[2])
    rows, s = _valid_rows(slots, pad_slot_id)
    if rows.numel() == 0:
        return out
    xf = x[rows].float()
    dt = dt_softplus(dt_raw[rows], dt_bias, clamp_min)
    dA = dt * A.float().view(1, -1)
    Bh = _expand_groups(B[rows], H)
    Ch = _expand_groups(C[rows], H)
    S = state[s]
    S = S * torch.exp(dA)[:, :, None, None] + (dt[:, :, None, None] * Bh[:, :, None, :]) * xf[..., None]
    state[s] = S
    out[rows] = torch.einsum("bhpn,bhn->bhp", S, Ch) + xf * D.float().view(1, H, 1)
    return out


def draft_step(draft: torch.Tensor, slots, x, dt_raw, B, C, A, D, dt_bias,
               clamp_min: float | None = 1e-3, pad_slot_id: int = -1) -> torch.Tensor:
    """One token of the hot-only self-speculative draft on ``draft [S, H, P, pb]``: the
    reference's install(cold="off"), i.e. selective_state_update on the hot slice alone
    (scale/v4_fused_decode.py:49-55) with no cold read, ring or flush (:140-142).  Its y and
    hot evolution are those of the tiered step in mode "coldoff" (scale/v4_native_decode.py:
    118-127), which the golden fixtures pin."""
    pb = draft.shape[-1]
    return fresh_step(draft, slots, x, dt_raw, B[..., :pb], C[..., :pb], A, D, dt_bias, clamp_min, pad_slot_id)


def _check_window(pool: TieredPoolRef, slots, n: int, pad_slot_id: int):
    _, s = _valid_rows(slots, pad_slot_id)
    r = pool.t[s] % pool.c
    if bool((r + n > pool.c).any()):
        raise ValueError("a verify / commit window crosses a chunk boundary")


def verify_steps(pool: TieredPoolRef, slots, xs, dts, Bs, Cs, A, D, dt_bias, clamp_min: float | None = 1e-3,
                 pad_slot_id: int = -1, mode: str = "stale") -> torch.Tensor:
    """y [b, n, H, P] of n tokens (xs [b, n, H, P], dts [b, n, H], Bs / Cs [b, n, G, N]) read
    against the committed state exactly as n successive ``tiered_step`` calls would read them;
    the pool is left unchanged (the verify of the draft -> verify -> accept cycle that
    scale/bench_selfspec_e2e.py times)."""
    import copy
    n = xs.shape[1]
    _check_window(pool, slots, n, pad_slot_id)
    work = copy.deepcopy(pool)
    return torch.stack([tiered_step(work, slots, xs[:, j], dts[:, j], Bs[:, j], Cs[:, j], A, D, dt_bias,
                                    clamp_min, pad_slot_id, mode) for j in range(n)], dim=1)


def commit_steps(pool: TieredPoolRef, slots, accept, xs, dts, Bs, A, dt_bias, clamp_min: float | None = 1e-3,
                 pad_slot_id: int = -1) -> None:
    """Advance row i by its first ``accept[i]`` tokens: ``tiered_step`` on the rows that keep
    token j, for j = 0 .. n-1 (the state update does not depend on the readout mode)."""
    n = xs.shape[1]
    accept = torch.as_tensor(accept).reshape(-1)
    _check_window(pool, slots, 0, pad_slot_id)
    _, s = _valid_rows(slots, pad_slot_id)
    rows, _ = _valid_rows(slots, pad_slot_id)
    if bool(((pool.t[s] % pool.c) + accept[rows] > pool.c).any()):
        raise ValueError("a commit window crosses a chunk boundary")
    for j in range(n):
        sl = torch.as_tensor(slots).clone().reshape(-1)
        sl[accept <= j] = pad_slot_id
        tiered_step(pool, sl, xs[:, j], dts[:, j], Bs[:, j], Bs[:, j], A, torch.zeros_like(A), dt_bias, clamp_min,
                    pad_slot_id)


def materialize(pool: TieredPoolRef, slots, A) -> torch.Tensor:
    """Exact current full fp32 state ``[b, H, P, N]`` of each slot: hot slice plus
    the cold slice replayed through the partial ring (tokens since the last flush).
    Read-only.  This is the state the native path would hold."""
    rows, s = _valid_rows(slots, -1)
    H, P, pb, c, G = pool.H, pool.P, pool.pb, pool.c, pool.G
    HG = H // G
    out = torch.zeros(len(slots), H, P, pool.N)
    A = A.float()
    for i, si in zip(rows.tolist(), s.tolist()):
        k = int(pool.t[si]) % c                           # ring entries since the last flush
        cold = dequantize_rows(pool.cold[si], None if pool.scale is None else pool.scale[si])
        if k:
            dAs = pool.ring_dt[si, :, :k] * A.view(-1, 1)       # [H,k]
            tot = torch.zeros(H)
            for j in range(k):
                tot = tot + dAs[:, j]
            suf = torch.zeros_like(dAs)
            for j in range(k - 2, -1, -1):
                suf[:, j] = suf[:, j + 1] + dAs[:, j + 1]
            W = torch.exp(suf)[..., None] * (pool.ring_dt[si, :, :k, None] * pool.ring_x[si, :, :k].float())
            bsh = pool.ring_b[si, :, :k].float().repeat_interleave(HG, dim=0)  # [H,k,Nc]
            upd = torch.zeros_like(cold)
            for j in range(k):
                upd = upd + W[:, j, :, None] * bsh[:, j, None, :]
            cold = cold * torch.exp(tot)[:, None, None] + upd
        out[i, ..., :pb] = pool.hot[si]
        out[i, ..., pb:] = cold
    return out


# --------------------------------------------------------------------------
# synthetic inputs with the BASELINE distributions
# --------------------------------------------------------------------------
def make_params(H: int, G: int, N: int, seed: int = 0, layers: int = 1):
    """Per-layer parameters: A = -exp(U(0, log 16)), D ~ N(0,1),
    dt_bias = log(expm1(U(1e-3, 0.1))), R = per-group QR of a Gaussian."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(layers):
        A = -torch.exp(torch.rand(H, generator=g) * math.log(16.0))
        D = torch.randn(H, generator=g)
        u = torch.rand(H, generator=g) * (0.1 - 1e-3) + 1e-3
        dt_bias = torch.log(torch.expm1(u))
        R = torch.linalg.qr(torch.randn(G, N, N, generator=g))[0].contiguous()
        out.append(dict(A=A.float(), D=D.float(), dt_bias=dt_bias.float(), R=R.float()))
    return out


def make_inputs(b: int, H: int, P: int, G: int, N: int, steps: int, seed: int = 0,
                io_dtype=torch.bfloat16):
    """Per-step inputs: x ~ N(0,1), B/C ~ N(0, 1/N), dt_raw ~ N(0,1)."""
    g = torch.Generator().manual_seed(seed + 1)
    xs = torch.randn(steps, b, H, P, generator=g).to(io_dtype)
    Bs = (torch.randn(steps, b, G, N, generator=g) / math.sqrt(N)).to(io_dtype)
    Cs = (torch.randn(steps, b, G, N, generator=g) / math.sqrt(N)).to(io_dtype)
    dts = torch.randn(steps, b, H, generator=g).to(io_dtype)
    return xs, dts, Bs, Cs
