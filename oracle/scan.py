"""TEST INFRASTRUCTURE ONLY -- CPU oracle for the prefill chunked scan.

The reference's memory-lean prefill (``scale/v4_native_decode.py:175-220``, ``_lean_prefill``)
runs the conv, rotates B and C, and calls the third-party ``mamba_chunk_scan_combined`` of
mamba_ssm 2.3.2.post1 (``mamba_ssm/ops/triton/ssd_combined.py``; the pinned version of
the reference's ``mamba_ssm_build.log``) with ``z=None``, ``dt_softplus=True``,
``initial_states=None``, ``dt_limit=mixer.time_step_limit`` and ``return_final_states``.
mamba_ssm is not installed here, so its published algorithm is restated:

* ``_chunk_cumsum_fwd``: ``dt = dt + dt_bias``; ``softplus`` where ``dt <= 20``; clamp to
  ``dt_limit``; zero past the sequence end; ``dA_cs = cumsum(dt * A)`` inside each chunk.
* ``_chunk_state_fwd``: ``B_s = (B * exp(dA_cs[last] - dA_cs) * dt)`` rounded to the input
  dtype; ``states[p, n] = sum_s x[s, p] B_s[s, n]`` accumulated in fp32.
* ``_state_passing_fwd``: ``S = exp(dA_cs[last]) * S + states`` in fp32; the state entering
  each chunk is stored in the input dtype (``out_dtype=C.dtype``), the final one in fp32.
* ``_bmm_chunk_fwd``: ``CB = C B^T`` in fp32.
* ``_chunk_scan_fwd``: ``y = (C . S_prev) * exp(dA_cs[l])`` plus ``sum_s M[l, s] x[s]`` with
  ``M = (CB * exp(dA_cs[l] - dA_cs[s]) * dt[s])`` masked to ``s <= l`` and rounded to the input
  dtype; ``y += D x``; stored in the input dtype.

``rounding=False`` keeps every operand in fp32; that is the HF ``torch_forward`` prefill
(transformers' NemotronH mixer, the reference's ``_orig_forward`` and its prefill when
``lean_prefill=0``) up to fp32 reassociation, and what ``tests/golden/make_golden.py`` pins.
``scan_recurrent`` is the token-by-token recurrence the chunked form factorises.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

__all__ = ["scan_dt", "chunk_scan", "scan_recurrent"]


def scan_dt(dt, dt_bias=None, dt_softplus=False, dt_limit=(0.0, math.inf)):
    """fp32 dt of ``_chunk_cumsum_fwd``: bias, softplus (threshold 20), clamp to dt_limit."""
    d = dt.float()
    if dt_bias is not None:
        d = d + dt_bias.float().view(*([1] * (d.dim() - 1)), -1)
    if dt_softplus:
        d = torch.where(d <= 20.0, F.softplus(d), d)
    return d.clamp(float(dt_limit[0]), float(dt_limit[1]))


def chunk_scan(x, dt, A, B, C, chunk_size=128, D=None, dt_bias=None, initial_states=None, dt_softplus=False,
               dt_limit=(0.0, math.inf), rounding=True):
    """Chunked SSD scan of one layer (restated ``mamba_chunk_scan_combined`` forward).

    x [b, T, H, P], dt [b, T, H] (pre-bias), A [H], B / C [b, T, G, N], D [H] or None,
    initial_states [b, H, P, N] or None.  Returns (y [b, T, H, P] in x's dtype when
    ``rounding`` else fp32, final state [b, H, P, N] fp32).
    """
    b, T, H, P = x.shape
    G, N = B.shape[2], B.shape[3]
    rd = x.dtype if rounding else torch.float32

    def r(t):
        return t.to(rd).float()

    xf, Bf, Cf = x.float(), B.float(), C.float()
    Af = A.float().view(1, 1, H)
    d_all = scan_dt(dt, dt_bias, dt_softplus, dt_limit)
    Bh = Bf.repeat_interleave(H // G, dim=2)
    Ch = Cf.repeat_interleave(H // G, dim=2)
    S = torch.zeros(b, H, P, N) if initial_states is None else initial_states.float().clone()
    y = torch.empty(b, T, H, P)
    for c0 in range(0, T, chunk_size):
        c1 = min(c0 + chunk_size, T)
        L = c1 - c0
        d = d_all[:, c0:c1]                                       # [b, L, H]
        cs = torch.cumsum(d * Af, dim=1)                          # dA_cs
        last = cs[:, -1]                                          # [b, H]
        xc, Bc, Cc = xf[:, c0:c1], Bh[:, c0:c1], Ch[:, c0:c1]
        # _chunk_state_fwd
        sc = torch.exp(last[:, None] - cs) * d
        Bs = r(Bc * sc[..., None])
        Sc = torch.einsum("blhp,blhn->bhpn", xc, Bs)
        # _chunk_scan_fwd, off-diagonal: the state entering the chunk, stored in the input dtype
        yoff = torch.einsum("blhn,bhpn->blhp", Cc, r(S)) * torch.exp(cs)[..., None]
        # _bmm_chunk_fwd + the diagonal block
        CB = torch.einsum("blhn,bshn->bhls", Cc, Bc)
        csh = cs.permute(0, 2, 1)                                 # [b, H, L]
        seg = csh[..., :, None] - csh[..., None, :]
        causal = torch.ones(L, L, dtype=torch.bool).tril()
        M = CB * torch.exp(torch.where(causal, seg, torch.zeros(())))
        M = M * d.permute(0, 2, 1)[..., None, :]
        M = r(torch.where(causal, M, torch.zeros(())))
        yc = yoff + torch.einsum("bhls,bshp->blhp", M, xc)
        if D is not None:
            yc = yc + xc * D.float().view(1, 1, H, 1)
        y[:, c0:c1] = yc
        # _state_passing_fwd
        S = torch.exp(last)[..., None, None] * S + Sc
    return (y.to(rd) if rounding else y), S


def scan_recurrent(x, dt, A, B, C, D=None, dt_bias=None, initial_states=None, dt_softplus=False,
                   dt_limit=(0.0, math.inf)):
    """Token-by-token fp32 recurrence ``h <- exp(dt A) h + dt x B^T``, ``y = h C + D x``."""
    b, T, H, P = x.shape
    G, N = B.shape[2], B.shape[3]
    d_all = scan_dt(dt, dt_bias, dt_softplus, dt_limit)
    Bh = B.float().repeat_interleave(H // G, dim=2)
    Ch = C.float().repeat_interleave(H // G, dim=2)
    h = torch.zeros(b, H, P, N) if initial_states is None else initial_states.float().clone()
    y = torch.empty(b, T, H, P)
    for t in range(T):
        d = d_all[:, t]                                           # [b, H]
        h = torch.exp(d * A.float().view(1, H))[..., None, None] * h + \
            (d[..., None] * x[:, t].float())[..., None] * Bh[:, t, :, None, :]
        yt = torch.einsum("bhpn,bhn->bhp", h, Ch[:, t])
        if D is not None:
            yt = yt + x[:, t].float() * D.float().view(1, H, 1)
        y[:, t] = yt
    return y, h
