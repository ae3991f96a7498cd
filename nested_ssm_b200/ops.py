"""Functional API over the C ABI, with the reference's call surface.

* :func:`tiered_state_update` -- the tiered per-layer decode with continuous-batching
  ``state_batch_indices``; replaces vLLM ``selective_state_update`` + ``decode_readout``
  (scale/vllm_v4_patch.py:140-179) and the state-op part of ``_v4_fused_decode``
  (scale/v4_fused_decode.py:45-93).
* :func:`selective_state_update` -- the untiered fp32 update (the fresh control),
  mamba_ssm/vLLM argument order.
* :func:`prefill_snapshot` / :func:`prefill_split` -- scale/vllm_v4_patch.py:123-137.
* :func:`rot_flat` -- scale/vllm_v4_patch.py:41-45 (fp32 accumulation, cast back).
* :func:`materialize` -- exact full fp32 state of slots (read-only).

All tensors must live on the same CUDA device; work is enqueued on the current
stream and never synchronised.  There is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .pool import TieredSlotPool, nssm_dtype

MODES = {"stale": _lib.NSSM_MODE_STALE, "corr": _lib.NSSM_MODE_CORR, "coldoff": _lib.NSSM_MODE_COLDOFF}
DEFAULT_DT_MIN = 1e-3   # NemotronH time_step_min (scale/v4_native_decode.py:55)


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*ts):
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("nested_ssm_b200 ops take CUDA tensors only (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} vs {t.device}")
    return dev


def _per_head(v: torch.Tensor | None, H: int, name: str) -> torch.Tensor | None:
    """[H] fp32 contiguous from [H], [H, P] or [H, P, N] (expanded, as the SSU takes them)."""
    if v is None:
        return None
    while v.dim() > 1:
        v = v[..., 0]
    if v.numel() != H:
        raise ValueError(f"{name} must have {H} heads, got shape {tuple(v.shape)}")
    if v.dtype != torch.float32 or not v.is_contiguous():
        v = v.float().contiguous()
    return v


def _dt_2d(dt: torch.Tensor) -> torch.Tensor:
    if dt.dim() == 3:        # [b, H, P] expanded over P (the SSU layout)
        dt = dt[..., 0]
    if dt.dim() != 2:
        raise ValueError(f"dt must be [b, H] or [b, H, P], got {tuple(dt.shape)}")
    return dt


def _bc_2d(v: torch.Tensor, b: int) -> torch.Tensor:
    v = v.reshape(b, -1) if v.is_contiguous() else v
    if v.dim() == 3:
        if v.stride(2) != 1 or v.stride(1) != v.shape[2]:
            v = v.contiguous()
        return v
    if v.stride(-1) != 1:
        v = v.contiguous()
    return v


def build_step_args(x, dt, A, B, C_, D=None, dt_bias=None, dt_softplus=True,
                    state_batch_indices=None, pad_slot_id=-1, out=None, R=None,
                    dt_min=DEFAULT_DT_MIN, mode="stale", workspace=None, status=None,
                    nheads=None):
    """Validate and pack the per-token inputs into an ``nssm_step_args`` struct.

    Returns ``(args, out, keepalive)``; ``keepalive`` holds converted tensors that
    must outlive the launch."""
    if x.dim() != 3 or x.stride(2) != 1:
        raise ValueError(f"x must be [b, H, P] with unit inner stride, got {tuple(x.shape)}")
    b, H, P = x.shape
    if nheads is not None and H != nheads:
        raise ValueError(f"x has {H} heads, pool has {nheads}")
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"x dtype {x.dtype} unsupported (bf16 / fp32)")
    dt2 = _dt_2d(dt)
    if dt2.shape[0] != b or dt2.shape[1] != H:
        raise ValueError(f"dt shape {tuple(dt.shape)} does not match x {tuple(x.shape)}")
    if B.dtype != x.dtype or C_.dtype != x.dtype:
        raise ValueError("B and C must have x's dtype")
    B2, C2 = _bc_2d(B, b), _bc_2d(C_, b)
    A1 = _per_head(A, H, "A")
    D1 = _per_head(D, H, "D")
    db1 = _per_head(dt_bias, H, "dt_bias")
    if out is None:
        out = torch.empty(b, H, P, dtype=x.dtype, device=x.device)
    if out.shape != (b, H, P) or out.stride(2) != 1 or out.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"out must be [b, H, P] bf16/fp32 with unit inner stride, got {tuple(out.shape)} {out.dtype}")
    idx = None
    if state_batch_indices is not None:
        idx = state_batch_indices
        if idx.dim() > 1:      # vLLM non-cache-all decode passes [b, 1] (scale/vllm_v4_patch.py:151-152)
            idx = idx[:, -1]
        if idx.dtype != torch.int32 or not idx.is_contiguous():
            idx = idx.to(torch.int32).contiguous()
        if idx.numel() != b:
            raise ValueError(f"state_batch_indices has {idx.numel()} rows, x has {b}")
    Rf = None
    if R is not None:
        Rf = R if (R.dtype == torch.float32 and R.is_contiguous()) else R.float().contiguous()
    if mode not in MODES:
        raise ValueError(f"mode must be one of {sorted(MODES)}")
    _require_cuda(x, dt2, A1, B2, C2, D1, db1, out, idx, Rf)
    a = _lib.NssmStepArgs()
    a.batch = b
    a.io_dtype = nssm_dtype(x.dtype)
    a.x, a.x_stride_b, a.x_stride_h = x.data_ptr(), x.stride(0), x.stride(1)
    a.dt, a.dt_stride_b, a.dt_stride_h = dt2.data_ptr(), dt2.stride(0), dt2.stride(1)
    a.dt_dtype = nssm_dtype(dt2.dtype)
    a.dt_softplus = 1 if dt_softplus else 0
    a.A = A1.data_ptr()
    a.B, a.B_stride_b = B2.data_ptr(), B2.stride(0)
    a.C, a.C_stride_b = C2.data_ptr(), C2.stride(0)
    a.D = _ptr(D1)
    a.dt_bias = _ptr(db1)
    a.dt_min = float(dt_min) if dt_min is not None else 0.0
    a.mode = MODES[mode]
    a.R = _ptr(Rf)
    a.state_batch_indices = _ptr(idx)
    a.pad_slot_id = int(pad_slot_id)
    a.out_dtype = nssm_dtype(out.dtype)
    a.out, a.out_stride_b, a.out_stride_h = out.data_ptr(), out.stride(0), out.stride(1)
    if workspace is not None:
        a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    a.status = _ptr(status)
    keep = (x, dt2, A1, B2, C2, D1, db1, out, idx, Rf, workspace, status)
    return a, out, keep


def tiered_state_update(pool: TieredSlotPool, layer: int, x, dt, A, B, C_, D=None, dt_bias=None,
                        dt_softplus=True, state_batch_indices=None, pad_slot_id=-1, out=None,
                        R=None, dt_min=DEFAULT_DT_MIN, mode="stale"):
    """One decode token of one layer on the tiered pool; returns ``out`` [b, H, P].

    Rows whose slot is ``pad_slot_id`` are skipped (their ``out`` rows untouched).
    ``R`` ([G, N, N]) rotates B and C first (fp32 accumulation, cast back to x's dtype).
    """
    if x.dtype != pool.io_dtype:
        raise ValueError(f"x dtype {x.dtype} differs from the pool's io dtype {pool.io_dtype}")
    if R is not None and x.shape[0] > pool.max_batch:
        raise ValueError(f"batch {x.shape[0]} exceeds the pool's max_batch {pool.max_batch}")
    a, out, keep = build_step_args(x, dt, A, B, C_, D, dt_bias, dt_softplus, state_batch_indices,
                                   pad_slot_id, out, R, dt_min, mode, pool.workspace, pool.status,
                                   nheads=pool.H)
    lib = _lib.load()
    _lib.check(lib.nssm_tiered_step(C.byref(pool.struct(layer)), C.byref(a), _stream(x.device)))
    return out


def selective_state_update(state: torch.Tensor, x, dt, A, B, C_, D=None, z=None, dt_bias=None,
                           dt_softplus=True, state_batch_indices=None, pad_slot_id=-1, out=None,
                           R=None, dt_min=DEFAULT_DT_MIN, workspace=None):
    """Untiered fp32 update of ``state [S, H, P, N]`` in place (the fresh control)."""
    if z is not None:
        raise NotImplementedError("z gating is applied by the caller's gated norm")
    if state.dtype != torch.float32 or not state.is_contiguous() or state.dim() != 4:
        raise ValueError("state must be a contiguous fp32 [S, H, P, N] tensor")
    S, H, P, N = state.shape
    G = (B.shape[1] if B.dim() == 3 else B.shape[-1] // N)
    if R is not None and workspace is None:
        lib = _lib.load()
        wsb = lib.nssm_step_workspace_bytes(x.shape[0], G, N, nssm_dtype(x.dtype), 1)
        workspace = torch.empty(max(wsb, 256), dtype=torch.uint8, device=x.device)
    a, out, keep = build_step_args(x, dt, A, B, C_, D, dt_bias, dt_softplus, state_batch_indices,
                                   pad_slot_id, out, R, dt_min, "stale", workspace, None, nheads=H)
    _require_cuda(state, x)
    lib = _lib.load()
    _lib.check(lib.nssm_fresh_step(state.data_ptr(), S, H, P, N, G, C.byref(a), _stream(x.device)))
    return out


def prefill_split(pool: TieredSlotPool, layer: int, states: torch.Tensor, slots: torch.Tensor,
                  pad_slot_id: int = -1) -> None:
    """Row i of ``states [b, H, P, N]`` (fp32) -> pool slot ``slots[i]``: hot, quantised
    cold, glog = 0, t = 0 (scale/vllm_v4_patch.py:123-137)."""
    if states.dtype != torch.float32:
        states = states.float()
    if states.dim() != 4 or states.shape[1:] != (pool.H, pool.P, pool.N):
        raise ValueError(f"states must be [b, {pool.H}, {pool.P}, {pool.N}], got {tuple(states.shape)}")
    if states.stride(3) != 1 or states.stride(2) != pool.N or states.stride(1) != pool.P * pool.N:
        states = states.contiguous()
    slots = slots.reshape(-1).to(device=pool.device, dtype=torch.int32).contiguous()
    if slots.numel() != states.shape[0]:
        raise ValueError("slots and states disagree on the batch size")
    _require_cuda(states, slots)
    lib = _lib.load()
    _lib.check(lib.nssm_prefill_split(C.byref(pool.struct(layer)), states.data_ptr(), states.stride(0),
                                      slots.data_ptr(), slots.numel(), int(pad_slot_id),
                                      _stream(states.device)))


def prefill_snapshot(pool: TieredSlotPool, layer: int, ssm_state: torch.Tensor, slots: torch.Tensor) -> None:
    """vLLM-style: ``ssm_state`` is the full cache ``[S, H, P, N]`` already holding the
    prefill's final states at ``slots`` (scale/vllm_v4_patch.py:123-137)."""
    slots = slots.reshape(-1)
    prefill_split(pool, layer, ssm_state[slots.to(ssm_state.device, torch.long)], slots)


def materialize(pool: TieredSlotPool, layer: int, slots: torch.Tensor, A: torch.Tensor,
                out: torch.Tensor | None = None, pad_slot_id: int = -1) -> torch.Tensor:
    """Exact current full fp32 state ``[b, H, P, N]`` of each slot (read-only)."""
    slots = slots.reshape(-1).to(device=pool.device, dtype=torch.int32).contiguous()
    A1 = _per_head(A.to(pool.device), pool.H, "A")
    if out is None:
        out = torch.zeros(slots.numel(), pool.H, pool.P, pool.N, device=pool.device)
    lib = _lib.load()
    _lib.check(lib.nssm_materialize(C.byref(pool.struct(layer)), A1.data_ptr(), slots.data_ptr(),
                                    slots.numel(), int(pad_slot_id), out.data_ptr(), out.stride(0),
                                    _stream(pool.device)))
    return out


def rot_flat(x: torch.Tensor, R: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``x [T, G*N]`` (or ``[T, G, N]``) rotated per group by ``R [G, N, N]``: fp32
    accumulation, rounded to x's dtype (scale/vllm_v4_patch.py:41-45 / v4_fused_decode.py:47)."""
    G, N, _ = R.shape
    T = x.shape[0]
    x2 = x.reshape(T, G * N) if x.is_contiguous() else x.contiguous().reshape(T, G * N)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    Rf = R.float().contiguous()
    if out is None:
        out = torch.empty(T, G * N, dtype=x.dtype, device=x.device)
    _require_cuda(x2, Rf, out)
    lib = _lib.load()
    _lib.check(lib.nssm_rot_flat(x2.data_ptr(), x2.stride(0), nssm_dtype(x.dtype), Rf.data_ptr(), T, G, N,
                                 out.data_ptr(), out.stride(0), _stream(x.device)))
    return out.view(x.shape) if out.shape != x.shape and out.numel() == x.numel() else out
