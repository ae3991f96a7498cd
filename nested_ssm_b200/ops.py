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
* :func:`draft_state_update` / :func:`verify_state_update` / :func:`commit_state_update` --
  self-speculative decoding: the hot-only draft (install(cold="off"),
  scale/v4_fused_decode.py:49-55 and :140-142) and the draft -> verify -> accept cycle that
  scale/bench_selfspec_e2e.py times, on the tiered state.
* :func:`mamba_chunk_scan_combined` -- the prefill chunked scan of the lean prefill
  (scale/v4_native_decode.py:209-216), mamba_ssm's argument order; its final states feed
  :func:`prefill_split`.

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
                        R=None, dt_min=DEFAULT_DT_MIN, mode="stale", norm=None):
    """One decode token of one layer on the tiered pool; returns ``out`` [b, H, P].

    Rows whose slot is ``pad_slot_id`` are skipped (their ``out`` rows untouched).
    ``R`` ([G, N, N]) rotates B and C first (fp32 accumulation, cast back to x's dtype).
    ``norm = (gate [b, H*P], weight [H*P], eps)``: ``out`` receives the mixer's gated RMS norm
    of y instead of y (scale/v4_native_decode.py:171; the same result as ``gated_rmsnorm`` on
    the step's y), fused into the step; the norm group is one SSM group of a row, H/G*P
    channels, and ``out`` must have x's dtype.
    """
    if x.dtype != pool.io_dtype:
        raise ValueError(f"x dtype {x.dtype} differs from the pool's io dtype {pool.io_dtype}")
    if R is not None and x.shape[0] > pool.max_batch:
        raise ValueError(f"batch {x.shape[0]} exceeds the pool's max_batch {pool.max_batch}")
    a, out, keep = build_step_args(x, dt, A, B, C_, D, dt_bias, dt_softplus, state_batch_indices,
                                   pad_slot_id, out, R, dt_min, mode, pool.workspace, pool.status,
                                   nheads=pool.H)
    if norm is not None:
        gate, weight, eps = norm
        b = x.shape[0]
        g2 = gate.reshape(b, -1)
        if g2.shape[1] != pool.H * pool.P or g2.stride(-1) != 1 or g2.dtype != out.dtype:
            raise ValueError(f"norm gate must be [b, {pool.H * pool.P}] in out's dtype with a unit inner stride")
        w = weight if weight.is_contiguous() else weight.contiguous()
        if w.numel() != pool.H * pool.P or w.dtype not in (torch.bfloat16, torch.float32):
            raise ValueError("norm weight must have H*P bf16 / fp32 entries")
        _require_cuda(g2, w)
        a.norm_gate, a.norm_gate_stride_b = g2.data_ptr(), g2.stride(0)
        a.norm_weight, a.norm_weight_dtype = w.data_ptr(), nssm_dtype(w.dtype)
        a.norm_group_size = (pool.H // pool.G) * pool.P
        a.norm_eps = float(eps)
        keep = keep + (g2, w)
    lib = _lib.load()
    _lib.check(lib.nssm_tiered_step(C.byref(pool.struct(layer)), C.byref(a), _stream(x.device)))
    return out


def draft_state_update(pool: TieredSlotPool, layer: int, draft: torch.Tensor, x, dt, A, B, C_, D=None,
                       dt_bias=None, dt_softplus=True, state_batch_indices=None, pad_slot_id=-1, out=None,
                       R=None, dt_min=DEFAULT_DT_MIN, from_pool=False):
    """One token of the hot-only draft model (the reference's install(cold="off"): the SSU on
    the hot slice alone, scale/v4_fused_decode.py:49-55, :140-142); returns ``out`` [b, H, P].

    ``draft`` is this layer's draft state, fp32 [S, H, P, hot_dim] indexed by slot
    (``pool.new_draft()[layer]``).  ``from_pool=True`` (the cycle's first draft token) starts
    from the pool's committed hot slice; otherwise the draft state is advanced in place.
    ``y = C_hot . h + D x``; the pool itself is not written."""
    if x.dtype != pool.io_dtype:
        raise ValueError(f"x dtype {x.dtype} differs from the pool's io dtype {pool.io_dtype}")
    if draft.dtype != torch.float32 or not draft.is_contiguous() or tuple(draft.shape) != tuple(pool.hot.shape[1:]):
        raise ValueError(f"draft must be contiguous fp32 {tuple(pool.hot.shape[1:])}")
    if R is not None and x.shape[0] > pool.max_batch:
        raise ValueError(f"batch {x.shape[0]} exceeds the pool's max_batch {pool.max_batch}")
    a, out, keep = build_step_args(x, dt, A, B, C_, D, dt_bias, dt_softplus, state_batch_indices,
                                   pad_slot_id, out, R, dt_min, "stale", pool.workspace, pool.status,
                                   nheads=pool.H)
    _require_cuda(x, draft)
    lib = _lib.load()
    _lib.check(lib.nssm_draft_step(C.byref(pool.struct(layer)), draft.data_ptr(), 1 if from_pool else 0,
                                   C.byref(a), _stream(x.device)))
    return out


def _token_inputs(pool, x, dt, B, C_, out, want_out=True):
    """Token-0 views and token strides of multi-token inputs x [b, n, H, P], dt [b, n, H]
    (or [b, n, H, P] expanded), B / C [b, n, G, N] or [b, n, G*N], out [b, n, H, P]."""
    if x.dim() != 4 or x.stride(3) != 1:
        raise ValueError(f"x must be [b, n, H, P] with unit inner stride, got {tuple(x.shape)}")
    b, n = x.shape[:2]
    if dt.dim() == 4:
        dt = dt[..., 0]
    if dt.dim() != 3 or tuple(dt.shape[:2]) != (b, n):
        raise ValueError(f"dt must be [b, n, H], got {tuple(dt.shape)}")
    bc = []
    for name, v in (("B", B), ("C", C_)):
        if v is None:
            bc.append(None)
            continue
        if v.dim() == 4:
            if v.stride(3) != 1 or v.stride(2) != v.shape[3]:
                v = v.contiguous()
            v = v.reshape(b, n, -1) if v.is_contiguous() else v.flatten(2)
        if v.dim() != 3 or tuple(v.shape[:2]) != (b, n) or v.stride(2) != 1:
            raise ValueError(f"{name} must be [b, n, G, N] or [b, n, G*N], got {tuple(v.shape)}")
        bc.append(v)
    if not want_out:
        return dt, bc[0], bc[1], None
    if out is None:
        out = torch.empty(b, n, pool.H, pool.P, dtype=x.dtype, device=x.device)
    if out.dim() != 4 or tuple(out.shape[:2]) != (b, n):
        raise ValueError(f"out must be [b, n, H, P], got {tuple(out.shape)}")
    return dt, bc[0], bc[1], out


def _token_struct(n, x, dt, B, C_, out, accept=None):
    t = _lib.NssmTokenArgs()
    t.ntok = n
    t.x_stride_t, t.dt_stride_t = x.stride(1), dt.stride(1)
    t.B_stride_t = B.stride(1)
    t.C_stride_t = C_.stride(1) if C_ is not None else 0
    t.out_stride_t = out.stride(1) if out is not None else 0
    t.accept = _ptr(accept)
    return t


def _spec_workspace(pool, b, n, with_rot):
    lib = _lib.load()
    nbytes = lib.nssm_spec_workspace_bytes(b, n, pool.G, pool.N, nssm_dtype(pool.io_dtype), 1 if with_rot else 0)
    return torch.empty(max(nbytes, 256), dtype=torch.uint8, device=pool.device)


def verify_state_update(pool: TieredSlotPool, layer: int, x, dt, A, B, C_, D=None, dt_bias=None,
                        dt_softplus=True, state_batch_indices=None, pad_slot_id=-1, out=None, R=None,
                        dt_min=DEFAULT_DT_MIN, mode="stale"):
    """y of n drafted tokens per row from the committed tiered state, as n successive
    :func:`tiered_state_update` calls would give them; returns ``out`` [b, n, H, P].  Read-only
    on the pool.  x [b, n, H, P], dt [b, n, H], B / C [b, n, G, N]; every row needs
    ``t % c + n <= c`` (checked on the device: bit 2 of the pool's status).  Modes "stale" and
    "coldoff"."""
    if x.dtype != pool.io_dtype:
        raise ValueError(f"x dtype {x.dtype} differs from the pool's io dtype {pool.io_dtype}")
    dt, B3, C3, out = _token_inputs(pool, x, dt, B, C_, out)
    b, n = x.shape[:2]
    ws = _spec_workspace(pool, b, n, R is not None)
    a, _, keep = build_step_args(x[:, 0], dt[:, 0], A, B3[:, 0], C3[:, 0], D, dt_bias, dt_softplus,
                                 state_batch_indices, pad_slot_id, out[:, 0], R, dt_min, mode, ws, pool.status,
                                 nheads=pool.H)
    t = _token_struct(n, x, dt, B3, C3, out)
    lib = _lib.load()
    _lib.check(lib.nssm_verify_step(C.byref(pool.struct(layer)), C.byref(a), C.byref(t), _stream(x.device)))
    return out


def commit_state_update(pool: TieredSlotPool, layer: int, accept, x, dt, A, B, dt_bias=None, dt_softplus=True,
                        state_batch_indices=None, pad_slot_id=-1, R=None, dt_min=DEFAULT_DT_MIN) -> None:
    """Make the first ``accept[b]`` of the n verified tokens of row b permanent: the pool ends
    exactly as after ``accept[b]`` :func:`tiered_state_update` calls with those inputs (hot
    slice, ring, glog, t, and the flush when they complete a chunk).  ``accept`` int32 [b] on
    the device, each in 0..n; x, dt, B and R as given to :func:`verify_state_update`."""
    if x.dtype != pool.io_dtype:
        raise ValueError(f"x dtype {x.dtype} differs from the pool's io dtype {pool.io_dtype}")
    dt, B3, _, _ = _token_inputs(pool, x, dt, B, None, None, want_out=False)
    b, n = x.shape[:2]
    acc = accept if (accept.dtype == torch.int32 and accept.is_contiguous()) else accept.to(torch.int32).contiguous()
    if acc.numel() != b:
        raise ValueError(f"accept has {acc.numel()} entries, x has {b} rows")
    ws = _spec_workspace(pool, b, n, R is not None)
    dummy = torch.empty(b, pool.H, pool.P, dtype=x.dtype, device=x.device)   # out is not written
    a, _, keep = build_step_args(x[:, 0], dt[:, 0], A, B3[:, 0], B3[:, 0], None, dt_bias, dt_softplus,
                                 state_batch_indices, pad_slot_id, dummy, R, dt_min, "stale", ws, pool.status,
                                 nheads=pool.H)
    _require_cuda(acc)
    t = _token_struct(n, x, dt, B3, B3, None, acc)
    t.C_stride_t = t.B_stride_t
    lib = _lib.load()
    _lib.check(lib.nssm_commit_step(C.byref(pool.struct(layer)), C.byref(a), C.byref(t), _stream(x.device)))


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


ACTIVATIONS = {None: 0, "none": 0, "identity": 0, "silu": 1, "swish": 1}


def conv_step(xbc: torch.Tensor, conv_state: torch.Tensor, weight: torch.Tensor, bias=None,
              activation="silu", conv_state_indices=None, pad_slot_id: int = -1, R=None, *,
              nheads: int, headdim: int, ngroups: int, dstate: int = 128,
              x_out=None, B_out=None, C_out=None, status=None):
    """Decode-token conv of one layer ahead of the state update: the causal conv1d update
    of ``xbc [b, conv_dim]`` (the in_proj slice [x | B | C]) with ``conv_state
    [num_slots, conv_dim, L]`` (updated in place, rows by ``conv_state_indices``; L
    innermost, or channels-last as the HF cache keeps it), the activation, the split, and
    the rotation of B and C by ``R [G, N, N]``.

    Replaces ``causal_conv1d_update`` + split + the R einsums of
    scale/v4_fused_decode.py:39-48.  Returns ``(x [b, H, P], B [b, G, N], C [b, G, N])`` in
    xbc's dtype, ready for :func:`tiered_state_update` with ``R=None``."""
    if xbc.dim() != 2 or xbc.stride(1) != 1:
        raise ValueError(f"xbc must be [b, conv_dim] with unit inner stride, got {tuple(xbc.shape)}")
    b, conv_dim = xbc.shape
    I, GN = nheads * headdim, ngroups * dstate
    if conv_dim != I + 2 * GN:
        raise ValueError(f"conv_dim {conv_dim} != nheads*headdim + 2*ngroups*dstate = {I + 2 * GN}")
    if xbc.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"xbc dtype {xbc.dtype} unsupported (bf16 / fp32)")
    if conv_state.dim() != 3 or conv_state.shape[1] != conv_dim or conv_state.dtype != xbc.dtype:
        raise ValueError(f"conv_state must be [S, {conv_dim}, L] of xbc's dtype, got {tuple(conv_state.shape)} "
                         f"{conv_state.dtype}")
    L = conv_state.shape[2]
    if not ((conv_state.stride(2) == 1 and conv_state.stride(1) == L)          # [S, conv_dim, L]
            or (conv_state.stride(1) == 1 and conv_state.stride(2) >= conv_dim)):   # channels-last (HF cache)
        raise ValueError("conv_state must be laid out [S, conv_dim, L] (L innermost) or channels-last")
    w = weight.reshape(weight.shape[0], -1) if weight.dim() == 3 else weight     # HF conv1d [D, 1, K]
    if w.dim() != 2 or w.shape[0] != conv_dim or not w.is_contiguous() or w.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"weight must be a contiguous [{conv_dim}, K] (or [{conv_dim}, 1, K]) bf16 / fp32 tensor")
    if bias is not None and (bias.shape != (conv_dim,) or bias.dtype != w.dtype or not bias.is_contiguous()):
        raise ValueError(f"bias must be a contiguous [{conv_dim}] tensor of weight's dtype")
    if activation not in ACTIVATIONS:
        raise ValueError(f"activation must be one of {sorted(k for k in ACTIVATIONS if k)}")
    idx = None
    if conv_state_indices is not None:
        idx = conv_state_indices.reshape(-1)
        if idx.dtype != torch.int32 or not idx.is_contiguous():
            idx = idx.to(torch.int32).contiguous()
        if idx.numel() != b:
            raise ValueError(f"conv_state_indices has {idx.numel()} rows, xbc has {b}")
    Rf = None
    if R is not None:
        Rf = R if (R.dtype == torch.float32 and R.is_contiguous()) else R.float().contiguous()
    dev = _require_cuda(xbc, conv_state, w, bias, idx, Rf)
    if x_out is None:
        x_out = torch.empty(b, nheads, headdim, dtype=xbc.dtype, device=dev)
    if B_out is None:
        B_out = torch.empty(b, ngroups, dstate, dtype=xbc.dtype, device=dev)
    if C_out is None:
        C_out = torch.empty(b, ngroups, dstate, dtype=xbc.dtype, device=dev)
    for t, name in ((x_out, "x_out"), (B_out, "B_out"), (C_out, "C_out")):
        if t.dtype != xbc.dtype or not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous with xbc's dtype")
    a = _lib.NssmConvArgs()
    a.batch, a.nheads, a.headdim, a.ngroups, a.dstate = b, nheads, headdim, ngroups, dstate
    a.width, a.state_len, a.num_slots = w.shape[1], conv_state.shape[2], conv_state.shape[0]
    a.io_dtype, a.weight_dtype = nssm_dtype(xbc.dtype), nssm_dtype(w.dtype)
    a.activation = ACTIVATIONS[activation]
    a.pad_slot_id = int(pad_slot_id)
    a.xbc, a.xbc_stride_b = xbc.data_ptr(), xbc.stride(0)
    a.conv_state, a.state_stride_s = conv_state.data_ptr(), conv_state.stride(0)
    a.state_stride_d, a.state_stride_l = conv_state.stride(1), conv_state.stride(2)
    a.weight, a.bias, a.R = w.data_ptr(), _ptr(bias), _ptr(Rf)
    a.state_batch_indices = _ptr(idx)
    a.x_out, a.x_out_stride_b = x_out.data_ptr(), I
    a.B_out, a.C_out, a.bc_out_stride_b = B_out.data_ptr(), C_out.data_ptr(), GN
    a.status = _ptr(status)
    keep = (xbc, conv_state, w, bias, idx, Rf, x_out, B_out, C_out, status)  # noqa: F841
    _lib.check(_lib.load().nssm_conv_step(C.byref(a), _stream(dev)))
    return x_out, B_out, C_out


def gated_rmsnorm(y: torch.Tensor, gate: torch.Tensor, weight: torch.Tensor, eps: float, group_size: int,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """The NemotronH mixer's ``norm(y, gate)`` in one launch: ``h = y * silu(gate)``, per group
    of ``group_size`` channels ``h / sqrt(mean(h^2) + eps)``, rounded to y's dtype, times
    ``weight`` (transformers Zamba2RMSNormGated; scale/nemotron_retrofit.py:146-161).
    ``y``, ``gate``: ``[..., dim]``; returns the same shape in y's dtype."""
    shape = y.shape
    dim = shape[-1]
    y2 = y.reshape(-1, dim)
    g2 = gate.reshape(-1, dim)
    if y2.stride(-1) != 1 or g2.stride(-1) != 1:
        raise ValueError("y and gate need a unit inner stride")
    if y.dtype not in (torch.bfloat16, torch.float32) or gate.dtype != y.dtype:
        raise ValueError("y and gate must share a bf16 / fp32 dtype")
    w = weight if weight.is_contiguous() else weight.contiguous()
    if w.numel() != dim or w.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"weight must have {dim} bf16 / fp32 entries")
    dev = _require_cuda(y2, g2, w)
    if out is None:
        out = torch.empty(y2.shape, dtype=y.dtype, device=dev)
    o2 = out.reshape(-1, dim)
    _lib.check(_lib.load().nssm_gated_rmsnorm(y2.data_ptr(), y2.stride(0), g2.data_ptr(), g2.stride(0), w.data_ptr(),
                                              nssm_dtype(w.dtype), float(eps), y2.shape[0], dim, int(group_size),
                                              nssm_dtype(y.dtype), o2.data_ptr(), o2.stride(0), _stream(dev)))
    return out.reshape(shape)


def mamba_chunk_scan_combined(x, dt, A, B, C_, chunk_size, D=None, z=None, dt_bias=None, initial_states=None,
                              seq_idx=None, cu_seqlens=None, dt_softplus=False, dt_limit=(0.0, float("inf")),
                              return_final_states=False, *, out=None, final_states=None, status=None):
    """Prefill chunked scan of one layer with mamba_ssm's call surface (as the reference's
    lean prefill makes it, scale/v4_native_decode.py:209-216): ``x [b, T, H, P]``,
    ``dt [b, T, H]`` (before bias and softplus), ``A [H]``, ``B``/``C_ [b, T, G, N]`` in bf16,
    ``D``/``dt_bias [H]``, ``initial_states [b, H, P, N]`` or None.  Returns ``y [b, T, H, P]``
    (bf16), and with ``return_final_states`` also the fp32 ``[b, H, P, N]`` final states.
    ``z``, ``seq_idx`` and ``cu_seqlens`` are not supported (the reference passes none)."""
    if z is not None or seq_idx is not None or cu_seqlens is not None:
        raise NotImplementedError("z / seq_idx / cu_seqlens are not supported by the chunk scan")
    if x.dim() != 4 or dt.dim() != 3 or B.dim() != 4 or C_.dim() != 4:
        raise ValueError("x [b, T, H, P], dt [b, T, H], B / C [b, T, G, N] expected")
    b, T, H, P = x.shape
    G, N = B.shape[2], B.shape[3]
    if dt.shape != (b, T, H) or B.shape != (b, T, G, N) or C_.shape != (b, T, G, N):
        raise ValueError(f"shape mismatch: x {tuple(x.shape)} dt {tuple(dt.shape)} B {tuple(B.shape)} "
                         f"C {tuple(C_.shape)}")
    if x.dtype != torch.bfloat16 or B.dtype != torch.bfloat16 or C_.dtype != torch.bfloat16:
        raise ValueError("x, B and C must be bf16")
    if dt.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("dt must be bf16 or fp32")
    if D is not None and D.dim() > 1:
        raise NotImplementedError("D with a headdim axis is not supported (D must be [H])")

    def rows(t, inner):   # unit innermost stride and packed inner dims
        if t.stride(-1) != 1 or (t.dim() == 4 and t.stride(2) != inner):
            t = t.contiguous()
        return t

    x, B, C_ = rows(x, P), rows(B, N), rows(C_, N)
    if dt.stride(-1) != 1:
        dt = dt.contiguous()
    Af, Df, bf = _per_head(A, H, "A"), _per_head(D, H, "D"), _per_head(dt_bias, H, "dt_bias")
    init = None
    if initial_states is not None:
        if initial_states.shape != (b, H, P, N):
            raise ValueError(f"initial_states must be [{b}, {H}, {P}, {N}]")
        init = initial_states.float().contiguous()
    dev = _require_cuda(x, dt, Af, B, C_, Df, bf, init)
    if out is None:
        out = torch.empty(b, T, H, P, dtype=torch.bfloat16, device=dev)
    if out.shape != (b, T, H, P) or out.dtype != torch.bfloat16 or out.stride(-1) != 1 or out.stride(2) != P:
        raise ValueError("out must be bf16 [b, T, H, P] with packed (H, P)")
    if return_final_states and final_states is None:
        final_states = torch.empty(b, H, P, N, dtype=torch.float32, device=dev)
    if final_states is not None and (final_states.shape != (b, H, P, N) or final_states.dtype != torch.float32
                                     or not final_states[0].is_contiguous()):
        raise ValueError("final_states must be fp32 [b, H, P, N] with contiguous rows")
    a = _lib.NssmScanArgs()
    a.batch, a.seqlen, a.nheads, a.headdim, a.ngroups, a.dstate = b, T, H, P, G, N
    a.chunk_size, a.io_dtype = int(chunk_size), _lib.NSSM_BF16
    a.x, a.x_stride_b, a.x_stride_t = x.data_ptr(), x.stride(0), x.stride(1)
    a.dt, a.dt_stride_b, a.dt_stride_t = dt.data_ptr(), dt.stride(0), dt.stride(1)
    a.dt_dtype, a.dt_softplus = nssm_dtype(dt.dtype), int(bool(dt_softplus))
    a.dt_min, a.dt_max = float(dt_limit[0]), float(dt_limit[1])
    a.A, a.D, a.dt_bias = Af.data_ptr(), _ptr(Df), _ptr(bf)
    a.B, a.B_stride_b, a.B_stride_t = B.data_ptr(), B.stride(0), B.stride(1)
    a.C, a.C_stride_b, a.C_stride_t = C_.data_ptr(), C_.stride(0), C_.stride(1)
    a.initial_states, a.init_stride_b = _ptr(init), (H * P * N)
    a.y, a.y_stride_b, a.y_stride_t = out.data_ptr(), out.stride(0), out.stride(1)
    a.final_states = _ptr(final_states)
    a.final_stride_b = final_states.stride(0) if final_states is not None else 0
    a.status = _ptr(status)
    keep = (x, dt, Af, B, C_, Df, bf, init, out, final_states, status)  # noqa: F841
    _lib.check(_lib.load().nssm_chunk_scan(C.byref(a), _stream(dev)))
    return (out, final_states) if return_final_states else out
