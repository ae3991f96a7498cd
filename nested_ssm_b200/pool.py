"""Tiered slot pool: the per-layer device buffers the C-ABI kernels update in place.

Ownership follows the reference's preallocation (scale/v4_fused_decode.py:129-137,
scale/vllm_v4_patch.py:90-103): every buffer is allocated once here, with a
leading layer axis, and the kernels never allocate.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib

COLD_DTYPES = {
    "fp8": (torch.float8_e4m3fn, _lib.NSSM_F8E4M3),
    "bf16": (torch.bfloat16, _lib.NSSM_BF16),
    "fp32": (torch.float32, _lib.NSSM_F32),
}
IO_DTYPES = {torch.bfloat16: _lib.NSSM_BF16, torch.float32: _lib.NSSM_F32}


def nssm_dtype(t: torch.dtype) -> int:
    if t in IO_DTYPES:
        return IO_DTYPES[t]
    raise ValueError(f"dtype {t} is not supported (bf16 or fp32)")


def _zeros(shape, dtype, device):
    if dtype == torch.float8_e4m3fn:
        return torch.zeros(shape, dtype=torch.uint8, device=device).view(dtype)
    return torch.zeros(shape, dtype=dtype, device=device)


class TieredSlotPool:
    """Per-layer tiered state for ``num_slots`` continuous-batching slots.

    Buffers (leading axis = layer):
      hot [L,S,H,P,pb] f32, cold [L,S,H,P,N-pb] (fp8|bf16|fp32), scale [L,S,H,P] f32 (fp8),
      glog [L,S,H] f32, t [L,S,H] i32, ring_x [L,S,H,c,P] io, ring_dt [L,S,H,round_up(c,4)] f32,
      ring_b [L,S,G,c,N-pb] f32 (the group's rotated B_cold of each chunk token; exact copies).
    """

    def __init__(self, num_layers: int, num_slots: int, nheads: int = 128, headdim: int = 80,
                 dstate: int = 128, ngroups: int = 8, hot_dim: int = 32, chunk: int = 4,
                 cold: str = "fp8", io_dtype: torch.dtype = torch.bfloat16,
                 device: torch.device | str | None = None, max_batch: int | None = None):
        if cold not in COLD_DTYPES:
            raise ValueError(f"cold must be one of {sorted(COLD_DTYPES)}, got {cold!r}")
        if not 0 < hot_dim < dstate:
            raise ValueError(f"hot_dim {hot_dim} must be in (0, {dstate})")
        if nheads % ngroups:
            raise ValueError(f"nheads {nheads} not divisible by ngroups {ngroups}")
        device = torch.device(device if device is not None else "cuda")
        if device.type != "cuda":
            raise RuntimeError("TieredSlotPool lives on a CUDA device (no CPU fallback)")
        self.L, self.S, self.H, self.P, self.N, self.G = num_layers, num_slots, nheads, headdim, dstate, ngroups
        self.pb, self.c, self.cold_kind = hot_dim, chunk, cold
        self.Nc = dstate - hot_dim
        self.io_dtype = io_dtype
        self.device = device
        cdt, self.cold_code = COLD_DTYPES[cold]
        L, S, H, P, G, Nc, c = self.L, self.S, self.H, self.P, self.G, self.Nc, self.c
        self.hot = torch.zeros(L, S, H, P, hot_dim, device=device)
        self.cold = _zeros((L, S, H, P, Nc), cdt, device)
        self.scale = torch.ones(L, S, H, P, device=device) if cold == "fp8" else None
        self.glog = torch.zeros(L, S, H, device=device)
        self.t = torch.zeros(L, S, H, dtype=torch.int32, device=device)
        self.ring_x = torch.zeros(L, S, H, c, P, dtype=io_dtype, device=device)
        self.ring_dt = torch.zeros(L, S, H, (c + 3) // 4 * 4, device=device)
        self.ring_b = torch.zeros(L, S, G, c, Nc, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.max_batch = max_batch if max_batch is not None else num_slots
        lib = _lib.load()
        ws = lib.nssm_step_workspace_bytes(self.max_batch, G, dstate, nssm_dtype(io_dtype), 1)
        self.workspace = torch.empty(max(ws, 256), dtype=torch.uint8, device=device)
        self._structs = [self._make_struct(l) for l in range(L)]

    # ------------------------------------------------------------------
    def _make_struct(self, l: int) -> _lib.NssmPool:
        s = _lib.NssmPool()
        s.num_slots, s.nheads, s.headdim, s.dstate = self.S, self.H, self.P, self.N
        s.ngroups, s.hot_dim, s.chunk = self.G, self.pb, self.c
        s.cold_dtype, s.io_dtype = self.cold_code, nssm_dtype(self.io_dtype)
        s.hot = self.hot[l].data_ptr()
        s.cold = self.cold[l].data_ptr()
        s.cold_scale = self.scale[l].data_ptr() if self.scale is not None else None
        s.glog = self.glog[l].data_ptr()
        s.t = self.t[l].data_ptr()
        s.ring_x = self.ring_x[l].data_ptr()
        s.ring_dt = self.ring_dt[l].data_ptr()
        s.ring_b = self.ring_b[l].data_ptr()
        return s

    def struct(self, layer: int) -> _lib.NssmPool:
        return self._structs[layer]

    @property
    def bytes_per_slot_layer(self) -> int:
        """HBM bytes one slot occupies in one layer."""
        tot = 0
        for t in (self.hot, self.cold, self.scale, self.glog, self.t, self.ring_x, self.ring_dt, self.ring_b):
            if t is not None:
                tot += t[0, 0].numel() * t.element_size()
        return tot

    def check_status(self) -> None:
        """Raise if a kernel flagged an error since the last reset (synchronises): bit 0 a slot
        index outside the pool, bit 1 a pipeline wait that timed out, bit 2 a verify / commit
        window across a chunk boundary or an accept count out of range."""
        v = int(self.status.item())
        if v:
            self.status.zero_()
            what = []
            if v & 1:
                what.append(f"a slot index outside [0, {self.S})")
            if v & 2:
                what.append("a pipeline wait timed out")
            if v & 4:
                what.append("a verify / commit window crosses a chunk boundary or accept is out of range")
            raise IndexError(f"nested_ssm: {'; '.join(what) or 'error'} (status {v})")

    def new_draft(self) -> torch.Tensor:
        """A draft state for the hot-only self-speculative draft: fp32 [L, S, H, P, hot_dim]
        (indexed by slot like the pool's hot slice; nssm_draft_step fills it)."""
        return torch.zeros_like(self.hot)

    def reset_slots(self, slots: torch.Tensor) -> None:
        """Zero the bookkeeping of the given slots (state buffers untouched)."""
        idx = slots.to(self.device, torch.long)
        self.t[:, idx] = 0
        self.glog[:, idx] = 0.0
