"""Slot sharding of the tiered state over the GPUs of one node.

Sequences are independent, so the slot pool is partitioned by slot: rank r owns the
contiguous global slots ``[r*S/n, (r+1)*S/n)`` in its own ``TieredSlotPool`` (local slot =
global slot - first owned slot) and runs the state op on the rows of the global batch whose
slot it owns.  Nothing crosses GPUs on the data path; :func:`gather_rows` (one all_gather)
exists only to assemble outputs for checks.
"""
from __future__ import annotations

import torch


def slot_range(num_slots: int, rank: int, world: int) -> tuple[int, int]:
    """Global slots ``[lo, hi)`` owned by ``rank`` (sizes differ by at most one)."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside [0, {world})")
    base, extra = divmod(num_slots, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def owner_of(slots: torch.Tensor, num_slots: int, world: int) -> torch.Tensor:
    """Rank owning each global slot (−1 for slots outside ``[0, num_slots)``)."""
    s = slots.long()
    base, extra = divmod(num_slots, world)
    cut = extra * (base + 1)               # first slot of the ranks holding `base` slots
    own = torch.where(s < cut, s // (base + 1), extra + (s - cut) // max(base, 1))
    return torch.where((s >= 0) & (s < num_slots), own, torch.full_like(own, -1))


def local_batch(slots: torch.Tensor, rank: int, world: int, num_slots: int,
                pad_slot_id: int = -1) -> tuple[torch.Tensor, torch.Tensor]:
    """Rows of a global batch that ``rank`` serves, and their local slot indices.

    Returns ``(rows, local_slots)``: ``rows`` indexes the global batch (padded rows are
    never owned), ``local_slots`` is int32 for the rank's own pool."""
    s = slots.reshape(-1).long()
    own = owner_of(s, num_slots, world)
    rows = torch.nonzero((own == rank) & (s != pad_slot_id)).reshape(-1)
    lo, _ = slot_range(num_slots, rank, world)
    return rows, (s[rows] - lo).to(torch.int32)


def gather_rows(y_local: torch.Tensor, rows: torch.Tensor, batch: int, group=None) -> torch.Tensor:
    """Assemble the global ``[batch, ...]`` output from every rank's rows (rows no rank
    served stay zero).  One all_gather of a padded buffer; for checks, not the hot path."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    dev = y_local.device
    n = torch.tensor([rows.numel()], device=dev, dtype=torch.int64)
    counts = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(counts, n, group=group)
    cap = int(max(int(c.item()) for c in counts))
    tail = tuple(y_local.shape[1:])
    buf = torch.zeros((cap + 1,) + tail, dtype=y_local.dtype, device=dev)
    buf[: rows.numel()] = y_local
    idx = torch.full((cap + 1,), -1, dtype=torch.int64, device=dev)
    idx[: rows.numel()] = rows.to(dev, torch.int64)
    bufs = [torch.empty_like(buf) for _ in range(world)]
    idxs = [torch.empty_like(idx) for _ in range(world)]
    dist.all_gather(bufs, buf, group=group)
    dist.all_gather(idxs, idx, group=group)
    out = torch.zeros((batch,) + tail, dtype=y_local.dtype, device=dev)
    for b_, i_ in zip(bufs, idxs):
        keep = i_ >= 0
        out[i_[keep]] = b_[keep]
    return out
