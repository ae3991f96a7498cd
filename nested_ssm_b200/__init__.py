"""nested_ssm_b200 -- B200-native (sm_100a) tiered Mamba2 decode state op.

A drop-in for the hot path of nested_ssm: the per-layer tiered
("dense-but-stale") selective-state update with continuous-batching slot
indices, the per-group rotation R of B and C, the ring buffer of the last c
tokens and the rank-c cold flush with fp8 requantisation.  Python/PyTorch is
the host; the work runs in hand-written CUDA behind the C ABI of
``include/nested_ssm.h`` (``libnested_ssm.so``), loaded with ctypes.
"""
from ._lib import load as load_library, supported_hot_dims  # noqa: F401
from .ops import (  # noqa: F401
    commit_state_update,
    conv_step,
    draft_state_update,
    gated_rmsnorm,
    mamba_chunk_scan_combined,
    materialize,
    prefill_snapshot,
    prefill_split,
    rot_flat,
    selective_state_update,
    tiered_state_update,
    verify_state_update,
)
from .pool import TieredSlotPool  # noqa: F401

__version__ = "0.1.0"
