"""The C-ABI library without a GPU: it loads, exports every entry point the header
declares, its structs match the ctypes binding, and host-side validation answers
before any device work."""
import ctypes as C
import os
import re

import pytest
import torch

from nested_ssm_b200 import _lib
from nested_ssm_b200 import build as B

HEADER = os.path.join(B.INCLUDE, "nested_ssm.h")


def _declared():
    src = open(HEADER).read()
    return set(re.findall(r"NSSM_API\s+[\w\s\*]+?\b(nssm_\w+)\s*\(", src))


def test_header_declares_what_the_binding_lists():
    assert _declared() == set(_lib.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name
    assert lib.nssm_abi_version() == _lib.ABI_VERSION
    assert lib.nssm_sizeof_pool() == C.sizeof(_lib.NssmPool)
    assert lib.nssm_sizeof_step_args() == C.sizeof(_lib.NssmStepArgs)


def test_workspace_bytes_and_hot_widths():
    lib = _lib.load()
    assert lib.nssm_step_workspace_bytes(448, 8, 128, _lib.NSSM_BF16, 1) == 2 * 448 * 8 * 128 * 2
    assert lib.nssm_step_workspace_bytes(3, 8, 128, _lib.NSSM_F32, 1) == 2 * 12288   # 256-byte rounded halves
    assert lib.nssm_step_workspace_bytes(448, 8, 128, _lib.NSSM_BF16, 0) == 0
    assert _lib.supported_hot_dims(128) == [16, 32, 64]
    assert _lib.supported_hot_dims(64) == []


def test_null_arguments_are_rejected_on_the_host():
    lib = _lib.load()
    assert lib.nssm_tiered_step(None, None, None) == _lib.NSSM_ERR_INVALID
    assert lib.nssm_last_error()
    assert lib.nssm_tiered_step_static(None, None, None) == _lib.NSSM_ERR_INVALID
    a = _lib.NssmStepArgs()
    assert lib.nssm_fresh_step(None, 1, 1, 1, 128, 1, C.byref(a), None) == _lib.NSSM_ERR_INVALID


def test_static_entry_rejects_oversized_batch_before_device_work():
    """Size check comes first: batch 1025 of bf16 B, C at G=8, N=128 needs 4 MiB + 8 KiB."""
    lib = _lib.load()
    p = _lib.NssmPool()
    p.num_slots, p.nheads, p.headdim, p.dstate, p.ngroups, p.hot_dim, p.chunk = 8, 128, 80, 128, 8, 32, 4
    a = _lib.NssmStepArgs()
    a.batch, a.io_dtype, a.R = 1025, _lib.NSSM_BF16, 16     # R non-NULL: rotation requested
    rc = lib.nssm_tiered_step_static(C.byref(p), C.byref(a), None)
    assert rc == _lib.NSSM_ERR_INVALID
    msg = lib.nssm_last_error().decode()
    assert "static scratch" in msg and "4194304" in msg


def test_ops_validate_shapes_and_refuse_cpu_tensors():
    from nested_ssm_b200 import ops
    x = torch.zeros(2, 4, 8)
    dt = torch.zeros(2, 4)
    A = torch.zeros(4)
    Bm = torch.zeros(2, 1, 16)
    with pytest.raises(ValueError):
        ops.build_step_args(torch.zeros(2, 4), dt, A, Bm, Bm)               # x not 3-D
    with pytest.raises(ValueError):
        ops.build_step_args(x, torch.zeros(3, 4), A, Bm, Bm)                # dt rows
    with pytest.raises(ValueError):
        ops.build_step_args(x, dt, torch.zeros(5), Bm, Bm)                  # A heads
    with pytest.raises(ValueError):
        ops.build_step_args(x, dt, A, Bm.bfloat16(), Bm)                    # B dtype
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ops.build_step_args(x, dt, A, Bm, Bm)


def test_pool_refuses_cpu_device():
    from nested_ssm_b200 import TieredSlotPool
    with pytest.raises(RuntimeError, match="CUDA device"):
        TieredSlotPool(1, 2, 4, 8, 32, 1, 8, 2, device="cpu")
    with pytest.raises(ValueError):
        TieredSlotPool(1, 2, 4, 8, 32, 1, 40, 2, device="cpu")             # hot >= dstate


def _fake_pool_and_args():
    """A pool and step args whose pointers are never dereferenced (every case below is
    answered by host-side validation)."""
    p = _lib.NssmPool()
    p.num_slots, p.nheads, p.headdim, p.dstate, p.ngroups, p.hot_dim, p.chunk = 8, 128, 80, 128, 8, 32, 4
    p.cold_dtype, p.io_dtype = _lib.NSSM_F8E4M3, _lib.NSSM_BF16
    for i, f in enumerate(("hot", "cold", "cold_scale", "glog", "t", "ring_x", "ring_dt", "ring_b")):
        setattr(p, f, 0x10000 * (i + 1))
    a = _lib.NssmStepArgs()
    a.batch, a.io_dtype, a.dt_dtype, a.out_dtype = 4, _lib.NSSM_BF16, _lib.NSSM_BF16, _lib.NSSM_BF16
    for i, f in enumerate(("x", "dt", "A", "B", "C", "out")):
        setattr(a, f, 0x100000 * (i + 1))
    return p, a


def test_spec_entry_points_validate_on_the_host():
    lib = _lib.load()
    assert lib.nssm_sizeof_token_args() == C.sizeof(_lib.NssmTokenArgs)
    # rotated B and C of batch * ntok rows, then one int32 per row (256-byte rounded)
    assert lib.nssm_spec_workspace_bytes(448, 4, 8, 128, _lib.NSSM_BF16, 1) == 2 * 448 * 4 * 8 * 128 * 2 + 1792
    assert lib.nssm_spec_workspace_bytes(448, 4, 8, 128, _lib.NSSM_BF16, 0) == 1792
    p, a = _fake_pool_and_args()
    t = _lib.NssmTokenArgs()
    t.ntok = 2
    assert lib.nssm_verify_step(C.byref(p), C.byref(a), None, None) == _lib.NSSM_ERR_INVALID
    assert lib.nssm_commit_step(C.byref(p), C.byref(a), C.byref(t), None) == _lib.NSSM_ERR_INVALID   # accept NULL
    assert "accept" in lib.nssm_last_error().decode()
    a.mode = _lib.NSSM_MODE_CORR
    assert lib.nssm_verify_step(C.byref(p), C.byref(a), C.byref(t), None) == _lib.NSSM_ERR_UNSUPPORTED
    a.mode = _lib.NSSM_MODE_STALE
    t.ntok = 5                                                      # longer than the chunk (4)
    assert lib.nssm_verify_step(C.byref(p), C.byref(a), C.byref(t), None) == _lib.NSSM_ERR_INVALID
    assert "chunk" in lib.nssm_last_error().decode()
    t.ntok = 0
    assert lib.nssm_verify_step(C.byref(p), C.byref(a), C.byref(t), None) == _lib.NSSM_ERR_INVALID
    assert lib.nssm_draft_step(C.byref(p), None, 1, C.byref(a), None) == _lib.NSSM_ERR_INVALID   # draft NULL
