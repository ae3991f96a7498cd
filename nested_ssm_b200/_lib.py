"""ctypes binding of ``libnested_ssm.so`` (declarations in ``include/nested_ssm.h``).

This is the same binding a reference-side maintainer would add: plain ctypes
over the C ABI, device pointers and sizes only.  Loading fails loudly if the
library is missing -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

from . import build as _build

NSSM_OK, NSSM_ERR_INVALID, NSSM_ERR_UNSUPPORTED, NSSM_ERR_CUDA = 0, 1, 2, 3
NSSM_F32, NSSM_BF16, NSSM_F8E4M3 = 0, 1, 2
NSSM_MODE_STALE, NSSM_MODE_CORR, NSSM_MODE_COLDOFF = 0, 1, 2
ABI_VERSION = 3

EXPORTED = (
    "nssm_step_workspace_bytes", "nssm_tiered_step", "nssm_fresh_step", "nssm_prefill_split",
    "nssm_materialize", "nssm_rot_flat", "nssm_supported_hot_dims", "nssm_sizeof_pool",
    "nssm_sizeof_step_args", "nssm_abi_version", "nssm_last_error", "nssm_tiered_step_static",
    "nssm_conv_step", "nssm_sizeof_conv_args", "nssm_gated_rmsnorm", "nssm_chunk_scan",
    "nssm_sizeof_scan_args", "nssm_set_wait_polls", "nssm_test_inject_stuck_copy",
    "nssm_spec_workspace_bytes", "nssm_draft_step", "nssm_verify_step", "nssm_commit_step",
    "nssm_sizeof_token_args",
)


class NssmPool(C.Structure):
    _fields_ = [
        ("num_slots", C.c_int32), ("nheads", C.c_int32), ("headdim", C.c_int32),
        ("dstate", C.c_int32), ("ngroups", C.c_int32), ("hot_dim", C.c_int32),
        ("chunk", C.c_int32), ("cold_dtype", C.c_int32), ("io_dtype", C.c_int32),
        ("_pad0", C.c_int32),
        ("hot", C.c_void_p), ("cold", C.c_void_p), ("cold_scale", C.c_void_p),
        ("glog", C.c_void_p), ("t", C.c_void_p), ("ring_x", C.c_void_p),
        ("ring_dt", C.c_void_p), ("ring_b", C.c_void_p),
    ]


class NssmStepArgs(C.Structure):
    _fields_ = [
        ("batch", C.c_int32), ("io_dtype", C.c_int32),
        ("x", C.c_void_p), ("x_stride_b", C.c_int64), ("x_stride_h", C.c_int64),
        ("dt", C.c_void_p), ("dt_stride_b", C.c_int64), ("dt_stride_h", C.c_int64),
        ("dt_dtype", C.c_int32), ("dt_softplus", C.c_int32),
        ("A", C.c_void_p),
        ("B", C.c_void_p), ("B_stride_b", C.c_int64),
        ("C", C.c_void_p), ("C_stride_b", C.c_int64),
        ("D", C.c_void_p), ("dt_bias", C.c_void_p),
        ("dt_min", C.c_float), ("mode", C.c_int32),
        ("R", C.c_void_p),
        ("state_batch_indices", C.c_void_p),
        ("pad_slot_id", C.c_int32), ("out_dtype", C.c_int32),
        ("out", C.c_void_p), ("out_stride_b", C.c_int64), ("out_stride_h", C.c_int64),
        ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
        ("status", C.c_void_p),
        ("norm_gate", C.c_void_p), ("norm_gate_stride_b", C.c_int64),
        ("norm_weight", C.c_void_p), ("norm_weight_dtype", C.c_int32), ("norm_group_size", C.c_int32),
        ("norm_eps", C.c_float), ("_pad1", C.c_int32),
    ]


class NssmTokenArgs(C.Structure):
    _fields_ = [
        ("ntok", C.c_int32), ("_pad0", C.c_int32),
        ("x_stride_t", C.c_int64), ("dt_stride_t", C.c_int64), ("B_stride_t", C.c_int64),
        ("C_stride_t", C.c_int64), ("out_stride_t", C.c_int64), ("accept", C.c_void_p),
    ]


class NssmConvArgs(C.Structure):
    _fields_ = [
        ("batch", C.c_int32), ("nheads", C.c_int32), ("headdim", C.c_int32), ("ngroups", C.c_int32),
        ("dstate", C.c_int32), ("width", C.c_int32), ("state_len", C.c_int32), ("num_slots", C.c_int32),
        ("io_dtype", C.c_int32), ("weight_dtype", C.c_int32), ("activation", C.c_int32),
        ("pad_slot_id", C.c_int32),
        ("xbc", C.c_void_p), ("xbc_stride_b", C.c_int64),
        ("conv_state", C.c_void_p), ("state_stride_s", C.c_int64), ("state_stride_d", C.c_int64),
        ("state_stride_l", C.c_int64),
        ("weight", C.c_void_p), ("bias", C.c_void_p), ("R", C.c_void_p),
        ("state_batch_indices", C.c_void_p),
        ("x_out", C.c_void_p), ("x_out_stride_b", C.c_int64),
        ("B_out", C.c_void_p), ("C_out", C.c_void_p), ("bc_out_stride_b", C.c_int64),
        ("status", C.c_void_p),
    ]


class NssmScanArgs(C.Structure):
    _fields_ = [
        ("batch", C.c_int32), ("seqlen", C.c_int32), ("nheads", C.c_int32), ("headdim", C.c_int32),
        ("ngroups", C.c_int32), ("dstate", C.c_int32), ("chunk_size", C.c_int32), ("io_dtype", C.c_int32),
        ("x", C.c_void_p), ("x_stride_b", C.c_int64), ("x_stride_t", C.c_int64),
        ("dt", C.c_void_p), ("dt_stride_b", C.c_int64), ("dt_stride_t", C.c_int64),
        ("dt_dtype", C.c_int32), ("dt_softplus", C.c_int32), ("dt_min", C.c_float), ("dt_max", C.c_float),
        ("A", C.c_void_p), ("D", C.c_void_p), ("dt_bias", C.c_void_p),
        ("B", C.c_void_p), ("B_stride_b", C.c_int64), ("B_stride_t", C.c_int64),
        ("C", C.c_void_p), ("C_stride_b", C.c_int64), ("C_stride_t", C.c_int64),
        ("initial_states", C.c_void_p), ("init_stride_b", C.c_int64),
        ("y", C.c_void_p), ("y_stride_b", C.c_int64), ("y_stride_t", C.c_int64),
        ("final_states", C.c_void_p), ("final_stride_b", C.c_int64),
        ("status", C.c_void_p),
    ]


_lib = None
_lock = threading.Lock()


def lib_path() -> str:
    """The library to load: $NESTED_SSM_LIB (a prebuilt libnested_ssm.so) or the in-tree build."""
    return os.environ.get("NESTED_SSM_LIB") or _build.LIB_PATH


def load(auto_build: bool = True) -> C.CDLL:
    """Load (building first if stale and nvcc is present) the C-ABI library."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if auto_build and path == _build.LIB_PATH and _build.is_stale(path):
            try:
                _build.build(quiet=True)
            except RuntimeError:
                if not os.path.exists(path):
                    raise
        if not os.path.exists(path):
            raise RuntimeError(
                f"nested_ssm_b200: {path} is missing; build it with `python -m nested_ssm_b200.build` "
                "(the package has no CPU fallback)")
        lib = C.CDLL(path)
        vp, i32, i64, sz = C.c_void_p, C.c_int32, C.c_int64, C.c_size_t
        P_pool, P_args = C.POINTER(NssmPool), C.POINTER(NssmStepArgs)
        sig = {
            "nssm_step_workspace_bytes": (sz, [i32, i32, i32, i32, i32]),
            "nssm_tiered_step": (C.c_int, [P_pool, P_args, vp]),
            "nssm_tiered_step_static": (C.c_int, [P_pool, P_args, vp]),
            "nssm_conv_step": (C.c_int, [C.POINTER(NssmConvArgs), vp]),
            "nssm_sizeof_conv_args": (sz, []),
            "nssm_chunk_scan": (C.c_int, [C.POINTER(NssmScanArgs), vp]),
            "nssm_sizeof_scan_args": (sz, []),
            "nssm_gated_rmsnorm": (C.c_int, [vp, i64, vp, i64, vp, i32, C.c_float, i32, i32, i32, i32, vp, i64, vp]),
            "nssm_fresh_step": (C.c_int, [vp, i32, i32, i32, i32, i32, P_args, vp]),
            "nssm_prefill_split": (C.c_int, [P_pool, vp, i64, vp, i32, i32, vp]),
            "nssm_materialize": (C.c_int, [P_pool, vp, vp, i32, i32, vp, i64, vp]),
            "nssm_rot_flat": (C.c_int, [vp, i64, i32, vp, i32, i32, i32, vp, i64, vp]),
            "nssm_supported_hot_dims": (i32, [i32, C.POINTER(i32), i32]),
            "nssm_sizeof_pool": (sz, []),
            "nssm_sizeof_step_args": (sz, []),
            "nssm_abi_version": (i32, []),
            "nssm_last_error": (C.c_char_p, []),
            "nssm_set_wait_polls": (C.c_uint32, [C.c_uint32]),
            "nssm_test_inject_stuck_copy": (i32, [i32]),
            "nssm_spec_workspace_bytes": (sz, [i32, i32, i32, i32, i32, i32]),
            "nssm_draft_step": (C.c_int, [P_pool, vp, i32, P_args, vp]),
            "nssm_verify_step": (C.c_int, [P_pool, P_args, C.POINTER(NssmTokenArgs), vp]),
            "nssm_commit_step": (C.c_int, [P_pool, P_args, C.POINTER(NssmTokenArgs), vp]),
            "nssm_sizeof_token_args": (sz, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype, fn.argtypes = res, args
        if lib.nssm_abi_version() != ABI_VERSION:
            raise RuntimeError(f"libnested_ssm ABI {lib.nssm_abi_version()} != binding {ABI_VERSION}")
        if (lib.nssm_sizeof_pool() != C.sizeof(NssmPool) or lib.nssm_sizeof_step_args() != C.sizeof(NssmStepArgs)
                or lib.nssm_sizeof_conv_args() != C.sizeof(NssmConvArgs)
                or lib.nssm_sizeof_scan_args() != C.sizeof(NssmScanArgs)
                or lib.nssm_sizeof_token_args() != C.sizeof(NssmTokenArgs)):
            raise RuntimeError("libnested_ssm struct layout differs from the ctypes binding")
        _lib = lib
        return lib


class NssmError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"nested_ssm error {code}: {msg}")
        self.code = code


def check(rc: int) -> None:
    if rc != NSSM_OK:
        msg = load().nssm_last_error()
        msg = msg.decode() if msg else ""
        if rc == NSSM_ERR_INVALID:
            raise ValueError(f"nested_ssm: {msg}")
        raise NssmError(rc, msg)


def supported_hot_dims(dstate: int = 128) -> list[int]:
    lib = load()
    buf = (C.c_int32 * 16)()
    n = lib.nssm_supported_hot_dims(dstate, buf, 16)
    return [buf[i] for i in range(min(n, 16))]
