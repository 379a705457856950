"""ctypes binding of the sas_b200 C ABI (``include/sas_b200.h``).

The shared library is built in-tree by ``dsv4_planb_b200.build`` and loaded
from ``dsv4_planb_b200/_lib/libsas_b200.so``.  There is no fallback: if the
library is missing, every operator raises.
"""

from __future__ import annotations

import ctypes
import os

from . import build as _build

SAS_OK = 0
SAS_ERR_INVALID_ARG = 1
SAS_ERR_UNSUPPORTED = 2
SAS_ERR_WORKSPACE = 3
SAS_ERR_CUDA = 4
SAS_ERR_DEVICE = 5

SAS_STATUS_BAD_INDEX = 0x1
SAS_STATUS_BAD_BLOCK = 0x2
SAS_STATUS_NO_PROGRESS = 0x4
SAS_STATUS_WAIT_TIMEOUT = 0x8
SAS_STATUS_BAD_TOKEN = 0x10

SAS_NOALLOC_SCRATCH_BYTES = 16 << 20

SAS_DTYPE_BF16 = 0
SAS_DTYPE_FP16 = 1

SAS_FWD_FLAG_CU_SEQLENS = 0x1
SAS_FWD_FLAG_TEST_STALL = 0x100
SAS_FWD_FLAG_LAZY_RESCALE = 0x200

KERNELS = {"auto": 0, "simt": 1, "tc": 2, "tc2": 3}
LAYOUT_Q = {"BSND": 0, "BSH": 1, "TND": 2}
LAYOUT_KV = {"PA_ND": 0, "TND": 1}

# Every symbol include/sas_b200.h declares.
EXPORTS = (
    "sas_workspace_size",
    "sas_forward_kernel_count",
    "sas_forward",
    "sas_forward_noalloc",
    "sas_backward",
    "sas_noalloc_read_status",
    "sas_resolve_rows",
    "sas_split_plan",
    "sas_split_metadata",
    "sas_read_status",
    "sas_set_kernel_events",
    "sas_metadata_workspace_size",
    "sas_metadata",
    "sas_strerror",
    "sas_abi_version",
)


class SasFwdArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32),
        ("num_tokens", ctypes.c_int32),
        ("max_q_len", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("v_head_dim", ctypes.c_int32),
        ("ori_block_num", ctypes.c_int32),
        ("ori_block_size", ctypes.c_int32),
        ("ori_table_len", ctypes.c_int32),
        ("cmp_block_num", ctypes.c_int32),
        ("cmp_block_size", ctypes.c_int32),
        ("cmp_table_len", ctypes.c_int32),
        ("topk", ctypes.c_int32),
        ("cmp_ratio", ctypes.c_int32),
        ("scenario", ctypes.c_int32),
        ("max_cmp_len", ctypes.c_int32),
        ("ori_win_left", ctypes.c_int32),
        ("ori_win_right", ctypes.c_int32),
        ("ori_mask_mode", ctypes.c_int32),
        ("cmp_mask_mode", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("softmax_scale", ctypes.c_float),
        ("kernel", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("split_tiles", ctypes.c_int32),
        ("reserved", ctypes.c_int32 * 4),
    ]


class SasMetaArgs(ctypes.Structure):
    _fields_ = [
        ("num_heads_q", ctypes.c_int32),
        ("num_heads_kv", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("n_cu_seqlens_q", ctypes.c_int32),
        ("n_cu_seqlens_ori_kv", ctypes.c_int32),
        ("n_seqused_q", ctypes.c_int32),
        ("n_seqused_kv", ctypes.c_int32),
        ("batch_size", ctypes.c_int32),
        ("max_seqlen_q", ctypes.c_int32),
        ("max_seqlen_kv", ctypes.c_int32),
        ("ori_topk", ctypes.c_int32),
        ("cmp_topk", ctypes.c_int32),
        ("cmp_ratio", ctypes.c_int32),
        ("ori_mask_mode", ctypes.c_int32),
        ("cmp_mask_mode", ctypes.c_int32),
        ("ori_win_left", ctypes.c_int32),
        ("ori_win_right", ctypes.c_int32),
        ("layout_q", ctypes.c_int32),
        ("layout_kv", ctypes.c_int32),
        ("has_ori_kv", ctypes.c_int32),
        ("has_cmp_kv", ctypes.c_int32),
        ("aic_core_num", ctypes.c_int32),
        ("aiv_core_num", ctypes.c_int32),
        ("reserved", ctypes.c_int32 * 5),
    ]


_P = ctypes.c_void_p
_SZ = ctypes.c_size_t

_SIGNATURES = {
    "sas_workspace_size": (ctypes.c_int, [ctypes.POINTER(SasFwdArgs), ctypes.POINTER(_SZ)]),
    "sas_forward_kernel_count": (ctypes.c_int, [ctypes.POINTER(SasFwdArgs), ctypes.POINTER(ctypes.c_int32)]),
    "sas_forward": (ctypes.c_int, [ctypes.POINTER(SasFwdArgs)] + [_P] * 13 + [_P, _SZ, _P]),
    "sas_forward_noalloc": (ctypes.c_int, [ctypes.POINTER(SasFwdArgs)] + [_P] * 13 + [_P]),
    "sas_noalloc_read_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32), _P]),
    "sas_backward": (ctypes.c_int, [ctypes.POINTER(SasFwdArgs)] + [_P] * 18 + [_P, _SZ, _P]),
    "sas_resolve_rows": (ctypes.c_int, [ctypes.POINTER(SasFwdArgs)] + [_P] * 8 + [_P, _SZ, _P]),
    "sas_split_plan": (ctypes.c_int, [ctypes.POINTER(SasFwdArgs), ctypes.POINTER(ctypes.c_int32),
                                      ctypes.POINTER(ctypes.c_int32)]),
    "sas_split_metadata": (ctypes.c_int, [ctypes.POINTER(SasFwdArgs)] + [_P] * 7 + [_P, _SZ, _P]),
    "sas_read_status": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_uint32), _P]),
    "sas_set_kernel_events": (ctypes.c_int, [_P, _P]),
    "sas_metadata_workspace_size": (ctypes.c_int, [ctypes.POINTER(SasMetaArgs), ctypes.POINTER(_SZ)]),
    "sas_metadata": (ctypes.c_int, [ctypes.POINTER(SasMetaArgs)] + [_P] * 5 + [_P, _SZ, _P]),
    "sas_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "sas_abi_version": (ctypes.c_int, []),
}

_lib = None


def lib_path() -> str:
    return _build.LIB


def load(build_if_missing: bool = False) -> ctypes.CDLL:
    """Load the library (optionally building it first).  Raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not os.path.exists(path):
        if build_if_missing:
            _build.build()
        else:
            raise RuntimeError(
                f"sas_b200 CUDA library not found at {path}; build it with "
                "`python -m dsv4_planb_b200.build` (no CPU fallback exists)"
            )
    lib = ctypes.CDLL(path)
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def strerror(rc: int) -> str:
    return load().sas_strerror(rc).decode()


def check(rc: int, what: str) -> None:
    if rc != SAS_OK:
        raise RuntimeError(f"{what} failed: {strerror(rc)} (status {rc})")


def status_names(bits: int):
    names = []
    for name, bit in (
        ("bad_index", SAS_STATUS_BAD_INDEX),
        ("bad_block", SAS_STATUS_BAD_BLOCK),
        ("no_progress", SAS_STATUS_NO_PROGRESS),
        ("wait_timeout", SAS_STATUS_WAIT_TIMEOUT),
        ("bad_token", SAS_STATUS_BAD_TOKEN),
    ):
        if bits & bit:
            names.append(name)
    return names
