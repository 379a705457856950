"""ctypes wrapper of the C metadata-scheduler oracle -- TEST INFRASTRUCTURE ONLY.

``metadata_ref(**kw)`` takes the keyword arguments of the reference's public
``sparse_attn_sharedkv_metadata`` (``metadata.py:1018-1045``) and returns the
packed ``int32[1024]`` array computed by ``sas_metadata_ref.c``.
``build_oracle()`` compiles the C file with gcc into ``oracle/_build/``.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SRC = os.path.join(_HERE, "sas_metadata_ref.c")
_BUILD = os.path.join(_HERE, "_build")
_LIB = os.path.join(_BUILD, "libsas_metadata_ref.so")

SAS_META_SIZE = 1024
AIC_CORE_NUM = 36
AIV_CORE_NUM = 72
FA_METADATA_SIZE = 8

_LAYOUT_Q = {"BSND": 0, "BSH": 1, "TND": 2}
_LAYOUT_KV = {"TND": 1}

ERRORS = {0: "ok", 1: "bad argument", 2: "index out of range", 3: "scheduler made no progress"}


class _Args(ctypes.Structure):
    _fields_ = [
        ("num_heads_q", ctypes.c_int64),
        ("num_heads_kv", ctypes.c_int64),
        ("head_dim", ctypes.c_int64),
        ("cu_seqlens_q", ctypes.POINTER(ctypes.c_int64)),
        ("n_cu_q", ctypes.c_int64),
        ("cu_seqlens_ori_kv", ctypes.POINTER(ctypes.c_int64)),
        ("n_cu_kv", ctypes.c_int64),
        ("seqused_q", ctypes.POINTER(ctypes.c_int64)),
        ("n_seqused_q", ctypes.c_int64),
        ("seqused_kv", ctypes.POINTER(ctypes.c_int64)),
        ("n_seqused_kv", ctypes.c_int64),
        ("batch_size", ctypes.c_int64),
        ("max_seqlen_q", ctypes.c_int64),
        ("max_seqlen_kv", ctypes.c_int64),
        ("ori_topk", ctypes.c_int64),
        ("cmp_topk", ctypes.c_int64),
        ("cmp_ratio", ctypes.c_int64),
        ("ori_mask_mode", ctypes.c_int64),
        ("cmp_mask_mode", ctypes.c_int64),
        ("ori_win_left", ctypes.c_int64),
        ("ori_win_right", ctypes.c_int64),
        ("layout_q", ctypes.c_int64),
        ("layout_kv", ctypes.c_int64),
        ("has_ori_kv", ctypes.c_int64),
        ("has_cmp_kv", ctypes.c_int64),
        ("aic_core_num", ctypes.c_int64),
        ("aiv_core_num", ctypes.c_int64),
    ]


def build_oracle(force: bool = False) -> str:
    """Compile ``sas_metadata_ref.c`` into ``oracle/_build/libsas_metadata_ref.so``."""
    if not force and os.path.exists(_LIB) and os.path.getmtime(_LIB) >= os.path.getmtime(_SRC):
        return _LIB
    os.makedirs(_BUILD, exist_ok=True)
    tmp = _LIB + f".tmp{os.getpid()}"
    subprocess.check_call(["gcc", "-O2", "-std=c11", "-shared", "-fPIC", "-o", tmp, _SRC])
    os.replace(tmp, _LIB)
    return _LIB


_lib = None


def _load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(build_oracle())
        lib.sasm_ref_metadata.restype = ctypes.c_int
        lib.sasm_ref_metadata.argtypes = [ctypes.POINTER(_Args), ctypes.POINTER(ctypes.c_int32)]
        _lib = lib
    return _lib


def _as_i64(x) -> Optional[np.ndarray]:
    if x is None:
        return None
    if hasattr(x, "detach"):
        x = x.detach().cpu().numpy()
    a = np.ascontiguousarray(np.asarray(x, dtype=np.int64).reshape(-1))
    return a if a.size else None


def metadata_ref(
    *,
    num_heads_q: int,
    num_heads_kv: int,
    head_dim: int,
    cu_seqlens_q=None,
    cu_seqlens_ori_kv=None,
    cu_seqlens_cmp_kv=None,
    seqused_q=None,
    seqused_kv=None,
    batch_size: int = 0,
    max_seqlen_q: int = 0,
    max_seqlen_kv: int = 0,
    ori_topk: int = 0,
    cmp_topk: int = 0,
    cmp_ratio: int = -1,
    ori_mask_mode: int = 4,
    cmp_mask_mode: int = 3,
    ori_win_left: int = 127,
    ori_win_right: int = 0,
    layout_q: str = "BSND",
    layout_kv: str = "PA_ND",
    has_ori_kv: bool = True,
    has_cmp_kv: bool = True,
    aic_core_num: int = 24,
    aiv_core_num: int = 48,
    device=None,
) -> np.ndarray:
    """C restatement of ``sparse_attn_sharedkv_metadata`` (``metadata.py:1018-1086``)."""
    del cu_seqlens_cmp_kv, device  # unused by the reference scheduler as well
    lib = _load()
    keep = []

    def ptr(x):
        a = _as_i64(x)
        if a is None:
            return ctypes.POINTER(ctypes.c_int64)(), 0
        keep.append(a)
        return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), a.size

    cu_q, n_cu_q = ptr(cu_seqlens_q)
    cu_kv, n_cu_kv = ptr(cu_seqlens_ori_kv)
    sq, n_sq = ptr(seqused_q)
    skv, n_skv = ptr(seqused_kv)
    args = _Args(
        num_heads_q,
        num_heads_kv,
        head_dim,
        cu_q,
        n_cu_q,
        cu_kv,
        n_cu_kv,
        sq,
        n_sq,
        skv,
        n_skv,
        batch_size,
        max_seqlen_q,
        max_seqlen_kv,
        ori_topk,
        cmp_topk,
        cmp_ratio,
        ori_mask_mode,
        cmp_mask_mode,
        ori_win_left,
        ori_win_right,
        _LAYOUT_Q.get(layout_q, 3),
        _LAYOUT_KV.get(layout_kv, 0),
        int(bool(has_ori_kv)),
        int(bool(has_cmp_kv)),
        aic_core_num,
        aiv_core_num,
    )
    out = np.zeros(SAS_META_SIZE, dtype=np.int32)
    rc = lib.sasm_ref_metadata(ctypes.byref(args), out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)))
    if rc != 0:
        raise RuntimeError(f"metadata oracle failed: {ERRORS.get(rc, rc)}")
    return out
