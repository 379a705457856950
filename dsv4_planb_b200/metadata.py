"""Drop-in ``sparse_attn_sharedkv_metadata`` running the CUDA scheduler kernel.

Same keyword arguments and result as the reference
``sparse_attn_sharedkv_tilelang/metadata.py:1018-1086``: an ``int32[1024]``
tensor holding ``faMetadata[36][8]`` then ``fdMetadata[72][8]``, bit-identical
to the reference for the same arguments.  Like the reference, the result is a
CPU tensor unless ``device`` is given.  The constants of the packed layout are
re-exported under the reference's names.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib

AIC_CORE_NUM = 36
AIV_CORE_NUM = 72
SAS_META_SIZE = 1024
FA_METADATA_SIZE = 8
FD_METADATA_SIZE = 8
FA_CORE_ENABLE_INDEX = 0
FA_BN2_START_INDEX = 1
FA_M_START_INDEX = 2
FA_S2_START_INDEX = 3
FA_BN2_END_INDEX = 4
FA_M_END_INDEX = 5
FA_S2_END_INDEX = 6
FA_FIRST_FD_DATA_WORKSPACE_IDX_INDEX = 7


def _host_list(t):
    if t is None:
        return None
    if isinstance(t, torch.Tensor):
        if t.numel() == 0:
            return None
        return t.detach().to("cpu", torch.int64).reshape(-1).tolist()
    t = [int(x) for x in t]
    return t or None


def sparse_attn_sharedkv_metadata(
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
    device: Optional[str] = None,
    cuda_device=None,
) -> torch.Tensor:
    """Per-core FA / FD work table of the reference scheduler, computed on the GPU."""
    del cu_seqlens_cmp_kv  # not read by the reference scheduler either
    dev = torch.device(cuda_device) if cuda_device is not None else torch.device("cuda", torch.cuda.current_device())
    lists = {
        "cu_q": _host_list(cu_seqlens_q),
        "cu_kv": _host_list(cu_seqlens_ori_kv),
        "sq": _host_list(seqused_q),
        "skv": _host_list(seqused_kv),
    }
    # Bound on the number of query rows, so the kernel can keep a per-row table.
    if lists["sq"] is not None:
        rows = sum(max(x, 0) for x in lists["sq"])
    elif layout_q == "TND" and lists["cu_q"] is not None:
        cu = lists["cu_q"]
        rows = sum(max(cu[i + 1] - cu[i], 0) for i in range(len(cu) - 1))
    else:
        rows = max(batch_size, 0) * max(max_seqlen_q, 0)
    rows = min(rows, 1 << 26)

    args = _lib.SasMetaArgs()
    args.num_heads_q, args.num_heads_kv, args.head_dim = num_heads_q, num_heads_kv, head_dim
    args.n_cu_seqlens_q = len(lists["cu_q"]) if lists["cu_q"] else 0
    args.n_cu_seqlens_ori_kv = len(lists["cu_kv"]) if lists["cu_kv"] else 0
    args.n_seqused_q = len(lists["sq"]) if lists["sq"] else 0
    args.n_seqused_kv = len(lists["skv"]) if lists["skv"] else 0
    args.batch_size, args.max_seqlen_q, args.max_seqlen_kv = batch_size, max_seqlen_q, max_seqlen_kv
    args.ori_topk, args.cmp_topk, args.cmp_ratio = ori_topk, cmp_topk, cmp_ratio
    args.ori_mask_mode, args.cmp_mask_mode = ori_mask_mode, cmp_mask_mode
    args.ori_win_left, args.ori_win_right = ori_win_left, ori_win_right
    args.layout_q = _lib.LAYOUT_Q.get(layout_q, 3)
    args.layout_kv = _lib.LAYOUT_KV.get(layout_kv, 0)
    args.has_ori_kv, args.has_cmp_kv = int(bool(has_ori_kv)), int(bool(has_cmp_kv))
    args.aic_core_num, args.aiv_core_num = aic_core_num, aiv_core_num
    args.reserved[0] = rows

    def dev_i32(x):
        return None if x is None else torch.tensor(x, dtype=torch.int32, device=dev)

    t_cu_q, t_cu_kv, t_sq, t_skv = (dev_i32(lists[k]) for k in ("cu_q", "cu_kv", "sq", "skv"))
    lib = _lib.load()
    nbytes = _lib.ctypes.c_size_t(0)
    _lib.check(lib.sas_metadata_workspace_size(_lib.ctypes.byref(args), _lib.ctypes.byref(nbytes)),
               "sas_metadata_workspace_size")
    ws = torch.empty(max(nbytes.value, 256), dtype=torch.uint8, device=dev)
    out = torch.empty(SAS_META_SIZE, dtype=torch.int32, device=dev)
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(lib.sas_metadata(_lib.ctypes.byref(args), ptr(t_cu_q), ptr(t_cu_kv), ptr(t_sq), ptr(t_skv), ptr(out),
                                ptr(ws), ws.numel(), stream), "sas_metadata")
    st = _lib.ctypes.c_uint32(0)
    _lib.check(lib.sas_read_status(ptr(ws), _lib.ctypes.byref(st), stream), "sas_read_status")
    if st.value:
        raise RuntimeError(f"sas_metadata: {_lib.status_names(st.value)}")
    return out.to(device) if device is not None else out.cpu()
