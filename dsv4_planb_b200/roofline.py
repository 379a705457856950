"""Algorithmic work of a workload: the denominators of the roofline.

FLOPs = sum over tokens of 2 * N1 * (n_win + n_cmp) * (D_qk + D_v)
Bytes = sum over requests of (distinct window rows + distinct compressed rows) * D_qk * elem
        + Q (N1 * D_qk * elem per token) + O (N1 * D_v * elem per token)
        + LSE (N1 * 4 per token) + indices (K * 4 per token) + block-table bytes
Each distinct KV row of a request is charged once: a kernel that re-reads it
(across tokens of one request, or across CTAs) spends traffic above this.
The counts come from the product's own key resolution (``resolve_rows``).
"""

from __future__ import annotations

import torch


def algorithmic_figures(wl, device=None) -> dict:
    from .api import resolve_rows

    dev = device or wl.q.device
    scen = 3 if wl.cmp_sparse_indices is not None else (2 if wl.cmp_kv is not None else 1)
    tinfo, rows, status = resolve_rows(
        cmp_sparse_indices=None if wl.cmp_sparse_indices is None else wl.cmp_sparse_indices.to(dev),
        ori_block_table=wl.ori_block_table.to(dev),
        cmp_block_table=None if wl.cmp_block_table is None else wl.cmp_block_table.to(dev),
        cu_seqlens_q=wl.cu_seqlens_q.to(dev), seqused_kv=wl.seqused_kv.to(dev), num_heads=wl.q.shape[1],
        head_dim=wl.q.shape[2], ori_block_num=wl.ori_kv.shape[0], ori_block_size=wl.ori_kv.shape[1],
        cmp_block_num=1 if wl.cmp_kv is None else wl.cmp_kv.shape[0],
        cmp_block_size=1 if wl.cmp_kv is None else wl.cmp_kv.shape[1], cmp_ratio=wl.cmp_ratio, scenario=scen)
    T, N1, Dq = wl.q.shape
    Dv = wl.v_head_dim
    elem = wl.q.element_size()
    b = tinfo[:, 0].long()
    left = tinfo[:, 2].long()
    n_win = tinfo[:, 3].long()
    n_cmp = tinfo[:, 4].long()
    keys = int((n_win + n_cmp).sum().item())
    flops = 2.0 * N1 * keys * (Dq + Dv)
    # distinct window rows per request: union of [left, left + n_win) intervals
    B = wl.cu_seqlens_q.numel() - 1
    win_rows = 0
    lo = torch.full((B,), 1 << 62, dtype=torch.long, device=dev).scatter_reduce(0, b, left, "amin")
    hi = torch.zeros((B,), dtype=torch.long, device=dev).scatter_reduce(0, b, left + n_win, "amax")
    # windows of consecutive queries of one request overlap or touch, so the union is one interval
    win_rows = int((hi - lo).clamp(min=0).sum().item())
    cmp_rows = 0
    if rows.numel():
        cap = rows.shape[1]
        slot = torch.arange(cap, device=dev)[None, :]
        valid = slot < n_cmp[:, None]
        pair = b[:, None] * (1 << 32) + rows.long().clamp(min=0)
        pair = pair[valid]
        cmp_rows = int(torch.unique(pair).numel())
    kv_bytes = (win_rows + cmp_rows) * Dq * elem
    topk = rows.shape[1] if scen == 3 else 0
    table_bytes = 4 * (wl.ori_block_table.numel() + (0 if wl.cmp_block_table is None else wl.cmp_block_table.numel()))
    io_bytes = T * N1 * (Dq * elem + Dv * elem + 4) + T * topk * 4 + table_bytes
    return dict(flops=flops, bytes=float(kv_bytes + io_bytes), kv_bytes=float(kv_bytes), keys=keys, tokens=T,
                status=status)
