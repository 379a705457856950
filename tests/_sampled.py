"""fp32 oracle on sampled tokens of a device-resident workload (test infrastructure).

Full BASELINE configurations do not fit a CPU copy (c5's pools are ~20 GB), so
each sampled token's key rows are resolved on the host with the oracle's own
rules (``oracle.golden_np.resolve_token_rows``, golden.py:28-66, 125-150),
mapped through the block tables as ``unpack_paged_kv`` would (golden.py:247-268,
unmapped blocks read as zero rows), gathered from the device pools, and fed to
``oracle.golden_np.attend_token`` (golden.py:156-200) in fp32.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import golden_np as O


def _phys_rows(table_row: np.ndarray, pos: np.ndarray, block_size: int, block_num: int) -> np.ndarray:
    pos = np.asarray(pos, dtype=np.int64)
    blk = pos // block_size
    phys = np.full(pos.shape, -1, dtype=np.int64)
    inside = blk < table_row.shape[0]
    phys[inside] = table_row[blk[inside]]
    ok = (phys >= 0) & (phys < block_num)
    return np.where(ok, phys * block_size + pos % block_size, -1)


def _gather(pool2d: torch.Tensor, rows: np.ndarray) -> np.ndarray:
    if rows.size == 0:
        return np.zeros((0, pool2d.shape[1]), dtype=np.float32)
    idx = torch.as_tensor(np.maximum(rows, 0), device=pool2d.device)
    got = pool2d.index_select(0, idx).float().cpu().numpy()
    got[rows < 0] = 0.0
    return got


def oracle_tokens(wl, tokens):
    """``(out [n, N1, Dv], lse [n, N1])`` of the fp32 oracle for flat token rows ``tokens``."""
    scen = 3 if wl.cmp_sparse_indices is not None else (2 if wl.cmp_kv is not None else 1)
    cu = wl.cu_seqlens_q.cpu().numpy().astype(np.int64)
    kv = wl.seqused_kv.cpu().numpy().astype(np.int64)
    D = wl.q.shape[2]
    ori2d = wl.ori_kv.view(-1, D)
    ori_bt = wl.ori_block_table.cpu().numpy().astype(np.int64)
    bs_o, bn_o = wl.ori_kv.shape[1], wl.ori_kv.shape[0]
    if scen >= 2:
        cmp2d = wl.cmp_kv.view(-1, D)
        cmp_bt = wl.cmp_block_table.cpu().numpy().astype(np.int64)
        bs_c, bn_c = wl.cmp_kv.shape[1], wl.cmp_kv.shape[0]
    sinks = wl.sinks.float().cpu().numpy()
    outs, lses = [], []
    for t in tokens:
        t = int(t)
        b = int(np.searchsorted(cu, t, side="right") - 1)
        s = t - int(cu[b])
        act_q = int(cu[b + 1] - cu[b])
        idx_row = wl.cmp_sparse_indices[t, 0].cpu().numpy() if scen == 3 else None
        win, cpos, _ = O.resolve_token_rows(scenario=scen, b=b, s=s, act_q=act_q, act_kv=int(kv[b]),
                                            cmp_idx_row=idx_row, topk=wl.topk, cmp_ratio=wl.cmp_ratio,
                                            ori_win_left=wl.ori_win_left)
        ok = _gather(ori2d, _phys_rows(ori_bt[b], win, bs_o, bn_o))
        ck = _gather(cmp2d, _phys_rows(cmp_bt[b], cpos, bs_c, bn_c)) if scen >= 2 else np.zeros((0, D), np.float32)
        q = wl.q[t].float().cpu().numpy()
        o, l = O.attend_token(q, ok, ck, sinks, wl.softmax_scale)
        outs.append(o[:, : wl.v_head_dim])
        lses.append(l)
    return np.stack(outs), np.stack(lses)


def stratified_tokens(wl, per_request_prefill=None, max_requests=None, seed=0):
    """Flat token rows to check: every request (or ``max_requests`` spread over the length order)
    at its last token; for prefill requests also the first tokens, the tokens at the window edge
    (s_global 127 / 128), where thr reaches topk, the middle and a few random ones."""
    cu = wl.cu_seqlens_q.cpu().numpy().astype(np.int64)
    kv = np.asarray(wl.kv_lens, dtype=np.int64)
    B = len(cu) - 1
    reqs = list(range(B))
    if max_requests and B > max_requests:
        order = np.argsort(kv, kind="stable")
        reqs = sorted(int(order[i]) for i in np.linspace(0, B - 1, max_requests).round().astype(int))
    rng = np.random.default_rng(seed)
    toks = set()
    for b in reqs:
        n = int(cu[b + 1] - cu[b])
        toks.add(int(cu[b]) + n - 1)
        if n > 1 and per_request_prefill:
            ctx = int(kv[b]) - n  # s_global = ctx + s
            cand = [0, 1, 2, 127 - ctx, 128 - ctx, 129 - ctx, wl.cmp_ratio * wl.topk - 1 - ctx, wl.cmp_ratio * wl.topk - ctx, n // 2,
                    n - 2]
            cand += rng.integers(0, n, size=per_request_prefill).tolist()
            for s in cand:
                if 0 <= s < n:
                    toks.add(int(cu[b]) + int(s))
    return sorted(toks)
