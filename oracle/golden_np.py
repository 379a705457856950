"""numpy restatement of the reference fp32 golden attention -- TEST INFRASTRUCTURE ONLY.

Restates ``sparse_attn_sharedkv_tilelang/golden.py`` of the reference
(``yangqiang2018/dsv4_planB``) so that it runs without the reference tree:

* ``resolve_cmp_positions``  <- ``_gather_cmp_kv_tokens``  (golden.py:28-66)
* ``token_window``           <- window bounds in ``sparse_attn_sharedkv_golden_bnsd``
                                (golden.py:125-131)
* ``attend_token``           <- the sink-seeded online softmax loop
                                (golden.py:156-200)
* ``paged_rows``             <- ``unpack_paged_kv`` (golden.py:247-268), evaluated
                                per requested position instead of materialising the
                                dense BNSD copy
* ``sparse_attn_sharedkv_oracle`` <- the whole op over the flat token layout that
                                the kernel ABI uses (``api.py:204-242``)

One deliberate difference: a cmp index below -1 is skipped (and reported in the
returned flags) instead of being used as a negative Python index into the
dense BNSD tensor, which is what ``golden.py:62-66`` would do.  Such indices are
outside the operator contract; the reference generators never produce them.

This module is a checker.  Nothing in the product package imports it.
"""

from __future__ import annotations

from typing import Optional, Sequence

import numpy as np

GOLDEN_S2_TILE = 512  # golden.py:25

FLAG_BAD_INDEX = 1  # a cmp index < -1 was seen and skipped
FLAG_BAD_BLOCK = 2  # a block-table entry >= block_num, or a position past the table


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 value (ties to even), kept as fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    r = ((u + rounding) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(x)
    out[nan] = x[nan]
    return out


def fp16_round(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def cmp_threshold(act_kv: int, act_q: int, s: int, cmp_ratio: int) -> int:
    """``floor((act_kv - act_q + s + 1) / cmp_ratio)`` (golden.py:43-44, mask mode 3)."""
    return (act_kv - act_q + s + 1) // cmp_ratio


def resolve_cmp_positions(idx_row: np.ndarray, thr: int, topk: int):
    """Valid compressed positions of one query token, in slot order.

    Restates golden.py:41-62 with sparse_block_size 1: slots are scanned while
    ``i < min(K, thr)``; the first -1 stops the scan; an index ``>= thr`` is
    skipped; duplicates are kept (each occurrence is its own key).
    Returns ``(positions int64[n], flags)``.
    """
    n = min(int(topk), int(thr))
    if n <= 0:
        return np.zeros(0, dtype=np.int64), 0
    seg = np.asarray(idx_row[:n], dtype=np.int64)
    stops = np.nonzero(seg == -1)[0]
    if stops.size:
        seg = seg[: stops[0]]
    flags = FLAG_BAD_INDEX if np.any(seg < -1) else 0
    keep = (seg >= 0) & (seg < thr)
    return seg[keep], flags


def token_window(act_kv: int, act_q: int, s: int, win_left: int, win_right: int = 0):
    """``(s_global, ori_left, n_win)`` of query ``s`` (golden.py:125-131).

    A negative ``s_global`` (more query tokens than kv tokens) is outside the
    contract; the window is then empty.
    """
    s_global = act_kv - act_q + s
    if s_global < 0:
        return s_global, 0, 0
    ori_left = max(s_global - win_left, 0)
    ori_right = s_global + win_right + 1
    return s_global, ori_left, ori_right - ori_left


def paged_rows(pool: np.ndarray, table_row: np.ndarray, positions: np.ndarray, block_size: int):
    """Rows of logical ``positions`` of one request from a paged pool.

    ``pool`` is ``[block_num * block_size, D]`` fp32.  An unmapped block (-1,
    golden.py:258-260) or a position past the table gives a zero row, as the
    dense copy built by ``unpack_paged_kv`` would.  A table entry
    ``>= block_num`` also gives a zero row and sets ``FLAG_BAD_BLOCK``.
    """
    positions = np.asarray(positions, dtype=np.int64)
    D = pool.shape[1]
    block_num = pool.shape[0] // block_size
    out = np.zeros((positions.size, D), dtype=np.float32)
    if positions.size == 0:
        return out, 0
    blk = positions // block_size
    row = positions % block_size
    in_table = blk < table_row.shape[0]
    phys = np.full(positions.shape, -1, dtype=np.int64)
    phys[in_table] = table_row[blk[in_table]]
    flags = 0
    if np.any(phys >= block_num) or np.any(~in_table):
        flags |= FLAG_BAD_BLOCK
    ok = (phys >= 0) & (phys < block_num)
    out[ok] = pool[phys[ok] * block_size + row[ok]]
    return out, flags


def attend_token(
    q: np.ndarray,
    ori_keys: np.ndarray,
    cmp_keys: np.ndarray,
    sinks: np.ndarray,
    softmax_scale: float,
    s2_tile: int = GOLDEN_S2_TILE,
    p_round=None,
):
    """Sink-seeded online softmax of one query token over its keys (golden.py:156-200).

    ``q`` is ``[G, D]``; ``ori_keys`` / ``cmp_keys`` are ``[n, D]`` (K = V).
    Window keys are walked first, then compressed keys, each in ``s2_tile``
    chunks.  ``p_round`` (e.g. ``bf16_round``) rounds P before the PV product
    as golden.py:193-194 does for low-precision inputs; ``None`` keeps fp32.
    Returns ``(out [G, D], lse [G])`` in fp32 with ``lse = max + ln(sum)``.
    """
    q = np.asarray(q, dtype=np.float32)
    G, D = q.shape
    row_max = np.asarray(sinks, dtype=np.float32).copy()
    row_sum = np.ones(G, dtype=np.float32)
    acc = np.zeros((G, D), dtype=np.float32)
    tiles = []
    for keys in (ori_keys, cmp_keys):
        n = keys.shape[0]
        for t in range(0, n, s2_tile):
            tiles.append(keys[t : t + s2_tile])
    for k_tile in tiles:
        if k_tile.shape[0] == 0:
            continue
        score = (q @ k_tile.T) * np.float32(softmax_scale)
        new_max = np.maximum(row_max, score.max(axis=1))
        alpha = np.exp(row_max - new_max)
        p = np.exp(score - new_max[:, None])
        row_sum = alpha * row_sum + p.sum(axis=1)
        p_low = p_round(p) if p_round is not None else p
        acc = acc * alpha[:, None] + p_low @ k_tile
        row_max = new_max
    out = acc / row_sum[:, None]
    lse = row_max + np.log(row_sum)
    return out.astype(np.float32), lse.astype(np.float32)


def _to_f32(x) -> np.ndarray:
    """Accept a numpy array or a torch tensor (any float dtype) and return fp32 numpy."""
    if hasattr(x, "detach"):
        import torch  # local: the oracle itself does not need torch

        return x.detach().to(torch.float32).cpu().numpy()
    return np.asarray(x, dtype=np.float32)


def _to_i64(x) -> np.ndarray:
    if hasattr(x, "detach"):
        return x.detach().cpu().numpy().astype(np.int64)
    return np.asarray(x, dtype=np.int64)


def resolve_token_rows(
    *,
    scenario: int,
    b: int,
    s: int,
    act_q: int,
    act_kv: int,
    cmp_idx_row,
    topk: int,
    cmp_ratio: int,
    ori_win_left: int,
    ori_win_right: int = 0,
):
    """Logical key positions of one query token.

    Returns ``(window_positions, cmp_positions, flags)``: window positions
    ``ori_left .. s_global`` (golden.py:129-131) and the compressed positions of
    the scenario: none (SWA), ``0 .. thr-1`` (CFA, golden.py:146-150) or the
    resolved top-k slots (SCFA, golden.py:134-145).
    """
    s_global, ori_left, n_win = token_window(act_kv, act_q, s, ori_win_left, ori_win_right)
    win_pos = np.arange(ori_left, ori_left + n_win, dtype=np.int64)
    flags = 0
    if scenario == 1:
        cmp_pos = np.zeros(0, dtype=np.int64)
    else:
        thr = cmp_threshold(act_kv, act_q, s, cmp_ratio)
        if scenario == 2:
            cmp_pos = np.arange(max(thr, 0), dtype=np.int64)
        else:
            cmp_pos, flags = resolve_cmp_positions(cmp_idx_row, thr, topk)
    return win_pos, cmp_pos, flags


def sparse_attn_sharedkv_oracle(
    q,
    *,
    ori_kv,
    ori_block_table,
    seqused_kv: Sequence[int],
    q_prefix: Sequence[int],
    act_q: Sequence[int],
    sinks,
    softmax_scale: float,
    cmp_kv=None,
    cmp_block_table=None,
    cmp_sparse_indices=None,
    cmp_ratio: Optional[int] = None,
    ori_win_left: int = 127,
    ori_win_right: int = 0,
    v_head_dim: Optional[int] = None,
    p_round=None,
    tokens: Optional[Sequence[int]] = None,
):
    """The whole operator on the flat token layout of the kernel ABI.

    ``q`` ``[T, N1, Dq]``; ``ori_kv`` ``[block_num, block_size, 1, Dq]``; tables
    ``[B, table_len]``; ``cmp_sparse_indices`` ``[T, 1, K]``; query token ``s``
    of request ``b`` lives at flat row ``q_prefix[b] + s`` (``api.py:204-242``).
    The scenario follows ``api.py:196-202``.  Returns ``(out [T, N1, Dv],
    lse [T, N1], flags)`` in fp32; rows that belong to no ``(b, s < act_q[b])``
    stay zero (golden.py:97).  ``tokens`` restricts the work to the listed flat
    rows (the others stay zero).
    """
    qf = _to_f32(q)
    T, N1, Dq = qf.shape
    Dv = Dq if v_head_dim is None else int(v_head_dim)
    ori = _to_f32(ori_kv)
    bs_o = ori.shape[1]
    ori_pool = ori.reshape(-1, Dq)
    ori_bt = _to_i64(ori_block_table)
    sinks_f = _to_f32(sinks).reshape(-1)
    seqused_kv = [int(x) for x in _to_i64(seqused_kv).reshape(-1)]
    q_prefix = [int(x) for x in _to_i64(q_prefix).reshape(-1)]
    act_q = [int(x) for x in _to_i64(act_q).reshape(-1)]
    if cmp_kv is None:
        scenario = 1
    elif cmp_sparse_indices is None:
        scenario = 2
    else:
        scenario = 3
    if scenario >= 2:
        cmp = _to_f32(cmp_kv)
        bs_c = cmp.shape[1]
        cmp_pool = cmp.reshape(-1, Dq)
        cmp_bt = _to_i64(cmp_block_table)
    idx = _to_i64(cmp_sparse_indices) if scenario == 3 else None
    topk = idx.shape[-1] if idx is not None else 0

    out = np.zeros((T, N1, Dv), dtype=np.float32)
    lse = np.zeros((T, N1), dtype=np.float32)
    want = None if tokens is None else set(int(t) for t in tokens)
    flags = 0
    for b in range(len(act_q)):
        for s in range(act_q[b]):
            t = q_prefix[b] + s
            if want is not None and t not in want:
                continue
            win_pos, cmp_pos, f = resolve_token_rows(
                scenario=scenario,
                b=b,
                s=s,
                act_q=act_q[b],
                act_kv=seqused_kv[b],
                cmp_idx_row=idx[t, 0] if idx is not None else None,
                topk=topk,
                cmp_ratio=cmp_ratio if cmp_ratio is not None else 4,
                ori_win_left=ori_win_left,
                ori_win_right=ori_win_right,
            )
            flags |= f
            ori_keys, f = paged_rows(ori_pool, ori_bt[b], win_pos, bs_o)
            flags |= f
            if scenario >= 2:
                cmp_keys, f = paged_rows(cmp_pool, cmp_bt[b], cmp_pos, bs_c)
                flags |= f
            else:
                cmp_keys = np.zeros((0, Dq), dtype=np.float32)
            o, l = attend_token(qf[t], ori_keys, cmp_keys, sinks_f, softmax_scale, p_round=p_round)
            out[t] = o[:, :Dv]
            lse[t] = l
    return out, lse, flags


def algorithmic_counts(
    *,
    scenario: int,
    seqused_kv: Sequence[int],
    act_q: Sequence[int],
    q_prefix: Sequence[int],
    cmp_sparse_indices=None,
    cmp_ratio: int = 4,
    ori_win_left: int = 127,
):
    """Per-token ``(n_win, n_cmp)`` and per-request unique-row counts.

    Used for the algorithmic bytes / FLOPs of a workload: FLOPs count every key
    of every token; bytes count each distinct KV row of a request once.
    """
    idx = _to_i64(cmp_sparse_indices) if cmp_sparse_indices is not None else None
    topk = idx.shape[-1] if idx is not None else 0
    n_win_tok, n_cmp_tok, uniq_rows = [], [], []
    for b in range(len(act_q)):
        win_set, cmp_set = set(), set()
        for s in range(int(act_q[b])):
            t = int(q_prefix[b]) + s
            w, c, _ = resolve_token_rows(
                scenario=scenario,
                b=b,
                s=s,
                act_q=int(act_q[b]),
                act_kv=int(seqused_kv[b]),
                cmp_idx_row=idx[t, 0] if idx is not None else None,
                topk=topk,
                cmp_ratio=cmp_ratio,
                ori_win_left=ori_win_left,
            )
            n_win_tok.append(w.size)
            n_cmp_tok.append(c.size)
            if w.size:
                win_set.update(range(int(w[0]), int(w[-1]) + 1))
            cmp_set.update(c.tolist())
        uniq_rows.append(len(win_set) + len(cmp_set))
    return np.array(n_win_tok), np.array(n_cmp_tok), np.array(uniq_rows)


__all__ = [
    "GOLDEN_S2_TILE",
    "FLAG_BAD_INDEX",
    "FLAG_BAD_BLOCK",
    "bf16_round",
    "fp16_round",
    "cmp_threshold",
    "resolve_cmp_positions",
    "token_window",
    "paged_rows",
    "attend_token",
    "resolve_token_rows",
    "sparse_attn_sharedkv_oracle",
    "algorithmic_counts",
]
