"""Restated reference input generators -- TEST INFRASTRUCTURE ONLY.

Reproduces, call for call on torch / numpy RNGs, how the reference test suite
builds its cases, so that the reference's own paramsets can be regenerated on a
machine without the reference tree:

* ``PARAMSETS``         <- ``SCENARIOS`` (test_sparse_attn_sharedkv.py:81-220)
                           plus the S1=1024 prefill shrink
                           (test_sparse_attn_sharedkv_fast.py:76-105)
* ``ref_build_case``    <- ``_build_case`` (test_sparse_attn_sharedkv.py:238-326),
                           using restatements of ``gen_ori_kv_paged`` /
                           ``gen_cmp_kv_paged`` / ``gen_cmp_sparse_indices_tnd``
                           (golden.py:315-473)

The fixtures record sha256 digests of the inputs the reference produced, and
``tests/test_oracle_pins.py`` checks these restatements against them.
"""

from __future__ import annotations

import hashlib
import math

import numpy as np
import torch

_BASE = dict(
    layout_q="TND",
    B=1,
    N1=64,
    N2=1,
    D=512,
    block_size1=128,
    softmax_scale=0.04419417,
    ori_win_left=127,
    ori_win_right=0,
    ori_mask_mode=4,
    cmp_mask_mode=3,
)

PARAMSETS = {
    "scfa_decode": dict(_BASE, scenario=3, S1=1, T1=1, K=512, block_num1=65, block_num2=17, block_size2=128,
                        cu_seqlens_q=[0, 1], seqused_kv=[8193], cmp_ratio=4),
    "swa_decode": dict(_BASE, scenario=1, S1=1, T1=1, K=0, block_num1=65, block_num2=1, block_size2=1,
                       cu_seqlens_q=[0, 1], seqused_kv=[8193], cmp_ratio=4),
    "cfa_decode": dict(_BASE, scenario=2, S1=1, T1=1, K=512, block_num1=65, block_num2=17, block_size2=128,
                       cu_seqlens_q=[0, 1], seqused_kv=[8193], cmp_ratio=128),
    "scfa_prefill": dict(_BASE, scenario=3, S1=8192, T1=8192, K=512, block_num1=65, block_num2=17, block_size2=128,
                         cu_seqlens_q=[0, 8192], seqused_kv=[8192], cmp_ratio=4),
    "swa_prefill": dict(_BASE, scenario=1, S1=8192, T1=8192, K=0, block_num1=65, block_num2=1, block_size2=1,
                        cu_seqlens_q=[0, 8192], seqused_kv=[8192], cmp_ratio=4),
    "cfa_prefill": dict(_BASE, scenario=2, S1=8192, T1=8192, K=512, block_num1=65, block_num2=17, block_size2=128,
                        cu_seqlens_q=[0, 8192], seqused_kv=[8192], cmp_ratio=128),
}


def shrink(name: str, s1: int = 1024) -> dict:
    """Small-S1 prefill paramset (test_sparse_attn_sharedkv_fast.py:79-99)."""
    cfg = dict(PARAMSETS[name])
    cfg.update(S1=s1, T1=s1, cu_seqlens_q=[0, s1], seqused_kv=[s1])
    cfg["block_num1"] = math.ceil(s1 / cfg["block_size1"]) + 2
    if cfg["scenario"] >= 2:
        cfg["block_num2"] = max(1, math.ceil((s1 // cfg["cmp_ratio"]) / cfg["block_size2"])) + 1
    return cfg


for _n in ("swa_prefill", "cfa_prefill", "scfa_prefill"):
    PARAMSETS[_n.replace("_prefill", "_prefill_fast")] = shrink(_n)


def _ori_paged(B, N2, D, block_num, block_size, seqused_kv, dtype, lo, hi, rng):
    """golden.py:315-360."""
    max_s = max(seqused_kv)
    max_blk = math.ceil(max_s / block_size)
    dense = (torch.rand((B, N2, max_s, D)) * (hi - lo) + lo).to(dtype)
    per_b = [math.ceil(s / block_size) for s in seqused_kv]
    if block_num < sum(per_b):
        raise ValueError("ori block_num too small")
    phys = rng.permutation(block_num).astype(np.int32)
    table = np.full((B, max_blk), -1, dtype=np.int32)
    cur = 0
    for b, nb in enumerate(per_b):
        for i in range(nb):
            table[b, i] = phys[cur]
            cur += 1
    pa = torch.zeros((block_num, block_size, N2, D), dtype=dtype)
    for b in range(B):
        for i in range(per_b[b]):
            p = int(table[b, i])
            s0 = i * block_size
            s1 = min(s0 + block_size, max_s)
            pa[p, : s1 - s0] = dense[b, :, s0:s1, :].permute(1, 0, 2)
    return pa, torch.tensor(table, dtype=torch.int32)


def _cmp_paged(B, N2, D, block_num, block_size, seqused_kv, cmp_ratio, dtype, lo, hi, rng):
    """golden.py:363-408."""
    cmp_seqs = [s // cmp_ratio for s in seqused_kv]
    max_cmp = max(cmp_seqs) if cmp_seqs else 0
    max_blk = math.ceil(max_cmp / block_size) if max_cmp > 0 else 1
    dense = (torch.rand((B, N2, max(max_cmp, 1), D)) * (hi - lo) + lo).to(dtype)
    per_b = [math.ceil(s / block_size) if s > 0 else 0 for s in cmp_seqs]
    if block_num < max(sum(per_b), 1):
        raise ValueError("cmp block_num too small")
    phys = rng.permutation(block_num).astype(np.int32)
    table = np.full((B, max(max_blk, 1)), -1, dtype=np.int32)
    cur = 0
    for b, nb in enumerate(per_b):
        for i in range(nb):
            table[b, i] = phys[cur]
            cur += 1
    pa = torch.zeros((block_num, block_size, N2, D), dtype=dtype)
    for b in range(B):
        for i in range(per_b[b]):
            p = int(table[b, i])
            s0 = i * block_size
            s1 = min(s0 + block_size, cmp_seqs[b])
            if s1 - s0 > 0:
                pa[p, : s1 - s0] = dense[b, :, s0:s1, :].permute(1, 0, 2)
    return pa, torch.tensor(table, dtype=torch.int32)


def _indices_tnd(B, T1, N2, K, cu, seqused_kv, cmp_ratio, gen):
    """golden.py:442-473."""
    idx = torch.full((T1, N2, K), -1, dtype=torch.int32)
    for b in range(B):
        s0, s1 = int(cu[b]), int(cu[b + 1])
        act_q = s1 - s0
        act_kv = int(seqused_kv[b])
        for n2 in range(N2):
            for s in range(act_q):
                cur = max(0, (act_kv - act_q + s + 1) // cmp_ratio)
                perm = torch.randperm(cur, generator=gen).to(torch.int32) if cur > 0 else torch.empty((0,), dtype=torch.int32)
                take = min(cur, K)
                idx[s0 + s, n2, :take] = perm[:take]
    return idx


def ref_build_case(cfg: dict, dtype: torch.dtype, seed: int = 42) -> dict:
    """Inputs of the reference ``_build_case`` for a TND paramset (no golden run)."""
    assert cfg["layout_q"] == "TND"
    torch.manual_seed(seed)
    np.random.seed(seed)
    B, T1, N1, N2, D = cfg["B"], cfg["T1"], cfg["N1"], cfg["N2"], cfg["D"]
    scen = cfg["scenario"]
    q = (torch.rand((T1, N1, D)) * 20 - 10).to(dtype)
    ori, ori_bt = _ori_paged(B, N2, D, cfg["block_num1"], cfg["block_size1"], cfg["seqused_kv"], dtype, -10, 10,
                             np.random.default_rng(seed))
    cmp = cmp_bt = idx = None
    if scen >= 2:
        cmp, cmp_bt = _cmp_paged(B, N2, D, cfg["block_num2"], cfg["block_size2"], cfg["seqused_kv"], cfg["cmp_ratio"],
                                 dtype, -5, 10, np.random.default_rng(seed + 1))
    if scen == 3:
        g = torch.Generator()
        g.manual_seed(seed + 7)
        idx = _indices_tnd(B, T1, N2, cfg["K"], cfg["cu_seqlens_q"], cfg["seqused_kv"], cfg["cmp_ratio"], g)
    sinks = (torch.rand(N1) * 2 - 1).to(torch.float32)
    return dict(q=q, ori_kv=ori, ori_block_table=ori_bt, cmp_kv=cmp, cmp_block_table=cmp_bt,
                cmp_sparse_indices=idx, sinks=sinks,
                cu_seqlens_q=torch.tensor(cfg["cu_seqlens_q"], dtype=torch.int32),
                seqused_kv=torch.tensor(cfg["seqused_kv"], dtype=torch.int32))


def digest(t) -> str:
    """sha256 of a tensor's raw bytes (None -> "none")."""
    if t is None:
        return "none"
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()
