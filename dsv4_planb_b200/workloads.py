"""Seeded synthetic workloads for the five BASELINE configurations.

The reference publishes no dataset for this operator; its tests regenerate
inputs from seeds (``test_sparse_attn_sharedkv.py:238-391``).  These
generators follow the same recipe at the BASELINE shapes:

* q, ori_kv and cmp_kv are N(0, 1) * 0.5 drawn in fp32 and stored as bf16;
* the ori / cmp paged pools are filled block by block in a seeded random
  permutation of physical blocks, unused table slots are -1
  (``golden.py:315-408``);
* each query token takes ``min(thr, K)`` distinct random compressed indices
  below its causal limit ``thr = (act_kv - act_q + s + 1) // cmp_ratio``,
  padded with -1 (``golden.py:442-473``);
* sinks are U[-1, 1] fp32 and ``softmax_scale = 1 / sqrt(D_qk)``.

Seeds: ``seed`` for q / lengths, ``seed + 1`` for the compressed pool,
``seed + 7`` for the indices, as the reference tests do
(``test_sparse_attn_sharedkv.py:243-298``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np
import torch


@dataclass
class Workload:
    name: str
    q: torch.Tensor  # [T, N1, Dq]
    ori_kv: torch.Tensor  # [ori_block_num, bs, 1, Dq]
    ori_block_table: torch.Tensor  # [B, ori_table_len] int32
    cmp_kv: Optional[torch.Tensor]  # [cmp_block_num, bs, 1, Dq]
    cmp_block_table: Optional[torch.Tensor]  # [B, cmp_table_len] int32
    cmp_sparse_indices: Optional[torch.Tensor]  # [T, 1, K] int32
    cu_seqlens_q: torch.Tensor  # [B + 1] int32
    seqused_kv: torch.Tensor  # [B] int32
    sinks: torch.Tensor  # [N1] fp32
    softmax_scale: float
    cmp_ratio: int
    topk: int
    v_head_dim: int
    ori_win_left: int = 127
    q_lens: List[int] = field(default_factory=list)
    kv_lens: List[int] = field(default_factory=list)

    @property
    def num_tokens(self) -> int:
        return int(self.q.shape[0])

    def api_kwargs(self) -> dict:
        """Keyword arguments of ``sparse_attn_sharedkv`` for this workload (TND layout)."""
        return dict(
            ori_kv=self.ori_kv,
            cmp_kv=self.cmp_kv,
            cmp_sparse_indices=self.cmp_sparse_indices,
            ori_block_table=self.ori_block_table,
            cmp_block_table=self.cmp_block_table,
            cu_seqlens_q=self.cu_seqlens_q,
            seqused_kv=self.seqused_kv,
            sinks=self.sinks,
            softmax_scale=self.softmax_scale,
            cmp_ratio=self.cmp_ratio,
            ori_win_left=self.ori_win_left,
            layout_q="TND",
            layout_kv="PA_ND",
            v_head_dim=self.v_head_dim,
        )

    def to(self, device) -> "Workload":
        def mv(t):
            return None if t is None else t.to(device)

        return Workload(
            name=self.name,
            q=mv(self.q),
            ori_kv=mv(self.ori_kv),
            ori_block_table=mv(self.ori_block_table),
            cmp_kv=mv(self.cmp_kv),
            cmp_block_table=mv(self.cmp_block_table),
            cmp_sparse_indices=mv(self.cmp_sparse_indices),
            cu_seqlens_q=mv(self.cu_seqlens_q),
            seqused_kv=mv(self.seqused_kv),
            sinks=mv(self.sinks),
            softmax_scale=self.softmax_scale,
            cmp_ratio=self.cmp_ratio,
            topk=self.topk,
            v_head_dim=self.v_head_dim,
            ori_win_left=self.ori_win_left,
            q_lens=list(self.q_lens),
            kv_lens=list(self.kv_lens),
        )


def _paged_pool(lens, block_size, dim, dtype, gen, device, std, rng):
    """A paged pool holding ``lens[b]`` rows per request, in a random block order."""
    per_req = [math.ceil(n / block_size) if n > 0 else 0 for n in lens]
    total = sum(per_req)
    block_num = max(total, 1)
    pool = torch.empty((block_num, block_size, 1, dim), dtype=dtype, device=device)
    chunk = 4096  # blocks per fill, bounds the fp32 staging buffer
    for s in range(0, block_num, chunk):
        e = min(block_num, s + chunk)
        x = torch.randn((e - s, block_size, 1, dim), generator=gen, device=device, dtype=torch.float32)
        pool[s:e] = (x * std).to(dtype)
    phys = rng.permutation(block_num).astype(np.int32)
    table_len = max(max(per_req) if per_req else 0, 1)
    table = np.full((len(lens), table_len), -1, dtype=np.int32)
    cur = 0
    for b, nb in enumerate(per_req):
        table[b, :nb] = phys[cur : cur + nb]
        cur += nb
    return pool, torch.from_numpy(table).to(device)


def _indices(q_lens, kv_lens, topk, cmp_ratio, gen, device, method):
    """Per-token random distinct top-k indices below the causal limit, -1 padded."""
    T = sum(q_lens)
    idx = torch.full((T, 1, topk), -1, dtype=torch.int32, device=device)
    if topk == 0:
        return idx
    t0 = 0
    thr_all = []
    for b, (ql, kl) in enumerate(zip(q_lens, kv_lens)):
        for s in range(ql):
            thr_all.append(max(0, (kl - ql + s + 1) // cmp_ratio))
        t0 += ql
    if method == "randperm":
        for t, thr in enumerate(thr_all):
            if thr > 0:
                take = min(thr, topk)
                perm = torch.randperm(thr, generator=gen, device="cpu").to(torch.int32)
                idx[t, 0, :take] = perm[:take].to(device)
        return idx
    # "keys": a uniformly random subset per token from the top-k of random keys,
    # evaluated in token chunks so the key matrix stays small.
    thr_t = torch.tensor(thr_all, dtype=torch.int64, device=device)
    max_thr = int(thr_t.max().item()) if T else 0
    if max_thr == 0:
        return idx
    step = max(1, (1 << 27) // max_thr)
    for s in range(0, T, step):
        e = min(T, s + step)
        keys = torch.rand((e - s, max_thr), generator=gen, device=device)
        col = torch.arange(max_thr, device=device)[None, :]
        keys = torch.where(col < thr_t[s:e, None], keys, torch.full_like(keys, -1.0))
        k = min(topk, max_thr)
        vals, pos = torch.topk(keys, k, dim=1)
        pos = torch.where(vals >= 0, pos, torch.full_like(pos, -1)).to(torch.int32)
        idx[s:e, 0, :k] = pos
    return idx


def make_workload(
    *,
    name: str,
    q_lens: List[int],
    kv_lens: List[int],
    num_heads: int,
    head_dim: int = 576,
    v_head_dim: int = 512,
    topk: int = 2048,
    cmp_ratio: int = 4,
    block_size: int = 128,
    seed: int = 42,
    dtype: torch.dtype = torch.bfloat16,
    device="cpu",
    std: float = 0.5,
    index_method: Optional[str] = None,
    scenario: int = 3,
) -> Workload:
    """Build one seeded workload (see the module docstring for the recipe)."""
    assert len(q_lens) == len(kv_lens)
    device = torch.device(device)
    if index_method is None:
        index_method = "randperm" if device.type == "cpu" else "keys"
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    rng = np.random.default_rng(seed)
    T = sum(q_lens)
    q = (torch.randn((T, num_heads, head_dim), generator=g, device=device) * std).to(dtype)
    ori_kv, ori_bt = _paged_pool(kv_lens, block_size, head_dim, dtype, g, device, std, rng)
    sinks = (torch.rand((num_heads,), generator=g, device=device) * 2 - 1).to(torch.float32)
    cmp_kv = cmp_bt = idx = None
    if scenario >= 2:
        g1 = torch.Generator(device=device)
        g1.manual_seed(seed + 1)
        cmp_lens = [k // cmp_ratio for k in kv_lens]
        cmp_kv, cmp_bt = _paged_pool(cmp_lens, block_size, head_dim, dtype, g1, device, std, np.random.default_rng(seed + 1))
    if scenario == 3:
        gi = torch.Generator(device="cpu" if index_method == "randperm" else device)
        gi.manual_seed(seed + 7)
        idx = _indices(q_lens, kv_lens, topk, cmp_ratio, gi, device, index_method)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32), device=device)
    seq = torch.tensor(np.asarray(kv_lens, dtype=np.int32), device=device)
    return Workload(
        name=name,
        q=q,
        ori_kv=ori_kv,
        ori_block_table=ori_bt,
        cmp_kv=cmp_kv,
        cmp_block_table=cmp_bt,
        cmp_sparse_indices=idx,
        cu_seqlens_q=cu,
        seqused_kv=seq,
        sinks=sinks,
        softmax_scale=1.0 / math.sqrt(head_dim),
        cmp_ratio=cmp_ratio,
        topk=topk if scenario == 3 else 0,
        v_head_dim=v_head_dim,
        q_lens=list(q_lens),
        kv_lens=list(kv_lens),
    )


def config_lengths(cfg: str, seed: int = 42, batch=None):
    """``(q_lens, kv_lens, num_heads, topk)`` of a BASELINE configuration.

    ``batch`` overrides the request count of the decode configs c2 and c3 (same length
    distribution), for small-batch measurements."""
    rng = np.random.default_rng(seed)
    if cfg == "c1":
        kv = rng.integers(512, 2048 + 1, size=4).tolist()
        return [1] * 4, kv, 16, 256
    if cfg == "c2":
        b = batch or 64
        kv = rng.integers(8192, 32768 + 1, size=b).tolist()
        return [1] * b, kv, 128, 2048
    if cfg == "c3":
        b = batch or 32
        kv = rng.integers(4096, 65536 + 1, size=b).tolist()
        return [2] * b, kv, 128, 2048
    if cfg == "c4":
        ctx = rng.integers(0, 16384 + 1, size=4).tolist()
        return [8192] * 4, [c + 8192 for c in ctx], 128, 2048
    if cfg == "c5":
        kv = np.floor(np.exp(rng.uniform(math.log(1024), math.log(131072), size=512))).astype(np.int64).tolist()
        return [1] * 512, kv, 128, 2048
    raise ValueError(f"unknown config {cfg!r}")


CONFIG_DESCRIPTIONS = {
    "c1": "CPU decode: B=4, q_len 1, N1=16, D_qk 576 / D_v 512, seq U[512, 2048], K=256",
    "c2": "production decode: B=64, q_len 1, N1=128, D_qk 576 / D_v 512, seq U[8K, 32K], K=2048",
    "c3": "MTP decode: B=32, q_len 2, N1=128, seq U[4K, 64K], K=2048",
    "c4": "chunked prefill: 4 x 8192 new tokens on ctx U[0, 16K], N1=128, K=2048",
    "c5": "mixed: 512 decode requests, seq log-U[1K, 128K], N1=128, K=2048",
}


def config_workload(cfg: str, *, seed: int = 42, device="cpu", dtype=torch.bfloat16, batch=None, **kw) -> Workload:
    q_lens, kv_lens, n1, topk = config_lengths(cfg, seed, batch)
    return make_workload(
        name=cfg, q_lens=q_lens, kv_lens=kv_lens, num_heads=n1, topk=topk, seed=seed, device=device, dtype=dtype, **kw
    )
