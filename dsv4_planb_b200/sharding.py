"""Request sharding of one decode batch across the GPUs of a node.

Requests are independent (no step of the path exchanges data between
requests), so each rank runs ``sparse_attn_sharedkv`` on its own subset of requests over its own
slice of the paged pools, with block ids remapped to that slice.  NCCL is used
only to bring outputs back together for verification.

* ``partition_requests``  greedy LPT over a per-request cost (window keys plus
  compressed keys; by default ``min(128, kv) + min(topk, kv // ratio)`` per
  query token), so ranks get equal work rather than equal counts;
* ``shard_workload``      the rank's sub-workload: its requests' query rows,
  indices, lengths, and the physical blocks its block tables reference,
  compacted into a local pool with remapped tables;
* ``gather_outputs``      ``all_gather`` of every rank's (out, lse, request ids)
  padded to a common size, reassembled in the original token order;
* ``split_hint``          the piece size (``split_tiles``) that best balances a
  rank's tokens over the tensor-core kernel's clusters, by simulating its queue.
"""

from __future__ import annotations

import heapq
from typing import List, Sequence

import torch

from .workloads import Workload


def request_costs(q_lens: Sequence[int], kv_lens: Sequence[int], topk: int, cmp_ratio: int = 4,
                  win: int = 128) -> List[int]:
    costs = []
    for ql, kv in zip(q_lens, kv_lens):
        c = 0
        for s in range(ql):
            sg = kv - ql + s
            c += min(win, max(sg + 1, 0)) + min(topk, max((sg + 1) // cmp_ratio, 0))
        costs.append(c)
    return costs


def token_tiles(q_lens: Sequence[int], kv_lens: Sequence[int], topk: int, cmp_ratio: int = 4,
                win: int = 128, tile: int = 64) -> List[int]:
    """Tiles of ``tile`` keys of every query token, in flat token order (SCFA, as the kernel counts
    them: window tiles plus compressed tiles, assuming every top-k slot below the causal limit is
    a valid index)."""
    tiles = []
    for ql, kv in zip(q_lens, kv_lens):
        for s in range(ql):
            sg = kv - ql + s
            n_win = min(win, max(sg + 1, 0))
            n_cmp = min(topk, max((sg + 1) // cmp_ratio, 0))
            tiles.append(-(-n_win // tile) + -(-n_cmp // tile))
    return tiles


def queue_makespan(tiles: Sequence[int], split_tiles: int, clusters: int = 74, unit_cost: float = 2.25,
                   piece_cost: float = 4.0) -> float:
    """Simulated duration, in tile periods, of the tensor-core kernel's dynamic queue over
    ``tiles``: units in the kernel's order (piece-major: the first piece of every token, then the
    second pieces, ...), each taken by the cluster that frees first.  A unit costs its tiles plus
    ``unit_cost`` (Q load and pipeline turn-over); a piece of a split token ``piece_cost`` more
    (its partial output and share of the merge).  The default costs are fitted to B200 timings
    of c5 request shards split at 12-28 tiles."""
    pieces = []
    for n in tiles:
        if split_tiles and n > split_tiles:
            k = -(-n // split_tiles)
            pieces.append([split_tiles] * (k - 1) + [n - split_tiles * (k - 1)])
        else:
            pieces.append([n])
    heap = [0.0] * clusters
    depth = max((len(p) for p in pieces), default=0)
    for k in range(depth):
        for p in pieces:
            if k < len(p):
                cost = p[k] + unit_cost + (piece_cost if len(p) > 1 else 0.0)
                heapq.heapreplace(heap, heap[0] + cost)
    return max(heap) if heap else 0.0


def split_hint(tiles: Sequence[int], clusters: int = 74, min_gain: float = 0.25) -> int:
    """``split_tiles`` for a batch whose tokens have ``tiles`` tiles each: the piece size with the
    shortest simulated queue, or 0 (no split) unless that beats no split by ``min_gain``.

    The queue model overrates splitting where most clusters already hold a token: on B200 the c5
    request shards of 2, 4 and 8 ranks gained at most 4 % from any piece size (4 ranks: 176 us at 17
    tiles against 183 us whole) and lost at 8 ranks (105 us whole, 108-122 us split), while the
    model promised 14-16 %.  Hence the high threshold: split when the model's gain is large, as for
    batches of far fewer tokens than clusters."""
    if not tiles:
        return 0
    base = queue_makespan(tiles, 0, clusters)
    best, best_m = base, 0
    for m in range(4, max(tiles)):
        t = queue_makespan(tiles, m, clusters)
        if t < best:
            best, best_m = t, m
    return best_m if best < (1.0 - min_gain) * base else 0


def partition_requests(costs: Sequence[int], world: int) -> List[List[int]]:
    """Longest-processing-time assignment of requests to ``world`` ranks.

    Each rank's list comes in descending cost, the order in which the rank should submit its
    requests: the attention kernel hands tokens to its clusters in index order from a dynamic
    queue, so the long requests start first and the short ones fill the tail."""
    heap = [(0, r) for r in range(world)]
    heapq.heapify(heap)
    parts: List[List[int]] = [[] for _ in range(world)]
    for b in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        load, r = heapq.heappop(heap)
        parts[r].append(b)
        heapq.heappush(heap, (load + costs[b], r))
    return parts


def _compact_pool(pool: torch.Tensor, table: torch.Tensor):
    """Copy the blocks ``table`` references into a new pool; return it and the remapped table."""
    used = table[table >= 0].unique(sorted=True)
    remap = torch.full((pool.shape[0],), -1, dtype=torch.int32, device=table.device)
    remap[used.long()] = torch.arange(used.numel(), dtype=torch.int32, device=table.device)
    new_table = torch.where(table >= 0, remap[table.clamp(min=0).long()], table)
    new_pool = pool[used.long()] if used.numel() else pool[:1]
    return new_pool.contiguous(), new_table.contiguous()


def shard_workload(wl: Workload, requests: Sequence[int]) -> Workload:
    """The sub-workload of ``requests`` (original request ids, in the order given)."""
    cu = wl.cu_seqlens_q.tolist()
    rows = [t for b in requests for t in range(cu[b], cu[b + 1])]
    row_idx = torch.tensor(rows, dtype=torch.long, device=wl.q.device)
    req_idx = torch.tensor(list(requests), dtype=torch.long, device=wl.q.device)
    q_lens = [wl.q_lens[b] for b in requests]
    kv_lens = [wl.kv_lens[b] for b in requests]
    ori_kv, ori_bt = _compact_pool(wl.ori_kv, wl.ori_block_table[req_idx])
    cmp_kv = cmp_bt = None
    if wl.cmp_kv is not None:
        cmp_kv, cmp_bt = _compact_pool(wl.cmp_kv, wl.cmp_block_table[req_idx])
    cu_new = torch.zeros(len(requests) + 1, dtype=torch.int32, device=wl.q.device)
    if q_lens:
        cu_new[1:] = torch.tensor(q_lens, dtype=torch.int32, device=wl.q.device).cumsum(0)
    return Workload(
        name=f"{wl.name}[shard]", q=wl.q[row_idx].contiguous(), ori_kv=ori_kv, ori_block_table=ori_bt, cmp_kv=cmp_kv,
        cmp_block_table=cmp_bt,
        cmp_sparse_indices=None if wl.cmp_sparse_indices is None else wl.cmp_sparse_indices[row_idx].contiguous(),
        cu_seqlens_q=cu_new, seqused_kv=wl.seqused_kv[req_idx].contiguous(), sinks=wl.sinks,
        softmax_scale=wl.softmax_scale, cmp_ratio=wl.cmp_ratio, topk=wl.topk, v_head_dim=wl.v_head_dim,
        ori_win_left=wl.ori_win_left, q_lens=q_lens, kv_lens=kv_lens)


def gather_outputs(out: torch.Tensor, lse: torch.Tensor, requests: Sequence[int], q_lens_all: Sequence[int],
                   group=None):
    """Reassemble every rank's outputs in the original flat token order (collective)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    dev = out.device
    cu = [0]
    for ql in q_lens_all:
        cu.append(cu[-1] + ql)
    rows = torch.tensor([t for b in requests for t in range(cu[b], cu[b + 1])], dtype=torch.long, device=dev)
    n = torch.tensor([rows.numel()], dtype=torch.long, device=dev)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    cap = int(max(int(s.item()) for s in sizes))
    pad = cap - rows.numel()
    o = torch.cat([out.float(), out.new_zeros((pad,) + tuple(out.shape[1:])).float()]) if pad else out.float()
    l_ = torch.cat([lse, lse.new_zeros((pad, lse.shape[1]))]) if pad else lse
    r = torch.cat([rows, rows.new_full((pad,), -1)]) if pad else rows
    os_ = [torch.empty_like(o) for _ in range(world)]
    ls_ = [torch.empty_like(l_) for _ in range(world)]
    rs_ = [torch.empty_like(r) for _ in range(world)]
    dist.all_gather(os_, o.contiguous(), group=group)
    dist.all_gather(ls_, l_.contiguous(), group=group)
    dist.all_gather(rs_, r.contiguous(), group=group)
    T = cu[-1]
    full_o = torch.zeros((T,) + tuple(out.shape[1:]), dtype=torch.float32, device=dev)
    full_l = torch.zeros((T, lse.shape[1]), dtype=lse.dtype, device=dev)
    for o_i, l_i, r_i in zip(os_, ls_, rs_):
        keep = r_i >= 0
        full_o[r_i[keep]] = o_i[keep]
        full_l[r_i[keep]] = l_i[keep]
    return full_o, full_l
