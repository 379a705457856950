"""Request sharding across ranks, with world-size-2 gloo process groups on the CPU.

Each rank takes its LPT share of the requests, compacts the pools its block
tables touch, computes its shard (the CPU oracle stands in for the GPU kernel
here; the per-token math does not depend on which rank runs it) and the
outputs are all-gathered back into the original token order.  The result must
equal the unsharded computation exactly.  A second test kills one rank before
the collective and checks that the survivor fails with an error (bounded by the
process-group timeout) rather than hanging.
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dsv4_planb_b200 import sharding as S
from dsv4_planb_b200 import workloads as W
from oracle import golden_np as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _wl():
    return W.make_workload(name="shard", q_lens=[1, 2, 1, 3, 1], kv_lens=[700, 1500, 300, 2600, 900], num_heads=16,
                           topk=128, seed=3)


def _oracle(wl):
    out, lse, _ = O.sparse_attn_sharedkv_oracle(
        wl.q, ori_kv=wl.ori_kv, ori_block_table=wl.ori_block_table, seqused_kv=wl.seqused_kv,
        q_prefix=wl.cu_seqlens_q[:-1], act_q=wl.cu_seqlens_q[1:] - wl.cu_seqlens_q[:-1], sinks=wl.sinks,
        softmax_scale=wl.softmax_scale, cmp_kv=wl.cmp_kv, cmp_block_table=wl.cmp_block_table,
        cmp_sparse_indices=wl.cmp_sparse_indices, cmp_ratio=wl.cmp_ratio, v_head_dim=wl.v_head_dim)
    return torch.from_numpy(out), torch.from_numpy(lse)


def _worker(rank, world, port, result_path, fail_rank):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        wl = _wl()
        costs = S.request_costs(wl.q_lens, wl.kv_lens, wl.topk, wl.cmp_ratio)
        parts = S.partition_requests(costs, world)
        mine = parts[rank]
        shard = S.shard_workload(wl, mine)
        if rank == fail_rank:
            os._exit(3)  # this rank dies between steps, before the collective
        out, lse = _oracle(shard)
        full_o, full_l = S.gather_outputs(out, lse, mine, wl.q_lens)
        if rank == 0:
            torch.save({"out": full_o, "lse": full_l, "parts": parts}, result_path)
    except Exception as e:  # noqa: BLE001
        if rank == 0:
            torch.save({"error": repr(e)}, result_path)
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def test_partition_balances_cost():
    costs = [100, 90, 80, 70, 10, 10, 5]
    parts = S.partition_requests(costs, 2)
    loads = [sum(costs[i] for i in p) for p in parts]
    assert sorted(sum(parts, [])) == list(range(len(costs)))
    assert max(loads) - min(loads) <= max(costs)


def test_rank_lists_run_largest_first():
    costs = [5, 100, 10, 90, 80, 70, 10]
    for p in S.partition_requests(costs, 2):
        assert [costs[i] for i in p] == sorted((costs[i] for i in p), reverse=True)


def test_token_tiles_and_split_hint():
    # window tiles + compressed tiles per token, as the kernel counts them
    assert S.token_tiles([1, 1, 2], [20000, 300, 129], 2048) == [2 + 32, 2 + 2, 2 + 1, 2 + 1]
    # a uniform decode batch of fewer tokens than clusters gains nothing from cutting tokens
    assert S.split_hint([34] * 64) == 0
    # far fewer long tokens than clusters: cutting them fills the idle clusters
    tiles = [34] * 16
    m = S.split_hint(tiles)
    assert 4 <= m < 34
    assert S.queue_makespan(tiles, m) < 0.75 * S.queue_makespan(tiles, 0)
    assert S.queue_makespan([], 0) == 0.0 and S.split_hint([]) == 0
    # the c5 request shards of 1-8 ranks: measured on B200, no piece size gains more than 4 %
    q_all, kv_all, _, topk = W.config_lengths("c5", 42)
    for world in (1, 2, 4, 8):
        for part in S.partition_requests(S.request_costs(q_all, kv_all, topk), world):
            assert S.split_hint(S.token_tiles([q_all[i] for i in part], [kv_all[i] for i in part], topk)) == 0


def test_shard_remaps_blocks_and_keeps_rows():
    wl = _wl()
    sh = S.shard_workload(wl, [1, 3])
    assert sh.q.shape[0] == 5 and sh.ori_kv.shape[0] <= wl.ori_kv.shape[0]
    assert int(sh.ori_block_table.max()) < sh.ori_kv.shape[0]
    out_full, _ = _oracle(wl)
    out_sh, _ = _oracle(sh)
    cu = wl.cu_seqlens_q.tolist()
    rows = [t for b in (1, 3) for t in range(cu[b], cu[b + 1])]
    np.testing.assert_array_equal(out_sh.numpy(), out_full.numpy()[rows])


def test_two_rank_sharded_run_equals_unsharded(tmp_path):
    port = _free_port()
    path = str(tmp_path / "res.pt")
    mp.start_processes(_worker, args=(2, port, path, -1), nprocs=2, join=True, start_method="spawn")
    res = torch.load(path)
    assert "error" not in res, res.get("error")
    ref_o, ref_l = _oracle(_wl())
    np.testing.assert_array_equal(res["out"].numpy(), ref_o.numpy())
    np.testing.assert_array_equal(res["lse"].numpy(), ref_l.numpy())
    assert all(len(p) > 0 for p in res["parts"])


def test_dead_rank_is_detected_not_hung(tmp_path):
    port = _free_port()
    path = str(tmp_path / "res.pt")
    ctx = mp.start_processes(_worker, args=(2, port, path, 1), nprocs=2, join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=120)
    assert all(not p.is_alive() for p in ctx.processes), "a rank hung"
    assert ctx.processes[1].exitcode == 3
    res = torch.load(path)
    assert "error" in res  # rank 0's collective failed instead of waiting forever


# dtypes torch's NCCL backend moves (int16 is not among them)
NCCL_DTYPES = {torch.uint8, torch.int8, torch.int32, torch.int64, torch.float16, torch.bfloat16, torch.float32,
               torch.float64, torch.bool}


class _NcclDtypeCheck:
    """torch.distributed as bench.py uses it, refusing what an NCCL process group refuses."""

    ReduceOp = dist.ReduceOp

    @staticmethod
    def all_reduce(t, op=dist.ReduceOp.SUM):
        assert t.dtype in NCCL_DTYPES, t.dtype
        return dist.all_reduce(t, op=op)

    @staticmethod
    def all_gather(lst, t):
        assert t.dtype in NCCL_DTYPES and all(x.dtype in NCCL_DTYPES for x in lst), t.dtype
        return dist.all_gather(lst, t)


def _verify_worker(rank, world, port, result_path):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        # each rank has its own requests (different seeds and lengths), as under bench.py --gpus N
        wl = W.make_workload(name=f"verify{rank}", q_lens=[1, 2, 1][: 2 + rank], kv_lens=[700, 1500, 900][: 2 + rank],
                             num_heads=16, topk=128, seed=5 + rank)
        out, lse = _oracle(wl)
        res = bench.verify_gather(wl, out.to(torch.bfloat16), lse.float(), torch.device("cpu"), rank, world,
                                  _NcclDtypeCheck, 3)
        if rank == 0:
            torch.save(res, result_path)
    finally:
        dist.destroy_process_group()


def test_bench_verify_gather_uses_nccl_dtypes(tmp_path):
    """bench.py's multi-GPU verification gathers every rank's out / lse and sampled token inputs and
    checks them against the oracle on rank 0.  Run over gloo with a wrapper that refuses the dtypes
    NCCL refuses, on shards of different sizes: it must pass and report its check."""
    port = _free_port()
    path = str(tmp_path / "verify.pt")
    mp.start_processes(_verify_worker, args=(2, port, path), nprocs=2, join=True, start_method="spawn")
    res = torch.load(path)
    assert res["parity_checked"] and res["pass"] and res["ranks"] == 2, res
