"""The tensor-core path's split-KV plan in the reference's FD-row metadata format.

The reference scheduler declares flash-decoding (FD) rows but never enables them
(supportFd = False, metadata.py:323-325; row packing metadata.py:995-1008).
``sas_split_metadata`` emits the plan the B200 attention kernel actually runs:
one FD row per token cut into np > 1 pieces, {1, b, s, t * pieces, np, 0, N1, 0},
FA rows zero, and the count of split tokens at int 864.  The expected rows are
recomputed here from the key-resolution records (``resolve_rows``) and the plan
shape (``sas_split_plan``) with the kernel's own cut rule: a token of n tiles of
64 keys is cut when n > tiles_per_piece, into min(ceil(n / tiles_per_piece),
pieces) pieces.
"""

import numpy as np
import pytest
import torch

from dsv4_planb_b200 import api
from dsv4_planb_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _expected(wl, P, M):
    tinfo, _, st = api.resolve_rows(
        cmp_sparse_indices=wl.cmp_sparse_indices, ori_block_table=wl.ori_block_table,
        cmp_block_table=wl.cmp_block_table, cu_seqlens_q=wl.cu_seqlens_q, seqused_kv=wl.seqused_kv,
        num_heads=wl.q.shape[1], head_dim=wl.q.shape[2], ori_block_num=wl.ori_kv.shape[0],
        ori_block_size=wl.ori_kv.shape[1], cmp_block_num=wl.cmp_kv.shape[0], cmp_block_size=wl.cmp_kv.shape[1],
        cmp_ratio=wl.cmp_ratio)
    assert st == 0
    ti = tinfo.cpu().numpy()
    out = np.zeros(1024, dtype=np.int32)
    n = 0
    for t in range(ti.shape[0]):
        ntiles = (-(-ti[t, 3] // 64) + -(-ti[t, 4] // 64)) if ti[t, 5] else 0
        np_ = min(-(-ntiles // M), P) if P > 1 and ntiles > M else 1
        if np_ > 1:
            if n < 72:
                out[288 + 8 * n: 296 + 8 * n] = [1, ti[t, 0], ti[t, 6], t * P, np_, 0, wl.q.shape[1], 0]
            n += 1
    out[864] = n
    return out


@pytest.mark.parametrize("case", ["b4", "b16", "b64", "shard_split"])
def test_split_metadata_matches_the_kernel_plan(cuda_device, case):
    if case == "shard_split":
        wl = W.make_workload(name="sm", q_lens=[1] * 48, kv_lens=[700 + 1500 * i for i in range(48)],
                             num_heads=128, topk=2048, seed=3, device=cuda_device)
        split = 8
    else:
        wl = W.config_workload("c2", device=cuda_device, batch=int(case[1:]))
        split = 0
    md, args = api.split_metadata(
        cmp_sparse_indices=wl.cmp_sparse_indices, ori_block_table=wl.ori_block_table,
        cmp_block_table=wl.cmp_block_table, cu_seqlens_q=wl.cu_seqlens_q, seqused_kv=wl.seqused_kv,
        num_heads=wl.q.shape[1], head_dim=wl.q.shape[2], v_head_dim=wl.v_head_dim,
        ori_block_num=wl.ori_kv.shape[0], ori_block_size=wl.ori_kv.shape[1], cmp_block_num=wl.cmp_kv.shape[0],
        cmp_block_size=wl.cmp_kv.shape[1], cmp_ratio=wl.cmp_ratio, split_tiles=split)
    P, M = api.split_plan(args)
    got = md.cpu().numpy()
    exp = _expected(wl, P, M)
    np.testing.assert_array_equal(got, exp)
    assert not got[:288].any(), "FA rows stay zero: clusters take units from a dynamic queue"
    if case == "b64":
        assert (P, M) == (1, 0) and got[864] == 0
    else:
        assert P > 1 and got[864] > 0
    # the plan is the one the attention call runs: it launches the combine kernel iff a token is split
    out, lse = api.sparse_attn_sharedkv(wl.q, return_softmax_lse=True, check_status=True, split_tiles=split,
                                        **wl.api_kwargs())
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
