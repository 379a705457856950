"""Failure path of the tensor-core kernel, exercised without a GPU fault.

Every wait in the tcgen05 kernel is bounded (4 s by %globaltimer).  When one
runs out, the waiting role raises SAS_STATUS_WAIT_TIMEOUT, sets the abort flag
of both CTAs of its cluster, every other role leaves its loop at its next
wait, and the teardown lets in-flight copies land, joins the cluster and frees
tensor memory.  The test makes one wait run out on purpose: with
SAS_FWD_FLAG_TEST_STALL the output CTAs never release their first P slot, so
the score CTAs' wait for that slot expires.  The call must then complete in
bounded time with the timeout bit set, and the next call on the same context
must produce the same results as before.  Collected near the end: a failure
here leaves the other GPU tests already run.
"""

import ctypes
import time

import pytest
import torch

from dsv4_planb_b200 import _lib
from dsv4_planb_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _call(lib, wl, flags):
    a = _lib.SasFwdArgs()
    B = len(wl.q_lens)
    a.batch, a.num_tokens, a.max_q_len = B, wl.num_tokens, max(wl.q_lens)
    a.num_heads, a.num_kv_heads, a.head_dim, a.v_head_dim = wl.q.shape[1], 1, wl.q.shape[2], wl.v_head_dim
    a.ori_block_num, a.ori_block_size, a.ori_table_len = wl.ori_kv.shape[0], wl.ori_kv.shape[1], wl.ori_block_table.shape[1]
    a.cmp_block_num, a.cmp_block_size, a.cmp_table_len = wl.cmp_kv.shape[0], wl.cmp_kv.shape[1], wl.cmp_block_table.shape[1]
    a.topk, a.cmp_ratio, a.scenario = wl.topk, wl.cmp_ratio, 3
    a.ori_win_left, a.ori_win_right, a.ori_mask_mode, a.cmp_mask_mode = 127, 0, 4, 3
    a.dtype, a.softmax_scale, a.kernel = _lib.SAS_DTYPE_BF16, wl.softmax_scale, 2  # the tensor-core kernel
    a.flags = _lib.SAS_FWD_FLAG_CU_SEQLENS | flags
    dev = wl.q.device
    n = ctypes.c_size_t(0)
    assert lib.sas_workspace_size(ctypes.byref(a), ctypes.byref(n)) == 0
    ws = torch.empty(n.value, dtype=torch.uint8, device=dev)
    out = torch.zeros((wl.num_tokens, wl.q.shape[1], wl.v_head_dim), dtype=wl.q.dtype, device=dev)
    lse = torch.zeros((wl.num_tokens, wl.q.shape[1]), dtype=torch.float32, device=dev)
    cu = wl.cu_seqlens_q.to(torch.int32).contiguous()
    ptrs = [t.data_ptr() for t in (wl.q, wl.ori_kv, wl.ori_block_table, wl.cmp_kv, wl.cmp_block_table,
                                   wl.cmp_sparse_indices, cu)]
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = lib.sas_forward(ctypes.byref(a), *ptrs, None, wl.seqused_kv.data_ptr(), wl.sinks.data_ptr(), None,
                         out.data_ptr(), lse.data_ptr(), ws.data_ptr(), n.value, stream)
    assert rc == 0, _lib.strerror(rc)
    st = ctypes.c_uint32(0)
    assert lib.sas_read_status(ws.data_ptr(), ctypes.byref(st), stream) == 0
    torch.cuda.synchronize()
    return out, lse, st.value


def test_wait_timeout_is_reported_and_the_context_survives(cuda_device):
    lib = _lib.load()
    wl = W.make_workload(name="stall", q_lens=[1, 1, 1], kv_lens=[3000, 700, 9000], num_heads=128, topk=256,
                         device=cuda_device, index_method="keys")
    ref_out, ref_lse, st0 = _call(lib, wl, 0)
    assert st0 == 0
    t0 = time.monotonic()
    _, _, st = _call(lib, wl, _lib.SAS_FWD_FLAG_TEST_STALL)
    elapsed = time.monotonic() - t0
    assert st & _lib.SAS_STATUS_WAIT_TIMEOUT, _lib.status_names(st)
    assert elapsed < 60.0
    out, lse, st2 = _call(lib, wl, 0)  # same context, same workspace sizes: must work as before
    assert st2 == 0
    assert torch.equal(out, ref_out) and torch.equal(lse, ref_lse)
