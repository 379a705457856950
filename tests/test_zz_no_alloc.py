"""sas_forward_noalloc: the entry point for hosts that cannot allocate device memory.

Some hosts of this operator own all device memory -- a serving engine that
reserves almost all of HBM for its paged KV pool up front, or a thin FFI host
with no device allocator -- and cannot hand sas_forward a workspace.  For them
sas_forward_noalloc runs the same kernels over a scratch array compiled into
the library.  This test calls both entry points through the C ABI on the same
inputs, twice in a row with different workloads (the scratch keeps the
previous call's contents), and requires identical bits: both entry points run
the same deterministic kernels on the same inputs, only the workspace differs.
It also reads the scratch's status word back (clean after a valid call, the
bad-index bit after a call with an index below -1).  It is collected last on
purpose: a failure here leaves every other test already run.
"""

import ctypes

import numpy as np
import pytest
import torch

from dsv4_planb_b200 import _lib
from dsv4_planb_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _args(wl):
    a = _lib.SasFwdArgs()
    B = len(wl.q_lens)
    a.batch, a.num_tokens, a.max_q_len = B, wl.num_tokens, max(wl.q_lens)
    a.num_heads, a.num_kv_heads, a.head_dim, a.v_head_dim = wl.q.shape[1], 1, wl.q.shape[2], wl.v_head_dim
    a.ori_block_num, a.ori_block_size, a.ori_table_len = wl.ori_kv.shape[0], wl.ori_kv.shape[1], wl.ori_block_table.shape[1]
    a.cmp_block_num, a.cmp_block_size, a.cmp_table_len = wl.cmp_kv.shape[0], wl.cmp_kv.shape[1], wl.cmp_block_table.shape[1]
    a.topk, a.cmp_ratio, a.scenario = wl.topk, wl.cmp_ratio, 3
    a.ori_win_left, a.ori_win_right, a.ori_mask_mode, a.cmp_mask_mode = 127, 0, 4, 3
    a.dtype, a.softmax_scale, a.kernel = _lib.SAS_DTYPE_BF16, wl.softmax_scale, 0
    return a


def _call(lib, wl, noalloc):
    dev = wl.q.device
    a = _args(wl)
    cu = wl.cu_seqlens_q.to(torch.int32)
    q_prefix = cu[:-1].contiguous()
    act_q = (cu[1:] - cu[:-1]).contiguous()
    out = torch.full((wl.num_tokens, wl.q.shape[1], wl.v_head_dim), float("nan"), dtype=wl.q.dtype, device=dev)
    lse = torch.full((wl.num_tokens, wl.q.shape[1]), float("nan"), dtype=torch.float32, device=dev)
    ins = [wl.q, wl.ori_kv, wl.ori_block_table, wl.cmp_kv, wl.cmp_block_table, wl.cmp_sparse_indices, q_prefix,
           act_q, wl.seqused_kv, wl.sinks]
    ptrs = [t.data_ptr() for t in ins]
    stream = torch.cuda.current_stream(dev).cuda_stream
    if noalloc:
        rc = lib.sas_forward_noalloc(ctypes.byref(a), *ptrs, None, out.data_ptr(), lse.data_ptr(), stream)
    else:
        n = ctypes.c_size_t(0)
        assert lib.sas_workspace_size(ctypes.byref(a), ctypes.byref(n)) == 0
        ws = torch.empty(n.value, dtype=torch.uint8, device=dev)
        rc = lib.sas_forward(ctypes.byref(a), *ptrs, None, out.data_ptr(), lse.data_ptr(), ws.data_ptr(), n.value,
                             stream)
    assert rc == 0, _lib.strerror(rc)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), lse.cpu().numpy()


def test_noalloc_matches_workspace_entry_point(cuda_device):
    lib = _lib.load()
    first = W.make_workload(name="na1", q_lens=[1, 2, 1], kv_lens=[3000, 900, 20000], num_heads=128, topk=2048,
                            device=cuda_device, index_method="keys")
    second = W.make_workload(name="na2", q_lens=[1, 1], kv_lens=[700, 5000], num_heads=128, topk=512, seed=7,
                             device=cuda_device, index_method="keys")
    for wl in (first, second):  # two calls in a row on the shared scratch
        ref_out, ref_lse = _call(lib, wl, noalloc=False)
        out, lse = _call(lib, wl, noalloc=True)
        assert np.isfinite(out).all() and np.isfinite(lse).all()
        np.testing.assert_array_equal(out, ref_out)
        np.testing.assert_array_equal(lse, ref_lse)
        st = ctypes.c_uint32(0xFFFFFFFF)
        assert lib.sas_noalloc_read_status(ctypes.byref(st), torch.cuda.current_stream().cuda_stream) == 0
        assert st.value == 0


def test_noalloc_status_word_reports_bad_indices(cuda_device):
    lib = _lib.load()
    wl = W.make_workload(name="na4", q_lens=[1, 1], kv_lens=[900, 900], num_heads=128, topk=64, device=cuda_device,
                         index_method="keys")
    wl.cmp_sparse_indices[0, 0, 3] = -5  # below -1: skipped, and the status word says so
    _call(lib, wl, noalloc=True)
    st = ctypes.c_uint32(0)
    assert lib.sas_noalloc_read_status(ctypes.byref(st), torch.cuda.current_stream().cuda_stream) == 0
    assert st.value & _lib.SAS_STATUS_BAD_INDEX


def test_noalloc_rejects_oversized_calls(cuda_device):
    lib = _lib.load()
    wl = W.make_workload(name="na3", q_lens=[1], kv_lens=[600], num_heads=16, topk=64, device=cuda_device,
                         index_method="keys")
    a = _args(wl)
    a.num_tokens = (_lib.SAS_NOALLOC_SCRATCH_BYTES // (4 * 64)) + 1024  # more rows than the scratch holds
    n = ctypes.c_size_t(0)
    assert lib.sas_workspace_size(ctypes.byref(a), ctypes.byref(n)) == 0 and n.value > _lib.SAS_NOALLOC_SCRATCH_BYTES
    null = None
    rc = lib.sas_forward_noalloc(ctypes.byref(a), 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, null, 1, 1, null)
    assert rc == _lib.SAS_ERR_WORKSPACE
