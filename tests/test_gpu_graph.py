"""The decode call is capturable in a CUDA graph and replays on new data.

A serving loop captures one ``sparse_attn_sharedkv`` call per batch shape and
replays it every decode step after writing the step's tokens, indices, lengths
and block tables into the captured buffers.  That needs a host path with no
synchronisation (``max_seqlen_q`` given, outputs passed in) and kernels that
read everything per-step from device memory.  The test captures once, replays
for two different workloads of the same shapes, and requires each replay to
equal an eager call on the same data exactly (the kernels are deterministic).
"""

import pytest
import torch

from dsv4_planb_b200 import workloads as W
from dsv4_planb_b200.api import sparse_attn_sharedkv

pytestmark = pytest.mark.gpu


def _wl(seed, dev, scenario=3):
    return W.make_workload(name=f"g{seed}", q_lens=[1, 2, 1, 1], kv_lens=[3000, 9000, 700, 20000], num_heads=128,
                           topk=512, seed=seed, device=dev, index_method="keys", scenario=scenario)


def _eager(wl, kernel):
    out, lse = sparse_attn_sharedkv(wl.q, return_softmax_lse=True, max_seqlen_q=max(wl.q_lens), kernel=kernel,
                                    **wl.api_kwargs())
    torch.cuda.synchronize()
    return out, lse


@pytest.mark.parametrize("kernel,scenario", [("tc", 3), ("simt", 3), ("tc", 2), ("simt", 2), ("tc2", 3), ("tc2", 2)])
def test_graph_capture_replays_new_inputs(cuda_device, kernel, scenario):
    """Scenario 3 (SCFA) and scenario 2 (CFA, whose dense compressed range the kernels take from
    the block table on the device: no host read of seqused_kv)."""
    first, second = _wl(11, cuda_device, scenario), _wl(12, cuda_device, scenario)
    kw = first.api_kwargs()
    static = {k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in kw.items()}
    q = first.q.clone()
    T, N1, _ = q.shape
    out = torch.empty((T, N1, first.v_head_dim), dtype=q.dtype, device=cuda_device)
    lse = torch.empty((T, N1), dtype=torch.float32, device=cuda_device)

    def call():
        sparse_attn_sharedkv(q, out=out, lse_out=lse, return_softmax_lse=True, max_seqlen_q=2, kernel=kernel,
                             **static)

    side = torch.cuda.Stream(device=cuda_device)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        call()  # warm-up outside the capture (kernel attributes, allocator pools)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        call()
    torch.cuda.synchronize()

    for wl in (first, second, first):
        q.copy_(wl.q)
        for k, v in wl.api_kwargs().items():
            if isinstance(v, torch.Tensor):
                assert static[k].shape == v.shape, k
                static[k].copy_(v)
        out.fill_(float("nan"))
        lse.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        ref_out, ref_lse = _eager(wl, kernel)
        assert torch.equal(out, ref_out)
        assert torch.equal(lse, ref_lse)
    graph.reset()


def test_registered_op_under_torch_compile_and_in_a_graph(cuda_device):
    """The launch is the registered op torch.ops.sas_b200.sparse_attn_sharedkv: torch.compile with
    fullgraph=True traces the public function in one graph (the op is opaque, its fake
    implementation gives the output shapes), the compiled function gives the eager bits, and the
    op-owned-output form captures in a CUDA graph and replays on new data."""
    wl, wl2 = _wl(21, cuda_device), _wl(22, cuda_device)
    kw = wl.api_kwargs()

    def fn(q, ori_kv, cmp_kv, idx, ori_bt, cmp_bt, cu, kv, sinks):
        return sparse_attn_sharedkv(q, ori_kv=ori_kv, cmp_kv=cmp_kv, cmp_sparse_indices=idx, ori_block_table=ori_bt,
                                    cmp_block_table=cmp_bt, cu_seqlens_q=cu, seqused_kv=kv, sinks=sinks,
                                    softmax_scale=wl.softmax_scale, cmp_ratio=wl.cmp_ratio, v_head_dim=wl.v_head_dim,
                                    return_softmax_lse=True, max_seqlen_q=2)

    args = (wl.q, kw["ori_kv"], kw["cmp_kv"], kw["cmp_sparse_indices"], kw["ori_block_table"], kw["cmp_block_table"],
            kw["cu_seqlens_q"], kw["seqused_kv"], kw["sinks"])
    ref_out, ref_lse = fn(*args)
    compiled = torch.compile(fn, fullgraph=True)
    out, lse = compiled(*args)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out) and torch.equal(lse, ref_lse)

    static = [a.clone() for a in args]
    side = torch.cuda.Stream(device=cuda_device)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn(*static)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        g_out, g_lse = fn(*static)
    kw2 = wl2.api_kwargs()
    new = (wl2.q, kw2["ori_kv"], kw2["cmp_kv"], kw2["cmp_sparse_indices"], kw2["ori_block_table"],
           kw2["cmp_block_table"], kw2["cu_seqlens_q"], kw2["seqused_kv"], kw2["sinks"])
    for dst, src in zip(static, new):
        assert dst.shape == src.shape
        dst.copy_(src)
    graph.replay()
    torch.cuda.synchronize()
    e_out, e_lse = fn(*new)
    torch.cuda.synchronize()
    assert torch.equal(g_out, e_out) and torch.equal(g_lse, e_lse)
    graph.reset()
