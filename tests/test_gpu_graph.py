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


def _wl(seed, dev):
    return W.make_workload(name=f"g{seed}", q_lens=[1, 2, 1, 1], kv_lens=[3000, 9000, 700, 20000], num_heads=128,
                           topk=512, seed=seed, device=dev, index_method="keys")


def _eager(wl, kernel):
    out, lse = sparse_attn_sharedkv(wl.q, return_softmax_lse=True, max_seqlen_q=max(wl.q_lens), kernel=kernel,
                                    **wl.api_kwargs())
    torch.cuda.synchronize()
    return out, lse


@pytest.mark.parametrize("kernel", ["tc", "simt"])
def test_graph_capture_replays_new_inputs(cuda_device, kernel):
    first, second = _wl(11, cuda_device), _wl(12, cuda_device)
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
