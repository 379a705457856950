"""Backward pass (``sas_backward`` through the registered op's autograd) against torch autograd.

The reference has no backward; the check is a plain fp32 PyTorch restatement of the same op (each
token's key rows resolved with the oracle's rules, golden.py:28-66 and 125-150, unmapped blocks read
as zero rows as in unpack_paged_kv, golden.py:247-268; softmax over the keys and the sink logit;
out = P V with V the first D_v columns of each K = V row; lse = logsumexp), differentiated by torch
autograd on the same bf16 / fp16 input values.  The kernel differentiates the exact softmax but
reads D = dO . out from the forward's rounded out, key-row gradients are sums of fp32 atomics, and
the gradients come back in the inputs' dtype (bf16 keeps 8 bits: a relative rounding of 2^-9).
The bar is max |g - g_ref| <= 5e-3 * max |g_ref| per gradient; measured on B200: 2.0-2.9e-3 with
bf16 inputs, 3.5e-4 with fp16.
"""

import numpy as np
import pytest
import torch

from dsv4_planb_b200 import workloads as W
from dsv4_planb_b200.api import sparse_attn_sharedkv
from oracle import golden_np as O

pytestmark = pytest.mark.gpu

RTOL = 5e-3


def _phys(table_row, pos, block_size, block_num):
    pos = np.asarray(pos, dtype=np.int64)
    blk = pos // block_size
    phys = np.full(pos.shape, -1, dtype=np.int64)
    inside = blk < table_row.shape[0]
    phys[inside] = table_row[blk[inside]]
    ok = (phys >= 0) & (phys < block_num)
    return np.where(ok, phys * block_size + pos % block_size, -1)


def _token_rows(wl):
    """Per flat token row: (window rows, compressed rows) as physical pool rows, -1 = zero row."""
    scen = 3 if wl.cmp_sparse_indices is not None else (2 if wl.cmp_kv is not None else 1)
    cu = wl.cu_seqlens_q.cpu().numpy().astype(np.int64)
    kv = wl.seqused_kv.cpu().numpy().astype(np.int64)
    ori_bt = wl.ori_block_table.cpu().numpy().astype(np.int64)
    cmp_bt = wl.cmp_block_table.cpu().numpy().astype(np.int64) if scen >= 2 else None
    idx = wl.cmp_sparse_indices.cpu().numpy() if scen == 3 else None
    res = []
    for b in range(len(cu) - 1):
        for s in range(int(cu[b + 1] - cu[b])):
            t = int(cu[b]) + s
            win, cpos, _ = O.resolve_token_rows(scenario=scen, b=b, s=s, act_q=int(cu[b + 1] - cu[b]),
                                                act_kv=int(kv[b]), cmp_idx_row=None if idx is None else idx[t, 0],
                                                topk=wl.topk, cmp_ratio=wl.cmp_ratio, ori_win_left=wl.ori_win_left)
            wr = _phys(ori_bt[b], win, wl.ori_kv.shape[1], wl.ori_kv.shape[0])
            cr = (_phys(cmp_bt[b], cpos, wl.cmp_kv.shape[1], wl.cmp_kv.shape[0]) if scen >= 2
                  else np.zeros(0, dtype=np.int64))
            res.append((wr, cr))
    return res


def _reference(wl, q, ori, cmp, sinks, rows):
    """fp32 torch restatement: (out [T, N1, Dv], lse [T, N1]); q, ori, cmp, sinks are fp32 leaves."""
    D, Dv = q.shape[-1], wl.v_head_dim
    ori2 = torch.cat([ori.reshape(-1, D), ori.new_zeros(1, D)])  # the extra row stands for -1
    cmp2 = torch.cat([cmp.reshape(-1, D), cmp.new_zeros(1, D)]) if cmp is not None else None
    outs, lses = [], []
    for t, (wr, cr) in enumerate(rows):
        wi = torch.as_tensor(np.where(wr >= 0, wr, ori2.shape[0] - 1), device=q.device)
        keys = [ori2.index_select(0, wi)]
        if cr.size:
            ci = torch.as_tensor(np.where(cr >= 0, cr, cmp2.shape[0] - 1), device=q.device)
            keys.append(cmp2.index_select(0, ci))
        k = torch.cat(keys)
        s = wl.softmax_scale * q[t] @ k.T
        lse = torch.logsumexp(torch.cat([s, sinks[:, None]], dim=1), dim=1)
        outs.append(torch.exp(s - lse[:, None]) @ k[:, :Dv])
        lses.append(lse)
    return torch.stack(outs), torch.stack(lses)


def _check(name, got, ref):
    got, ref = got.float(), ref.float()
    err = float((got - ref).abs().max())
    mag = float(ref.abs().max())
    assert torch.isfinite(got).all(), name
    assert err <= RTOL * mag + 1e-6, f"{name}: max |err| {err:.3e} against max |ref| {mag:.3e}"
    return err / max(mag, 1e-30)


def _run(wl, with_lse_grad=True, kernel="auto"):
    dev = wl.q.device
    kw = wl.api_kwargs()
    q = wl.q.detach().clone().requires_grad_(True)
    ori = kw.pop("ori_kv").detach().clone().requires_grad_(True)
    cmp = kw.pop("cmp_kv")
    cmp = cmp.detach().clone().requires_grad_(True) if cmp is not None else None
    sinks = kw.pop("sinks").detach().clone().float().requires_grad_(True)
    out, lse = sparse_attn_sharedkv(q, ori_kv=ori, cmp_kv=cmp, sinks=sinks, return_softmax_lse=True,
                                    check_status=True, kernel=kernel, max_seqlen_q=max(wl.q_lens), **kw)
    gen = torch.Generator(device=dev).manual_seed(5)
    g_out = torch.randn(out.shape, generator=gen, device=dev).to(out.dtype)
    g_lse = torch.randn(lse.shape, generator=gen, device=dev) if with_lse_grad else None
    if with_lse_grad:
        torch.autograd.backward([out, lse], [g_out, g_lse])
    else:
        torch.autograd.backward([out], [g_out])

    rows = _token_rows(wl)
    q32 = wl.q.detach().float().requires_grad_(True)
    ori32 = wl.ori_kv.detach().float().requires_grad_(True)
    cmp32 = wl.cmp_kv.detach().float().requires_grad_(True) if wl.cmp_kv is not None else None
    sinks32 = wl.sinks.detach().float().requires_grad_(True)
    r_out, r_lse = _reference(wl, q32, ori32, cmp32, sinks32, rows)
    loss = (r_out * g_out.float()).sum() + ((r_lse * g_lse).sum() if with_lse_grad else 0.0)
    loss.backward()
    rel = {"dq": _check("dq", q.grad, q32.grad), "d_ori_kv": _check("d_ori_kv", ori.grad, ori32.grad),
           "d_sinks": _check("d_sinks", sinks.grad, sinks32.grad)}
    if cmp is not None:
        rel["d_cmp_kv"] = _check("d_cmp_kv", cmp.grad, cmp32.grad)
    print("\n[backward] " + ", ".join(f"{k} rel err {v:.2e}" for k, v in rel.items()))


@pytest.mark.parametrize("scenario", [3, 2, 1])
def test_backward_matches_torch_autograd(cuda_device, scenario):
    """SCFA, CFA and SWA: gradients of q, both pools and the sinks, with gradients on out and lse."""
    wl = W.make_workload(name=f"bwd{scenario}", q_lens=[1, 3, 2], kv_lens=[700, 1500, 2900], num_heads=16, topk=128,
                         seed=31 + scenario, device=cuda_device, scenario=scenario)
    _run(wl)


def test_backward_128_heads_fp16_and_out_only(cuda_device):
    """Every head group of a 128-head token, fp16 inputs, and a loss on out alone (lse unused)."""
    wl = W.make_workload(name="bwd128", q_lens=[2, 1], kv_lens=[1300, 2200], num_heads=128, topk=256, seed=41,
                         dtype=torch.float16, device=cuda_device)
    _run(wl, with_lse_grad=False)


def test_backward_unmapped_blocks_and_tensor_core_forward(cuda_device):
    """-1 table entries inside the used range are zero rows with no gradient destination; the
    forward runs on the tensor-core kernel (the backward reads its out and lse)."""
    wl = W.make_workload(name="bwdholes", q_lens=[2, 1], kv_lens=[1000, 3000], num_heads=128, topk=128, seed=43,
                         device=cuda_device)
    wl.ori_block_table[0, 7] = -1
    wl.cmp_block_table[1, 0] = -1
    _run(wl, kernel="tc")


def test_backward_bsnd_matches_tnd(cuda_device):
    """The BSND layout (q [B, S, N1, D], indices [B, S, 1, K]) gives the TND call's gradients."""
    wl = W.make_workload(name="bwdbsnd", q_lens=[2, 2], kv_lens=[900, 2100], num_heads=32, topk=128, seed=47,
                         device=cuda_device)
    kw = wl.api_kwargs()
    grads = []
    for layout in ("TND", "BSND"):
        q = wl.q.detach().clone()
        idx = kw["cmp_sparse_indices"]
        if layout == "BSND":
            q = q.reshape(2, 2, *q.shape[1:])
            idx = idx.reshape(2, 2, *idx.shape[1:])
        q.requires_grad_(True)
        ori = wl.ori_kv.detach().clone().requires_grad_(True)
        cmp = wl.cmp_kv.detach().clone().requires_grad_(True)
        sinks = wl.sinks.detach().clone().requires_grad_(True)
        args = dict(kw, ori_kv=ori, cmp_kv=cmp, sinks=sinks, cmp_sparse_indices=idx, layout_q=layout)
        out = sparse_attn_sharedkv(q, check_status=True, **args)
        g = torch.ones_like(out)
        out.backward(g)
        grads.append((q.grad.reshape(wl.q.shape).float(), ori.grad.float(), cmp.grad.float(), sinks.grad.float()))
    for name, a, b in zip(("dq", "d_ori_kv", "d_cmp_kv", "d_sinks"), *grads):
        assert float((a - b).abs().max()) <= 1e-3 * float(b.abs().max()) + 1e-6, name
