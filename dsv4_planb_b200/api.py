"""Drop-in ``sparse_attn_sharedkv`` for B200, over the sas_b200 C ABI.

Mirrors the reference entry point ``sparse_attn_sharedkv_tilelang/api.py:129-397``
of yangqiang2018/dsv4_planB: the same keyword arguments with the same meaning,
the same scenario dispatch (``cmp_kv`` / ``cmp_sparse_indices`` present or not,
api.py:196-202), the same TND / BSND handling (api.py:204-240), the same
assertions (api.py:186-191, 247-249, 362-364) and the same return value
(``out``, or ``(out, lse)`` when ``return_softmax_lse``, api.py:388-397).

The launch itself is a registered torch operator, ``torch.ops.sas_b200.sparse_attn_sharedkv``
(outputs allocated by the op) and ``torch.ops.sas_b200.sparse_attn_sharedkv_out`` (writes
caller-owned ``out`` / ``lse``), each with a fake (meta) implementation: the dispatcher, fake
tensors, ``torch.compile(fullgraph=True)`` and CUDA-graph capture see one opaque op, where the
reference calls its JIT kernel directly (api.py:372-384).

Differences, all widenings of the reference contract:

* any head count N1 and any ``D_qk % 8 == 0`` (the reference pins N1 = 64,
  D = 512, api.py:279-282); ``v_head_dim`` (default ``D_qk``) selects the
  DeepSeek-V4 split of a 576-wide K = V row into D_v = 512 value columns;
* ``metadata`` is accepted and checked for size but not needed: the B200
  kernels plan their own work split over 148 SMs (no scheduler call and no
  host sync when it is omitted); ``core_num`` is accepted and ignored;
* no host synchronisation: scenario 2 (CFA) takes each token's compressed range
  from the block table on the device (the reference reads ``seqused_kv.max()``
  on the host, api.py:260), and TND needs none once ``max_seqlen_q`` is given;
* extra keywords ``kernel`` ("auto" | "simt" | "tc" | "tc2"), ``max_seqlen_q`` (skips
  the host read of ``cu_seqlens_q``), ``out`` / ``lse_out`` (preallocated
  outputs), ``check_status`` (read the device status word, synchronising),
  ``split_tiles`` and ``lazy_rescale``.
"""

from __future__ import annotations

from typing import List, Optional, Tuple, Union

import torch

from . import _lib

SAS_META_SIZE = 1024
DEFAULT_CORE_NUM = 24

def _dtype_code(t: torch.dtype) -> int:
    if t == torch.bfloat16:
        return _lib.SAS_DTYPE_BF16
    if t == torch.float16:
        return _lib.SAS_DTYPE_FP16
    raise ValueError(f"unsupported torch dtype {t}")


def _i32(t: torch.Tensor, device) -> torch.Tensor:
    return t.to(device=device, dtype=torch.int32).contiguous()


def _dense16(t: torch.Tensor) -> torch.Tensor:
    """Contiguous, with a 16-byte aligned base: the kernels move rows in 16-byte vectors and the
    tensor-core kernel reads q and the pools through TMA tensor maps.  A view that starts inside a
    vector (an odd element offset) is copied; the C ABI rejects such a pointer.  For per-call
    tensors (q); the KV pools go through _pool16."""
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _pool16(t: torch.Tensor, name: str) -> torch.Tensor:
    """A paged KV pool must already be dense with a 16-byte aligned base: copying a pool (which can
    be gigabytes) on every call to re-home it would hide a large cost behind a slow step."""
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous (a paged KV pool is not copied per call)")
    if t.data_ptr() % 16:
        raise ValueError(f"{name} must start on a 16-byte boundary (a paged KV pool is not copied per call)")
    return t


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _workspace(nbytes: int, device) -> torch.Tensor:
    # The caching allocator makes this cheap and keeps it stream-ordered.
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def _scenario(cmp_kv, cmp_sparse_indices) -> int:
    if cmp_kv is None:
        return 1
    return 2 if cmp_sparse_indices is None else 3


def _out_shapes(q: torch.Tensor, layout_q: str, v_head_dim: int):
    if layout_q == "TND":
        T, N1, _ = q.shape
        return (T, N1, v_head_dim), (T, N1)
    B, S, N1, _ = q.shape
    return (B, S, N1, v_head_dim), (B, S, N1)


class _Call:
    """The device arguments of one call, as sas_forward and sas_backward take them."""

    __slots__ = ("args", "lib", "ws", "q", "ori_kv", "ori_bt", "cmp_kv", "cmp_bt", "idx", "q_prefix", "act_q",
                 "seq_kv", "sinks", "metadata", "T", "N1", "Dv", "stream")


def _marshal(q, ori_kv, cmp_kv, cmp_sparse_indices, ori_block_table, cmp_block_table, cu_seqlens_q, seqused_kv,
             sinks, metadata, softmax_scale, cmp_ratio, ori_win_left, layout_q, v_head_dim, kernel, max_seqlen_q,
             split_tiles, lazy_rescale) -> _Call:
    """Flatten the layouts, check the shapes and fill SasFwdArgs; ``max_seqlen_q`` < 0 reads it from
    ``cu_seqlens_q`` (host sync).  Allocates the call's workspace."""
    dev = q.device
    scenario = _scenario(cmp_kv, cmp_sparse_indices)
    if layout_q == "TND":
        T, N1, D = q.shape
        q_flat = q
        cu = _i32(cu_seqlens_q, dev)
        B = cu.numel() - 1
        q_prefix = cu  # with SAS_FWD_FLAG_CU_SEQLENS the kernels derive act_q = cu[b+1] - cu[b]
        act_q = None
        if max_seqlen_q < 0:
            cu_h = cu_seqlens_q.detach().to("cpu", torch.int64)
            max_seqlen_q = int((cu_h[1:] - cu_h[:-1]).max().item()) if B > 0 else 0
        idx_flat = _i32(cmp_sparse_indices, dev) if scenario == 3 else None
    else:
        B, S_max, N1, D = q.shape
        T = B * S_max
        q_flat = q.reshape(T, N1, D)
        q_prefix = torch.arange(B, dtype=torch.int32, device=dev) * S_max
        if cu_seqlens_q is not None:
            cu = _i32(cu_seqlens_q, dev)
            act_q = (cu[1:] - cu[:-1]).contiguous()
        else:
            act_q = torch.full((B,), S_max, dtype=torch.int32, device=dev)
        max_seqlen_q = S_max if max_seqlen_q < 0 else max_seqlen_q
        if scenario == 3:
            ci = cmp_sparse_indices
            idx_flat = _i32(ci.reshape(T, ci.shape[2], ci.shape[3]), dev)
        else:
            idx_flat = None
    seq_kv = _i32(seqused_kv, dev)
    if scenario == 3:
        N2 = idx_flat.shape[1]
        K = idx_flat.shape[2]
    else:
        N2 = (cmp_kv if scenario == 2 else ori_kv).shape[2]
        K = 0
    if N2 != 1:
        raise ValueError(f"only one KV head is supported (got N2={N2})")
    Dv = v_head_dim
    ori_kv_d = _pool16(ori_kv, "ori_kv")
    ori_bt = _i32(ori_block_table, dev)
    if ori_bt.dim() != 2 or ori_bt.shape[0] < B:
        raise ValueError(f"ori_block_table must be [B>={B}, table_len] (got {tuple(ori_bt.shape)})")
    if cmp_block_table is not None and (cmp_block_table.dim() != 2 or cmp_block_table.shape[0] < B):
        raise ValueError(f"cmp_block_table must be [B>={B}, table_len] (got {tuple(cmp_block_table.shape)})")
    if idx_flat is not None and (idx_flat.dim() != 3 or idx_flat.shape[0] != T):
        raise ValueError(f"cmp_sparse_indices must hold one row per query token (got {tuple(idx_flat.shape)})")
    if scenario >= 2:
        cmp_kv_d = _pool16(cmp_kv, "cmp_kv")
        cmp_bt = _i32(cmp_block_table, dev)
    else:
        cmp_kv_d = cmp_bt = None
    sinks_d = sinks.to(device=dev, dtype=torch.float32).contiguous()
    if metadata is not None:
        metadata = _i32(metadata.reshape(SAS_META_SIZE), dev)

    args = _lib.SasFwdArgs()
    args.batch = B
    args.num_tokens = T
    args.max_q_len = int(max_seqlen_q)
    args.num_heads = N1
    args.num_kv_heads = N2
    args.head_dim = D
    args.v_head_dim = Dv
    args.ori_block_num, args.ori_block_size = ori_kv_d.shape[0], ori_kv_d.shape[1]
    args.ori_table_len = ori_bt.shape[1]
    if scenario >= 2:
        args.cmp_block_num, args.cmp_block_size = cmp_kv_d.shape[0], cmp_kv_d.shape[1]
        args.cmp_table_len = cmp_bt.shape[1]
    args.topk = K
    args.cmp_ratio = int(cmp_ratio)
    args.scenario = scenario
    args.max_cmp_len = 0  # the kernels resolve CFA's dense range through the table
    args.ori_win_left = ori_win_left
    args.ori_win_right = 0
    args.ori_mask_mode = 4
    args.cmp_mask_mode = 3
    args.dtype = _dtype_code(q.dtype)
    args.softmax_scale = float(softmax_scale)
    args.kernel = _lib.KERNELS[kernel]
    args.flags = (_lib.SAS_FWD_FLAG_CU_SEQLENS if layout_q == "TND" else 0) | (
        _lib.SAS_FWD_FLAG_LAZY_RESCALE if lazy_rescale else 0)
    args.split_tiles = int(split_tiles)

    lib = _lib.load()
    nbytes = _lib.ctypes.c_size_t(0)
    _lib.check(lib.sas_workspace_size(_lib.ctypes.byref(args), _lib.ctypes.byref(nbytes)), "sas_workspace_size")
    c = _Call()
    c.args, c.lib, c.ws = args, lib, _workspace(nbytes.value, dev)
    c.q, c.ori_kv, c.ori_bt, c.cmp_kv, c.cmp_bt, c.idx = _dense16(q_flat), ori_kv_d, ori_bt, cmp_kv_d, cmp_bt, idx_flat
    c.q_prefix, c.act_q, c.seq_kv, c.sinks, c.metadata = q_prefix, act_q, seq_kv, sinks_d, metadata
    c.T, c.N1, c.Dv = T, N1, Dv
    c.stream = torch.cuda.current_stream(dev).cuda_stream
    return c


def _check_status(c: _Call, what: str) -> None:
    st = _lib.ctypes.c_uint32(0)
    _lib.check(c.lib.sas_read_status(_ptr(c.ws), _lib.ctypes.byref(st), c.stream), "sas_read_status")
    if st.value:
        raise RuntimeError(f"{what} device status: {_lib.status_names(st.value)}")


def _launch(q, ori_kv, cmp_kv, cmp_sparse_indices, ori_block_table, cmp_block_table, cu_seqlens_q, seqused_kv,
            sinks, metadata, softmax_scale, cmp_ratio, ori_win_left, layout_q, v_head_dim, kernel, max_seqlen_q,
            split_tiles, check_status, lazy_rescale, out, lse_out):
    """One sas_forward call (the body of both registered forward ops).  ``out`` / ``lse_out`` are
    the outputs in the layout of ``q``."""
    c = _marshal(q, ori_kv, cmp_kv, cmp_sparse_indices, ori_block_table, cmp_block_table, cu_seqlens_q, seqused_kv,
                 sinks, metadata, softmax_scale, cmp_ratio, ori_win_left, layout_q, v_head_dim, kernel, max_seqlen_q,
                 split_tiles, lazy_rescale)
    T, N1, Dv = c.T, c.N1, c.Dv
    out_flat = out.view(T, N1, Dv)
    out_user = None  # a caller's out that starts inside a 16-byte vector: written through a copy
    if out_flat.data_ptr() % 16:
        out_user, out_flat = out_flat, torch.empty_like(out_flat)
    lse_flat = lse_out.view(T, N1)
    rc = c.lib.sas_forward(
        _lib.ctypes.byref(c.args),
        _ptr(c.q),
        _ptr(c.ori_kv),
        _ptr(c.ori_bt),
        _ptr(c.cmp_kv),
        _ptr(c.cmp_bt),
        _ptr(c.idx),
        _ptr(c.q_prefix),
        _ptr(c.act_q),
        _ptr(c.seq_kv),
        _ptr(c.sinks),
        _ptr(c.metadata),
        _ptr(out_flat),
        _ptr(lse_flat),
        _ptr(c.ws),
        c.ws.numel(),
        c.stream,
    )
    _lib.check(rc, "sas_forward")
    if out_user is not None:
        out_user.copy_(out_flat)
    if check_status:
        _check_status(c, "sas_forward")


@torch.library.custom_op("sas_b200::sparse_attn_sharedkv", mutates_args=(), device_types="cuda")
def _op(q: torch.Tensor, ori_kv: torch.Tensor, cmp_kv: Optional[torch.Tensor],
        cmp_sparse_indices: Optional[torch.Tensor], ori_block_table: torch.Tensor,
        cmp_block_table: Optional[torch.Tensor], cu_seqlens_q: Optional[torch.Tensor], seqused_kv: torch.Tensor,
        sinks: torch.Tensor, metadata: Optional[torch.Tensor], softmax_scale: float, cmp_ratio: int,
        ori_win_left: int, layout_q: str, v_head_dim: int, kernel: str, max_seqlen_q: int, split_tiles: int,
        check_status: bool, lazy_rescale: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    """sparse_attn_sharedkv with op-owned outputs: returns ``(out, lse)`` in the layout of ``q``."""
    o_shape, l_shape = _out_shapes(q, layout_q, v_head_dim)
    out = torch.empty(o_shape, dtype=q.dtype, device=q.device)
    lse = torch.empty(l_shape, dtype=torch.float32, device=q.device)
    _launch(q, ori_kv, cmp_kv, cmp_sparse_indices, ori_block_table, cmp_block_table, cu_seqlens_q, seqused_kv,
            sinks, metadata, softmax_scale, cmp_ratio, ori_win_left, layout_q, v_head_dim, kernel, max_seqlen_q,
            split_tiles, check_status, lazy_rescale, out, lse)
    return out, lse


@_op.register_fake
def _op_fake(q, ori_kv, cmp_kv, cmp_sparse_indices, ori_block_table, cmp_block_table, cu_seqlens_q, seqused_kv,
             sinks, metadata, softmax_scale, cmp_ratio, ori_win_left, layout_q, v_head_dim, kernel, max_seqlen_q,
             split_tiles, check_status, lazy_rescale):
    o_shape, l_shape = _out_shapes(q, layout_q, v_head_dim)
    return q.new_empty(o_shape), q.new_empty(l_shape, dtype=torch.float32)


@torch.library.custom_op("sas_b200::sparse_attn_sharedkv_out", mutates_args=("out", "lse"), device_types="cuda")
def _op_out(q: torch.Tensor, ori_kv: torch.Tensor, cmp_kv: Optional[torch.Tensor],
            cmp_sparse_indices: Optional[torch.Tensor], ori_block_table: torch.Tensor,
            cmp_block_table: Optional[torch.Tensor], cu_seqlens_q: Optional[torch.Tensor], seqused_kv: torch.Tensor,
            sinks: torch.Tensor, metadata: Optional[torch.Tensor], softmax_scale: float, cmp_ratio: int,
            ori_win_left: int, layout_q: str, v_head_dim: int, kernel: str, max_seqlen_q: int, split_tiles: int,
            check_status: bool, lazy_rescale: bool, out: torch.Tensor, lse: torch.Tensor) -> None:
    """sparse_attn_sharedkv into caller-owned ``out`` / ``lse`` (layout of ``q``)."""
    _launch(q, ori_kv, cmp_kv, cmp_sparse_indices, ori_block_table, cmp_block_table, cu_seqlens_q, seqused_kv,
            sinks, metadata, softmax_scale, cmp_ratio, ori_win_left, layout_q, v_head_dim, kernel, max_seqlen_q,
            split_tiles, check_status, lazy_rescale, out, lse)


@_op_out.register_fake
def _op_out_fake(q, ori_kv, cmp_kv, cmp_sparse_indices, ori_block_table, cmp_block_table, cu_seqlens_q, seqused_kv,
                 sinks, metadata, softmax_scale, cmp_ratio, ori_win_left, layout_q, v_head_dim, kernel, max_seqlen_q,
                 split_tiles, check_status, lazy_rescale, out, lse):
    return None


def _launch_backward(q, ori_kv, cmp_kv, cmp_sparse_indices, ori_block_table, cmp_block_table, cu_seqlens_q,
                     seqused_kv, sinks, out, lse, grad_out, grad_lse, softmax_scale, cmp_ratio, ori_win_left,
                     layout_q, v_head_dim, max_seqlen_q, check_status):
    """One sas_backward call: (dq, d_ori_kv, d_cmp_kv, d_sinks) in the inputs' shapes and dtypes
    (d_cmp_kv empty when there is no compressed cache)."""
    c = _marshal(q, ori_kv, cmp_kv, cmp_sparse_indices, ori_block_table, cmp_block_table, cu_seqlens_q, seqused_kv,
                 sinks, None, softmax_scale, cmp_ratio, ori_win_left, layout_q, v_head_dim, "simt", max_seqlen_q, 0,
                 False)
    dev, T, N1, Dv, D = q.device, c.T, c.N1, c.Dv, q.shape[-1]
    dq = torch.empty((T, N1, D), dtype=torch.float32, device=dev)
    d_ori = torch.zeros(ori_kv.shape, dtype=torch.float32, device=dev)
    d_cmp = (torch.zeros(cmp_kv.shape, dtype=torch.float32, device=dev) if cmp_kv is not None
             else torch.zeros(0, dtype=torch.float32, device=dev))
    d_sinks = torch.zeros(N1, dtype=torch.float32, device=dev)
    out_c = _dense16(out.reshape(T, N1, Dv))
    lse_c = lse.reshape(T, N1).to(torch.float32).contiguous()
    dout_c = _dense16(grad_out.reshape(T, N1, Dv).to(q.dtype))
    dlse_c = None if grad_lse is None else grad_lse.reshape(T, N1).to(torch.float32).contiguous()
    rc = c.lib.sas_backward(
        _lib.ctypes.byref(c.args), _ptr(c.q), _ptr(c.ori_kv), _ptr(c.ori_bt), _ptr(c.cmp_kv), _ptr(c.cmp_bt),
        _ptr(c.idx), _ptr(c.q_prefix), _ptr(c.act_q), _ptr(c.seq_kv), _ptr(c.sinks), _ptr(out_c), _ptr(lse_c),
        _ptr(dout_c), _ptr(dlse_c), _ptr(dq), _ptr(d_ori), _ptr(d_cmp if cmp_kv is not None else None),
        _ptr(d_sinks), _ptr(c.ws), c.ws.numel(), c.stream)
    _lib.check(rc, "sas_backward")
    if check_status:
        _check_status(c, "sas_backward")
    return (dq.view(q.shape).to(q.dtype), d_ori.to(ori_kv.dtype),
            d_cmp.to(cmp_kv.dtype) if cmp_kv is not None else d_cmp, d_sinks.to(sinks.dtype))


@torch.library.custom_op("sas_b200::sparse_attn_sharedkv_backward", mutates_args=(), device_types="cuda")
def _op_bwd(q: torch.Tensor, ori_kv: torch.Tensor, cmp_kv: Optional[torch.Tensor],
            cmp_sparse_indices: Optional[torch.Tensor], ori_block_table: torch.Tensor,
            cmp_block_table: Optional[torch.Tensor], cu_seqlens_q: Optional[torch.Tensor], seqused_kv: torch.Tensor,
            sinks: torch.Tensor, out: torch.Tensor, lse: torch.Tensor, grad_out: torch.Tensor,
            grad_lse: Optional[torch.Tensor], softmax_scale: float, cmp_ratio: int, ori_win_left: int,
            layout_q: str, v_head_dim: int, max_seqlen_q: int,
            check_status: bool) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Gradients of sparse_attn_sharedkv with respect to q, ori_kv, cmp_kv and sinks."""
    return _launch_backward(q, ori_kv, cmp_kv, cmp_sparse_indices, ori_block_table, cmp_block_table, cu_seqlens_q,
                            seqused_kv, sinks, out, lse, grad_out, grad_lse, softmax_scale, cmp_ratio, ori_win_left,
                            layout_q, v_head_dim, max_seqlen_q, check_status)


@_op_bwd.register_fake
def _op_bwd_fake(q, ori_kv, cmp_kv, cmp_sparse_indices, ori_block_table, cmp_block_table, cu_seqlens_q, seqused_kv,
                 sinks, out, lse, grad_out, grad_lse, softmax_scale, cmp_ratio, ori_win_left, layout_q, v_head_dim,
                 max_seqlen_q, check_status):
    d_cmp = cmp_kv.new_empty(cmp_kv.shape) if cmp_kv is not None else q.new_empty(0, dtype=torch.float32)
    return q.new_empty(q.shape), ori_kv.new_empty(ori_kv.shape), d_cmp, sinks.new_empty(sinks.shape)


def _setup_context(ctx, inputs, output):
    (q, ori_kv, cmp_kv, cmp_sparse_indices, ori_block_table, cmp_block_table, cu_seqlens_q, seqused_kv, sinks,
     _metadata, softmax_scale, cmp_ratio, ori_win_left, layout_q, v_head_dim, _kernel, max_seqlen_q, _split,
     check_status, _lazy) = inputs
    out, lse = output
    ctx.save_for_backward(q, ori_kv, cmp_kv, cmp_sparse_indices, ori_block_table, cmp_block_table, cu_seqlens_q,
                          seqused_kv, sinks, out, lse)
    ctx.consts = (softmax_scale, cmp_ratio, ori_win_left, layout_q, v_head_dim, max_seqlen_q, check_status)
    ctx.has_cmp = cmp_kv is not None


def _backward(ctx, grad_out, grad_lse):
    q, ori_kv, cmp_kv, idx, ori_bt, cmp_bt, cu, seqused_kv, sinks, out, lse = ctx.saved_tensors
    if grad_out is None:
        grad_out = torch.zeros_like(out)
    dq, d_ori, d_cmp, d_sinks = torch.ops.sas_b200.sparse_attn_sharedkv_backward(
        q, ori_kv, cmp_kv, idx, ori_bt, cmp_bt, cu, seqused_kv, sinks, out, lse, grad_out, grad_lse, *ctx.consts)
    return (dq, d_ori, d_cmp if ctx.has_cmp else None, None, None, None, None, None, d_sinks) + (None,) * 11


# the op with op-owned outputs is differentiable (q, ori_kv, cmp_kv, sinks); the ``_out`` form is not
torch.library.register_autograd("sas_b200::sparse_attn_sharedkv", _backward, setup_context=_setup_context)


def sparse_attn_sharedkv(
    q: torch.Tensor,
    *,
    ori_kv: torch.Tensor,
    cmp_kv: Optional[torch.Tensor] = None,
    cmp_sparse_indices: Optional[torch.Tensor] = None,
    ori_block_table: torch.Tensor,
    cmp_block_table: Optional[torch.Tensor] = None,
    cu_seqlens_q: Optional[torch.Tensor] = None,
    seqused_q: Optional[torch.Tensor] = None,
    seqused_kv: torch.Tensor,
    sinks: torch.Tensor,
    metadata: Optional[torch.Tensor] = None,
    softmax_scale: float,
    cmp_ratio: Optional[int] = None,
    ori_mask_mode: int = 4,
    cmp_mask_mode: int = 3,
    ori_win_left: int = 127,
    ori_win_right: int = 0,
    layout_q: str = "TND",
    layout_kv: str = "PA_ND",
    return_softmax_lse: bool = False,
    core_num: int = DEFAULT_CORE_NUM,
    topk_cmp: Optional[int] = None,
    v_head_dim: Optional[int] = None,
    kernel: str = "auto",
    max_seqlen_q: Optional[int] = None,
    out: Optional[torch.Tensor] = None,
    lse_out: Optional[torch.Tensor] = None,
    check_status: bool = False,
    split_tiles: int = 0,
    lazy_rescale: bool = False,
) -> Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]:
    """Sink-seeded sliding-window + compressed attention over a shared K = V cache.

    Scenario 1 (SWA) when ``cmp_kv`` is None, 2 (CFA) when only
    ``cmp_sparse_indices`` is None, 3 (SCFA) otherwise.  Returns ``out`` in
    the layout of ``q`` (last dim ``v_head_dim``), and with
    ``return_softmax_lse`` also the fp32 natural-log LSE ``[T, N1]`` (TND) or
    ``[B, S, N1]`` (BSND) with the sink folded in.

    B200 extensions of the reference signature: ``kernel`` ("auto", "tc", "tc2", "simt"),
    ``max_seqlen_q`` (no host synchronisation when given), ``out`` / ``lse_out``
    (caller-owned outputs), ``check_status`` (raise on device-side status bits) and
    ``split_tiles`` (piece size, in 64-key tiles, for cutting long tokens across the
    tensor-core path's clusters; 0 lets the library decide; see ``sharding.split_hint``) and
    ``lazy_rescale`` (``SAS_FWD_FLAG_LAZY_RESCALE``: raise the softmax's running max only past a
    threshold, faster, P rounded at another scale than the golden's; off by default).
    Everything here is shape logic that ``torch.compile`` traces; the launch is the
    registered op ``torch.ops.sas_b200.sparse_attn_sharedkv`` (``..._out`` with ``out``).
    Without ``out`` / ``lse_out`` the call is differentiable in q, ori_kv, cmp_kv and sinks
    (``sas_backward``, CUDA cores; the reference has no backward).
    """
    del seqused_q, core_num  # API parity (the reference kernel does not read them either)
    assert ori_mask_mode == 4, "only ori_mask_mode=4 supported"
    assert cmp_mask_mode == 3 or cmp_kv is None, "only cmp_mask_mode=3 supported"
    assert ori_win_right == 0, "only ori_win_right=0 supported"
    assert layout_kv == "PA_ND", "only layout_kv=PA_ND supported"
    assert layout_q in ("TND", "BSND"), f"unsupported layout_q={layout_q!r}"
    if kernel not in _lib.KERNELS:
        raise ValueError(f"kernel must be one of {sorted(_lib.KERNELS)}")
    if not q.is_cuda:
        raise ValueError("q must be a CUDA tensor (sas_b200 has no CPU path)")
    scenario = _scenario(cmp_kv, cmp_sparse_indices)
    if layout_q == "TND":
        assert cu_seqlens_q is not None, "cu_seqlens_q is required for TND"
    D = q.shape[-1]
    if scenario == 3:
        K = cmp_sparse_indices.shape[-1]
        assert topk_cmp is None or topk_cmp == K, "topk_cmp does not match cmp_sparse_indices last dim"
    elif scenario == 2:
        assert cmp_ratio is not None, "cmp_ratio is required with cmp_kv"
    Dv = D if v_head_dim is None else int(v_head_dim)
    if ori_kv.shape[-1] != D:
        raise ValueError(f"ori_kv row width {ori_kv.shape[-1]} != head_dim {D}")
    if ori_kv.dtype != q.dtype or (cmp_kv is not None and cmp_kv.dtype != q.dtype):
        raise ValueError("q, ori_kv and cmp_kv must share one dtype")
    if metadata is not None:
        assert metadata.numel() == SAS_META_SIZE, (
            f"metadata must have {SAS_META_SIZE} int32 entries (got {metadata.numel()})"
        )
    if split_tiles < 0:
        raise ValueError("split_tiles must be >= 0")
    ratio = int(cmp_ratio) if cmp_ratio is not None else 4
    mq = -1 if max_seqlen_q is None else int(max_seqlen_q)
    common = (q, ori_kv, cmp_kv, cmp_sparse_indices, ori_block_table, cmp_block_table, cu_seqlens_q, seqused_kv,
              sinks, metadata, float(softmax_scale), ratio, int(ori_win_left), layout_q, Dv, kernel, mq,
              int(split_tiles), bool(check_status), bool(lazy_rescale))
    if out is None and lse_out is None:
        out_r, lse_r = torch.ops.sas_b200.sparse_attn_sharedkv(*common)
    else:
        o_shape, l_shape = _out_shapes(q, layout_q, Dv)
        out_r = out.view(o_shape) if out is not None else torch.empty(o_shape, dtype=q.dtype, device=q.device)
        lse_r = lse_out.view(l_shape) if lse_out is not None else torch.empty(l_shape, dtype=torch.float32,
                                                                             device=q.device)
        torch.ops.sas_b200.sparse_attn_sharedkv_out(*common, out_r, lse_r)
    if return_softmax_lse:
        return out_r, lse_r
    return out_r


def resolve_rows(
    *,
    cmp_sparse_indices: Optional[torch.Tensor],
    ori_block_table: torch.Tensor,
    cmp_block_table: Optional[torch.Tensor],
    cu_seqlens_q: torch.Tensor,
    seqused_kv: torch.Tensor,
    num_heads: int,
    head_dim: int,
    ori_block_num: int,
    ori_block_size: int,
    cmp_block_num: int = 1,
    cmp_block_size: int = 1,
    cmp_ratio: int = 4,
    scenario: int = 3,
    ori_win_left: int = 127,
    max_cmp_len: int = 0,
):
    """Run only the key-resolution step (TND) and return ``(token_info [T, 8], cmp_rows [T, cap])``.

    ``token_info`` columns: b, s_global, ori_left, n_win, n_cmp, valid, s, 0.
    ``cmp_rows`` holds physical compressed rows (-1 = unmapped block).
    """
    dev = ori_block_table.device
    cu = _i32(cu_seqlens_q, dev)
    cu_h = cu_seqlens_q.detach().to("cpu", torch.int64)
    B = cu.numel() - 1
    T = int(cu_h[-1].item()) if B > 0 else 0
    max_q = int((cu_h[1:] - cu_h[:-1]).max().item()) if B > 0 else 0
    args = _lib.SasFwdArgs()
    args.batch, args.num_tokens, args.max_q_len = B, T, max_q
    args.num_heads, args.num_kv_heads, args.head_dim, args.v_head_dim = num_heads, 1, head_dim, min(head_dim, 512)
    args.ori_block_num, args.ori_block_size, args.ori_table_len = ori_block_num, ori_block_size, ori_block_table.shape[1]
    if scenario >= 2:
        args.cmp_block_num, args.cmp_block_size = cmp_block_num, cmp_block_size
        args.cmp_table_len = cmp_block_table.shape[1]
    args.topk = cmp_sparse_indices.shape[-1] if scenario == 3 else 0
    args.cmp_ratio, args.scenario, args.max_cmp_len = cmp_ratio, scenario, max_cmp_len
    args.ori_win_left, args.ori_mask_mode, args.cmp_mask_mode = ori_win_left, 4, 3
    args.dtype, args.softmax_scale, args.kernel = 0, 1.0, _lib.KERNELS["simt"]
    lib = _lib.load()
    nbytes = _lib.ctypes.c_size_t(0)
    _lib.check(lib.sas_workspace_size(_lib.ctypes.byref(args), _lib.ctypes.byref(nbytes)), "sas_workspace_size")
    ws = _workspace(nbytes.value, dev)
    cap = args.topk if scenario == 3 else (max_cmp_len if scenario == 2 else 0)
    tinfo = torch.zeros((T, 8), dtype=torch.int32, device=dev)
    rows = torch.full((T, max(cap, 1)), -7, dtype=torch.int32, device=dev)
    idx = _i32(cmp_sparse_indices, dev) if scenario == 3 else None
    bt_c = _i32(cmp_block_table, dev) if scenario >= 2 else None
    ori_bt = _i32(ori_block_table, dev)
    seq = _i32(seqused_kv, dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = lib.sas_resolve_rows(_lib.ctypes.byref(args), _ptr(ori_bt), _ptr(bt_c), _ptr(idx), _ptr(cu[:-1]),
                              _ptr((cu[1:] - cu[:-1]).contiguous()), _ptr(seq), _ptr(tinfo), _ptr(rows), _ptr(ws),
                              ws.numel(), stream)
    _lib.check(rc, "sas_resolve_rows")
    st = _lib.ctypes.c_uint32(0)
    _lib.check(lib.sas_read_status(_ptr(ws), _lib.ctypes.byref(st), stream), "sas_read_status")
    return tinfo, rows[:, :cap], st.value


def split_plan(args) -> Tuple[int, int]:
    """``(pieces, tiles_per_piece)`` of the split-KV plan ``sas_forward`` runs for ``args`` (an
    ``_lib.SasFwdArgs``); ``(1, 0)``: whole tokens."""
    lib = _lib.load()
    p, m = _lib.ctypes.c_int32(0), _lib.ctypes.c_int32(0)
    _lib.check(lib.sas_split_plan(_lib.ctypes.byref(args), _lib.ctypes.byref(p), _lib.ctypes.byref(m)),
               "sas_split_plan")
    return p.value, m.value


def split_metadata(
    *,
    cmp_sparse_indices: torch.Tensor,
    ori_block_table: torch.Tensor,
    cmp_block_table: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    seqused_kv: torch.Tensor,
    num_heads: int,
    head_dim: int,
    v_head_dim: int,
    ori_block_num: int,
    ori_block_size: int,
    cmp_block_num: int,
    cmp_block_size: int,
    cmp_ratio: int = 4,
    ori_win_left: int = 127,
    split_tiles: int = 0,
    max_seqlen_q: Optional[int] = None,
    kernel: str = "auto",
):
    """The tensor-core path's split-KV plan for a TND SCFA call, as ``int32[1024]`` in the reference
    metadata layout (FD rows, ``sas_split_metadata``), plus the ``SasFwdArgs`` it was planned for."""
    dev = ori_block_table.device
    cu = _i32(cu_seqlens_q, dev)
    B = cu.numel() - 1
    T = cmp_sparse_indices.shape[0]
    if max_seqlen_q is None:
        cu_h = cu_seqlens_q.detach().to("cpu", torch.int64)
        max_seqlen_q = int((cu_h[1:] - cu_h[:-1]).max().item()) if B > 0 else 0
    args = _lib.SasFwdArgs()
    args.batch, args.num_tokens, args.max_q_len = B, T, int(max_seqlen_q)
    args.num_heads, args.num_kv_heads, args.head_dim, args.v_head_dim = num_heads, 1, head_dim, v_head_dim
    args.ori_block_num, args.ori_block_size, args.ori_table_len = ori_block_num, ori_block_size, ori_block_table.shape[1]
    args.cmp_block_num, args.cmp_block_size, args.cmp_table_len = cmp_block_num, cmp_block_size, cmp_block_table.shape[1]
    args.topk, args.cmp_ratio, args.scenario = cmp_sparse_indices.shape[-1], cmp_ratio, 3
    args.ori_win_left, args.ori_mask_mode, args.cmp_mask_mode = ori_win_left, 4, 3
    args.dtype, args.softmax_scale, args.kernel = _lib.SAS_DTYPE_BF16, 1.0, _lib.KERNELS[kernel]
    args.flags = _lib.SAS_FWD_FLAG_CU_SEQLENS
    args.split_tiles = int(split_tiles)
    lib = _lib.load()
    nbytes = _lib.ctypes.c_size_t(0)
    _lib.check(lib.sas_workspace_size(_lib.ctypes.byref(args), _lib.ctypes.byref(nbytes)), "sas_workspace_size")
    ws = _workspace(nbytes.value, dev)
    out = torch.empty(SAS_META_SIZE, dtype=torch.int32, device=dev)
    idx = _i32(cmp_sparse_indices, dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = lib.sas_split_metadata(_lib.ctypes.byref(args), _ptr(_i32(ori_block_table, dev)),
                                _ptr(_i32(cmp_block_table, dev)), _ptr(idx), _ptr(cu), None,
                                _ptr(_i32(seqused_kv, dev)), _ptr(out), _ptr(ws), ws.numel(), stream)
    _lib.check(rc, "sas_split_metadata")
    return out, args
