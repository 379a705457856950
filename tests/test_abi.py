"""The C ABI library: it loads, exports what include/sas_b200.h declares, its
structs agree with the ctypes mirror, and its argument checks reject
out-of-contract calls before touching the device.  No GPU needed."""

import ctypes
import os
import re
import subprocess

import pytest

from dsv4_planb_b200 import _lib, build

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "sas_b200.h")


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sas_[a-z_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert declared_functions() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.lib_path()], capture_output=True, text=True, check=True)
    exported = set(line.split()[-1] for line in out.stdout.splitlines() if line.strip())
    for name in declared_functions():
        assert name in exported, name
        assert getattr(lib, name) is not None


def test_struct_layout_matches_header(tmp_path):
    src = tmp_path / "probe.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "sas_b200.h"\n'
        "int main(void){printf(\"%zu %zu %zu %zu\\n\", sizeof(SasFwdArgs), sizeof(SasMetaArgs),"
        " offsetof(SasFwdArgs, softmax_scale), offsetof(SasMetaArgs, reserved));return 0;}\n"
    )
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-I", os.path.dirname(HEADER), str(src), "-o", str(exe)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert vals == [ctypes.sizeof(_lib.SasFwdArgs), ctypes.sizeof(_lib.SasMetaArgs),
                    _lib.SasFwdArgs.softmax_scale.offset, _lib.SasMetaArgs.reserved.offset]


def good_args():
    a = _lib.SasFwdArgs()
    a.batch, a.num_tokens, a.max_q_len = 2, 2, 1
    a.num_heads, a.num_kv_heads, a.head_dim, a.v_head_dim = 128, 1, 576, 512
    a.ori_block_num, a.ori_block_size, a.ori_table_len = 64, 128, 32
    a.cmp_block_num, a.cmp_block_size, a.cmp_table_len = 16, 128, 8
    a.topk, a.cmp_ratio, a.scenario = 2048, 4, 3
    a.ori_win_left, a.ori_win_right, a.ori_mask_mode, a.cmp_mask_mode = 127, 0, 4, 3
    a.dtype, a.softmax_scale = _lib.SAS_DTYPE_BF16, 576 ** -0.5
    return a


def ws_size(lib, a):
    n = ctypes.c_size_t(0)
    rc = lib.sas_workspace_size(ctypes.byref(a), ctypes.byref(n))
    return rc, n.value


def test_workspace_size_and_validation(lib):
    a = good_args()
    rc, n = ws_size(lib, a)
    assert rc == _lib.SAS_OK and n >= 2 * 8 * 4 + 2 * 2048 * 4
    bad = [
        ("num_kv_heads", 2, _lib.SAS_ERR_UNSUPPORTED),
        ("ori_mask_mode", 3, _lib.SAS_ERR_UNSUPPORTED),
        ("ori_win_right", 1, _lib.SAS_ERR_UNSUPPORTED),
        ("cmp_mask_mode", 1, _lib.SAS_ERR_UNSUPPORTED),
        ("scenario", 4, _lib.SAS_ERR_INVALID_ARG),
        ("head_dim", 570, _lib.SAS_ERR_UNSUPPORTED),
        ("v_head_dim", 600, _lib.SAS_ERR_UNSUPPORTED),
        ("dtype", 7, _lib.SAS_ERR_INVALID_ARG),
        ("cmp_ratio", 0, _lib.SAS_ERR_INVALID_ARG),
        ("batch", -1, _lib.SAS_ERR_INVALID_ARG),
        ("kernel", 9, _lib.SAS_ERR_INVALID_ARG),
        ("ori_win_left", -1, _lib.SAS_ERR_INVALID_ARG),
    ]
    for field, value, want in bad:
        b = good_args()
        setattr(b, field, value)
        assert ws_size(lib, b)[0] == want, field
    b = good_args()
    b.reserved[2] = 1
    assert ws_size(lib, b)[0] == _lib.SAS_ERR_INVALID_ARG


def test_forward_rejects_before_touching_the_device(lib):
    a = good_args()
    null = None
    # missing workspace
    rc = lib.sas_forward(ctypes.byref(a), 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, null, 1, 1, null, 0, null)
    assert rc == _lib.SAS_ERR_WORKSPACE
    # missing indices in scenario 3
    rc = lib.sas_forward(ctypes.byref(a), 1, 1, 1, 1, 1, null, 1, 1, 1, 1, null, 1, 1, 1, 1 << 30, null)
    assert rc == _lib.SAS_ERR_INVALID_ARG
    # missing cmp pool in scenario 2
    a.scenario, a.max_cmp_len = 2, 100
    rc = lib.sas_forward(ctypes.byref(a), 1, 1, 1, null, 1, null, 1, 1, 1, 1, null, 1, 1, 1, 1 << 30, null)
    assert rc == _lib.SAS_ERR_INVALID_ARG
    assert lib.sas_forward(None, *([None] * 13), None, 0, None) == _lib.SAS_ERR_INVALID_ARG


def test_forward_rejects_misaligned_pointers(lib):
    # q, the pools, out and the workspace need 16-byte alignment (vector accesses, TMA tensor maps);
    # the int32 / fp32 arrays 4-byte.  The check runs before any device work, so fake addresses do.
    a = good_args()
    base = [0x10000 * (i + 1) for i in range(16)]  # q .. lse, all 256-byte aligned
    names = ["q", "ori_kv", "ori_bt", "cmp_kv", "cmp_bt", "idx", "q_prefix", "act_q", "act_kv", "sinks",
             "metadata", "out", "lse"]
    wide = {"q", "ori_kv", "cmp_kv", "out"}
    for i, name in enumerate(names):
        if name == "metadata":
            continue  # not read by the kernels
        ptrs = list(base[:13])
        ptrs[i] += 8 if name in wide else 2
        rc = lib.sas_forward(ctypes.byref(a), *ptrs, 0x1000000, 1 << 30, None)
        assert rc == _lib.SAS_ERR_INVALID_ARG, name
    rc = lib.sas_forward(ctypes.byref(a), *base[:13], 0x1000008, 1 << 30, None)
    assert rc == _lib.SAS_ERR_INVALID_ARG, "workspace"


def test_noalloc_rejects_misaligned_pointers(lib):
    # the entry point without a workspace follows the same pointer rule, checked before any device work
    a = good_args()
    base = [0x10000 * (i + 1) for i in range(13)]
    for i, wide in [(0, True), (1, True), (3, True), (11, True), (2, False), (9, False), (12, False)]:
        ptrs = list(base)
        ptrs[i] += 8 if wide else 2
        assert lib.sas_forward_noalloc(ctypes.byref(a), *ptrs, None) == _lib.SAS_ERR_INVALID_ARG, i


def test_cu_seqlens_flag(lib):
    # act_q_len may be NULL only with SAS_FWD_FLAG_CU_SEQLENS; unknown flag bits are rejected
    a = good_args()
    null = None
    rc = lib.sas_forward(ctypes.byref(a), 1, 1, 1, 1, 1, 1, 1, null, 1, 1, null, 1, 1, 1, 1 << 30, null)
    assert rc == _lib.SAS_ERR_INVALID_ARG
    a.flags = 0x2
    assert ws_size(lib, a)[0] == _lib.SAS_ERR_INVALID_ARG
    a.flags = _lib.SAS_FWD_FLAG_CU_SEQLENS
    assert ws_size(lib, a)[0] == _lib.SAS_OK


def kernel_count(lib, a):
    n = ctypes.c_int32(-1)
    rc = lib.sas_forward_kernel_count(ctypes.byref(a), ctypes.byref(n))
    return rc, n.value


def test_kernel_count_and_split_workspace(lib):
    # clear + prep + attention; small SCFA batches on the tensor-core path are cut into pieces
    # (split KV), which adds the LSE-combine kernel and per-piece partials to the workspace
    a = good_args()  # 2 tokens: split
    rc, n = kernel_count(lib, a)
    assert rc == _lib.SAS_OK and n == 4
    split_ws = ws_size(lib, a)[1]
    a.kernel = _lib.KERNELS["simt"]
    assert kernel_count(lib, a) == (_lib.SAS_OK, 3)
    assert ws_size(lib, a)[1] < split_ws
    a.kernel = _lib.KERNELS["auto"]
    a.batch, a.num_tokens = 64, 64  # a full decode batch: one unit per token
    assert kernel_count(lib, a) == (_lib.SAS_OK, 3)
    a.batch, a.num_tokens = 37, 37  # the largest batch that is still split
    assert kernel_count(lib, a) == (_lib.SAS_OK, 4)
    a.scenario = 1  # window only: never split
    assert kernel_count(lib, a) == (_lib.SAS_OK, 3)
    a.scenario, a.num_tokens = 3, 0  # only the status word is cleared
    assert kernel_count(lib, a) == (_lib.SAS_OK, 1)
    a.num_tokens, a.num_heads = 4, 0
    assert kernel_count(lib, a)[0] == _lib.SAS_ERR_INVALID_ARG


def test_split_tiles_hint(lib):
    # a caller-chosen piece size cuts tokens whatever the batch size; negative sizes are rejected
    a = good_args()
    a.batch, a.num_tokens = 128, 128
    plain = ws_size(lib, a)[1]
    assert kernel_count(lib, a) == (_lib.SAS_OK, 3)
    a.split_tiles = 16
    assert kernel_count(lib, a) == (_lib.SAS_OK, 4)
    assert ws_size(lib, a)[1] > plain
    a.split_tiles = 64  # no token has more tiles than that: nothing to cut
    assert kernel_count(lib, a) == (_lib.SAS_OK, 3)
    a.split_tiles = -1
    assert ws_size(lib, a)[0] == _lib.SAS_ERR_INVALID_ARG
    # a prefill-sized batch would need more than 1 GiB of partials: whole tokens instead
    a.split_tiles, a.batch, a.num_tokens, a.max_q_len = 16, 4, 32768, 8192
    assert kernel_count(lib, a) == (_lib.SAS_OK, 3)


def test_metadata_validation(lib):
    m = _lib.SasMetaArgs()
    m.num_heads_q, m.num_heads_kv, m.head_dim = 64, 1, 512
    m.batch_size, m.aic_core_num, m.aiv_core_num = 1, 24, 48
    n = ctypes.c_size_t(0)
    assert lib.sas_metadata_workspace_size(ctypes.byref(m), ctypes.byref(n)) == _lib.SAS_OK and n.value > 0
    m.num_heads_kv = 0
    assert lib.sas_metadata_workspace_size(ctypes.byref(m), ctypes.byref(n)) == _lib.SAS_ERR_INVALID_ARG
    m.num_heads_kv = 128
    assert lib.sas_metadata_workspace_size(ctypes.byref(m), ctypes.byref(n)) == _lib.SAS_ERR_INVALID_ARG


def test_strerror_and_version(lib):
    assert lib.sas_abi_version() == 1
    for rc in range(6):
        assert _lib.strerror(rc)


def test_api_rehomes_views_that_start_inside_a_vector():
    # The Python layer hands the C ABI only 16-byte aligned q bases: a view at an odd element
    # offset is copied (same values), an aligned one passes through untouched.
    import torch

    from dsv4_planb_b200.api import _dense16

    base = torch.arange(64, dtype=torch.bfloat16)
    aligned = base[8:40].view(4, 8)  # 16 bytes into a (>= 16-byte aligned) allocation
    assert _dense16(aligned).data_ptr() == aligned.data_ptr()
    odd = base[1:33].view(4, 8)
    fixed = _dense16(odd)
    assert fixed.data_ptr() % 16 == 0 and fixed.data_ptr() != odd.data_ptr()
    assert torch.equal(fixed, odd)
    strided = base.view(8, 8)[:, :4]  # non-contiguous: made dense
    assert _dense16(strided).is_contiguous() and torch.equal(_dense16(strided), strided)


def test_api_rejects_misaligned_or_strided_pools():
    # A paged KV pool is never copied per call (it can be gigabytes): a pool view that starts
    # inside a 16-byte vector, or is not contiguous, is an argument error.
    import pytest
    import torch

    from dsv4_planb_b200.api import _pool16

    base = torch.zeros(4 * 128 * 576 + 1, dtype=torch.bfloat16)
    good = base[:-1].view(4, 128, 1, 576)
    assert _pool16(good, "ori_kv") is good
    with pytest.raises(ValueError, match="16-byte"):
        _pool16(base[1:].view(4, 128, 1, 576), "ori_kv")
    with pytest.raises(ValueError, match="contiguous"):
        _pool16(good.transpose(0, 1), "cmp_kv")


def test_registered_op_fake_shapes():
    # The op is registered with the dispatcher; its fake (meta) implementation gives the output
    # shapes and dtypes without a device, which is what torch.compile traces against.
    import torch
    from torch._subclasses.fake_tensor import FakeTensorMode

    import dsv4_planb_b200.api  # noqa: F401  (registers the ops)

    with FakeTensorMode():
        q = torch.empty(6, 128, 576, dtype=torch.bfloat16)
        pool = torch.empty(10, 128, 1, 576, dtype=torch.bfloat16)
        bt = torch.empty(2, 5, dtype=torch.int32)
        idx = torch.empty(6, 1, 2048, dtype=torch.int32)
        cu = torch.empty(3, dtype=torch.int32)
        kv = torch.empty(2, dtype=torch.int32)
        sinks = torch.empty(128, dtype=torch.float32)
        out, lse = torch.ops.sas_b200.sparse_attn_sharedkv(q, pool, pool, idx, bt, bt, cu, kv, sinks, None, 0.04, 4,
                                                           127, "TND", 512, "auto", 3, 0, False, False)
        assert out.shape == (6, 128, 512) and out.dtype == torch.bfloat16
        assert lse.shape == (6, 128) and lse.dtype == torch.float32
        qb = torch.empty(2, 3, 128, 576, dtype=torch.bfloat16)
        out, lse = torch.ops.sas_b200.sparse_attn_sharedkv(qb, pool, None, None, bt, None, None, kv, sinks, None,
                                                           0.04, 4, 127, "BSND", 512, "tc", -1, 0, False, True)
        assert out.shape == (2, 3, 128, 512) and lse.shape == (2, 3, 128)


def test_split_plan_shape_matches_the_workspace(lib):
    # The plan sas_split_plan reports is the one sas_workspace_size sizes: bf16 partial outputs and
    # fp32 (m, l, lr, 0) statistics for T x pieces slots.  Small SCFA batches on the tensor-core path
    # split; large ones, the CUDA-core kernel and a caller's piece size >= a token's tiles do not.
    def plan(a):
        p, m = ctypes.c_int32(-1), ctypes.c_int32(-1)
        assert lib.sas_split_plan(ctypes.byref(a), ctypes.byref(p), ctypes.byref(m)) == 0
        return p.value, m.value

    for T in (1, 4, 16, 37, 38, 64):
        a = good_args()
        a.batch, a.num_tokens, a.max_q_len = T, T, 1
        a.num_heads, a.head_dim, a.v_head_dim, a.topk, a.kernel = 128, 576, 512, 2048, 0
        P, M = plan(a)
        if T <= 37:
            assert P > 1 and M >= 4 and P * M >= 34 and (P - 1) * M < 34, (T, P, M)
        else:
            assert (P, M) == (1, 0)
        base = ws_size(lib, a)[1]
        a.kernel = _lib.KERNELS["simt"]
        assert plan(a) == (1, 0)
        simt = ws_size(lib, a)[1]
        assert base - simt >= (T * P * 128 * (512 * 2 + 16) if P > 1 else 0)
        assert base - simt < (T * P * 128 * (512 * 2 + 16) if P > 1 else 0) + 512
        a.kernel, a.split_tiles = 0, 40  # a piece size no token exceeds: whole tokens
        assert plan(a) == (1, 0)
        a.split_tiles = 6
        P, M = plan(a)
        assert M == 6 and P == -(-34 // 6)


def test_backward_op_fake_shapes():
    # The backward op's fake implementation: gradients in the shapes and dtypes of q, the pools and
    # the sinks (an empty fp32 tensor for the compressed pool when there is none).
    import torch
    from torch._subclasses.fake_tensor import FakeTensorMode

    import dsv4_planb_b200.api  # noqa: F401  (registers the ops)

    with FakeTensorMode():
        q = torch.empty(6, 128, 576, dtype=torch.bfloat16)
        pool = torch.empty(10, 128, 1, 576, dtype=torch.bfloat16)
        bt = torch.empty(2, 5, dtype=torch.int32)
        idx = torch.empty(6, 1, 2048, dtype=torch.int32)
        cu = torch.empty(3, dtype=torch.int32)
        kv = torch.empty(2, dtype=torch.int32)
        sinks = torch.empty(128, dtype=torch.float32)
        out = torch.empty(6, 128, 512, dtype=torch.bfloat16)
        lse = torch.empty(6, 128, dtype=torch.float32)
        dq, d_ori, d_cmp, d_s = torch.ops.sas_b200.sparse_attn_sharedkv_backward(
            q, pool, pool, idx, bt, bt, cu, kv, sinks, out, lse, out, lse, 0.04, 4, 127, "TND", 512, 3, False)
        assert dq.shape == q.shape and dq.dtype == q.dtype
        assert d_ori.shape == pool.shape and d_cmp.shape == pool.shape and d_s.shape == sinks.shape
        dq, d_ori, d_cmp, d_s = torch.ops.sas_b200.sparse_attn_sharedkv_backward(
            q, pool, None, None, bt, None, cu, kv, sinks, out, lse, out, None, 0.04, 4, 127, "TND", 512, 3, False)
        assert d_cmp.numel() == 0 and d_ori.shape == pool.shape


def test_backward_rejects_bad_pointers(lib):
    # sas_backward checks its pointers before any device work: a missing or misaligned gradient
    # buffer and a short workspace are argument errors.
    a = good_args()
    base = [0x10000 * (i + 1) for i in range(18)]  # q .. d_sinks, all 256-byte aligned
    for i, off in [(12, 8), (14, 8), (15, 2), (17, 2), (16, 2)]:  # dout, dq, d_ori, d_sinks, d_cmp
        ptrs = list(base)
        ptrs[i] += off
        assert lib.sas_backward(ctypes.byref(a), *ptrs, 0x1000000, 1 << 30, None) == _lib.SAS_ERR_INVALID_ARG, i
    for i in (10, 11, 12, 14, 15, 17):  # out, lse, dout, dq, d_ori, d_sinks are required
        ptrs = list(base)
        ptrs[i] = None
        assert lib.sas_backward(ctypes.byref(a), *ptrs, 0x1000000, 1 << 30, None) == _lib.SAS_ERR_INVALID_ARG, i
    assert lib.sas_backward(ctypes.byref(a), *base, 0x1000000, 16, None) == _lib.SAS_ERR_WORKSPACE
