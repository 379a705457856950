// C-ABI entry points of the sas_b200 library: argument validation, workspace
// layout and launch sequencing for sparse_attn_sharedkv.
//
// Validation follows the reference API's contract (api.py:186-191, 279-282):
// band mask (mode 4) with win_right 0, cmp mask mode 3, one KV head.  The
// reference additionally pins N1 = 64 and D = 512 for its TileLang kernel; this
// library accepts any N1 and D_qk % 8 == 0, with D_v <= D_qk (V = the first D_v
// columns of each K = V row), which covers the D_qk 576 / D_v 512 shapes of the
// DeepSeek-V4 configurations.

#include <stdio.h>

#include "sas_common.cuh"

namespace sas_host {

int launch_prep(const SasFwdArgs &a, const sas::FwdLayout &L, char *ws, const int32_t *cmp_bt, const int32_t *idx,
                const int32_t *q_prefix, const int32_t *act_q, const int32_t *act_kv, cudaStream_t s);
int launch_fwd_simt(const SasFwdArgs &a, const sas::FwdLayout &L, char *ws, const void *q, const void *ori_kv,
                    const int32_t *ori_bt, const void *cmp_kv, const int32_t *cmp_bt, const float *sinks, void *out,
                    float *lse, cudaStream_t s);
bool tc_supported(const SasFwdArgs &a);
size_t tc_workspace(const SasFwdArgs &a);
int tc_kernel_count(const SasFwdArgs &a);
void tc_split_shape(const SasFwdArgs &a, int32_t *pieces, int32_t *tiles);
int launch_split_metadata(const SasFwdArgs &a, const sas::FwdLayout &L, char *ws, bool tc, int32_t *out,
                          cudaStream_t s);
int launch_fwd_tc(const SasFwdArgs &a, const sas::FwdLayout &L, char *ws, const void *q, const void *ori_kv,
                  const int32_t *ori_bt, const void *cmp_kv, const int32_t *cmp_bt, const float *sinks, void *out,
                  float *lse, cudaStream_t s, bool pair);
int launch_bwd_simt(const SasFwdArgs &a, const sas::FwdLayout &L, char *ws, const void *q, const void *ori_kv,
                    const int32_t *ori_bt, const void *cmp_kv, const int32_t *cmp_bt, const float *sinks,
                    const void *out, const float *lse, const void *dout, const float *dlse, float *dq, float *d_ori,
                    float *d_cmp, float *d_sinks, cudaStream_t s);

int check_cuda(cudaError_t e) {
    if (e == cudaSuccess) return SAS_OK;
    fprintf(stderr, "sas_b200: CUDA error %d (%s)\n", (int)e, cudaGetErrorString(e));
    return SAS_ERR_CUDA;
}

int validate_fwd(const SasFwdArgs &a) {
    if (a.batch < 0 || a.batch > 65535 || a.num_tokens < 0 || a.max_q_len < 0) return SAS_ERR_INVALID_ARG;
    if (a.num_heads <= 0 || a.head_dim <= 0 || a.v_head_dim <= 0) return SAS_ERR_INVALID_ARG;
    if (a.num_kv_heads != 1) return SAS_ERR_UNSUPPORTED;
    if (a.scenario < 1 || a.scenario > 3) return SAS_ERR_INVALID_ARG;
    if (a.ori_mask_mode != 4 || a.ori_win_right != 0) return SAS_ERR_UNSUPPORTED;
    if (a.scenario >= 2 && a.cmp_mask_mode != 3) return SAS_ERR_UNSUPPORTED;
    if (a.ori_win_left < 0) return SAS_ERR_INVALID_ARG;
    if (a.head_dim % 8 != 0 || a.head_dim > 1024) return SAS_ERR_UNSUPPORTED;
    if (a.v_head_dim > a.head_dim || a.v_head_dim % 32 != 0 || a.v_head_dim > 512) return SAS_ERR_UNSUPPORTED;
    if (a.dtype != SAS_DTYPE_BF16 && a.dtype != SAS_DTYPE_FP16) return SAS_ERR_INVALID_ARG;
    if (a.ori_block_num <= 0 || a.ori_block_size <= 0 || a.ori_table_len <= 0) return SAS_ERR_INVALID_ARG;
    if ((int64_t)a.ori_block_num * a.ori_block_size >= ((int64_t)1 << 31)) return SAS_ERR_UNSUPPORTED;
    if (a.scenario >= 2) {
        if (a.cmp_block_num <= 0 || a.cmp_block_size <= 0 || a.cmp_table_len <= 0 || a.cmp_ratio <= 0)
            return SAS_ERR_INVALID_ARG;
        if ((int64_t)a.cmp_block_num * a.cmp_block_size >= ((int64_t)1 << 31)) return SAS_ERR_UNSUPPORTED;
    }
    if (a.scenario == 3 && a.topk < 0) return SAS_ERR_INVALID_ARG;
    if (a.scenario == 2 && a.max_cmp_len < 0) return SAS_ERR_INVALID_ARG;
    if (a.kernel < SAS_KERNEL_AUTO || a.kernel > SAS_KERNEL_TC2) return SAS_ERR_INVALID_ARG;
    if ((a.flags & ~(SAS_FWD_FLAG_CU_SEQLENS | SAS_FWD_FLAG_TEST_STALL | SAS_FWD_FLAG_LAZY_RESCALE)) != 0)
        return SAS_ERR_INVALID_ARG;
    if (a.split_tiles < 0) return SAS_ERR_INVALID_ARG;
    for (int i = 0; i < 4; ++i)
        if (a.reserved[i] != 0) return SAS_ERR_INVALID_ARG;
    if ((a.kernel == SAS_KERNEL_TC || a.kernel == SAS_KERNEL_TC2) && !tc_supported(a)) return SAS_ERR_UNSUPPORTED;
    return SAS_OK;
}

// cfa_rows: also room for scenario 2's compressed rows (max_cmp_len per token), which only the
// sas_resolve_rows export writes; the attention kernels resolve CFA rows through the table directly.
sas::FwdLayout fwd_layout(const SasFwdArgs &a, bool cfa_rows) {
    sas::FwdLayout L{};
    L.row_cap = a.scenario == 3 ? a.topk : (a.scenario == 2 && cfa_rows ? a.max_cmp_len : 0);
    const size_t T = (size_t)(a.num_tokens > 0 ? a.num_tokens : 0);
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off = sas::align_up(off + bytes); return o; };
    L.status = take(sas::kAlign);
    L.token_info = take(sizeof(int32_t) * sas::TI_INTS * T);
    L.cmp_rows = take(sizeof(int32_t) * (size_t)L.row_cap * T);
    L.tc = take(tc_supported(a) ? tc_workspace(a) : 0);
    L.total = off;
    return L;
}

thread_local cudaEvent_t g_kernel_start = nullptr, g_kernel_stop = nullptr;

int record_kernel_event(bool start, cudaStream_t s) {
    cudaEvent_t e = start ? g_kernel_start : g_kernel_stop;
    if (!e || !g_kernel_start || !g_kernel_stop) return SAS_OK;
    // Inside a stream capture a plain record only orders the capture; the
    // external flag makes it a node that takes a timestamp at every replay.
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (check_cuda(cudaStreamIsCapturing(s, &cs))) return SAS_ERR_CUDA;
    if (cs == cudaStreamCaptureStatusActive) return check_cuda(cudaEventRecordWithFlags(e, s, cudaEventRecordExternal));
    return check_cuda(cudaEventRecord(e, s));
}

static bool use_tc(const SasFwdArgs &a) {
    if (a.kernel == SAS_KERNEL_SIMT) return false;
    return tc_supported(a);
}

} // namespace sas_host

using namespace sas_host;

extern "C" {

int sas_abi_version(void) { return SAS_ABI_VERSION; }

const char *sas_strerror(int status) {
    switch (status) {
    case SAS_OK: return "ok";
    case SAS_ERR_INVALID_ARG: return "invalid argument";
    case SAS_ERR_UNSUPPORTED: return "unsupported shape or mode";
    case SAS_ERR_WORKSPACE: return "workspace missing or too small";
    case SAS_ERR_CUDA: return "CUDA runtime error";
    case SAS_ERR_DEVICE: return "device-side check failed (see status bits)";
    default: return "unknown status";
    }
}

int sas_workspace_size(const SasFwdArgs *args, size_t *bytes) {
    if (!args || !bytes) return SAS_ERR_INVALID_ARG;
    int rc = validate_fwd(*args);
    if (rc) return rc;
    *bytes = fwd_layout(*args, true).total;  // enough for sas_forward and for sas_resolve_rows
    return SAS_OK;
}

int sas_forward_kernel_count(const SasFwdArgs *args, int32_t *count) {
    if (!args || !count) return SAS_ERR_INVALID_ARG;
    const SasFwdArgs &a = *args;
    int rc = validate_fwd(a);
    if (rc) return rc;
    const int clear = 1;  // the status word and token records, always
    const int prep = (a.batch == 0 || a.max_q_len == 0 || a.num_tokens == 0) ? 0 : 1;
    int attn = 0;
    if (a.num_tokens > 0) attn = use_tc(a) ? tc_kernel_count(a) : (a.num_heads > 0 ? 1 : 0);
    *count = clear + prep + attn;
    return SAS_OK;
}

static int check_inputs(const SasFwdArgs &a, const void *ori_kv, const int32_t *ori_bt, const void *cmp_kv,
                        const int32_t *cmp_bt, const int32_t *idx, const int32_t *q_prefix, const int32_t *act_q,
                        const int32_t *act_kv) {
    const bool need_act_q = (a.flags & SAS_FWD_FLAG_CU_SEQLENS) == 0;
    if (a.batch > 0 && (!q_prefix || (need_act_q && !act_q) || !act_kv || !ori_bt || !ori_kv))
        return SAS_ERR_INVALID_ARG;
    if (a.scenario >= 2 && (!cmp_kv || !cmp_bt)) return SAS_ERR_INVALID_ARG;
    if (a.scenario == 3 && a.topk > 0 && a.num_tokens > 0 && !idx) return SAS_ERR_INVALID_ARG;
    return SAS_OK;
}

// The kernels move rows of q, the pools, out and the workspace in 16-byte vectors (and the
// tensor-core kernel reads q and the pools through TMA tensor maps); int32 and fp32 arrays are read
// and written per element.  A misaligned pointer is an argument error, not a device fault.
static bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

static int check_alignment(const void *q, const void *ori_kv, const int32_t *ori_bt, const void *cmp_kv,
                           const int32_t *cmp_bt, const int32_t *idx, const int32_t *q_prefix, const int32_t *act_q,
                           const int32_t *act_kv, const float *sinks, const void *out, const float *lse,
                           const void *workspace) {
    for (const void *p : {q, ori_kv, cmp_kv, out, workspace})
        if (!aligned(p, 16)) return SAS_ERR_INVALID_ARG;
    for (const void *p : {(const void *)ori_bt, (const void *)cmp_bt, (const void *)idx, (const void *)q_prefix,
                          (const void *)act_q, (const void *)act_kv, (const void *)sinks, (const void *)lse})
        if (!aligned(p, 4)) return SAS_ERR_INVALID_ARG;
    return SAS_OK;
}

int sas_forward(const SasFwdArgs *args, const void *q, const void *ori_kv, const int32_t *ori_block_table,
                const void *cmp_kv, const int32_t *cmp_block_table, const int32_t *cmp_indices,
                const int32_t *q_prefix, const int32_t *act_q_len, const int32_t *act_kv_len, const float *sinks,
                const int32_t *metadata, void *out, float *lse, void *workspace, size_t workspace_bytes,
                void *stream) {
    (void)metadata;  // interface parity; the B200 kernels plan their own split
    if (!args) return SAS_ERR_INVALID_ARG;
    const SasFwdArgs &a = *args;
    int rc = validate_fwd(a);
    if (rc) return rc;
    rc = check_inputs(a, ori_kv, ori_block_table, cmp_kv, cmp_block_table, cmp_indices, q_prefix, act_q_len,
                      act_kv_len);
    if (rc) return rc;
    if (a.num_tokens > 0 && (!q || !out || !sinks)) return SAS_ERR_INVALID_ARG;
    const sas::FwdLayout L = fwd_layout(a);
    if (!workspace || workspace_bytes < L.total) return SAS_ERR_WORKSPACE;
    rc = check_alignment(q, ori_kv, ori_block_table, cmp_kv, cmp_block_table, cmp_indices, q_prefix, act_q_len,
                         act_kv_len, sinks, out, lse, workspace);
    if (rc) return rc;
    char *ws = static_cast<char *>(workspace);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    rc = launch_prep(a, L, ws, cmp_block_table, cmp_indices, q_prefix, act_q_len, act_kv_len, s);
    if (rc) return rc;
    if ((rc = record_kernel_event(true, s))) return rc;
    if (use_tc(a)) rc = launch_fwd_tc(a, L, ws, q, ori_kv, ori_block_table, cmp_kv, cmp_block_table, sinks, out, lse, s,
                                     a.kernel == SAS_KERNEL_TC2);
    else rc = launch_fwd_simt(a, L, ws, q, ori_kv, ori_block_table, cmp_kv, cmp_block_table, sinks, out, lse, s);
    if (rc) return rc;
    return record_kernel_event(false, s);
}

int sas_backward(const SasFwdArgs *args, const void *q, const void *ori_kv, const int32_t *ori_block_table,
                 const void *cmp_kv, const int32_t *cmp_block_table, const int32_t *cmp_indices,
                 const int32_t *q_prefix, const int32_t *act_q_len, const int32_t *act_kv_len, const float *sinks,
                 const void *out, const float *lse, const void *dout, const float *dlse, float *dq,
                 float *d_ori_kv, float *d_cmp_kv, float *d_sinks, void *workspace, size_t workspace_bytes,
                 void *stream) {
    if (!args) return SAS_ERR_INVALID_ARG;
    const SasFwdArgs &a = *args;
    int rc = validate_fwd(a);
    if (rc) return rc;
    if (a.head_dim > 1024) return SAS_ERR_UNSUPPORTED;
    rc = check_inputs(a, ori_kv, ori_block_table, cmp_kv, cmp_block_table, cmp_indices, q_prefix, act_q_len,
                      act_kv_len);
    if (rc) return rc;
    if (a.num_tokens > 0 && (!q || !out || !lse || !dout || !sinks || !dq || !d_ori_kv || !d_sinks))
        return SAS_ERR_INVALID_ARG;
    if (a.num_tokens > 0 && a.scenario >= 2 && !d_cmp_kv) return SAS_ERR_INVALID_ARG;
    const sas::FwdLayout L = fwd_layout(a);
    if (!workspace || workspace_bytes < L.total) return SAS_ERR_WORKSPACE;
    rc = check_alignment(q, ori_kv, ori_block_table, cmp_kv, cmp_block_table, cmp_indices, q_prefix, act_q_len,
                         act_kv_len, sinks, out, lse, workspace);
    if (rc) return rc;
    if (!aligned(dout, 16) || !aligned(dq, 16) || !aligned(dlse, 4) || !aligned(d_ori_kv, 4) ||
        !aligned(d_cmp_kv, 4) || !aligned(d_sinks, 4))
        return SAS_ERR_INVALID_ARG;
    char *ws = static_cast<char *>(workspace);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    rc = launch_prep(a, L, ws, cmp_block_table, cmp_indices, q_prefix, act_q_len, act_kv_len, s);
    if (rc) return rc;
    return launch_bwd_simt(a, L, ws, q, ori_kv, ori_block_table, cmp_kv, cmp_block_table, sinks, out, lse, dout,
                           dlse, dq, d_ori_kv, d_cmp_kv, d_sinks, s);
}

int sas_set_kernel_events(void *start_event, void *stop_event) {
    g_kernel_start = static_cast<cudaEvent_t>(start_event);
    g_kernel_stop = static_cast<cudaEvent_t>(stop_event);
    return SAS_OK;
}

int sas_resolve_rows(const SasFwdArgs *args, const int32_t *ori_block_table, const int32_t *cmp_block_table,
                     const int32_t *cmp_indices, const int32_t *q_prefix, const int32_t *act_q_len,
                     const int32_t *act_kv_len, int32_t *token_info, int32_t *cmp_rows, void *workspace,
                     size_t workspace_bytes, void *stream) {
    if (!args) return SAS_ERR_INVALID_ARG;
    const SasFwdArgs &a = *args;
    int rc = validate_fwd(a);
    if (rc) return rc;
    // the pools are not read here; pass the table pointer as a non-null stand-in
    rc = check_inputs(a, ori_block_table, ori_block_table, cmp_block_table, cmp_block_table, cmp_indices, q_prefix,
                      act_q_len, act_kv_len);
    if (rc) return rc;
    const sas::FwdLayout L = fwd_layout(a, true);
    if (!workspace || workspace_bytes < L.total) return SAS_ERR_WORKSPACE;
    if (a.num_tokens > 0 && !token_info) return SAS_ERR_INVALID_ARG;
    rc = check_alignment(nullptr, nullptr, ori_block_table, nullptr, cmp_block_table, cmp_indices, q_prefix,
                         act_q_len, act_kv_len, nullptr, nullptr, nullptr, workspace);
    if (rc || !aligned(token_info, 4) || !aligned(cmp_rows, 4)) return SAS_ERR_INVALID_ARG;
    char *ws = static_cast<char *>(workspace);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    rc = launch_prep(a, L, ws, cmp_block_table, cmp_indices, q_prefix, act_q_len, act_kv_len, s);
    if (rc) return rc;
    const size_t T = (size_t)a.num_tokens;
    if (T && check_cuda(cudaMemcpyAsync(token_info, ws + L.token_info, sizeof(int32_t) * sas::TI_INTS * T,
                                        cudaMemcpyDeviceToDevice, s)))
        return SAS_ERR_CUDA;
    if (T && L.row_cap > 0 && cmp_rows &&
        check_cuda(cudaMemcpyAsync(cmp_rows, ws + L.cmp_rows, sizeof(int32_t) * (size_t)L.row_cap * T,
                                   cudaMemcpyDeviceToDevice, s)))
        return SAS_ERR_CUDA;
    return SAS_OK;
}

int sas_split_plan(const SasFwdArgs *args, int32_t *pieces, int32_t *tiles_per_piece) {
    if (!args || !pieces || !tiles_per_piece) return SAS_ERR_INVALID_ARG;
    const int rc = validate_fwd(*args);
    if (rc) return rc;
    if (use_tc(*args)) {
        tc_split_shape(*args, pieces, tiles_per_piece);
    } else {
        *pieces = 1;
        *tiles_per_piece = 0;
    }
    return SAS_OK;
}

int sas_split_metadata(const SasFwdArgs *args, const int32_t *ori_block_table, const int32_t *cmp_block_table,
                       const int32_t *cmp_indices, const int32_t *q_prefix, const int32_t *act_q_len,
                       const int32_t *act_kv_len, int32_t *metadata_out, void *workspace, size_t workspace_bytes,
                       void *stream) {
    if (!args || !metadata_out) return SAS_ERR_INVALID_ARG;
    const SasFwdArgs &a = *args;
    int rc = validate_fwd(a);
    if (rc) return rc;
    rc = check_inputs(a, ori_block_table, ori_block_table, cmp_block_table, cmp_block_table, cmp_indices, q_prefix,
                      act_q_len, act_kv_len);
    if (rc) return rc;
    const sas::FwdLayout L = fwd_layout(a);
    if (!workspace || workspace_bytes < L.total) return SAS_ERR_WORKSPACE;
    rc = check_alignment(nullptr, nullptr, ori_block_table, nullptr, cmp_block_table, cmp_indices, q_prefix,
                         act_q_len, act_kv_len, nullptr, nullptr, nullptr, workspace);
    if (rc || !aligned(metadata_out, 4)) return SAS_ERR_INVALID_ARG;
    char *ws = static_cast<char *>(workspace);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    rc = launch_prep(a, L, ws, cmp_block_table, cmp_indices, q_prefix, act_q_len, act_kv_len, s);
    if (rc) return rc;
    return launch_split_metadata(a, L, ws, use_tc(a), metadata_out, s);
}

int sas_read_status(const void *workspace, uint32_t *status, void *stream) {
    if (!workspace || !status) return SAS_ERR_INVALID_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (check_cuda(cudaMemcpyAsync(status, workspace, sizeof(uint32_t), cudaMemcpyDeviceToHost, s)))
        return SAS_ERR_CUDA;
    if (check_cuda(cudaStreamSynchronize(s))) return SAS_ERR_CUDA;
    return SAS_OK;
}

} // extern "C"
