// sas_forward_noalloc: sas_forward over a scratch array compiled into the
// library, for callers that cannot allocate device memory (see sas_b200.h).
//
// The array is a file-scope __device__ object.  In host code its name stands
// for a host-side shadow, not a device address, so the device address is looked
// up once per device with cudaGetSymbolAddress (with that device current) and
// cached; the kernels are then given that pointer like any workspace.

#include <mutex>

#include "sas_common.cuh"

namespace sas_host {
int launch_prep(const SasFwdArgs &a, const sas::FwdLayout &L, char *ws, const int32_t *cmp_bt, const int32_t *idx,
                const int32_t *q_prefix, const int32_t *act_q, const int32_t *act_kv, cudaStream_t s);
int launch_fwd_simt(const SasFwdArgs &a, const sas::FwdLayout &L, char *ws, const void *q, const void *ori_kv,
                    const int32_t *ori_bt, const void *cmp_kv, const float *sinks, void *out, float *lse,
                    cudaStream_t s);
bool tc_supported(const SasFwdArgs &a);
int launch_fwd_tc(const SasFwdArgs &a, const sas::FwdLayout &L, char *ws, const void *q, const void *ori_kv,
                  const int32_t *ori_bt, const void *cmp_kv, const float *sinks, void *out, float *lse,
                  cudaStream_t s);
} // namespace sas_host

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[SAS_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once per device).
int scratch_for_current_device(char **out) {
    int dev = 0;
    if (sas_host::check_cuda(cudaGetDevice(&dev))) return SAS_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return SAS_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        if (sas_host::check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch))) return SAS_ERR_CUDA;
        g_scratch_addr[dev] = p;
    }
    *out = static_cast<char *>(g_scratch_addr[dev]);
    return SAS_OK;
}

// The same pointer rule as sas_forward: 16-byte vectors and TMA tensor maps over q, the pools and
// out; per-element access to the int32 and fp32 arrays.  A misaligned pointer is an argument error.
bool misaligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) != 0; }

} // namespace

extern "C" int sas_forward_noalloc(const SasFwdArgs *args, const void *q, const void *ori_kv,
                                   const int32_t *ori_block_table, const void *cmp_kv,
                                   const int32_t *cmp_block_table, const int32_t *cmp_indices,
                                   const int32_t *q_prefix, const int32_t *act_q_len, const int32_t *act_kv_len,
                                   const float *sinks, const int32_t *metadata, void *out, float *lse, void *stream) {
    (void)metadata;
    if (!args) return SAS_ERR_INVALID_ARG;
    const SasFwdArgs &a = *args;
    int rc = sas_host::validate_fwd(a);
    if (rc) return rc;
    if (a.batch > 0 && (!q_prefix || (!act_q_len && !(a.flags & SAS_FWD_FLAG_CU_SEQLENS)) || !act_kv_len ||
                        !ori_block_table || !ori_kv))
        return SAS_ERR_INVALID_ARG;
    if (a.scenario >= 2 && (!cmp_kv || !cmp_block_table)) return SAS_ERR_INVALID_ARG;
    if (a.scenario == 3 && a.topk > 0 && a.num_tokens > 0 && !cmp_indices) return SAS_ERR_INVALID_ARG;
    if (a.num_tokens > 0 && (!q || !out || !sinks)) return SAS_ERR_INVALID_ARG;
    const sas::FwdLayout L = sas_host::fwd_layout(a);
    if (L.total > (size_t)SAS_NOALLOC_SCRATCH_BYTES) return SAS_ERR_WORKSPACE;
    for (const void *p : {q, ori_kv, cmp_kv, (const void *)out})
        if (misaligned(p, 16)) return SAS_ERR_INVALID_ARG;
    for (const void *p : {(const void *)ori_block_table, (const void *)cmp_block_table, (const void *)cmp_indices,
                          (const void *)q_prefix, (const void *)act_q_len, (const void *)act_kv_len,
                          (const void *)sinks, (const void *)lse})
        if (misaligned(p, 4)) return SAS_ERR_INVALID_ARG;
    char *ws = nullptr;
    if ((rc = scratch_for_current_device(&ws))) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // launch_prep clears the status word and the token records the kernels read
    rc = sas_host::launch_prep(a, L, ws, cmp_block_table, cmp_indices, q_prefix, act_q_len, act_kv_len, s);
    if (rc) return rc;
    if (a.kernel != SAS_KERNEL_SIMT && sas_host::tc_supported(a))
        return sas_host::launch_fwd_tc(a, L, ws, q, ori_kv, ori_block_table, cmp_kv, sinks, out, lse, s);
    return sas_host::launch_fwd_simt(a, L, ws, q, ori_kv, ori_block_table, cmp_kv, sinks, out, lse, s);
}
