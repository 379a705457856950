// sas_forward_noalloc: sas_forward over a scratch array compiled into the
// library, for callers that cannot allocate device memory (see sas_b200.h).
//
// The array is a file-scope __device__ object.  In host code its name stands
// for a host-side shadow, not a device address, so the device address is looked
// up with cudaGetSymbolAddress (with that device current) and cached; the
// kernels are then given that pointer like any workspace.  The address belongs
// to the module instance loaded in one CUDA context: the cache is keyed on the
// current context as well as the device ordinal, so after a cudaDeviceReset (or
// any new primary context) the next call looks the address up again instead of
// handing the kernels a pointer into freed memory.

#include <cuda.h>

#include <mutex>

#include "sas_common.cuh"

namespace sas_host {
int launch_prep(const SasFwdArgs &a, const sas::FwdLayout &L, char *ws, const int32_t *cmp_bt, const int32_t *idx,
                const int32_t *q_prefix, const int32_t *act_q, const int32_t *act_kv, cudaStream_t s);
int launch_fwd_simt(const SasFwdArgs &a, const sas::FwdLayout &L, char *ws, const void *q, const void *ori_kv,
                    const int32_t *ori_bt, const void *cmp_kv, const int32_t *cmp_bt, const float *sinks, void *out,
                    float *lse, cudaStream_t s);
bool tc_supported(const SasFwdArgs &a);
int launch_fwd_tc(const SasFwdArgs &a, const sas::FwdLayout &L, char *ws, const void *q, const void *ori_kv,
                  const int32_t *ori_bt, const void *cmp_kv, const int32_t *cmp_bt, const float *sinks, void *out,
                  float *lse, cudaStream_t s, bool pair);
} // namespace sas_host

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[SAS_NOALLOC_SCRATCH_BYTES];

struct ScratchSlot {
    CUcontext ctx;  // context the address was looked up in
    void *addr;
};
std::mutex g_mu;
ScratchSlot g_scratch[sas::kMaxDevices] = {};

typedef CUresult (*CtxGetCurrentFn)(CUcontext *);

CtxGetCurrentFn ctx_get_current() {
    static CtxGetCurrentFn fn = [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<CtxGetCurrentFn>(ptr);
        return static_cast<CtxGetCurrentFn>(nullptr);
    }();
    return fn;
}

// Device address of the scratch array in the current device's current context.  Looked up on the
// first call in a context and cached; the lookup allocates nothing (it may initialise the context,
// which is why the first call on a device belongs before any stream capture).
int scratch_for_current_device(char **out) {
    int dev = 0;
    if (sas_host::check_cuda(cudaGetDevice(&dev))) return SAS_ERR_CUDA;
    if (dev < 0 || dev >= sas::kMaxDevices) return SAS_ERR_UNSUPPORTED;
    CtxGetCurrentFn get = ctx_get_current();
    if (!get) return SAS_ERR_CUDA;
    // NULL before the runtime's first use of the device on this thread: the lookup below binds it
    CUcontext ctx = nullptr;
    if (get(&ctx) != CUDA_SUCCESS) return SAS_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_mu);
    ScratchSlot &slot = g_scratch[dev];
    if (!ctx || !slot.addr || slot.ctx != ctx) {
        void *p = nullptr;
        if (sas_host::check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch))) return SAS_ERR_CUDA;
        if (get(&ctx) != CUDA_SUCCESS || !ctx) return SAS_ERR_CUDA;
        slot.ctx = ctx;
        slot.addr = p;
    }
    *out = static_cast<char *>(slot.addr);
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
        return sas_host::launch_fwd_tc(a, L, ws, q, ori_kv, ori_block_table, cmp_kv, cmp_block_table, sinks, out, lse, s,
                                     a.kernel == SAS_KERNEL_TC2);
    return sas_host::launch_fwd_simt(a, L, ws, q, ori_kv, ori_block_table, cmp_kv, cmp_block_table, sinks, out, lse, s);
}

extern "C" int sas_noalloc_read_status(uint32_t *status, void *stream) {
    if (!status) return SAS_ERR_INVALID_ARG;
    char *ws = nullptr;
    int rc = scratch_for_current_device(&ws);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // the status word is the first word of the workspace layout (sas_forward's as well)
    uint32_t word = 0;
    if (sas_host::check_cuda(cudaMemcpyAsync(&word, ws, sizeof(uint32_t), cudaMemcpyDeviceToHost, s)))
        return SAS_ERR_CUDA;
    if (sas_host::check_cuda(cudaStreamSynchronize(s))) return SAS_ERR_CUDA;
    *status = word;
    return SAS_OK;
}
