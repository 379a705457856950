// Shared definitions of the sas_b200 CUDA library (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "sas_b200.h"

namespace sas {

// Per-token record written by the key-resolution kernel (sas_prep.cu) and read
// by the attention kernels.  One record per flat token row, int32 each.
enum TokenInfo : int {
    TI_B = 0,       // request index b
    TI_SGLOBAL = 1, // s_global = act_kv - act_q + s (golden.py:125)
    TI_LEFT = 2,    // first window position max(s_global - win_left, 0) (golden.py:130)
    TI_NWIN = 3,    // window keys
    TI_NCMP = 4,    // resolved compressed keys (rows in the cmp row list)
    TI_VALID = 5,   // 1 if some (b, s < act_q[b]) maps to this row
    TI_S = 6,       // s, the query index inside its request
    TI_PAD = 7,
    TI_INTS = 8
};

constexpr size_t kAlign = 256;
// Byte offset, inside the status block, of the tensor-core kernel's token counter (cleared with
// the status word before every launch).
constexpr size_t kTokenCounterOff = 64;
inline size_t align_up(size_t x, size_t a = kAlign) { return (x + a - 1) / a * a; }

// Workspace layout of sas_forward / sas_resolve_rows.
struct FwdLayout {
    size_t status;     // uint32 status word (+ spare words)
    size_t token_info; // int32 [T][TI_INTS]
    size_t cmp_rows;   // int32 [T][row_cap]
    size_t tc;         // scratch of the tensor-core path
    size_t total;
    int64_t row_cap;
};

// Bounded spin used by every device-side wait: ~2^26 polls (well under a second
// of wall time at B200 clocks with the nanosleep back-off) before giving up.
constexpr uint32_t kSpinLimit = 1u << 26;

// Devices a process may drive (per-device launch attribute caches).
constexpr int kMaxDevices = 64;

// First-time set-up per device (kernel attributes belong to a device's context).  Each bit of
// `done` marks one finished step; `run` performs a step under a mutex the first time, so host
// threads that make their first calls at once neither race on the flags nor launch before the
// attribute is raised.  Steps are idempotent: after a context reset a repeat would be harmless.
struct DeviceOnce {
    std::atomic<uint32_t> done{0};
    std::mutex mu;
    template <typename F> int run(uint32_t bit, F &&step) {
        if (done.load(std::memory_order_acquire) & bit) return 0;
        std::lock_guard<std::mutex> lock(mu);
        if (done.load(std::memory_order_relaxed) & bit) return 0;
        const int rc = step();
        if (rc == 0) done.fetch_or(bit, std::memory_order_release);
        return rc;
    }
};

template <typename T> struct DT;
template <> struct DT<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
    static __device__ __forceinline__ float2 to_f2(uint32_t w) {
        __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162 *>(&w);
        return __bfloat1622float2(v);
    }
    static __device__ __forceinline__ float round_p(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
};
template <> struct DT<__half> {
    static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
    static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
    static __device__ __forceinline__ float2 to_f2(uint32_t w) {
        __half2 v = *reinterpret_cast<__half2 *>(&w);
        return __half22float2(v);
    }
    static __device__ __forceinline__ float round_p(float x) { return __half2float(__float2half_rn(x)); }
};

__device__ __forceinline__ void set_status(uint32_t *status, uint32_t bits) {
    if (status) atomicOr(status, bits);
}

// Physical row (block * block_size + offset) of logical `pos` of request `b`
// in a paged pool, or -1 when the block is unmapped / out of range.  Entries
// >= block_num and positions past the table raise SAS_STATUS_BAD_BLOCK.
__device__ __forceinline__ int64_t paged_row(const int32_t *__restrict__ table, int b, int table_len,
                                             int block_size, int block_num, int64_t pos, uint32_t *status) {
    int64_t blk = pos / block_size;
    if (pos < 0) return -1;
    if (blk >= table_len) {
        set_status(status, SAS_STATUS_BAD_BLOCK);
        return -1;
    }
    int32_t phys = __ldg(table + (int64_t)b * table_len + blk);
    if (phys < 0) {
        if (phys != -1) set_status(status, SAS_STATUS_BAD_BLOCK);
        return -1;
    }
    if (phys >= block_num) {
        set_status(status, SAS_STATUS_BAD_BLOCK);
        return -1;
    }
    return (int64_t)phys * block_size + (pos - blk * block_size);
}

} // namespace sas

// Host-side helpers shared by the launch code.
namespace sas_host {
int check_cuda(cudaError_t e);
sas::FwdLayout fwd_layout(const SasFwdArgs &a, bool cfa_rows = false);
int validate_fwd(const SasFwdArgs &a);
} // namespace sas_host
