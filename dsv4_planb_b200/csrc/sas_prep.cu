// Key resolution: for every query token, its window bounds and the list of
// physical compressed rows it attends to.
//
// One CTA per (request b, query s < act_q[b]); the flat token row is
// q_prefix[b] + s (kernel.py:421-474 decodes the same pair).  Semantics:
//   window      keys [max(s_g - win_left, 0), s_g], s_g = act_kv - act_q + s
//               (golden.py:125-131)
//   SCFA (3)    scan slots i < min(K, thr), thr = (act_kv - act_q + s + 1) // ratio;
//               the first -1 stops the scan, an index >= thr is skipped, duplicates
//               stay (golden.py:41-62).  An index < -1 is outside the contract: it
//               is skipped and SAS_STATUS_BAD_INDEX is raised.
//   CFA (2)     positions 0 .. thr-1 (golden.py:146-150): only the count is recorded;
//               the attention kernels map the positions through the table themselves
//               (the rows are written only for the sas_resolve_rows export)
//   SWA (1)     no compressed keys
// Each kept position p maps through the cmp block table to a physical row
// (table[b][p / bs] * bs + p % bs); an unmapped block gives -1, which the
// attention kernels read as a zero row, as unpack_paged_kv (golden.py:247-268)
// leaves unmapped blocks zero.
//
// The scan is data-parallel: each thread holds kPer consecutive slots, the
// stop position is a block-wide minimum and the compaction a block-wide
// exclusive prefix sum, so the kept rows keep their slot order.

#include "sas_common.cuh"

namespace {

struct PrepArgs {
    int B, T, K, row_cap, scenario, ratio, win_left, win_right, max_q_len;
    int cu;  // q_prefix is cu_seqlens_q [B + 1]; act_q is derived from it
    int cmp_block_num, cmp_block_size, cmp_table_len;
    const int32_t *cmp_bt, *idx, *q_prefix, *act_q, *act_kv;
    int32_t *tinfo, *rows;
    uint32_t *status;
};

constexpr int kThreads = 256;
constexpr int kTableSmem = 2048;  // block-table entries staged in shared memory

__device__ __forceinline__ int floordiv_i(int a, int b) {
    int q = a / b, r = a % b;
    return (r != 0 && ((r < 0) != (b < 0))) ? q - 1 : q;
}

// Physical row of compressed position v of request b (table staged in smem when it fits).
__device__ __forceinline__ int32_t cmp_row(const PrepArgs &p, const int32_t *tab_s, int b, int v) {
    const int blk = v / p.cmp_block_size;
    if (blk >= p.cmp_table_len) {
        sas::set_status(p.status, SAS_STATUS_BAD_BLOCK);
        return -1;
    }
    const int32_t phys = tab_s ? tab_s[blk] : __ldg(p.cmp_bt + (int64_t)b * p.cmp_table_len + blk);
    if (phys < 0) {
        if (phys != -1) sas::set_status(p.status, SAS_STATUS_BAD_BLOCK);
        return -1;
    }
    if (phys >= p.cmp_block_num) {
        sas::set_status(p.status, SAS_STATUS_BAD_BLOCK);
        return -1;
    }
    return phys * p.cmp_block_size + (v - blk * p.cmp_block_size);
}

// Block-wide exclusive prefix sum of `v` (also returns the total).
__device__ __forceinline__ int block_exscan(int v, int *total, int *warp_sums) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < kThreads / 32 ? warp_sums[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < kThreads / 32) warp_sums[lane] = w;  // inclusive per-warp totals
    }
    __syncthreads();
    const int before = (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
    *total = warp_sums[kThreads / 32 - 1];
    __syncthreads();
    return before;
}

// Zeroes the status word and the token records (n16 16-byte words), then lets the prep grid launch.
__global__ void __launch_bounds__(kThreads) clear_kernel(uint4 *words, int64_t n16) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n16; i += (int64_t)gridDim.x * kThreads)
        words[i] = make_uint4(0, 0, 0, 0);
}

template <int kPer>
__global__ void __launch_bounds__(kThreads, 1) prep_kernel(PrepArgs p) {
    __shared__ int32_t tab_s[kTableSmem];
    __shared__ int warp_sums[kThreads / 32];
    __shared__ int s_stop;
    __shared__ int s_bad;
    // the attention kernel is launched as a programmatic dependent of this one: let it start its
    // prologue now (it waits for this grid's completion before reading the records)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int s = blockIdx.x;
    const int b = blockIdx.y;
    const int tid = threadIdx.x;
    if (b >= p.B) return;
    // Everything that depends on the request alone is loaded in one round trip (these reads miss
    // L2 after a flush; the indices, which need the token row, form the second and last round).
    const int q0 = __ldg(p.q_prefix + b);
    const int aq = p.cu ? __ldg(p.q_prefix + b + 1) - q0 : __ldg(p.act_q + b);
    const int akv = __ldg(p.act_kv + b);
    const bool staged = (p.scenario == 3 || (p.scenario == 2 && p.row_cap > 0)) && p.cmp_table_len <= kTableSmem;
    int32_t tabv[kTableSmem / kThreads];
#pragma unroll
    for (int k = 0; k < kTableSmem / kThreads; ++k) {
        const int i = tid + k * kThreads;
        tabv[k] = staged && i < p.cmp_table_len ? __ldg(p.cmp_bt + (int64_t)b * p.cmp_table_len + i) : 0;
    }
    // launched as a programmatic dependent of clear_kernel: the status word and the token records
    // are zero after this wait (the request-level loads above already overlap the clear)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (s == 0 && tid == 0 && aq > p.max_q_len) sas::set_status(p.status, SAS_STATUS_BAD_TOKEN);
    if (s >= aq) return;
    const int64_t t = (int64_t)q0 + s;
    if (t < 0 || t >= p.T) {
        if (tid == 0) sas::set_status(p.status, SAS_STATUS_BAD_TOKEN);
        return;
    }
    const int s_g = akv - aq + s;
    int left = 0, n_win = 0;
    if (s_g >= 0) {
        left = max(s_g - p.win_left, 0);
        n_win = s_g + p.win_right + 1 - left;
    }
    int n_cmp = 0;
    int32_t *rows = p.rows + t * (int64_t)p.row_cap;
    if (p.scenario >= 2) {
        if (staged) {
#pragma unroll
            for (int k = 0; k < kTableSmem / kThreads; ++k) {
                const int i = tid + k * kThreads;
                if (i < p.cmp_table_len) tab_s[i] = tabv[k];
            }
        }
        if (tid == 0) {
            s_stop = 0x7fffffff;
            s_bad = 0;
        }
        __syncthreads();
        const int32_t *tab = staged ? tab_s : nullptr;
        const int thr = floordiv_i(akv - aq + s + 1, p.ratio);
        if (p.scenario == 2) {
            n_cmp = max(thr, 0);
            if (p.row_cap > 0) {  // the export: as many rows as the caller's max_cmp_len holds
                if (thr > p.row_cap && tid == 0) sas::set_status(p.status, SAS_STATUS_BAD_TOKEN);
                for (int i = tid; i < min(n_cmp, p.row_cap); i += kThreads) rows[i] = cmp_row(p, tab, b, i);
            }
        } else {
            const int n_scan = min(p.K, thr);
            const int32_t *ir = p.idx + t * (int64_t)p.K;
            // process the scan window in chunks of kThreads * kPer slots
            for (int base = 0; base < n_scan; base += kThreads * kPer) {
                int v[kPer];
                const int i0 = base + tid * kPer;
                int first_stop = 0x7fffffff;
#pragma unroll
                for (int k = 0; k < kPer; ++k) {
                    v[k] = i0 + k < n_scan ? __ldg(ir + i0 + k) : 0;
                    if (i0 + k < n_scan && v[k] == -1 && first_stop == 0x7fffffff) first_stop = i0 + k;
                }
                if (first_stop != 0x7fffffff) atomicMin(&s_stop, first_stop);
                __syncthreads();
                const int stop = min(s_stop, n_scan);
                int cnt = 0;
                bool bad = false;
#pragma unroll
                for (int k = 0; k < kPer; ++k) {
                    const bool live = i0 + k < stop;
                    bad |= live && v[k] < -1;
                    cnt += (live && v[k] >= 0 && v[k] < thr) ? 1 : 0;
                }
                if (bad) s_bad = 1;
                int total;
                int pos = n_cmp + block_exscan(cnt, &total, warp_sums);
#pragma unroll
                for (int k = 0; k < kPer; ++k) {
                    if (i0 + k < stop && v[k] >= 0 && v[k] < thr) rows[pos++] = cmp_row(p, tab, b, v[k]);
                }
                n_cmp += total;
                if (stop < n_scan) break;  // uniform: s_stop is shared
            }
            __syncthreads();
            if (tid == 0 && s_bad) sas::set_status(p.status, SAS_STATUS_BAD_INDEX);
        }
    }
    if (tid == 0) {
        int32_t *ti = p.tinfo + t * sas::TI_INTS;
        ti[sas::TI_B] = b;
        ti[sas::TI_SGLOBAL] = s_g;
        ti[sas::TI_LEFT] = left;
        ti[sas::TI_NWIN] = n_win;
        ti[sas::TI_NCMP] = n_cmp;
        ti[sas::TI_VALID] = 1;
        ti[sas::TI_S] = s;
        ti[sas::TI_PAD] = 0;
    }
}

} // namespace

namespace sas_host {

// Zero the status word and the token records, then resolve every token.
int launch_prep(const SasFwdArgs &a, const sas::FwdLayout &L, char *ws, const int32_t *cmp_bt, const int32_t *idx,
                const int32_t *q_prefix, const int32_t *act_q, const int32_t *act_kv, cudaStream_t s) {
    const bool cu = (a.flags & SAS_FWD_FLAG_CU_SEQLENS) != 0;
    // the status word and the token records are adjacent: one kernel clears both, and prep follows
    // it as a programmatic dependent (its launch and first loads overlap the clear)
    static_assert(sizeof(int32_t) * sas::TI_INTS % 16 == 0, "token record size");
    const size_t clear = L.token_info + sizeof(int32_t) * sas::TI_INTS * (size_t)(a.num_tokens > 0 ? a.num_tokens : 0);
    const int64_t n16 = (int64_t)((clear - L.status) / 16);
    const int cblocks = (int)std::min<int64_t>((n16 + kThreads - 1) / kThreads, 148);
    clear_kernel<<<cblocks, kThreads, 0, s>>>(reinterpret_cast<uint4 *>(ws + L.status), n16);
    if (check_cuda(cudaGetLastError())) return SAS_ERR_CUDA;
    if (a.batch == 0 || a.max_q_len == 0 || a.num_tokens == 0) return SAS_OK;
    PrepArgs p;
    p.B = a.batch;
    p.T = a.num_tokens;
    p.K = a.topk;
    p.row_cap = (int)L.row_cap;
    p.scenario = a.scenario;
    p.ratio = a.cmp_ratio;
    p.win_left = a.ori_win_left;
    p.win_right = a.ori_win_right;
    p.max_q_len = a.max_q_len;
    p.cu = cu ? 1 : 0;
    p.cmp_block_num = a.cmp_block_num;
    p.cmp_block_size = a.cmp_block_size;
    p.cmp_table_len = a.cmp_table_len;
    p.cmp_bt = cmp_bt;
    p.idx = idx;
    p.q_prefix = q_prefix;
    p.act_q = act_q;
    p.act_kv = act_kv;
    p.tinfo = reinterpret_cast<int32_t *>(ws + L.token_info);
    p.rows = reinterpret_cast<int32_t *>(ws + L.cmp_rows);
    p.status = reinterpret_cast<uint32_t *>(ws + L.status);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.max_q_len, a.batch, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = (a.scenario == 3 && a.topk > kThreads * 4) ? cudaLaunchKernelEx(&cfg, prep_kernel<8>, p)
                                                                      : cudaLaunchKernelEx(&cfg, prep_kernel<4>, p);
    return check_cuda(e);
}

} // namespace sas_host
