// Key resolution: for every query token, its window bounds and the list of
// physical compressed rows it attends to.
//
// One warp per (request b, query s < act_q[b]); the flat token row is
// q_prefix[b] + s (kernel.py:421-474 decodes the same pair).  Semantics:
//   window      keys [max(s_g - win_left, 0), s_g], s_g = act_kv - act_q + s
//               (golden.py:125-131)
//   SCFA (3)    scan slots i < min(K, thr), thr = (act_kv - act_q + s + 1) // ratio;
//               the first -1 stops the scan, an index >= thr is skipped, duplicates
//               stay (golden.py:41-62).  An index < -1 is outside the contract: it
//               is skipped and SAS_STATUS_BAD_INDEX is raised.
//   CFA (2)     positions 0 .. thr-1 (golden.py:146-150)
//   SWA (1)     no compressed keys
// Each kept position p maps through the cmp block table to a physical row
// (table[b][p / bs] * bs + p % bs); an unmapped block gives -1, which the
// attention kernels read as a zero row, as unpack_paged_kv (golden.py:247-268)
// leaves unmapped blocks zero.

#include "sas_common.cuh"

namespace {

struct PrepArgs {
    int B, T, K, row_cap, scenario, ratio, win_left, win_right, max_q_len;
    int cmp_block_num, cmp_block_size, cmp_table_len;
    const int32_t *cmp_bt, *idx, *q_prefix, *act_q, *act_kv;
    int32_t *tinfo, *rows;
    uint32_t *status;
};

constexpr int kWarps = 8;

__device__ __forceinline__ int floordiv_i(int a, int b) {
    int q = a / b, r = a % b;
    return (r != 0 && ((r < 0) != (b < 0))) ? q - 1 : q;
}

__global__ void __launch_bounds__(kWarps * 32) prep_kernel(PrepArgs p) {
    const int lane = threadIdx.x & 31;
    const int s = blockIdx.x * kWarps + (threadIdx.x >> 5);
    const int b = blockIdx.y;
    if (b >= p.B) return;
    const int aq = __ldg(p.act_q + b);
    if (s == 0 && lane == 0 && aq > p.max_q_len) sas::set_status(p.status, SAS_STATUS_BAD_TOKEN);
    if (s >= aq) return;
    const int akv = __ldg(p.act_kv + b);
    const int64_t t = (int64_t)__ldg(p.q_prefix + b) + s;
    if (t < 0 || t >= p.T) {
        if (lane == 0) sas::set_status(p.status, SAS_STATUS_BAD_TOKEN);
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
        const int thr = floordiv_i(akv - aq + s + 1, p.ratio);
        if (p.scenario == 2) {
            if (thr > p.row_cap && lane == 0) sas::set_status(p.status, SAS_STATUS_BAD_TOKEN);
            const int n = min(max(thr, 0), p.row_cap);
            for (int i = lane; i < n; i += 32)
                rows[i] = (int32_t)sas::paged_row(p.cmp_bt, b, p.cmp_table_len, p.cmp_block_size, p.cmp_block_num,
                                                  i, p.status);
            n_cmp = n;
        } else {
            const int n_scan = min(p.K, thr);
            const int32_t *ir = p.idx + t * (int64_t)p.K;
            bool bad = false;
            for (int base = 0; base < n_scan; base += 32) {
                const int i = base + lane;
                const int v = i < n_scan ? __ldg(ir + i) : 0;
                const unsigned stop = __ballot_sync(0xffffffffu, i < n_scan && v == -1);
                const int stop_lane = stop ? __ffs(stop) - 1 : 32;
                const bool live = i < n_scan && lane < stop_lane;
                bad |= live && v < -1;
                const bool keep = live && v >= 0 && v < thr;
                const unsigned km = __ballot_sync(0xffffffffu, keep);
                if (keep) {
                    const int slot = n_cmp + __popc(km & ((1u << lane) - 1u));
                    rows[slot] = (int32_t)sas::paged_row(p.cmp_bt, b, p.cmp_table_len, p.cmp_block_size,
                                                         p.cmp_block_num, v, p.status);
                }
                n_cmp += __popc(km);
                if (stop) break;
            }
            if (__any_sync(0xffffffffu, bad) && lane == 0) sas::set_status(p.status, SAS_STATUS_BAD_INDEX);
        }
    }
    if (lane == 0) {
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
    if (check_cuda(cudaMemsetAsync(ws + L.status, 0, sas::kAlign, s))) return SAS_ERR_CUDA;
    if (a.num_tokens > 0 &&
        check_cuda(cudaMemsetAsync(ws + L.token_info, 0, sizeof(int32_t) * sas::TI_INTS * (size_t)a.num_tokens, s)))
        return SAS_ERR_CUDA;
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
    dim3 grid((a.max_q_len + kWarps - 1) / kWarps, a.batch);
    prep_kernel<<<grid, kWarps * 32, 0, s>>>(p);
    return check_cuda(cudaGetLastError());
}

} // namespace sas_host
