// CUDA port of the reference metadata tile scheduler.
//
// Reproduces sparse_attn_sharedkv_metadata (metadata.py:1018-1086 of
// yangqiang2018/dsv4_planB, itself the Python port of the Ascend aicpu
// SparseAttnSharedkvMetadata op) bit for bit.  One CTA:
//   phase 0  per-request sizes, row counts and the all-zero test (parallel over b)
//   phase 1  the cost of every (request, row) -- metadata.py:634-714 -- in
//            parallel over the flattened rows, summed per request with
//            atomics; each row's {cost, last block cost, blocks, s2 start} is
//            kept in a table so the sequential phase reads it back
//   phase 2  the greedy assignment of metadata.py:718-923, one thread (it is
//            inherently sequential: each core's limit depends on what the
//            previous cores took)
//   phase 3  packing into int32[1024] (metadata.py:974-1009)
// Python integer semantics: the pre/next-token sums can involve INT64_MAX, so
// they are evaluated in __int128, and // and % follow Python's floor rules.
// supportFd is False in the reference and never flipped: the block-level
// reassignment and FD bookkeeping (metadata.py:777-827, 925-954) cannot run,
// and the FD rows and first-FD-workspace fields stay zero.

#include <stdint.h>

#include "sas_common.cuh"

namespace {

constexpr int kMetaSize = 1024;
constexpr int kAicRows = 36;
constexpr int kFaInts = 8;
constexpr int64_t kS2Base = 512;
constexpr int kThreads = 1024;

typedef __int128 i128;

__device__ __forceinline__ int64_t fdiv(int64_t a, int64_t b) {
    int64_t q = a / b, r = a % b;
    return (r != 0 && ((r < 0) != (b < 0))) ? q - 1 : q;
}
__device__ __forceinline__ int64_t fmod_py(int64_t a, int64_t b) {
    int64_t r = a % b;
    return (r != 0 && ((r < 0) != (b < 0))) ? r + b : r;
}
__device__ __forceinline__ i128 fdiv128(i128 a, i128 b) {
    i128 q = a / b, r = a % b;
    return (r != 0 && ((r < 0) != (b < 0))) ? q - 1 : q;
}
__device__ __forceinline__ i128 fmod128(i128 a, i128 b) {
    i128 r = a % b;
    return (r != 0 && ((r < 0) != (b < 0))) ? r + b : r;
}

struct MetaIn {
    SasMetaArgs a;
    const int32_t *cu_q, *cu_kv, *seq_q, *seq_kv;
    int32_t *out;
    // workspace carve-up
    uint32_t *status;
    int64_t *s1, *s2, *base, *tail, *prefix;              // [B] / [B+1]
    unsigned long long *bcost, *bblock, *blast;           // [B]
    int64_t *row_cost, *row_last, *row_block, *row_s2s;   // [row_cap]
    int64_t row_cap;
    int64_t bufB;                                          // capacity of the [B] arrays
};

// Everything phase 2 needs about one (request, row): the fields of S1GCache
// that metadata.py:718-923 reads.
struct RowR {
    int64_t cost, last_cost, block, s2_start;
};

struct Params {
    int64_t B, G, m_base, pre_token, next_token;
    int attn_mode, is_s1g, is_cfa, is_scfa;
};

struct Batch {
    int64_t b, s1, s2;
    i128 pre_lu, next_lu;
};

__device__ int64_t q_len(const MetaIn &m, int64_t b, uint32_t &err) {
    const SasMetaArgs &a = m.a;
    if (a.n_seqused_q > 0) {
        if (b < 0 || b >= a.n_seqused_q) { err |= 1; return 0; }
        return m.seq_q[b];
    }
    if (a.layout_q == SAS_LAYOUT_TND && a.n_cu_seqlens_q > 0) {
        if (b < 0 || b + 1 >= a.n_cu_seqlens_q) { err |= 1; return 0; }
        return (int64_t)m.cu_q[b + 1] - m.cu_q[b];
    }
    return a.max_seqlen_q;
}

__device__ int64_t kv_len(const MetaIn &m, int64_t b, uint32_t &err) {
    const SasMetaArgs &a = m.a;
    if (a.n_seqused_kv > 0) {
        if (b < 0 || b >= a.n_seqused_kv) { err |= 1; return 0; }
        return m.seq_kv[b];
    }
    if (a.layout_kv == SAS_LAYOUT_KV_TND && a.n_cu_seqlens_ori_kv > 0) {
        if (b < 0 || b + 1 >= a.n_cu_seqlens_ori_kv) { err |= 1; return 0; }
        return (int64_t)m.cu_kv[b + 1] - m.cu_kv[b];
    }
    return a.max_seqlen_kv;
}

// metadata.py:409-426
__device__ Batch make_batch(const MetaIn &m, const Params &p, int64_t b) {
    Batch r;
    r.b = b;
    r.s1 = m.s1[b];
    r.s2 = m.s2[b];
    const int mode = m.a.ori_mask_mode;
    r.pre_lu = mode == 4 ? (i128)r.s1 - r.s2 + p.pre_token : (i128)p.pre_token;
    if (mode == 0 || mode == 1 || mode == 2) r.next_lu = p.next_token;
    else if (mode == 3) r.next_lu = (i128)r.s2 - r.s1;
    else if (mode == 4) r.next_lu = (i128)r.s2 - r.s1 + p.next_token;
    else r.next_lu = p.next_token;
    return r;
}

// metadata.py:428-438
__device__ __forceinline__ int64_t block_cost(int64_t m, int64_t s2) {
    return 6 * ((m + 15) >> 4) + 10 * ((s2 + 63) >> 6);
}

// One row's cost fields: metadata.py:479-501, 512-547, 440-477, 549-632, 623-667.
__device__ RowR eval_row(const MetaIn &m, const Params &p, const Batch &bc, int64_t idx) {
    RowR r{0, 0, 0, 0};
    const int64_t base = m.base[bc.b];
    if (base == 0) return r;  // metadata.py:642-653
    // --- s2 token range, metadata.py:479-501
    i128 f, l;
    if (bc.s1 == 0 || bc.s2 == 0) {
        f = 0; l = 0;
    } else if (!p.attn_mode) {
        f = 0; l = (i128)bc.s2 - 1;
    } else {
        int64_t g_first = idx * p.m_base;
        int64_t g_last = min(g_first + p.m_base, bc.s1 * p.G) - 1;
        int64_t s1f, s1l;
        if (p.is_s1g) {
            s1f = fdiv(g_first, p.G);
            s1l = fdiv(g_last, p.G);
        } else if (fdiv(g_first, bc.s1) == fdiv(g_last, bc.s1)) {
            s1f = fmod_py(g_first, bc.s1);
            s1l = fmod_py(g_last, bc.s1);
        } else {
            s1f = 0;
            s1l = bc.s1;
        }
        f = (i128)s1f - bc.pre_lu;
        l = (i128)s1l + bc.next_lu;
    }
    // --- block range and tails, metadata.py:512-547
    int64_t win_end, win_tail;
    if (f >= bc.s2 || l < 0 || l < f) {
        f = 0; l = 0; win_end = 0; win_tail = 0;
    } else {
        const i128 hi = (i128)bc.s2 - 1;
        f = f < hi ? f : hi; f = f > 0 ? f : 0;
        l = l < hi ? l : hi; l = l > 0 ? l : 0;
        win_end = (int64_t)fdiv128(l - f, kS2Base) + 1;
        win_tail = (int64_t)fmod128(l - f + 1, kS2Base);
    }
    const int64_t cmp_start = win_end;
    int64_t cmp_last = 0;
    if (m.a.has_cmp_kv && m.a.cmp_ratio > 0) cmp_last = (int64_t)fdiv128(l + 1, m.a.cmp_ratio);
    int64_t act = 0;
    if (p.is_cfa) act = cmp_last;
    else if (p.is_scfa) act = min(cmp_last, (int64_t)m.a.cmp_topk);
    const int64_t cmp_end = act == 0 ? cmp_start : cmp_start + fdiv(act - 1, kS2Base) + 1;
    const int64_t cmp_tail = fmod_py(act, kS2Base);
    // --- per-type block costs, metadata.py:440-477 (row type: normal or tail)
    const int64_t s1t = m.tail[bc.b];
    const bool tail_row = (idx == base - 1) && s1t != 0;
    const int64_t c_nn = block_cost(p.m_base, kS2Base);
    const int64_t c_tn = s1t == 0 ? 0 : block_cost(s1t, kS2Base);
    // --- window part, metadata.py:549-584
    int64_t win_block = 0, win_cost = 0, win_last = 0;
    if (0 < win_end) {
        const int64_t c_nt = win_tail == 0 ? 0 : block_cost(p.m_base, win_tail);
        const int64_t c_tt = (s1t == 0 || win_tail == 0) ? 0 : block_cost(s1t, win_tail);
        win_block = win_end;
        const int64_t t = win_tail != 0, n = win_block - t;
        if (tail_row) {
            win_cost = c_tn * n + c_tt * t;
            win_last = t > 0 ? c_tt : c_tn;
        } else {
            win_cost = c_nn * n + c_nt * t;
            win_last = t > 0 ? c_nt : c_nn;
        }
    }
    // --- compressed part, metadata.py:586-621
    int64_t cmp_block = 0, cmp_cost = 0, cmp_lastc = 0;
    if (cmp_start < cmp_end) {
        // the CMP cost entries are only written when has_cmp_kv (metadata.py:463);
        // with no cmp pool act is 0, so this branch is not reached then.
        const int64_t c_nt = cmp_tail == 0 ? 0 : block_cost(p.m_base, cmp_tail);
        const int64_t c_tt = (s1t == 0 || cmp_tail == 0) ? 0 : block_cost(s1t, cmp_tail);
        cmp_block = cmp_end - cmp_start;
        const int64_t t = cmp_tail != 0, n = cmp_block - t;
        if (tail_row) {
            cmp_cost = c_tn * n + c_tt * t;
            cmp_lastc = t > 0 ? c_tt : c_tn;
        } else {
            cmp_cost = c_nn * n + c_nt * t;
            cmp_lastc = t > 0 ? c_nt : c_nn;
        }
    }
    // --- merge, metadata.py:623-632
    r.s2_start = win_block > 0 ? 0 : cmp_start;
    r.last_cost = cmp_block > 0 ? cmp_lastc : win_last;
    r.block = win_block + cmp_block;
    r.cost = win_cost + cmp_cost;
    return r;
}

__device__ __forceinline__ RowR get_row(const MetaIn &m, const Params &p, const Batch &bc, int64_t idx, bool table) {
    if (table && idx >= 0 && idx < m.base[bc.b]) {
        const int64_t k = m.prefix[bc.b] + idx;
        return RowR{m.row_cost[k], m.row_last[k], m.row_block[k], m.row_s2s[k]};
    }
    return eval_row(m, p, bc, idx);
}

__global__ void __launch_bounds__(kThreads, 1) metadata_kernel(MetaIn m) {
    __shared__ Params sp;
    __shared__ int64_t s_total_rows;
    __shared__ int s_all_zero;
    __shared__ uint32_t s_err;
    __shared__ unsigned long long s_max_cost;
    const int tid = threadIdx.x;
    const SasMetaArgs &a = m.a;

    for (int i = tid; i < kMetaSize; i += blockDim.x) m.out[i] = 0;
    if (tid == 0) {
        Params p;
        if (a.n_seqused_q > 0) p.B = a.n_seqused_q;
        else if (a.layout_q == SAS_LAYOUT_TND && a.n_cu_seqlens_q > 0) p.B = a.n_cu_seqlens_q - 1;
        else p.B = a.batch_size;
        if (a.ori_mask_mode == 0) { p.pre_token = INT64_MAX; p.next_token = INT64_MAX; p.attn_mode = 0; }
        else if (a.ori_mask_mode == 3) { p.pre_token = INT64_MAX; p.next_token = 0; p.attn_mode = 1; }
        else { p.pre_token = a.ori_win_left > -1 ? (int64_t)a.ori_win_left : INT64_MAX; p.next_token = 0; p.attn_mode = 1; }
        p.is_s1g = a.layout_q == SAS_LAYOUT_BSND || a.layout_q == SAS_LAYOUT_BSH || a.layout_q == SAS_LAYOUT_TND;
        p.G = a.num_heads_q / a.num_heads_kv;
        p.is_scfa = a.has_cmp_kv && a.cmp_topk > 0;
        p.is_cfa = a.has_cmp_kv && !(a.cmp_topk > 0);
        p.m_base = p.G;
        sp = p;
        s_all_zero = 1;
        s_err = 0;
        s_max_cost = 0;
    }
    __syncthreads();
    const Params p = sp;
    if (p.B > m.bufB || p.B < 0) {
        if (tid == 0) sas::set_status(m.status, SAS_STATUS_NO_PROGRESS);
        return;
    }

    // ---- phase 0: sizes, split info (metadata.py:671-683)
    uint32_t err = 0;
    for (int64_t b = tid; b < p.B; b += blockDim.x) {
        const int64_t s1 = q_len(m, b, err), s2 = kv_len(m, b, err);
        m.s1[b] = s1;
        m.s2[b] = s2;
        m.base[b] = fdiv(s1 * p.G + p.m_base - 1, p.m_base);
        m.tail[b] = fmod_py(s1 * p.G, p.m_base);
        const int64_t s2_base = fdiv(s2 + kS2Base - 1, kS2Base);
        if (m.base[b] != 0 && s2_base != 0) s_all_zero = 0;
        m.bcost[b] = 0;
        m.bblock[b] = 0;
        m.blast[b] = 0;
    }
    if (err) atomicOr(&s_err, err);
    __syncthreads();
    if (s_err) {
        if (tid == 0) sas::set_status(m.status, SAS_STATUS_NO_PROGRESS);
        return;
    }
    if (tid == 0) {
        int64_t acc = 0;
        for (int64_t b = 0; b < p.B; ++b) {
            m.prefix[b] = acc;
            acc += m.base[b] > 0 ? m.base[b] : 0;
        }
        m.prefix[p.B] = acc;
        s_total_rows = acc;
    }
    __syncthreads();
    const int64_t total_rows = s_total_rows;
    const bool table = total_rows <= m.row_cap;

    if (!s_all_zero) {
        // ---- phase 1: row costs (metadata.py:685-714)
        for (int64_t r = tid; r < total_rows; r += blockDim.x) {
            int64_t lo = 0, hi = p.B;  // find b with prefix[b] <= r < prefix[b+1]
            while (hi - lo > 1) {
                const int64_t mid = (lo + hi) >> 1;
                if (m.prefix[mid] <= r) lo = mid; else hi = mid;
            }
            const int64_t b = lo, idx = r - m.prefix[b];
            const Batch bc = make_batch(m, p, b);
            const RowR row = eval_row(m, p, bc, idx);
            if (table) {
                m.row_cost[r] = row.cost;
                m.row_last[r] = row.last_cost;
                m.row_block[r] = row.block;
                m.row_s2s[r] = row.s2_start;
            }
            if (bc.s1 == 0 || bc.s2 == 0) continue;  // metadata.py:690-691
            atomicAdd(&m.bcost[b], (unsigned long long)row.cost);
            atomicAdd(&m.bblock[b], (unsigned long long)row.block);
            atomicMax(&s_max_cost, (unsigned long long)row.cost);
            if (row.block > 0) atomicMax(&m.blast[b], ((unsigned long long)(idx + 1) << 32) | (uint32_t)row.last_cost);
        }
        __syncthreads();
    }
    if (tid != 0) return;

    // ---- phase 2: greedy assignment (metadata.py:718-923), one thread
    const int64_t N2 = a.num_heads_kv;
    const int64_t aic = a.aic_core_num;
    int64_t used = 0;
    int64_t bn2_end[kAicRows], g_s1_end[kAicRows], s2_end[kAicRows];
    for (int i = 0; i < kAicRows; ++i) bn2_end[i] = g_s1_end[i] = s2_end[i] = 0;

    if (s_all_zero) {
        if (aic <= 0) { sas::set_status(m.status, SAS_STATUS_NO_PROGRESS); return; }
        used = 1;
        bn2_end[0] = p.B * N2;
    } else {
        int64_t total_cost = 0;
        for (int64_t b = 0; b < p.B; ++b) total_cost += (int64_t)m.bcost[b] * N2;
        const int64_t max_row_cost = (int64_t)s_max_cost;
        if (aic > 0) {
            int64_t cur_b = 0, cur_bn2 = 0, cur_s1g = 0, cur_s2 = 0, cur_core = 0;
            int64_t unassigned = total_cost;
            int64_t bn2_cost = (int64_t)m.bcost[0], bn2_block = (int64_t)m.bblock[0];
            bool finished = false;
            Batch bc = make_batch(m, p, 0);
            RowR rc = get_row(m, p, bc, 0, table);
            cur_s2 = rc.s2_start;
            for (int64_t i = 0; i < aic; ++i) {
                if (finished || unassigned <= 0) break;
                cur_core = i;
                const int64_t avg = fdiv(unassigned, max((int64_t)1, aic - cur_core));
                int64_t core_cost = 0, core_block = 0;
                const int64_t limit = max(avg, max_row_cost);
                // _assign_by_batch, metadata.py:718-745
                if (!finished) {
                    while (bn2_cost == 0 ||
                           limit + fdiv((int64_t)(m.blast[cur_b] & 0xffffffffull), 2) >= core_cost + bn2_cost) {
                        core_cost += bn2_cost;
                        core_block += bn2_block;
                        cur_bn2 += 1;
                        if (cur_bn2 == p.B * N2) {
                            cur_s1g = 0;
                            cur_s2 = 0;
                            finished = true;
                            break;
                        }
                        if (fdiv(cur_bn2, N2) != cur_b) {
                            cur_b = fdiv(cur_bn2, N2);
                            bc = make_batch(m, p, cur_b);
                        }
                        bn2_cost = (int64_t)m.bcost[cur_b];
                        bn2_block = (int64_t)m.bblock[cur_b];
                        cur_s1g = 0;
                        rc = get_row(m, p, bc, 0, table);
                        cur_s2 = rc.s2_start;
                    }
                }
                // _assign_by_row, metadata.py:747-764
                if (!finished) {
                    while (limit + fdiv(rc.last_cost, 2) >= core_cost + rc.cost) {
                        core_cost += rc.cost;
                        core_block += rc.block;
                        bn2_cost = max((int64_t)0, bn2_cost - rc.cost);
                        bn2_block = max((int64_t)0, bn2_block - rc.block);
                        // Advance to the next row with blocks.  The reference spins
                        // forever if there is none; every row past this cap is empty.
                        const int64_t cap = m.base[bc.b] + (a.ori_win_left < 0 ? -(int64_t)a.ori_win_left
                                                                                : (int64_t)a.ori_win_left) +
                                            (bc.s2 < 0 ? -bc.s2 : bc.s2) + 64;
                        for (;;) {
                            cur_s1g += 1;
                            rc = get_row(m, p, bc, cur_s1g, table);
                            if (rc.block != 0) break;
                            if (cur_s1g > cap) {
                                sas::set_status(m.status, SAS_STATUS_NO_PROGRESS);
                                return;
                            }
                        }
                        cur_s2 = rc.s2_start;
                    }
                }
                if (i < kAicRows) {
                    bn2_end[i] = cur_bn2;
                    g_s1_end[i] = cur_s1g;
                    s2_end[i] = cur_s2;
                }
                unassigned -= core_cost;
                (void)core_block;
            }
            used = cur_core + 1;
        }
        if (used < 1) used = 1;
    }

    // ---- phase 3: packing (metadata.py:974-1009)
    for (int64_t i = 0; i < kAicRows; ++i) {
        if (i >= used || i >= aic) continue;
        int32_t *row = m.out + i * kFaInts;
        row[0] = 1;
        row[1] = (int32_t)(i == 0 ? 0 : bn2_end[i - 1]);
        row[2] = (int32_t)(i == 0 ? 0 : g_s1_end[i - 1]);
        row[3] = (int32_t)(i == 0 ? 0 : s2_end[i - 1]);
        row[4] = (int32_t)bn2_end[i];
        row[5] = (int32_t)g_s1_end[i];
        row[6] = (int32_t)s2_end[i];
        row[7] = 0;
    }
}

struct MetaLayout {
    size_t status, s1, s2, base, tail, prefix, bcost, bblock, blast, rcost, rlast, rblock, rs2s, total;
    int64_t bufB, row_cap;
};

MetaLayout meta_layout(const SasMetaArgs &a) {
    MetaLayout L{};
    int64_t B = a.batch_size;
    if (a.n_seqused_q > 0) B = a.n_seqused_q;
    else if (a.layout_q == SAS_LAYOUT_TND && a.n_cu_seqlens_q > 0) B = a.n_cu_seqlens_q - 1;
    if (B < 1) B = 1;
    L.bufB = B;
    // row table capacity: reserved[0] = caller's bound on the total number of
    // query rows (0 = none; phase 2 then evaluates rows on the fly)
    L.row_cap = a.reserved[0] > 0 ? a.reserved[0] : 0;
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off = sas::align_up(off + bytes); return o; };
    L.status = take(64);
    L.s1 = take(sizeof(int64_t) * B);
    L.s2 = take(sizeof(int64_t) * B);
    L.base = take(sizeof(int64_t) * B);
    L.tail = take(sizeof(int64_t) * B);
    L.prefix = take(sizeof(int64_t) * (B + 1));
    L.bcost = take(sizeof(int64_t) * B);
    L.bblock = take(sizeof(int64_t) * B);
    L.blast = take(sizeof(int64_t) * B);
    L.rcost = take(sizeof(int64_t) * L.row_cap);
    L.rlast = take(sizeof(int64_t) * L.row_cap);
    L.rblock = take(sizeof(int64_t) * L.row_cap);
    L.rs2s = take(sizeof(int64_t) * L.row_cap);
    L.total = off;
    return L;
}

int validate_meta(const SasMetaArgs &a) {
    if (a.num_heads_kv <= 0 || a.num_heads_q <= 0 || a.num_heads_q < a.num_heads_kv) return SAS_ERR_INVALID_ARG;
    if (a.aic_core_num < 0 || a.aiv_core_num < 0) return SAS_ERR_INVALID_ARG;
    if (a.n_cu_seqlens_q < 0 || a.n_cu_seqlens_ori_kv < 0 || a.n_seqused_q < 0 || a.n_seqused_kv < 0)
        return SAS_ERR_INVALID_ARG;
    if (a.layout_q < 0 || a.layout_q > 3 || a.layout_kv < 0 || a.layout_kv > 1) return SAS_ERR_INVALID_ARG;
    if (a.reserved[0] < 0) return SAS_ERR_INVALID_ARG;
    for (int i = 1; i < 5; ++i)
        if (a.reserved[i] != 0) return SAS_ERR_INVALID_ARG;
    return SAS_OK;
}

} // namespace

extern "C" int sas_metadata_workspace_size(const SasMetaArgs *args, size_t *bytes) {
    if (!args || !bytes) return SAS_ERR_INVALID_ARG;
    int rc = validate_meta(*args);
    if (rc) return rc;
    *bytes = meta_layout(*args).total;
    return SAS_OK;
}

extern "C" int sas_metadata(const SasMetaArgs *args, const int32_t *cu_seqlens_q, const int32_t *cu_seqlens_ori_kv,
                            const int32_t *seqused_q, const int32_t *seqused_kv, int32_t *metadata_out,
                            void *workspace, size_t workspace_bytes, void *stream) {
    if (!args || !metadata_out) return SAS_ERR_INVALID_ARG;
    int rc = validate_meta(*args);
    if (rc) return rc;
    const SasMetaArgs &a = *args;
    if ((a.n_cu_seqlens_q > 0 && !cu_seqlens_q) || (a.n_cu_seqlens_ori_kv > 0 && !cu_seqlens_ori_kv) ||
        (a.n_seqused_q > 0 && !seqused_q) || (a.n_seqused_kv > 0 && !seqused_kv))
        return SAS_ERR_INVALID_ARG;
    const MetaLayout L = meta_layout(a);
    if (!workspace || workspace_bytes < L.total) return SAS_ERR_WORKSPACE;
    char *ws = static_cast<char *>(workspace);
    MetaIn m;
    m.a = a;
    m.cu_q = cu_seqlens_q;
    m.cu_kv = cu_seqlens_ori_kv;
    m.seq_q = seqused_q;
    m.seq_kv = seqused_kv;
    m.out = metadata_out;
    m.status = reinterpret_cast<uint32_t *>(ws + L.status);
    m.s1 = reinterpret_cast<int64_t *>(ws + L.s1);
    m.s2 = reinterpret_cast<int64_t *>(ws + L.s2);
    m.base = reinterpret_cast<int64_t *>(ws + L.base);
    m.tail = reinterpret_cast<int64_t *>(ws + L.tail);
    m.prefix = reinterpret_cast<int64_t *>(ws + L.prefix);
    m.bcost = reinterpret_cast<unsigned long long *>(ws + L.bcost);
    m.bblock = reinterpret_cast<unsigned long long *>(ws + L.bblock);
    m.blast = reinterpret_cast<unsigned long long *>(ws + L.blast);
    m.row_cost = reinterpret_cast<int64_t *>(ws + L.rcost);
    m.row_last = reinterpret_cast<int64_t *>(ws + L.rlast);
    m.row_block = reinterpret_cast<int64_t *>(ws + L.rblock);
    m.row_s2s = reinterpret_cast<int64_t *>(ws + L.rs2s);
    m.row_cap = L.row_cap;
    m.bufB = L.bufB;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (sas_host::check_cuda(cudaMemsetAsync(m.status, 0, 64, s))) return SAS_ERR_CUDA;
    metadata_kernel<<<1, kThreads, 0, s>>>(m);
    return sas_host::check_cuda(cudaGetLastError());
}
