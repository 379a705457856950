// Portable CUDA-core path of the fused attention (any head count, D_qk <= 1024,
// D_v <= 512).  One CTA per (token, group of 16 heads); keys are streamed in
// chunks of 32 rows through shared memory.
//
// Per token the math is the reference golden (golden.py:156-200): a sink-seeded
// online softmax over the window keys then the compressed keys, K = V, P rounded
// to the input dtype before the PV product and lse = m + ln(l).  The output is
// normalised by the sum of the rounded P (the weights actually applied), which
// keeps out a convex combination of V rows; l for the LSE sums the exact P.
// Scores are kept in the log2 domain (q pre-scaled by softmax_scale * log2 e).
// The tensor-core path (sas_fwd_tc.cu) is the fast path for the production
// shapes; this kernel serves the shapes it does not take.

#include "sas_common.cuh"

namespace {

constexpr int kHG = 16;      // heads per CTA
constexpr int kKC = 32;      // keys per chunk
constexpr int kThreads = 256;
constexpr int kMaxPairs = 16; // D_v / 32 <= 16

struct SimtArgs {
    const void *q, *ori, *cmp;
    const int32_t *ori_bt, *tinfo, *rows;
    const int32_t *cmp_bt;  // scenario 2: compressed rows are positions 0 .. n_cmp-1 of this table
    const float *sinks;
    void *out;
    float *lse;
    uint32_t *status;
    int T, N1, Dq, Dv, row_cap;
    int ori_block_num, ori_block_size, ori_table_len;
    int dense_cmp, cmp_block_num, cmp_block_size, cmp_table_len;
    float scale_log2;
};

template <typename T>
__global__ void __launch_bounds__(kThreads) fwd_simt_kernel(SimtArgs p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int KS = p.Dq + 8;  // K row stride (elements): 16-byte aligned, conflict-free 16-byte reads
    float *qs = reinterpret_cast<float *>(smem);                       // [kHG][Dq]
    T *ks = reinterpret_cast<T *>(qs + kHG * p.Dq);                    // [kKC][KS]
    float *ps = reinterpret_cast<float *>(ks + kKC * KS);              // [kHG][kKC]
    float *ms = ps + kHG * kKC;                                        // [kHG]
    float *ls = ms + kHG;
    float *al = ls + kHG;
    float *lr = al + kHG;                                              // [kHG] sum of rounded P
    int64_t *rid = reinterpret_cast<int64_t *>(lr + kHG);              // [kKC]
    int *rsrc = reinterpret_cast<int *>(rid + kKC);                    // [kKC]: 0 ori, 1 cmp, 2 masked

    const int t = blockIdx.x;
    const int h0 = blockIdx.y * kHG;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int32_t *ti = p.tinfo + (int64_t)t * sas::TI_INTS;
    const int valid = ti[sas::TI_VALID];
    const int npair = p.Dv >> 5;
    T *out = reinterpret_cast<T *>(p.out);

    if (!valid) {  // rows that belong to no (b, s) stay zero (golden.py:97)
        for (int e = tid; e < kHG * p.Dv; e += kThreads) {
            const int h = h0 + e / p.Dv;
            if (h < p.N1) out[((int64_t)t * p.N1 + h) * p.Dv + e % p.Dv] = sas::DT<T>::from_f(0.f);
        }
        if (p.lse && tid < kHG && h0 + tid < p.N1) p.lse[(int64_t)t * p.N1 + h0 + tid] = 0.f;
        return;
    }
    const int b = ti[sas::TI_B];
    const int left = ti[sas::TI_LEFT];
    const int n_win = ti[sas::TI_NWIN];
    const int n_keys = n_win + ti[sas::TI_NCMP];
    const T *q = reinterpret_cast<const T *>(p.q) + (int64_t)t * p.N1 * p.Dq;
    const T *ori = reinterpret_cast<const T *>(p.ori);
    const T *cmp = reinterpret_cast<const T *>(p.cmp);
    const int32_t *crow = p.rows + (int64_t)t * p.row_cap;

    for (int e = tid; e < kHG * p.Dq; e += kThreads) {
        const int h = e / p.Dq, d = e % p.Dq;
        qs[e] = (h0 + h < p.N1) ? sas::DT<T>::to_f(q[(int64_t)(h0 + h) * p.Dq + d]) * p.scale_log2 : 0.f;
    }
    if (tid < kHG) {
        ms[tid] = (h0 + tid < p.N1) ? p.sinks[h0 + tid] * 1.4426950408889634f : 0.f;
        ls[tid] = 1.f;
        lr[tid] = 1.f;
    }
    float o[2 * kMaxPairs];
#pragma unroll
    for (int k = 0; k < 2 * kMaxPairs; ++k) o[k] = 0.f;

    const int n_chunks = (n_keys + kKC - 1) / kKC;
    const int c16n = p.Dq >> 3;
    for (int c = 0; c < n_chunks; ++c) {
        __syncthreads();
        if (tid < kKC) {
            const int slot = c * kKC + tid;
            int64_t r = -1;
            int src = 2;
            if (slot < n_win) {
                r = sas::paged_row(p.ori_bt, b, p.ori_table_len, p.ori_block_size, p.ori_block_num, left + slot,
                                   p.status);
                src = 0;
            } else if (slot < n_keys) {
                r = p.dense_cmp ? sas::paged_row(p.cmp_bt, b, p.cmp_table_len, p.cmp_block_size, p.cmp_block_num,
                                                 slot - n_win, p.status)
                                : crow[slot - n_win];
                src = 1;
            }
            rid[tid] = r;
            rsrc[tid] = src;
        }
        __syncthreads();
        for (int e = tid; e < kKC * c16n; e += kThreads) {
            const int j = e / c16n, c16 = e % c16n;
            const int64_t r = rid[j];
            uint4 v = make_uint4(0, 0, 0, 0);
            if (r >= 0) {
                const T *src = (rsrc[j] == 0 ? ori : cmp) + r * p.Dq;
                v = __ldg(reinterpret_cast<const uint4 *>(src) + c16);
            }
            *reinterpret_cast<uint4 *>(ks + j * KS + c16 * 8) = v;
        }
        __syncthreads();
        // scores: warp w owns heads 2w, 2w+1; lane = key
        {
            float acc0 = 0.f, acc1 = 0.f;
            const T *kr = ks + lane * KS;
            const float *q0 = qs + (2 * warp) * p.Dq;
            const float *q1 = q0 + p.Dq;
            for (int c16 = 0; c16 < c16n; ++c16) {
                const uint4 kv = *reinterpret_cast<const uint4 *>(kr + c16 * 8);
                const float2 k0 = sas::DT<T>::to_f2(kv.x), k1 = sas::DT<T>::to_f2(kv.y);
                const float2 k2 = sas::DT<T>::to_f2(kv.z), k3 = sas::DT<T>::to_f2(kv.w);
                const float4 a0 = *reinterpret_cast<const float4 *>(q0 + c16 * 8);
                const float4 a1 = *reinterpret_cast<const float4 *>(q0 + c16 * 8 + 4);
                const float4 b0 = *reinterpret_cast<const float4 *>(q1 + c16 * 8);
                const float4 b1 = *reinterpret_cast<const float4 *>(q1 + c16 * 8 + 4);
                acc0 += a0.x * k0.x + a0.y * k0.y + a0.z * k1.x + a0.w * k1.y + a1.x * k2.x + a1.y * k2.y +
                        a1.z * k3.x + a1.w * k3.y;
                acc1 += b0.x * k0.x + b0.y * k0.y + b0.z * k1.x + b0.w * k1.y + b1.x * k2.x + b1.y * k2.y +
                        b1.z * k3.x + b1.w * k3.y;
            }
            const bool masked = rsrc[lane] == 2;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int h = 2 * warp + hh;
                const float s = masked ? -INFINITY : (hh ? acc1 : acc0);
                float mx = s;
#pragma unroll
                for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
                const float m_old = ms[h];
                const float m_new = fmaxf(m_old, mx);
                const float alpha = exp2f(m_old - m_new);
                const float pv = masked ? 0.f : exp2f(s - m_new);
                const float pr = sas::DT<T>::round_p(pv);
                float sum = pv, sumr = pr;
#pragma unroll
                for (int off = 16; off; off >>= 1) {
                    sum += __shfl_xor_sync(0xffffffffu, sum, off);
                    sumr += __shfl_xor_sync(0xffffffffu, sumr, off);
                }
                ps[h * kKC + lane] = pr;
                __syncwarp();
                if (lane == 0) {
                    ls[h] = ls[h] * alpha + sum;
                    lr[h] = lr[h] * alpha + sumr;
                    ms[h] = m_new;
                    al[h] = alpha;
                }
            }
        }
        __syncthreads();
        // PV: thread = (head h = tid / 16, word column sub = tid % 16)
        {
            const int h = tid >> 4, sub = tid & 15;
            const float a = al[h];
#pragma unroll
            for (int k = 0; k < 2 * kMaxPairs; ++k) o[k] *= a;
            const int nk = min(kKC, n_keys - c * kKC);
            for (int j = 0; j < nk; ++j) {
                const float pj = ps[h * kKC + j];
                const uint32_t *row = reinterpret_cast<const uint32_t *>(ks + j * KS);
#pragma unroll
                for (int k = 0; k < kMaxPairs; ++k) {
                    if (k < npair) {
                        const float2 v = sas::DT<T>::to_f2(row[sub + 16 * k]);
                        o[2 * k] += pj * v.x;
                        o[2 * k + 1] += pj * v.y;
                    }
                }
            }
        }
    }
    __syncthreads();
    {
        const int h = tid >> 4, sub = tid & 15;
        if (h0 + h < p.N1) {
            const float inv = 1.f / lr[h];
            T *orow = out + ((int64_t)t * p.N1 + h0 + h) * p.Dv;
#pragma unroll
            for (int k = 0; k < kMaxPairs; ++k) {
                if (k < npair) {
                    const int d = 2 * (sub + 16 * k);
                    orow[d] = sas::DT<T>::from_f(o[2 * k] * inv);
                    orow[d + 1] = sas::DT<T>::from_f(o[2 * k + 1] * inv);
                }
            }
            if (sub == 0 && p.lse) p.lse[(int64_t)t * p.N1 + h0 + h] = (ms[h] + log2f(ls[h])) * 0.6931471805599453f;
        }
    }
}

size_t simt_smem(int Dq) {
    return sizeof(float) * kHG * Dq + 2 * (size_t)kKC * (Dq + 8) + sizeof(float) * (kHG * kKC + 5 * kHG) +
           sizeof(int64_t) * kKC + sizeof(int) * kKC + 64;
}

} // namespace

namespace sas_host {

int launch_fwd_simt(const SasFwdArgs &a, const sas::FwdLayout &L, char *ws, const void *q, const void *ori_kv,
                    const int32_t *ori_bt, const void *cmp_kv, const int32_t *cmp_bt, const float *sinks, void *out,
                    float *lse, cudaStream_t s) {
    if (a.num_tokens == 0 || a.num_heads == 0) return SAS_OK;
    SimtArgs p;
    p.q = q;
    p.ori = ori_kv;
    p.cmp = cmp_kv;
    p.ori_bt = ori_bt;
    p.tinfo = reinterpret_cast<const int32_t *>(ws + L.token_info);
    p.rows = reinterpret_cast<const int32_t *>(ws + L.cmp_rows);
    p.sinks = sinks;
    p.out = out;
    p.lse = lse;
    p.status = reinterpret_cast<uint32_t *>(ws + L.status);
    p.T = a.num_tokens;
    p.N1 = a.num_heads;
    p.Dq = a.head_dim;
    p.Dv = a.v_head_dim;
    p.row_cap = (int)L.row_cap;
    p.ori_block_num = a.ori_block_num;
    p.ori_block_size = a.ori_block_size;
    p.ori_table_len = a.ori_table_len;
    p.dense_cmp = a.scenario == 2 ? 1 : 0;
    p.cmp_bt = cmp_bt;
    p.cmp_block_num = a.cmp_block_num;
    p.cmp_block_size = a.cmp_block_size;
    p.cmp_table_len = a.cmp_table_len;
    p.scale_log2 = a.softmax_scale * 1.4426950408889634f;
    const size_t smem = simt_smem(a.head_dim);
    dim3 grid(a.num_tokens, (a.num_heads + kHG - 1) / kHG);
    // The opt-in shared-memory size is raised once per device and dtype to the
    // largest layout (D_qk = 1024), so the call inside a stream capture is a no-op.
    int dev = 0;
    if (check_cuda(cudaGetDevice(&dev))) return SAS_ERR_CUDA;
    if (dev < 0 || dev >= sas::kMaxDevices) return SAS_ERR_UNSUPPORTED;
    static sas::DeviceOnce attr_done[sas::kMaxDevices];
    const int di = a.dtype == SAS_DTYPE_BF16 ? 0 : 1;
    const int rc = attr_done[dev].run(1u << di, [&] {
        const int max_smem = (int)simt_smem(1024);
        cudaError_t e = di == 0 ? cudaFuncSetAttribute(fwd_simt_kernel<__nv_bfloat16>,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem)
                                : cudaFuncSetAttribute(fwd_simt_kernel<__half>,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
        return check_cuda(e);
    });
    if (rc) return rc;
    if (a.dtype == SAS_DTYPE_BF16) fwd_simt_kernel<__nv_bfloat16><<<grid, kThreads, smem, s>>>(p);
    else fwd_simt_kernel<__half><<<grid, kThreads, smem, s>>>(p);
    return check_cuda(cudaGetLastError());
}

} // namespace sas_host
