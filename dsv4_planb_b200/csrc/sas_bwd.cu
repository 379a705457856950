// Backward pass of sparse_attn_sharedkv (CUDA cores, fp32 arithmetic).
//
// The reference has no backward (test_graph_mode.py:314-324).  This kernel differentiates the
// forward's softmax over each token's resolved keys (the window rows then the compressed rows,
// the same lists prep_kernel builds for the forward) plus the per-head sink logit:
//
//   P_j    = exp(scale q.k_j - lse)           P_sink = exp(sink - lse)
//   D      = sum_d dO[d] out[d]               (out as the forward returned it)
//   dS_j   = P_j (dO.v_j - D + dlse)          (dlse: the LSE output's gradient, 0 if absent)
//   dq     = scale sum_j dS_j k_j
//   d row  += scale sum_h dS_hj q_h  (all D_qk dims)  +  sum_h P_hj dO_h  (the first D_v dims: V)
//   dsink  += P_sink (dlse - D)
//
// K = V share one row per key, so a row's gradient collects both terms.  P is the exact softmax
// weight (the forward's rounding of P to the input dtype before PV is not differentiated).
// Rows are shared across tokens and heads: their gradients are added with fp32 atomics into
// caller-zeroed [rows][D_qk] buffers, so the sum's order (and the last bits) vary between runs.
// Keys whose block is unmapped read as zero rows in the forward; they take part in the softmax
// and receive no gradient.
//
// One CTA per (token, group of 16 heads), keys streamed in chunks of 32 rows through shared
// memory, as in the CUDA-core forward.  A correctness-first path: there is no reference
// performance to match.

#include "sas_common.cuh"

namespace {

constexpr int kHG = 16;       // heads per CTA
constexpr int kKC = 32;       // keys per chunk
constexpr int kThreads = 256;
constexpr int kMaxQPairs = 32;  // D_qk / 2 / 16 <= 32 (D_qk <= 1024)

struct BwdArgs {
    const void *q, *ori, *cmp, *out, *dout;
    const float *lse, *dlse, *sinks;
    const int32_t *ori_bt, *tinfo, *rows, *cmp_bt;
    float *dq, *dori, *dcmp, *dsinks;
    uint32_t *status;
    int T, N1, Dq, Dv, row_cap;
    int ori_block_num, ori_block_size, ori_table_len;
    int dense_cmp, cmp_block_num, cmp_block_size, cmp_table_len;
    float scale;
};

template <typename T>
__global__ void __launch_bounds__(kThreads) bwd_simt_kernel(BwdArgs p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int KS = p.Dq + 8;  // K row stride (elements), as in the forward
    float *qs = reinterpret_cast<float *>(smem);            // [kHG][Dq]   q (unscaled)
    float *dos = qs + kHG * p.Dq;                           // [kHG][Dv]   dO
    T *ks = reinterpret_cast<T *>(dos + kHG * p.Dv);        // [kKC][KS]   key rows of the chunk
    float *ps = reinterpret_cast<float *>(ks + kKC * KS);   // [kHG][kKC]  P
    float *dss = ps + kHG * kKC;                            // [kHG][kKC]  scale * dS
    float *lse_s = dss + kHG * kKC;                         // [kHG]
    float *dm = lse_s + kHG;                                // [kHG]       D - dlse
    int64_t *rid = reinterpret_cast<int64_t *>(dm + kHG);   // [kKC]
    int *rsrc = reinterpret_cast<int *>(rid + kKC);         // [kKC]: 0 ori, 1 cmp, 2 no key

    const int t = blockIdx.x;
    const int h0 = blockIdx.y * kHG;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int32_t *ti = p.tinfo + (int64_t)t * sas::TI_INTS;
    const int nqp = p.Dq >> 1;  // dim pairs of a q / k row
    const int hq = tid >> 4, sub = tid & 15;

    if (!ti[sas::TI_VALID]) {  // a row of no request: its out is zero and depends on nothing
        for (int e = tid; e < kHG * p.Dq; e += kThreads) {
            const int h = h0 + e / p.Dq;
            if (h < p.N1) p.dq[((int64_t)t * p.N1 + h) * p.Dq + e % p.Dq] = 0.f;
        }
        return;
    }
    const int b = ti[sas::TI_B];
    const int left = ti[sas::TI_LEFT];
    const int n_win = ti[sas::TI_NWIN];
    const int n_keys = n_win + ti[sas::TI_NCMP];
    const T *q = reinterpret_cast<const T *>(p.q) + (int64_t)t * p.N1 * p.Dq;
    const T *out = reinterpret_cast<const T *>(p.out) + (int64_t)t * p.N1 * p.Dv;
    const T *dout = reinterpret_cast<const T *>(p.dout) + (int64_t)t * p.N1 * p.Dv;
    const T *ori = reinterpret_cast<const T *>(p.ori);
    const T *cmp = reinterpret_cast<const T *>(p.cmp);
    const int32_t *crow = p.rows + (int64_t)t * p.row_cap;

    for (int e = tid; e < kHG * p.Dq; e += kThreads) {
        const int h = e / p.Dq, d = e % p.Dq;
        qs[e] = h0 + h < p.N1 ? sas::DT<T>::to_f(q[(int64_t)(h0 + h) * p.Dq + d]) : 0.f;
    }
    for (int e = tid; e < kHG * p.Dv; e += kThreads) {
        const int h = e / p.Dv, d = e % p.Dv;
        dos[e] = h0 + h < p.N1 ? sas::DT<T>::to_f(dout[(int64_t)(h0 + h) * p.Dv + d]) : 0.f;
    }
    __syncthreads();
    // D = dO . out per head (warp w: heads 2w, 2w + 1), and the sink's gradient
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int h = 2 * warp + hh;
        float acc = 0.f;
        if (h0 + h < p.N1)
            for (int d = lane; d < p.Dv; d += 32)
                acc += dos[h * p.Dv + d] * sas::DT<T>::to_f(out[(int64_t)(h0 + h) * p.Dv + d]);
#pragma unroll
        for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (lane == 0) {
            const bool hv = h0 + h < p.N1;
            const float l = hv ? p.lse[(int64_t)t * p.N1 + h0 + h] : 0.f;
            const float g = hv && p.dlse ? p.dlse[(int64_t)t * p.N1 + h0 + h] : 0.f;
            lse_s[h] = l;
            dm[h] = acc - g;
            if (hv) atomicAdd(p.dsinks + h0 + h, -expf(p.sinks[h0 + h] - l) * (acc - g));
        }
    }

    float dq[2 * kMaxQPairs];
#pragma unroll
    for (int k = 0; k < 2 * kMaxQPairs; ++k) dq[k] = 0.f;

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
        // P and scale * dS: warp w owns heads 2w, 2w + 1; lane = key of the chunk
        {
            float s0 = 0.f, s1 = 0.f, v0 = 0.f, v1 = 0.f;
            const T *kr = ks + lane * KS;
            const float *q0 = qs + (2 * warp) * p.Dq, *q1 = q0 + p.Dq;
            const float *g0 = dos + (2 * warp) * p.Dv, *g1 = g0 + p.Dv;
            for (int c16 = 0; c16 < c16n; ++c16) {
                const uint4 kv = *reinterpret_cast<const uint4 *>(kr + c16 * 8);
                const float2 k0 = sas::DT<T>::to_f2(kv.x), k1 = sas::DT<T>::to_f2(kv.y);
                const float2 k2 = sas::DT<T>::to_f2(kv.z), k3 = sas::DT<T>::to_f2(kv.w);
                const float kf[8] = {k0.x, k0.y, k1.x, k1.y, k2.x, k2.y, k3.x, k3.y};
                const int d0 = c16 * 8;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    s0 += q0[d0 + i] * kf[i];
                    s1 += q1[d0 + i] * kf[i];
                }
                if (d0 < p.Dv) {  // D_v % 32 == 0, so a 16-byte group is wholly in V or not
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        v0 += g0[d0 + i] * kf[i];
                        v1 += g1[d0 + i] * kf[i];
                    }
                }
            }
            const bool key = rsrc[lane] != 2;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int h = 2 * warp + hh;
                const bool live = key && h0 + h < p.N1;
                const float pj = live ? expf(p.scale * (hh ? s1 : s0) - lse_s[h]) : 0.f;
                ps[h * kKC + lane] = pj;
                dss[h * kKC + lane] = p.scale * pj * ((hh ? v1 : v0) - dm[h]);
            }
        }
        __syncthreads();
        const int nk = min(kKC, n_keys - c * kKC);
        // dq: thread = (head hq, dim pairs sub + 16 k)
        for (int j = 0; j < nk; ++j) {
            const float g = dss[hq * kKC + j];
            const uint32_t *row = reinterpret_cast<const uint32_t *>(ks + j * KS);
#pragma unroll
            for (int k = 0; k < kMaxQPairs; ++k) {
                const int pi = sub + 16 * k;
                if (pi < nqp) {
                    const float2 kv = sas::DT<T>::to_f2(row[pi]);
                    dq[2 * k] += g * kv.x;
                    dq[2 * k + 1] += g * kv.y;
                }
            }
        }
        // the chunk's row gradients: consecutive threads take consecutive dims of one row
        for (int e = tid; e < nk * p.Dq; e += kThreads) {
            const int j = e / p.Dq, d = e - j * p.Dq;
            const int64_t r = rid[j];
            if (r < 0) continue;
            float acc = 0.f;
#pragma unroll
            for (int h = 0; h < kHG; ++h) acc += dss[h * kKC + j] * qs[h * p.Dq + d];
            if (d < p.Dv) {
#pragma unroll
                for (int h = 0; h < kHG; ++h) acc += ps[h * kKC + j] * dos[h * p.Dv + d];
            }
            atomicAdd((rsrc[j] == 0 ? p.dori : p.dcmp) + r * p.Dq + d, acc);
        }
    }
    if (h0 + hq < p.N1) {
        float *dqrow = p.dq + ((int64_t)t * p.N1 + h0 + hq) * p.Dq;
#pragma unroll
        for (int k = 0; k < kMaxQPairs; ++k) {
            const int pi = sub + 16 * k;
            if (pi < nqp) *reinterpret_cast<float2 *>(dqrow + 2 * pi) = make_float2(dq[2 * k], dq[2 * k + 1]);
        }
    }
}

size_t bwd_smem(int Dq, int Dv) {
    return sizeof(float) * kHG * (size_t)(Dq + Dv) + 2 * (size_t)kKC * (Dq + 8) + sizeof(float) * (2 * kHG * kKC + 2 * kHG) +
           sizeof(int64_t) * kKC + sizeof(int) * kKC + 64;
}

} // namespace

namespace sas_host {

int check_cuda(cudaError_t e);

// The backward grid over the records prep_kernel left in the workspace (the same key lists as the
// forward).  dq is written; d_ori, d_cmp and d_sinks are added into.
int launch_bwd_simt(const SasFwdArgs &a, const sas::FwdLayout &L, char *ws, const void *q, const void *ori_kv,
                    const int32_t *ori_bt, const void *cmp_kv, const int32_t *cmp_bt, const float *sinks,
                    const void *out, const float *lse, const void *dout, const float *dlse, float *dq, float *d_ori,
                    float *d_cmp, float *d_sinks, cudaStream_t s) {
    if (a.num_tokens == 0 || a.num_heads == 0) return SAS_OK;
    BwdArgs p;
    p.q = q;
    p.ori = ori_kv;
    p.cmp = cmp_kv;
    p.out = out;
    p.dout = dout;
    p.lse = lse;
    p.dlse = dlse;
    p.sinks = sinks;
    p.ori_bt = ori_bt;
    p.tinfo = reinterpret_cast<const int32_t *>(ws + L.token_info);
    p.rows = reinterpret_cast<const int32_t *>(ws + L.cmp_rows);
    p.cmp_bt = cmp_bt;
    p.dq = dq;
    p.dori = d_ori;
    p.dcmp = d_cmp;
    p.dsinks = d_sinks;
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
    p.cmp_block_num = a.cmp_block_num;
    p.cmp_block_size = a.cmp_block_size;
    p.cmp_table_len = a.cmp_table_len;
    p.scale = a.softmax_scale;
    const size_t smem = bwd_smem(a.head_dim, a.v_head_dim);
    dim3 grid(a.num_tokens, (a.num_heads + kHG - 1) / kHG);
    // raised once per device and dtype to the largest layout (D_qk 1024, D_v 512)
    int dev = 0;
    if (check_cuda(cudaGetDevice(&dev))) return SAS_ERR_CUDA;
    if (dev < 0 || dev >= sas::kMaxDevices) return SAS_ERR_UNSUPPORTED;
    static sas::DeviceOnce attr_done[sas::kMaxDevices];
    const int di = a.dtype == SAS_DTYPE_BF16 ? 0 : 1;
    const int rc = attr_done[dev].run(1u << di, [&] {
        const int max_smem = (int)bwd_smem(1024, 512);
        cudaError_t e = di == 0 ? cudaFuncSetAttribute(bwd_simt_kernel<__nv_bfloat16>,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem)
                                : cudaFuncSetAttribute(bwd_simt_kernel<__half>,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
        return check_cuda(e);
    });
    if (rc) return rc;
    if (a.dtype == SAS_DTYPE_BF16) bwd_simt_kernel<__nv_bfloat16><<<grid, kThreads, smem, s>>>(p);
    else bwd_simt_kernel<__half><<<grid, kThreads, smem, s>>>(p);
    return check_cuda(cudaGetLastError());
}

} // namespace sas_host
