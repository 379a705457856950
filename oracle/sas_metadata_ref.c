/*
 * Plain-C restatement of the reference metadata tile scheduler -- TEST
 * INFRASTRUCTURE ONLY (the checker for the CUDA scheduler, and its timed CPU
 * baseline).  Nothing in the product library links this file.
 *
 * Follows sparse_attn_sharedkv_tilelang/metadata.py of yangqiang2018/dsv4_planB
 * (itself a port of the Ascend aicpu SparseAttnSharedkvMetadata kernel):
 *   params_init ............ metadata.py:359-390
 *   s1/s2 sizes, pre/next .. metadata.py:345-426
 *   block cost ............. metadata.py:428-477
 *   s2 token range ......... metadata.py:479-501
 *   block range / tails .... metadata.py:512-547
 *   win/cmp row caches ..... metadata.py:549-632
 *   row cache .............. metadata.py:634-667
 *   split info / costs ..... metadata.py:671-714
 *   greedy assignment ...... metadata.py:718-923 (FD paths: supportFd is False in
 *                            the reference and is never flipped, so block-level
 *                            reassignment and FD bookkeeping are inert)
 *   packing ................ metadata.py:974-1009
 *
 * Python integers do not overflow; the pre/next-token arithmetic involves
 * INT64_MAX when the window is unbounded, so those sums are done in __int128.
 * Python floor division and modulo are reproduced by floordiv()/pymod().
 * metadata.py:759-763 loops forever when no later row has work; this port
 * stops after a bounded number of empty rows and returns SASM_ERR_NO_PROGRESS.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define AIC_CORE_NUM 36
#define AIV_CORE_NUM 72
#define SAS_META_SIZE 1024
#define FA_METADATA_SIZE 8
#define FD_METADATA_SIZE 8
#define S2_BASE 512
#define TOL_RATIO 2

enum { SASM_OK = 0, SASM_ERR_ARG = 1, SASM_ERR_INDEX = 2, SASM_ERR_NO_PROGRESS = 3 };
enum { LQ_BSND = 0, LQ_BSH = 1, LQ_TND = 2, LQ_OTHER = 3 };
enum { LKV_PA_ND = 0, LKV_TND = 1 };
enum { M_DEFAULT = 0, M_ALL = 1, M_LEFT_UP = 2, M_RIGHT_DOWN = 3, M_BAND = 4 };

typedef __int128 i128;
static const int64_t I64MAX = INT64_MAX;

typedef struct {
    int64_t num_heads_q, num_heads_kv, head_dim;
    const int64_t *cu_seqlens_q; int64_t n_cu_q;
    const int64_t *cu_seqlens_ori_kv; int64_t n_cu_kv;
    const int64_t *seqused_q; int64_t n_seqused_q;
    const int64_t *seqused_kv; int64_t n_seqused_kv;
    int64_t batch_size, max_seqlen_q, max_seqlen_kv;
    int64_t ori_topk, cmp_topk, cmp_ratio;
    int64_t ori_mask_mode, cmp_mask_mode, ori_win_left, ori_win_right;
    int64_t layout_q, layout_kv, has_ori_kv, has_cmp_kv;
    int64_t aic_core_num, aiv_core_num;
} SasmArgs;

static int64_t floordiv(int64_t a, int64_t b) {
    int64_t q = a / b, r = a % b;
    return (r != 0 && ((r < 0) != (b < 0))) ? q - 1 : q;
}
static int64_t pymod(int64_t a, int64_t b) {
    int64_t r = a % b;
    return (r != 0 && ((r < 0) != (b < 0))) ? r + b : r;
}
static i128 floordiv128(i128 a, i128 b) {
    i128 q = a / b, r = a % b;
    return (r != 0 && ((r < 0) != (b < 0))) ? q - 1 : q;
}
static i128 pymod128(i128 a, i128 b) {
    i128 r = a % b;
    return (r != 0 && ((r < 0) != (b < 0))) ? r + b : r;
}
static int64_t imax(int64_t a, int64_t b) { return a > b ? a : b; }
static int64_t imin(int64_t a, int64_t b) { return a < b ? a : b; }

typedef struct { int64_t b, s1, s2; i128 pre_lu, next_lu; } BatchC;

typedef struct {
    int64_t b, s1g, s2_start, s2_end, win_s2_start, win_s2_end, cmp_s2_start, cmp_s2_end;
    int64_t cost, last_cost, block;
    int64_t win_block, win_cost, win_last_cost, win_normal_cost;
    int64_t cmp_block, cmp_cost, cmp_last_cost, cmp_normal_cost;
    int64_t cmp_tail, win_tail;
} RowC;

typedef struct {
    const SasmArgs *a;
    int err;
    int64_t B, G, m_base, pre_token, next_token;
    int attn_mode, is_s1g, is_cfa, is_scfa;
    int64_t tc[4][4];
    /* split info, per batch */
    int64_t *s1g_base, *s1g_tail;
    int all_zero;
    /* cost info, per batch */
    int64_t *bcost, *bblock, *blast;
    int64_t total_cost, total_block, max_row_cost;
} Sched;

static int64_t s1_size(Sched *S, int64_t b) {
    const SasmArgs *a = S->a;
    if (a->n_seqused_q > 0) {
        if (b < 0 || b >= a->n_seqused_q) { S->err = SASM_ERR_INDEX; return 0; }
        return a->seqused_q[b];
    }
    if (a->layout_q == LQ_TND && a->n_cu_q > 0) {
        if (b < 0 || b + 1 >= a->n_cu_q) { S->err = SASM_ERR_INDEX; return 0; }
        return a->cu_seqlens_q[b + 1] - a->cu_seqlens_q[b];
    }
    return a->max_seqlen_q;
}

static int64_t s2_size(Sched *S, int64_t b) {
    const SasmArgs *a = S->a;
    if (a->n_seqused_kv > 0) {
        if (b < 0 || b >= a->n_seqused_kv) { S->err = SASM_ERR_INDEX; return 0; }
        return a->seqused_kv[b];
    }
    if (a->layout_kv == LKV_TND && a->n_cu_kv > 0) {
        if (b < 0 || b + 1 >= a->n_cu_kv) { S->err = SASM_ERR_INDEX; return 0; }
        return a->cu_seqlens_ori_kv[b + 1] - a->cu_seqlens_ori_kv[b];
    }
    return a->max_seqlen_kv;
}

static void batch_cache(Sched *S, int64_t b, BatchC *bc) {
    bc->b = b;
    bc->s1 = s1_size(S, b);
    bc->s2 = s2_size(S, b);
    int64_t mode = S->a->ori_mask_mode;
    bc->pre_lu = (mode == M_BAND) ? (i128)bc->s1 - bc->s2 + S->pre_token : (i128)S->pre_token;
    if (mode == M_DEFAULT || mode == M_ALL || mode == M_LEFT_UP) bc->next_lu = S->next_token;
    else if (mode == M_RIGHT_DOWN) bc->next_lu = (i128)bc->s2 - bc->s1;
    else if (mode == M_BAND) bc->next_lu = (i128)bc->s2 - bc->s1 + S->next_token;
    else bc->next_lu = S->next_token;
}

static int64_t blk_cost(int64_t m, int64_t s2) {
    return 6 * ((m + 15) >> 4) + 10 * ((s2 + 63) >> 6);
}

static void cost_table(Sched *S, int64_t s1n, int64_t s2n, int64_t s1t, int64_t wt, int64_t ct) {
    int64_t (*tc)[4] = S->tc;
    tc[0][0] = blk_cost(s1n, s2n);
    tc[1][0] = s1t == 0 ? 0 : blk_cost(s1t, s2n);
    tc[0][1] = wt == 0 ? 0 : blk_cost(s1n, wt);
    tc[1][1] = (s1t == 0 || wt == 0) ? 0 : blk_cost(s1t, wt);
    if (S->a->has_cmp_kv) {
        tc[2][2] = blk_cost(s1n, s2n);
        tc[3][2] = s1t == 0 ? 0 : blk_cost(s1t, s2n);
        tc[2][3] = ct == 0 ? 0 : blk_cost(s1n, ct);
        tc[3][3] = (s1t == 0 || ct == 0) ? 0 : blk_cost(s1t, ct);
    }
}

static void s2_range(Sched *S, int64_t s1g, const BatchC *bc, i128 *first, i128 *last) {
    if (bc->s1 == 0 || bc->s2 == 0) { *first = 0; *last = 0; return; }
    if (!S->attn_mode) { *first = 0; *last = (i128)bc->s2 - 1; return; }
    int64_t s1g_first = s1g * S->m_base;
    int64_t s1g_last = imin(s1g_first + S->m_base, bc->s1 * S->G) - 1;
    int64_t s1_first, s1_last;
    if (S->is_s1g) {
        s1_first = floordiv(s1g_first, S->G);
        s1_last = floordiv(s1g_last, S->G);
    } else if (floordiv(s1g_first, bc->s1) == floordiv(s1g_last, bc->s1)) {
        s1_first = pymod(s1g_first, bc->s1);
        s1_last = pymod(s1g_last, bc->s1);
    } else {
        s1_first = 0;
        s1_last = bc->s1;
    }
    *first = (i128)s1_first - bc->pre_lu;
    *last = (i128)s1_last + bc->next_lu;
}

static void block_range(Sched *S, i128 f, i128 l, const BatchC *bc, RowC *r) {
    if (f >= bc->s2 || l < 0 || l < f) {
        f = 0; l = 0;
        r->win_s2_start = 0; r->win_s2_end = 0; r->win_tail = 0;
    } else {
        i128 hi = (i128)bc->s2 - 1;
        /* _clip(v, 0, hi) = max(0, min(v, hi)), metadata.py:84-85 */
        f = f < hi ? f : hi; f = f > 0 ? f : 0;
        l = l < hi ? l : hi; l = l > 0 ? l : 0;
        r->win_s2_start = 0;
        r->win_s2_end = (int64_t)floordiv128(l - f, S2_BASE) + 1;
        r->win_tail = (int64_t)pymod128(l - f + 1, S2_BASE);
    }
    r->cmp_s2_start = r->win_s2_end;
    int64_t cmp_last = 0;
    if (S->a->has_cmp_kv && S->a->cmp_ratio > 0)
        cmp_last = (int64_t)floordiv128(l + 1, S->a->cmp_ratio);
    int64_t act = 0;
    if (S->is_cfa) act = cmp_last;
    else if (S->is_scfa) act = imin(cmp_last, S->a->cmp_topk);
    if (act == 0) r->cmp_s2_end = r->cmp_s2_start;
    else r->cmp_s2_end = r->cmp_s2_start + floordiv(act - 1, S2_BASE) + 1;
    r->cmp_tail = pymod(act, S2_BASE);
}

static int is_tail_row(Sched *S, const RowC *r) {
    return r->s1g == S->s1g_base[r->b] - 1 && S->s1g_tail[r->b] != 0;
}

static void win_row(Sched *S, RowC *r) {
    int64_t (*tc)[4] = S->tc;
    if (r->win_s2_start >= r->win_s2_end) {
        r->win_block = 0; r->win_cost = 0; r->win_last_cost = 0; r->win_normal_cost = 0;
        return;
    }
    r->win_block = r->win_s2_end - r->win_s2_start;
    int64_t t = r->win_tail != 0 ? 1 : 0, n = r->win_block - t;
    int row = is_tail_row(S, r) ? 1 : 0;
    r->win_cost = tc[row][0] * n + tc[row][1] * t;
    r->win_last_cost = t > 0 ? tc[row][1] : tc[row][0];
    r->win_normal_cost = tc[row][0];
}

static void cmp_row(Sched *S, RowC *r) {
    int64_t (*tc)[4] = S->tc;
    if (r->cmp_s2_start >= r->cmp_s2_end) {
        r->cmp_block = 0; r->cmp_cost = 0; r->cmp_last_cost = 0; r->cmp_normal_cost = 0;
        return;
    }
    r->cmp_block = r->cmp_s2_end - r->cmp_s2_start;
    int64_t t = r->cmp_tail != 0 ? 1 : 0, n = r->cmp_block - t;
    int row = is_tail_row(S, r) ? 3 : 2;
    r->cmp_cost = tc[row][2] * n + tc[row][3] * t;
    r->cmp_last_cost = t > 0 ? tc[row][3] : tc[row][2];
    r->cmp_normal_cost = tc[row][2];
}

static void row_cache(Sched *S, int64_t s1g, const BatchC *bc, RowC *r) {
    if (bc->b < 0 || bc->b >= S->B) { S->err = SASM_ERR_INDEX; return; }
    if (S->s1g_base[bc->b] == 0) {
        /* metadata.py:642-653 resets only these fields */
        r->cost = 0; r->last_cost = 0;
        r->win_normal_cost = 0; r->win_last_cost = 0;
        r->cmp_normal_cost = 0; r->cmp_last_cost = 0;
        r->block = 0; r->s2_start = 0; r->cmp_s2_start = 0; r->s2_end = 0;
        return;
    }
    r->b = bc->b;
    r->s1g = s1g;
    i128 f, l;
    s2_range(S, s1g, bc, &f, &l);
    block_range(S, f, l, bc, r);
    cost_table(S, S->m_base, S2_BASE, S->s1g_tail[r->b], r->win_tail, r->cmp_tail);
    win_row(S, r);
    cmp_row(S, r);
    r->s2_start = r->win_block > 0 ? r->win_s2_start : r->cmp_s2_start;
    if (r->cmp_block > 0) { r->last_cost = r->cmp_last_cost; r->s2_end = r->cmp_s2_end; }
    else { r->last_cost = r->win_last_cost; r->s2_end = r->win_s2_end; }
    r->block = r->win_block + r->cmp_block;
    r->cost = r->win_cost + r->cmp_cost;
}

typedef struct {
    int64_t cur_b, cur_bn2, cur_s1g, cur_s2, cur_core, unassigned;
    int64_t kv_split_part, fd_data_num, bn2_cost, bn2_block;
    int finished;
    BatchC bc;
    RowC rc;
    int64_t core_limit, core_cost, core_block;
} Assign;

static int within(int64_t limit, int64_t tol, int64_t value) { return limit + tol >= value; }

static void by_batch(Sched *S, Assign *A) {
    if (A->finished) return;
    int64_t N2 = S->a->num_heads_kv;
    while (A->bn2_cost == 0 ||
           within(A->core_limit, floordiv(S->blast[A->cur_b], TOL_RATIO), A->core_cost + A->bn2_cost)) {
        A->core_cost += A->bn2_cost;
        A->core_block += A->bn2_block;
        A->cur_bn2 += 1;
        if (A->cur_bn2 == S->B * N2) {
            A->cur_s1g = 0; A->cur_s2 = 0; A->finished = 1;
            return;
        }
        if (floordiv(A->cur_bn2, N2) != A->cur_b) {
            A->cur_b = floordiv(A->cur_bn2, N2);
            batch_cache(S, A->cur_b, &A->bc);
        }
        if (A->cur_b < 0 || A->cur_b >= S->B) { S->err = SASM_ERR_INDEX; return; }
        A->bn2_cost = S->bcost[A->cur_b];
        A->bn2_block = S->bblock[A->cur_b];
        A->cur_s1g = 0;
        row_cache(S, A->cur_s1g, &A->bc, &A->rc);
        A->cur_s2 = A->rc.s2_start;
        if (S->err) return;
    }
}

static void by_row(Sched *S, Assign *A) {
    if (A->finished) return;
    while (within(A->core_limit, floordiv(A->rc.last_cost, TOL_RATIO), A->core_cost + A->rc.cost)) {
        A->core_cost += A->rc.cost;
        A->core_block += A->rc.block;
        A->bn2_cost = imax(0, A->bn2_cost - A->rc.cost);
        A->bn2_block = imax(0, A->bn2_block - A->rc.block);
        /* metadata.py:759-763: advance to the next row that has blocks.  The
         * reference spins forever when none exists; rows past
         * base + |win_left| + s2 + 64 are all empty, so stop there. */
        int64_t cap = S->s1g_base[A->bc.b] + (S->a->ori_win_left < 0 ? -S->a->ori_win_left : S->a->ori_win_left) +
                      (A->bc.s2 < 0 ? -A->bc.s2 : A->bc.s2) + 64;
        for (;;) {
            A->cur_s1g += 1;
            row_cache(S, A->cur_s1g, &A->bc, &A->rc);
            if (S->err) return;
            if (A->rc.block != 0) break;
            if (A->cur_s1g > cap) { S->err = SASM_ERR_NO_PROGRESS; return; }
        }
        A->cur_s2 = A->rc.s2_start;
    }
}

static int sched_run(Sched *Sp, const SasmArgs *a, int64_t aic, int64_t *bn2_end, int64_t *g_s1_end,
                     int64_t *s2_end, int32_t *out);

int sasm_ref_metadata(const SasmArgs *a, int32_t *out) {
    Sched S;
    memset(&S, 0, sizeof(S));
    memset(out, 0, sizeof(int32_t) * SAS_META_SIZE);
    S.a = a;
    if (a->num_heads_kv <= 0 || a->num_heads_q <= 0 || a->num_heads_q < a->num_heads_kv) return SASM_ERR_ARG;
    if (a->aic_core_num < 0 || a->aiv_core_num < 0) return SASM_ERR_ARG;

    /* params_init, metadata.py:359-390 */
    if (a->n_seqused_q > 0) S.B = a->n_seqused_q;
    else if (a->layout_q == LQ_TND && a->n_cu_q > 0) S.B = a->n_cu_q - 1;
    else S.B = a->batch_size;
    if (S.B < 0) return SASM_ERR_ARG;
    if (a->ori_mask_mode == M_DEFAULT) { S.pre_token = I64MAX; S.next_token = I64MAX; S.attn_mode = 0; }
    else if (a->ori_mask_mode == M_RIGHT_DOWN) { S.pre_token = I64MAX; S.next_token = 0; S.attn_mode = 1; }
    else { S.pre_token = a->ori_win_left > -1 ? a->ori_win_left : I64MAX; S.next_token = 0; S.attn_mode = 1; }
    S.is_s1g = (a->layout_q == LQ_BSND || a->layout_q == LQ_BSH || a->layout_q == LQ_TND);
    S.G = a->num_heads_q / a->num_heads_kv;
    if (a->has_cmp_kv) {
        if (a->cmp_topk > 0) S.is_scfa = 1; else S.is_cfa = 1;
    }
    S.m_base = S.G;

    int64_t aic = a->aic_core_num;
    int64_t Bn = S.B > 0 ? S.B : 1;
    int64_t an = aic > 0 ? aic : 1;
    int64_t *mem = (int64_t *)calloc((size_t)(5 * Bn + 3 * an), sizeof(int64_t));
    if (!mem) return SASM_ERR_ARG;
    S.s1g_base = mem; S.s1g_tail = mem + Bn;
    S.bcost = mem + 2 * Bn; S.bblock = mem + 3 * Bn; S.blast = mem + 4 * Bn;
    int64_t *bn2_end = mem + 5 * Bn, *g_s1_end = bn2_end + an, *s2_end = g_s1_end + an;
    int rc = sched_run(&S, a, aic, bn2_end, g_s1_end, s2_end, out);
    free(mem);
    return rc;
}

static int sched_run(Sched *Sp, const SasmArgs *a, int64_t aic, int64_t *bn2_end, int64_t *g_s1_end,
                     int64_t *s2_end, int32_t *out) {
    Sched S = *Sp;
    int64_t used = 0;

    /* split info, metadata.py:671-683 */
    S.all_zero = 1;
    for (int64_t b = 0; b < S.B; ++b) {
        int64_t s1 = s1_size(&S, b), s2 = s2_size(&S, b);
        if (S.err) return S.err;
        S.s1g_base[b] = floordiv(s1 * S.G + S.m_base - 1, S.m_base);
        S.s1g_tail[b] = pymod(s1 * S.G, S.m_base);
        int64_t s2_base = floordiv(s2 + S2_BASE - 1, S2_BASE);
        if (S.s1g_base[b] != 0 && s2_base != 0) S.all_zero = 0;
    }
    if (S.all_zero) {
        /* metadata.py:959-964 */
        if (aic <= 0) return SASM_ERR_INDEX;
        used = 1;
        bn2_end[0] = S.B * a->num_heads_kv;
    } else {
        /* cost info, metadata.py:685-714 */
        for (int64_t b = 0; b < S.B; ++b) {
            S.bcost[b] = 0; S.bblock[b] = 0; S.blast[b] = 0;
            if (s1_size(&S, b) == 0 || s2_size(&S, b) == 0) continue;
            BatchC bc; RowC rc;
            memset(&bc, 0, sizeof(bc)); memset(&rc, 0, sizeof(rc));
            batch_cache(&S, b, &bc);
            for (int64_t i = 0; i < S.s1g_base[b]; ++i) {
                row_cache(&S, i, &bc, &rc);
                S.bcost[b] += rc.cost;
                S.bblock[b] += rc.block;
                if (rc.cost > S.max_row_cost) S.max_row_cost = rc.cost;
                if (rc.block > 0) S.blast[b] = rc.last_cost;
            }
            if (S.err) return S.err;
            S.total_cost += S.bcost[b] * a->num_heads_kv;
            S.total_block += S.bblock[b] * a->num_heads_kv;
        }
        /* split plan, metadata.py:898-923 */
        if (aic > 0) {
            Assign A;
            memset(&A, 0, sizeof(A));
            A.kv_split_part = 1; A.fd_data_num = 1;
            A.unassigned = S.total_cost;
            A.bn2_cost = S.bcost[0];
            A.bn2_block = S.bblock[0];
            batch_cache(&S, 0, &A.bc);
            row_cache(&S, 0, &A.bc, &A.rc);
            A.cur_s2 = A.rc.s2_start;
            int64_t max_cost = 0;
            for (int64_t i = 0; i < aic; ++i) {
                if (A.finished || A.unassigned <= 0) break;
                A.cur_core = i;
                /* metadata.py:872-896 */
                int64_t avg = floordiv(A.unassigned, imax(1, aic - A.cur_core));
                A.core_cost = 0; A.core_block = 0;
                A.core_limit = imax(avg, S.max_row_cost);
                by_batch(&S, &A);
                if (S.err) return S.err;
                by_row(&S, &A);
                if (S.err) return S.err;
                bn2_end[i] = A.cur_bn2;
                g_s1_end[i] = A.cur_s1g;
                s2_end[i] = A.cur_s2;
                max_cost = imax(max_cost, A.core_cost);
                A.unassigned -= A.core_cost;
                /* metadata.py:892-896: the FD record needs kv_split_part > 1,
                 * which cannot happen while supportFd is False. */
                if (A.rc.s2_start < A.cur_s2 && A.cur_s2 <= A.rc.s2_end) A.kv_split_part += 1;
            }
            used = A.cur_core + 1;
        }
        if (used < 1) used = 1;
    }

    /* gen_metadata, metadata.py:974-1009 */
    for (int64_t i = 0; i < AIC_CORE_NUM; ++i) {
        int32_t *row = out + i * FA_METADATA_SIZE;
        if (i >= used || i >= aic) continue;
        row[0] = 1;
        row[1] = (int32_t)(i == 0 ? 0 : bn2_end[i - 1]);
        row[2] = (int32_t)(i == 0 ? 0 : g_s1_end[i - 1]);
        row[3] = (int32_t)(i == 0 ? 0 : s2_end[i - 1]);
        row[4] = (int32_t)bn2_end[i];
        row[5] = (int32_t)g_s1_end[i];
        row[6] = (int32_t)s2_end[i];
        row[7] = 0; /* first FD workspace index: never set while supportFd is False */
    }
    /* FD rows (offset 288) stay zero: no FD head is ever recorded. */
    return SASM_OK;
}
