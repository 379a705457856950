/*
 * sas_b200.h -- C ABI of the B200-native sparse_attn_sharedkv operator.
 *
 * Drop-in boundary for the reference yangqiang2018/dsv4_planB
 * (sparse_attn_sharedkv_tilelang/).  Every entry point is stream-ordered,
 * takes plain device pointers and sizes, performs no host synchronisation
 * (except sas_read_status, whose job is to read a device word back), and
 * returns an int status (SAS_OK or an error below; sas_strerror names it).
 * The caller owns every buffer, including the workspace.  Pointers are CUDA
 * device pointers on the current device; `stream` is a cudaStream_t passed
 * as void* (NULL = the legacy default stream).
 */
#ifndef SAS_B200_H
#define SAS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SAS_ABI_VERSION 1

/* ---- status codes ------------------------------------------------------- */
enum {
    SAS_OK = 0,
    SAS_ERR_INVALID_ARG = 1,  /* a size, pointer or mode is outside the contract */
    SAS_ERR_UNSUPPORTED = 2,  /* valid for the reference, not implemented here */
    SAS_ERR_WORKSPACE = 3,    /* workspace missing or smaller than *_workspace_size */
    SAS_ERR_CUDA = 4,         /* a CUDA runtime call failed (launch, attribute, ...) */
    SAS_ERR_DEVICE = 5        /* sas_read_status found a device-side problem */
};

/* ---- device status bits (sas_read_status) ------------------------------- */
#define SAS_STATUS_BAD_INDEX 0x1u    /* a compressed index < -1 was skipped */
#define SAS_STATUS_BAD_BLOCK 0x2u    /* a block-table entry >= block_num, or a position past the
                                        table: the row was read as zeros */
#define SAS_STATUS_NO_PROGRESS 0x4u  /* metadata: the scheduler found no row with work where the
                                        reference loops forever (metadata.py:759-763) */
#define SAS_STATUS_WAIT_TIMEOUT 0x8u /* a bounded device-side wait gave up */
#define SAS_STATUS_BAD_TOKEN 0x10u   /* q_prefix[b] + s fell outside [0, num_tokens) */

typedef enum { SAS_DTYPE_BF16 = 0, SAS_DTYPE_FP16 = 1 } SasDtype;

/*
 * Kernel choice for sas_forward (SasFwdArgs.kernel).  SAS_KERNEL_TC: tensor
 * cores, a two-SM cluster per unit that splits the work by role (one SM
 * gathers K and computes S and P, the other gathers V and accumulates O).
 * SAS_KERNEL_TC2: tensor cores, a two-SM cluster that issues one
 * cta_group::2 MMA stream, each SM gathering half of every tile's key rows.
 * Both take the same shapes (D_qk 512 or 576, D_v 512, up to 128 heads).
 */
typedef enum { SAS_KERNEL_AUTO = 0, SAS_KERNEL_SIMT = 1, SAS_KERNEL_TC = 2, SAS_KERNEL_TC2 = 3 } SasKernel;

/*
 * Shape and mode of one sas_forward call.  Mirrors the compile-time
 * parameters of the reference kernel builder
 * (kernel.py:62-85 build_sparse_attn_sharedkv, keyed in api.py:81-101).
 */
typedef struct SasFwdArgs {
    int32_t batch;          /* B: entries of q_prefix/act_q_len/act_kv_len, rows of both tables */
    int32_t num_tokens;     /* T: rows of q, out, lse and cmp_indices */
    int32_t max_q_len;      /* max over requests of act_q_len (the reference's max_seq) */
    int32_t num_heads;      /* N1 query heads */
    int32_t num_kv_heads;   /* N2; must be 1 (api.py:279-282) */
    int32_t head_dim;       /* D_qk: row width of q and of both KV pools */
    int32_t v_head_dim;     /* D_v <= D_qk: V is the first D_v columns of the K=V row */
    int32_t ori_block_num, ori_block_size, ori_table_len;
    int32_t cmp_block_num, cmp_block_size, cmp_table_len;
    int32_t topk;           /* K: last dim of cmp_indices (scenario 3) */
    int32_t cmp_ratio;      /* compression ratio (scenarios 2, 3) */
    int32_t scenario;       /* 1 SWA, 2 CFA, 3 SCFA (api.py:196-202) */
    int32_t max_cmp_len;    /* scenario 2, sas_resolve_rows only: row capacity of its cmp_rows
                               export (>= max over requests of floor(act_kv / cmp_ratio)).
                               sas_forward needs no bound (0 is fine): it resolves CFA's dense
                               compressed range through the table in the attention kernel */
    int32_t ori_win_left;   /* sliding window: keys [s_g - ori_win_left, s_g] */
    int32_t ori_win_right;  /* must be 0 */
    int32_t ori_mask_mode;  /* must be 4 (band) */
    int32_t cmp_mask_mode;  /* must be 3 */
    int32_t dtype;          /* SasDtype of q, both pools and out */
    float softmax_scale;
    int32_t kernel;         /* SasKernel */
    int32_t flags;          /* SAS_FWD_FLAG_* bits (0: the reference's q_prefix / act_q_len inputs) */
    int32_t split_tiles;    /* 0, or a piece size in 64-key tiles: see below */
    int32_t reserved[4];    /* must be 0 */
} SasFwdArgs;

/*
 * SasFwdArgs.split_tiles.  The tensor-core path processes a batch as units
 * handed to its 74 two-SM clusters by a dynamic queue.  A unit is a whole
 * token, or, for batches of at most 37 tokens (SCFA), a piece of one: tokens
 * are then cut into pieces that fill the clusters and an LSE-combine kernel
 * merges them.  A host that knows its requests' lengths (the device tensors
 * hold them, so the library does not) may set split_tiles > 0 instead: every
 * SCFA token with more than split_tiles tiles of 64 keys is cut into pieces of
 * split_tiles tiles, whatever the batch size.  This balances batches of a few
 * long and many short requests, as a request shard of a multi-GPU batch is.
 * The workspace then holds a bf16 partial output per piece; a request whose
 * partials would exceed 1 GiB runs on whole tokens instead.  Ignored by the
 * CUDA-core kernel and for the SWA and CFA scenarios.
 */

/*
 * SasFwdArgs.flags.
 * SAS_FWD_FLAG_CU_SEQLENS: q_prefix points at cu_seqlens_q (batch + 1 entries,
 *   the TND layout's cumulative lengths) and act_q_len may be NULL; the kernels
 *   take act_q_len[b] = q_prefix[b + 1] - q_prefix[b].  A TND caller then needs
 *   no device work of its own before the call (no act_q_len subtraction kernel).
 *   No counterpart in the reference, whose API derives act_q_len with a tensor
 *   op (api.py:208-240).
 */
#define SAS_FWD_FLAG_CU_SEQLENS 0x1
/*
 * SAS_FWD_FLAG_TEST_STALL: test hook for the failure path of the tensor-core
 * kernel.  Its output CTAs withhold the release of their first P slot, so the
 * score CTA's bounded wait for that slot runs out: the call completes, the
 * status word reports SAS_STATUS_WAIT_TIMEOUT, and the context stays usable.
 * Nothing faults, traps or spins without bound.
 */
#define SAS_FWD_FLAG_TEST_STALL 0x100
/*
 * SAS_FWD_FLAG_LAZY_RESCALE: performance mode of the tensor-core kernel.  By
 * default its online softmax raises the running max on every increase, so P
 * is rounded to bf16 / fp16 at the scale the reference golden rounds it
 * (golden.py:186-194) and the reference's own low-precision acceptance
 * (test_sparse_attn_sharedkv.py:394-467) holds.  With this flag the max is
 * raised only when it grows by more than 8 (log2 units), so the 128 x 512
 * fp32 O accumulator is rarely rescaled (about 15 % faster at the c2 decode
 * shape); P is then rounded at another scale, and results stay within the
 * north-star bars against the fp32 golden.  Ignored by the CUDA-core kernel.
 * No counterpart in the reference.
 */
#define SAS_FWD_FLAG_LAZY_RESCALE 0x200

/* Bytes of workspace sas_forward needs for `args` (256-byte aligned base). */
int sas_workspace_size(const SasFwdArgs *args, size_t *bytes);

/*
 * Number of kernels one sas_forward call with `args` launches: the clear of the
 * workspace's status word and token records, key resolution, attention, and
 * the split-KV combine when the tensor-core path cuts tokens into pieces.  No
 * counterpart in the reference API: a launch count for profilers and
 * benchmarks.
 */
int sas_forward_kernel_count(const SasFwdArgs *args, int32_t *count);

/*
 * The fused attention.  Replaces the JIT kernel the reference API launches
 * (api.py:372-384; inputs kernel.py:209-237): the same eleven inputs in the
 * same order, then the two outputs, then the workspace and stream.
 *   q            [T, N1, D_qk]                      dtype
 *   ori_kv       [ori_block_num, ori_block_size, 1, D_qk]
 *   ori_block_table [B, ori_table_len] int32 (-1 = unmapped)
 *   cmp_kv       [cmp_block_num, cmp_block_size, 1, D_qk]   (scenarios 2, 3; else NULL)
 *   cmp_block_table [B, cmp_table_len] int32                (scenarios 2, 3; else NULL)
 *   cmp_indices  [T, 1, K] int32, -1 padded                  (scenario 3; else NULL)
 *   q_prefix     [B] int32: flat row of request b's first query token
 *                ([B + 1] cu_seqlens_q with SAS_FWD_FLAG_CU_SEQLENS)
 *   act_q_len    [B] int32 (NULL allowed with SAS_FWD_FLAG_CU_SEQLENS)
 *   act_kv_len   [B] int32 (seqused_kv)
 *   sinks        [N1] fp32
 *   metadata     int32[1024] from sas_metadata / the reference scheduler, or
 *                NULL.  Accepted for interface parity; the B200 kernels plan
 *                their own split over 148 SMs, so it is not read.
 *   out          [T, N1, D_v] dtype; rows of no (b, s < act_q_len[b]) are zeroed
 *   lse          [T, N1] fp32 natural-log LSE (sink folded in), or NULL
 * All tensors are dense.  The tensor-core kernel reads q, ori_kv and cmp_kv
 * through TMA tensor maps: their base addresses must be 16-byte aligned, else
 * the call returns SAS_ERR_INVALID_ARG.
 */
int sas_forward(const SasFwdArgs *args, const void *q, const void *ori_kv, const int32_t *ori_block_table,
                const void *cmp_kv, const int32_t *cmp_block_table, const int32_t *cmp_indices,
                const int32_t *q_prefix, const int32_t *act_q_len, const int32_t *act_kv_len,
                const float *sinks, const int32_t *metadata, void *out, float *lse, void *workspace,
                size_t workspace_bytes, void *stream);

/*
 * Backward pass (no counterpart in the reference, which has none,
 * test_graph_mode.py:314-324).  Same arguments as sas_forward up to sinks,
 * then the forward's out and lse, the gradient of out (dout, the layout and
 * dtype of out) and optionally of lse (dlse, fp32 [T][N1], NULL = zero), and
 * the gradients:
 *   dq        fp32 [T][N1][D_qk], written;
 *   d_ori_kv  fp32 [ori_block_num * ori_block_size][D_qk], added into;
 *   d_cmp_kv  fp32 [cmp_block_num * cmp_block_size][D_qk], added into
 *             (scenarios 2 and 3; may be NULL in scenario 1);
 *   d_sinks   fp32 [N1], added into.
 * K = V share a row, so a row's gradient holds its key and its value parts.
 * Rows are shared across tokens and heads and their gradients are summed with
 * atomics: the order of the sum, and so the last bits, vary between calls.
 * The softmax weights are differentiated exactly (the forward's rounding of P
 * to the input dtype is not).  Runs on CUDA cores for every shape with
 * D_qk <= 1024; args->kernel is ignored.  The workspace is sas_forward's
 * (sas_workspace_size).  dout and dq need 16-byte aligned bases.
 */
int sas_backward(const SasFwdArgs *args, const void *q, const void *ori_kv, const int32_t *ori_block_table,
                 const void *cmp_kv, const int32_t *cmp_block_table, const int32_t *cmp_indices,
                 const int32_t *q_prefix, const int32_t *act_q_len, const int32_t *act_kv_len, const float *sinks,
                 const void *out, const float *lse, const void *dout, const float *dlse, float *dq,
                 float *d_ori_kv, float *d_cmp_kv, float *d_sinks, void *workspace, size_t workspace_bytes,
                 void *stream);

/*
 * Index-handling export: runs only the key-resolution step of sas_forward and
 * copies, per flat token row, {b, s_global, ori_left, n_win, n_cmp, valid}
 * into token_info[T][8] (int32) and the physical compressed rows
 * (block * block_size + offset, or -1 for an unmapped block) into
 * cmp_rows[T][row_cap], row_cap = K (scenario 3) or max_cmp_len (scenario 2).
 * Same arguments as sas_forward minus the outputs.  No counterpart in the
 * reference API: it exposes what golden.py:28-66 computes, for parity tests.
 */
int sas_resolve_rows(const SasFwdArgs *args, const int32_t *ori_block_table, const int32_t *cmp_block_table,
                     const int32_t *cmp_indices, const int32_t *q_prefix, const int32_t *act_q_len,
                     const int32_t *act_kv_len, int32_t *token_info, int32_t *cmp_rows, void *workspace,
                     size_t workspace_bytes, void *stream);

/*
 * Shape of the split-KV plan sas_forward would run for `args` (host only, no
 * device work): the tensor-core path cuts every token of more than
 * *tiles_per_piece tiles of 64 keys into at most *pieces pieces; *pieces == 1
 * (and *tiles_per_piece == 0) means whole tokens.  The workspace then holds
 * partials for T x pieces slots: bf16 out [T][pieces][N1][D_v] and fp32
 * (m, l, lr, 0) [T][pieces][N1][4].  No counterpart in the reference.
 */
int sas_split_plan(const SasFwdArgs *args, int32_t *pieces, int32_t *tiles_per_piece);

/*
 * The split-KV plan of one sas_forward call with the same arguments, written to
 * metadata_out (device int32[1024]) in the layout of the reference's metadata
 * (metadata.py:38-60, packed at metadata.py:974-1009).  It completes what the
 * reference's scheduler declares but never enables (supportFd = False,
 * metadata.py:323-325; FD bookkeeping metadata.py:795-827, 925-954):
 *   - FA rows (ints 0..287): all zero.  The B200 kernel's 74 two-SM clusters take
 *     units (whole tokens, or pieces of split tokens) from a dynamic queue, so
 *     there is no static per-core range to describe.
 *   - FD row i (ints 288 + 8i .. +7, i < 72): the i-th token, in flat-row order,
 *     that the tensor-core kernel cuts into np > 1 pieces:
 *     {enable 1, bn2 = b (one KV head), m = s (query index in its request; the
 *     reference's mBaseSize is the group size, so its s1g index is s), ws_idx =
 *     t * pieces (first slot of the token in the partial buffers), ws_num = np,
 *     m_start = 0, m_num = N1 (the combine merges every head of the token), 0}.
 *     The Ascend meaning differs in m_start / m_num, which there split one
 *     token's heads across vector cores.
 *   - int 864 (zero in the reference): how many tokens are split; rows past the
 *     72nd are not listed.
 * Runs the key resolution (like sas_resolve_rows) into `workspace` (sized by
 * sas_workspace_size), then one small kernel.  No host synchronisation.
 */
int sas_split_metadata(const SasFwdArgs *args, const int32_t *ori_block_table, const int32_t *cmp_block_table,
                       const int32_t *cmp_indices, const int32_t *q_prefix, const int32_t *act_q_len,
                       const int32_t *act_kv_len, int32_t *metadata_out, void *workspace, size_t workspace_bytes,
                       void *stream);

/*
 * Reads the device status word a previous call on `workspace` left behind
 * (SAS_STATUS_* bits, 0 = clean).  Synchronises `stream`.
 */
int sas_read_status(const void *workspace, uint32_t *status, void *stream);

/*
 * sas_forward for callers that cannot allocate device memory.  Some hosts of
 * this operator own every byte of the GPU and forbid device allocations once
 * they are running -- a serving engine that reserves nearly all of HBM for its
 * paged KV pool up front, or a thin FFI host (ctypes, cgo) that embeds the op
 * with no device allocator of its own -- so they cannot provide the workspace
 * sas_forward asks for.  This entry point takes the same arguments minus the
 * workspace and uses a scratch array compiled into the library instead
 * (SAS_NOALLOC_SCRATCH_BYTES per GPU that loads the library, held until the
 * process exits).  It allocates nothing: no cudaMalloc, no cudaFree.
 *   - Calls whose sas_workspace_size exceeds SAS_NOALLOC_SCRATCH_BYTES are
 *     rejected with SAS_ERR_WORKSPACE (use sas_forward for those).
 *   - The first call on a device looks up the array's device address on the
 *     current device; make that first call before any stream capture.  The
 *     address is cached per device and CUDA context: after a cudaDeviceReset
 *     the next call looks it up again (again outside any capture).
 *   - Every call shares the one array: calls that overlap on the GPU (other
 *     streams, other host threads) race.  Serialise them on one stream.
 *   - The device status word lives in the private scratch: read it with
 *     sas_noalloc_read_status, not sas_read_status.
 * No counterpart in the reference.
 */
#define SAS_NOALLOC_SCRATCH_BYTES (16u << 20)
int sas_forward_noalloc(const SasFwdArgs *args, const void *q, const void *ori_kv, const int32_t *ori_block_table,
                        const void *cmp_kv, const int32_t *cmp_block_table, const int32_t *cmp_indices,
                        const int32_t *q_prefix, const int32_t *act_q_len, const int32_t *act_kv_len,
                        const float *sinks, const int32_t *metadata, void *out, float *lse, void *stream);

/*
 * The device status word (SAS_STATUS_* bits) the last sas_forward_noalloc call
 * on the current device left in the library's scratch array: bad indices or
 * table entries, or a bounded wait that gave up.  Synchronises `stream`;
 * allocates nothing.  No counterpart in the reference.
 */
int sas_noalloc_read_status(uint32_t *status, void *stream);

/* ---- metadata scheduler ----------------------------------------------------
 * Replaces sparse_attn_sharedkv_metadata (metadata.py:1018-1086, the Python
 * port of the aicpu SparseAttnSharedkvMetadata op) with a CUDA kernel whose
 * int32[1024] output is bit-identical to it.
 */
typedef enum { SAS_LAYOUT_BSND = 0, SAS_LAYOUT_BSH = 1, SAS_LAYOUT_TND = 2, SAS_LAYOUT_OTHER = 3 } SasLayoutQ;
typedef enum { SAS_LAYOUT_PA_ND = 0, SAS_LAYOUT_KV_TND = 1 } SasLayoutKv;

typedef struct SasMetaArgs {
    int32_t num_heads_q, num_heads_kv, head_dim;
    int32_t n_cu_seqlens_q;      /* entries of cu_seqlens_q (0 = absent) */
    int32_t n_cu_seqlens_ori_kv; /* entries of cu_seqlens_ori_kv (0 = absent) */
    int32_t n_seqused_q;         /* entries of seqused_q (0 = absent) */
    int32_t n_seqused_kv;        /* entries of seqused_kv (0 = absent) */
    int32_t batch_size, max_seqlen_q, max_seqlen_kv;
    int32_t ori_topk, cmp_topk, cmp_ratio;
    int32_t ori_mask_mode, cmp_mask_mode, ori_win_left, ori_win_right;
    int32_t layout_q;            /* SasLayoutQ */
    int32_t layout_kv;           /* SasLayoutKv */
    int32_t has_ori_kv, has_cmp_kv;
    int32_t aic_core_num, aiv_core_num;
    int32_t reserved[5];
} SasMetaArgs;

int sas_metadata_workspace_size(const SasMetaArgs *args, size_t *bytes);

/* metadata_out: device int32[1024]. */
int sas_metadata(const SasMetaArgs *args, const int32_t *cu_seqlens_q, const int32_t *cu_seqlens_ori_kv,
                 const int32_t *seqused_q, const int32_t *seqused_kv, int32_t *metadata_out, void *workspace,
                 size_t workspace_bytes, void *stream);

/*
 * Measurement aid: when both are non-NULL, sas_forward calls made afterwards
 * by this host thread record `start_event` / `stop_event` (cudaEvent_t) on
 * their stream immediately before and after the attention kernel itself, so
 * a caller can time that kernel alone.  NULL, NULL switches it off.  Results
 * are unaffected.  No counterpart in the reference.
 */
int sas_set_kernel_events(void *start_event, void *stop_event);

/* ---- misc ---------------------------------------------------------------- */
const char *sas_strerror(int status);
int sas_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* SAS_B200_H */
