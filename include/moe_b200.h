/*
 * moe_b200.h -- C ABI of the B200 (sm_100a) fused Mixture-of-Experts operator.
 *
 * This is the drop-in boundary for the fused-MoE operator of the kernelswift
 * track-1 suite. The reference operator is the pure-torch
 * `Model.forward(hidden_states, router_logits)` of
 * kernels/track1-triton/fused_moe/base.py:35-76; each entry point below names
 * the lines of that file (or of the library pipeline in
 * kernels/track1-triton/fused_moe/mlu/triton_fused_moe_006.py) whose work it
 * replaces.
 *
 * Conventions shared by every entry point:
 *   - All tensor arguments are raw device pointers to dense row-major arrays.
 *     Row, weight, output and workspace pointers are 16-byte aligned (the
 *     kernels move them in 16-byte vectors, TMA and bulk copies); the
 *     compute entry points refuse others with MOE_ERR_INVALID_ARG. Ids,
 *     routing weights and fp32 block scales need only element alignment.
 *   - Memory is owned by the caller. Entry points that need temporary device
 *     memory take a `workspace` pointer and its size; the matching
 *     *_workspace_size() query returns the required number of bytes.
 *   - Work is enqueued on the caller's CUDA stream (`stream` is a
 *     cudaStream_t passed as void*; NULL means the legacy default stream).
 *     Nothing synchronises the host unless the entry point says so.
 *   - Every entry point returns a moe_status_t. Arguments are validated on the
 *     host before anything is launched; a failed validation launches nothing.
 *     moe_last_error() returns a thread-local message for the last failure.
 *   - Kernels that wait on on-chip barriers wait with a time limit. When a
 *     wait runs out, the kernel stores MOE_ERR_TIMEOUT into the optional
 *     device status word (`status`, may be NULL) and returns; the CUDA
 *     context stays usable. moe_read_status() copies that word to the host.
 */
#ifndef MOE_B200_H_
#define MOE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_B200_ABI_VERSION 2

typedef enum moe_status {
  MOE_OK = 0,
  MOE_ERR_INVALID_ARG = 1,  /* bad pointer, size, dtype or layout            */
  MOE_ERR_UNSUPPORTED = 2,  /* valid request this build does not implement   */
  MOE_ERR_CUDA = 3,         /* a CUDA runtime/driver call failed             */
  MOE_ERR_TIMEOUT = 4,      /* a device-side bounded wait ran out            */
  MOE_ERR_WORKSPACE = 5,    /* workspace missing or smaller than required    */
  MOE_ERR_DEVICE = 6        /* current device is not an sm_100 part          */
} moe_status_t;

typedef enum moe_dtype {
  MOE_DTYPE_F32 = 0,
  MOE_DTYPE_F16 = 1,
  MOE_DTYPE_BF16 = 2,
  MOE_DTYPE_E4M3 = 3,       /* float8_e4m3fn                                  */
  MOE_DTYPE_I8 = 4,
  MOE_DTYPE_I32 = 5,
  MOE_DTYPE_I64 = 6
} moe_dtype_t;

typedef enum moe_quant {
  MOE_QUANT_NONE = 0,         /* bf16/fp16 weights and activations            */
  MOE_QUANT_FP8_BLOCK = 1,    /* e4m3 W8A8: weight scales per 128x128 block,
                                 activation scales per token per 128 columns  */
  MOE_QUANT_INT8_CHANNEL = 2, /* int8 W8A8: weight scale per output channel,
                                 activation scale per token                   */
  MOE_QUANT_FP8_UE8M0 = 3     /* e4m3 W8A8 with power-of-two (UE8M0) scales,
                                 the FP8_BLOCK granularity, applied by the
                                 tensor core; scales travel as scale-factor
                                 images (below)                                */
} moe_quant_t;

/*
 * MOE_QUANT_FP8_UE8M0 scales. A scale is one byte b meaning 2^(b - 127); it
 * is the smallest power of two s with absmax / s <= 448 over its group (a
 * 128x128 weight block, or 128 columns of one activation row), 127 (s = 1)
 * for an all-zero group; q = e4m3_rn(x / s). The tensor core applies the
 * scales itself (tcgen05.mma kind::mxf8f6f4.block_scale), so the products of
 * every k-block accumulate in tensor memory with no per-block promotion.
 *
 * The scales of a matrix group g (expert g of a weight tensor; g = 0 for the
 * gathered activations) with R rows and KB = C / 128 column blocks are stored
 * as a "scale-factor image" of 512-byte chunks, one chunk per 128 rows and 4
 * column blocks, in the order the tensor memory copy (tcgen05.cp 32x128b)
 * takes them. The scale of row r, column block kb is the byte at
 *   ((g * Q + kb / 4) * RS + r / 128) * 512
 *     + 16 * (r % 32) + 4 * ((r % 128) / 32) + kb % 4
 * with Q = ceil(KB / 4) and RS = ceil(R / 128). For the gate/up weights, r is
 * the row of the regrouped w13 (each row carries the scale of its block in
 * the original w1 layout).
 */
int64_t moe_ue8m0_scale_bytes(int64_t groups, int64_t rows, int64_t cols);

/* ------------------------------------------------------------------------ */
/* Status helpers                                                           */
/* ------------------------------------------------------------------------ */

/* Name of a status code ("MOE_OK", ...). Never returns NULL. */
const char* moe_status_string(int status);

/* Thread-local detail message of the last non-OK status returned on this
 * host thread ("" when none). */
const char* moe_last_error(void);

/* ABI version of the loaded library (MOE_B200_ABI_VERSION). */
int moe_abi_version(void);

/* Synchronises `stream`, copies the device status word to *host_status and,
 * when `reset` is non-zero, clears it. */
int moe_read_status(int32_t* device_status, int32_t* host_status, int reset,
                    void* stream);

/* ------------------------------------------------------------------------ */
/* Routing: softmax -> top-k -> renormalise -> cast                          */
/* Replaces base.py:44-48 (torch.softmax, torch.topk, the renormalising      */
/* division and the cast of the weights to the activation dtype).           */
/* ------------------------------------------------------------------------ */

/*
 * For every token t: w_e = exp(l_e - max) / sum_e' exp(l_e' - max) over the
 * router logits l = router_logits[t, :] (fp32 arithmetic); the top_k experts
 * by logit, largest first, ties broken by the lower expert index (softmax is
 * strictly increasing, so this is the top-k of the probabilities); with
 * renormalize != 0 each selected weight is divided by the sum of the
 * selected weights. Writes topk_weights [T, top_k] (F32/F16/BF16) and
 * topk_ids [T, top_k] (I32/I64). logits dtype F32/F16/BF16;
 * 1 <= num_experts <= 1024, 1 <= top_k <= min(32, num_experts).
 */
int moe_topk_softmax(const void* router_logits, int logits_dtype,
                     int64_t num_tokens, int num_experts, int top_k,
                     int renormalize, void* topk_weights, int weights_dtype,
                     void* topk_ids, int ids_dtype, void* stream);

/* ------------------------------------------------------------------------ */
/* Routing metadata: moe_align_block_size                                   */
/* Replaces the per-expert grouping of base.py:64-68 (`mask = flat_ids == e`,
 * `x_rep[mask]`) and tmo.moe_gen_idx of triton_fused_moe_006.py:38.         */
/* ------------------------------------------------------------------------ */

/* Number of int32 entries of `sorted_token_ids`:
 * round_up(numel + num_experts * (block_m - 1), block_m).
 * `expert_ids` has moe_align_buffer_len(...) / block_m entries. */
int64_t moe_align_buffer_len(int64_t numel, int num_experts, int block_m);

/* Bytes of workspace moe_align_block_size needs for this problem. */
int moe_align_workspace_size(int64_t numel, int num_experts, int block_m,
                             size_t* bytes);

/*
 * Groups the flat (token, slot) assignments `topk_ids[numel]` by expert.
 *
 * For flat index r (= token * top_k + slot, the row order of base.py:52-58):
 *   cnt[e]    = #{r : topk_ids[r] == e}
 *   padded[e] = ceil(cnt[e] / block_m) * block_m
 *   off[e]    = sum of padded[e'] for e' < e
 *   sorted_token_ids[off[e] + j] = j-th r (ascending) with topk_ids[r] == e
 *   padding slots and the tail up to the buffer length hold `numel`
 *   expert_ids[b] = e for every block b of expert e, -1 for unused blocks
 *   *num_tokens_post_pad = sum of padded[e]
 * Ids outside [0, num_experts) are dropped (used by expert parallelism).
 * Bit-exact and deterministic: no atomics decide an element's position.
 *
 * ids_dtype: MOE_DTYPE_I32 or MOE_DTYPE_I64. Requires 1 <= num_experts <= 1024,
 * block_m in {16, 32, 64, 128, 256}.
 */
int moe_align_block_size(const void* topk_ids, int ids_dtype, int64_t numel,
                         int num_experts, int block_m,
                         int32_t* sorted_token_ids, int32_t* expert_ids,
                         int32_t* num_tokens_post_pad, void* workspace,
                         size_t workspace_bytes, void* stream);

/*
 * Same result as moe_align_block_size, but allocates nothing and takes no
 * workspace. No counterpart in the reference: this entry point exists for
 * callers that cannot allocate device memory -- e.g. a serving runtime that
 * has given all free HBM to its own pool and offers operators no workspace,
 * or a latency-critical path that must not call cudaMalloc because it can
 * synchronise the device.
 *
 * Its scratch is one static device array of MOE_ALIGN_NOALLOC_SCRATCH_BYTES
 * (1 MiB) that every GPU loading the library holds until the process exits.
 * Problems needing more (more than MOE_ALIGN_NOALLOC_SCRATCH_BYTES / 4 ints of
 * per-chunk histograms: ceil(numel / 4096) * num_experts) are rejected with
 * MOE_ERR_UNSUPPORTED and a message; up to 8192 ids need no scratch at all.
 * The first call on each device looks up the array's device address with
 * cudaGetSymbolAddress (that device must be current) and should come before
 * any stream capture. The address is kept for the life of the process: after
 * cudaDeviceReset of a device (or any teardown of its primary context) the
 * library may be loaded again at another address, so do not call this entry
 * point on that device again in the same process. All calls share the
 * array: calls whose work overlaps on the GPU race on it, so order them on
 * one stream or with events. Nothing in the array has to start at zero.
 */
#define MOE_ALIGN_NOALLOC_SCRATCH_BYTES (1u << 20)
int moe_align_block_size_noalloc(const void* topk_ids, int ids_dtype,
                                 int64_t numel, int num_experts, int block_m,
                                 int32_t* sorted_token_ids, int32_t* expert_ids,
                                 int32_t* num_tokens_post_pad, void* stream);

/* ------------------------------------------------------------------------ */
/* Weight preparation (one-time per weight version)                         */
/* Replaces the per-call casts `self.w1.to(dtype)` / `self.w2.to(dtype)` of
 * base.py:60-61.                                                           */
/* ------------------------------------------------------------------------ */

/*
 * w1 [E, 2I, H] (gate rows [0, I), up rows [I, 2I), base.py:25-27,70) ->
 * w13 [E, 2I, H] in the layout the gate/up GEMM reads: rows are regrouped in
 * 16-row pairs, w13 row 32g + c = w1 row 16g + c (gate) and
 * w13 row 32g + 16 + c = w1 row I + 16g + c (up), c in [0, 16).
 *
 * quant == MOE_QUANT_NONE:   src F32/F16/BF16 -> dst_dtype F16/BF16 (cast).
 * quant == MOE_QUANT_FP8_BLOCK: src F32/F16/BF16 is quantised to e4m3 with one
 *   scale per 128x128 block of the ORIGINAL layout, scale = absmax / 448;
 *   `scale_out` receives [E, ceil(2I/128), ceil(H/128)] fp32.
 *   src E4M3 is taken as already quantised: rows are regrouped and
 *   `scale_in` ([E, ceil(2I/128), ceil(H/128)]) is copied to `scale_out`.
 * quant == MOE_QUANT_INT8_CHANNEL: src F32/F16/BF16 is quantised to int8 with
 *   one scale per output row, scale = absmax / 127; `scale_out` receives
 *   [E, 2I] fp32 in the regrouped row order.
 * quant == MOE_QUANT_FP8_UE8M0: src F32/F16/BF16 is quantised to e4m3 with one
 *   power-of-two scale per 128x128 block of the original layout; `scale_out`
 *   (cast to float*, moe_ue8m0_scale_bytes(E, 2I, H) bytes) receives the
 *   scale-factor image. Requires I % 128 == 0 and H % 128 == 0.
 * Requires I % 16 == 0 and H % 16 == 0.
 */
int moe_prepare_w13(const void* w1, int src_dtype, const float* scale_in,
                    int64_t num_experts, int64_t inter_size,
                    int64_t hidden_size, int quant, void* w13_out,
                    int dst_dtype, float* scale_out, void* stream);

/*
 * w2 [E, H, I] (base.py:29-31) -> the down-projection operand, same layout.
 * quant NONE: cast. FP8_BLOCK: e4m3 + [E, ceil(H/128), ceil(I/128)] scales
 * (or pass-through of an already-e4m3 source with `scale_in`). INT8_CHANNEL:
 * int8 + [E, H] scales. FP8_UE8M0: e4m3 + the scale-factor image
 * (moe_ue8m0_scale_bytes(E, H, I) bytes).
 */
int moe_prepare_w2(const void* w2, int src_dtype, const float* scale_in,
                   int64_t num_experts, int64_t hidden_size,
                   int64_t inter_size, int quant, void* w2_out, int dst_dtype,
                   float* scale_out, void* stream);

/* ------------------------------------------------------------------------ */
/* The fused expert computation                                             */
/* Replaces base.py:50-76: the replicate (52-58), the per-expert loop of
 * gate/up GEMM, SiLU(gate)*up and down GEMM (64-72) and the weighted top-k
 * reduction (75-76); equivalently group_gemm x2 + combine of
 * triton_fused_moe_006.py:40-65.                                           */
/* ------------------------------------------------------------------------ */

typedef struct moe_problem {
  int64_t num_tokens;       /* T                                             */
  int64_t hidden_size;      /* H                                             */
  int64_t inter_size;       /* I                                             */
  int32_t num_experts;      /* E experts held by this process                */
  int32_t top_k;            /* k                                             */
  int32_t act_dtype;        /* hidden/out dtype: F32, F16 or BF16            */
  int32_t quant;            /* moe_quant_t                                   */
  int32_t ids_dtype;        /* I32 or I64                                    */
  int32_t weights_dtype;    /* topk_weights dtype: F32, F16 or BF16          */
  const void* hidden;       /* [T, H] act_dtype                              */
  const void* w13;          /* moe_prepare_w13 output [E, 2I, H]             */
  const void* w2;           /* moe_prepare_w2 output  [E, H, I]              */
  const float* w13_scale;   /* per moe_prepare_w13 (NULL for QUANT_NONE)     */
  const float* w2_scale;    /* per moe_prepare_w2  (NULL for QUANT_NONE)     */
  const void* topk_weights; /* [T, k] weights_dtype                          */
  const void* topk_ids;     /* [T, k] ids_dtype; ids outside [0,E) are dropped*/
  void* out;                /* [T, H] act_dtype                              */
  int32_t* status;          /* optional device status word (may be NULL)     */
  void** stage_events;      /* optional cudaEvent_t[MOE_NUM_STAGES + 1]: event
                               i is recorded on `stream` before stage i and
                               event MOE_NUM_STAGES after the last one, for
                               per-kernel timing (may be NULL)               */
  const int32_t* num_tokens_dev; /* optional device int: only tokens
                               t < *num_tokens_dev (<= num_tokens) take part;
                               the rest are neither read nor written. Lets an
                               expert-parallel receive buffer sized for the
                               worst case be processed at the size it got
                               this step without a host sync (NULL: all
                               num_tokens). Not with the decode path's sizes
                               (at most 16 routed rows).                     */
} moe_problem_t;

/* Stages of moe_fused_experts, in launch order (for stage_events). */
#define MOE_STAGE_ALIGN 0
#define MOE_STAGE_GATHER 1
#define MOE_STAGE_GATE_UP 2
#define MOE_STAGE_QUANT 3
#define MOE_STAGE_DOWN 4
#define MOE_STAGE_SUM 5
#define MOE_NUM_STAGES 6

/* Bytes of workspace moe_fused_experts needs for `p` (pointers unused). */
int moe_fused_experts_workspace_size(const moe_problem_t* p, size_t* bytes);

/*
 * out[t] = sum_j topk_weights[t, j] *
 *          W2[e] . (silu(W1g[e] . x_t) * (W1u[e] . x_t)),  e = topk_ids[t, j]
 * Matmuls run on the tcgen05 tensor cores (bf16/fp16, tf32, e4m3 or int8
 * operands, fp32/int32 accumulation in tensor memory); SiLU, scaling and the
 * top-k sum run in fp32. F32 activations with unquantised weights take tf32
 * MMAs: the weights (prepared as F32) and the operand rows are rounded to
 * tf32 (10-bit mantissa, nearest, ties away from zero) where they are
 * written. The operand rows are gathered token by token (each token read
 * and, for fp8, quantised once; MOE_NO_TOKEN_GATHER=1 gathers them row by
 * row, with the same bytes). With at most
 * 16 routed rows, 16-bit activations, unquantised weights and at most 256 MB
 * of weights to stream, two weight-streaming CUDA-core kernels do the whole
 * computation instead (fp32 dot products; MOE_NO_DECODE_PATH=1 disables
 * them). Kernels are launched with programmatic dependent launch
 * (MOE_NO_PDL=1 disables it).
 * hidden, w13, w2, out, workspace and the INT8_CHANNEL / FP8_UE8M0 weight
 * scales must be 16-byte aligned (the kernels move them in 16-byte vectors
 * and bulk copies; FP8_BLOCK scales need only float alignment); otherwise
 * MOE_ERR_INVALID_ARG, checked before anything else.
 */
int moe_fused_experts(const moe_problem_t* p, void* workspace,
                      size_t workspace_bytes, void* stream);

/*
 * The whole forward of base.py:35-76 in one call: routing of
 * router_logits [T, num_experts] (F32, F16 or BF16) as moe_topk_softmax does
 * it (softmax in fp32, top-k, renormalised when `renormalize`; base.py:44-48)
 * into p->topk_weights / p->topk_ids -- OUTPUTS here, [T, k] in
 * p->weights_dtype / p->ids_dtype -- then moe_fused_experts with those
 * weights (moe_topk_softmax's kernel, then moe_fused_experts' launches, on
 * `stream`; on the decode path -- at most 16 routed rows -- with F32 logits
 * over at most 256 experts the first decode kernel routes the tokens itself,
 * with the same code, and no routing kernel is launched). Workspace as for
 * moe_fused_experts_workspace_size. Replaces Model.forward (base.py:35-76).
 */
int moe_fused_moe(const moe_problem_t* p, const void* router_logits, int logits_dtype,
                  int renormalize, void* workspace, size_t workspace_bytes, void* stream);

/* Number of kernels moe_fused_moe launches for `p` with logits of
 * `logits_dtype` (pointers unused; answers without a GPU). No reference
 * counterpart (measurement aid). */
int moe_fused_moe_launches(const moe_problem_t* p, int logits_dtype, int* launches);

/* moe_fused_experts for top_k == 1 where only the rows of tokens with a
 * valid expert id are wanted (the expert-parallel receive buffer): out[t] =
 * w[t] * expert(x_t) for those tokens; rows of tokens whose id is dropped are
 * unspecified (moe_fused_experts writes zeros there). When the down
 * GEMM runs without a K split its epilogue writes these rows directly and
 * no top-k sum is launched. No reference counterpart (an expert-parallel
 * building block). */
int moe_fused_experts_rows(const moe_problem_t* p, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Number of kernels moe_fused_experts (rows_only = 0) or
 * moe_fused_experts_rows (rows_only = 1) launches for `p` (pointers unused;
 * answers without a GPU). No reference counterpart (measurement aid). */
int moe_fused_experts_launches(const moe_problem_t* p, int rows_only, int* launches);

/* The plan moe_fused_experts makes for `p` (pointers unused; answers without
 * a GPU, for 148 SMs): info[0] gate-up tile width, [1] gate-up K splits,
 * [2] down tile width, [3] down K splits, [4] dtype of the down GEMM's rows,
 * [5] 1 when the operand rows are gathered token by token (the align's
 * slot map; 0 for the row-major gather, MOE_NO_TOKEN_GATHER=1, int8, or the
 * decode kernels), [6] 1 when the decode kernels run instead of the GEMM
 * pipeline, [7] SMs planned for. No reference counterpart (inspection aid). */
int moe_fused_experts_plan(const moe_problem_t* p, int32_t* info);

/* ------------------------------------------------------------------------ */
/* The stages of moe_fused_experts, one entry point each. Used by the expert-
 * parallel path (which inserts the token exchange between them) and by tests.
 * `buffer_len` is moe_align_buffer_len(numel, E, 128); the grouped GEMMs need
 * routing metadata made with block_m = 128.                                */
/* ------------------------------------------------------------------------ */

/*
 * dst[m] = src[sorted_token_ids[m] / top_k] for m < *num_tokens_post_pad whose
 * slot is not padding (base.py:52-58 replicate + base.py:68 gather); padding
 * rows are left untouched. top_k == 0 copies row m itself (valid rows only).
 * quant NONE: dst_dtype F16/BF16 (F32 sources are rounded), or F32 from
 *   F32 rows rounded to tf32 (nearest, ties away: the operand of the tf32
 *   GEMMs that fp32 activations use).
 * quant FP8_BLOCK: dst e4m3 + dst_scale [buffer_len, ceil(H/128)],
 *   scale = absmax/448 per 128 columns. INT8_CHANNEL: dst int8 + dst_scale
 *   [buffer_len], scale = absmax/127 per row. FP8_UE8M0: dst e4m3 +
 *   dst_scale (cast to float*) the scale-factor image of the rows,
 *   moe_ue8m0_scale_bytes(1, buffer_len, H) bytes; H % 128 == 0.
 */
int moe_gather_rows(const void* src, int src_dtype, int64_t src_rows,
                    int64_t hidden_size, int top_k,
                    const int32_t* sorted_token_ids,
                    const int32_t* num_tokens_post_pad, int64_t buffer_len,
                    int64_t numel, int quant, void* dst, int dst_dtype,
                    float* dst_scale, void* stream);

/*
 * act[m, :] = silu(gate) * up for every operand row m of a used block whose
 * slot is not padding, gate/up = a[m] . w13[e]^T (base.py:69-71).
 * act_out: [buffer_len, I] in compute_dtype (bf16 for the W8A8 modes).
 * FP8_UE8M0: a_scale and w13_scale are scale-factor images (cast to float*).
 * block_n: 0 picks the N tile, else 64, 128 or 256 (128 or 256 for fp8).
 */
int moe_gemm_gate_up(int quant, int compute_dtype, const void* a,
                     const float* a_scale, const void* w13,
                     const float* w13_scale, const int32_t* sorted_token_ids,
                     const int32_t* expert_ids,
                     const int32_t* num_tokens_post_pad, int64_t buffer_len,
                     int64_t numel, int num_experts, int64_t hidden_size,
                     int64_t inter_size, void* act_out, int block_n,
                     int32_t* status, void* stream);

/*
 * partial[s, r, :] = row_weights[r] * (act[m] . w2[e]^T over K split s) for
 * r = sorted_token_ids[m] (base.py:72 and the weight multiply of base.py:75).
 * partial_out: [splits, numel, H] fp32; rows of dropped slots are not written.
 * `splits` must leave no split empty: with kb = ceil(I * elem_bytes / 128)
 * k-blocks, ceil(kb / ceil(kb / splits)) == splits.
 * FP8_UE8M0: act_scale and w2_scale are scale-factor images (cast to float*).
 */
int moe_gemm_down(int quant, int compute_dtype, const void* act,
                  const float* act_scale, const void* w2,
                  const float* w2_scale, const int32_t* sorted_token_ids,
                  const int32_t* expert_ids, const int32_t* num_tokens_post_pad,
                  int64_t buffer_len, int64_t numel, int num_experts,
                  int64_t hidden_size, int64_t inter_size,
                  const void* row_weights, int weights_dtype, int splits,
                  float* partial_out, int block_n, int32_t* status,
                  void* stream);

/*
 * out[t, :] = sum_j sum_s partial[s, t*top_k + j, :] over slots whose id is in
 * [0, num_experts) (all slots when topk_ids is NULL), in fixed order, fp32,
 * then cast to out_dtype (base.py:75-76).
 */
int moe_sum_topk(const float* partial, int splits, int64_t num_tokens,
                 int top_k, int64_t hidden_size, const void* topk_ids,
                 int ids_dtype, int num_experts, void* out, int out_dtype,
                 void* stream);

/*
 * Expert-parallel combine on the token's own rank: rows[inv_index[r]] is the
 * expert output for flat slot r = t*top_k + j (computed on whichever rank
 * holds that expert and sent back);
 *   out[t, :] = sum_j weights[r] * rows[inv_index[r], :]   (j ascending, fp32)
 * Slots with inv_index < 0 contribute nothing. rows and out share a dtype
 * (F32/F16/BF16). The weighted top-k reduction of base.py:75-76 for rows
 * that were not computed locally.
 */
int moe_combine_rows(const void* rows, int rows_dtype, const int32_t* inv_index,
                     const void* weights, int weights_dtype, int64_t num_tokens,
                     int top_k, int64_t hidden_size, void* out, int out_dtype,
                     void* stream);

/*
 * Grouped top-k routing of kernels/track1-triton/groupedtopk/base.py:31-72
 * (Model.forward): scores = softmax (scoring_func 0) or sigmoid (1) of
 * gating_output [num_tokens, num_experts] (F32/F16/BF16); the experts form
 * num_expert_group equal groups; the topk_group groups with the highest
 * maximum score are kept and the top_k experts are chosen among them, in
 * descending score order; topk_weights (fp32) = their scores, divided by
 * their sum when renormalize, times routed_scaling_factor; topk_ids int32.
 * Ties go to the lower index. num_experts <= 1024, num_expert_group <= 32,
 * top_k <= min(32, topk_group * num_experts / num_expert_group).
 */
int moe_grouped_topk(const void* gating_output, int logits_dtype, int64_t num_tokens,
                     int num_experts, int top_k, int renormalize, int num_expert_group,
                     int topk_group, int scoring_func, float routed_scaling_factor,
                     float* topk_weights, int32_t* topk_ids, void* stream);

/*
 * Expert-parallel dispatch plan for this rank's routing (experts sharded in
 * contiguous blocks of num_experts / world per rank). For flat slot r with
 * expert id e = topk_ids[r] and destination rank d = e / (num_experts/world):
 *   order[p]     slot at send position p: slots grouped by d (ascending),
 *                ascending r within a rank; send positions run over
 *                [0, counts[0] + ... + counts[world-1])
 *   send_eid[p]  e - d * (num_experts / world), the id on the receiving rank
 *   inv_index[r] send position of slot r (-1 for ids outside [0, num_experts))
 *   counts[d]    slots for rank d (int64, d < world); counts[world] = slots
 *                with ids outside [0, num_experts)
 * order/send_eid/inv_index hold numel int32 each; counts world + 1 int64.
 * Deterministic (stable counting sort, no atomics decide positions).
 * Replaces the per-expert grouping of base.py:64-68 across ranks.
 * 1 <= world <= 128.
 */
int moe_ep_plan(const void* topk_ids, int ids_dtype, int64_t numel,
                int num_experts, int world, int32_t* order, int32_t* send_eid,
                int32_t* inv_index, int64_t* counts, void* stream);

/* moe_ep_plan with the slots spread over CTAs when there are more than 8192
 * (three launches: per-chunk histograms, a scan, the placement; one CTA
 * otherwise). Same outputs, bit for bit. `workspace` holds
 * moe_ep_plan_workspace_size bytes (0 up to 8192 slots). */
int moe_ep_plan_workspace_size(int64_t numel, int world, size_t* bytes);
int moe_ep_plan_ws(const void* topk_ids, int ids_dtype, int64_t numel,
                   int num_experts, int world, int32_t* order, int32_t* send_eid,
                   int32_t* inv_index, int64_t* counts, void* workspace,
                   size_t workspace_bytes, void* stream);

/*
 * Deduplicated send plan: one send row per (token, destination rank) that
 * holds any of the token's k slots, so a token crosses to a rank once
 * however many of its experts live there (top-8 of 256 experts over 8 ranks
 * reaches about 5.3 ranks per token). Rows are grouped by rank (ascending),
 * tokens ascending inside a rank; for send row p:
 *   send_token[p]        the token (row of hidden_states)
 *   send_eid[p*k + j]    topk_ids[t, j] - d * E_local when slot j is on rank d,
 *                        else -1
 *   send_w[p*k + j]      topk_weights[t, j] (as f32) for those slots, else 0
 * inv_index[t*world + d] = the row of (t, d), -1 when the token has no slot
 * on d; counts[d] = rows for rank d (d < world), counts[world] = tokens with
 * an id outside [0, num_experts). Outputs hold num_tokens * world rows at
 * most. One CTA; deterministic. Replaces the cross-rank grouping of
 * base.py:64-68. 1 <= world <= 32, num_experts % world == 0.
 */
int moe_ep_plan_dedup(const void* topk_ids, int ids_dtype, const void* topk_weights,
                      int weights_dtype, int64_t num_tokens, int top_k, int num_experts,
                      int world, int32_t* send_token, int32_t* send_eid, float* send_w,
                      int32_t* inv_index, int64_t* counts, void* stream);

/* ------------------------------------------------------------------------ */
/* Expert parallelism over NVLink peer memory. No reference counterpart (the */
/* reference has no expert parallelism): it replaces, across the ranks of    */
/* one node, the per-expert loop and weighted sum of                         */
/* kernels/track1-triton/fused_moe/base.py:64-76, with token rows moved by   */
/* the dispatch and combine kernels themselves (stores into and loads from   */
/* the other GPUs' buffers) and no host synchronisation.                     */
/*                                                                          */
/* Each rank owns one device buffer (created here, shared with the others   */
/* through CUDA IPC handles): a control block, `capacity` x top_k received   */
/* expert ids and weights, `capacity` received rows and `capacity` result    */
/* rows of hidden_size act_dtype (F16/BF16) elements. A token travels to a   */
/* rank once, with its top_k ids local to that rank (-1 for slots held       */
/* elsewhere) and their weights. One step, all on the caller's stream:       */
/*   moe_ep_plan_dedup -> moe_ep_peer_dispatch -> moe_fused_experts over the */
/*   received rows (num_tokens = capacity, top_k = k, ids and weights from   */
/*   the buffer, num_tokens_dev = the received-count word, out = the result  */
/*   rows: each the weighted sum over the slots this rank holds)            */
/*   -> moe_ep_peer_combine (out[t] = sum over the ranks of their rows).    */
/* Every rank must take every step. Waits on other ranks are bounded;       */
/* on expiry, or when a rank would receive more than `capacity` rows, the    */
/* kernels store an error code (MOE_ERR_TIMEOUT / MOE_ERR_WORKSPACE) in the  */
/* optional device status word and skip their work.                         */
/* ------------------------------------------------------------------------ */
#define MOE_EP_MAX_RANKS 8
#define MOE_EP_HANDLE_BYTES 64

typedef struct moe_ep_peer moe_ep_peer_t;

/* Allocates this rank's buffer for `capacity` received token rows (the most
 * a step can bring: max tokens per rank * world) with top_k id and weight
 * slots each; writes its IPC handle (MOE_EP_HANDLE_BYTES) to handle_out.
 * 2 <= world <= MOE_EP_MAX_RANKS. wait_limit_ms bounds every wait on
 * another rank (0: 5000 ms). After a timeout the object is unusable (ranks
 * may disagree on the step) and must be destroyed. */
int moe_ep_peer_create(int world, int rank, int64_t capacity, int64_t hidden_size, int top_k,
                       int act_dtype, int wait_limit_ms, moe_ep_peer_t** out,
                       void* handle_out);

/* Opens the other ranks' buffers: `handles` holds world handles, rank order. */
int moe_ep_peer_connect(moe_ep_peer_t* ep, const void* handles);

/* This rank's received rows [capacity, hidden_size], their expert ids
 * [capacity, top_k] (int32, local to this rank, -1 for slots held elsewhere)
 * and weights [capacity, top_k] (f32), the result rows [capacity,
 * hidden_size], and the device int that holds how many rows the last
 * dispatch delivered (pass it as moe_problem_t.num_tokens_dev). */
int moe_ep_peer_buffers(const moe_ep_peer_t* ep, void** recv_rows, int32_t** recv_ids,
                        float** recv_weights, void** result_rows, int32_t** recv_count);

/* Sends this rank's rows: for send row p of moe_ep_plan_dedup (send_token,
 * send_eid, send_w, counts), row hidden[send_token[p]] with its top_k ids
 * and weights goes to the destination rank's buffer; returns (on the
 * stream) once every rank's rows for this rank have arrived, with the
 * received count in the recv_count word. hidden is [num_tokens,
 * hidden_size] in the buffer's act dtype. */
int moe_ep_peer_dispatch(moe_ep_peer_t* ep, const void* hidden, int64_t num_tokens,
                         const int32_t* send_token, const int32_t* send_eid,
                         const float* send_w, const int64_t* counts, int32_t* status,
                         void* stream);

/* Signals that this rank's result rows (each already the weighted sum over
 * its slots) are complete, waits for the other ranks' signals and computes
 * out[t] = sum over ranks d, ascending, with inv_index[t*world + d] >= 0 of
 * the result row d computed for (t, d), read from d's buffer, in fp32. out
 * is [num_tokens, hidden_size] in the act dtype. Ends the step. */
int moe_ep_peer_combine(moe_ep_peer_t* ep, const int32_t* inv_index, int64_t num_tokens,
                        void* out, int32_t* status, void* stream);

/* Closes the mappings of the other ranks' buffers. */
int moe_ep_peer_disconnect(moe_ep_peer_t* ep);

/* Frees this rank's buffer (closing any mappings still open). Call it after
 * the stream has drained and every rank has disconnected: other ranks must
 * not hold a mapping of a buffer that is freed. */
int moe_ep_peer_destroy(moe_ep_peer_t* ep);

/* ------------------------------------------------------------------------ */
/* Self-test of the bounded device waits (failure detection without a GPU   */
/* fault): launches one CTA whose mbarrier wait is never satisfied, with a   */
/* limit of `limit_us` microseconds. The kernel stores MOE_ERR_TIMEOUT into  */
/* `device_status` and returns.                                             */
/* ------------------------------------------------------------------------ */
int moe_selftest_wait_timeout(int32_t* device_status, int limit_us,
                              void* stream);

/* Self-test of the MOE_QUANT_FP8_UE8M0 scale-factor path: copies one
 * 512-byte chunk (`chunk`, device, 16-byte aligned) into tensor memory as the
 * block-scaled GEMM does and reads the four columns of all 128 lanes back
 * into out[lane * 4 + column] (uint32, device). A correct copy gives
 * out[l * 4 + c] = 32-bit word 4 * (l % 32) + c of the chunk. A bounded wait
 * that runs out stores MOE_ERR_TIMEOUT in `device_status`. */
int moe_selftest_sf_copy(const void* chunk, uint32_t* out, int32_t* device_status,
                         void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* MOE_B200_H_ */
