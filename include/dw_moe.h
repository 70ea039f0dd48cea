/*
 * dw_moe.h -- C ABI of the B200 FP4 MoE hot path (libdw_moe.so).
 *
 * Plain pointers, sizes and a cudaStream_t passed as void*; no torch types.
 * Every device pointer is caller-allocated; every call is stream-ordered and
 * does not synchronise the host. Return codes: 0 = ok, negative = invalid
 * argument or unsupported shape (message in dwm_last_error()), positive =
 * a CUDA runtime error code. Device-side faults that a kernel detects (a wait
 * that ran out, an index out of range, a buffer overflow) are OR-ed into a
 * per-device status word read with dwm_device_status().
 *
 * Reference interfaces each entry point replaces are cited as file:line in
 * jamesdborin/dw-tpu, with these aliases for its files:
 *   TK  = patches/tokamax/0001-gmm_v2-fp4-emulation-v6e.patch
 *   B01 = patches/tpu-inference/0001-dsv4-v6e-enablement.patch
 *   KD  = kernels/tpu_inference/layers/common/moe_fast_dispatch.py
 *   KC  = kernels/tpu_inference/layers/common/moe_fast_combine.py
 *   KO  = kernels/tpu_inference/kernels/collectives/oneshot.py
 *   KE  = kernels/tpu_inference/layers/common/quantization/e8m0_scale.py
 *   E0901 = patches/tpu-inference-experimental/fused-moe-fp4/0901-*.patch
 *   X0101.. = patches/tpu-inference-ext/0101-*.patch ..
 */
#ifndef DW_MOE_H_
#define DW_MOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define DWM_OK 0
#define DWM_ERR_INVALID (-1)     /* bad argument: raised as ValueError */
#define DWM_ERR_UNSUPPORTED (-2) /* shape/dtype this build does not take */
#define DWM_ERR_STATE (-3)       /* context misuse (EP) */

/* device status bits (dwm_device_status) */
#define DWM_DEV_TIMEOUT 1   /* a bounded device-side wait ran out */
#define DWM_DEV_BAD_INDEX 2 /* an expert id / row index out of range */
#define DWM_DEV_OVERFLOW 4  /* a receive buffer was too small */

/* ---- dtype / option enums ----------------------------------------------- */
#define DWM_BF16 0
#define DWM_F32 1
#define DWM_U8 2 /* E8M0 exponent codes (scales only) */

#define DWM_ACT_NONE 0
#define DWM_ACT_SWIGLU 1       /* silu(gate) * up on [gate | up] halves */
#define DWM_ACT_SWIGLU_CLAMP 2 /* gate = min(gate, L), up = clip(up, -L, L) */

#define DWM_FP4_E2M1 0    /* OCP e2m1 nibbles (sign | e1 e0 | m) */
#define DWM_FP4_TOKAMAX 1 /* tokamax codes q = sign*(2e+m), int4 two's compl. */
#define DWM_FP4_B200 2    /* the B200 load-time layout (dwm_fp4_to_b200):
                             u32 words [groups][n/16][k/16][32] (as many
                             bytes as [groups, n, k/2]); word l of a 16x16
                             (k, column) block is lane l's A fragment of an
                             m16n8k16 MMA for W^T, its bits permuted for a
                             one-PRMT bf16 decode */

#define DWM_SCORE_SOFTMAX 0
#define DWM_SCORE_SIGMOID 1
#define DWM_SCORE_SQRTSOFTPLUS 2

/* ---- library ------------------------------------------------------------ */
const char* dwm_version(void);
/* Message of the last negative return on this host thread. */
const char* dwm_last_error(void);
/* Synchronises `stream`, returns the device status bits seen since the last
 * call into *bits and clears them. */
int dwm_device_status(void* stream, int* bits);

/* ---- FP4 grouped matmul --------------------------------------------------
 * Replaces tokamax gmm_v2(lhs, rhs, group_sizes, rhs_scale=..., group_offset,
 * zero_initialize, fuse_act, preferred_element_type, rhs_fp4_codes)
 * (TK:107-153; decode TK:33-41,62-63; dequant order E0901:84-95) as reached
 * through gmm_wrapper (B01:218-232, X0401:56-64, X0403:64-70, X0106:18-29).
 *
 *   lhs     bf16 [m, k], rows sorted by group (group g owns rows
 *           [sum(group_sizes[:g]), +group_sizes[g]))
 *   codes   DWM_FP4_E2M1: uint8 [num_local_groups, k, n/2], two e2m1 nibbles
 *           per byte, element 2j in the low nibble; DWM_FP4_B200: the same
 *           values re-laid by dwm_fp4_to_b200 (faster decode); convert
 *           tokamax codes once with dwm_fp4_codes_convert
 *   scales  [num_local_groups, k/32, n] of scale_dtype: DWM_U8 (E8M0 codes,
 *           KE:37-40), DWM_BF16 or DWM_F32 (cast to bf16 before use)
 *   group_sizes int32 [num_groups] on the device
 *   act     DWM_ACT_*; with SwiGLU the output has n/2 columns
 *   out     [m, n or n/2] of out_dtype (DWM_BF16 or DWM_F32)
 *   zero_init  rows outside the local groups are zeroed (else untouched,
 *           like zero_initialize=False)
 * Constraints: k % 64 == 0, n % 256 == 0, 16-byte aligned pointers. */
int dwm_gmm_fp4(const void* lhs, const void* codes, int codes_format, const void* scales,
                int scale_dtype, const int32_t* group_sizes, int num_groups, int m, int k,
                int n, int group_offset, int num_local_groups, int act, float act_limit,
                int out_dtype, int zero_init, void* out, void* stream);

/* dwm_gmm_fp4 with the kernel variant fixed: 0 = automatic (as dwm_gmm_fp4),
 * 1 = tcgen05 MMA on weights decoded into shared memory (128-row tiles; the
 * automatic choice for groups averaging 49-95 rows),
 * 2 = mma.sync on weights decoded straight into registers (decode-sized
 * groups; 8-row token tiles up to 6 rows per group on average, 16-row tiles
 * above), 3 / 4 = the same with 8 / 16-row token tiles (2: the automatic
 * choice for B200 codes whose groups average at most 16 rows), 5 = the same
 * with 32-row token tiles (four n8 tiles per decoded weight fragment; E8M0
 * scales multiplied into the decoded weights in bf16 before the MMA),
 * 7 = tcgen05 on CTA pairs: M = 256 UMMAs (cta_group::2) over two SMs, each
 * decoding half of the weight columns, up to 256 token rows per tile and
 * double-buffered accumulators, a group above 256 rows in tiles of equal
 * size (the automatic choice for B200 codes whose groups average 96-223
 * rows); 8 = the same kernel for each group's full 256-row tiles (and a last
 * tile of 96 rows or more), the mma.sync kernel for a shorter remainder,
 * which then costs one weight stream per 16 rows instead of a whole tile's
 * decode; 9 = 7 with tiles of up to 512 token rows: two UMMAs per k-step
 * (N = 256 and the rest) into both 256-column TMEM accumulator slots over
 * one decoded stage, so a group of 257-512 rows costs one tile's decode;
 * tiles of up to 256 rows keep the two slots double-buffered (the automatic
 * choice for B200 codes whose groups average 224 rows or more); 10 = each
 * group on the kernel for its size, in four launches over disjoint rows:
 * 1-16 rows on the mma.sync kernel's 16-row tiles, 17-32 on its 32-row tiles,
 * 33-95 on variant 1's kernel, larger groups on variant 9's (the automatic
 * choice for groups averaging 17-48 rows; for skewed routing at any size).
 * 1-5 and 7-10 need DWM_FP4_B200 codes; 6 is not assigned. Every variant decodes
 * the same bf16 weights and accumulates in f32; results differ between
 * variants only by f32 summation order (1, 7 and 9 give identical bits; 8
 * gives them on every group's first 256 rows, 10 on groups above 32 rows). Same reference interface as
 * dwm_gmm_fp4 (TK:107-153). */
int dwm_gmm_fp4_variant(const void* lhs, const void* codes, int codes_format, const void* scales,
                        int scale_dtype, const int32_t* group_sizes, int num_groups, int m,
                        int k, int n, int group_offset, int num_local_groups, int act,
                        float act_limit, int out_dtype, int zero_init, void* out, int variant,
                        void* stream);

/* Dequantise FP4 weights to bf16 with the reference's order (decode to bf16,
 * scale cast to bf16, one bf16 multiply; E0901:84-95): codes as for
 * dwm_gmm_fp4 (DWM_FP4_E2M1 [g, k, n/2] or DWM_FP4_B200 [g, n, k/2]), scales
 * [g, k/32, n] -> out bf16 [g, k, n]. The same decode the GEMM uses.
 * Counterpart of tokamax decode_codes (TK:33-41) plus the block-scale
 * multiply. */
int dwm_fp4_dequant(const void* codes, int codes_format, const void* scales, int scale_dtype,
                    int groups, int k, int n, void* out, void* stream);

/* Load-time re-layout of packed e2m1 weights: raw [g, k, n/2] -> DWM_FP4_B200
 * [g, n, k/2] (inverse = 0) or back (inverse = 1); lossless, out of place.
 * Counterpart of the reference's one-time stored-code re-encoding
 * fp4_weight_to_codes (B01:276-299, TK:17-30). k % 16 == 0, n % 16 == 0. */
int dwm_fp4_to_b200(const void* in, void* out, int groups, int k, int n, int inverse,
                    void* stream);

/* On-device weight preparation: quantize_tensor(float4_e2m1fn, w, block 32,
 * power_of_two_scale) (B01:319-347) of w [groups, k, n] (bf16 or f32) over
 * blocks of 32 consecutive k of each column -> codes uint8 [groups, k, n/2]
 * (packed e2m1, element 2j in the low nibble) and scales [groups, k/32, n]:
 * DWM_U8 E8M0 codes (needs pow2 = 1; *lossless_dev, int32 on the device, is
 * set to 1 and cleared if a scale is not a positive normal power of two or
 * +0, as e8m0_encode's flag, KE:28-34) or DWM_F32. With pow2 = 1,
 * re-quantising MXFP4 data reproduces it exactly (B01:131-157). k % 32 == 0,
 * n % 2 == 0. */
int dwm_fp4_quantize(const void* w, int w_dtype, int groups, int k, int n, int pow2, void* codes,
                     void* scales, int scale_dtype, int32_t* lossless_dev, void* stream);

/* Re-encode packed nibbles between DWM_FP4_E2M1 and DWM_FP4_TOKAMAX
 * (tokamax e2m1_to_codes, TK:17-30, and its inverse); in == out allowed. */
int dwm_fp4_codes_convert(const void* in, void* out, size_t nbytes, int from_format,
                          int to_format, void* stream);

/* ---- E8M0 scales (KE:28-40) ---------------------------------------------- */
/* f32 -> uint8 exponent codes; *lossless_dev (int32, device) is set to 1 and
 * cleared to 0 if any scale is not a positive power of two or +0. */
int dwm_e8m0_encode(const float* scale, size_t n, uint8_t* codes, int32_t* lossless_dev,
                    void* stream);
int dwm_e8m0_decode(const uint8_t* codes, size_t n, float* out, void* stream);

/* ---- routing (E0901:656-687, X0101:131) --------------------------------- */
/* logits [t, e] (DWM_BF16 or DWM_F32) -> top_k ids int32 [t, top_k] and
 * weights (f32 [t, top_k] and/or bf16 [t, top_k]; either may be NULL).
 * Ties resolve to the lower expert index (lax.top_k). bias (f32 [e], may be
 * NULL) is added for selection only. Rows >= num_valid_tokens (if >= 0) get
 * expert 0 with weight 0. */
int dwm_route_topk(const void* logits, int logits_dtype, int t, int e, int top_k, int scoring,
                   int renormalize, const float* bias, int num_valid_tokens, int32_t* topk_ids,
                   float* topk_weights_f32, void* topk_weights_bf16, void* stream);

/* Hash routing (E0901:667-671): the ids come precomputed (hash_ids int32
 * [t, top_k], e.g. DeepSeek-V4's hash layers) and the weights are the scores
 * at those ids; renormalisation and padding as dwm_route_topk. Ids outside
 * [0, e) are reported (DWM_DEV_BAD_INDEX) and read as expert 0. */
int dwm_route_hash(const void* logits, int logits_dtype, int t, int e, int top_k, int scoring,
                   int renormalize, const int32_t* hash_ids, int num_valid_tokens,
                   int32_t* topk_ids, float* topk_weights_f32, void* topk_weights_bf16,
                   void* stream);

/* dedupe_topk (E0901:98-121), in place: a repeated expert id within a token
 * adds its f32 weight to the first occurrence and is re-pointed at the lowest
 * of experts 0 .. min(2*top_k, num_experts)-1 the token does not use, with
 * weight 0. topk_weights_bf16 (may be NULL) receives the bf16 cast. */
int dwm_dedupe_topk(float* topk_weights_f32, int32_t* topk_ids, int t, int top_k,
                    int num_experts, void* topk_weights_bf16, void* stream);

/* ---- permute / dispatch (KD, X0405:70-98) -------------------------------- */
/* KD:41-44: out[j] = argsort[j] / topk. */
int dwm_sorted_token_indices(const int32_t* topk_argsort, int64_t n, int topk, int32_t* out,
                             void* stream);

/* Stable sort of the flattened ids by expert (jnp.argsort is stable):
 * argsort [t*topk], token_indices_sorted [t*topk] (= argsort / topk),
 * revert [t*topk] (inverse permutation; the combine's indices),
 * group_sizes [e] (bincount). Any output except group_sizes may be NULL. */
int dwm_permute(const int32_t* topk_ids, int t, int topk, int e, int32_t* topk_argsort,
                int32_t* token_indices_sorted, int32_t* revert, int32_t* group_sizes,
                void* stream);

/* KD:134-194: out[r] = hidden[token_indices_sorted[r]] for bf16 rows
 * (bit-exact data movement). hidden [t, h], out [rows, h]. */
int dwm_dispatch_gather(const void* hidden, int t, int h, const int32_t* token_indices_sorted,
                        int64_t rows, void* out, void* stream);

/* ---- combine (KC:44-54,57-122; contract KC:14-21) ------------------------ */
/* out[t] = round(sum_{k=0..topk-1} f32(x[indices[t*topk+k]]) * f32(w[t,k])),
 * f32 products, summed left to right from +0.0, one rounding to out_dtype.
 * x [x_rows, h] (DWM_BF16 or DWM_F32); w [t, topk] (DWM_BF16 or DWM_F32). */
int dwm_combine(const void* x, int x_dtype, int64_t x_rows, const int32_t* indices,
                const void* w, int w_dtype, int t, int h, int topk, void* out, int out_dtype,
                void* stream);

/* The combine with the shared expert summed in (MOE_SHARED_EXPERT_TP,
 * X0104:80-87): out[t] = round(f32(mid(routed[t])) * routed_scale + shared[t])
 * where routed[t] is dwm_combine's k-order f32 sum, mid rounds it to bf16
 * (mid_dtype DWM_BF16, the combine's own output dtype) or keeps it
 * (DWM_F32, MOE_F32_REDUCE), and each step is rounded to f32. shared [t, h]
 * (DWM_BF16 or DWM_F32) is the shared expert's output (or this shard's
 * partial of it); NULL gives dwm_combine. */
int dwm_combine_shared(const void* x, int x_dtype, int64_t x_rows, const int32_t* indices,
                       const void* w, int w_dtype, int t, int h, int topk, const void* shared,
                       int shared_dtype, float routed_scale, int mid_dtype, void* out,
                       int out_dtype, void* stream);

/* ---- the single-device layer in one call ---------------------------------
 * fused_moe_func's GMM path (X0104:88-98, X0405, X0404 on one device):
 * dwm_route_topk -> dwm_permute -> dwm_dispatch_gather -> dwm_gmm_fp4 (gmm1,
 * SwiGLU) -> dwm_gmm_fp4 (gmm2) -> dwm_combine, bit-identical to making those
 * calls in turn. hidden bf16 [num_tokens, hidden_size]; logits [num_tokens,
 * num_experts] (bf16 or f32); w13 / s13 / w2 / s2 as dwm_gmm_fp4 takes them
 * (w13: k = hidden_size, n = 2*inter; w2: k = inter, n = hidden_size);
 * y_f32 = 1 keeps gmm2's output in f32 (MOE_F32_REDUCE, X0106:18-29);
 * out bf16 [num_tokens, hidden_size]. The intermediates live in `workspace`
 * (256-byte aligned, at least dwm_moe_layer_workspace_bytes bytes; nothing in
 * it needs to start at zero). */
size_t dwm_moe_layer_workspace_bytes(int num_tokens, int hidden, int inter, int topk,
                                     int num_experts, int y_f32);
int dwm_moe_layer_fp4(const void* hidden, const void* logits, int logits_dtype, int num_tokens,
                      int hidden_size, int num_experts, int topk, int scoring, int renormalize,
                      const void* w13, const void* s13, const void* w2, const void* s2,
                      int codes_format, int scale_dtype, int inter, int act, float act_limit,
                      int y_f32, void* workspace, size_t workspace_bytes, void* out,
                      void* stream);

/* dwm_moe_layer_fp4 for callers that cannot allocate device memory: no
 * workspace argument; the intermediates live in one file-scope device array
 * of DWM_LAYER_SCRATCH_BYTES (32 MiB: e.g. 128 tokens x top-8 at hidden 4096,
 * intermediate 2048 with f32 gmm2 output), one per device, whose address is
 * resolved once per device. Inputs needing more scratch are rejected
 * (DWM_ERR_INVALID). Nothing in the scratch needs to start at zero. Calls that
 * overlap on one device (other streams or host threads) race on that one
 * array. The first call on a device (a num_tokens = 0 call does only that
 * setup) must come before any stream capture. No counterpart in the
 * reference. */
#define DWM_LAYER_SCRATCH_BYTES 33554432
int dwm_moe_layer_fp4_noalloc(const void* hidden, const void* logits, int logits_dtype,
                              int num_tokens, int hidden_size, int num_experts, int topk,
                              int scoring, int renormalize, const void* w13, const void* s13,
                              const void* w2, const void* s2, int codes_format, int scale_dtype,
                              int inter, int act, float act_limit, int y_f32, void* out,
                              void* stream);

/* ---- expert-parallel exchange over NVLink peer memory ---------------------
 * Replaces the GMM_EP exchange: all_gather_local + the per-shard stable sort
 * (KO:152-164, X0101:56-104, X0107:34-51) on the way in, and the masked f32
 * combine + reduce_scatter_local (X0107:15-29, KO:167-185) on the way out,
 * with one-shot kernels over peer memory: the dispatch stores rows straight
 * into the expert owners' receive buffers, and the combine loads each
 * token's expert outputs straight from the owners' output buffers.
 * One context per rank (one process per GPU); rank r owns experts
 * [r*E/world, (r+1)*E/world). Receive order on rank r: expert-major over its
 * experts, then (source rank, source token, k slot), i.e. the rows the
 * reference's global stable argsort over the rank-major gathered batch keeps
 * on rank r. The combine is the k-order f32 weighted sum of each token's
 * expert outputs from +0.0, rounded once (KC:14-21, the combine contract of
 * the single-device path). Every rank must make the same sequence of calls
 * with the same dtypes, one combine per dispatch; calls on one context are
 * stream-ordered and must not overlap. The exchange keeps its step counter
 * in device memory, so the calls can be captured in a CUDA graph and
 * replayed. Device-side waits give up after 2 s (dwm_ep_set_wait_limit) with
 * DWM_DEV_TIMEOUT; the reference's barrier waits without bound
 * (KO:70-77). */
#define DWM_EP_HANDLE_BYTES 64 /* size of one rank's IPC handle */
#define DWM_EP_COUNTS 1        /* dispatch phases (DWM_EP_ALL = all three) */
#define DWM_EP_ROWS 2
#define DWM_EP_WAIT 4
#define DWM_EP_ALL 7
#define DWM_EP_PUSH 1          /* combine phases: make this rank's outputs readable, */
#define DWM_EP_REDUCE 2        /* then reduce every own token */
#define DWM_EP_GATED 8         /* dispatch flag: per-expert arrivals for dwm_ep_gmm_fp4 */
#define DWM_EP_PUSHED 4        /* combine flag: outputs were pushed by dwm_ep_gmm_fp4 */
#define DWM_EP_RANK_ORDER 16   /* combine flag: the reference GMM_EP sum order (below) */
#define DWM_EP_GEMM_GATED 1    /* dwm_ep_gmm_fp4 modes: the up projection, gated, */
#define DWM_EP_GEMM_PUSH 2     /* the down projection, pushing its rows to the owners */

typedef struct dwm_ep dwm_ep;

/* Allocate this rank's symmetric buffer on the current device: receive rows
 * (bf16) and expert outputs (4-byte capacity) for world*max_tokens*topk
 * pairs, plus counts and flags. num_experts % world == 0,
 * num_experts <= 1024, hidden % 8 == 0, world <= 8,
 * world*max_tokens*topk <= 2^28. */
int dwm_ep_create(int rank, int world, int max_tokens, int hidden, int topk, int num_experts,
                  dwm_ep** ctx);
/* This rank's CUDA IPC handle (DWM_EP_HANDLE_BYTES bytes) for the exchange. */
int dwm_ep_ipc_handle(dwm_ep* ctx, void* handle);
/* Map every peer's buffer: handles = world handles, rank-major. */
int dwm_ep_connect(dwm_ep* ctx, const void* handles);
/* Single-process form: `ranks` holds all world contexts, created on the same
 * device (an emulation of the exchange on one GPU: the phases of all ranks
 * must then be issued phase by phase, COUNTS of every rank before ROWS of any,
 * and so on, so that no wait depends on a later launch). */
int dwm_ep_connect_local(dwm_ep* ctx, dwm_ep* const* ranks);
/* The receive buffer (bf16 [capacity_rows, hidden]) inside the symmetric
 * buffer; rows [0, sum(recv_group_sizes)) are valid after a dispatch. */
int dwm_ep_recv_buffer(dwm_ep* ctx, void** recv, int64_t* capacity_rows);
/* The output buffer inside the symmetric buffer: room for [capacity_rows,
 * hidden] bf16 or f32 expert outputs in receive order. A grouped matmul that
 * writes its output here saves the combine a copy. */
int dwm_ep_output_buffer(dwm_ep* ctx, void** y, int64_t* capacity_rows);
/* hidden bf16 [num_tokens, hidden], topk_ids int32 [num_tokens, topk] (ids
 * outside [0, num_experts) are reported and dropped) -> the receive buffer
 * and recv_group_sizes int32 [num_experts/world] (device). Counterpart of
 * all_gather_local + sort (X0101:56-104). */
int dwm_ep_dispatch(dwm_ep* ctx, const void* hidden, const int32_t* topk_ids, int num_tokens,
                    int32_t* recv_group_sizes, int phases, void* stream);
/* y [rows, hidden] (bf16 or f32: expert outputs of the received rows, in
 * receive order; copied into the output buffer first unless y is that
 * buffer) -> out [num_tokens, hidden] of out_dtype, with topk_weights
 * [num_tokens, topk] (bf16 or f32) of the dispatch's tokens. Counterpart of
 * the masked combine + reduce_scatter_local (X0107:15-29, KO:167-185) with
 * the k-order contract of fast_combine (KC:14-21). With DWM_EP_RANK_ORDER
 * (top_k <= 8) the sum instead follows the reference's GMM_EP order: for each
 * rank r, an f32 partial over the k slots whose expert rank r owns (k order,
 * from +0.0, a slot of another rank adding +0.0), and the partials summed in
 * f32 in rank order 0..world-1 (X0107:15-29, KO:181-184), rounded once. */
int dwm_ep_combine(dwm_ep* ctx, const void* y, int y_dtype, const void* topk_weights,
                   int w_dtype, void* out, int out_dtype, int phases, void* stream);
/* dwm_ep_combine with the shared expert summed into each own token's sum
 * (MOE_SHARED_EXPERT_TP, X0104:80-87), as dwm_combine_shared does; shared
 * [num_tokens, hidden] is read in the REDUCE phase. */
int dwm_ep_combine_shared(dwm_ep* ctx, const void* y, int y_dtype, const void* topk_weights,
                          int w_dtype, const void* shared, int shared_dtype, float routed_scale,
                          int mid_dtype, void* out, int out_dtype, int phases, void* stream);
/* The overlapped form of the exchange (prefill): the grouped matmuls run on a
 * kernel of `variant` 1 (tcgen05, one CTA), 3 / 4 / 5 (mma.sync decode
 * kernel, 8 / 16 / 32-row tiles), 7 (CTA pairs) or 9 (CTA pairs, 512-row
 * tiles), as in dwm_gmm_fp4_variant, with the exchange folded in,
 * instead of the dispatch waiting for every row and the combine pulling every
 * output after the GEMMs.
 *   dwm_ep_dispatch(..., DWM_EP_COUNTS | DWM_EP_ROWS | DWM_EP_GATED): stores
 *       the rows with their (source rank, pair) tags; each CTA adds the rows it
 *       stored for each expert to the owner's arrival counter of that expert;
 *       no wait at the end.
 *   dwm_ep_gmm_fp4(..., DWM_EP_GEMM_GATED): lhs = the receive buffer
 *       (dwm_ep_recv_buffer), k = hidden; the tiles of a local expert load its
 *       rows only once all of them have arrived, so the GEMM starts on the
 *       experts that are complete while other rows are still in flight
 *       (out: [capacity, n or n/2], e.g. the SwiGLU activations).
 *   dwm_ep_gmm_fp4(..., DWM_EP_GEMM_PUSH): act = none, n = hidden; the
 *       epilogue stores each output row straight into its token owner's
 *       buffer (over NVLink), at the row of its (token, k) pair; the last CTA
 *       tells every rank (out is not written).
 *   dwm_ep_combine(..., DWM_EP_REDUCE | DWM_EP_PUSHED): waits until every
 *       rank has pushed, then forms the k-order f32 sum from local memory
 *       (y is not read; y_dtype = the down projection's out_dtype).
 * Bits are those of the serial exchange with the same kernels. Counterpart
 * of the reference's fused dispatch-GEMM-combine kernel
 * (E0901:361-449,690-767) and next-expert prefetch (E0902:48-66). The
 * recv_group_sizes are the dispatch's; codes in the B200 layout. */
int dwm_ep_gmm_fp4(dwm_ep* ctx, const void* lhs, const void* codes, int codes_format,
                   const void* scales, int scale_dtype, const int32_t* recv_group_sizes, int k,
                   int n, int act, float act_limit, int out_dtype, void* out, int mode,
                   int variant, void* stream);
/* Link measurement: copies `bytes` of this rank's receive buffer into rank
 * `peer`'s receive buffer over NVLink (one copy-engine copy on `stream`).
 * It overwrites the peer's receive rows: call it only between steps, with
 * every rank idle. No counterpart in the reference. */
int dwm_ep_link_probe(dwm_ep* ctx, int peer, int64_t bytes, void* stream);
/* Limit of every device-side wait of this context's later launches (default
 * 2 s; 1 us .. 60 s). A wait that runs out sets DWM_DEV_TIMEOUT, the kernel
 * drops the step's rows and returns; the contexts of all ranks must then be
 * destroyed and created again before the next exchange (their step counters
 * no longer agree). No counterpart in the reference, whose one-shot barrier
 * waits without bound (KO:70-77). */
int dwm_ep_set_wait_limit(dwm_ep* ctx, uint64_t limit_ns);
/* Synchronise the context's device, unmap peers and free the buffers. */
int dwm_ep_destroy(dwm_ep* ctx);

#ifdef __cplusplus
}
#endif

#endif /* DW_MOE_H_ */
