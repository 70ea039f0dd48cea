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
 * Reference interfaces each entry point replaces are cited as project-relative
 * paths of jamesdborin/dw-tpu (see the alias table in DESIGN.md):
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
 *   codes   uint8 [num_local_groups, k, n/2]: two e2m1 nibbles per byte,
 *           element 2j in the low nibble (DWM_FP4_E2M1 only; convert tokamax
 *           codes once with dwm_fp4_codes_convert)
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

/* Dequantise FP4 weights to bf16 with the reference's order (decode to bf16,
 * scale cast to bf16, one bf16 multiply; E0901:84-95): codes [g, k, n/2],
 * scales [g, k/32, n] -> out bf16 [g, k, n]. The same decode the GEMM uses. */
int dwm_fp4_dequant(const void* codes, const void* scales, int scale_dtype, int groups, int k,
                    int n, void* out, void* stream);

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

#ifdef __cplusplus
}
#endif

#endif /* DW_MOE_H_ */
