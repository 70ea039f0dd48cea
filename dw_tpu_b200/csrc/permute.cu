// MOE_FAST_DISPATCH / MOE_FAST_COMBINE for sm_100a: the stable
// sort-by-expert permutation, the row gather and the k-order weighted combine.
//
//   permute   KD:41-44 + X0405:73-88 (stable argsort, argsort // topk,
//             bincount) as a one-CTA counting sort: per-warp histograms,
//             an exclusive scan, then an in-order scatter in which each warp
//             ranks equal experts with __match_any_sync. Stability holds
//             because warps own contiguous, ordered segments.
//   gather    KD:134-194, 16-byte vector copies of bf16 rows (HBM-bound).
//   combine   KC:44-54 (contract KC:14-21): f32 products, left-to-right f32
//             sum from +0.0, one rounding; mul and add are kept separate
//             (no FMA contraction) so the result is bit-identical to that
//             sequence.
#include <algorithm>

#include "moe_common.cuh"

namespace dwm {
namespace perm {

using namespace moe;

__global__ void sorted_token_indices_kernel(const int32_t* __restrict__ in, int64_t n, int topk,
                                            int32_t* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = in[i] / topk;
}

__global__ void __launch_bounds__(SORT_THREADS, 1)
    permute_kernel(const int32_t* __restrict__ ids, int n, int topk, int e,
                   int32_t* __restrict__ argsort, int32_t* __restrict__ tok,
                   int32_t* __restrict__ revert, int32_t* __restrict__ group_sizes, int* status) {
  extern __shared__ int sm[];
  counting_sort_block(ids, n, topk, e, argsort, tok, revert, group_sizes, nullptr, status, sm);
}

// out[r, :] = hidden[tok[r], :], rows of h bf16 (h % 8 == 0).
__global__ void gather_rows_kernel(const uint4* __restrict__ hidden, int t, int64_t h16,
                                   const int32_t* __restrict__ tok, int64_t rows,
                                   uint4* __restrict__ out, int* status) {
  const int64_t total = rows * h16;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / h16;
    const int64_t c = i - r * h16;
    const int src = tok[r];
    if (src < 0 || src >= t) {
      report(status, DWM_DEV_BAD_INDEX);
      out[i] = make_uint4(0, 0, 0, 0);
      continue;
    }
    out[i] = hidden[(int64_t)src * h16 + c];
  }
}

// One thread per 8 output columns of one token.
template <int XD, int WD, int OD>
__global__ void combine_kernel(const void* __restrict__ x, int64_t x_rows,
                               const int32_t* __restrict__ idx, const void* __restrict__ w,
                               int t, int h, int topk, void* __restrict__ out,
                               const moe::SharedAdd sa, int* status) {
  const int h8 = h / 8;
  const int64_t total = (int64_t)t * h8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tt = i / h8;
    const int c = (int)(i - tt * h8);
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.0f;
    for (int k = 0; k < topk; ++k) {
      const int64_t r = idx[tt * topk + k];
      const float wk = load_weight<WD>(w, tt * topk + k);
      if (r < 0 || r >= x_rows) {
        report(status, DWM_DEV_BAD_INDEX);
        continue;
      }
      float v[8];
      load8<XD>(x, r * h + (int64_t)c * 8, v);
      mul_add8(acc, v, wk);
    }
    moe::shared_add8(acc, sa, tt * h + (int64_t)c * 8);
    store8<OD>(out, tt * h + (int64_t)c * 8, acc);
  }
}

}  // namespace perm
}  // namespace dwm

using namespace dwm;

extern "C" int dwm_sorted_token_indices(const int32_t* topk_argsort, int64_t n, int topk,
                                        int32_t* out, void* stream) {
  DWM_CHECK_ARG(topk >= 1, "topk must be >= 1");
  DWM_CHECK_ARG(n >= 0 && (n == 0 || (topk_argsort && out)), "bad arguments");
  if (n == 0) return DWM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  perm::sorted_token_indices_kernel<<<moe::grid_for(n, 256), 256, 0, s>>>(topk_argsort, n, topk,
                                                                           out);
  return check_cuda(cudaGetLastError(), "sorted_token_indices launch");
}

extern "C" int dwm_permute(const int32_t* topk_ids, int t, int topk, int e, int32_t* topk_argsort,
                           int32_t* token_indices_sorted, int32_t* revert, int32_t* group_sizes,
                           void* stream) {
  DWM_CHECK_ARG(t >= 0 && topk >= 1 && e >= 1, "bad shape t=%d topk=%d e=%d", t, topk, e);
  DWM_CHECK_ARG(e <= 1024, "e=%d exceeds 1024 experts", e);
  DWM_CHECK_ARG((int64_t)t * topk < (1LL << 31), "t*topk too large");
  DWM_CHECK_ARG(t == 0 || topk_ids, "NULL topk_ids");
  DWM_CHECK_ARG(group_sizes, "group_sizes is required");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int n = t * topk;
  const size_t smem = (size_t)(moe::SORT_WARPS * e + e) * sizeof(int);
  int rc = set_smem_limit(reinterpret_cast<const void*>(perm::permute_kernel),
                          (int)((moe::SORT_WARPS * 1024 + 1024) * sizeof(int)),
                          "permute smem attribute");
  if (rc) return rc;
  perm::permute_kernel<<<1, moe::SORT_THREADS, smem, s>>>(
      topk_ids, n, topk, e, topk_argsort, token_indices_sorted, revert, group_sizes,
      status_ptr());
  return check_cuda(cudaGetLastError(), "permute launch");
}

extern "C" int dwm_dispatch_gather(const void* hidden, int t, int h,
                                   const int32_t* token_indices_sorted, int64_t rows, void* out,
                                   void* stream) {
  DWM_CHECK_ARG(t >= 0 && h > 0 && rows >= 0, "bad shape");
  DWM_CHECK_ARG(h % 8 == 0, "h=%d must be a multiple of 8", h);
  DWM_CHECK_ARG(rows == 0 || (hidden && token_indices_sorted && out), "NULL pointer");
  DWM_CHECK_ARG(moe::aligned16(hidden) && moe::aligned16(out), "pointers must be 16-byte aligned");
  if (rows == 0) return DWM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t h16 = h / 8;
  perm::gather_rows_kernel<<<moe::grid_for(rows * h16, 256), 256, 0, s>>>(
      static_cast<const uint4*>(hidden), t, h16, token_indices_sorted, rows,
      static_cast<uint4*>(out), status_ptr());
  return check_cuda(cudaGetLastError(), "gather launch");
}

extern "C" int dwm_combine_shared(const void* x, int x_dtype, int64_t x_rows,
                                  const int32_t* indices, const void* w, int w_dtype, int t, int h,
                                  int topk, const void* shared, int shared_dtype,
                                  float routed_scale, int mid_dtype, void* out, int out_dtype,
                                  void* stream) {
  DWM_CHECK_ARG(t >= 0 && h > 0 && topk >= 1 && x_rows >= 0, "bad shape");
  DWM_CHECK_ARG(h % 8 == 0, "h=%d must be a multiple of 8", h);
  DWM_CHECK_ARG(x_dtype == DWM_BF16 || x_dtype == DWM_F32, "x dtype must be bf16 or f32");
  DWM_CHECK_ARG(w_dtype == DWM_BF16 || w_dtype == DWM_F32, "w dtype must be bf16 or f32");
  DWM_CHECK_ARG(out_dtype == DWM_BF16 || out_dtype == DWM_F32, "out dtype must be bf16 or f32");
  DWM_CHECK_ARG(t == 0 || (x && indices && w && out), "NULL pointer");
  DWM_CHECK_ARG(moe::aligned16(x) && moe::aligned16(out), "pointers must be 16-byte aligned");
  DWM_CHECK_ARG(shared == nullptr || ((shared_dtype == DWM_BF16 || shared_dtype == DWM_F32) &&
                                      (mid_dtype == DWM_BF16 || mid_dtype == DWM_F32) &&
                                      moe::aligned16(shared)),
                "shared partial: bf16/f32, 16-byte aligned; mid dtype bf16/f32");
  if (t == 0) return DWM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned grid = moe::grid_for((int64_t)t * (h / 8), 256);
  const moe::SharedAdd sa{shared, shared_dtype == DWM_F32, routed_scale, mid_dtype == DWM_BF16};
  int* st = status_ptr();
#define DWM_COMBINE(XD, WD, OD)                                                             \
  if (x_dtype == XD && w_dtype == WD && out_dtype == OD) {                                  \
    perm::combine_kernel<XD, WD, OD><<<grid, 256, 0, s>>>(x, x_rows, indices, w, t, h, topk, \
                                                          out, sa, st);                      \
    return check_cuda(cudaGetLastError(), "combine launch");                                \
  }
  DWM_COMBINE(DWM_BF16, DWM_BF16, DWM_BF16)
  DWM_COMBINE(DWM_BF16, DWM_F32, DWM_BF16)
  DWM_COMBINE(DWM_F32, DWM_BF16, DWM_BF16)
  DWM_COMBINE(DWM_F32, DWM_F32, DWM_BF16)
  DWM_COMBINE(DWM_BF16, DWM_BF16, DWM_F32)
  DWM_COMBINE(DWM_BF16, DWM_F32, DWM_F32)
  DWM_COMBINE(DWM_F32, DWM_BF16, DWM_F32)
  DWM_COMBINE(DWM_F32, DWM_F32, DWM_F32)
#undef DWM_COMBINE
  return set_error(DWM_ERR_UNSUPPORTED, "combine dtype combination");
}

extern "C" int dwm_combine(const void* x, int x_dtype, int64_t x_rows, const int32_t* indices,
                           const void* w, int w_dtype, int t, int h, int topk, void* out,
                           int out_dtype, void* stream) {
  return dwm_combine_shared(x, x_dtype, x_rows, indices, w, w_dtype, t, h, topk, nullptr, DWM_F32,
                            1.0f, DWM_BF16, out, out_dtype, stream);
}
