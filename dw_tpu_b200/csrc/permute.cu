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

#include "common.cuh"

namespace dwm {
namespace perm {

constexpr int PERMUTE_THREADS = 1024;
constexpr int PERMUTE_WARPS = PERMUTE_THREADS / 32;

__global__ void sorted_token_indices_kernel(const int32_t* __restrict__ in, int64_t n, int topk,
                                            int32_t* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = in[i] / topk;
}

// hist: [PERMUTE_WARPS][e] ints in dynamic shared memory, then the scan.
__global__ void __launch_bounds__(PERMUTE_THREADS, 1)
    permute_kernel(const int32_t* __restrict__ ids, int n, int topk, int e,
                   int32_t* __restrict__ argsort, int32_t* __restrict__ tok,
                   int32_t* __restrict__ revert, int32_t* __restrict__ group_sizes, int* status) {
  extern __shared__ int sm[];
  int* hist = sm;                          // [W][e]
  int* totals = sm + PERMUTE_WARPS * e;    // [e]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < PERMUTE_WARPS * e; i += blockDim.x) hist[i] = 0;
  __syncthreads();

  // Contiguous segment per warp, a multiple of 32 entries.
  const int seg = ((n + PERMUTE_WARPS - 1) / PERMUTE_WARPS + 31) & ~31;
  const int s0 = warp * seg, s1 = min(n, s0 + seg);
  int* my = hist + warp * e;
  for (int base = s0; base < s1; base += 32) {
    const int j = base + lane;
    int x = -1;
    if (j < s1) {
      x = ids[j];
      if (x < 0 || x >= e) { report(status, DWM_DEV_BAD_INDEX); x = -1; }
    }
    const unsigned act = __ballot_sync(0xffffffffu, x >= 0);
    const unsigned peers = __match_any_sync(0xffffffffu, x);
    if (x >= 0 && (peers & act) && (__ffs(peers) - 1) == lane) my[x] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();

  // totals[x] = sum over warps; hist[w][x] <- sum over earlier warps.
  for (int x = threadIdx.x; x < e; x += blockDim.x) {
    int run = 0;
    for (int w = 0; w < PERMUTE_WARPS; ++w) {
      const int v = hist[w * e + x];
      hist[w * e + x] = run;
      run += v;
    }
    totals[x] = run;
    if (group_sizes) group_sizes[x] = run;
  }
  __syncthreads();
  // Exclusive scan of totals (e entries) by warp 0, chunked per lane.
  if (warp == 0) {
    const int per = (e + 31) / 32;
    int sum = 0;
    for (int i = 0; i < per; ++i) {
      const int x = lane * per + i;
      if (x < e) sum += totals[x];
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    int run = incl - sum;
    for (int i = 0; i < per; ++i) {
      const int x = lane * per + i;
      if (x < e) {
        const int v = totals[x];
        totals[x] = run;
        run += v;
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < PERMUTE_WARPS * e; i += blockDim.x) hist[i] += totals[i % e];
  __syncthreads();

  // In-order scatter.
  for (int base = s0; base < s1; base += 32) {
    const int j = base + lane;
    int x = -1;
    if (j < s1) {
      x = ids[j];
      if (x < 0 || x >= e) x = -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, x);
    const unsigned lower = peers & ((1u << lane) - 1u);
    int pos = -1;
    if (x >= 0) pos = my[x] + __popc(lower);
    __syncwarp();
    if (x >= 0 && lower == 0) my[x] += __popc(peers);
    __syncwarp();
    if (x >= 0) {
      if (argsort) argsort[pos] = j;
      if (tok) tok[pos] = j / topk;
      if (revert) revert[j] = pos;
    } else if (j < s1 && revert) {
      revert[j] = -1;
    }
  }
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

template <int XD>
__device__ __forceinline__ void load8(const void* x, int64_t off, float (&v)[8]) {
  if constexpr (XD == DWM_BF16) {
    const uint4 q = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + off);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  } else {
    const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + off);
    const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + off + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

// One thread per 8 output columns of one token.
template <int XD, int WD, int OD>
__global__ void combine_kernel(const void* __restrict__ x, int64_t x_rows,
                               const int32_t* __restrict__ idx, const void* __restrict__ w,
                               int t, int h, int topk, void* __restrict__ out, int* status) {
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
      float wk;
      if constexpr (WD == DWM_BF16)
        wk = __uint_as_float((uint32_t)static_cast<const uint16_t*>(w)[tt * topk + k] << 16);
      else
        wk = static_cast<const float*>(w)[tt * topk + k];
      if (r < 0 || r >= x_rows) {
        report(status, DWM_DEV_BAD_INDEX);
        continue;
      }
      float v[8];
      load8<XD>(x, r * h + (int64_t)c * 8, v);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = __fadd_rn(acc[q], __fmul_rn(v[q], wk));
    }
    if constexpr (OD == DWM_BF16) {
      uint4 o;
      o.x = f32_to_bf16_bits(acc[0]) | (f32_to_bf16_bits(acc[1]) << 16);
      o.y = f32_to_bf16_bits(acc[2]) | (f32_to_bf16_bits(acc[3]) << 16);
      o.z = f32_to_bf16_bits(acc[4]) | (f32_to_bf16_bits(acc[5]) << 16);
      o.w = f32_to_bf16_bits(acc[6]) | (f32_to_bf16_bits(acc[7]) << 16);
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + tt * h + (int64_t)c * 8) = o;
    } else {
      float* o = static_cast<float*>(out) + tt * h + (int64_t)c * 8;
      *reinterpret_cast<float4*>(o) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *reinterpret_cast<float4*>(o + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline unsigned grid_for(int64_t work, int threads, int per_sm = 16) {
  int64_t b = (work + threads - 1) / threads;
  int64_t cap = (int64_t)num_sms() * per_sm;
  return (unsigned)std::max<int64_t>(1, std::min(b, cap));
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
  perm::sorted_token_indices_kernel<<<perm::grid_for(n, 256), 256, 0, s>>>(topk_argsort, n, topk,
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
  const size_t smem = (size_t)(perm::PERMUTE_WARPS * e + e) * sizeof(int);
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    int rc = check_cuda(cudaFuncSetAttribute(perm::permute_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)((perm::PERMUTE_WARPS * 1024 + 1024) * sizeof(int))),
                        "permute smem attribute");
    if (rc) return rc;
    attr_set[dev] = true;
  }
  perm::permute_kernel<<<1, perm::PERMUTE_THREADS, smem, s>>>(
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
  DWM_CHECK_ARG(perm::aligned16(hidden) && perm::aligned16(out), "pointers must be 16-byte aligned");
  if (rows == 0) return DWM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t h16 = h / 8;
  perm::gather_rows_kernel<<<perm::grid_for(rows * h16, 256), 256, 0, s>>>(
      static_cast<const uint4*>(hidden), t, h16, token_indices_sorted, rows,
      static_cast<uint4*>(out), status_ptr());
  return check_cuda(cudaGetLastError(), "gather launch");
}

extern "C" int dwm_combine(const void* x, int x_dtype, int64_t x_rows, const int32_t* indices,
                           const void* w, int w_dtype, int t, int h, int topk, void* out,
                           int out_dtype, void* stream) {
  DWM_CHECK_ARG(t >= 0 && h > 0 && topk >= 1 && x_rows >= 0, "bad shape");
  DWM_CHECK_ARG(h % 8 == 0, "h=%d must be a multiple of 8", h);
  DWM_CHECK_ARG(x_dtype == DWM_BF16 || x_dtype == DWM_F32, "x dtype must be bf16 or f32");
  DWM_CHECK_ARG(w_dtype == DWM_BF16 || w_dtype == DWM_F32, "w dtype must be bf16 or f32");
  DWM_CHECK_ARG(out_dtype == DWM_BF16 || out_dtype == DWM_F32, "out dtype must be bf16 or f32");
  DWM_CHECK_ARG(t == 0 || (x && indices && w && out), "NULL pointer");
  DWM_CHECK_ARG(perm::aligned16(x) && perm::aligned16(out), "pointers must be 16-byte aligned");
  if (t == 0) return DWM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned grid = perm::grid_for((int64_t)t * (h / 8), 256);
  int* st = status_ptr();
#define DWM_COMBINE(XD, WD, OD)                                                             \
  if (x_dtype == XD && w_dtype == WD && out_dtype == OD) {                                  \
    perm::combine_kernel<XD, WD, OD><<<grid, 256, 0, s>>>(x, x_rows, indices, w, t, h, topk, \
                                                          out, st);                          \
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
