// Top-k routing (E0901:656-687, cast X0101:131) and E8M0 scale codes
// (KE:28-40) for sm_100a.
//
// route_topk: one warp per token. Scores (softmax / sigmoid / sqrtsoftplus,
// in f32 from f32-widened logits) live in shared memory; top-k is k rounds
// of a warp arg-max whose ties resolve to the lower expert index, the order
// lax.top_k returns. The optional correction bias only steers selection.
#include <algorithm>

#include "common.cuh"

namespace dwm {
namespace route {

constexpr int WARPS = 4;

__device__ __forceinline__ bool better(float a, int ia, float b, int ib) {
  return a > b || (a == b && ia < ib);
}

// hash_ids (optional, [t, top_k]): precomputed expert ids (hash routing,
// E0901:667-671); the weights are the scores at those ids.
template <int LD>
__global__ void route_topk_kernel(const void* __restrict__ logits, int t, int e, int top_k,
                                  int scoring, int renormalize, const float* __restrict__ bias,
                                  int num_valid, const int32_t* __restrict__ hash_ids,
                                  int32_t* __restrict__ ids, float* __restrict__ w32,
                                  uint16_t* __restrict__ w16, int* status) {
  extern __shared__ float sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* score = sm + warp * 2 * e;
  float* sel = score + e;
  const int tok = blockIdx.x * WARPS + warp;
  if (tok >= t) return;
  const int64_t row = (int64_t)tok * e;

  float mx = -INFINITY;
  for (int x = lane; x < e; x += 32) {
    float v;
    if constexpr (LD == DWM_BF16)
      v = __uint_as_float((uint32_t)static_cast<const uint16_t*>(logits)[row + x] << 16);
    else
      v = static_cast<const float*>(logits)[row + x];
    score[x] = v;
    mx = fmaxf(mx, v);
  }
  if (scoring == DWM_SCORE_SOFTMAX) {
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    for (int x = lane; x < e; x += 32) {
      const float ex = expf(score[x] - mx);
      score[x] = ex;
      sum += ex;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    for (int x = lane; x < e; x += 32) score[x] = score[x] / sum;
  } else if (scoring == DWM_SCORE_SIGMOID) {
    for (int x = lane; x < e; x += 32) score[x] = 1.0f / (1.0f + expf(-score[x]));
  } else {
    for (int x = lane; x < e; x += 32) {
      const float v = score[x];
      score[x] = sqrtf(fmaxf(v, 0.0f) + log1pf(expf(-fabsf(v))));
    }
  }
  for (int x = lane; x < e; x += 32) sel[x] = bias ? score[x] + bias[x] : score[x];
  __syncwarp();

  const bool valid = num_valid < 0 || tok < num_valid;
  float wk_mine = 0.0f;  // lane k keeps the k-th weight
  int id_mine = 0;
  if (hash_ids) {
    if (lane < top_k) {
      int id = hash_ids[(int64_t)tok * top_k + lane];
      if (id < 0 || id >= e) {
        report(status, DWM_DEV_BAD_INDEX);
        id = 0;
      }
      id_mine = id;
      wk_mine = score[id];
    }
  }
  for (int k = 0; k < (hash_ids ? 0 : top_k); ++k) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int x = lane; x < e; x += 32) {
      const float v = sel[x];
      if (better(v, x, bv, bi)) { bv = v; bi = x; }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (bi < 0 || bi >= e) bi = 0;  // all -inf / NaN row: fall back to expert 0
    if (lane == k) {
      id_mine = bi;
      wk_mine = score[bi];
    }
    __syncwarp();
    if (lane == 0) sel[bi] = -INFINITY;
    __syncwarp();
  }
  if (renormalize) {
    // Sum in k order by lane 0, then broadcast.
    float s = 0.0f;
    for (int k = 0; k < top_k; ++k) s += __shfl_sync(0xffffffffu, wk_mine, k);
    wk_mine = wk_mine / s;
  }
  if (!valid) {
    id_mine = 0;
    wk_mine = 0.0f;
  }
  if (lane < top_k) {
    ids[(int64_t)tok * top_k + lane] = id_mine;
    if (w32) w32[(int64_t)tok * top_k + lane] = wk_mine;
    if (w16) w16[(int64_t)tok * top_k + lane] = (uint16_t)f32_to_bf16_bits(wk_mine);
  }
}

__global__ void e8m0_encode_kernel(const float* __restrict__ s, size_t n, uint8_t* __restrict__ c,
                                   int32_t* violation) {
  bool bad = false;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t bits = __float_as_uint(s[i]);
    const uint32_t ex = bits >> 23;
    bad |= ((bits & 0x807FFFFFu) != 0u) || ex == 255u;
    c[i] = (uint8_t)ex;
  }
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(violation, 1);
}

__global__ void flip_flag_kernel(int32_t* f) { *f = (*f == 0) ? 1 : 0; }

__global__ void e8m0_decode_kernel(const uint8_t* __restrict__ c, size_t n, float* __restrict__ o) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    o[i] = __uint_as_float((uint32_t)c[i] << 23);
}

inline unsigned grid_for(size_t work, int threads) {
  size_t b = (work + threads - 1) / threads;
  size_t cap = (size_t)num_sms() * 16;
  return (unsigned)std::max<size_t>(1, std::min(b, cap));
}

}  // namespace route
}  // namespace dwm

using namespace dwm;

namespace dwm {
namespace route {

static int route_impl(const void* logits, int logits_dtype, int t, int e, int top_k, int scoring,
                      int renormalize, const float* bias, const int32_t* hash_ids,
                      int num_valid_tokens, int32_t* topk_ids, float* topk_weights_f32,
                      void* topk_weights_bf16, void* stream) {
  DWM_CHECK_ARG(logits_dtype == DWM_BF16 || logits_dtype == DWM_F32,
                "logits dtype must be bf16 or f32");
  DWM_CHECK_ARG(t >= 0 && e >= 1 && e <= 4096, "bad shape t=%d e=%d", t, e);
  DWM_CHECK_ARG(top_k >= 1 && top_k <= 32 && top_k <= e, "top_k=%d must be in [1, min(32, e)]",
                top_k);
  DWM_CHECK_ARG(scoring == DWM_SCORE_SOFTMAX || scoring == DWM_SCORE_SIGMOID ||
                    scoring == DWM_SCORE_SQRTSOFTPLUS,
                "unknown scoring function %d", scoring);
  DWM_CHECK_ARG(t == 0 || (logits && topk_ids), "NULL pointer");
  if (t == 0) return DWM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t smem = (size_t)WARPS * 2 * e * sizeof(float);
  if (smem > 48 * 1024) {
    auto fn = logits_dtype == DWM_BF16 ? route_topk_kernel<DWM_BF16> : route_topk_kernel<DWM_F32>;
    int rc = check_cuda(
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
        "route smem attribute");
    if (rc) return rc;
  }
  const unsigned grid = (unsigned)((t + WARPS - 1) / WARPS);
  auto w16 = static_cast<uint16_t*>(topk_weights_bf16);
  if (logits_dtype == DWM_BF16)
    route_topk_kernel<DWM_BF16><<<grid, 32 * WARPS, smem, s>>>(
        logits, t, e, top_k, scoring, renormalize, bias, num_valid_tokens, hash_ids, topk_ids,
        topk_weights_f32, w16, status_ptr());
  else
    route_topk_kernel<DWM_F32><<<grid, 32 * WARPS, smem, s>>>(
        logits, t, e, top_k, scoring, renormalize, bias, num_valid_tokens, hash_ids, topk_ids,
        topk_weights_f32, w16, status_ptr());
  return check_cuda(cudaGetLastError(), "route_topk launch");
}

// dedupe_topk (E0901:98-121), one thread per token, in place: a repeated
// expert id adds its f32 weight to the first occurrence and is re-pointed at
// the lowest of experts 0 .. min(2k, e) - 1 the token does not use, weight 0.
__global__ void dedupe_kernel(float* __restrict__ w, int32_t* __restrict__ ids, int t, int top_k,
                              int e, uint16_t* __restrict__ w16) {
  const int tok = blockIdx.x * blockDim.x + threadIdx.x;
  if (tok >= t) return;
  float* wr = w + (int64_t)tok * top_k;
  int32_t* ir = ids + (int64_t)tok * top_k;
  const int ncand = min(2 * top_k, e);
  for (int j = 1; j < top_k; ++j) {
    int first = -1;
    for (int q = 0; q < j; ++q)
      if (ir[q] == ir[j]) {
        first = q;
        break;
      }
    if (first < 0) continue;
    wr[first] = __fadd_rn(wr[first], wr[j]);
    int free_id = 0;  // argmin over "used": the first unused candidate, else 0
    for (int c = 0; c < ncand; ++c) {
      bool used = false;
      for (int q = 0; q < top_k; ++q) used |= ir[q] == c;
      if (!used) {
        free_id = c;
        break;
      }
    }
    ir[j] = free_id;
    wr[j] = 0.0f;
  }
  if (w16)
    for (int q = 0; q < top_k; ++q)
      w16[(int64_t)tok * top_k + q] = (uint16_t)f32_to_bf16_bits(wr[q]);
}

}  // namespace route
}  // namespace dwm

extern "C" int dwm_route_topk(const void* logits, int logits_dtype, int t, int e, int top_k,
                              int scoring, int renormalize, const float* bias,
                              int num_valid_tokens, int32_t* topk_ids, float* topk_weights_f32,
                              void* topk_weights_bf16, void* stream) {
  return route::route_impl(logits, logits_dtype, t, e, top_k, scoring, renormalize, bias, nullptr,
                           num_valid_tokens, topk_ids, topk_weights_f32, topk_weights_bf16,
                           stream);
}

extern "C" int dwm_route_hash(const void* logits, int logits_dtype, int t, int e, int top_k,
                              int scoring, int renormalize, const int32_t* hash_ids,
                              int num_valid_tokens, int32_t* topk_ids, float* topk_weights_f32,
                              void* topk_weights_bf16, void* stream) {
  DWM_CHECK_ARG(t == 0 || hash_ids, "NULL hash_ids");
  return route::route_impl(logits, logits_dtype, t, e, top_k, scoring, renormalize, nullptr,
                           hash_ids, num_valid_tokens, topk_ids, topk_weights_f32,
                           topk_weights_bf16, stream);
}

extern "C" int dwm_dedupe_topk(float* topk_weights_f32, int32_t* topk_ids, int t, int top_k,
                               int num_experts, void* topk_weights_bf16, void* stream) {
  DWM_CHECK_ARG(t >= 0 && top_k >= 1 && top_k <= 32 && num_experts >= 1, "bad shape");
  DWM_CHECK_ARG(t == 0 || (topk_weights_f32 && topk_ids), "NULL pointer");
  if (t == 0) return DWM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  route::dedupe_kernel<<<(t + 127) / 128, 128, 0, s>>>(topk_weights_f32, topk_ids, t, top_k,
                                                       num_experts,
                                                       static_cast<uint16_t*>(topk_weights_bf16));
  return check_cuda(cudaGetLastError(), "dedupe_topk launch");
}

extern "C" int dwm_e8m0_encode(const float* scale, size_t n, uint8_t* codes,
                               int32_t* lossless_dev, void* stream) {
  DWM_CHECK_ARG(lossless_dev && (n == 0 || (scale && codes)), "NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = check_cuda(cudaMemsetAsync(lossless_dev, 0, sizeof(int32_t), s), "e8m0 flag");
  if (rc) return rc;
  if (n) {
    route::e8m0_encode_kernel<<<route::grid_for(n, 256), 256, 0, s>>>(scale, n, codes,
                                                                      lossless_dev);
    rc = check_cuda(cudaGetLastError(), "e8m0_encode launch");
    if (rc) return rc;
  }
  route::flip_flag_kernel<<<1, 1, 0, s>>>(lossless_dev);
  return check_cuda(cudaGetLastError(), "e8m0 flag launch");
}

extern "C" int dwm_e8m0_decode(const uint8_t* codes, size_t n, float* out, void* stream) {
  DWM_CHECK_ARG(n == 0 || (codes && out), "NULL pointer");
  if (n == 0) return DWM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  route::e8m0_decode_kernel<<<route::grid_for(n, 256), 256, 0, s>>>(codes, n, out);
  return check_cuda(cudaGetLastError(), "e8m0_decode launch");
}
