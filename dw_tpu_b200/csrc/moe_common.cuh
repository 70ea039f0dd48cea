// Device pieces shared by the single-device permute/combine kernels
// (permute.cu) and the expert-parallel exchange (ep.cu), so both produce the
// same bits.
#pragma once

#include "common.cuh"

namespace dwm {
namespace moe {

constexpr int SORT_THREADS = 1024;
constexpr int SORT_WARPS = SORT_THREADS / 32;

// Dynamic shared memory the counting sort needs for e experts.
inline size_t sort_smem_bytes(int e) { return (size_t)(SORT_WARPS * e + e) * sizeof(int); }

// Stable counting sort of the n = t * topk expert ids by expert (KD:41-44,
// X0405:73-88: stable argsort of the flattened ids, argsort // topk, bincount)
// run by one CTA of SORT_THREADS threads: per-warp histograms, an exclusive
// scan, then an in-order scatter in which each warp ranks equal experts with
// __match_any_sync. Stability holds because warps own contiguous, ordered
// segments. Outputs (each optional): argsort[pos] = j, tok[pos] = j / topk,
// revert[j] = pos (-1 for an id outside [0, e), which is also reported),
// group_sizes[x] = count of expert x, prefix[x] = exclusive prefix of the
// counts. sm: sort_smem_bytes(e) of shared memory.
__device__ __forceinline__ void counting_sort_block(const int32_t* __restrict__ ids, int n,
                                                    int topk, int e, int32_t* argsort,
                                                    int32_t* tok, int32_t* revert,
                                                    int32_t* group_sizes, int32_t* prefix,
                                                    int* status, int* sm) {
  int* hist = sm;                     // [W][e]
  int* totals = sm + SORT_WARPS * e;  // [e]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < SORT_WARPS * e; i += blockDim.x) hist[i] = 0;
  __syncthreads();

  // Contiguous segment per warp, a multiple of 32 entries.
  const int seg = ((n + SORT_WARPS - 1) / SORT_WARPS + 31) & ~31;
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
    for (int w = 0; w < SORT_WARPS; ++w) {
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
        if (prefix) prefix[x] = run;
        run += v;
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < SORT_WARPS * e; i += blockDim.x) hist[i] += totals[i % e];
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

// 8 consecutive elements (bf16 or f32) at element offset off, as f32.
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

// Same, bypassing L1 (data another GPU wrote during this kernel's lifetime).
template <int XD>
__device__ __forceinline__ void load8_cg(const void* x, int64_t off, float (&v)[8]) {
  if constexpr (XD == DWM_BF16) {
    const uint4 q = __ldcg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + off));
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  } else {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(static_cast<const float*>(x) + off));
    const float4 b =
        __ldcg(reinterpret_cast<const float4*>(static_cast<const float*>(x) + off + 4));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

// 8 consecutive bf16 elements kept packed (4 registers), bypassing L1.
__device__ __forceinline__ uint4 load8_bf16_raw_cg(const void* x, int64_t off) {
  return __ldcg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + off));
}

// acc <- acc + bf16x8(q) * w, as mul_add8 on the unpacked values.
__device__ __forceinline__ void mul_add8_bf16raw(float (&acc)[8], const uint4& q, float w) {
  const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    acc[2 * i] = __fadd_rn(acc[2 * i], __fmul_rn(__uint_as_float(u[i] << 16), w));
    acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], __fmul_rn(__uint_as_float(u[i] & 0xFFFF0000u), w));
  }
}

template <int WD>
__device__ __forceinline__ float load_weight(const void* w, int64_t i) {
  if constexpr (WD == DWM_BF16)
    return __uint_as_float((uint32_t)static_cast<const uint16_t*>(w)[i] << 16);
  else
    return static_cast<const float*>(w)[i];
}

// acc <- acc + v * w with the product and the sum rounded separately (no FMA
// contraction), the combine contract of KC:14-21.
__device__ __forceinline__ void mul_add8(float (&acc)[8], const float (&v)[8], float w) {
#pragma unroll
  for (int q = 0; q < 8; ++q) acc[q] = __fadd_rn(acc[q], __fmul_rn(v[q], w));
}

template <int OD>
__device__ __forceinline__ void store8(void* out, int64_t off, const float (&acc)[8]) {
  if constexpr (OD == DWM_BF16) {
    uint4 o;
    o.x = f32_to_bf16_bits(acc[0]) | (f32_to_bf16_bits(acc[1]) << 16);
    o.y = f32_to_bf16_bits(acc[2]) | (f32_to_bf16_bits(acc[3]) << 16);
    o.z = f32_to_bf16_bits(acc[4]) | (f32_to_bf16_bits(acc[5]) << 16);
    o.w = f32_to_bf16_bits(acc[6]) | (f32_to_bf16_bits(acc[7]) << 16);
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + off) = o;
  } else {
    float* o = static_cast<float*>(out) + off;
    *reinterpret_cast<float4*>(o) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    *reinterpret_cast<float4*>(o + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
}

// The shared expert summed into the routed combine (MOE_SHARED_EXPERT_TP,
// X0104:80-87 of the patch): out = f32(mid(routed)) * scale + shared, where
// mid rounds the routed k-order sum to bf16 (the combine's own output dtype)
// or keeps it f32 (MOE_F32_REDUCE); each step is rounded to f32 on its own.
// p == nullptr: no shared expert (the plain combine).
struct SharedAdd {
  const void* p;
  int f32;       // shared partial dtype: 1 = f32, 0 = bf16
  float scale;   // routed_scale
  int mid_bf16;  // 1: round the routed sum to bf16 first
};

__device__ __forceinline__ void shared_add8(float (&acc)[8], const SharedAdd& s, int64_t off) {
  if (s.p == nullptr) return;
  float sh[8];
  if (s.f32)
    load8<DWM_F32>(s.p, off, sh);
  else
    load8<DWM_BF16>(s.p, off, sh);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    float v = acc[q];
    if (s.mid_bf16) v = __uint_as_float(f32_to_bf16_bits(v) << 16);
    acc[q] = __fadd_rn(__fmul_rn(v, s.scale), sh[q]);
  }
}

inline unsigned grid_for(int64_t work, int threads, int per_sm = 16) {
  const int64_t b = (work + threads - 1) / threads;
  const int64_t cap = (int64_t)num_sms() * per_sm;
  return (unsigned)(b < 1 ? 1 : (b < cap ? b : cap));
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace moe
}  // namespace dwm
