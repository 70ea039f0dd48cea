// On-device FP4 weight preparation: quantize_tensor(float4_e2m1fn, w,
// block_size=32, power_of_two_scale) (B01:319-347) over blocks of 32
// consecutive k of each column of a [groups, k, n] expert weight, straight
// into the layouts the grouped matmul reads: packed e2m1 codes [g, k, n/2]
// (element 2j in the low nibble) and per-32 scales [g, k/32, n] as E8M0 codes
// (KE:28-40) or f32. Re-quantising an MXFP4 checkpoint (e2m1 + power-of-two
// scale per 32) this way with power-of-two scales reproduces it exactly
// (B01:131-157).
//
// Per block: scale = absmax / 6 (f32); with power_of_two_scale, the scale is
// rounded up to 2^ceil(log2 scale) (frexp: a mantissa of exactly 0.5 means it
// already is a power of two); q = w / scale (0 for a zero scale) rounded to
// the nearest e2m1 value, ties to the even mantissa, saturating at 6; a
// negative value that rounds to 0 becomes +0.
#include <algorithm>

#include "common.cuh"

namespace dwm {
namespace quant {

// e2m1 magnitude grid: 0 .5 1 1.5 2 3 4 6 (codes 0..7).
__device__ __forceinline__ uint32_t round_to_e2m1(float x) {
  const float a = fminf(fabsf(x), 6.0f);
  // Midpoints between grid values; a tie goes to the even code (even
  // mantissa bit), so the comparison is strict or not per midpoint.
  uint32_t c;
  if (a <= 0.25f) c = 0;        // tie 0.25 -> 0 (even)
  else if (a < 0.75f) c = 1;    // tie 0.75 -> 2 (even)
  else if (a <= 1.25f) c = 2;   // tie 1.25 -> 2 (even)
  else if (a < 1.75f) c = 3;    // tie 1.75 -> 4 (even)
  else if (a <= 2.5f) c = 4;    // tie 2.5 -> 4 (even)
  else if (a < 3.5f) c = 5;     // tie 3.5 -> 6 (even)
  else if (a <= 5.0f) c = 6;    // tie 5 -> 6 (even)
  else c = 7;
  return (c != 0 && signbit(x)) ? (c | 8u) : c;
}

__device__ __forceinline__ float pow2_ceil(float s) {
  int e;
  const float m = frexpf(s, &e);  // s = m * 2^e, m in [0.5, 1)
  return ldexpf(1.0f, m == 0.5f ? e - 1 : e);
}

// One thread per (group, k block, column pair): two columns' blocks of 32,
// so the two nibbles of each output byte come from one thread.
template <typename T>
__global__ void quantize_kernel(const T* __restrict__ w, int groups, int k, int n, int pow2,
                                uint8_t* __restrict__ codes, void* __restrict__ scales,
                                int scale_u8, int32_t* lossless) {
  const int np = n / 2;
  const int kb32 = k / 32;
  const int64_t total = (int64_t)groups * kb32 * np;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int cp = (int)(i % np);
    const int64_t gk = i / np;
    const int kb = (int)(gk % kb32);
    const int64_t g = gk / kb32;
    const int64_t base = (g * k + (int64_t)kb * 32) * n + 2 * cp;  // w[g, 32kb, 2cp]
    float amax[2] = {0.0f, 0.0f};
#pragma unroll 8
    for (int r = 0; r < 32; ++r) {
#pragma unroll
      for (int h = 0; h < 2; ++h)
        amax[h] = fmaxf(amax[h], fabsf((float)w[base + (int64_t)r * n + h]));
    }
    float sc[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      sc[h] = __fdiv_rn(amax[h], 6.0f);
      if (pow2 && sc[h] > 0.0f) sc[h] = pow2_ceil(sc[h]);
      const int64_t so = (g * kb32 + kb) * (int64_t)n + 2 * cp + h;
      if (scale_u8) {
        const uint32_t bits = __float_as_uint(sc[h]);
        // E8M0 holds the exponent of a positive power of two (or +0).
        if ((bits & 0x807FFFFFu) != 0u || (bits >> 23) == 255u) atomicAnd(lossless, 0);
        static_cast<uint8_t*>(scales)[so] = (uint8_t)(bits >> 23);
      } else {
        static_cast<float*>(scales)[so] = sc[h];
      }
    }
#pragma unroll 8
    for (int r = 0; r < 32; ++r) {
      uint32_t byte = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float v = (float)w[base + (int64_t)r * n + h];
        const float q = sc[h] > 0.0f ? __fdiv_rn(v, sc[h]) : 0.0f;
        byte |= round_to_e2m1(q) << (4 * h);
      }
      codes[(g * k + (int64_t)kb * 32 + r) * np + cp] = (uint8_t)byte;
    }
  }
}

__global__ void set_one_kernel(int32_t* p) { *p = 1; }

}  // namespace quant
}  // namespace dwm

using namespace dwm;

extern "C" int dwm_fp4_quantize(const void* w, int w_dtype, int groups, int k, int n, int pow2,
                                void* codes, void* scales, int scale_dtype,
                                int32_t* lossless_dev, void* stream) {
  DWM_CHECK_ARG(w_dtype == DWM_BF16 || w_dtype == DWM_F32, "weights must be bf16 or f32");
  DWM_CHECK_ARG(scale_dtype == DWM_U8 || scale_dtype == DWM_F32,
                "scales are written as u8 (E8M0) or f32");
  DWM_CHECK_ARG(groups >= 0 && k > 0 && n > 0 && k % 32 == 0 && n % 2 == 0,
                "bad shape groups=%d k=%d n=%d (k %% 32, n %% 2)", groups, k, n);
  DWM_CHECK_ARG(scale_dtype != DWM_U8 || (pow2 && lossless_dev),
                "E8M0 scales need power_of_two_scale and a lossless flag");
  DWM_CHECK_ARG(groups == 0 || (w && codes && scales), "NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int su8 = scale_dtype == DWM_U8;
  if (su8) {
    quant::set_one_kernel<<<1, 1, 0, s>>>(lossless_dev);
    int rc = check_cuda(cudaGetLastError(), "quantize flag");
    if (rc) return rc;
  }
  const int64_t total = (int64_t)groups * (k / 32) * (n / 2);
  if (total == 0) return DWM_OK;
  const unsigned grid = (unsigned)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 16);
  if (w_dtype == DWM_BF16)
    quant::quantize_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(w), groups, k, n, pow2, static_cast<uint8_t*>(codes),
        scales, su8, lossless_dev);
  else
    quant::quantize_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(w), groups, k, n,
                                                        pow2, static_cast<uint8_t*>(codes),
                                                        scales, su8, lossless_dev);
  return check_cuda(cudaGetLastError(), "fp4_quantize launch");
}
