// FP4 (e2m1) decode shared by the grouped-matmul kernels, and the B200
// load-time weight layout.
//
// Every decode produces, for a 32-bit word of 8 FP4 values, four bf16x2 words
// t[0..3] holding the e2m1 values times 2^-126 exactly: the 3 magnitude bits
// land in the bf16 exponent LSBs and the top mantissa bit, so the e2m1
// subnormal 0.5 becomes the bf16 subnormal 2^-127. One bf16 multiply by
// m1 = 2^(126 - delta) * scale then yields value * scale * 2^-delta rounded
// once, which is exact (power-of-two scales) and equals the reference's
// bf16(value) * bf16(scale) (E0901:84-95) up to the 2^-delta factor the
// epilogues remove exactly in f32. When m1 is not representable (E8M0 code 0
// or above 128 + delta, or non-E8M0 scales) the multiply is split in two
// (m1 = 2^(126 - delta), m2 = scale).
//
//   raw e2m1 word  8 columns c..c+7 at one k, column c+j in bits 4j..4j+3.
//                  Word i of the decode holds columns (c+i, c+i+4).
//   B200 word      the 8 A-fragment values of one lane of an m16n8k16 MMA
//                  (weight columns gid, gid+8 x k pairs 2t, 2t+8 of a 16x16
//                  block) with their bits permuted so each bf16x2 pair is one
//                  PRMT lookup in an 8-byte table; word i is fragment
//                  register i.
#pragma once

#include "common.cuh"

namespace dwm {
namespace fp4 {

template <int SD>
struct ScaleTraits;
template <>
struct ScaleTraits<DWM_U8> {
  static constexpr int bytes = 1;
  static constexpr CUtensorMapDataType tma = CU_TENSOR_MAP_DATA_TYPE_UINT8;
};
template <>
struct ScaleTraits<DWM_BF16> {
  static constexpr int bytes = 2;
  static constexpr CUtensorMapDataType tma = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
};
template <>
struct ScaleTraits<DWM_F32> {
  static constexpr int bytes = 4;
  static constexpr CUtensorMapDataType tma = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
};

// PRMT table: bytes 0-3 give the bf16 low byte by (e0, m), bytes 4-7 the high
// byte by (sign, e1).
constexpr uint32_t kLutLo = 0xC0804000u;
constexpr uint32_t kLutHi = 0x81800100u;

// PTX prmt in its default mode. The selectors built below never set bit 3
// of a nibble (the sign-replicate bit), so this is exactly __byte_perm, whose
// documented semantics would make the compiler mask every selector first.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

template <bool B200>
__device__ __forceinline__ void tvals(uint32_t w, uint32_t (&t)[4]) {
  if constexpr (!B200) {
    t[0] = ((w << 6) & 0x01C001C0u) | ((w << 12) & 0x80008000u);
    t[1] = ((w << 2) & 0x01C001C0u) | ((w << 8) & 0x80008000u);
    t[2] = ((w >> 2) & 0x01C001C0u) | ((w << 4) & 0x80008000u);
    t[3] = ((w >> 6) & 0x01C001C0u) | (w & 0x80008000u);
  } else {
    const uint32_t x = (w & 0x33333333u) | 0x40404040u;
    const uint32_t y = ((w >> 2) & 0x33333333u) | 0x40404040u;
    t[0] = prmt(kLutLo, kLutHi, x);
    t[1] = prmt(kLutLo, kLutHi, y);
    t[2] = prmt(kLutLo, kLutHi, x >> 16);
    t[3] = prmt(kLutLo, kLutHi, y >> 16);
  }
}

// The B200 decode with its constants held in registers. pin() hides a value
// from the compiler, so the four constants are materialised once per kernel
// and stay in registers, and each selector is one LOP3 ((w & m33) | c40).
__device__ __forceinline__ uint32_t pin(uint32_t v) {
  asm volatile("mov.b32 %0, %0;" : "+r"(v));
  return v;
}
struct DecodeRegs {
  uint32_t lut_lo, lut_hi, m33, c40;
  __device__ __forceinline__ static DecodeRegs make() {
    return {pin(kLutLo), pin(kLutHi), pin(0x33333333u), pin(0x40404040u)};
  }
};
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));  // (a & b) | c
  return d;
}
__device__ __forceinline__ void tvals_b200(uint32_t w, const DecodeRegs& R, uint32_t (&t)[4]) {
  const uint32_t x = lop3_and_or(w, R.m33, R.c40);
  const uint32_t y = lop3_and_or(w >> 2, R.m33, R.c40);
  t[0] = prmt(R.lut_lo, R.lut_hi, x);
  t[1] = prmt(R.lut_lo, R.lut_hi, y);
  t[2] = prmt(R.lut_lo, R.lut_hi, x >> 16);
  t[3] = prmt(R.lut_lo, R.lut_hi, y >> 16);
}

template <bool B200, bool TWO>
__device__ __forceinline__ uint4 decode8(uint32_t w, const uint32_t (&m1)[4],
                                         const uint32_t (&m2)[4]) {
  uint32_t t[4];
  tvals<B200>(w, t);
  uint4 v;
  v.x = hmul2_bf16(t[0], m1[0]);
  v.y = hmul2_bf16(t[1], m1[1]);
  v.z = hmul2_bf16(t[2], m1[2]);
  v.w = hmul2_bf16(t[3], m1[3]);
  if constexpr (TWO) {
    v.x = hmul2_bf16(v.x, m2[0]);
    v.y = hmul2_bf16(v.y, m2[1]);
    v.z = hmul2_bf16(v.z, m2[2]);
    v.w = hmul2_bf16(v.w, m2[3]);
  }
  return v;
}

// Exponent bias folded into the decode for E8M0 scales (removed in the
// epilogue): one multiply then covers codes 1..128 + kDelta.
constexpr int kDelta = 4;

template <int SD>
__host__ __device__ constexpr int decode_delta() { return SD == DWM_U8 ? kDelta : 0; }

template <int DELTA>
__host__ __device__ constexpr uint32_t pow2_126_minus_delta_x2() {
  return ((uint32_t)(253 - DELTA) << 7) * 0x10001u;  // bf16 2^(126-delta), twice
}

// Multiplier pair for one scale (both bf16 halves the same). Returns true if
// the two-step multiply is needed.
template <int SD, int DELTA>
__device__ __forceinline__ bool col_mult(const uint8_t* sp, uint32_t& m1, uint32_t& m2) {
  constexpr uint32_t kPow2x2 = pow2_126_minus_delta_x2<DELTA>();
  if constexpr (SD == DWM_U8) {
    const uint32_t c = *sp;
    m2 = (c << 7) * 0x10001u;  // 2^(c-127); c = 0 -> +0
    if (c >= 1u && c <= 128u + DELTA) {
      m1 = ((c + 126u - DELTA) << 7) * 0x10001u;  // 2^(c-1-delta)
      return false;
    }
    m1 = kPow2x2;
    return true;
  } else if constexpr (SD == DWM_BF16) {
    m2 = (uint32_t)(*reinterpret_cast<const uint16_t*>(sp)) * 0x10001u;
    m1 = kPow2x2;
    return true;
  } else {
    m2 = f32_to_bf16_bits(*reinterpret_cast<const float*>(sp)) * 0x10001u;
    m1 = kPow2x2;
    return true;
  }
}

// Multipliers for the 8 scales of raw columns c..c+7, paired (i, i+4) like
// the raw decode's output words.
template <int SD, int DELTA>
__device__ __forceinline__ bool raw_mults(const uint8_t* sp, uint32_t (&m1)[4],
                                          uint32_t (&m2)[4]) {
  constexpr uint32_t kPow2x2 = pow2_126_minus_delta_x2<DELTA>();
  if constexpr (SD == DWM_U8) {
    const uint2 raw = *reinterpret_cast<const uint2*>(sp);  // c0..c3 | c4..c7
    const uint32_t a = __byte_perm(raw.x, raw.y, 0x5140);   // c0 c4 c1 c5
    const uint32_t b = __byte_perm(raw.x, raw.y, 0x7362);   // c2 c6 c3 c7
    uint32_t p[4];                                           // (c_lo, c_hi) per half
    p[0] = __byte_perm(a, 0, 0x4140);
    p[1] = __byte_perm(a, 0, 0x4342);
    p[2] = __byte_perm(b, 0, 0x4140);
    p[3] = __byte_perm(b, 0, 0x4342);
    // Fast path needs every code in [1, 128 + DELTA]: bit 8 of c + 255 set
    // (c >= 1) and bit 8 of c + 127 - DELTA clear (c <= 128 + DELTA).
    uint32_t bad = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      bad |= ~(p[i] + 0x00FF00FFu) | (p[i] + (uint32_t)(127 - DELTA) * 0x10001u);
      m1[i] = p[i] * 128u + (uint32_t)((126 - DELTA) << 7) * 0x10001u;
      m2[i] = p[i] << 7;
    }
    if (bad & 0x01000100u) {
#pragma unroll
      for (int i = 0; i < 4; ++i) m1[i] = kPow2x2;
      return true;
    }
    return false;
  } else if constexpr (SD == DWM_BF16) {
    const uint4 raw = *reinterpret_cast<const uint4*>(sp);  // (s0,s1),(s2,s3),(s4,s5),(s6,s7)
    m2[0] = __byte_perm(raw.x, raw.z, 0x5410);               // s0 s4
    m2[1] = __byte_perm(raw.x, raw.z, 0x7632);               // s1 s5
    m2[2] = __byte_perm(raw.y, raw.w, 0x5410);               // s2 s6
    m2[3] = __byte_perm(raw.y, raw.w, 0x7632);               // s3 s7
#pragma unroll
    for (int i = 0; i < 4; ++i) m1[i] = kPow2x2;
    return true;
  } else {
    const float4 a = *reinterpret_cast<const float4*>(sp);
    const float4 b = *reinterpret_cast<const float4*>(sp + 16);
    const float sc[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      m1[i] = kPow2x2;
      m2[i] = f32_to_bf16_bits(sc[i]) | (f32_to_bf16_bits(sc[i + 4]) << 16);
    }
    return true;
  }
}

// --- the B200 word permutation --------------------------------------------
// Output pair p (nibbles 2p, 2p+1 of the plain word, byte p) moves its 2-bit
// fields (bits 1:0, 3:2 of the low nibble, 1:0, 3:2 of the high nibble) to
// bits B, B+4, B+8, B+12 with B = 0, 2, 16, 18 for p = 0..3.
__host__ __device__ __forceinline__ uint32_t b200_swizzle_word(uint32_t w) {
  uint32_t o = 0;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t byte = (w >> (8 * p)) & 0xFFu;
    const int base = (p & 1) * 2 + (p >> 1) * 16;
    o |= ((byte >> 0) & 3u) << base;
    o |= ((byte >> 2) & 3u) << (base + 4);
    o |= ((byte >> 4) & 3u) << (base + 8);
    o |= ((byte >> 6) & 3u) << (base + 12);
  }
  return o;
}

__host__ __device__ __forceinline__ uint32_t b200_unswizzle_word(uint32_t o) {
  uint32_t w = 0;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const int base = (p & 1) * 2 + (p >> 1) * 16;
    uint32_t byte = ((o >> base) & 3u) | (((o >> (base + 4)) & 3u) << 2) |
                    (((o >> (base + 8)) & 3u) << 4) | (((o >> (base + 12)) & 3u) << 6);
    w |= byte << (8 * p);
  }
  return w;
}

// --- the B200 weight layout ---------------------------------------------------
// Weights [g, k, n] are stored as u32 words [g][n/16][k/16][32]: the 16x16
// block (column block cb, k block kb) is 32 words, word l (gid = l/4, t = l%4)
// holding, in nibble order j = 0..7 before the permutation,
//   (k, col) = (2t, gid) (2t+1, gid) (2t, gid+8) (2t+1, gid+8)
//              (2t+8, gid) (2t+9, gid) (2t+8, gid+8) (2t+9, gid+8)
// relative to (16 kb, 16 cb): the A fragment of mma.m16n8k16 for W^T.
__host__ __device__ __forceinline__ void b200_nibble_coord(int l, int j, int& dk, int& dc) {
  const int gid = l >> 2, t = l & 3;
  dk = 2 * t + (j & 1) + ((j >> 2) << 3);
  dc = gid + (((j >> 1) & 1) << 3);
}

__host__ __device__ __forceinline__ int64_t b200_word_index(int64_t g, int cb, int kb, int l,
                                                            int n, int k) {
  return ((g * (n / 16) + cb) * (int64_t)(k / 16) + kb) * 32 + l;
}

}  // namespace fp4
}  // namespace dwm
