// FP4 grouped matmul for sm_100a: tokamax gmm_v2 with rhs_fp4_codes
// (TK:107-153), decoded in shared memory and multiplied on tcgen05 tensor
// cores with the accumulator in TMEM.
//
// Design (one persistent CTA per SM, 16 warps):
//   warps 0-3   epilogue: TMEM -> registers -> (SwiGLU) -> global
//   warp  4     TMA producer: e2m1 codes + scales ring, token-row ring
//   warp  5     TMEM allocator and single-thread UMMA issuer
//   warps 8-15  decode: e2m1 nibbles x scale -> bf16 tiles in swizzled SMEM
//
// The product is computed transposed ("swap AB"): the decoded weight tile
// W[k, n0:n0+128] is UMMA operand A (M = 128 weight columns, MN-major, 128B
// swizzle) and the token rows X[r0:r0+rows, k] are operand B (N = rows
// rounded up to 16, K-major, 128B swizzle, loaded by TMA). A decode-sized
// group of 2 rows then costs an N = 16 MMA instead of wasting a 128-row
// tile, and prefill-sized groups run N = 128. Each tile carries two 128-column
// sub-tiles (two accumulators): adjacent columns for a plain GEMM, or the
// matching gate and up columns for the fused SwiGLU.
//
// Numerics follow the reference order (E0901:84-95): each e2m1 value is
// decoded exactly to bf16, multiplied by the bf16 scale in one bf16 multiply
// (round to nearest even), then the MMA accumulates bf16 x bf16 products in
// f32; the epilogue applies SwiGLU in f32 and rounds once to the output type.
#include "common.cuh"

namespace dwm {
namespace gmm {

constexpr int NSUB = 2;    // sub-tiles (accumulators) per tile
constexpr int BW = 128;    // weight columns per sub-tile (UMMA M)
constexpr int BK = 64;     // K per pipeline stage (128 bytes of bf16)
constexpr int BT = 128;    // max token rows per tile (UMMA N)
constexpr int CS = 6;      // codes+scales stages
constexpr int TS = 3;      // token-row stages
constexpr int AS = 3;      // decoded-weight stages
constexpr int NUM_THREADS = 512;
constexpr int PRODUCER_WARP = 4;
constexpr int MMA_WARP = 5;
constexpr int DEC_WARP0 = 8;
constexpr int NUM_DEC_WARPS = 8;
constexpr int MAX_GROUPS = 1024;
constexpr int TMEM_COLS = 512;  // 2 buffers x NSUB x BT f32 columns

constexpr int A_SUB_BYTES = BW * BK * 2;     // 16 KiB, MN-major SW128
constexpr int A_STAGE = NSUB * A_SUB_BYTES;  // 32 KiB
constexpr int A_LBO = 8192;                  // MN-atom (64 columns) stride
constexpr int A_SBO = 1024;                  // K-atom (8 rows) stride
constexpr int T_STAGE = BT * BK * 2;         // 16 KiB, K-major SW128
constexpr int T_BOX_ROWS = 16;
constexpr int T_BOX_BYTES = T_BOX_ROWS * BK * 2;  // 2 KiB
constexpr int C_SUB_BYTES = BK * (BW / 2);        // 4 KiB of packed nibbles
// TMA writes shared memory at 128-byte aligned addresses only.
constexpr int C_SUB1_OFF = C_SUB_BYTES;
constexpr int C_STAGE = NSUB * C_SUB_BYTES;
static_assert(C_SUB1_OFF % 128 == 0 && C_STAGE % 128 == 0, "TMA needs 128 B alignment");

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

template <int SD>
struct Smem {
  static constexpr int S_STAGE = NSUB * 2 * BW * ScaleTraits<SD>::bytes;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_T = OFF_A + AS * A_STAGE;
  static constexpr int OFF_C = OFF_T + TS * T_STAGE;
  static constexpr int OFF_S = OFF_C + CS * C_STAGE;
  static constexpr int OFF_BAR = OFF_S + CS * S_STAGE;
  static constexpr int NUM_BARS = 2 * CS + 2 * TS + 2 * AS + 4 + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int OFF_ROWS = OFF_MISC + 16;
  static constexpr int OFF_TILES = OFF_ROWS + (MAX_GROUPS + 1) * 4;
  static constexpr int BYTES = OFF_TILES + (MAX_GROUPS + 1) * 4;
  static constexpr int ALLOC = BYTES + 1024;  // slack for 1 KiB alignment
};

struct Args {
  const int32_t* group_sizes;
  int num_groups, group_offset, n_local;
  int m, k, n;
  int act;
  float limit;
  int out_f32;
  int zero_init;
  void* out;
  int ldo;  // output row length (n, or n/2 with SwiGLU)
  int n_tiles;  // column tiles per group
  int* status;
};

// Column permutation inside each 8-column group produced by decode8: SMEM
// position p holds column (p >> 1) + 4 * (p & 1).
__device__ __forceinline__ int perm8(int p) { return (p >> 1) + ((p & 1) << 2); }

// Decode one 32-bit word of 8 e2m1 nibbles (columns c..c+7, column c+j in
// bits 4j..4j+3) into 8 bf16 values. Output word i holds columns (c+i,
// c+i+4) in its low/high halves.
//
// (w << s) & 0x01C001C0 drops the 3 magnitude bits into the bf16 exponent
// LSBs and top mantissa bit, and (w << s') & 0x80008000 moves the sign: the
// result is the e2m1 value times 2^-126 exactly (the e2m1 subnormal 0.5 lands
// on the bf16 subnormal 2^-127). One bf16 multiply by 2^126 * scale (m1)
// then gives value * scale rounded once; when that factor would overflow
// bf16 the caller passes m1 = 2^126 and the scale in m2 (two_step).
__device__ __forceinline__ uint4 decode8(uint32_t w, const uint32_t (&m1)[4],
                                         const uint32_t (&m2)[4], bool two_step) {
  uint32_t t0 = ((w << 6) & 0x01C001C0u) | ((w << 12) & 0x80008000u);
  uint32_t t1 = ((w << 2) & 0x01C001C0u) | ((w << 8) & 0x80008000u);
  uint32_t t2 = ((w >> 2) & 0x01C001C0u) | ((w << 4) & 0x80008000u);
  uint32_t t3 = ((w >> 6) & 0x01C001C0u) | (w & 0x80008000u);
  uint4 v;
  v.x = hmul2_bf16(t0, m1[0]);
  v.y = hmul2_bf16(t1, m1[1]);
  v.z = hmul2_bf16(t2, m1[2]);
  v.w = hmul2_bf16(t3, m1[3]);
  if (two_step) {
    v.x = hmul2_bf16(v.x, m2[0]);
    v.y = hmul2_bf16(v.y, m2[1]);
    v.z = hmul2_bf16(v.z, m2[2]);
    v.w = hmul2_bf16(v.w, m2[3]);
  }
  return v;
}

constexpr uint32_t kBf16Pow2_126x2 = 0x7E807E80u;  // bf16 2^126, twice

// Multipliers for the 8 scales s[0..7] of columns c..c+7 (pairs (i, i+4)).
// Returns true if the two-step form is needed for this thread.
template <int SD>
__device__ __forceinline__ bool scale_mults(const uint8_t* sp, uint32_t (&m1)[4],
                                            uint32_t (&m2)[4]) {
  if constexpr (SD == DWM_U8) {
    const uint2 raw = *reinterpret_cast<const uint2*>(sp);
    uint32_t c[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      c[i] = (raw.x >> (8 * i)) & 0xFFu;
      c[i + 4] = (raw.y >> (8 * i)) & 0xFFu;
    }
    bool two = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) two |= c[i] > 128u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // 2^(c-127) has bf16 bits c << 7 (c = 0 -> +0); 2^126 * 2^(c-127) =
      // 2^(c-1) has bits (c + 126) << 7 and is finite for c <= 128.
      uint32_t lo1 = c[i] ? ((c[i] + 126u) << 7) : 0u;
      uint32_t hi1 = c[i + 4] ? ((c[i + 4] + 126u) << 7) : 0u;
      m1[i] = lo1 | (hi1 << 16);
      m2[i] = (c[i] << 7) | (c[i + 4] << 23);
    }
    return two;
  } else if constexpr (SD == DWM_BF16) {
    const uint4 raw = *reinterpret_cast<const uint4*>(sp);
    const uint32_t r[4] = {raw.x, raw.y, raw.z, raw.w};  // (s0,s1),(s2,s3),..
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t lo = (r[i >> 1] >> ((i & 1) * 16)) & 0xFFFFu;
      uint32_t hi = (r[(i + 4) >> 1] >> (((i + 4) & 1) * 16)) & 0xFFFFu;
      m1[i] = kBf16Pow2_126x2;
      m2[i] = lo | (hi << 16);
    }
    return true;
  } else {
    const float4 a = *reinterpret_cast<const float4*>(sp);
    const float4 b = *reinterpret_cast<const float4*>(sp + 16);
    const float s[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      m1[i] = kBf16Pow2_126x2;
      m2[i] = f32_to_bf16_bits(s[i]) | (f32_to_bf16_bits(s[i + 4]) << 16);
    }
    return true;
  }
}

struct Tile {
  int g;      // local group
  int row0;   // first lhs row
  int rows;   // valid rows (1..BT)
  int n_idx;  // column tile
};

__device__ __forceinline__ Tile get_tile(int idx, const int* row_start, const int* tile_prefix,
                                         const Args& a) {
  int lo = 0, hi = a.n_local;  // tile_prefix[lo] <= idx < tile_prefix[hi]
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (tile_prefix[mid] <= idx) lo = mid; else hi = mid;
  }
  Tile t;
  t.g = lo;
  int local = idx - tile_prefix[lo];
  int t_idx = local / a.n_tiles;
  t.n_idx = local - t_idx * a.n_tiles;
  int gs_start = row_start[a.group_offset + lo];
  int gs_rows = row_start[a.group_offset + lo + 1] - gs_start;
  t.row0 = gs_start + t_idx * BT;
  t.rows = min(BT, gs_rows - t_idx * BT);
  return t;
}

template <int SD>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gmm_fp4_kernel(const __grid_constant__ CUtensorMap tm_lhs,
                   const __grid_constant__ CUtensorMap tm_codes,
                   const __grid_constant__ CUtensorMap tm_scales, const Args a) {
  using L = Smem<SD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* cs_full = bars;
  uint64_t* cs_empty = cs_full + CS;
  uint64_t* tk_full = cs_empty + CS;
  uint64_t* tk_empty = tk_full + TS;
  uint64_t* a_full = tk_empty + TS;
  uint64_t* a_empty = a_full + AS;
  uint64_t* acc_full = a_empty + AS;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);
  int* row_start = reinterpret_cast<int*>(smem + L::OFF_ROWS);
  int* tile_prefix = reinterpret_cast<int*>(smem + L::OFF_TILES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < CS; ++i) {
      mbar_init(&cs_full[i], 1);
      mbar_init(&cs_empty[i], NUM_DEC_WARPS);
    }
    for (int i = 0; i < TS; ++i) {
      mbar_init(&tk_full[i], 1);
      mbar_init(&tk_empty[i], 1);
    }
    for (int i = 0; i < AS; ++i) {
      mbar_init(&a_full[i], NUM_DEC_WARPS);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == PRODUCER_WARP && lane == 0) {
    tma_prefetch_desc(&tm_lhs);
    tma_prefetch_desc(&tm_codes);
    tma_prefetch_desc(&tm_scales);
  }
  if (warp == 0) {
    // Row starts over all groups (rows are sorted by group), then tile
    // prefix over the local groups. Each lane scans a contiguous chunk.
    const int G = a.num_groups;
    const int per = (G + 31) / 32;
    int sum = 0;
    for (int i = 0; i < per; ++i) {
      int g = lane * per + i;
      if (g < G) {
        int v = a.group_sizes[g];
        if (v < 0) { report(a.status, DWM_DEV_BAD_INDEX); v = 0; }
        sum += v;
      }
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    int run = incl - sum;
    for (int i = 0; i < per; ++i) {
      int g = lane * per + i;
      if (g < G) {
        int v = max(a.group_sizes[g], 0);
        int s = min(run, a.m);
        row_start[g] = s;
        run += v;
      }
    }
    if (lane == 31) {
      row_start[G] = min(run, a.m);
      if (run > a.m) report(a.status, DWM_DEV_BAD_INDEX);
    }
    __syncwarp();
    const int NL = a.n_local;
    const int per2 = (NL + 31) / 32;
    int tsum = 0;
    for (int i = 0; i < per2; ++i) {
      int g = lane * per2 + i;
      if (g < NL) {
        int rows = row_start[a.group_offset + g + 1] - row_start[a.group_offset + g];
        tsum += ((rows + BT - 1) / BT) * a.n_tiles;
      }
    }
    int tincl = tsum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, tincl, o);
      if (lane >= o) tincl += y;
    }
    int trun = tincl - tsum;
    for (int i = 0; i < per2; ++i) {
      int g = lane * per2 + i;
      if (g < NL) {
        tile_prefix[g] = trun;
        int rows = row_start[a.group_offset + g + 1] - row_start[a.group_offset + g];
        trun += ((rows + BT - 1) / BT) * a.n_tiles;
      }
    }
    if (lane == 31) tile_prefix[NL] = trun;
  }
  if (warp == MMA_WARP) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int total = tile_prefix[a.n_local];
  const int KT = a.k / BK;

  if (warp < 4) {
    // ---------------- epilogue ----------------
    const int es = a.out_f32 ? 4 : 2;
    if (a.zero_init) {
      // Rows outside the local groups: [0, lo) and [hi, m).
      const int lo = row_start[a.group_offset];
      const int hi = row_start[a.group_offset + a.n_local];
      const int64_t row_bytes = (int64_t)a.ldo * es;
      const int64_t n16 = row_bytes / 16;
      uint4 z = make_uint4(0, 0, 0, 0);
      const int64_t tid = (int64_t)blockIdx.x * 128 + threadIdx.x;
      const int64_t stride = (int64_t)gridDim.x * 128;
      uint4* o = reinterpret_cast<uint4*>(a.out);
      for (int64_t i = tid; i < (int64_t)lo * n16; i += stride) o[i] = z;
      for (int64_t i = (int64_t)hi * n16 + tid; i < (int64_t)a.m * n16; i += stride) o[i] = z;
    }
    const int mrow = warp * 32 + lane;  // TMEM lane = A row = weight column slot
    const int col = (mrow & ~7) + perm8(mrow & 7);
    int it = 0;
    for (int idx = blockIdx.x; idx < total; idx += gridDim.x, ++it) {
      const Tile t = get_tile(idx, row_start, tile_prefix, a);
      const int buf = it & 1;
      const uint32_t ph = (it >> 1) & 1;
      const bool got = mbar_wait(&acc_full[buf], ph, abort_flag, a.status);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(buf * NSUB * BT);
      const int nchunks = (t.rows + 15) >> 4;
      for (int c = 0; c < nchunks; ++c) {
        uint32_t r0[16], r1[16];
        tmem_ld16(tbase + c * 16, r0);
        tmem_ld16(tbase + BT + c * 16, r1);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int r = c * 16 + e;
          if (r < t.rows) {
            const int64_t row = t.row0 + r;
            const float v0 = __uint_as_float(r0[e]);
            const float v1 = __uint_as_float(r1[e]);
            if (a.act == DWM_ACT_NONE) {
              const int64_t base = row * a.ldo + (int64_t)t.n_idx * (NSUB * BW) + col;
              if (a.out_f32) {
                float* o = reinterpret_cast<float*>(a.out);
                o[base] = v0;
                o[base + BW] = v1;
              } else {
                uint16_t* o = reinterpret_cast<uint16_t*>(a.out);
                o[base] = (uint16_t)f32_to_bf16_bits(v0);
                o[base + BW] = (uint16_t)f32_to_bf16_bits(v1);
              }
            } else {
              float g = v0, u = v1;
              if (a.act == DWM_ACT_SWIGLU_CLAMP) {
                g = fminf(g, a.limit);
                u = fminf(fmaxf(u, -a.limit), a.limit);
              }
              const float sg = 1.0f / (1.0f + expf(-g));
              const float h = g * sg * u;
              const int64_t base = row * a.ldo + (int64_t)t.n_idx * BW + col;
              if (a.out_f32) {
                reinterpret_cast<float*>(a.out)[base] = h;
              } else {
                reinterpret_cast<uint16_t*>(a.out)[base] = (uint16_t)f32_to_bf16_bits(h);
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  } else if (warp == PRODUCER_WARP) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint64_t pol_stream = policy_evict_first();
      const uint64_t pol_keep = policy_evict_last();
      constexpr uint32_t cs_bytes = NSUB * C_SUB_BYTES + L::S_STAGE;
      int cs = 0, ts = 0;
      uint32_t cs_ph = 0, ts_ph = 0;
      uint32_t cs_armed = 0, cs_par = 0, ts_armed = 0, ts_par = 0;
      const int half = a.n / 2;
      for (int idx = blockIdx.x; idx < total; idx += gridDim.x) {
        const Tile t = get_tile(idx, row_start, tile_prefix, a);
        int col[NSUB];
        if (a.act == DWM_ACT_NONE) {
          col[0] = t.n_idx * (NSUB * BW);
          col[1] = col[0] + BW;
        } else {
          col[0] = t.n_idx * BW;
          col[1] = half + t.n_idx * BW;
        }
        const int nb = (t.rows + T_BOX_ROWS - 1) / T_BOX_ROWS;
        bool ok = true;
        for (int kk = 0; kk < KT && ok; ++kk) {
          if (!mbar_wait(&cs_empty[cs], cs_ph ^ 1, abort_flag, a.status)) { ok = false; break; }
          mbar_arrive_expect_tx(&cs_full[cs], cs_bytes);
          cs_armed |= 1u << cs;
          cs_par = (cs_par & ~(1u << cs)) | (cs_ph << cs);
          uint8_t* cdst = smem + L::OFF_C + cs * C_STAGE;
          uint8_t* sdst = smem + L::OFF_S + cs * L::S_STAGE;
#pragma unroll
          for (int s = 0; s < NSUB; ++s) {
            tma_load_2d(cdst + s * C_SUB1_OFF, &tm_codes, &cs_full[cs], col[s] / 2,
                        t.g * a.k + kk * BK, pol_stream);
            tma_load_2d(sdst + s * (L::S_STAGE / NSUB), &tm_scales, &cs_full[cs], col[s],
                        t.g * (a.k / 32) + kk * 2, pol_stream);
          }
          if (++cs == CS) { cs = 0; cs_ph ^= 1; }

          if (!mbar_wait(&tk_empty[ts], ts_ph ^ 1, abort_flag, a.status)) { ok = false; break; }
          mbar_arrive_expect_tx(&tk_full[ts], nb * T_BOX_BYTES);
          ts_armed |= 1u << ts;
          ts_par = (ts_par & ~(1u << ts)) | (ts_ph << ts);
          uint8_t* tdst = smem + L::OFF_T + ts * T_STAGE;
          for (int b = 0; b < nb; ++b)
            tma_load_2d(tdst + b * T_BOX_BYTES, &tm_lhs, &tk_full[ts], kk * BK,
                        t.row0 + b * T_BOX_ROWS, pol_keep);
          if (++ts == TS) { ts = 0; ts_ph ^= 1; }
        }
        if (!ok) break;
      }
      // Let every issued copy land before the CTA can exit.
      for (int s = 0; s < CS; ++s)
        if (cs_armed & (1u << s)) mbar_wait(&cs_full[s], (cs_par >> s) & 1, nullptr, a.status);
      for (int s = 0; s < TS; ++s)
        if (ts_armed & (1u << s)) mbar_wait(&tk_full[s], (ts_par >> s) & 1, nullptr, a.status);
    }
  } else if (warp == MMA_WARP) {
    // ---------------- UMMA issuer ----------------
    if (lane == 0) {
      int as = 0, ts = 0;
      uint32_t as_ph = 0, ts_ph = 0;
      int it = 0;
      bool ok = true;
      for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x, ++it) {
        const Tile t = get_tile(idx, row_start, tile_prefix, a);
        const int nmma = (t.rows + 15) & ~15;
        const uint32_t idesc = idesc_bf16(128, nmma, /*a_mn=*/true, /*b_mn=*/false);
        const int buf = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        if (!mbar_wait(&acc_empty[buf], ph ^ 1, abort_flag, a.status)) break;
        tc_fence_after();
        const uint32_t d0 = tmem + (uint32_t)(buf * NSUB * BT);
        for (int kk = 0; kk < KT; ++kk) {
          if (!mbar_wait(&a_full[as], as_ph, abort_flag, a.status) ||
              !mbar_wait(&tk_full[ts], ts_ph, abort_flag, a.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + L::OFF_A + as * A_STAGE);
          const uint32_t t_base = smem_u32(smem + L::OFF_T + ts * T_STAGE);
#pragma unroll
          for (int j = 0; j < BK / 16; ++j) {
            const uint64_t bdesc = smem_desc_sw128(t_base + j * 32, 16, 1024);
#pragma unroll
            for (int s = 0; s < NSUB; ++s) {
              const uint64_t adesc =
                  smem_desc_sw128(a_base + s * A_SUB_BYTES + j * 2048, A_LBO, A_SBO);
              umma_bf16(d0 + s * BT, adesc, bdesc, idesc, (kk | j) != 0);
            }
          }
          umma_commit(&a_empty[as]);
          umma_commit(&tk_empty[ts]);
          if (++as == AS) { as = 0; as_ph ^= 1; }
          if (++ts == TS) { ts = 0; ts_ph ^= 1; }
        }
        if (!ok) break;
        umma_commit(&acc_full[buf]);
      }
      // Every issued MMA completes before TMEM is released.
      umma_commit(drain_bar);
      mbar_wait(drain_bar, 0, nullptr, a.status);
    }
  } else if (warp >= DEC_WARP0) {
    // ---------------- decode ----------------
    // Warps 0-3 of the decode group take sub-tile 0, warps 4-7 sub-tile 1.
    // A warp decodes two adjacent 64-byte code rows per step (lanes 0-15 row
    // r, lanes 16-31 row r+1: 128 contiguous bytes, conflict-free), rows
    // r = 2*(dw%4) + 8j (+1), j = 0..7, covering all 64 rows of the stage.
    const int dw = warp - DEC_WARP0;
    const int sub = dw >> 2;
    const int half = lane >> 4;
    const int g = lane & 15;          // 8-column group inside the sub-tile
    int cs = 0, as = 0;
    uint32_t cs_ph = 0, as_ph = 0;
    bool ok = true;
    for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x) {
      for (int kk = 0; kk < KT; ++kk) {
        bool got = mbar_wait(&cs_full[cs], cs_ph, abort_flag, a.status);
        got = got && mbar_wait(&a_empty[as], as_ph ^ 1, abort_flag, a.status);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        const uint8_t* csrc = smem + L::OFF_C + cs * C_STAGE + sub * C_SUB1_OFF;
        const uint8_t* ssrc = smem + L::OFF_S + cs * L::S_STAGE +
                              sub * (L::S_STAGE / NSUB) + g * 8 * ScaleTraits<SD>::bytes;
        uint8_t* adst = smem + L::OFF_A + as * A_STAGE + sub * A_SUB_BYTES + (g >> 3) * A_LBO;
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          uint32_t m1[4], m2[4];
          bool two = scale_mults<SD>(ssrc + kb * BW * ScaleTraits<SD>::bytes, m1, m2);
          two = __any_sync(0xffffffffu, two);
          if (two) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if (SD == DWM_U8) m1[i] = kBf16Pow2_126x2;
          }
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const int r = kb * 32 + jj * 8 + 2 * (dw & 3) + half;
            const uint32_t w = *reinterpret_cast<const uint32_t*>(csrc + r * (BW / 2) + g * 4);
            const uint4 v = decode8(w, m1, m2, two);
            const int chunk = (g & 7) ^ (r & 7);
            *reinterpret_cast<uint4*>(adst + (r >> 3) * A_SBO + (r & 7) * 128 + chunk * 16) = v;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&cs_empty[cs]);
          mbar_arrive(&a_full[as]);
        }
        if (++cs == CS) { cs = 0; cs_ph ^= 1; }
        if (++as == AS) { as = 0; as_ph ^= 1; }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// Elementwise dequantisation with the same decode (natural column order).
template <int SD>
__global__ void fp4_dequant_kernel(const uint8_t* __restrict__ codes,
                                   const uint8_t* __restrict__ scales, int groups, int k, int n,
                                   uint4* __restrict__ out) {
  const int64_t words_per_row = n / 8;
  const int64_t total = (int64_t)groups * k * words_per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / words_per_row;  // g * k + kk
    const int c8 = (int)(i - row * words_per_row);
    const int64_t g = row / k;
    const int kk = (int)(row - g * k);
    const uint32_t w = reinterpret_cast<const uint32_t*>(codes)[i];
    const uint8_t* sp =
        scales + ((g * (k / 32) + kk / 32) * (int64_t)n + (int64_t)c8 * 8) * ScaleTraits<SD>::bytes;
    uint32_t m1[4], m2[4];
    bool two = scale_mults<SD>(sp, m1, m2);
    if (SD == DWM_U8 && two) {
#pragma unroll
      for (int q = 0; q < 4; ++q) m1[q] = kBf16Pow2_126x2;
    }
    const uint4 v = decode8(w, m1, m2, two);
    uint4 o;
    o.x = __byte_perm(v.x, v.y, 0x5410);  // columns 0,1
    o.y = __byte_perm(v.z, v.w, 0x5410);  // columns 2,3
    o.z = __byte_perm(v.x, v.y, 0x7632);  // columns 4,5
    o.w = __byte_perm(v.z, v.w, 0x7632);  // columns 6,7
    out[i] = o;
  }
}

// tokamax codes <-> OCP e2m1 nibbles, one byte (two nibbles) per step.
__device__ __forceinline__ uint32_t nib_convert(uint32_t c, int to_tokamax) {
  if (to_tokamax) {
    const uint32_t mag = c & 7u;
    return (c & 8u) ? ((16u - mag) & 0xFu) : mag;  // -0 -> +0
  }
  return (c >= 8u) ? (8u | ((16u - c) & 7u)) : c;
}

__global__ void fp4_codes_convert_kernel(const uint8_t* __restrict__ in, uint8_t* out,
                                         size_t nbytes, int to_tokamax) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nbytes;
       i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t b = in[i];
    out[i] = (uint8_t)(nib_convert(b & 0xFu, to_tokamax) | (nib_convert(b >> 4, to_tokamax) << 4));
  }
}

template <int SD>
int launch(const void* lhs, const void* codes, const void* scales, const int32_t* group_sizes,
           int num_groups, int m, int k, int n, int group_offset, int n_local, int act,
           float limit, int out_dtype, int zero_init, void* out, cudaStream_t stream) {
  using L = Smem<SD>;
  CUtensorMap tm_lhs, tm_codes, tm_scales;
  int rc = encode_tmap_2d(&tm_lhs, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, lhs, (uint64_t)k,
                          (uint64_t)m, (uint64_t)k * 2, BK, T_BOX_ROWS,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_tmap_2d(&tm_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, codes, (uint64_t)n / 2,
                      (uint64_t)n_local * k, (uint64_t)n / 2, BW / 2, BK,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  rc = encode_tmap_2d(&tm_scales, ScaleTraits<SD>::tma, scales, (uint64_t)n,
                      (uint64_t)n_local * (k / 32), (uint64_t)n * ScaleTraits<SD>::bytes, BW, 2,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;

  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    rc = check_cuda(cudaFuncSetAttribute(gmm_fp4_kernel<SD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC),
                    "gmm smem attribute");
    if (rc) return rc;
    attr_set[dev] = true;
  }
  Args a;
  a.group_sizes = group_sizes;
  a.num_groups = num_groups;
  a.group_offset = group_offset;
  a.n_local = n_local;
  a.m = m;
  a.k = k;
  a.n = n;
  a.act = act;
  a.limit = limit;
  a.out_f32 = out_dtype == DWM_F32;
  a.zero_init = zero_init;
  a.out = out;
  a.ldo = act == DWM_ACT_NONE ? n : n / 2;
  a.n_tiles = n / (NSUB * BW);
  a.status = status_ptr();
  gmm_fp4_kernel<SD><<<num_sms(), NUM_THREADS, L::ALLOC, stream>>>(tm_lhs, tm_codes, tm_scales,
                                                                   a);
  return check_cuda(cudaGetLastError(), "gmm_fp4 launch");
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace gmm
}  // namespace dwm

using namespace dwm;

extern "C" int dwm_gmm_fp4(const void* lhs, const void* codes, int codes_format,
                           const void* scales, int scale_dtype, const int32_t* group_sizes,
                           int num_groups, int m, int k, int n, int group_offset,
                           int num_local_groups, int act, float act_limit, int out_dtype,
                           int zero_init, void* out, void* stream) {
  DWM_CHECK_ARG(codes_format == DWM_FP4_E2M1,
                "gmm_fp4 takes e2m1 nibbles; convert tokamax codes once with "
                "dwm_fp4_codes_convert");
  DWM_CHECK_ARG(scale_dtype == DWM_U8 || scale_dtype == DWM_BF16 || scale_dtype == DWM_F32,
                "scale dtype must be u8 (e8m0), bf16 or f32");
  DWM_CHECK_ARG(out_dtype == DWM_BF16 || out_dtype == DWM_F32, "out dtype must be bf16 or f32");
  DWM_CHECK_ARG(act == DWM_ACT_NONE || act == DWM_ACT_SWIGLU || act == DWM_ACT_SWIGLU_CLAMP,
                "unknown activation %d", act);
  DWM_CHECK_ARG(m >= 0 && k > 0 && n > 0, "bad shape m=%d k=%d n=%d", m, k, n);
  DWM_CHECK_ARG(k % gmm::BK == 0, "k=%d must be a multiple of %d", k, gmm::BK);
  DWM_CHECK_ARG(n % (gmm::NSUB * gmm::BW) == 0, "n=%d must be a multiple of 256", n);
  DWM_CHECK_ARG(num_groups >= 1 && num_groups <= gmm::MAX_GROUPS,
                "num_groups=%d out of [1, %d]", num_groups, gmm::MAX_GROUPS);
  DWM_CHECK_ARG(group_offset >= 0 && num_local_groups >= 0 &&
                    group_offset + num_local_groups <= num_groups,
                "group_offset=%d + num_local_groups=%d exceeds num_groups=%d", group_offset,
                num_local_groups, num_groups);
  DWM_CHECK_ARG(group_sizes && out && (m == 0 || lhs), "NULL pointer");
  DWM_CHECK_ARG(num_local_groups == 0 || (codes && scales), "NULL weights");
  DWM_CHECK_ARG(gmm::aligned16(lhs) && gmm::aligned16(codes) && gmm::aligned16(scales) &&
                    gmm::aligned16(out),
                "pointers must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int n_out = act == DWM_ACT_NONE ? n : n / 2;
  const size_t es = out_dtype == DWM_F32 ? 4 : 2;
  if (m == 0) return DWM_OK;
  if (num_local_groups == 0) {
    if (zero_init)
      return check_cuda(cudaMemsetAsync(out, 0, (size_t)m * n_out * es, s), "gmm zero");
    return DWM_OK;
  }
  switch (scale_dtype) {
    case DWM_U8:
      return gmm::launch<DWM_U8>(lhs, codes, scales, group_sizes, num_groups, m, k, n,
                                 group_offset, num_local_groups, act, act_limit, out_dtype,
                                 zero_init, out, s);
    case DWM_BF16:
      return gmm::launch<DWM_BF16>(lhs, codes, scales, group_sizes, num_groups, m, k, n,
                                   group_offset, num_local_groups, act, act_limit, out_dtype,
                                   zero_init, out, s);
    default:
      return gmm::launch<DWM_F32>(lhs, codes, scales, group_sizes, num_groups, m, k, n,
                                  group_offset, num_local_groups, act, act_limit, out_dtype,
                                  zero_init, out, s);
  }
}

extern "C" int dwm_fp4_dequant(const void* codes, const void* scales, int scale_dtype,
                               int groups, int k, int n, void* out, void* stream) {
  DWM_CHECK_ARG(codes && scales && out, "NULL pointer");
  DWM_CHECK_ARG(groups >= 0 && k > 0 && n > 0 && k % 32 == 0 && n % 8 == 0,
                "bad shape groups=%d k=%d n=%d (k %% 32, n %% 8)", groups, k, n);
  DWM_CHECK_ARG(gmm::aligned16(out) && (reinterpret_cast<uintptr_t>(codes) & 3) == 0,
                "misaligned pointer");
  DWM_CHECK_ARG(scale_dtype == DWM_U8 || scale_dtype == DWM_BF16 || scale_dtype == DWM_F32,
                "scale dtype must be u8, bf16 or f32");
  const int64_t total = (int64_t)groups * k * (n / 8);
  if (total == 0) return DWM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((total + threads - 1) / threads, 148LL * 16);
  auto c = static_cast<const uint8_t*>(codes);
  auto sc = static_cast<const uint8_t*>(scales);
  auto o = static_cast<uint4*>(out);
  if (scale_dtype == DWM_U8)
    gmm::fp4_dequant_kernel<DWM_U8><<<(int)blocks, threads, 0, s>>>(c, sc, groups, k, n, o);
  else if (scale_dtype == DWM_BF16)
    gmm::fp4_dequant_kernel<DWM_BF16><<<(int)blocks, threads, 0, s>>>(c, sc, groups, k, n, o);
  else
    gmm::fp4_dequant_kernel<DWM_F32><<<(int)blocks, threads, 0, s>>>(c, sc, groups, k, n, o);
  return check_cuda(cudaGetLastError(), "fp4_dequant launch");
}

extern "C" int dwm_fp4_codes_convert(const void* in, void* out, size_t nbytes, int from_format,
                                     int to_format, void* stream) {
  DWM_CHECK_ARG(in && out, "NULL pointer");
  DWM_CHECK_ARG((from_format == DWM_FP4_E2M1 || from_format == DWM_FP4_TOKAMAX) &&
                    (to_format == DWM_FP4_E2M1 || to_format == DWM_FP4_TOKAMAX),
                "unknown fp4 code format");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (nbytes == 0) return DWM_OK;
  if (from_format == to_format) {
    if (in == out) return DWM_OK;
    return check_cuda(cudaMemcpyAsync(out, in, nbytes, cudaMemcpyDeviceToDevice, s),
                      "codes copy");
  }
  const int threads = 256;
  const size_t blocks = std::min<size_t>((nbytes + threads - 1) / threads, 148 * 32);
  gmm::fp4_codes_convert_kernel<<<(unsigned)blocks, threads, 0, s>>>(
      static_cast<const uint8_t*>(in), static_cast<uint8_t*>(out), nbytes,
      to_format == DWM_FP4_TOKAMAX);
  return check_cuda(cudaGetLastError(), "codes_convert launch");
}
