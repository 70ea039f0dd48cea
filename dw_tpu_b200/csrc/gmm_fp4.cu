// FP4 grouped matmul for sm_100a: tokamax gmm_v2 with rhs_fp4_codes
// (TK:107-153), decoded on the SM and multiplied on tcgen05 tensor cores with
// f32 accumulators in TMEM. Decode-sized groups go to the mma.sync kernel in
// gmv_fp4.cu instead (see the dispatcher at the end of this file).
//
// The product is computed transposed ("swap AB"): the decoded weight tile
// W[k, n0:n0+128] is UMMA operand A (M = 128 weight columns) and the token
// rows X[r0:r0+rows, k] are operand B (N = rows rounded up to 16, K-major,
// 128-byte swizzled, loaded by TMA). Each tile carries two 128-column
// sub-tiles (two accumulators): adjacent columns for a plain GEMM, or the
// matching gate and up columns for the fused SwiGLU. Two variants share the
// producers, the tile scheduler and the epilogue:
//   kMN  raw e2m1 weights [g, k, n/2] decoded into a 128-byte swizzled,
//        MN-major A tile in shared memory.
//   kKS  B200-layout weights (fp4_decode.cuh) decoded into a K-major,
//        128-byte swizzled A tile in shared memory.
//
// One persistent CTA per SM, 24 warps:
//   warps 0-3   epilogue: TMEM -> registers -> (SwiGLU) -> global
//   warp  4     TMA producer: FP4 codes + scales ring (the HBM stream)
//   warp  5     TMEM allocator and single-thread UMMA issuer
//   warp  6     TMA producer: token-row ring (L2-resident rows)
//   warps 8-23  decode, two groups of 8 on alternate stages
//
// Numerics follow the reference order (E0901:84-95): each e2m1 value is
// decoded exactly to bf16, multiplied by the bf16 scale in one bf16 multiply
// (round to nearest even), then the MMA accumulates bf16 x bf16 products in
// f32; the epilogue applies SwiGLU in f32 and rounds once to the output type.
#include <algorithm>
#include <type_traits>

#include "fp4_decode.cuh"

namespace dwm {

int launch_gmv(const void* lhs, const void* codes, const void* scales, int scale_dtype,
               const int32_t* group_sizes, int num_groups, int m, int k, int n, int group_offset,
               int n_local, int act, float limit, int out_dtype, int zero_init, void* out, int nt,
               cudaStream_t stream, int tail_min = 0, int grp_lo = 0, int grp_hi = 1 << 30,
               const EpHooks* hooks = nullptr);
int launch_gmm_pair(const void* lhs, const void* codes, const void* scales, int scale_dtype,
                    const int32_t* group_sizes, int num_groups, int m, int k, int n,
                    int group_offset, int n_local, int act, float limit, int out_dtype,
                    int zero_init, void* out, const EpHooks* hooks, cudaStream_t stream,
                    int tail_min, int wide, int grp_lo = 0);

namespace gmm {

using namespace fp4;

// Variant 8: a group's last tile goes to the CTA-pair kernel only with at
// least this many rows (a whole tile's decode costs about as much as the
// decode kernel's six 16-row weight streams).
constexpr int kPairTailMin = 96;
// Variant 10's size classes: groups of up to kSplitRows16 rows on the decode
// kernel's 16-row tiles, up to kSplitRows32 on its 32-row tiles, up to
// kSplitRows96 on the single-CTA tcgen05 kernel, larger ones on CTA pairs.
constexpr int kSplitRows16 = 16;
constexpr int kSplitRows32 = 32;
constexpr int kSplitRows96 = 95;  // 33-95 rows: the single-CTA tcgen05 kernel

enum Variant { kMN = 0, kKS = 1 };

constexpr int NSUB = 2;    // sub-tiles (accumulators) per tile
constexpr int BW = 128;    // weight columns per sub-tile (UMMA M)
constexpr int BK = 64;     // K per pipeline stage (128 bytes of bf16)
constexpr int BT = 128;    // token rows per tile at most (the UMMA N)
constexpr int NUM_THREADS = 768;
constexpr int PRODUCER_WARP = 4;
constexpr int MMA_WARP = 5;
constexpr int TOKEN_WARP = 6;
constexpr int DEC_WARP0 = 8;
constexpr int NUM_DEC_WARPS = 8;  // per group; two groups
constexpr int MAX_GROUPS = 1024;
constexpr int TMEM_COLS = 512;    // two buffers x NSUB x BT f32 columns

constexpr int A_SUB_BYTES = BW * BK * 2;     // 16 KiB bf16 sub-tile
constexpr int A_STAGE = NSUB * A_SUB_BYTES;  // 32 KiB
constexpr int A_LBO_MN = 8192;               // MN-major: MN-atom (64 columns) stride
constexpr int A_SBO_MN = 1024;               // MN-major: K-atom (8 rows) stride
constexpr int T_BOX_ROWS = 16;
constexpr int T_BOX_BYTES = T_BOX_ROWS * BK * 2;  // 2 KiB
constexpr int C_SUB_BYTES = BK * (BW / 2);        // 4 KiB of packed nibbles per sub-tile
constexpr int C_STAGE = NSUB * C_SUB_BYTES;       // TMA writes 128-byte aligned addresses
static_assert(C_SUB_BYTES % 128 == 0, "TMA needs 128 B alignment");

// Sleep (ns) between mbarrier polls per role: the epilogue waits a whole
// tile, the producers and the decode warps wait for ring slots, the MMA
// issuer waits for decoded stages (latency-critical).
#ifndef DWM_GMM_EPI_SLEEP
#define DWM_GMM_EPI_SLEEP 256
#endif
#ifndef DWM_GMM_PROD_SLEEP
#define DWM_GMM_PROD_SLEEP 0
#endif
#ifndef DWM_GMM_DEC_SLEEP
#define DWM_GMM_DEC_SLEEP 0
#endif
#ifndef DWM_GMM_MMA_SLEEP
#define DWM_GMM_MMA_SLEEP 0
#endif

// Epilogue staging: each epilogue warp turns its 32 columns x 8 token rows
// into 16-byte row vectors through 1 KiB of shared memory (8 x 32 x 4 bytes).
constexpr int EPI_ROWS = 8;
constexpr int EPI_WARP_BYTES = EPI_ROWS * 32 * 4;

// Pipeline depths (build-time tunables). Measured on cfg3-sized groups (256
// rows per expert): the token ring is the one that matters. A token stage
// reaches shared memory from L2 only after the UMMAs of the stage it
// replaces have completed, so its latency has to be covered by the stages
// ahead of it: 4 stages of 128 rows (2 A stages, 8 code stages) measured
// 599 TFLOP/s against 562 with 3 (3 A stages).
#ifndef DWM_GMM_TS
#define DWM_GMM_TS 4
#endif
#ifndef DWM_GMM_AS
#define DWM_GMM_AS 2
#endif
#ifndef DWM_GMM_CS
#define DWM_GMM_CS 8
#endif
// Two TMEM accumulator buffers, so a tile's epilogue overlaps the next
// tile's main loop.
template <int SD>
struct Smem {
  static constexpr int TS = DWM_GMM_TS;
  static constexpr int AS = DWM_GMM_AS;
  // A token stage: BT/16 boxes of 16 rows x 64 k (one k-step of a full tile).
  static constexpr int T_STAGE = BT * BK * 2;
  static constexpr int T_BOXES = T_STAGE / T_BOX_BYTES;
  static constexpr int NBUF = TMEM_COLS / (NSUB * BT);
  // Code ring: 8 stages (6 with f32 scales, 7 with bf16 scales, to fit the
  // epilogue's staging tiles in shared memory).
  static constexpr int CS_BASE = DWM_GMM_CS;
  static constexpr int CS = ScaleTraits<SD>::bytes == 4   ? (CS_BASE * 3 + 3) / 4
                            : ScaleTraits<SD>::bytes == 2 ? CS_BASE - (CS_BASE > 4)
                                                          : CS_BASE;
  static constexpr int S_STAGE = NSUB * 2 * BW * ScaleTraits<SD>::bytes;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_T = OFF_A + AS * A_STAGE;
  static constexpr int OFF_C = OFF_T + TS * T_STAGE;
  static constexpr int OFF_S = OFF_C + CS * C_STAGE;
  static constexpr int OFF_BAR = OFF_S + CS * S_STAGE;
  static constexpr int NUM_BARS = 2 * CS + 2 * TS + 2 * AS + 4 + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int OFF_ROWS = OFF_MISC + 32;
  static constexpr int OFF_TILES = OFF_ROWS + (MAX_GROUPS + 1) * 4;
  static constexpr int OFF_EPI = (OFF_TILES + (MAX_GROUPS + 1) * 4 + 15) & ~15;
  static constexpr int EPI_WARPS = 4;
  static constexpr int BYTES = OFF_EPI + EPI_WARPS * EPI_WARP_BYTES;
  static constexpr int ALLOC = BYTES + 1024;  // slack for 1 KiB alignment
  static_assert(ALLOC <= 232448, "exceeds the 227 KiB per-CTA shared memory");
  static_assert(CS <= 32 && TS <= 32, "ring masks are 32-bit");
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
  int ldo;      // output row length (n, or n/2 with SwiGLU)
  int n_tiles;  // column tiles per group
  int grp_lo, grp_hi;  // only groups of grp_lo < rows <= grp_hi (variant 10's size classes)
  int* status;
  EpHooks hk;   // expert-parallel gating / push (all null for a plain GEMM)
};

// Tiles of a group of `rows` rows in this launch.
__device__ __forceinline__ int group_tile_count(int rows, const Args& a) {
  return rows > a.grp_lo && rows <= a.grp_hi ? ((rows + BT - 1) / BT) * a.n_tiles : 0;
}

// SMEM slot p of an 8-column group holds column perm8(p) (kMN).
__device__ __forceinline__ int perm8(int p) { return (p >> 1) + ((p & 1) << 2); }

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

// Token-stage geometry: a tile needs nb 16-row boxes per k-step; rounded up
// to a power of two (nbp) a stage of `boxes` boxes covers boxes / nbp
// k-steps.
__device__ __forceinline__ int token_span(int nb, int& nbp, int boxes) {
  nbp = nb <= 1 ? 1 : nb <= 2 ? 2 : nb <= 4 ? 4 : nb <= 8 ? 8 : 16;
  return boxes / nbp;
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// A decode group's wait for its next stage: the group's first warp polls the
// two mbarriers (codes landed, A slot free) and publishes the outcome; the
// other seven warps wait on named barrier 1 + grp, which holds them in
// hardware instead of letting them spin and take issue slots from the warps
// with work (the epilogue, above all). The outcome is double-buffered by the
// group's step parity, so the first warp can publish the next step's value
// while a slow warp still reads this one.
// DWM_GMM_DEC_SYNC 0 instead lets every warp poll for itself.
#ifndef DWM_GMM_DEC_SYNC
#define DWM_GMM_DEC_SYNC 1
#endif
template <int SLEEP>
__device__ __forceinline__ bool group_wait(int grp, int dw, uint32_t step, uint64_t* full,
                                           uint32_t full_ph, uint64_t* empty, uint32_t empty_ph,
                                           volatile int* abort_flag, volatile int* go,
                                           int* status) {
  if (DWM_GMM_DEC_SYNC == 0) {
    bool got = mbar_wait<SLEEP>(full, full_ph, abort_flag, status);
    got = got && mbar_wait<SLEEP>(empty, empty_ph, abort_flag, status);
    return __all_sync(0xffffffffu, got);
  }
  volatile int* slot = go + grp * 2 + ((step >> 1) & 1);
  if (dw == 0) {
    bool got = mbar_wait<SLEEP>(full, full_ph, abort_flag, status);
    got = got && mbar_wait<SLEEP>(empty, empty_ph, abort_flag, status);
    got = __all_sync(0xffffffffu, got);
    if ((threadIdx.x & 31) == 0) *slot = got ? 1 : 0;
  }
  named_bar_sync(1 + grp, NUM_DEC_WARPS * 32);
  return *slot != 0;
}

template <int SD, int VAR>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gmm_fp4_kernel(const __grid_constant__ CUtensorMap tm_lhs,
                   const __grid_constant__ CUtensorMap tm_lhs_32,
                   const __grid_constant__ CUtensorMap tm_lhs_64,
                   const __grid_constant__ CUtensorMap tm_lhs_128,
                   const __grid_constant__ CUtensorMap tm_codes,
                   const __grid_constant__ CUtensorMap tm_scales, const Args a) {
  using L = Smem<SD>;
  constexpr int CS = L::CS;
  constexpr int TS = L::TS;
  constexpr int AS = L::AS;
  constexpr int T_STAGE = L::T_STAGE;
  constexpr int NBUF = L::NBUF;
  extern __shared__ uint8_t smem_raw[];
  // 1 KiB alignment by pointer arithmetic on the shared array itself, so the
  // compiler keeps every access below in the shared window (LDS/STS, not LD/ST).
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
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
  volatile int* group_go = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 16);  // [2][2]
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
      mbar_init(&acc_empty[i], L::EPI_WARPS);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == PRODUCER_WARP && lane == 0) {
    tma_prefetch_desc(&tm_lhs);
    tma_prefetch_desc(&tm_lhs_32);
    tma_prefetch_desc(&tm_lhs_64);
    tma_prefetch_desc(&tm_lhs_128);
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
        row_start[g] = min(run, a.m);
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
        tsum += group_tile_count(rows, a);
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
        trun += group_tile_count(rows, a);
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
    const int eq = warp;  // TMEM lane quarter
    if (a.zero_init) {
      // Rows outside the local groups: [0, lo) and [hi, m).
      const int lo = row_start[a.group_offset];
      const int hi = row_start[a.group_offset + a.n_local];
      const int64_t n16 = (int64_t)a.ldo * es / 16;
      const uint4 z = make_uint4(0, 0, 0, 0);
      const int64_t tid = (int64_t)blockIdx.x * 128 + threadIdx.x;
      const int64_t stride = (int64_t)gridDim.x * 128;
      uint4* o = reinterpret_cast<uint4*>(a.out);
      for (int64_t i = tid; i < (int64_t)lo * n16; i += stride) o[i] = z;
      for (int64_t i = (int64_t)hi * n16 + tid; i < (int64_t)a.m * n16; i += stride) o[i] = z;
    }
    const int mrow = eq * 32 + lane;  // TMEM lane = A row = weight column slot
    const uint32_t epi_s = smem_u32(smem + L::OFF_EPI + eq * EPI_WARP_BYTES);
    const int col = VAR == kMN ? (mrow & ~7) + perm8(mrow & 7) : mrow;
    constexpr float acc_scale = (float)(1 << decode_delta<SD>());  // undoes the decode bias
    int it = 0;
    for (int idx = blockIdx.x; idx < total; idx += gridDim.x, ++it) {
      const Tile t = get_tile(idx, row_start, tile_prefix, a);
      const int buf = it % NBUF;
      const uint32_t ph = (it / NBUF) & 1;
      const bool got = mbar_wait<DWM_GMM_EPI_SLEEP>(&acc_full[buf], ph, abort_flag, a.status);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(eq * 32) << 16) + (uint32_t)(buf * NSUB * BT);
      const int nchunks = (t.rows + 15) >> 4;
      // The warp's 32 output columns (per part): SwiGLU gives one part
      // (columns n_idx*BW + 32 warp ..), a plain GEMM two (sub-tile 0 and
      // sub-tile 1, BW apart).
      const bool act = a.act != DWM_ACT_NONE;
      const int nparts = act ? 1 : 2;
      const int64_t colw = act ? (int64_t)t.n_idx * BW + eq * 32
                               : (int64_t)t.n_idx * (NSUB * BW) + eq * 32;
      const int lcol = col - eq * 32;  // this lane's column inside the warp's 32
      const int row_bytes = 32 * es;     // one staged row: 64 or 128 bytes
      const int vec_per_row = row_bytes / 16;
      for (int c = 0; c < nchunks; ++c) {
        uint32_t r0[16], r1[16];
        tmem_ld16(tbase + c * 16, r0);
        tmem_ld16(tbase + BT + c * 16, r1);
        tmem_ld_wait();
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int rb = c * 16 + half * EPI_ROWS;  // first token row of this round
          if (rb >= t.rows) break;
          for (int part = 0; part < nparts; ++part) {
            // Stage: lane lcol writes its value of each of the round's rows.
#pragma unroll
            for (int e = 0; e < EPI_ROWS; ++e) {
              const int ee = half * EPI_ROWS + e;
              const float v0 = __uint_as_float(r0[ee]) * acc_scale;
              const float v1 = __uint_as_float(r1[ee]) * acc_scale;
              float v;
              if (act) {
                float g = v0, u = v1;
                if (a.act == DWM_ACT_SWIGLU_CLAMP) {
                  g = fminf(g, a.limit);
                  u = fminf(fmaxf(u, -a.limit), a.limit);
                }
                v = g * sigmoid_fast(g) * u;
              } else {
                v = part == 0 ? v0 : v1;
              }
              if (a.out_f32)
                sts_f32(epi_s + (uint32_t)(e * row_bytes + lcol * 4), v);
              else
                sts_u16(epi_s + (uint32_t)(e * row_bytes + lcol * 2),
                        (uint16_t)f32_to_bf16_bits(v));
            }
            __syncwarp();
            // Copy out: 16-byte vectors of consecutive columns, one row each.
            for (int q = lane; q < EPI_ROWS * vec_per_row; q += 32) {
              const int e = q / vec_per_row, j = q - e * vec_per_row;
              const int r = rb + e;
              if (r < t.rows) {
                const uint4 v = lds_u128(epi_s + (uint32_t)(e * row_bytes + j * 16));
                if (a.hk.push_tags != nullptr) {
                  // Expert parallel: straight into the token owner's buffer,
                  // at the row of its (token, k) pair (NVLink for a peer).
                  const int tag = a.hk.push_tags[t.row0 + r];
                  if (tag >= 0) {
                    const int64_t off = ((int64_t)(tag & ((1 << kEpTagBits) - 1)) * a.ldo +
                                         colw + part * BW) * es + j * 16;
                    *reinterpret_cast<uint4*>(a.hk.push_base[tag >> kEpTagBits] + off) = v;
                  }
                } else {
                  const int64_t off =
                      ((t.row0 + r) * (int64_t)a.ldo + colw + part * BW) * es + j * 16;
                  *reinterpret_cast<uint4*>(static_cast<uint8_t*>(a.out) + off) = v;
                }
              }
            }
            __syncwarp();
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  } else if (warp == PRODUCER_WARP) {
    // ---------------- TMA producer: codes + scales (HBM stream) ----------------
    if (lane == 0) {
      const uint64_t pol_stream = policy_evict_first();
      constexpr uint32_t cs_bytes = NSUB * C_SUB_BYTES + L::S_STAGE;
      int cs = 0;
      uint32_t cs_ph = 0, cs_armed = 0, cs_par = 0;
      const int half = a.n / 2;
      bool ok = true;
      for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x) {
        const Tile t = get_tile(idx, row_start, tile_prefix, a);
        int col[NSUB];
        if (a.act == DWM_ACT_NONE) {
          col[0] = t.n_idx * (NSUB * BW);
          col[1] = col[0] + BW;
        } else {
          col[0] = t.n_idx * BW;
          col[1] = half + t.n_idx * BW;
        }
        for (int kk = 0; kk < KT; ++kk) {
          if (!mbar_wait<DWM_GMM_PROD_SLEEP>(&cs_empty[cs], cs_ph ^ 1, abort_flag, a.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&cs_full[cs], cs_bytes);
          cs_armed |= 1u << cs;
          cs_par = (cs_par & ~(1u << cs)) | (cs_ph << cs);
          uint8_t* cdst = smem + L::OFF_C + cs * C_STAGE;
          uint8_t* sdst = smem + L::OFF_S + cs * L::S_STAGE;
#pragma unroll
          for (int s = 0; s < NSUB; ++s) {
            if constexpr (VAR == kMN)  // [g*k + kk, n/2 bytes]: 64 rows x 64 bytes
              tma_load_2d(cdst + s * C_SUB_BYTES, &tm_codes, &cs_full[cs], col[s] / 2,
                          t.g * a.k + kk * BK, pol_stream);
            else  // [g*n/16 + block, (k/16)*32 words]: 8 column blocks x 4 k-blocks
              tma_load_2d(cdst + s * C_SUB_BYTES, &tm_codes, &cs_full[cs], kk * 4 * 32,
                          t.g * (a.n / 16) + col[s] / 16, pol_stream);
            tma_load_2d(sdst + s * (L::S_STAGE / NSUB), &tm_scales, &cs_full[cs], col[s],
                        t.g * (a.k / 32) + kk * 2, pol_stream);
          }
          if (++cs == CS) { cs = 0; cs_ph ^= 1; }
        }
      }
      // Let every issued copy land before the CTA can exit.
      for (int s = 0; s < CS; ++s)
        if (cs_armed & (1u << s)) mbar_wait(&cs_full[s], (cs_par >> s) & 1, nullptr, a.status);
    }
  } else if (warp == TOKEN_WARP) {
    // ---------------- TMA producer: token rows (L2-resident) ----------------
    // A token stage holds 8 boxes of 16 rows x 64 k: one k-step of a 128-row
    // tile, or up to 8 k-steps of a small tile (see token_span).
    if (lane == 0) {
      const uint64_t pol_keep = policy_evict_last();
      int ts = 0;
      uint32_t ts_ph = 0, ts_armed = 0, ts_par = 0;
      bool ok = true;
      int gated = -1;  // last local expert whose rows were seen to have arrived
      for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x) {
        const Tile t = get_tile(idx, row_start, tile_prefix, a);
        if (a.hk.gate_arrive != nullptr && t.g != gated) {
          // Expert-parallel gating: every source rank's rows of this expert
          // have been stored here (and made visible) before TMA reads them.
          if (!wait_counter_ge(a.hk.gate_arrive + t.g, a.hk.gate_target[t.g], a.hk.wait_ns,
                               a.status)) {
            *abort_flag = 1;
            break;
          }
          fence_proxy_async_all();
          gated = t.g;
        }
        const int nb = (t.rows + T_BOX_ROWS - 1) / T_BOX_ROWS;
        int nbp;
        const int kspan = token_span(nb, nbp, L::T_BOXES);
        for (int k0 = 0; k0 < KT; k0 += kspan) {
          const int kn = min(kspan, KT - k0);
          if (!mbar_wait<DWM_GMM_PROD_SLEEP>(&tk_empty[ts], ts_ph ^ 1, abort_flag, a.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&tk_full[ts], kn * nb * T_BOX_BYTES);
          ts_armed |= 1u << ts;
          ts_par = (ts_par & ~(1u << ts)) | (ts_ph << ts);
          uint8_t* tdst = smem + L::OFF_T + ts * T_STAGE;
          // A k-step's nb boxes of 16 rows in at most three copies (one of
          // 128 rows, else 64 + 32 + 16): each copy costs the issuing thread
          // about as much as a full box. The boxes land where nb single boxes
          // would.
          for (int kl = 0; kl < kn; ++kl) {
            uint8_t* kdst = tdst + kl * nbp * T_BOX_BYTES;
            const int kx = (k0 + kl) * BK;
            if (nb == 8) {
              tma_load_2d(kdst, &tm_lhs_128, &tk_full[ts], kx, t.row0, pol_keep);
              continue;
            }
            int b = 0;
            if (nb & 4) {
              tma_load_2d(kdst, &tm_lhs_64, &tk_full[ts], kx, t.row0, pol_keep);
              b += 4;
            }
            if (nb & 2) {
              tma_load_2d(kdst + b * T_BOX_BYTES, &tm_lhs_32, &tk_full[ts], kx,
                          t.row0 + b * T_BOX_ROWS, pol_keep);
              b += 2;
            }
            if (nb & 1)
              tma_load_2d(kdst + b * T_BOX_BYTES, &tm_lhs, &tk_full[ts], kx,
                          t.row0 + b * T_BOX_ROWS, pol_keep);
          }
          if (++ts == TS) { ts = 0; ts_ph ^= 1; }
        }
      }
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
        const int nb = nmma / T_BOX_ROWS;
        int nbp;
        const int kspan = token_span(nb, nbp, L::T_BOXES);
        const uint32_t idesc = idesc_bf16(128, nmma, /*a_mn=*/VAR == kMN, /*b_mn=*/false);
        const int buf = it % NBUF;
        const uint32_t ph = (it / NBUF) & 1;
        if (!mbar_wait<DWM_GMM_MMA_SLEEP>(&acc_empty[buf], ph ^ 1, abort_flag, a.status)) break;
        tc_fence_after();
        const uint32_t d0 = tmem + (uint32_t)(buf * NSUB * BT);
        for (int kk = 0; kk < KT; ++kk) {
          const int kl = kk % kspan;
          if (kl == 0 && !mbar_wait<DWM_GMM_MMA_SLEEP>(&tk_full[ts], ts_ph, abort_flag, a.status)) {
            ok = false;
            break;
          }
          if (!mbar_wait<DWM_GMM_MMA_SLEEP>(&a_full[as], as_ph, abort_flag, a.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + L::OFF_A + as * A_STAGE);
          const uint32_t t_base =
              smem_u32(smem + L::OFF_T + ts * T_STAGE) + (uint32_t)(kl * nbp * T_BOX_BYTES);
#pragma unroll
          for (int j = 0; j < BK / 16; ++j) {
            const uint64_t bdesc = smem_desc_sw128(t_base + j * 32, 16, 1024);
            for (int s = 0; s < NSUB; ++s) {
              const uint64_t adesc =
                  VAR == kMN
                      ? smem_desc_sw128(a_base + s * A_SUB_BYTES + j * 2048, A_LBO_MN, A_SBO_MN)
                      : smem_desc_sw128(a_base + s * A_SUB_BYTES + j * 32, 16, 1024);
              umma_bf16(d0 + s * BT, adesc, bdesc, idesc, (kk | j) != 0);
            }
          }
          umma_commit(&a_empty[as]);
          if (++as == AS) { as = 0; as_ph ^= 1; }
          if (kl == kspan - 1 || kk == KT - 1) {
            umma_commit(&tk_empty[ts]);
            if (++ts == TS) { ts = 0; ts_ph ^= 1; }
          }
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
    // Two groups of 8 decode warps take alternate stages (group = stage
    // counter % 2), so two stages are decoded concurrently.
    const int grp = (warp - DEC_WARP0) / NUM_DEC_WARPS;
    const int dw = (warp - DEC_WARP0) % NUM_DEC_WARPS;
    constexpr int es = ScaleTraits<SD>::bytes;
    constexpr int DELTA = decode_delta<SD>();
    uint32_t step = 0;  // stage counter over all k-steps of all tiles
    bool ok = true;
    if constexpr (VAR == kMN) {
      // Warp dw owns sub-tile dw/4 and k-block (dw/2)%2 of every stage; lane
      // (half, g) decodes the 8-column group g of 8 rows kb*32 + q*8 +
      // (i ^ half), q = 2*(dw%2) + half, i = 0..7: one scale set per thread
      // per stage. Lanes 0-15 and 16-31 read 64-byte rows 512 +- 64 bytes
      // apart (disjoint banks); each quarter-warp stores one 128-byte
      // swizzled row.
      const int sub = dw >> 2;
      const int kb = (dw >> 1) & 1;
      const int half = lane >> 4;
      const int g = lane & 15;
      const int q = 2 * (dw & 1) + half;
      const int row0 = kb * 32 + q * 8;
      const int c_even = sub * C_SUB_BYTES + (row0 + half) * (BW / 2) + g * 4;
      const int c_odd = sub * C_SUB_BYTES + (row0 - half) * (BW / 2) + g * 4;
      const int a_rows = sub * A_SUB_BYTES + (g >> 3) * A_LBO_MN + (row0 >> 3) * A_SBO_MN;
      const int a_even = a_rows + half * 128;
      const int a_odd = a_rows - half * 128;
      const uint32_t gh = (uint32_t)((g & 7) ^ half) << 4;
      const int s_off = sub * (L::S_STAGE / NSUB) + (kb * BW + g * 8) * es;
      for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x) {
        for (int kk = 0; kk < KT; ++kk, ++step) {
          if ((int)(step & 1) != grp) continue;
          const int cs = (int)(step % CS);
          const uint32_t cs_ph = (step / CS) & 1;
          const int as = (int)(step % AS);
          const uint32_t as_ph = (step / AS) & 1;
          if (!group_wait<DWM_GMM_DEC_SLEEP>(grp, dw, step, &cs_full[cs], cs_ph, &a_empty[as],
                                             as_ph ^ 1, abort_flag, group_go, a.status)) {
            ok = false;
            break;
          }
          const uint8_t* cstage = smem + L::OFF_C + cs * C_STAGE;
          uint8_t* astage = smem + L::OFF_A + as * A_STAGE;
          uint32_t m1[4], m2[4];
          const bool two =
              raw_mults<SD, DELTA>(smem + L::OFF_S + cs * L::S_STAGE + s_off, m1, m2);
          auto run = [&](auto two_tag) {
            constexpr bool TWO = decltype(two_tag)::value;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const uint32_t w = *reinterpret_cast<const uint32_t*>(
                  cstage + ((i & 1) ? c_odd : c_even) + i * 64);
              const uint4 v = decode8<false, TWO>(w, m1, m2);
              *reinterpret_cast<uint4*>(astage + ((i & 1) ? a_odd : a_even) + i * 128 +
                                        (gh ^ (uint32_t)(i << 4))) = v;
            }
          };
          if (__any_sync(0xffffffffu, two)) {
            if (!two) {
#pragma unroll
              for (int i = 0; i < 4; ++i) m1[i] = pow2_126_minus_delta_x2<DELTA>();
            }
            run(std::true_type{});
          } else {
            run(std::false_type{});
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&cs_empty[cs]);
            mbar_arrive(&a_full[as]);
          }
        }
      }
    } else {
      // B200 layout: a stage holds, per sub-tile, 8 column blocks x 4 k-blocks
      // of 32 words. Warp dw owns sub-tile dw/4 and column blocks
      // 2*(dw%4), 2*(dw%4)+1; its lane l decodes word l of each of the 8
      // blocks (the A fragment of an m16n8k16 MMA: columns gid, gid+8, k
      // pairs t, t+4) and scatters the four bf16x2 pairs into the K-major,
      // 128-byte swizzled A tile with 32-bit stores (conflict-free: the
      // eight gid rows land on eight different 16-byte chunks).
      const int sub = dw >> 2;
      const int gid = lane >> 2, tig = lane & 3;
      const DecodeRegs dregs = DecodeRegs::make();  // decode constants held in registers
      for (int idx = blockIdx.x; idx < total && ok; idx += gridDim.x) {
        for (int kk = 0; kk < KT; ++kk, ++step) {
          if ((int)(step & 1) != grp) continue;
          const int cs = (int)(step % CS);
          const uint32_t cs_ph = (step / CS) & 1;
          const int as = (int)(step % AS);
          const uint32_t as_ph = (step / AS) & 1;
          if (!group_wait<DWM_GMM_DEC_SLEEP>(grp, dw, step, &cs_full[cs], cs_ph, &a_empty[as],
                                             as_ph ^ 1, abort_flag, group_go, a.status)) {
            ok = false;
            break;
          }
          const uint8_t* cstage = smem + L::OFF_C + cs * C_STAGE + sub * C_SUB_BYTES;
          const uint8_t* sstage = smem + L::OFF_S + cs * L::S_STAGE + sub * (L::S_STAGE / NSUB);
          uint8_t* asub = smem + L::OFF_A + as * A_STAGE + sub * A_SUB_BYTES;
#pragma unroll
          for (int bi = 0; bi < 2; ++bi) {
            const int cbl = 2 * (dw & 3) + bi;  // column block inside the sub-tile
            // The four lanes of a quad (same gid) need the same four scales:
            // k32 half h, column gid + 8c. Lane tig converts scale (h, c) =
            // (tig >> 1, tig & 1) and the quad exchanges the multipliers.
            uint32_t m1s, m2s;
            const bool two = col_mult<SD, DELTA>(
                sstage + ((tig >> 1) * BW + 16 * cbl + gid + 8 * (tig & 1)) * es, m1s, m2s);
            const bool two_any = __any_sync(0xffffffffu, two);
            uint32_t m1[2][2], m2[2][2];  // [k32 half][column gid / gid+8]
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int c = 0; c < 2; ++c) {
                const int src = (lane & ~3) + 2 * h + c;
                if (two_any) {  // both multiplies: 2^(126 - delta), then the scale
                  m1[h][c] = pow2_126_minus_delta_x2<DELTA>();
                  m2[h][c] = __shfl_sync(0xffffffffu, m2s, src);
                } else {
                  m1[h][c] = __shfl_sync(0xffffffffu, m1s, src);
                  m2[h][c] = 0u;
                }
              }
            const int r0 = 16 * cbl + gid;  // A rows r0 and r0 + 8
            uint8_t* row_a = asub + (r0 >> 3) * 1024 + (r0 & 7) * 128;
            uint8_t* row_b = asub + ((r0 + 8) >> 3) * 1024 + ((r0 + 8) & 7) * 128;
#pragma unroll
            for (int kb = 0; kb < 4; ++kb) {
              const uint32_t w = *reinterpret_cast<const uint32_t*>(cstage + cbl * 512 +
                                                                    kb * 128 + lane * 4);
              uint32_t tv[4];
              tvals_b200(w, dregs, tv);
              const int h = kb >> 1;
              uint32_t v0 = hmul2_bf16(tv[0], m1[h][0]);
              uint32_t v1 = hmul2_bf16(tv[1], m1[h][1]);
              uint32_t v2 = hmul2_bf16(tv[2], m1[h][0]);
              uint32_t v3 = hmul2_bf16(tv[3], m1[h][1]);
              if (two_any) {
                v0 = hmul2_bf16(v0, m2[h][0]);
                v1 = hmul2_bf16(v1, m2[h][1]);
                v2 = hmul2_bf16(v2, m2[h][0]);
                v3 = hmul2_bf16(v3, m2[h][1]);
              }
              // k pair (16 kb + 2 tig) sits in 16-byte chunk 2 kb, k pair
              // (16 kb + 2 tig + 8) in chunk 2 kb + 1, both at byte 4 tig.
              const int c0 = 2 * kb, c1 = 2 * kb + 1;
              *reinterpret_cast<uint32_t*>(row_a + ((c0 ^ (r0 & 7)) << 4) + 4 * tig) = v0;
              *reinterpret_cast<uint32_t*>(row_b + ((c0 ^ ((r0 + 8) & 7)) << 4) + 4 * tig) = v1;
              *reinterpret_cast<uint32_t*>(row_a + ((c1 ^ (r0 & 7)) << 4) + 4 * tig) = v2;
              *reinterpret_cast<uint32_t*>(row_b + ((c1 ^ ((r0 + 8) & 7)) << 4) + 4 * tig) = v3;
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&cs_empty[cs]);
            mbar_arrive(&a_full[as]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (a.hk.push_tags != nullptr && threadIdx.x == 0) {
    // Every row this CTA stored precedes (bar.sync, then an acq_rel ticket
    // at gpu scope) the last CTA's ticket, which precedes its system-scope
    // fence and relaxed add to every rank: one fence covers all CTAs and
    // every rank.
    if (atom_add_acq_rel_gpu(a.hk.ticket, 1u) == gridDim.x - 1) {
      *a.hk.ticket = 0;
      fence_acq_rel_sys();
      for (int p = 0; p < a.hk.world; ++p) red_relaxed_sys_add(a.hk.push_done[p], 1);
    }
  }
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Elementwise kernels: dequantisation, layout conversion, tokamax codes.
// ---------------------------------------------------------------------------

// Raw e2m1 dequantisation with the GEMM's decode (delta = 0: value * scale
// exactly as the reference's bf16 multiply), natural column order.
template <int SD>
__global__ void fp4_dequant_raw_kernel(const uint8_t* __restrict__ codes,
                                       const uint8_t* __restrict__ scales, int groups, int k,
                                       int n, uint4* __restrict__ out) {
  const int64_t words_per_row = n / 8;
  const int64_t total = (int64_t)groups * k * words_per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / words_per_row;  // g * k + kk
    const int c8 = (int)(i - row * words_per_row);
    const int64_t g = row / k;
    const int kk = (int)(row - g * k);
    const uint32_t w = reinterpret_cast<const uint32_t*>(codes)[i];
    const uint8_t* sp = scales + ((g * (k / 32) + kk / 32) * (int64_t)n + (int64_t)c8 * 8) *
                                     ScaleTraits<SD>::bytes;
    uint32_t m1[4], m2[4];
    const bool two = raw_mults<SD, 0>(sp, m1, m2);
    const uint4 v = two ? decode8<false, true>(w, m1, m2) : decode8<false, false>(w, m1, m2);
    uint4 o;
    o.x = __byte_perm(v.x, v.y, 0x5410);  // columns 0,1
    o.y = __byte_perm(v.z, v.w, 0x5410);  // columns 2,3
    o.z = __byte_perm(v.x, v.y, 0x7632);  // columns 4,5
    o.w = __byte_perm(v.z, v.w, 0x7632);  // columns 6,7
    out[i] = o;
  }
}

// B200-layout dequantisation: one word = one lane's A fragment of a block.
template <int SD>
__global__ void fp4_dequant_b200_kernel(const uint32_t* __restrict__ codes,
                                        const uint8_t* __restrict__ scales, int groups, int k,
                                        int n, uint16_t* __restrict__ out) {
  const int64_t total = (int64_t)groups * k * n / 8;
  const int kb16 = k / 16, cb16 = n / 16;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int l = (int)(i & 31);
    const int64_t blk = i >> 5;
    const int kb = (int)(blk % kb16);
    const int64_t gc = blk / kb16;
    const int cb = (int)(gc % cb16);
    const int64_t g = gc / cb16;
    uint32_t tv[4];
    tvals<true>(codes[i], tv);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        int dk, dc;
        b200_nibble_coord(l, 2 * p + hh, dk, dc);
        const int kk = 16 * kb + dk, col = 16 * cb + dc;
        uint32_t m1, m2;
        const bool two = col_mult<SD, 0>(
            scales + ((g * (k / 32) + kk / 32) * (int64_t)n + col) * ScaleTraits<SD>::bytes, m1,
            m2);
        uint32_t v = hmul2_bf16(tv[p], m1);
        if (two) v = hmul2_bf16(v, m2);
        out[(g * k + kk) * (int64_t)n + col] = (uint16_t)(hh ? (v >> 16) : (v & 0xFFFFu));
      }
    }
  }
}

// raw [g, k, n/2] (column-pair bytes) -> B200 words.
__global__ void fp4_to_b200_kernel(const uint8_t* __restrict__ raw, uint32_t* __restrict__ out,
                                   int groups, int k, int n) {
  const int64_t total = (int64_t)groups * k * n / 8;
  const int kb16 = k / 16, cb16 = n / 16;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int l = (int)(i & 31);
    const int64_t blk = i >> 5;
    const int kb = (int)(blk % kb16);
    const int64_t gc = blk / kb16;
    const int cb = (int)(gc % cb16);
    const int64_t g = gc / cb16;
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int dk, dc;
      b200_nibble_coord(l, j, dk, dc);
      const int col = 16 * cb + dc;
      const uint8_t b = raw[(g * k + 16 * kb + dk) * (int64_t)(n / 2) + col / 2];
      word |= (uint32_t)((col & 1) ? (b >> 4) : (b & 0xF)) << (4 * j);
    }
    out[i] = b200_swizzle_word(word);
  }
}

// B200 words -> raw [g, k, n/2] bytes (one raw byte = columns 2c, 2c+1).
__global__ void fp4_from_b200_kernel(const uint32_t* __restrict__ b200, uint8_t* __restrict__ raw,
                                     int groups, int k, int n) {
  const int64_t total = (int64_t)groups * k * (n / 2);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int cp = (int)(i % (n / 2));
    const int64_t gk = i / (n / 2);
    const int kk = (int)(gk % k);
    const int64_t g = gk / k;
    uint32_t byte = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int col = 2 * cp + h;
      const int dk = kk & 15, dc = col & 15;
      // Invert b200_nibble_coord: dc = gid + 8*bit1(j), dk = 2t + bit0(j) + 8*bit2(j).
      const int gid = dc & 7, t = (dk & 7) >> 1;
      const int j = (dk & 1) | ((dc >> 3) << 1) | ((dk >> 3) << 2);
      const int l = gid * 4 + t;
      const uint32_t w =
          b200_unswizzle_word(b200[b200_word_index(g, col / 16, kk / 16, l, n, k)]);
      byte |= ((w >> (4 * j)) & 0xFu) << (4 * h);
    }
    raw[i] = (uint8_t)byte;
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

// ---------------------------------------------------------------------------
// Host launch
// ---------------------------------------------------------------------------

template <int SD, int VAR>
int launch(const void* lhs, const void* codes, const void* scales, const int32_t* group_sizes,
           int num_groups, int m, int k, int n, int group_offset, int n_local, int act,
           float limit, int out_dtype, int zero_init, void* out, cudaStream_t stream,
           const EpHooks* hooks = nullptr, int grp_lo = 0, int grp_hi = 1 << 30) {
  using L = Smem<SD>;
  CUtensorMap tm_lhs, tm_lhs_32, tm_lhs_64, tm_lhs_128, tm_codes, tm_scales;
  CUtensorMap* lhs_maps[4] = {&tm_lhs, &tm_lhs_32, &tm_lhs_64, &tm_lhs_128};
  int rc = 0;
  for (int i = 0; i < 4 && !rc; ++i)  // boxes of 16, 32, 64 and 128 token rows
    rc = encode_tmap_2d(lhs_maps[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, lhs, (uint64_t)k,
                        (uint64_t)m, (uint64_t)k * 2, BK, T_BOX_ROWS << i,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (VAR == kMN)
    rc = encode_tmap_2d(&tm_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, codes, (uint64_t)n / 2,
                        (uint64_t)n_local * k, (uint64_t)n / 2, BW / 2, BK,
                        CU_TENSOR_MAP_SWIZZLE_NONE);
  else  // rows = column blocks, each (k/16) blocks x 32 words
    rc = encode_tmap_2d(&tm_codes, CU_TENSOR_MAP_DATA_TYPE_UINT32, codes,
                        (uint64_t)(k / 16) * 32, (uint64_t)n_local * (n / 16),
                        (uint64_t)(k / 16) * 128, 4 * 32, BW / 16, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  rc = encode_tmap_2d(&tm_scales, ScaleTraits<SD>::tma, scales, (uint64_t)n,
                      (uint64_t)n_local * (k / 32), (uint64_t)n * ScaleTraits<SD>::bytes, BW, 2,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;

  rc = set_smem_limit(reinterpret_cast<const void*>(gmm_fp4_kernel<SD, VAR>), L::ALLOC, "gmm smem attribute");
  if (rc) return rc;
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
  a.grp_lo = grp_lo;
  a.grp_hi = grp_hi;
  a.status = status_ptr();
  a.hk = hooks ? *hooks : EpHooks{};
  gmm_fp4_kernel<SD, VAR><<<num_sms(), NUM_THREADS, L::ALLOC, stream>>>(
      tm_lhs, tm_lhs_32, tm_lhs_64, tm_lhs_128, tm_codes, tm_scales, a);
  return check_cuda(cudaGetLastError(), "gmm_fp4 launch");
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline unsigned grid_for(int64_t work, int threads, int per_sm = 16) {
  int64_t b = (work + threads - 1) / threads;
  int64_t cap = (int64_t)num_sms() * per_sm;
  return (unsigned)std::max<int64_t>(1, std::min(b, cap));
}

// Argument checks shared by the GEMM entry points.
static int validate(const void* lhs, const void* codes, int codes_format, const void* scales,
                    int scale_dtype, const int32_t* group_sizes, int num_groups, int m, int k,
                    int n, int group_offset, int num_local_groups, int act, int out_dtype,
                    void* out) {
  DWM_CHECK_ARG(codes_format == DWM_FP4_E2M1 || codes_format == DWM_FP4_B200,
                "gmm_fp4 takes e2m1 nibbles (raw or B200 layout); convert tokamax codes once "
                "with dwm_fp4_codes_convert");
  DWM_CHECK_ARG(scale_dtype == DWM_U8 || scale_dtype == DWM_BF16 || scale_dtype == DWM_F32,
                "scale dtype must be u8 (e8m0), bf16 or f32");
  DWM_CHECK_ARG(out_dtype == DWM_BF16 || out_dtype == DWM_F32, "out dtype must be bf16 or f32");
  DWM_CHECK_ARG(act == DWM_ACT_NONE || act == DWM_ACT_SWIGLU || act == DWM_ACT_SWIGLU_CLAMP,
                "unknown activation %d", act);
  DWM_CHECK_ARG(m >= 0 && k > 0 && n > 0, "bad shape m=%d k=%d n=%d", m, k, n);
  DWM_CHECK_ARG(k % BK == 0, "k=%d must be a multiple of %d", k, BK);
  DWM_CHECK_ARG(n % (NSUB * BW) == 0, "n=%d must be a multiple of 256", n);
  DWM_CHECK_ARG(num_groups >= 1 && num_groups <= MAX_GROUPS, "num_groups=%d out of [1, %d]",
                num_groups, MAX_GROUPS);
  DWM_CHECK_ARG(group_offset >= 0 && num_local_groups >= 0 &&
                    group_offset + num_local_groups <= num_groups,
                "group_offset=%d + num_local_groups=%d exceeds num_groups=%d", group_offset,
                num_local_groups, num_groups);
  DWM_CHECK_ARG(group_sizes && out && (m == 0 || lhs), "NULL pointer");
  DWM_CHECK_ARG(num_local_groups == 0 || (codes && scales), "NULL weights");
  DWM_CHECK_ARG(aligned16(lhs) && aligned16(codes) && aligned16(scales) && aligned16(out),
                "pointers must be 16-byte aligned");
  return DWM_OK;
}

// variant: 0 = choose, 1 = tcgen05 (shared-memory decode) with 128-row
// tiles, 2 = mma.sync decode kernel (B200 layout only) with 8-row token tiles
// up to 6 rows per local group on average and 16-row tiles above, 3 / 4 = the
// same with 8 / 16-row tiles, 7 = tcgen05 on CTA pairs (gmm_pair.cu, B200
// layout), 8 = 7 for each group's 256-row tiles and a remainder of at least
// kPairTailMin rows, the decode kernel for shorter remainders, 9 = 7 with
// tiles of up to 512 rows (two UMMAs per k-step over one decoded stage).
// The automatic choice for the B200 layout: mma.sync when the local groups
// average at most 16 rows (8 or 16-row tiles), variant 10 (each group on the
// kernel for its size) at 17-48, where groups straddle the classes (the
// 32-row decode tiles run their four MMAs per decoded fragment at about 290
// TFLOP/s, so they beat the tcgen05 kernels only while a group fits one
// tile), variant 7 from 96 rows and variant 9 from 224
// (prefill; most groups then exceed 256 rows or come close), else the
// single-CTA tcgen05 kernel with 128-row tiles. Variant 8 is not chosen
// automatically: since the pair kernel loads a partial token half in at most
// three copies, equal tiles (7) match it below 224 rows and 9 beats it above.
static int run(const void* lhs, const void* codes, int codes_format, const void* scales,
               int scale_dtype, const int32_t* group_sizes, int num_groups, int m, int k, int n,
               int group_offset, int num_local_groups, int act, float act_limit, int out_dtype,
               int zero_init, void* out, int variant, cudaStream_t s) {
  const int n_out = act == DWM_ACT_NONE ? n : n / 2;
  const size_t es = out_dtype == DWM_F32 ? 4 : 2;
  if (m == 0) return DWM_OK;
  if (num_local_groups == 0) {
    if (zero_init)
      return check_cuda(cudaMemsetAsync(out, 0, (size_t)m * n_out * es, s), "gmm zero");
    return DWM_OK;
  }
  const int64_t avg = ((int64_t)m + num_local_groups - 1) / num_local_groups;
  if (variant == 0)
    variant = codes_format != DWM_FP4_B200 ? 1
              : avg <= 16                  ? 2
              : avg <= 48                  ? 10
              : avg >= 224                 ? 9
              : avg >= 96                  ? 7
                                           : 1;
  if (variant >= 2 && variant <= 5)
    return launch_gmv(lhs, codes, scales, scale_dtype, group_sizes, num_groups, m, k, n,
                      group_offset, num_local_groups, act, act_limit, out_dtype, zero_init, out,
                      variant == 3 ? 1 : variant == 4 ? 2 : variant == 5 ? 4 : (avg <= 6 ? 1 : 2),
                      s);
  if (variant == 7)
    return launch_gmm_pair(lhs, codes, scales, scale_dtype, group_sizes, num_groups, m, k, n,
                           group_offset, num_local_groups, act, act_limit, out_dtype, zero_init,
                           out, nullptr, s, 0, 0);
  if (variant == 9)
    return launch_gmm_pair(lhs, codes, scales, scale_dtype, group_sizes, num_groups, m, k, n,
                           group_offset, num_local_groups, act, act_limit, out_dtype, zero_init,
                           out, nullptr, s, 0, 1);
  if (variant == 10) {
    // Each group on the kernel for its size: up to 16 rows on the decode
    // kernel's 16-row tiles, 17-32 on its 32-row tiles (one weight stream
    // each), 33-95 on the single-CTA tcgen05 kernel, larger groups on CTA
    // pairs with tiles of up to 512 rows. For skewed routing, where a group
    // of a few rows would otherwise cost the pair kernel a whole tile's
    // decode. The launches write disjoint rows; the first zeroes the rows
    // outside the local groups. A launch that finds no group of its class
    // costs a few microseconds.
    int rc = launch_gmv(lhs, codes, scales, scale_dtype, group_sizes, num_groups, m, k, n,
                        group_offset, num_local_groups, act, act_limit, out_dtype, zero_init, out,
                        2, s, 0, 0, kSplitRows16);
    if (rc) return rc;
    rc = launch_gmv(lhs, codes, scales, scale_dtype, group_sizes, num_groups, m, k, n,
                    group_offset, num_local_groups, act, act_limit, out_dtype, 0, out, 4, s, 0,
                    kSplitRows16, kSplitRows32);
    if (rc) return rc;
#define DWM_GMM_CLASS(SD)                                                                   \
  rc = launch<SD, kKS>(lhs, codes, scales, group_sizes, num_groups, m, k, n, group_offset,  \
                       num_local_groups, act, act_limit, out_dtype, 0, out, s, nullptr,     \
                       kSplitRows32, kSplitRows96)
    if (scale_dtype == DWM_U8)
      DWM_GMM_CLASS(DWM_U8);
    else if (scale_dtype == DWM_BF16)
      DWM_GMM_CLASS(DWM_BF16);
    else
      DWM_GMM_CLASS(DWM_F32);
#undef DWM_GMM_CLASS
    if (rc) return rc;
    return launch_gmm_pair(lhs, codes, scales, scale_dtype, group_sizes, num_groups, m, k, n,
                           group_offset, num_local_groups, act, act_limit, out_dtype, 0, out,
                           nullptr, s, 0, 1, kSplitRows96);
  }
  if (variant == 8) {
    // Full 256-row tiles (and remainders of kPairTailMin rows or more) on CTA
    // pairs, shorter remainders on the decode kernel: a remainder of r rows
    // costs the pair kernel a whole tile's decode, the decode kernel one
    // weight stream per 16 rows.
    int rc = launch_gmm_pair(lhs, codes, scales, scale_dtype, group_sizes, num_groups, m, k, n,
                             group_offset, num_local_groups, act, act_limit, out_dtype,
                             zero_init, out, nullptr, s, kPairTailMin, 0);
    if (rc) return rc;
    return launch_gmv(lhs, codes, scales, scale_dtype, group_sizes, num_groups, m, k, n,
                      group_offset, num_local_groups, act, act_limit, out_dtype, 0, out, 2, s,
                      kPairTailMin);
  }
#define DWM_GMM_LAUNCH(SD, VAR)                                                        \
  return launch<SD, VAR>(lhs, codes, scales, group_sizes, num_groups, m, k, n, group_offset, \
                         num_local_groups, act, act_limit, out_dtype, zero_init, out, s)
#define DWM_GMM_BY_SCALE(VAR)                                   \
  do {                                                          \
    if (scale_dtype == DWM_U8) DWM_GMM_LAUNCH(DWM_U8, VAR);     \
    if (scale_dtype == DWM_BF16) DWM_GMM_LAUNCH(DWM_BF16, VAR); \
    DWM_GMM_LAUNCH(DWM_F32, VAR);                               \
  } while (0)
  if (codes_format == DWM_FP4_B200) DWM_GMM_BY_SCALE(kKS);
  DWM_GMM_BY_SCALE(kMN);
#undef DWM_GMM_BY_SCALE
#undef DWM_GMM_LAUNCH
}

}  // namespace gmm
}  // namespace dwm

using namespace dwm;

namespace dwm {
// The single-CTA tcgen05 kernel on B200-layout codes with expert-parallel
// hooks (dwm_ep_gmm_fp4); the caller has validated the arguments.
int launch_gmm_single_ep(const void* lhs, const void* codes, const void* scales, int scale_dtype,
                         const int32_t* group_sizes, int num_groups, int m, int k, int n,
                         int act, float limit, int out_dtype, void* out, const EpHooks* hooks,
                         cudaStream_t stream) {
  if (scale_dtype == DWM_U8)
    return gmm::launch<DWM_U8, gmm::kKS>(lhs, codes, scales, group_sizes, num_groups, m, k, n, 0,
                                         num_groups, act, limit, out_dtype, 0, out, stream, hooks);
  if (scale_dtype == DWM_BF16)
    return gmm::launch<DWM_BF16, gmm::kKS>(lhs, codes, scales, group_sizes, num_groups, m, k, n,
                                           0, num_groups, act, limit, out_dtype, 0, out, stream,
                                           hooks);
  return gmm::launch<DWM_F32, gmm::kKS>(lhs, codes, scales, group_sizes, num_groups, m, k, n, 0,
                                        num_groups, act, limit, out_dtype, 0, out, stream, hooks);
}
}  // namespace dwm

extern "C" int dwm_gmm_fp4(const void* lhs, const void* codes, int codes_format,
                           const void* scales, int scale_dtype, const int32_t* group_sizes,
                           int num_groups, int m, int k, int n, int group_offset,
                           int num_local_groups, int act, float act_limit, int out_dtype,
                           int zero_init, void* out, void* stream) {
  int rc = gmm::validate(lhs, codes, codes_format, scales, scale_dtype, group_sizes, num_groups,
                         m, k, n, group_offset, num_local_groups, act, out_dtype, out);
  if (rc) return rc;
  return gmm::run(lhs, codes, codes_format, scales, scale_dtype, group_sizes, num_groups, m, k,
                  n, group_offset, num_local_groups, act, act_limit, out_dtype, zero_init, out,
                  0, static_cast<cudaStream_t>(stream));
}

extern "C" int dwm_gmm_fp4_variant(const void* lhs, const void* codes, int codes_format,
                                   const void* scales, int scale_dtype,
                                   const int32_t* group_sizes, int num_groups, int m, int k,
                                   int n, int group_offset, int num_local_groups, int act,
                                   float act_limit, int out_dtype, int zero_init, void* out,
                                   int variant, void* stream) {
  DWM_CHECK_ARG(variant >= 0 && variant <= 10 && variant != 6,
                "variant must be 0 (auto), 1 (tcgen05, one CTA), 2-5 (mma.sync decode "
                "kernel), 7 (tcgen05 on CTA pairs), 8 (CTA pairs + decode-kernel tails), 9 "
                "(CTA pairs, 512-row tiles) or 10 (each group on the kernel for its size)");
  DWM_CHECK_ARG(variant == 0 || codes_format == DWM_FP4_B200,
                "variants 1-5 and 7-10 need the B200 layout");
  int rc = gmm::validate(lhs, codes, codes_format, scales, scale_dtype, group_sizes, num_groups,
                         m, k, n, group_offset, num_local_groups, act, out_dtype, out);
  if (rc) return rc;
  return gmm::run(lhs, codes, codes_format, scales, scale_dtype, group_sizes, num_groups, m, k,
                  n, group_offset, num_local_groups, act, act_limit, out_dtype, zero_init, out,
                  variant, static_cast<cudaStream_t>(stream));
}

extern "C" int dwm_fp4_dequant(const void* codes, int codes_format, const void* scales,
                               int scale_dtype, int groups, int k, int n, void* out,
                               void* stream) {
  DWM_CHECK_ARG(codes && scales && out, "NULL pointer");
  DWM_CHECK_ARG(codes_format == DWM_FP4_E2M1 || codes_format == DWM_FP4_B200,
                "codes_format must be DWM_FP4_E2M1 or DWM_FP4_B200");
  DWM_CHECK_ARG(groups >= 0 && k > 0 && n > 0 && k % 32 == 0 && n % 16 == 0,
                "bad shape groups=%d k=%d n=%d (k %% 32, n %% 16)", groups, k, n);
  DWM_CHECK_ARG(gmm::aligned16(out) && (reinterpret_cast<uintptr_t>(codes) & 3) == 0,
                "misaligned pointer");
  DWM_CHECK_ARG(scale_dtype == DWM_U8 || scale_dtype == DWM_BF16 || scale_dtype == DWM_F32,
                "scale dtype must be u8, bf16 or f32");
  const int64_t total = (int64_t)groups * k * (n / 8);
  if (total == 0) return DWM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int threads = 256;
  const unsigned blocks = gmm::grid_for(total, threads);
  auto sc = static_cast<const uint8_t*>(scales);
  if (codes_format == DWM_FP4_B200) {
    auto cw = static_cast<const uint32_t*>(codes);
    auto o = static_cast<uint16_t*>(out);
    if (scale_dtype == DWM_U8)
      gmm::fp4_dequant_b200_kernel<DWM_U8><<<blocks, threads, 0, s>>>(cw, sc, groups, k, n, o);
    else if (scale_dtype == DWM_BF16)
      gmm::fp4_dequant_b200_kernel<DWM_BF16><<<blocks, threads, 0, s>>>(cw, sc, groups, k, n, o);
    else
      gmm::fp4_dequant_b200_kernel<DWM_F32><<<blocks, threads, 0, s>>>(cw, sc, groups, k, n, o);
  } else {
    auto c = static_cast<const uint8_t*>(codes);
    auto o = static_cast<uint4*>(out);
    if (scale_dtype == DWM_U8)
      gmm::fp4_dequant_raw_kernel<DWM_U8><<<blocks, threads, 0, s>>>(c, sc, groups, k, n, o);
    else if (scale_dtype == DWM_BF16)
      gmm::fp4_dequant_raw_kernel<DWM_BF16><<<blocks, threads, 0, s>>>(c, sc, groups, k, n, o);
    else
      gmm::fp4_dequant_raw_kernel<DWM_F32><<<blocks, threads, 0, s>>>(c, sc, groups, k, n, o);
  }
  return check_cuda(cudaGetLastError(), "fp4_dequant launch");
}

extern "C" int dwm_fp4_to_b200(const void* in, void* out, int groups, int k, int n, int inverse,
                               void* stream) {
  DWM_CHECK_ARG(in && out && in != out, "NULL or aliased pointers (out-of-place only)");
  DWM_CHECK_ARG(groups >= 0 && k > 0 && n > 0 && k % 16 == 0 && n % 16 == 0,
                "bad shape groups=%d k=%d n=%d (k %% 16, n %% 16)", groups, k, n);
  DWM_CHECK_ARG(((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 3) == 0,
                "pointers must be 4-byte aligned");
  const int64_t words = (int64_t)groups * k * n / 8;
  if (words == 0) return DWM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!inverse)
    gmm::fp4_to_b200_kernel<<<gmm::grid_for(words, 256), 256, 0, s>>>(
        static_cast<const uint8_t*>(in), static_cast<uint32_t*>(out), groups, k, n);
  else
    gmm::fp4_from_b200_kernel<<<gmm::grid_for(words * 4, 256), 256, 0, s>>>(
        static_cast<const uint32_t*>(in), static_cast<uint8_t*>(out), groups, k, n);
  return check_cuda(cudaGetLastError(), "fp4_to_b200 launch");
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
  gmm::fp4_codes_convert_kernel<<<gmm::grid_for((int64_t)nbytes, 256), 256, 0, s>>>(
      static_cast<const uint8_t*>(in), static_cast<uint8_t*>(out), nbytes,
      to_format == DWM_FP4_TOKAMAX);
  return check_cuda(cudaGetLastError(), "codes_convert launch");
}
