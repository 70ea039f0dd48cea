// FP4 grouped matmul on CTA pairs for prefill-sized groups: tokamax gmm_v2
// with rhs_fp4_codes (TK:107-153), weights in the B200 layout
// (fp4_decode.cuh), decoded on the SM and multiplied with tcgen05
// cta_group::2 UMMAs.
//
// The product is computed transposed as in gmm_fp4.cu: decoded weight columns
// are UMMA operand A (rows), token rows are operand B. Two CTAs on
// neighbouring SMs (a cluster of 2) share one 256 x N tile:
//   - each CTA decodes its own 128 weight columns of a 64-k stage into its
//     shared memory (A) and loads half of the tile's N token rows (B);
//   - the even CTA issues the M = 256 UMMAs, which take the time of a
//     single-SM 128 x N UMMA;
//   - each CTA's TMEM holds its 128 x N f32 accumulator, double-buffered
//     (2 x 256 columns), so a tile's epilogue overlaps the next main loop.
// Against one CTA with two 128-column sub-tiles and N = 128 this halves the
// decode work per output and reaches the UMMA's full rate (N = 256).
//
// Tile geometry: a pair tile covers 128 SwiGLU features (their gate and up
// columns, 64 features per CTA) or 256 plain columns (128 per CTA), and up
// to 256 token rows of one group. A group of r rows takes ceil(r / 256) tiles
// of equal size, N rounded up to 32 so that each CTA's half is a whole number
// of 16-row TMA boxes. In A, each 16-feature gate block sits next to its up
// block, so one TMEM lane quarter holds both and the SwiGLU epilogue pairs
// them with one warp shuffle.
//
// Warp roles in each CTA (768 threads):
//   warps 0-3   epilogue: TMEM lane quarter = warp
//   warp  4     TMA: FP4 codes + scales of this CTA's columns (HBM stream)
//   warp  5     pair TMEM allocation; UMMA issuer in the even CTA (the whole
//               warp runs the loop so its operands stay warp-uniform, one
//               elected lane issues: a UMMA takes ~100 cycles to issue)
//   warps 6-7   TMA: this CTA's half of the token rows (L2-resident)
//   warps 8-23  decode, groups of warps taking the stages in turn
//
// A pipeline stage holds one 64-k step of both operands (the decoded A and
// this CTA's token rows) behind one "full" barrier in the even CTA, so the
// single issuing thread waits once and commits once per step: both CTAs'
// token copies complete on it (the even CTA expects the bytes of both
// halves) and both CTAs' decode warps arrive on it remotely. The issuer's
// commits arrive on the matching barrier of both CTAs. Every wait is bounded
// (common.cuh). Numerics are those of gmm_fp4.cu (E0901:84-95).
#include <algorithm>
#include <map>
#include <mutex>

#include "fp4_decode.cuh"

namespace dwm {
namespace gmm_pair {

using namespace fp4;

constexpr int ROWS = 128;        // A rows (weight columns) per CTA
constexpr int BK = 64;           // k per stage
constexpr int BT = 256;          // token rows per tile at most (pair UMMA N)
constexpr int HALF = BT / 2;     // token rows per CTA at most
constexpr int NUM_THREADS = 768;
constexpr int EPI_WARPS = 4;
constexpr int PRODUCER_WARP = 4;
constexpr int MMA_WARP = 5;
constexpr int TOKEN_WARP = 6;   // token copies of even index in a stage's list
constexpr int TOKEN_WARP2 = 7;  // and of odd index
constexpr int DEC_WARP0 = 8;
#ifndef DWM_PAIR_DEC_GROUPS
#define DWM_PAIR_DEC_GROUPS 2
#endif
#ifndef DWM_PAIR_DEC_SYNC
#define DWM_PAIR_DEC_SYNC 0
#endif
constexpr int DEC_WARPS = 16;                       // decode warps per CTA
constexpr int DEC_GROUPS = DWM_PAIR_DEC_GROUPS;      // groups taking stages in turn
constexpr int NUM_DEC_WARPS = DEC_WARPS / DEC_GROUPS;  // per group
constexpr int BLOCKS_PER_WARP = 8 / NUM_DEC_WARPS;     // 16-column code blocks per warp
static_assert(DEC_GROUPS == 2 || DEC_GROUPS == 4, "2 or 4 decode groups");
constexpr int MAX_GROUPS = 1024;
constexpr int TMEM_COLS = 512;    // two 256-column accumulator buffers
constexpr int ACC_COLS = 256;
constexpr int A_STAGE = ROWS * BK * 2;  // 16 KiB of bf16, 128-byte swizzled, K-major
constexpr int T_STAGE = HALF * BK * 2;  // 16 KiB: this CTA's token rows of one k-step
constexpr int C_STAGE = ROWS * BK / 2;  // 4 KiB of codes: 8 column blocks x 4 k-blocks x 32 words
constexpr int T_BOX_ROWS = 16;
constexpr int T_BOX_BYTES = T_BOX_ROWS * BK * 2;  // 2 KiB
constexpr int EPI_WARP_BYTES = 16 * 32 * 4;       // 16 token rows x 32 columns of f32

#ifndef DWM_PAIR_STAGES
#define DWM_PAIR_STAGES 5
#endif
#ifndef DWM_PAIR_CS
#define DWM_PAIR_CS 8
#endif
#ifndef DWM_PAIR_EPI_SLEEP
#define DWM_PAIR_EPI_SLEEP 256
#endif

// WIDE: tiles of up to 512 token rows as two UMMAs per k16 step (N = 256 and
// the rest) into both TMEM accumulator slots over one decoded A, so a group
// of 257-512 rows costs one tile's decode instead of two; each CTA then
// stages up to 256 token rows per k-step (a 32 KiB token stage), which leaves
// room for 4 stages. Such a tile holds both slots, so its epilogue overlaps
// only the next tile's wait for its first slot (AccRing).
template <int SD, bool WIDE>
struct Layout {
  static constexpr int S = WIDE ? 4 : DWM_PAIR_STAGES;
  static constexpr int CS = WIDE ? (ScaleTraits<SD>::bytes == 1 ? 4 : 3) : DWM_PAIR_CS;
  static constexpr int T_ST = (WIDE ? 2 : 1) * T_STAGE;  // this CTA's token rows of a k-step
  static constexpr int STG = A_STAGE + T_ST;
  static constexpr int S_STAGE = 2 * ROWS * ScaleTraits<SD>::bytes;  // [k32 block][128 rows]
  static constexpr int OFF_STAGE = 0;  // stage i: A at i * STG, tokens A_STAGE after it
  static constexpr int OFF_C = OFF_STAGE + S * STG;
  static constexpr int OFF_S = OFF_C + CS * C_STAGE;
  static constexpr int OFF_BAR = OFF_S + CS * S_STAGE;
  static constexpr int NUM_BARS = 2 * CS + 2 * S + 4 + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int OFF_ROWS = OFF_MISC + 64;
  static constexpr int OFF_TILES = OFF_ROWS + (MAX_GROUPS + 1) * 4;
  static constexpr int OFF_EPI = (OFF_TILES + (MAX_GROUPS + 1) * 4 + 15) & ~15;
  static constexpr int BYTES = OFF_EPI + EPI_WARPS * EPI_WARP_BYTES;
  static constexpr int ALLOC = BYTES + 1024;  // slack for 1 KiB alignment
  static_assert(ALLOC <= 232448, "exceeds the 227 KiB per-CTA shared memory");
  static_assert(STG % 1024 == 0 && A_STAGE % 1024 == 0, "swizzled tiles need 1 KiB alignment");
  static_assert(CS <= 32 && S <= 32, "ring masks are 32-bit");
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
  int n_tiles;  // pair column tiles per group (n / 256)
  int max_rows; // token rows per tile at most: 256, or 512 for the WIDE kernel
  int tail_min; // 0: a group's rows in tiles of equal size; > 0: tiles of 256 rows and
                // a last tile only if at least tail_min rows remain (fewer are left to
                // the decode kernel, which streams the weights once per 16 rows)
  int grp_lo;   // only groups of more than grp_lo rows (variant 10's size classes)
  int* status;
  EpHooks hk;   // expert-parallel gating / push (all null for a plain GEMM)
};

struct Tile {
  int g;      // local group
  int row0;   // first lhs row
  int rows;   // valid rows (1..BT)
  int n_idx;  // column tile
};

// Row tiles of a group of `rows` rows, tiles of at most bt rows (see
// Args::tail_min).
__device__ __forceinline__ int group_tiles(int rows, int bt, int tail_min, int grp_lo) {
  if (rows <= grp_lo) return 0;
  if (tail_min <= 0) return (rows + bt - 1) / bt;
  return rows / bt + (rows % bt >= tail_min ? 1 : 0);
}

// A group whose tiles exceed 256 rows (WIDE kernel, equal-size tiles): two
// UMMAs per k-step.
__device__ __forceinline__ bool wide_group(int rows, const Args& a) {
  if (a.max_rows <= BT || a.tail_min > 0 || rows <= BT) return false;
  const int nt = (rows + a.max_rows - 1) / a.max_rows;
  return (rows + nt - 1) / nt > BT;
}

// tile_prefix entries: first tile index (low kTileBits) | local group above.
constexpr int kTileBits = 21;
constexpr int kTileMask = (1 << kTileBits) - 1;

__device__ __forceinline__ Tile get_tile(int idx, const int* row_start, const int* tile_prefix,
                                         const Args& a) {
  int lo = 0, hi = a.n_local;  // first tile of position lo <= idx < that of position hi
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if ((tile_prefix[mid] & kTileMask) <= idx) lo = mid; else hi = mid;
  }
  Tile t;
  t.g = tile_prefix[lo] >> kTileBits;
  const int local = idx - (tile_prefix[lo] & kTileMask);
  const int t_idx = local / a.n_tiles;
  t.n_idx = local - t_idx * a.n_tiles;
  const int gs_start = row_start[a.group_offset + t.g];
  const int gs_rows = row_start[a.group_offset + t.g + 1] - gs_start;
  const int bt = a.max_rows;
  if (a.tail_min > 0) {
    t.row0 = gs_start + t_idx * bt;
    t.rows = min(bt, gs_rows - t_idx * bt);
    return t;
  }
  const int nt = (gs_rows + bt - 1) / bt;
  const int r_lo = (int)(((int64_t)t_idx * gs_rows) / nt);
  const int r_hi = (int)(((int64_t)(t_idx + 1) * gs_rows) / nt);
  t.row0 = gs_start + r_lo;
  t.rows = r_hi - r_lo;
  return t;
}

// The two 256-column TMEM accumulator slots. A tile of up to 256 rows takes
// the next slot and the one after alternates; a WIDE tile of more rows takes
// both (rows 0-255 in the next slot sa, the rest in the other, sb). Its
// epilogue drains sb first (at most 256 rows, often a few chunks) and the
// next tile starts in sb, so it waits for that short drain only. The UMMA
// issuer and the epilogue walk the same tile sequence with a ring each; par
// bit s is the phase parity of slot s's next fill.
struct AccRing {
  int nxt = 0;
  uint32_t par = 0;
  __device__ __forceinline__ void take(bool both, int& sa, int& sb, uint32_t& pa,
                                       uint32_t& pb) {
    sa = nxt;
    sb = nxt ^ 1;
    pa = (par >> sa) & 1u;
    pb = (par >> sb) & 1u;
    par ^= 1u << sa;
    if (both) {
      par ^= 1u << sb;
      nxt = sb;
    } else {
      nxt ^= 1;
    }
  }
};

// UMMA N of a tile: rows rounded up to 32 (each CTA's half a multiple of 16).
__device__ __forceinline__ int tile_n(int rows) { return max(32, (rows + 31) & ~31); }

// A 32-bit shared store that the compiler may schedule freely among the
// other loads and stores (no memory clobber); volatile asm keeps it before
// the proxy fence that publishes the stage.
__device__ __forceinline__ void sts_b32_free(uint32_t a, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(a), "r"(v));
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// A decode group's wait for its next stage (codes landed, stage released by
// the pair's UMMAs). DWM_PAIR_DEC_SYNC 0 (default): every warp polls for
// itself, so the group's warps drift apart within a stage (10% faster on
// 256-row tiles); 1: the group's first warp polls, the others park on named
// barrier 1 + grp, and the outcome is double-buffered by the group's step
// parity (3% faster on tiles of 16-32 rows).
__device__ __forceinline__ bool group_wait(int grp, int dw, uint32_t step, uint64_t* full,
                                           uint32_t full_ph, uint64_t* empty, uint32_t empty_ph,
                                           volatile int* abort_flag, volatile int* go,
                                           int* status) {
  if (DWM_PAIR_DEC_SYNC == 0) {
    bool got = mbar_wait(full, full_ph, abort_flag, status);
    got = got && mbar_wait(empty, empty_ph, abort_flag, status);
    return __all_sync(0xffffffffu, got);
  }
  volatile int* slot = go + grp * 2 + ((step / DEC_GROUPS) & 1);
  if (dw == 0) {
    bool got = mbar_wait(full, full_ph, abort_flag, status);
    got = got && mbar_wait(empty, empty_ph, abort_flag, status);
    got = __all_sync(0xffffffffu, got);
    if ((threadIdx.x & 31) == 0) *slot = got ? 1 : 0;
  }
  named_bar_sync(1 + grp, NUM_DEC_WARPS * 32);
  return *slot != 0;
}

template <int SD, bool WIDE>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gmm_pair_kernel(const __grid_constant__ CUtensorMap tm_lhs,
                    const __grid_constant__ CUtensorMap tm_lhs_32,
                    const __grid_constant__ CUtensorMap tm_lhs_64,
                    const __grid_constant__ CUtensorMap tm_lhs_half,
                    const __grid_constant__ CUtensorMap tm_codes,
                    const __grid_constant__ CUtensorMap tm_scales, const Args a) {
  using L = Layout<SD, WIDE>;
  constexpr int CS = L::CS;
  constexpr int S = L::S;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* cs_full = bars;             // local: code TMA landed
  uint64_t* cs_empty = cs_full + CS;    // local: decode group done with the codes
  uint64_t* full = cs_empty + CS;      // even CTA: both CTAs' A decoded and tokens landed
  uint64_t* empty = full + S;           // each CTA: the pair's UMMAs done with the stage
  uint64_t* acc_full = empty + S;       // each CTA: accumulator buffer complete
  uint64_t* acc_empty = acc_full + 2;   // even CTA: both CTAs drained the buffer
  uint64_t* drain_bar = acc_empty + 2;  // each CTA: every UMMA complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);
  volatile int* group_go = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 16);  // [4][2]
  int* row_start = reinterpret_cast<int*>(smem + L::OFF_ROWS);
  int* tile_prefix = reinterpret_cast<int*>(smem + L::OFF_TILES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cl = (int)cluster_index();
  const int ncl = (int)cluster_count();

  if (threadIdx.x == 0) {
    for (int i = 0; i < CS; ++i) {
      mbar_init(&cs_full[i], 1);
      mbar_init(&cs_empty[i], NUM_DEC_WARPS);
    }
    for (int i = 0; i < S; ++i) {
      // Decode warps of both CTAs, the even CTA's expect_tx for the token
      // bytes of both halves, and TOKEN_WARP2 of both CTAs.
      mbar_init(&full[i], 2 * NUM_DEC_WARPS + 3);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 2 * EPI_WARPS);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == PRODUCER_WARP && lane == 0) {
    tma_prefetch_desc(&tm_lhs);
    tma_prefetch_desc(&tm_lhs_32);
    tma_prefetch_desc(&tm_lhs_64);
    tma_prefetch_desc(&tm_lhs_half);
    tma_prefetch_desc(&tm_codes);
    tma_prefetch_desc(&tm_scales);
  }
  if (warp == 0) {
    // Row starts over all groups (rows are sorted by group), then the tile
    // prefix over the local groups.
    const int G = a.num_groups;
    const int per = (G + 31) / 32;
    int sum = 0;
    for (int i = 0; i < per; ++i) {
      const int g = lane * per + i;
      if (g < G) {
        int v = a.group_sizes[g];
        if (v < 0) { report(a.status, DWM_DEV_BAD_INDEX); v = 0; }
        sum += v;
      }
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    int run = incl - sum;
    for (int i = 0; i < per; ++i) {
      const int g = lane * per + i;
      if (g < G) {
        const int v = max(a.group_sizes[g], 0);
        row_start[g] = min(run, a.m);
        run += v;
      }
    }
    if (lane == 31) {
      row_start[G] = min(run, a.m);
      if (run > a.m) report(a.status, DWM_DEV_BAD_INDEX);
    }
    __syncwarp();
    // Local groups in schedule order: those with a tile above 256 rows (two
    // UMMAs per k-step, the costliest tiles) first, so that the round-robin
    // assignment of tiles to clusters spreads them evenly. tile_prefix[i] =
    // first tile of the i-th group in that order | its group << kTileBits.
    const int NL = a.n_local;
    const int per2 = (NL + 31) / 32;
    auto rows_of = [&](int g) {
      return row_start[a.group_offset + g + 1] - row_start[a.group_offset + g];
    };
    int nwide = 0;
    for (int i = 0; i < per2; ++i) {
      const int g = lane * per2 + i;
      if (g < NL && wide_group(rows_of(g), a)) ++nwide;
    }
    int wincl = nwide;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wincl, o);
      if (lane >= o) wincl += y;
    }
    const int wide_total = __shfl_sync(0xffffffffu, wincl, 31);
    int wpos = wincl - nwide;                           // next wide position
    int npos = wide_total + lane * per2 - (wincl - nwide);  // next narrow position
    for (int i = 0; i < per2; ++i) {
      const int g = lane * per2 + i;
      if (g < NL) tile_prefix[wide_group(rows_of(g), a) ? wpos++ : npos++] = g;
    }
    __syncwarp();
    int tsum = 0;
    for (int i = 0; i < per2; ++i) {
      const int pos = lane * per2 + i;
      if (pos < NL) tsum += group_tiles(rows_of(tile_prefix[pos]), a.max_rows, a.tail_min, a.grp_lo) * a.n_tiles;
    }
    int tincl = tsum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, tincl, o);
      if (lane >= o) tincl += y;
    }
    int trun = tincl - tsum;
    for (int i = 0; i < per2; ++i) {
      const int pos = lane * per2 + i;
      if (pos < NL) {
        const int g = tile_prefix[pos];
        tile_prefix[pos] = trun | (g << kTileBits);
        trun += group_tiles(rows_of(g), a.max_rows, a.tail_min, a.grp_lo) * a.n_tiles;
      }
    }
    if (lane == 31) tile_prefix[NL] = trun;
  }
  if (warp == MMA_WARP) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  // Barriers initialised and TMEM allocated in both CTAs before any
  // cross-CTA arrival.
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int total = tile_prefix[a.n_local];
  const int KT = a.k / BK;
  const bool act = a.act != DWM_ACT_NONE;
  // The even CTA's barriers, as shared::cluster addresses.
  const uint32_t full_0 = mapa_shared(full, 0);
  const uint32_t acc_empty_0 = mapa_shared(acc_empty, 0);

  if (warp < EPI_WARPS) {
    // ---------------- epilogue ----------------
    const int es = a.out_f32 ? 4 : 2;
    const int q = warp;  // TMEM lane quarter
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
    const uint32_t epi_s = smem_u32(smem + L::OFF_EPI + q * EPI_WARP_BYTES);
    constexpr float acc_scale = (float)(1 << decode_delta<SD>());  // undoes the decode bias
    const bool hi_lane = lane >= 16;
    AccRing ring;
    for (int idx = cl; idx < total; idx += ncl) {
      const Tile t = get_tile(idx, row_start, tile_prefix, a);
      const bool both = WIDE && tile_n(t.rows) > BT;
      int sa, sb;
      uint32_t pa, pb;
      ring.take(both, sa, sb, pa, pb);
      bool got = mbar_wait<DWM_PAIR_EPI_SLEEP>(&acc_full[sa], pa, abort_flag, a.status);
      if (both) got = got && mbar_wait<DWM_PAIR_EPI_SLEEP>(&acc_full[sb], pb, abort_flag, a.status);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
      const uint32_t ta = tq + (uint32_t)(sa * ACC_COLS), tb = tq + (uint32_t)(sb * ACC_COLS);
      // Chunk c of 16 token rows: rows 0-255 in slot sa, the rest in sb. A
      // two-slot tile drains chunks 16.. (slot sb) first: step ci takes
      // chunk chunk_of(ci), and sb is free once its chunks are in registers.
      const int nchunks = (t.rows + 15) >> 4;
      const int n_sb = both ? nchunks - 16 : 0;
      auto chunk_of = [&](int ci) { return ci < n_sb ? 16 + ci : ci - n_sb; };
      auto chunk_addr = [&](int c) { return (c < 16 ? ta : tb) + (uint32_t)((c & 15) * 16); };
      auto release_first = [&](int ci) {
        if (ci == n_sb - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_remote(acc_empty_0 + (uint32_t)(sb * 8));
        }
      };
      if (act) {
        // Lanes 0-15 hold the gate, lanes 16-31 the up column of features
        // fcol + (lane & 15); lane < 16 forms the even tokens of a chunk,
        // lane >= 16 the odd ones, each after one shuffle with its partner.
        const int64_t fcol = (int64_t)t.n_idx * 128 + rank * 64 + q * 16;
        const int row_bytes = 16 * es;  // one staged token row: 16 features
        const int vpr = row_bytes / 16;
        for (int ci = 0; ci < nchunks; ++ci) {
          const int c = chunk_of(ci);
          uint32_t r[16];
          tmem_ld16(chunk_addr(c), r);
          tmem_ld_wait();
          release_first(ci);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float even = __uint_as_float(r[2 * e]) * acc_scale;
            const float odd = __uint_as_float(r[2 * e + 1]) * acc_scale;
            const float recv = __shfl_xor_sync(0xffffffffu, hi_lane ? even : odd, 16);
            float g = hi_lane ? recv : even;
            float u = hi_lane ? odd : recv;
            if (a.act == DWM_ACT_SWIGLU_CLAMP) {
              g = fminf(g, a.limit);
              u = fminf(fmaxf(u, -a.limit), a.limit);
            }
            const float v = g * sigmoid_fast(g) * u;
            const uint32_t at = (uint32_t)((2 * e + (hi_lane ? 1 : 0)) * row_bytes + (lane & 15) * es);
            if (a.out_f32)
              sts_f32(epi_s + at, v);
            else
              sts_u16(epi_s + at, (uint16_t)f32_to_bf16_bits(v));
          }
          __syncwarp();
          for (int qv = lane; qv < 16 * vpr; qv += 32) {
            const int e = qv / vpr, j = qv - e * vpr;
            const int rr = c * 16 + e;
            if (rr < t.rows) {
              const uint4 v = lds_u128(epi_s + (uint32_t)(e * row_bytes + j * 16));
              const int64_t off = ((t.row0 + rr) * (int64_t)a.ldo + fcol) * es + j * 16;
              *reinterpret_cast<uint4*>(static_cast<uint8_t*>(a.out) + off) = v;
            }
          }
          __syncwarp();
        }
      } else {
        const int64_t ccol = (int64_t)t.n_idx * 256 + rank * 128 + q * 32;
        const int row_bytes = 32 * es;  // one staged token row: 32 columns
        const int vpr = row_bytes / 16;
        for (int ci = 0; ci < nchunks; ++ci) {
          const int c = chunk_of(ci);
          uint32_t r[16];
          tmem_ld16(chunk_addr(c), r);
          tmem_ld_wait();
          release_first(ci);
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float v = __uint_as_float(r[e]) * acc_scale;
            const uint32_t at = (uint32_t)(e * row_bytes + lane * es);
            if (a.out_f32)
              sts_f32(epi_s + at, v);
            else
              sts_u16(epi_s + at, (uint16_t)f32_to_bf16_bits(v));
          }
          __syncwarp();
          for (int qv = lane; qv < 16 * vpr; qv += 32) {
            const int e = qv / vpr, j = qv - e * vpr;
            const int rr = c * 16 + e;
            if (rr < t.rows) {
              const uint4 v = lds_u128(epi_s + (uint32_t)(e * row_bytes + j * 16));
              if (a.hk.push_tags != nullptr) {
                // Expert parallel: straight into the token owner's buffer, at
                // the row of its (token, k) pair (over NVLink for a peer).
                const int tag = a.hk.push_tags[t.row0 + rr];
                if (tag >= 0) {
                  const int64_t off =
                      ((int64_t)(tag & ((1 << kEpTagBits) - 1)) * a.ldo + ccol) * es + j * 16;
                  *reinterpret_cast<uint4*>(a.hk.push_base[tag >> kEpTagBits] + off) = v;
                }
              } else {
                const int64_t off = ((t.row0 + rr) * (int64_t)a.ldo + ccol) * es + j * 16;
                *reinterpret_cast<uint4*>(static_cast<uint8_t*>(a.out) + off) = v;
              }
            }
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(acc_empty_0 + (uint32_t)(sa * 8));
    }
  } else if (warp == PRODUCER_WARP) {
    // ---------------- TMA producer: codes + scales (HBM stream) ----------------
    if (lane == 0) {
      const uint64_t pol_stream = policy_evict_first();
      constexpr uint32_t cs_bytes = C_STAGE + L::S_STAGE;
      int cs = 0;
      uint32_t cs_ph = 0, cs_armed = 0, cs_par = 0;
      bool ok = true;
      for (int idx = cl; idx < total && ok; idx += ncl) {
        const Tile t = get_tile(idx, row_start, tile_prefix, a);
        // This CTA's first column: features (gate) with SwiGLU, else columns.
        const int col0 = act ? t.n_idx * 128 + (int)rank * 64 : t.n_idx * 256 + (int)rank * 128;
        const int blk = t.g * (a.n / 16) + col0 / 16;
        const int srow = t.g * (a.k / 32);
        for (int kk = 0; kk < KT; ++kk) {
          if (!mbar_wait(&cs_empty[cs], cs_ph ^ 1, abort_flag, a.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&cs_full[cs], cs_bytes);
          cs_armed |= 1u << cs;
          cs_par = (cs_par & ~(1u << cs)) | (cs_ph << cs);
          tma_load_3d(smem + L::OFF_C + cs * C_STAGE, &tm_codes, &cs_full[cs], kk * 128, blk, 0,
                      pol_stream);
          tma_load_3d(smem + L::OFF_S + cs * L::S_STAGE, &tm_scales, &cs_full[cs], col0, 0,
                      srow + kk * 2, pol_stream);
          if (++cs == CS) { cs = 0; cs_ph ^= 1; }
        }
      }
      for (int s = 0; s < CS; ++s)
        if (cs_armed & (1u << s)) mbar_wait(&cs_full[s], (cs_par >> s) & 1, nullptr, a.status);
    }
  } else if (warp == TOKEN_WARP || warp == TOKEN_WARP2) {
    // ---------------- TMA producers: this CTA's token rows ----------------
    // A tile's N rows are UMMA 1's first min(N, 256) and (WIDE) UMMA 2's rest;
    // this CTA loads its half of each part, the second 16 KiB after the
    // first. A full half (128 rows) is one copy, a partial one of nb boxes of
    // 16 rows at most three (64 + 32 + 16 rows). A copy costs its issuing
    // thread about 300 cycles, so two warps split a stage's copies (even and
    // odd positions in the list); TOKEN_WARP also arms the stage's bytes.
    // TOKEN_WARP2 arrives on every stage, with copies or without: a waiter
    // that no barrier waits for could fall a whole phase behind its stage's
    // barrier and then wait on a parity that has already passed.
    if (lane == 0) {
      const int which = warp - TOKEN_WARP;
      const uint64_t pol_keep = policy_evict_last();
      int st = 0;
      uint32_t ph = 0, armed = 0, par = 0;
      bool ok = true;
      int gated = -1;  // last local expert whose rows were seen to have arrived
      for (int idx = cl; idx < total && ok; idx += ncl) {
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
        const int n_all = tile_n(t.rows);
        const int n1 = min(n_all, BT), n2 = n_all - n1;  // n2 > 0 only in WIDE tiles
        const int nb1 = n1 / 2 / T_BOX_ROWS, nb2 = n2 / 2 / T_BOX_ROWS;
        const int rbase1 = t.row0 + (int)rank * (n1 / 2);
        const int rbase2 = t.row0 + n1 + (int)rank * (n2 / 2);
        for (int kk = 0; kk < KT; ++kk) {
          if (!mbar_wait(&empty[st], ph ^ 1, abort_flag, a.status)) {
            ok = false;
            break;
          }
          if (rank == 0 && which == 0)
            mbar_arrive_expect_tx(&full[st], (uint32_t)(2 * (nb1 + nb2) * T_BOX_BYTES));
          armed |= 1u << st;
          par = (par & ~(1u << st)) | (ph << st);
          const uint32_t bar0 = full_0 + (uint32_t)(st * 8);
          uint8_t* tdst = smem + L::OFF_STAGE + st * L::STG + A_STAGE;
          int ci = 0;  // position of the next copy in the stage's list
          auto copy = [&](uint8_t* dst, const CUtensorMap* map, int row) {
            if ((ci++ & 1) == which) tma_load_2d_pair(dst, map, bar0, kk * BK, row, pol_keep);
          };
          auto load_part = [&](uint8_t* dst, int nb, int rbase) {
            if (nb == HALF / T_BOX_ROWS) {
              copy(dst, &tm_lhs_half, rbase);
              return;
            }
            int bx = 0;
            if (nb & 4) {
              copy(dst, &tm_lhs_64, rbase);
              bx += 4;
            }
            if (nb & 2) {
              copy(dst + bx * T_BOX_BYTES, &tm_lhs_32, rbase + bx * T_BOX_ROWS);
              bx += 2;
            }
            if (nb & 1) copy(dst + bx * T_BOX_BYTES, &tm_lhs, rbase + bx * T_BOX_ROWS);
          };
          load_part(tdst, nb1, rbase1);
          if (WIDE && nb2 > 0) load_part(tdst + T_STAGE, nb2, rbase2);
          if (which == 1) mbar_arrive_remote(bar0);
          if (++st == S) { st = 0; ph ^= 1; }
        }
      }
      // Every stage this warp filled is released by the pair's UMMAs (so its
      // copies have landed) before the CTA can exit.
      for (int i = 0; i < S; ++i)
        if (armed & (1u << i)) mbar_wait(&empty[i], (par >> i) & 1, nullptr, a.status);
    }
  } else if (warp == MMA_WARP) {
    // ---------------- UMMA issuer (even CTA) ----------------
    if (rank == 0) {
      // The whole warp runs the loop (warp-uniform operands); one elected
      // lane issues.
      const bool issuer = elect_one();
      int st = 0;
      uint32_t ph = 0;
      AccRing ring;
      bool ok = true;
      for (int idx = cl; idx < total && ok; idx += ncl) {
        const Tile t = get_tile(idx, row_start, tile_prefix, a);
        const int n_all = tile_n(t.rows);
        const int n1 = min(n_all, BT), n2 = n_all - n1;  // n2 > 0 only in WIDE tiles
        const bool both = WIDE && n2 > 0;
        const uint32_t idesc = idesc_bf16(2 * ROWS, n1, false, false);
        const uint32_t idesc2 = idesc_bf16(2 * ROWS, n2 > 0 ? n2 : 32, false, false);
        int sa, sb;
        uint32_t pa, pb;
        ring.take(both, sa, sb, pa, pb);
        bool free_ok = mbar_wait(&acc_empty[sa], pa ^ 1, abort_flag, a.status);
        if (both) free_ok = free_ok && mbar_wait(&acc_empty[sb], pb ^ 1, abort_flag, a.status);
        if (!__all_sync(0xffffffffu, free_ok)) break;
        tc_fence_after();
        const uint32_t d0 = tmem + (uint32_t)(sa * ACC_COLS);
        const uint32_t d1 = tmem + (uint32_t)(sb * ACC_COLS);
        for (int kk = 0; kk < KT; ++kk) {
          if (!__all_sync(0xffffffffu, mbar_wait(&full[st], ph, abort_flag, a.status))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + L::OFF_STAGE + st * L::STG);
          const uint32_t t_base = a_base + A_STAGE;
          if (issuer) {
#pragma unroll
            for (int j = 0; j < BK / 16; ++j) {
              const uint64_t adesc = smem_desc_sw128(a_base + j * 32, 16, 1024);
              umma_pair_bf16(d0, adesc, smem_desc_sw128(t_base + j * 32, 16, 1024), idesc,
                             (kk | j) != 0);
              if (both)  // token rows 256.. into the other slot
                umma_pair_bf16(d1, adesc,
                               smem_desc_sw128(t_base + T_STAGE + j * 32, 16, 1024), idesc2,
                               (kk | j) != 0);
            }
            umma_commit_pair(&empty[st]);
          }
          __syncwarp();
          if (++st == S) { st = 0; ph ^= 1; }
        }
        if (!ok) break;
        if (issuer) {
          umma_commit_pair(&acc_full[sa]);
          if (both) umma_commit_pair(&acc_full[sb]);
        }
        __syncwarp();
      }
      if (issuer) umma_commit_pair(drain_bar);
      __syncwarp();
    }
    // Both CTAs: every UMMA (which writes both TMEMs) completes before TMEM
    // is released.
    if (lane == 0) mbar_wait(drain_bar, 0, nullptr, a.status);
  } else if (warp >= DEC_WARP0) {
    // ---------------- decode ----------------
    // DEC_GROUPS groups of NUM_DEC_WARPS warps take the stages in turn. Warp
    // dw of a group decodes code blocks dw + NUM_DEC_WARPS * i (16 weight
    // columns each) of its stage: lane l decodes word l of each of a block's
    // 4 k-blocks (columns gid, gid+8 of the block, k pairs t, t+4) into A
    // rows p*16 + gid and + 8, where the row block p puts gate block j next to
    // up block j with SwiGLU.
    const int grp = (warp - DEC_WARP0) / NUM_DEC_WARPS;
    const int dw = (warp - DEC_WARP0) % NUM_DEC_WARPS;
    constexpr int es = ScaleTraits<SD>::bytes;
    constexpr int DELTA = decode_delta<SD>();
    const int gid = lane >> 2, tig = lane & 3;
    const DecodeRegs dregs = DecodeRegs::make();  // decode constants held in registers
    // The lane's offset in a row pair of A: row gid of an 8-row swizzle atom,
    // byte 4 tig of a 16-byte chunk, and the atom's XOR phase (gid) in the
    // chunk bits, which the chunk index is XORed into.
    const uint32_t lane_sw = (uint32_t)(gid * 128 + (gid << 4) + 4 * tig);
    uint32_t step = 0;
    bool ok = true;
    for (int idx = cl; idx < total && ok; idx += ncl) {
      for (int kk = 0; kk < KT; ++kk, ++step) {
        if ((int)(step % DEC_GROUPS) != grp) continue;
        const int cs = (int)(step % CS);
        const uint32_t cs_ph = (step / CS) & 1;
        const int st = (int)(step % S);
        const uint32_t ph = (step / S) & 1;
        if (!group_wait(grp, dw, step, &cs_full[cs], cs_ph, &empty[st], ph ^ 1, abort_flag,
                        group_go, a.status)) {
          ok = false;
          break;
        }
        const uint8_t* sstage = smem + L::OFF_S + cs * L::S_STAGE;
        uint8_t* astage = smem + L::OFF_STAGE + st * L::STG;
#pragma unroll
        for (int bi = 0; bi < BLOCKS_PER_WARP; ++bi) {
          const int b = dw + NUM_DEC_WARPS * bi;
          const int p = act ? 2 * (b & 3) + (b >> 2) : b;
          const uint8_t* cstage = smem + L::OFF_C + cs * C_STAGE + b * 512;
          // The codes' loads and table lookups first: they do not wait for
          // the scale multipliers, whose loads and shuffles then overlap them.
          uint32_t tv[4][4];
#pragma unroll
          for (int kb = 0; kb < 4; ++kb)
            tvals_b200(*reinterpret_cast<const uint32_t*>(cstage + kb * 128 + lane * 4), dregs,
                       tv[kb]);
          // The four lanes of a quad (same gid) need the same four scales:
          // k32 half h, column gid + 8c. Lane tig converts scale (h, c) =
          // (tig >> 1, tig & 1) and the quad exchanges the multipliers.
          uint32_t m1s, m2s;
          const bool two = col_mult<SD, DELTA>(
              sstage + ((tig >> 1) * ROWS + 16 * b + gid + 8 * (tig & 1)) * es, m1s, m2s);
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
          // Rows r0 = 16 p + gid and r0 + 8 sit 1 KiB apart in the same
          // swizzle phase (gid), so one XOR of the 16-byte chunk index into
          // the lane's base address serves both (the stage is 1 KiB aligned).
          const uint32_t row_a = smem_u32(astage) + (uint32_t)(2 * p * 1024) + lane_sw;
#pragma unroll
          for (int kb = 0; kb < 4; ++kb) {
            const int h = kb >> 1;
            uint32_t v0 = hmul2_bf16(tv[kb][0], m1[h][0]);
            uint32_t v1 = hmul2_bf16(tv[kb][1], m1[h][1]);
            uint32_t v2 = hmul2_bf16(tv[kb][2], m1[h][0]);
            uint32_t v3 = hmul2_bf16(tv[kb][3], m1[h][1]);
            if (two_any) {
              v0 = hmul2_bf16(v0, m2[h][0]);
              v1 = hmul2_bf16(v1, m2[h][1]);
              v2 = hmul2_bf16(v2, m2[h][0]);
              v3 = hmul2_bf16(v3, m2[h][1]);
            }
            // k pair (16 kb + 2 tig) sits in 16-byte chunk 2 kb, k pair
            // (16 kb + 2 tig + 8) in chunk 2 kb + 1, both at byte 4 tig.
            const int c0 = 2 * kb, c1 = 2 * kb + 1;
            const uint32_t a0 = row_a ^ (uint32_t)(c0 << 4), a1 = row_a ^ (uint32_t)(c1 << 4);
            sts_b32_free(a0, v0);
            sts_b32_free(a0 + 1024, v1);
            sts_b32_free(a1, v2);
            sts_b32_free(a1 + 1024, v3);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&cs_empty[cs]);
          mbar_arrive_remote(full_0 + (uint32_t)(st * 8));
        }
      }
    }
  }

  // Both CTAs are done with every barrier, shared tile and TMEM column.
  tc_fence_before();
  cluster_sync();
  if (a.hk.push_tags != nullptr && threadIdx.x == 0) {
    // Every row this CTA stored precedes (cluster barrier, then an acq_rel
    // ticket at gpu scope) the last CTA's ticket, which precedes its
    // system-scope fence and relaxed add to every rank: one fence covers all
    // CTAs and every rank.
    if (atom_add_acq_rel_gpu(a.hk.ticket, 1u) == gridDim.x - 1) {
      *a.hk.ticket = 0;
      fence_acq_rel_sys();
      for (int p = 0; p < a.hk.world; ++p) red_relaxed_sys_add(a.hk.push_done[p], 1);
    }
  }
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
  cluster_sync();
}

// Largest number of 2-CTA clusters resident at once (one CTA per SM), per
// device (cached; safe to call from several host threads).
template <int SD, bool WIDE>
int max_pairs(cudaLaunchConfig_t cfg) {
  static std::mutex mu;
  static std::map<int, int> cached;  // device -> clusters
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cached.find(dev);
    if (it != cached.end()) return it->second;
  }
  int n = 0;
  cfg.gridDim = dim3(2 * (unsigned)std::max(1, num_sms() / 2));
  cudaError_t e = cudaOccupancyMaxActiveClusters(&n, gmm_pair_kernel<SD, WIDE>, &cfg);
  if (e != cudaSuccess || n < 1) {
    (void)cudaGetLastError();
    n = std::max(1, num_sms() / 2);
  }
  std::lock_guard<std::mutex> lk(mu);
  cached[dev] = n;
  return n;
}

template <int SD, bool WIDE>
int launch(const void* lhs, const void* codes, const void* scales, const int32_t* group_sizes,
           int num_groups, int m, int k, int n, int group_offset, int n_local, int act,
           float limit, int out_dtype, int zero_init, void* out, const EpHooks* hooks,
           int tail_min, int grp_lo, cudaStream_t stream) {
  using L = Layout<SD, WIDE>;
  constexpr int es = ScaleTraits<SD>::bytes;
  const bool act_on = act != DWM_ACT_NONE;
  // Tile indices fit the low kTileBits of a tile_prefix entry.
  DWM_CHECK_ARG((int64_t)(m / BT + n_local + 1) * (n / 256) < (int64_t)kTileMask,
                "m=%d rows over n=%d columns exceed the pair kernel's tile count", m, n);
  CUtensorMap tm_lhs, tm_lhs_32, tm_lhs_64, tm_lhs_half, tm_codes, tm_scales;
  int rc = encode_tmap_2d(&tm_lhs, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, lhs, (uint64_t)k,
                          (uint64_t)m, (uint64_t)k * 2, BK, T_BOX_ROWS,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_tmap_2d(&tm_lhs_32, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, lhs, (uint64_t)k,
                      (uint64_t)m, (uint64_t)k * 2, BK, 2 * T_BOX_ROWS, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_tmap_2d(&tm_lhs_64, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, lhs, (uint64_t)k,
                      (uint64_t)m, (uint64_t)k * 2, BK, 4 * T_BOX_ROWS, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_tmap_2d(&tm_lhs_half, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, lhs, (uint64_t)k,
                      (uint64_t)m, (uint64_t)k * 2, BK, HALF, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  {
    // Codes: rows = 16-column blocks ((k/16)*32 words each); a box is 4
    // consecutive blocks x 2 halves (the up blocks I/16 rows on with SwiGLU,
    // the next 4 blocks without) x one stage of 4 k-blocks.
    const uint64_t row_bytes = (uint64_t)(k / 16) * 128;
    const uint64_t dims[3] = {(uint64_t)(k / 16) * 32, (uint64_t)n_local * (n / 16), 2};
    const uint64_t strides[2] = {row_bytes, act_on ? (uint64_t)(n / 32) * row_bytes : 4 * row_bytes};
    const uint32_t box[3] = {128, 4, 2};
    rc = encode_tmap_nd(&tm_codes, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, codes, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  {
    // Scales [n_local * k/32][n]: 64 columns x the same 2 halves x 2 k32 rows.
    const uint64_t dims[3] = {(uint64_t)n, 2, (uint64_t)n_local * (k / 32)};
    const uint64_t strides[2] = {act_on ? (uint64_t)(n / 2) * es : (uint64_t)64 * es,
                                 (uint64_t)n * es};
    const uint32_t box[3] = {64, 2, 2};
    rc = encode_tmap_nd(&tm_scales, ScaleTraits<SD>::tma, 3, scales, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  rc = set_smem_limit(reinterpret_cast<const void*>(gmm_pair_kernel<SD, WIDE>), L::ALLOC, "gmm pair smem attribute");
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
  a.ldo = act_on ? n / 2 : n;
  a.n_tiles = n / 256;
  a.tail_min = tail_min;
  a.grp_lo = grp_lo;
  a.max_rows = WIDE ? 2 * BT : BT;
  a.status = status_ptr();
  a.hk = hooks ? *hooks : EpHooks{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = L::ALLOC;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(2 * (unsigned)max_pairs<SD, WIDE>(cfg));
  return check_cuda(cudaLaunchKernelEx(&cfg, gmm_pair_kernel<SD, WIDE>, tm_lhs, tm_lhs_32, tm_lhs_64, tm_lhs_half, tm_codes,
                                       tm_scales, a),
                    "gmm_pair launch");
}

}  // namespace gmm_pair

// Entry from the grouped-matmul dispatcher (gmm_fp4.cu): B200-layout weights,
// n a multiple of 256, k of 64; the caller has validated the arguments.
// hooks: expert-parallel gating / push (dwm_ep_gmm_fp4), or nullptr;
// tail_min: Args::tail_min; wide: tiles of up to 512 token rows (Layout);
// grp_lo: Args::grp_lo.
int launch_gmm_pair(const void* lhs, const void* codes, const void* scales, int scale_dtype,
                    const int32_t* group_sizes, int num_groups, int m, int k, int n,
                    int group_offset, int n_local, int act, float limit, int out_dtype,
                    int zero_init, void* out, const EpHooks* hooks, cudaStream_t stream,
                    int tail_min, int wide, int grp_lo) {
#define DWM_PAIR_LAUNCH(SD, W)                                                               \
  gmm_pair::launch<SD, W>(lhs, codes, scales, group_sizes, num_groups, m, k, n, group_offset, \
                          n_local, act, limit, out_dtype, zero_init, out, hooks, tail_min,   \
                          grp_lo, stream)
  if (scale_dtype == DWM_U8) return wide ? DWM_PAIR_LAUNCH(DWM_U8, true) : DWM_PAIR_LAUNCH(DWM_U8, false);
  if (scale_dtype == DWM_BF16)
    return wide ? DWM_PAIR_LAUNCH(DWM_BF16, true) : DWM_PAIR_LAUNCH(DWM_BF16, false);
  return wide ? DWM_PAIR_LAUNCH(DWM_F32, true) : DWM_PAIR_LAUNCH(DWM_F32, false);
#undef DWM_PAIR_LAUNCH
}

}  // namespace dwm
