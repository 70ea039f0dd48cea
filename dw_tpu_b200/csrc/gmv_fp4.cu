// FP4 grouped matmul for decode-sized groups (a few token rows per expert).
//
// At decode, a tcgen05 UMMA of M = 128 weight columns x K = 16 costs about
// 138 cycles whatever its N (measured on B200 for N = 16..256), so with N =
// the 2-16 token rows of an expert it consumes only 1 KiB of FP4 codes per
// 138 cycles: about 2 TB/s across the chip, a third of HBM. This kernel runs
// the same math on mma.sync.m16n8k16 (bf16 in, f32 accumulate): weights are
// decoded straight from the B200 layout into A-fragment registers (one 32-bit
// word per lane per 16x16 block, one PRMT per bf16 pair), token rows are the
// n8 tiles, and nothing decoded touches shared or tensor memory.
//
// The kernel is bound by instruction issue and the integer (ALU) pipe, not
// by the MMA: at the HBM roofline an SM must retire one 32-bit code word (8
// weights) per lane every ~22 issue slots, and the decode alone is 9 ALU
// operations (2 LOP3, 3 SHF, 4 PRMT, with its four constants held in
// registers). So everything else per word is kept off the ALU and small:
//   * E8M0 scales (the common case) are applied to the f32 partial of each
//     32-deep k block after the MMA: the decode yields value * 2^-126
//     (fp4_decode.cuh), the tokens are pre-scaled by 2^80 (exact), and the
//     partial is multiplied by 2^(c-81) (one mad builds the factor): the
//     reference's bf16(value * scale) x bf16 token products (E0901:84-95),
//     exactly, up to the f32 summation order, while |value * token| >= 2^-80
//     (a product value * token * 2^-46 stays a normal f32) and |token| < 2^48
//     (the pre-scaled token stays a finite bf16). A stage holding code 0
//     (scale +0) or a code above 208 instead forms bf16(value * scale) in two exact bf16
//     steps and multiplies the unscaled tokens, the reference's arithmetic
//     (one SWAR test per lane per stage decides). Built with
//     DWM_GMV_POST=0 the fast path instead multiplies each decoded weight
//     register by 2^(c-1-4) in bf16 (exact for codes 1..132; the epilogue
//     removes the 2^-4), about 3% slower.
//   * bf16 / f32 scales (reference: cast to bf16, one bf16 multiply) are
//     multiplied into the decoded weights, which reproduces that rounding.
//   * each warp streams its own tasks through a private ring of S stages of
//     64 or 128 k, filled by three TMA copies per stage issued by lane 0
//     (tokens; the task's 4 column blocks of codes as one 5-D box; their
//     scales as one 3-D box), with prefetch running ahead across task
//     boundaries; token rows land KS/2 + 4 words apart (a box KS + 8 k wide)
//     so B-fragment loads are bank-conflict free with plain offsets.
//   * warps are numbered SM-minor, so the last partial round of tasks is
//     spread one warp per SM.
#include <type_traits>

#include "fp4_decode.cuh"

namespace dwm {
namespace gmv {

using namespace fp4;

constexpr int MAX_GROUPS = 1024;
// Token pre-scale of the post-MMA path, 2^kTokExp: the raw decode is value *
// 2^-126, so products land at value * token * 2^(kTokExp - 126).
constexpr int kTokExp = 80;
constexpr uint32_t kBf16x2_TokScale = (uint32_t)(127 + kTokExp) * 0x00800080u;  // 2^80, both halves
constexpr uint32_t kBf16x2_Norm = (uint32_t)(127 + 126 - kTokExp) * 0x00800080u;  // 2^46
constexpr uint32_t kBf16x2_2p126 = 253u * 0x00800080u;                            // 2^126

// Ring depth per warp (stages of 64 k) for 1 and 2 n8 token tiles.
#ifndef DWM_GMV_STAGES1
#define DWM_GMV_STAGES1 4
#endif
// Ring depth per warp for stages of 128 k (one n8 token tile).
#ifndef DWM_GMV_STAGES1_K128
#define DWM_GMV_STAGES1_K128 2
#endif
// 1: two-tile (16-row) tasks on k % 128 == 0 also take stages of 128 k, with
// DWM_GMV_WARPS2_K128 warps per CTA (measured 17% faster than 64-k stages at
// 32 experts x 512 rows, the per-rank shape of 8 GPUs).
#ifndef DWM_GMV_K128_NT2
#define DWM_GMV_K128_NT2 1
#endif
#ifndef DWM_GMV_WARPS2_K128
#define DWM_GMV_WARPS2_K128 12
#endif
#ifndef DWM_GMV_STAGES2
#define DWM_GMV_STAGES2 3
#endif
// Warps per CTA (E8M0 / bf16 scales; f32 scales take 12).
#ifndef DWM_GMV_WARPS1
#define DWM_GMV_WARPS1 16
#endif
// 1: feed the raw decode (value * 2^-126, a bf16 subnormal for 0.5) to the
// MMA on the E8M0 path; 0: first normalise it by 2^46 (4 more multiplies per
// word, exact either way).
#ifndef DWM_GMV_RAW_TVALS
#define DWM_GMV_RAW_TVALS 1
#endif
// E8M0 scales: 1 = scale the f32 partial of each k32 block after the MMA;
// 0 = multiply each decoded weight register by 2^(c-1-4) in bf16 (exact for
// codes 1..132; the 2^-4 is removed in the epilogue).
#ifndef DWM_GMV_POST
#define DWM_GMV_POST 1
#endif
// 1: one-tile tasks on k % 128 == 0 take stages of 128 k.
#ifndef DWM_GMV_K128
#define DWM_GMV_K128 1
#endif
// 32-row tasks (four n8 token tiles, variant 5): k per stage, ring depth and
// warps per CTA. Their token tile (32 rows) outweighs the codes of a stage.
#ifndef DWM_GMV_KS4
#define DWM_GMV_KS4 64
#endif
#ifndef DWM_GMV_STAGES4
#define DWM_GMV_STAGES4 2
#endif
#ifndef DWM_GMV_WARPS4
#define DWM_GMV_WARPS4 16
#endif
// 1: 128-k launches whose 64-column tasks would give a warp fewer than three
// run half-width tasks (QB = 2); 0 (default): always 64 columns. Measured
// slower at the per-rank shapes of 4 and 8 GPUs (32 experts x 512 rows: gmm1
// 0.187 against 0.163 ms; 64 experts: 0.239 against 0.213): a half-width
// stage carries the same fixed cost for half the words.
#ifndef DWM_GMV_HALF_TASKS
#define DWM_GMV_HALF_TASKS 0
#endif
// 1: 128-k launches with few tasks split each task's k range over a warp pair
// (3-5% faster at the per-rank shapes of 4 and 8 GPUs); 0 (default): every
// task sums its whole k range in one warp, so the expert-parallel layer keeps
// the single-device layer's bits at every rank count (split-K sums the two
// halves of k separately: within 1 bf16 ulp, not bit-equal).
#ifndef DWM_GMV_SPLIT
#define DWM_GMV_SPLIT 0
#endif
// Sleep (ns) of a waiting warp between mbarrier polls (leaving issue slots to
// the warps that have data); 0 = poll.
#ifndef DWM_GMV_BACKOFF
#define DWM_GMV_BACKOFF 0
#endif

// KS: k per ring stage (64 or 128). QB: 16-column code blocks per task, 4 (64
// weight columns: 32 output features with SwiGLU) or 2 (half that: twice the
// tasks, for launches with too few tasks to fill every warp a few times).
template <int SD, int NT, int KS, int QB = 4>
struct Cfg {
  static constexpr int KSTAGE = KS;
  static constexpr int KS16 = KS / 16, KS32 = KS / 32;
  // [QB column blocks (gate ones first with SwiGLU)][KS16 k16 blocks][32
  // words], one TMA copy.
  static constexpr int CODE_BYTES = QB * KS16 * 128;
  // A token row in shared memory: KS + 8 k of bf16, of which the stage uses
  // KS. Rows KS/2 + 4 words apart put the 8 rows of a B-fragment load in 8
  // different bank quads.
  static constexpr int TOK_ROW = 2 * KS + 16;
  // E8M0: scale the f32 partials of each k32 block. Not for 32-row tasks:
  // there the partials would cost 2 * NT multiply-adds per code word and 64
  // registers, against 4 exact bf16 multiplies of the decoded weights.
  static constexpr bool POST = SD == DWM_U8 && DWM_GMV_POST && NT <= 2;
  static constexpr int DELTA = (SD == DWM_U8 && !POST) ? kDelta : 0;  // weight-side bias
  static constexpr int es = ScaleTraits<SD>::bytes;
  static constexpr int S = NT == 4      ? DWM_GMV_STAGES4
                           : KS == 128  ? DWM_GMV_STAGES1_K128
                           : NT == 1    ? DWM_GMV_STAGES1
                                        : DWM_GMV_STAGES2;
  static constexpr bool RAW = DWM_GMV_RAW_TVALS != 0;
  // Largest E8M0 code of the post-MMA path: the k-block factor
  // 2^(c-1-kTokExp) (raw decode) or 2^(c-127) (normalised) must be a finite f32.
  static constexpr uint32_t POST_MAX = POST ? (RAW ? 128u + kTokExp : 254u) : 128u + kDelta;
  static constexpr int TOK = 8 * NT * TOK_ROW;  // token tile: rows of KS + 8 k (KS used)
  // Scales of a stage: [KS32 k32 rows][2 tiles][8 * QB columns], one TMA copy.
  static constexpr int SC_ROW = 16 * QB * es;
  static constexpr int SC = KS32 * SC_ROW;
  static constexpr int WARP_BYTES = (S * (TOK + CODE_BYTES + SC) + 127) & ~127;
  // Split-K warp pairs: 128-k stages, and a token slot that holds a warp's
  // f32 partials (QB * NT quads of registers per lane).
  static constexpr bool SPLIT_OK = KS == 128 && QB * NT * 32 * 16 <= TOK;
  static constexpr int WARPS = NT == 4 ? (SD != DWM_F32 ? DWM_GMV_WARPS4 : 12)
                             : (NT == 2 && KS == 128) ? (SD != DWM_F32 ? DWM_GMV_WARPS2_K128 : 10)
                                                      : (SD != DWM_F32 ? DWM_GMV_WARPS1 : 12);
  static constexpr int OFF_BAR = WARPS * WARP_BYTES;
  // Split-K exchange barriers: [WARPS / 2 pairs][ready, consumed].
  static constexpr int OFF_XBAR = OFF_BAR + WARPS * S * 8;
  static constexpr int OFF_ROWS = OFF_XBAR + WARPS * 8;
  static constexpr int OFF_TASKS = OFF_ROWS + (MAX_GROUPS + 1) * 4;
  static constexpr int BYTES = OFF_TASKS + (MAX_GROUPS + 1) * 4;
  static constexpr int ALLOC = BYTES + 128;  // slack for 128-byte alignment (TMA destinations)
  static constexpr uint32_t TX = TOK + CODE_BYTES + SC;
  static_assert(ALLOC <= 232448, "exceeds the 227 KiB per-CTA shared memory");
  static_assert(TOK % 128 == 0 && CODE_BYTES % 128 == 0 && SC % 128 == 0 && KS32 % 2 == 0,
                "TMA destinations need 128-byte alignment");
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
  int ldo;
  int quads;  // tasks per row chunk: n / (16 * QB)
  int tail_min;  // 0: all rows; > 0: only the rows past a group's last full 256-row tile,
                 // and only if fewer than tail_min (the CTA-pair kernel takes the rest)
  int grp_lo, grp_hi;  // only groups of grp_lo < rows <= grp_hi (variant 10's size classes)
  int ksplit;  // 1, or 2: warp pairs split each task's k range (split-K in the CTA)
  int* status;
  EpHooks hk;  // expert-parallel gating / push (all null for a plain GEMM)
};

// The rows [w0, w0 + wn) of a group starting at row gs0 with gsn rows that
// this launch computes (see Args::tail_min, grp_lo and grp_hi).
__device__ __forceinline__ void row_window(int gs0, int gsn, const Args& a, int& w0, int& wn) {
  const int tail_min = a.tail_min;
  if (gsn <= a.grp_lo || gsn > a.grp_hi) {
    w0 = gs0;
    wn = 0;
    return;
  }
  if (tail_min <= 0) {
    w0 = gs0;
    wn = gsn;
    return;
  }
  const int rem = gsn % 256;
  wn = (rem > 0 && rem < tail_min) ? rem : 0;
  w0 = gs0 + gsn - wn;
}

__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// d = a * b + z, with z a zero quad the caller keeps in registers (the MMA
// reads C as four registers; a literal 0 would be rebuilt for every call).
__device__ __forceinline__ void mma_16816_z(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                            uint32_t b1, const float (&z)[4]) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(z[0]), "f"(z[1]),
        "f"(z[2]), "f"(z[3]));
}

struct Task {
  int g;     // local group
  int quad;  // 64-column task inside the group
  int row0;  // first lhs row of the chunk
  int rows;  // valid rows in the chunk (1..8*NT)
};

template <int NT>
__device__ __forceinline__ Task get_task(int idx, const int* row_start, const int* task_prefix,
                                         const Args& a) {
  int lo = 0, hi = a.n_local;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (task_prefix[mid] <= idx) lo = mid; else hi = mid;
  }
  Task t;
  t.g = lo;
  const int local = idx - task_prefix[lo];
  const int chunk = local / a.quads;
  t.quad = local - chunk * a.quads;
  int gs0, gsn;
  row_window(row_start[a.group_offset + lo],
             row_start[a.group_offset + lo + 1] - row_start[a.group_offset + lo], a, gs0, gsn);
  t.row0 = gs0 + chunk * 8 * NT;
  t.rows = min(8 * NT, gsn - chunk * 8 * NT);
  return t;
}

// First column block of each of the task's two halves of QB/2 blocks:
// adjacent columns, or the gate and up halves for SwiGLU.
template <int QB>
__device__ __forceinline__ void task_blocks(const Task& t, const Args& a, int& cb0, int& cb1) {
  constexpr int HB = QB / 2;
  if (a.act == DWM_ACT_NONE) {
    cb0 = QB * t.quad;
    cb1 = cb0 + HB;
  } else {
    cb0 = HB * t.quad;
    cb1 = a.n / 32 + HB * t.quad;
  }
}

template <int SD, int NT, int KS, int QB, bool SPLIT, bool EP>
__global__ void __launch_bounds__(Cfg<SD, NT, KS, QB>::WARPS * 32, 1)
    gmv_fp4_kernel(const __grid_constant__ CUtensorMap tm_lhs,
                   const __grid_constant__ CUtensorMap tm_codes,
                   const __grid_constant__ CUtensorMap tm_scales, const Args a) {
  using C = Cfg<SD, NT, KS, QB>;
  constexpr int S = C::S;
  constexpr int es = C::es;
  constexpr int KSTAGE = C::KSTAGE, CODE_BYTES = C::CODE_BYTES, TOK_ROW = C::TOK_ROW;
  extern __shared__ uint8_t smem_raw[];
  // 1 KiB alignment by pointer arithmetic on the shared array itself, so the
  // compiler keeps every access below in the shared window (LDS, not LD).
  uint8_t* smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  int* row_start = reinterpret_cast<int*>(smem + C::OFF_ROWS);
  int* task_prefix = reinterpret_cast<int*>(smem + C::OFF_TASKS);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint8_t* tok_s = smem + warp * C::WARP_BYTES;  // [S][TOK]
  uint8_t* code_s = tok_s + S * C::TOK;           // [S][CODE_BYTES]
  uint8_t* sc_s = code_s + S * CODE_BYTES;        // [S][SC]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR) + warp * S;
  // Split-K: warps 2p and 2p+1 take the same tasks, the first half of k and
  // the second; the second hands its f32 partials to the first through
  // shared memory (its just-consumed token slot) behind two mbarriers, and
  // the first adds them (own + partner, a fixed order) and stores.
  static_assert(!SPLIT || C::SPLIT_OK, "split-K needs 128-k stages and room for the partials");
  constexpr int ks = SPLIT ? 2 : 1;  // a.ksplit
  const int kh = SPLIT ? (warp & 1) : 0;
  uint64_t* xbar = reinterpret_cast<uint64_t*>(smem + C::OFF_XBAR) + 2 * (warp >> 1);

  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    if (SPLIT && kh == 0) {
      mbar_init(&xbar[0], 1);  // partials ready (the second warp)
      mbar_init(&xbar[1], 1);  // partials read (the first warp)
    }
    fence_mbar_init();
  }
  if (threadIdx.x == 32) {
    tma_prefetch_desc(&tm_lhs);
    tma_prefetch_desc(&tm_codes);
    tma_prefetch_desc(&tm_scales);
  }
  if (warp == 0) {
    // Row starts over all groups, then the task prefix over local groups.
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
        row_start[g] = min(run, a.m);
        run += max(a.group_sizes[g], 0);
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
      const int g = lane * per2 + i;
      if (g < NL) {
        int w0, rows;
        row_window(row_start[a.group_offset + g],
                   row_start[a.group_offset + g + 1] - row_start[a.group_offset + g], a, w0,
                   rows);
        tsum += ((rows + 8 * NT - 1) / (8 * NT)) * a.quads;
      }
    }
    int tincl = tsum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, tincl, o);
      if (lane >= o) tincl += y;
    }
    int trun = tincl - tsum;
    for (int i = 0; i < per2; ++i) {
      const int g = lane * per2 + i;
      if (g < NL) {
        task_prefix[g] = trun;
        int w0, rows;
        row_window(row_start[a.group_offset + g],
                   row_start[a.group_offset + g + 1] - row_start[a.group_offset + g], a, w0,
                   rows);
        trun += ((rows + 8 * NT - 1) / (8 * NT)) * a.quads;
      }
    }
    if (lane == 31) task_prefix[NL] = trun;
  }
  __syncthreads();
  const int total = task_prefix[a.n_local];

  if (a.zero_init) {
    const int oes = a.out_f32 ? 4 : 2;
    const int lo = row_start[a.group_offset];
    const int hi = row_start[a.group_offset + a.n_local];
    const int64_t n16 = (int64_t)a.ldo * oes / 16;
    const uint4 z = make_uint4(0, 0, 0, 0);
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    uint4* o = reinterpret_cast<uint4*>(a.out);
    for (int64_t i = tid; i < (int64_t)lo * n16; i += stride) o[i] = z;
    for (int64_t i = (int64_t)hi * n16 + tid; i < (int64_t)a.m * n16; i += stride) o[i] = z;
  }

  const int gid = lane >> 2, tig = lane & 3;
  const int NSTAGE = a.k / KSTAGE;
  const int NST = NSTAGE / ks;  // stages of this warp's part of a task
  const DecodeRegs dregs = DecodeRegs::make();
  // Register-held constants of the post-MMA path: the zero quad of the
  // partials' first MMA and the tokens' 2^kTokExp pre-scale.
  const float zq[4] = {__uint_as_float(pin(0u)), __uint_as_float(pin(0u)),
                       __uint_as_float(pin(0u)), __uint_as_float(pin(0u))};
  const uint32_t tok_scale = pin(kBf16x2_TokScale);
  // 2^(c-1-delta) for E8M0 code c, both bf16 halves: c * 0x00800080 + bias.
  const uint32_t wm_bias = pin((126u - C::DELTA) * 0x00800080u);
  const int wstride = gridDim.x * (C::WARPS / ks);
  // Warps (pairs with split-K) numbered SM-minor: the last, partial round of
  // tasks lands on one warp per SM (which then runs with the SM nearly to
  // itself) instead of on every warp of a few SMs.
  const int first = (SPLIT ? warp >> 1 : warp) * gridDim.x + blockIdx.x;

  // ---- producer state (lane 0): the next (task, stage) to fetch ----
  uint64_t pol_stream = 0, pol_keep = 0;
  int iss_idx = first, iss_st = 0, iss_end = NST;
  // Per-task TMA coordinates: token row, the group and the two quad
  // coordinates of the code map (the map's dimensions differ with the
  // activation; the task's quad goes into one of them), the scale map's two
  // column coordinates and the task's first scale row.
  int y_tok = 0, c_g = 0, c_a = 0, c_b = 0, s_x = 0, s_y = 0, y_s = 0;
  int gated = -1;  // expert-parallel gating: last local expert seen complete
  auto set_task = [&](int idx) {
    const Task t = get_task<NT>(idx, row_start, task_prefix, a);
    const bool act = a.act != DWM_ACT_NONE;
    if (EP && a.hk.gate_arrive != nullptr && t.g != gated) {
      // Every source rank's rows of this expert have been stored here (and
      // made visible) before TMA reads them. A wait that runs out reports a
      // timeout; the stages then load whatever has arrived.
      wait_counter_ge(a.hk.gate_arrive + t.g, a.hk.gate_target[t.g], a.hk.wait_ns, a.status);
      fence_proxy_async_all();
      gated = t.g;
    }
    y_tok = t.row0;
    c_g = t.g;
    if constexpr (QB == 4) {
      c_a = act ? t.quad : 0;
      c_b = act ? 0 : t.quad;
      s_x = act ? 32 * t.quad : 0;
      s_y = act ? 0 : 2 * t.quad;
    } else {  // the maps of launch_impl for QB = 2
      c_a = t.quad;
      c_b = 0;
      s_x = act ? 16 * t.quad : 0;
      s_y = act ? 0 : t.quad;
    }
    y_s = t.g * (a.k / 32);
    iss_st = kh * NST;
    iss_end = iss_st + NST;
  };
  uint32_t issued = 0;  // stages issued so far (ring sequence)
  auto issue_one = [&]() {
    const int slot = (int)(issued % S);
    uint64_t* bar = &bars[slot];
    mbar_arrive_expect_tx(bar, C::TX);
    const int xc = iss_st * C::KS16 * 32;
    tma_load_2d(tok_s + slot * C::TOK, &tm_lhs, bar, iss_st * KSTAGE, y_tok, pol_keep);
    tma_load_5d(code_s + slot * CODE_BYTES, &tm_codes, bar, xc, 0, c_a, c_b, c_g, pol_stream);
    tma_load_3d(sc_s + slot * C::SC, &tm_scales, bar, s_x, s_y, y_s + C::KS32 * iss_st,
                pol_stream);
    ++issued;
    if (++iss_st == iss_end) {
      iss_idx += wstride;
      if (iss_idx < total) set_task(iss_idx);
    }
  };
  if (lane == 0 && first < total) {
    pol_stream = policy_evict_first();
    pol_keep = policy_evict_last();
    set_task(first);
    while (issued < (uint32_t)S && iss_idx < total) issue_one();
  }
  __syncwarp();

  uint32_t seq = 0;  // stages consumed
  bool ok = true;
  uint32_t tcount = 0;  // tasks done (the exchange barriers' phase)
  for (int idx = first; idx < total && ok; idx += wstride, ++tcount) {
    const Task t = get_task<NT>(idx, row_start, task_prefix, a);
    int cb0, cb1;
    task_blocks<QB>(t, a, cb0, cb1);

    float acc[QB][NT][4];
#pragma unroll
    for (int i = 0; i < QB; ++i)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][nt][e] = 0.0f;

    for (int st = 0; st < NST; ++st, ++seq) {
      const int slot = (int)(seq % S);
      const bool got =
          mbar_wait<DWM_GMV_BACKOFF>(&bars[slot], (seq / S) & 1, nullptr, a.status);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      const uint8_t* tok = tok_s + slot * C::TOK;
      const uint8_t* code = code_s + slot * CODE_BYTES;
      const uint8_t* sc = sc_s + slot * C::SC;
      // PRE: multiply the decoded weights by their scale in bf16 (the
      // reference's rounding; bf16/f32 scales, or E8M0 codes outside the
      // post-MMA range) and the tokens as they are, else scale the f32
      // partial of each k32 block.
      auto stage = [&](auto pre_tag) {
        constexpr bool PRE = decltype(pre_tag)::value;
        constexpr uint32_t M1 = C::POST ? kBf16x2_2p126 : pow2_126_minus_delta_x2<C::DELTA>();
#pragma unroll
        for (int h = 0; h < C::KS32; ++h) {  // 32-deep k block inside the stage
          // Scales of the lane's columns: block i, column gid (+8 for hc =
          // 1); a k32 row holds the task's 16 * QB columns, block i's at
          // 16 i.
          uint32_t wm[QB][2];
          float post[QB][2];
#pragma unroll
          for (int i = 0; i < QB; ++i)
#pragma unroll
            for (int hc = 0; hc < 2; ++hc) {
              const uint8_t* p = sc + h * C::SC_ROW + (i * 16 + gid + 8 * hc) * es;
              uint32_t c;
              if constexpr (SD == DWM_U8)
                c = *p;
              else if constexpr (SD == DWM_BF16)
                c = *reinterpret_cast<const uint16_t*>(p);
              else
                c = f32_to_bf16_bits(*reinterpret_cast<const float*>(p));
              if constexpr (PRE) {
                wm[i][hc] = SD == DWM_U8 ? (c << 7) * 0x10001u  // bf16 2^(c-127), 0 -> +0
                                         : c * 0x10001u;        // the bf16 scale
              } else if constexpr (!C::POST) {
                asm("mad.lo.u32 %0, %1, 8388736, %2;"  // c * 0x00800080 + bias
                    : "=r"(wm[i][hc])
                    : "r"(c), "r"(wm_bias));
              } else {
                post[i][hc] = C::RAW ? __uint_as_float(c * 0x00800000u +  // 2^(c-1-kTokExp)
                                                       ((uint32_t)(126 - kTokExp) << 23))
                                     : __uint_as_float(c << 23);  // 2^(c-127)
              }
            }
          float part[QB][NT][4];
#pragma unroll
          for (int kk2 = 0; kk2 < 2; ++kk2) {
            const int kk = 2 * h + kk2;  // k16 block inside the stage
            // B fragments. Rows past the task (other groups' tokens or the
            // tile's zero fill) only reach output columns that are not stored.
            uint32_t b[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              // token row nt*8 + gid: k pairs 16 kk + 2 tig and + 8
              const uint8_t* row = tok + (nt * 8 + gid) * TOK_ROW + kk * 32 + 4 * tig;
              uint32_t b0 = *reinterpret_cast<const uint32_t*>(row);
              uint32_t b1 = *reinterpret_cast<const uint32_t*>(row + 16);
              if constexpr (C::POST && !PRE) {
                b0 = hmul2_bf16(b0, tok_scale);
                b1 = hmul2_bf16(b1, tok_scale);
              }
              b[nt][0] = b0;
              b[nt][1] = b1;
            }
#pragma unroll
            for (int i = 0; i < QB; ++i) {
              const uint32_t w =
                  *reinterpret_cast<const uint32_t*>(code + i * (C::KS16 * 128) + kk * 128 + lane * 4);
              uint32_t af[4];
              tvals_b200(w, dregs, af);
              if constexpr (PRE) {
                af[0] = hmul2_bf16(hmul2_bf16(af[0], M1), wm[i][0]);
                af[1] = hmul2_bf16(hmul2_bf16(af[1], M1), wm[i][1]);
                af[2] = hmul2_bf16(hmul2_bf16(af[2], M1), wm[i][0]);
                af[3] = hmul2_bf16(hmul2_bf16(af[3], M1), wm[i][1]);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma_16816(acc[i][nt], af, b[nt][0], b[nt][1]);
              } else if constexpr (!C::POST) {  // one exact multiply per register
                af[0] = hmul2_bf16(af[0], wm[i][0]);
                af[1] = hmul2_bf16(af[1], wm[i][1]);
                af[2] = hmul2_bf16(af[2], wm[i][0]);
                af[3] = hmul2_bf16(af[3], wm[i][1]);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma_16816(acc[i][nt], af, b[nt][0], b[nt][1]);
              } else {
                if constexpr (!C::RAW) {
#pragma unroll
                  for (int j = 0; j < 4; ++j) af[j] = hmul2_bf16(af[j], kBf16x2_Norm);
                }
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                  if (kk2 == 0)
                    mma_16816_z(part[i][nt], af, b[nt][0], b[nt][1], zq);
                  else
                    mma_16816(part[i][nt], af, b[nt][0], b[nt][1]);
                }
              }
            }
          }
          if constexpr (!PRE && C::POST) {
#pragma unroll
            for (int i = 0; i < QB; ++i)
#pragma unroll
              for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  acc[i][nt][e] = fmaf(part[i][nt][e], post[i][e >> 1], acc[i][nt][e]);
          }
        }
      };
      if constexpr (SD == DWM_U8) {
        // One check per stage for the whole warp: each lane tests SC / 128 of
        // the stage's SC / 4 scale words; the fast path needs every code in
        // [1, POST_MAX].
        uint32_t bad = 0;
#pragma unroll
        for (int q = 0; q < C::SC / 128; ++q) {
          const uint32_t v = *reinterpret_cast<const uint32_t*>(sc + (q * 32 + lane) * 4);
          const uint32_t zero_byte = (v - 0x01010101u) & ~v & 0x80808080u;
          uint32_t high_byte;
          if constexpr (C::POST_MAX >= 128u && C::POST_MAX < 255u)
            // a byte > POST_MAX: bit 7 set and low 7 bits + (255 - POST_MAX) >= 128
            high_byte = ((v & 0x7F7F7F7Fu) + (255u - C::POST_MAX) * 0x01010101u) & v &
                        0x80808080u;
          else  // a byte == 255
            high_byte = (~v - 0x01010101u) & v & 0x80808080u;
          bad |= zero_byte | high_byte;
        }
        if (__any_sync(0xffffffffu, bad != 0u))
          stage(std::true_type{});
        else
          stage(std::false_type{});
      } else {
        stage(std::true_type{});
      }
      __syncwarp();  // every lane is done with this slot
      // The second warp of a split pair keeps its last slot for the hand-over.
      const bool keep = SPLIT && kh == 1 && st == NST - 1;
      if (!keep && lane == 0 && iss_idx < total) issue_one();
      __syncwarp();
    }
    if (!ok) break;
    if constexpr (SPLIT) {
      // Hand-over area: the second warp's slot of its last stage (both warps
      // of the pair have consumed the same number of stages).
      const int xslot = (int)((seq - 1) % S);
      float4* xb = reinterpret_cast<float4*>(smem + (warp | 1) * C::WARP_BYTES + xslot * C::TOK);
      const uint32_t xph = tcount & 1;
      if (kh == 1) {
#pragma unroll
        for (int i = 0; i < QB; ++i)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            xb[(i * NT + nt) * 32 + lane] =
                make_float4(acc[i][nt][0], acc[i][nt][1], acc[i][nt][2], acc[i][nt][3]);
        fence_proxy_async_smem();  // before this warp's next TMA into the slot
        __syncwarp();
        if (lane == 0) mbar_arrive(&xbar[0]);
        const bool got = mbar_wait<DWM_GMV_BACKOFF>(&xbar[1], xph, nullptr, a.status);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        if (lane == 0 && iss_idx < total) issue_one();
        __syncwarp();
        continue;  // the first warp stores the task
      }
      const bool got = mbar_wait<DWM_GMV_BACKOFF>(&xbar[0], xph, nullptr, a.status);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int i = 0; i < QB; ++i)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float4 v = xb[(i * NT + nt) * 32 + lane];
          acc[i][nt][0] += v.x;
          acc[i][nt][1] += v.y;
          acc[i][nt][2] += v.z;
          acc[i][nt][3] += v.w;
        }
      fence_proxy_async_smem();  // these reads before the partner's TMA into the slot
      __syncwarp();
      if (lane == 0) mbar_arrive(&xbar[1]);
    }

    // Epilogue: c0,c1 = (column gid, tokens 2t, 2t+1), c2,c3 = (column gid+8, ...);
    // kAccScale removes the weight-side 2^-delta exactly.
    constexpr float kAccScale = (float)(1 << C::DELTA);
    int colbase[QB];
#pragma unroll
    for (int i = 0; i < QB; ++i) colbase[i] = 16 * (i < QB / 2 ? cb0 + i : cb1 + i - QB / 2);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int r = nt * 8 + 2 * tig + e;
        if (r >= t.rows) continue;
        const int64_t row = t.row0 + r;
        if (a.act == DWM_ACT_NONE) {
          // Expert parallel: straight into the token owner's buffer, at the
          // row of its (token, k) pair (over NVLink for a peer).
          void* obase = a.out;
          int64_t orow = row;
          if (EP && a.hk.push_tags != nullptr) {
            const int tag = a.hk.push_tags[row];
            if (tag < 0) continue;
            obase = a.hk.push_base[tag >> kEpTagBits];
            orow = tag & ((1 << kEpTagBits) - 1);
          }
#pragma unroll
          for (int i = 0; i < QB; ++i) {
#pragma unroll
            for (int hc = 0; hc < 2; ++hc) {
              const float v = acc[i][nt][hc * 2 + e] * kAccScale;
              const int64_t off = orow * a.ldo + colbase[i] + gid + 8 * hc;
              if (a.out_f32)
                reinterpret_cast<float*>(obase)[off] = v;
              else
                reinterpret_cast<uint16_t*>(obase)[off] = (uint16_t)f32_to_bf16_bits(v);
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < QB / 2; ++i) {
#pragma unroll
            for (int hc = 0; hc < 2; ++hc) {
              float g = acc[i][nt][hc * 2 + e] * kAccScale;
              float u = acc[i + QB / 2][nt][hc * 2 + e] * kAccScale;
              if (a.act == DWM_ACT_SWIGLU_CLAMP) {
                g = fminf(g, a.limit);
                u = fminf(fmaxf(u, -a.limit), a.limit);
              }
              const float hv = g * sigmoid_fast(g) * u;
              const int64_t off = row * a.ldo + colbase[i] + gid + 8 * hc;
              if (a.out_f32)
                reinterpret_cast<float*>(a.out)[off] = hv;
              else
                reinterpret_cast<uint16_t*>(a.out)[off] = (uint16_t)f32_to_bf16_bits(hv);
            }
          }
        }
      }
    }
  }
  // On abort, let every copy this warp issued land before the CTA can exit.
  if (!ok && lane == 0) {
    for (uint32_t q = seq; q < issued; ++q)
      mbar_wait(&bars[q % S], (q / S) & 1, nullptr, a.status);
  }
  if (EP && a.hk.push_tags != nullptr) {
    // Every row this CTA stored precedes (bar.sync, then an acq_rel ticket at
    // gpu scope) the last CTA's ticket, which precedes its system-scope fence
    // and relaxed add to every rank: one fence covers all CTAs and ranks.
    __syncthreads();
    if (threadIdx.x == 0 && atom_add_acq_rel_gpu(a.hk.ticket, 1u) == gridDim.x - 1) {
      *a.hk.ticket = 0;
      fence_acq_rel_sys();
      for (int p = 0; p < a.hk.world; ++p) red_relaxed_sys_add(a.hk.push_done[p], 1);
    }
  }
}

template <int SD, int NT, int KS, int QB = 4>
int launch_impl(const void* lhs, const void* codes, const void* scales, Args a,
                cudaStream_t stream) {
  using C = Cfg<SD, NT, KS, QB>;
  a.quads = a.n / (16 * QB);
  // Split-K warp pairs when the launch has too few tasks to give every warp
  // several (the last, partial round of tasks then dominates): each task's
  // two halves run concurrently, so a round costs half a task.
  a.ksplit = (DWM_GMV_SPLIT && C::SPLIT_OK && (a.k / KS) % 2 == 0 && C::WARPS % 2 == 0 &&
              (int64_t)a.n_local * a.quads < 4LL * num_sms() * C::WARPS)
                 ? 2
                 : 1;
  CUtensorMap tm_lhs, tm_codes, tm_scales;
  // lhs [m, k] bf16: box of KS + 8 k (KS used) x 8*NT rows, rows TOK_ROW bytes apart.
  int rc = encode_tmap_2d(&tm_lhs, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, lhs, (uint64_t)a.k,
                          (uint64_t)a.m, (uint64_t)a.k * 2, C::TOK_ROW / 2, 8 * NT,
                          CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  // codes: one row of (k/16) x 32 words per column block, n/16 rows per
  // group (R bytes each). One 5-D box holds the task's 4 column blocks as
  // two pairs: with SwiGLU the gate pair (blocks 2q, 2q+1) and the up pair
  // (n/32 blocks later); otherwise blocks 4q .. 4q+3. Dimensions: word,
  // block in pair, then (quad, half) or (half, quad), group.
  const bool act = a.act != DWM_ACT_NONE;
  const uint64_t R = (uint64_t)(a.k / 16) * 128;
  const uint64_t cw = (uint64_t)(a.k / 16) * 32, q64 = (uint64_t)a.n / 64, G = a.n_local;
  if (QB == 4) {
    const uint64_t dims[5] = {cw, 2, act ? q64 : 2, act ? 2 : q64, G};
    const uint64_t strides[4] = {R, 2 * R, act ? (uint64_t)(a.n / 32) * R : 4 * R,
                                 (uint64_t)(a.n / 16) * R};
    const uint32_t box[5] = {(uint32_t)(C::KS16 * 32), 2, act ? 1u : 2u, act ? 2u : 1u, 1};
    rc = encode_tmap_nd(&tm_codes, CU_TENSOR_MAP_DATA_TYPE_UINT32, 5, codes, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  } else {
    // Two blocks per task, coordinates (word, 0, task, 0, group): with SwiGLU
    // gate block `task` and its up block n/32 later, else blocks 2 task and
    // 2 task + 1. Dimensions of one are placeholders.
    const uint64_t q32 = (uint64_t)a.n / 32;
    const uint64_t dims[5] = {cw, act ? 1u : 2u, q32, act ? 2u : 1u, G};
    const uint64_t strides[4] = {R, act ? R : 2 * R, act ? q32 * R : q32 * 2 * R,
                                 (uint64_t)(a.n / 16) * R};
    const uint32_t box[5] = {(uint32_t)(C::KS16 * 32), act ? 1u : 2u, 1, act ? 2u : 1u, 1};
    rc = encode_tmap_nd(&tm_codes, CU_TENSOR_MAP_DATA_TYPE_UINT32, 5, codes, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  // scales [n_local * k/32, n]: one 3-D box of 32 columns x 2 tiles x KS32
  // k32 rows; the tiles are the gate and up halves (n/2 apart) with SwiGLU,
  // else two adjacent 32-column groups.
  {
    // QB = 2: 16 columns x (gate, up) with SwiGLU, else one 32-column group.
    constexpr uint64_t es = ScaleTraits<SD>::bytes;
    const uint64_t dims[3] = {act ? (uint64_t)a.n / 2 : 32, act ? 2 : (uint64_t)a.n / 32,
                              G * (a.k / 32)};
    const uint64_t strides[2] = {act ? (uint64_t)a.n / 2 * es : 32 * es, (uint64_t)a.n * es};
    const uint32_t box[3] = {act ? (uint32_t)(8 * QB) : 32u, act ? 2u : (uint32_t)(QB / 2),
                             (uint32_t)C::KS32};
    rc = encode_tmap_nd(&tm_scales, ScaleTraits<SD>::tma, 3, scales, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  // Expert-parallel hooks (their own instance, so the plain kernel keeps its
  // registers), or split-K pairs, or neither.
  const bool ep = a.hk.gate_arrive != nullptr || a.hk.push_tags != nullptr;
  if (ep) a.ksplit = 1;
  auto kernel = ep ? gmv_fp4_kernel<SD, NT, KS, QB, false, true>
                   : gmv_fp4_kernel<SD, NT, KS, QB, false, false>;
  if constexpr (C::SPLIT_OK)
    if (a.ksplit == 2) kernel = gmv_fp4_kernel<SD, NT, KS, QB, true, false>;
  rc = set_smem_limit(reinterpret_cast<const void*>(kernel), C::ALLOC, "gmv smem attribute");
  if (rc) return rc;
  kernel<<<num_sms(), C::WARPS * 32, C::ALLOC, stream>>>(tm_lhs, tm_codes, tm_scales, a);
  return check_cuda(cudaGetLastError(), "gmv_fp4 launch");
}

}  // namespace gmv

// Decode-regime grouped GEMM on the B200 layout (called by the dwm_gmm_fp4
// dispatcher after argument validation: k % 64 == 0, n % 256 == 0, 16-byte
// aligned pointers). nt: 1, 2 or 4 n8 token tiles per task (8, 16 or 32
// token rows; every weight is decoded once per task). hooks: expert-parallel
// gating / push (dwm_ep_gmm_fp4), or nullptr.
int launch_gmv(const void* lhs, const void* codes, const void* scales, int scale_dtype,
               const int32_t* group_sizes, int num_groups, int m, int k, int n, int group_offset,
               int n_local, int act, float limit, int out_dtype, int zero_init, void* out, int nt,
               cudaStream_t stream, int tail_min, int grp_lo, int grp_hi, const EpHooks* hooks) {
  gmv::Args a;
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
  a.quads = n / 64;
  a.tail_min = tail_min;
  a.grp_lo = grp_lo;
  a.grp_hi = grp_hi;
  a.ksplit = 1;
  a.status = status_ptr();
  a.hk = hooks ? *hooks : EpHooks{};
#define DWM_GMV(SD, NT) return gmv::launch_impl<SD, NT, 64>(lhs, codes, scales, a, stream)
  // Half-width tasks (QB = 2) when 64-column tasks, one per local group and
  // column quad, would not give every warp of the grid three.
  auto half_tasks = [&](int warps) {
    return DWM_GMV_HALF_TASKS && (int64_t)n_local * (n / 64) < 3LL * num_sms() * warps;
  };
#define DWM_GMV_K128_BY_QB(SD, NT)                                                       \
  do {                                                                                    \
    if (half_tasks(gmv::Cfg<SD, NT, 128, 2>::WARPS))                                      \
      return gmv::launch_impl<SD, NT, 128, 2>(lhs, codes, scales, a, stream);             \
    return gmv::launch_impl<SD, NT, 128, 4>(lhs, codes, scales, a, stream);               \
  } while (0)
  if (nt <= 1 && k % 128 == 0 && DWM_GMV_K128) {
    if (scale_dtype == DWM_U8) DWM_GMV_K128_BY_QB(DWM_U8, 1);
    if (scale_dtype == DWM_BF16) DWM_GMV_K128_BY_QB(DWM_BF16, 1);
    DWM_GMV_K128_BY_QB(DWM_F32, 1);
  }
  if (nt <= 1) {
    if (scale_dtype == DWM_U8) DWM_GMV(DWM_U8, 1);
    if (scale_dtype == DWM_BF16) DWM_GMV(DWM_BF16, 1);
    DWM_GMV(DWM_F32, 1);
  }
  if (nt == 2 && DWM_GMV_K128_NT2 && k % 128 == 0) {
    if (scale_dtype == DWM_U8) DWM_GMV_K128_BY_QB(DWM_U8, 2);
    if (scale_dtype == DWM_BF16) DWM_GMV_K128_BY_QB(DWM_BF16, 2);
    DWM_GMV_K128_BY_QB(DWM_F32, 2);
  }
  if (nt == 4) {
    if (scale_dtype == DWM_U8)
      return gmv::launch_impl<DWM_U8, 4, DWM_GMV_KS4>(lhs, codes, scales, a, stream);
    if (scale_dtype == DWM_BF16)
      return gmv::launch_impl<DWM_BF16, 4, DWM_GMV_KS4>(lhs, codes, scales, a, stream);
    return gmv::launch_impl<DWM_F32, 4, DWM_GMV_KS4>(lhs, codes, scales, a, stream);
  }
  if (scale_dtype == DWM_U8) DWM_GMV(DWM_U8, 2);
  if (scale_dtype == DWM_BF16) DWM_GMV(DWM_BF16, 2);
  DWM_GMV(DWM_F32, 2);
#undef DWM_GMV
#undef DWM_GMV_K128_BY_QB
}

}  // namespace dwm
