// Expert-parallel token exchange for sm_100a over NVLink peer memory: the
// one-shot dispatch and combine that replace the reference's all-gather +
// per-shard sort (X0101:56-104, X0107:34-51) and its masked combine +
// reduce-scatter (X0107:15-29, KO:167-185).
//
// One process per GPU. Every rank owns one device allocation with the same
// layout (the "symmetric" buffer), exports it as a CUDA IPC handle, and maps
// every peer's; kernels then load and store peer memory over NVLink.
//
//   dispatch  one kernel of one CTA per SM. Every CTA histograms all of the
//             rank's (token, k) expert ids in shared memory (so no CTA waits
//             on another CTA of its grid). The first CTA to start publishes
//             the per-expert counts into every peer's count table as 64-bit
//             (epoch << 32 | count) words, which need no fence or flag.
//             Each CTA then waits for the peers' counts of this epoch, forms
//             the receive offsets, and stores the rows of its own slice of
//             pairs straight into the owners' receive buffers (the whole CTA
//             on a few rows, loads batched ahead of the stores). The CTA that
//             finishes last (a ticket) bumps every peer's arrival counter
//             once and waits until all ranks have bumped its own.
//   combine   one kernel. The first CTA to start announces that this rank's
//             expert outputs (the symmetric output buffer, written by the
//             preceding grouped matmul) are ready; every CTA waits for the
//             peers' announcements, then forms each token's k-order f32
//             weighted sum, loading each (token, k) row straight from the
//             owner's output buffer at the row the dispatch sent it to (the
//             single-device combine's arithmetic, bit for bit).
//
// The phases can also be issued as separate launches (DWM_EP_COUNTS, _ROWS,
// _WAIT; DWM_EP_PUSH, _REDUCE), which the single-GPU emulation of several
// ranks needs: there every rank's earlier phase runs before any later one.
//
// Receive order: rank r's rows are expert-major over its experts
// [r*E/n, (r+1)*E/n), and inside an expert ordered by (source rank, source
// token, k slot): the rows the reference's global stable argsort over the
// rank-major gathered batch keeps on rank r (X0101:56-104). A pair's row is
//   sum of all ranks' counts of the owner's earlier experts
//   + sum of lower ranks' counts of its expert
//   + its rank among the source's own pairs of that expert (stable).
//
// Waits are bounded (2 s by default, dwm_ep_set_wait_limit; then
// DWM_DEV_TIMEOUT in the status word and the kernel winds down). Every wait depends only on kernels of other ranks or of
// earlier launches, never on a particular CTA of the same grid: the counts are
// published by whichever CTA starts first, and only the last CTA to finish
// waits for the arrivals. Counters are monotonic and tagged with a
// per-rank epoch that lives in device memory (the dispatch advances it), so
// nothing is reset between steps and a captured CUDA graph of the exchange
// replays with a fresh epoch each time.
//
// Reuse across steps is safe without extra barriers: a rank starts its next
// dispatch only after its combine has read every peer's outputs, and a peer
// overwrites its receive rows, counts or outputs only after that next
// dispatch's counts from this rank have reached it.
#include <cstring>
#include <type_traits>
#include <new>

#include "moe_common.cuh"

namespace dwm {
namespace ep {

constexpr int MAX_WORLD = 8;
constexpr int XFER_THREADS = 512;  // dispatch CTA size (one CTA per SM)
constexpr int COPY_DEPTH = 8;      // 16-byte row loads in flight per dispatch thread
constexpr int COMBINE_THREADS = 128;
constexpr int ROW_BITS = 28;    // sent-row code: owner << ROW_BITS | row
constexpr int64_t MAX_CAP = 1LL << ROW_BITS;

struct Layout {  // byte offsets inside every rank's symmetric buffer
  size_t ready;      // uint32 [MAX_WORLD]: epoch whose outputs source s has made readable
  size_t arrive;     // uint64: dispatch arrivals (one per rank and epoch, monotonic)
  size_t delivered;  // uint64: ranks whose gmm2 pushed this rank's outputs (monotonic)
  size_t counts;     // uint64 [MAX_WORLD][E]: (epoch << 32) | count of expert x from source s
  size_t exp_arrive; // uint64 [E/world]: rows of each local expert received (monotonic)
  size_t tags;       // int32 [cap]: source rank << ROW_BITS | source pair of each received row
  size_t recv;       // bf16 [cap][H]: received rows, expert-major
  size_t outb;       // [cap][H], 4-byte capacity: expert outputs of the received rows, or
                     // (pushed mode) this rank's own pairs' outputs, row = pair
  size_t total;
};

// Per-rank control words (ordinary device memory, not shared with peers),
// followed by the per-local-expert arrival targets (uint64 [E/world]).
enum Ctl {
  CTL_EPOCH = 0, CTL_FIRST = 1, CTL_DONE = 2, CTL_RECV_ROWS = 3, CTL_GEMM_TICKET = 4,
  CTL_PUSH_STEPS = 5, CTL_WORDS = 6
};

struct Params {
  uint8_t* peer[MAX_WORLD];
  Layout L;
  int rank, world, E, LE, H, topk, T;
  int64_t cap;
  int32_t* sent;  // [max_pairs]: owner << ROW_BITS | row of each own pair, -1 if dropped
  uint32_t* ctl;  // [CTL_WORDS]
  uint64_t* target;  // [E/world]: rows each local expert must have received (monotonic)
  uint64_t wait_ns;  // limit of every device-side wait (dwm_ep_set_wait_limit)
};

// Bounded spin until *p >= target (32-bit epoch flag); gives up after `limit`
// ns (DWM_DEV_TIMEOUT).
__device__ __forceinline__ bool wait_flag(const uint32_t* p, uint32_t target, uint64_t limit,
                                          int* status) {
  if (ld_acquire_sys(p) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    __nanosleep(32);
    if (ld_acquire_sys(p) >= target) return true;
    if ((i & 63u) == 0 && globaltimer_ns() - t0 > limit) {
      report(status, DWM_DEV_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ bool wait_count(const uint64_t* p, uint64_t target, uint64_t limit,
                                           int* status) {
  if (ld_acquire_sys64(p) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    __nanosleep(32);
    if (ld_acquire_sys64(p) >= target) return true;
    if ((i & 63u) == 0 && globaltimer_ns() - t0 > limit) {
      report(status, DWM_DEV_TIMEOUT);
      return false;
    }
  }
}

// Bounded spin until the tagged count word carries `epoch`; its count or -1.
__device__ __forceinline__ int wait_tagged(const uint64_t* p, uint32_t epoch, uint64_t limit,
                                          int* status) {
  uint64_t v = ld_relaxed_sys64(p);
  if ((uint32_t)(v >> 32) == epoch) return (int)(uint32_t)v;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    __nanosleep(32);
    v = ld_relaxed_sys64(p);
    if ((uint32_t)(v >> 32) == epoch) return (int)(uint32_t)v;
    if ((i & 63u) == 0 && globaltimer_ns() - t0 > limit) {
      report(status, DWM_DEV_TIMEOUT);
      return -1;
    }
  }
}

__device__ __forceinline__ uint64_t* count_word(const Params& P, int rank_mem, int src, int x) {
  return reinterpret_cast<uint64_t*>(P.peer[rank_mem] + P.L.counts) + (size_t)src * P.E + x;
}

// Dynamic shared memory of the dispatch kernel (ints): tot, run, col, scan,
// dest, run0 [E] each, then the chunk's experts and rows [XFER_THREADS] each.
inline size_t dispatch_smem_bytes(int e) { return (size_t)(6 * e + 2 * XFER_THREADS) * 4; }

// Exclusive scan of in[0, n) into out by warp 0 (chunked per lane).
__device__ __forceinline__ void warp0_exclusive_scan(const int* in, int* out, int n) {
  const int lane = threadIdx.x & 31;
  if (threadIdx.x >= 32) return;
  const int per = (n + 31) / 32;
  int sum = 0;
  for (int i = 0; i < per; ++i) {
    const int x = lane * per + i;
    if (x < n) sum += in[x];
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
    if (x < n) {
      out[x] = run;
      run += in[x];
    }
  }
}

// The dispatch (phases: DWM_EP_COUNTS | DWM_EP_ROWS | DWM_EP_WAIT; with
// DWM_EP_GATED each row also carries its tag, and each CTA adds the rows it
// stored for every expert to the owner's arrival counter of that expert, so
// the owner's grouped matmul can start on an expert as soon as its rows are in).
__global__ void __launch_bounds__(XFER_THREADS)
    ep_dispatch_kernel(const __grid_constant__ Params P, const uint4* __restrict__ hidden,
                       const int32_t* __restrict__ ids, int32_t* recv_group_sizes, int ph,
                       int* status) {
  extern __shared__ int sm[];
  int* tot = sm;                 // this rank's count of each expert
  int* run = sm + P.E;           // count of each expert in pairs before the chunk
  int* col = sm + 2 * P.E;       // all ranks' count of each expert
  int* scan = sm + 3 * P.E;      // exclusive scan of col
  int* dest = sm + 4 * P.E;      // first receive row of this rank's pairs of each expert
  int* run0 = sm + 5 * P.E;      // run before this CTA's slice (gated arrivals)
  int* cx = sm + 6 * P.E;        // chunk: expert of each pair (-1: dropped)
  int* crow = cx + XFER_THREADS; // chunk: receive row of each pair (-1: dropped)
  __shared__ uint32_t s_epoch;
  __shared__ int s_first, s_last, s_fail;
  const int tid = threadIdx.x;
  const int n = P.T * P.topk;
  const bool counts = ph & DWM_EP_COUNTS, rows = ph & DWM_EP_ROWS;
  const bool gated = ph & DWM_EP_GATED;
  if (tid == 0) {
    s_epoch = P.ctl[CTL_EPOCH] + (counts ? 1u : 0u);
    s_first = counts ? atomicAdd(&P.ctl[CTL_FIRST], 1u) == 0u : 0;
    s_fail = 0;
  }
  for (int x = tid; x < 2 * P.E; x += blockDim.x) sm[x] = 0;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int slice = (n + gridDim.x - 1) / gridDim.x;
  const int j0 = min(n, (int)blockIdx.x * slice), j1 = min(n, j0 + slice);

  if (counts || rows) {
    for (int j = tid; j < n; j += blockDim.x) {
      const int x = ids[j];
      if (x < 0 || x >= P.E) {
        if (blockIdx.x == 0) report(status, DWM_DEV_BAD_INDEX);
        continue;
      }
      atomicAdd(&tot[x], 1);
      if (j < j0) atomicAdd(&run[x], 1);
    }
    __syncthreads();
  }
  if (s_first) {  // publish this rank's counts to every rank (itself included)
    for (int i = tid; i < P.world * P.E; i += blockDim.x) {
      const int p = i / P.E, x = i - p * P.E;
      st_relaxed_sys64(count_word(P, p, P.rank, x), ((uint64_t)epoch << 32) | (uint32_t)tot[x]);
    }
  }
  if (rows) {
    for (int x = tid; x < P.E; x += blockDim.x) {
      int c = 0, b = 0;
      for (int s = 0; s < P.world; ++s) {
        int v = tot[x];
        if (s != P.rank) {
          v = wait_tagged(count_word(P, P.rank, s, x), epoch, P.wait_ns, status);
          if (v < 0) {
            s_fail = 1;
            v = 0;
          }
        }
        c += v;
        if (s < P.rank) b += v;
      }
      col[x] = c;
      dest[x] = b;
    }
    __syncthreads();
    warp0_exclusive_scan(col, scan, P.E);
    __syncthreads();
    for (int x = tid; x < P.E; x += blockDim.x) {
      const int owner = x / P.LE;
      dest[x] += scan[x] - scan[owner * P.LE];
      run0[x] = run[x];
      if (blockIdx.x == 0 && owner == P.rank) {
        recv_group_sizes[x - owner * P.LE] = col[x];
        if (gated) P.target[x - owner * P.LE] += (uint64_t)col[x];
      }
    }
    if (blockIdx.x == 0 && tid == 0) {
      const int last = (P.rank + 1) * P.LE - 1;
      P.ctl[CTL_RECV_ROWS] = (uint32_t)(scan[last] + col[last] - scan[P.rank * P.LE]);
    }
    __syncthreads();
    const int h16 = P.H / 8;
    for (int c0 = j0; c0 < j1 && !s_fail; c0 += blockDim.x) {
      const int cn = min((int)blockDim.x, j1 - c0);
      if (tid < cn) {
        const int x = ids[c0 + tid];
        cx[tid] = (x < 0 || x >= P.E) ? -1 : x;
      }
      __syncthreads();
      if (tid < cn) {
        const int x = cx[tid];
        int row = -1;
        if (x >= 0) {
          int r = run[x];
          for (int u = 0; u < tid; ++u) r += cx[u] == x;
          row = dest[x] + r;
          if (row >= P.cap) {
            report(status, DWM_DEV_OVERFLOW);
            row = -1;
          }
        }
        crow[tid] = row;
        P.sent[c0 + tid] = row < 0 ? -1 : ((x / P.LE) << ROW_BITS) | row;
        if (gated && row >= 0)  // the owner's gmm2 sends this row's output back to pair c0+tid
          reinterpret_cast<int32_t*>(P.peer[x / P.LE] + P.L.tags)[row] =
              (P.rank << ROW_BITS) | (c0 + tid);
      }
      __syncthreads();
      if (tid < cn && cx[tid] >= 0) atomicAdd(&run[cx[tid]], 1);
      // Copy the chunk's rows: 16-byte units, COPY_DEPTH loads in flight per
      // thread ahead of the stores.
      const int units = cn * h16;
      for (int u0 = tid; u0 < units; u0 += COPY_DEPTH * blockDim.x) {
        uint4 v[COPY_DEPTH];
        uint4* to[COPY_DEPTH];
#pragma unroll
        for (int q = 0; q < COPY_DEPTH; ++q) {
          const int u = u0 + q * blockDim.x;
          to[q] = nullptr;
          if (u < units) {
            const int p = u / h16, c = u - p * h16;
            const int row = crow[p];
            if (row >= 0) {
              v[q] = __ldg(hidden + (int64_t)((c0 + p) / P.topk) * h16 + c);
              to[q] = reinterpret_cast<uint4*>(P.peer[cx[p] / P.LE] + P.L.recv) +
                      (int64_t)row * h16 + c;
            }
          }
        }
#pragma unroll
        for (int q = 0; q < COPY_DEPTH; ++q)
          if (to[q]) *to[q] = v[q];
      }
      __syncthreads();
    }
    if (s_fail)  // counts never came: this slice's pairs are dropped
      for (int j = j0 + tid; j < j1; j += blockDim.x) P.sent[j] = -1;
    if (gated && !s_fail) {
      // Every thread's row and tag stores precede (bar.sync) each release:
      // one system-scope add per (CTA, expert) publishes this CTA's rows.
      __syncthreads();
      for (int x = tid; x < P.E; x += blockDim.x) {
        const int d = run[x] - run0[x];
        if (d > 0) {
          const int owner = x / P.LE;
          red_release_sys_add(
              reinterpret_cast<uint64_t*>(P.peer[owner] + P.L.exp_arrive) + (x - owner * P.LE),
              (uint64_t)d);
        }
      }
    }
  }
  __syncthreads();
  // The last CTA to finish: reset the tickets, advance the epoch, signal the
  // peers once, and wait for all of them. Ordering: every CTA's row stores
  // precede (bar.sync, then an acq_rel ticket at gpu scope) the last CTA's
  // ticket, which precedes its system-scope fence and the relaxed adds after
  // it (a release pattern per peer), which the peers' acquire observes;
  // causality order is transitive across the two scopes, so one fence covers
  // all CTAs' stores and every peer.
  if (tid == 0) {
    s_last = atom_add_acq_rel_gpu(&P.ctl[CTL_DONE], 1u) == gridDim.x - 1;
    if (s_last) {
      P.ctl[CTL_DONE] = 0;
      P.ctl[CTL_FIRST] = 0;
      if (counts) P.ctl[CTL_EPOCH] = epoch;
      if (rows) {
        fence_acq_rel_sys();
        for (int p = 0; p < P.world; ++p)
          red_relaxed_sys_add(reinterpret_cast<uint64_t*>(P.peer[p] + P.L.arrive), 1);
      }
      if (ph & DWM_EP_WAIT)
        wait_count(reinterpret_cast<const uint64_t*>(P.peer[P.rank] + P.L.arrive),
                   (uint64_t)epoch * P.world, P.wait_ns, status);
    }
  }
}

// Copy the received rows' outputs y -> the symmetric output buffer (only when
// the caller's y is not that buffer).
__global__ void ep_stage_kernel(const __grid_constant__ Params P, const uint4* __restrict__ y,
                                int row_bytes) {
  uint4* to = reinterpret_cast<uint4*>(P.peer[P.rank] + P.L.outb);
  const int64_t units = (int64_t)P.ctl[CTL_RECV_ROWS] * (row_bytes / 16);
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < units;
       u += (int64_t)gridDim.x * blockDim.x)
    to[u] = __ldg(y + u);
}

// The combine (phases: DWM_EP_PUSH = announce outputs, DWM_EP_REDUCE):
// out[t] = sum_k y(t, k) * w[t, k] in k order (f32, from +0.0). A thread owns
// 8 consecutive elements of one token and keeps up to KB of its rows' loads in
// flight: the rows on this rank are loaded before the wait for the peers'
// announcements, the peers' rows after it.
template <int XD, int WD, int OD, bool RANK_ORDER>
__global__ void __launch_bounds__(COMBINE_THREADS)
    ep_combine_kernel(const __grid_constant__ Params P, const void* __restrict__ w,
                      void* __restrict__ out, const moe::SharedAdd sa, int ph, int* status) {
  constexpr int KB = 8;
  constexpr int ROW_MASK = (1 << ROW_BITS) - 1;
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  const int tid = threadIdx.x;
  const bool pushed = ph & DWM_EP_PUSHED;
  if (tid == 0) {
    s_epoch = P.ctl[CTL_EPOCH];
    s_ok = 1;
    // Pushed mode: every rank's gmm2 has stored its outputs of this rank's
    // pairs here once `delivered` has grown by world this step.
    if (pushed && (ph & DWM_EP_REDUCE) &&
        !wait_counter_ge(reinterpret_cast<const uint64_t*>(P.peer[P.rank] + P.L.delivered),
                         (uint64_t)(P.ctl[CTL_PUSH_STEPS] + 1) * P.world, P.wait_ns, status))
      s_ok = 0;
    // The outputs were written by earlier kernels on this stream: one
    // system-scope fence, then a relaxed flag store per peer, publishes them.
    if ((ph & DWM_EP_PUSH) && atomicAdd(&P.ctl[CTL_FIRST], 1u) == 0u) {
      fence_acq_rel_sys();
      for (int p = 0; p < P.world; ++p)
        st_relaxed_sys(reinterpret_cast<uint32_t*>(P.peer[p] + P.L.ready) + P.rank, P.ctl[CTL_EPOCH]);
    }
  }
  __syncthreads();
  if (ph & DWM_EP_REDUCE) {
    const int h8 = P.H / 8;
    const int64_t total = (int64_t)P.T * h8;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + tid;
    const int64_t t = i / h8;
    const int c = (int)(i - t * h8);
    const bool mine = i < total;
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.0f;
    for (int k0 = 0; k0 < P.topk || k0 == 0; k0 += KB) {
      // Rows in flight: packed bf16 (4 registers each) or f32 (8).
      using Row = std::conditional_t<XD == DWM_BF16, uint4, float[8]>;
      Row v[KB];
      int code[KB] = {};
      auto load = [&](int q) {
        // Pulled: the owner's output row; pushed: this rank's row of the pair.
        const uint8_t* base = pushed ? P.peer[P.rank] + P.L.outb
                                     : P.peer[code[q] >> ROW_BITS] + P.L.outb;
        const int64_t row = pushed ? t * P.topk + k0 + q : (int64_t)(code[q] & ROW_MASK);
        const int64_t off = row * P.H + (int64_t)c * 8;
        if constexpr (XD == DWM_BF16)
          v[q] = moe::load8_bf16_raw_cg(base, off);
        else
          moe::load8_cg<XD>(base, off, v[q]);
      };
#pragma unroll
      for (int q = 0; q < KB; ++q)
        code[q] = mine && k0 + q < P.topk ? __ldg(P.sent + t * P.topk + k0 + q) : -1;
#pragma unroll
      for (int q = 0; q < KB; ++q)
        if (code[q] >= 0 && (pushed || (code[q] >> ROW_BITS) == P.rank)) load(q);
      if (k0 == 0 && !pushed) {  // the peers' outputs: wait once for their announcements
        if (tid < P.world && tid != P.rank &&
            !wait_flag(reinterpret_cast<const uint32_t*>(P.peer[P.rank] + P.L.ready) + tid,
                       s_epoch, P.wait_ns, status))
          s_ok = 0;
        __syncthreads();
      }
      if (!s_ok) break;
#pragma unroll
      for (int q = 0; q < KB; ++q)
        if (code[q] >= 0 && !pushed && (code[q] >> ROW_BITS) != P.rank) load(q);
      if constexpr (RANK_ORDER) {
        // The reference's GMM_EP numerics (X0107:15-29 then KO:181-184):
        // rank r's masked f32 partial over the k slots of its experts, in k
        // order from +0.0 (a masked slot adds +0.0), then the partials summed
        // in rank order 0..world-1. All k rows are in v (top_k <= KB).
        float prod[KB][8];
#pragma unroll
        for (int q = 0; q < KB; ++q) {
          const float wk = code[q] >= 0 ? moe::load_weight<WD>(w, t * P.topk + q) : 0.0f;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            float y;
            if constexpr (XD == DWM_BF16) {
              const uint32_t u = (e >> 1) == 0   ? v[q].x
                                 : (e >> 1) == 1 ? v[q].y
                                 : (e >> 1) == 2 ? v[q].z
                                                 : v[q].w;
              y = __uint_as_float((e & 1) ? (u & 0xFFFF0000u) : (u << 16));
            } else {
              y = v[q][e];
            }
            prod[q][e] = code[q] >= 0 ? __fmul_rn(y, wk) : 0.0f;
          }
        }
        for (int r = 0; r < P.world; ++r) {
          float part[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) part[e] = 0.0f;
#pragma unroll
          for (int q = 0; q < KB; ++q) {
            if (q >= P.topk) break;  // the reference's partial runs over the k slots only
            const bool own = code[q] >= 0 && (code[q] >> ROW_BITS) == r;
#pragma unroll
            for (int e = 0; e < 8; ++e) part[e] = __fadd_rn(part[e], own ? prod[q][e] : 0.0f);
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] = r == 0 ? part[e] : __fadd_rn(acc[e], part[e]);
        }
      } else {
#pragma unroll
        for (int q = 0; q < KB; ++q)
          if (code[q] >= 0) {
            const float wk = moe::load_weight<WD>(w, t * P.topk + k0 + q);
            if constexpr (XD == DWM_BF16)
              moe::mul_add8_bf16raw(acc, v[q], wk);
            else
              moe::mul_add8(acc, v[q], wk);
          }
      }
    }
    if (mine && s_ok) {
      moe::shared_add8(acc, sa, t * P.H + (int64_t)c * 8);
      moe::store8<OD>(out, t * P.H + (int64_t)c * 8, acc);
    }
  }
  __syncthreads();
  if (tid == 0 && atomicAdd(&P.ctl[CTL_DONE], 1u) == gridDim.x - 1) {
    __threadfence();
    P.ctl[CTL_DONE] = 0;
    P.ctl[CTL_FIRST] = 0;
    if (pushed && (ph & DWM_EP_REDUCE)) P.ctl[CTL_PUSH_STEPS] += 1;
  }
}

}  // namespace ep
}  // namespace dwm

using namespace dwm;
using dwm::ep::MAX_WORLD;

struct dwm_ep {
  int rank, world, max_tokens, hidden, topk, num_experts, local_experts, device;
  int64_t cap, max_pairs;
  ep::Layout L;
  uint8_t* base = nullptr;     // own symmetric buffer
  int32_t* scratch = nullptr;  // sent [max_pairs], the control words, then targets [E/world]
  size_t target_off = 0;       // byte offset of the targets inside scratch
  uint8_t* peer[MAX_WORLD] = {};
  bool peer_ipc[MAX_WORLD] = {};
  bool connected = false;
  bool dispatched = false;  // a COUNTS phase was issued (host-side state check only)
  int last_t = -1;          // tokens of the current dispatch
  uint64_t wait_ns = kWaitLimitNs;  // device-side wait limit
};

namespace {

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

ep::Params make_params(const dwm_ep* c) {
  ep::Params P;
  for (int i = 0; i < MAX_WORLD; ++i) P.peer[i] = c->peer[i];
  P.L = c->L;
  P.rank = c->rank;
  P.world = c->world;
  P.E = c->num_experts;
  P.LE = c->local_experts;
  P.H = c->hidden;
  P.topk = c->topk;
  P.T = c->last_t < 0 ? 0 : c->last_t;
  P.cap = c->cap;
  P.wait_ns = c->wait_ns;
  P.sent = c->scratch;
  P.ctl = reinterpret_cast<uint32_t*>(c->scratch + c->max_pairs);
  P.target = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(c->scratch) + c->target_off);
  return P;
}

int check_ctx(const dwm_ep* c) {
  if (!c) return set_error(DWM_ERR_INVALID, "NULL ep context");
  if (!c->connected) return set_error(DWM_ERR_STATE, "ep context not connected");
  int dev = -1;
  cudaGetDevice(&dev);
  if (dev != c->device)
    return set_error(DWM_ERR_STATE, "current device %d is not the context's device %d", dev,
                     c->device);
  return DWM_OK;
}

}  // namespace

extern "C" int dwm_ep_create(int rank, int world, int max_tokens, int hidden, int topk,
                             int num_experts, dwm_ep** out) {
  DWM_CHECK_ARG(out, "NULL output pointer");
  *out = nullptr;
  DWM_CHECK_ARG(world >= 1 && world <= MAX_WORLD, "world=%d out of [1, %d]", world, MAX_WORLD);
  DWM_CHECK_ARG(rank >= 0 && rank < world, "rank=%d out of [0, %d)", rank, world);
  DWM_CHECK_ARG(num_experts >= 1 && num_experts <= 1024 && num_experts % world == 0,
                "num_experts=%d must be in [1, 1024] and divisible by world=%d", num_experts,
                world);
  DWM_CHECK_ARG(hidden > 0 && hidden % 8 == 0, "hidden=%d must be a positive multiple of 8",
                hidden);
  DWM_CHECK_ARG(topk >= 1 && max_tokens >= 1, "bad topk=%d / max_tokens=%d", topk, max_tokens);
  const int64_t max_pairs = (int64_t)max_tokens * topk;
  const int64_t cap = max_pairs * world;
  DWM_CHECK_ARG(cap <= ep::MAX_CAP, "max_tokens * topk * world above %lld",
                (long long)ep::MAX_CAP);
  dwm_ep* c = new (std::nothrow) dwm_ep();
  if (!c) return set_error(DWM_ERR_INVALID, "out of host memory");
  c->rank = rank;
  c->world = world;
  c->max_tokens = max_tokens;
  c->hidden = hidden;
  c->topk = topk;
  c->num_experts = num_experts;
  c->local_experts = num_experts / world;
  c->max_pairs = max_pairs;
  c->cap = cap;
  cudaGetDevice(&c->device);
  ep::Layout& L = c->L;
  L.ready = 0;
  L.arrive = 64;
  L.delivered = 72;
  L.counts = 128;
  L.exp_arrive = align_up(L.counts + (size_t)MAX_WORLD * num_experts * 8, 256);
  L.tags = align_up(L.exp_arrive + (size_t)c->local_experts * 8, 256);
  L.recv = align_up(L.tags + (size_t)cap * 4, 256);
  L.outb = align_up(L.recv + (size_t)cap * hidden * 2, 256);
  L.total = align_up(L.outb + (size_t)cap * hidden * 4, 256);
  int rc = check_cuda(cudaMalloc(&c->base, L.total), "ep symmetric buffer");
  if (!rc) rc = check_cuda(cudaMemset(c->base, 0, L.recv), "ep header clear");
  c->target_off = align_up((size_t)(max_pairs + ep::CTL_WORDS) * 4, 8);
  const size_t scratch_bytes = c->target_off + (size_t)c->local_experts * 8;
  if (!rc) rc = check_cuda(cudaMalloc(&c->scratch, scratch_bytes), "ep scratch");
  if (!rc)
    rc = check_cuda(cudaMemset(reinterpret_cast<uint8_t*>(c->scratch) + (size_t)max_pairs * 4, 0,
                               scratch_bytes - (size_t)max_pairs * 4),
                    "ep control clear");
  if (!rc) rc = check_cuda(cudaDeviceSynchronize(), "ep create");
  if (rc) {
    if (c->base) cudaFree(c->base);
    if (c->scratch) cudaFree(c->scratch);
    delete c;
    return rc;
  }
  c->peer[rank] = c->base;
  *out = c;
  return DWM_OK;
}

extern "C" int dwm_ep_ipc_handle(dwm_ep* c, void* handle) {
  DWM_CHECK_ARG(c && handle, "NULL pointer");
  cudaIpcMemHandle_t h;
  int rc = check_cuda(cudaIpcGetMemHandle(&h, c->base), "cudaIpcGetMemHandle");
  if (rc) return rc;
  static_assert(sizeof(cudaIpcMemHandle_t) == DWM_EP_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  return DWM_OK;
}

extern "C" int dwm_ep_connect(dwm_ep* c, const void* handles) {
  DWM_CHECK_ARG(c && handles, "NULL pointer");
  if (c->connected) return set_error(DWM_ERR_STATE, "ep context already connected");
  const uint8_t* hb = static_cast<const uint8_t*>(handles);
  for (int p = 0; p < c->world; ++p) {
    if (p == c->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hb + (size_t)p * DWM_EP_HANDLE_BYTES, sizeof(h));
    void* ptr = nullptr;
    int rc = check_cuda(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess),
                        "cudaIpcOpenMemHandle");
    if (rc) {
      for (int q = 0; q < p; ++q)
        if (c->peer_ipc[q]) {
          cudaIpcCloseMemHandle(c->peer[q]);
          c->peer_ipc[q] = false;
          c->peer[q] = nullptr;
        }
      return rc;
    }
    c->peer[p] = static_cast<uint8_t*>(ptr);
    c->peer_ipc[p] = true;
  }
  c->connected = true;
  return DWM_OK;
}

extern "C" int dwm_ep_connect_local(dwm_ep* c, dwm_ep* const* ranks) {
  DWM_CHECK_ARG(c && ranks, "NULL pointer");
  if (c->connected) return set_error(DWM_ERR_STATE, "ep context already connected");
  for (int p = 0; p < c->world; ++p) {
    const dwm_ep* o = ranks[p];
    DWM_CHECK_ARG(o && o->rank == p && o->world == c->world && o->num_experts == c->num_experts &&
                      o->hidden == c->hidden && o->topk == c->topk &&
                      o->max_tokens == c->max_tokens && o->device == c->device,
                  "context %d does not match (rank, world, shape, device)", p);
  }
  for (int p = 0; p < c->world; ++p) c->peer[p] = ranks[p]->base;
  c->connected = true;
  return DWM_OK;
}

extern "C" int dwm_ep_recv_buffer(dwm_ep* c, void** recv, int64_t* capacity_rows) {
  DWM_CHECK_ARG(c && recv && capacity_rows, "NULL pointer");
  *recv = c->base + c->L.recv;
  *capacity_rows = c->cap;
  return DWM_OK;
}

extern "C" int dwm_ep_output_buffer(dwm_ep* c, void** y, int64_t* capacity_rows) {
  DWM_CHECK_ARG(c && y && capacity_rows, "NULL pointer");
  *y = c->base + c->L.outb;
  *capacity_rows = c->cap;
  return DWM_OK;
}

extern "C" int dwm_ep_dispatch(dwm_ep* c, const void* hidden, const int32_t* topk_ids,
                               int num_tokens, int32_t* recv_group_sizes, int phases,
                               void* stream) {
  int rc = check_ctx(c);
  if (rc) return rc;
  DWM_CHECK_ARG(phases >= 1 && phases <= (DWM_EP_ALL | DWM_EP_GATED) &&
                    phases != DWM_EP_GATED,
                "phases=%d", phases);
  DWM_CHECK_ARG(num_tokens >= 0 && num_tokens <= c->max_tokens,
                "num_tokens=%d out of [0, max_tokens=%d]", num_tokens, c->max_tokens);
  DWM_CHECK_ARG(num_tokens == 0 || (hidden && topk_ids), "NULL input");
  DWM_CHECK_ARG(moe::aligned16(hidden), "hidden must be 16-byte aligned");
  if (phases & DWM_EP_COUNTS) {
    c->dispatched = true;
    c->last_t = num_tokens;
  }
  if (!c->dispatched) return set_error(DWM_ERR_STATE, "dispatch phases before COUNTS");
  if (phases & DWM_EP_ROWS) {
    DWM_CHECK_ARG(num_tokens == c->last_t, "num_tokens=%d differs from the COUNTS phase (%d)",
                  num_tokens, c->last_t);
    DWM_CHECK_ARG(recv_group_sizes, "NULL recv_group_sizes");
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned grid = (phases & DWM_EP_ROWS) ? (unsigned)num_sms() : 1;
  ep::ep_dispatch_kernel<<<grid, ep::XFER_THREADS, ep::dispatch_smem_bytes(c->num_experts), s>>>(
      make_params(c), static_cast<const uint4*>(hidden), topk_ids, recv_group_sizes, phases,
      status_ptr());
  return check_cuda(cudaGetLastError(), "ep dispatch launch");
}

extern "C" int dwm_ep_combine_shared(dwm_ep* c, const void* y, int y_dtype,
                                     const void* topk_weights, int w_dtype, const void* shared,
                                     int shared_dtype, float routed_scale, int mid_dtype,
                                     void* out, int out_dtype, int phases, void* stream) {
  int rc = check_ctx(c);
  if (rc) return rc;
  DWM_CHECK_ARG(phases >= 1 &&
                    phases <= (DWM_EP_PUSH | DWM_EP_REDUCE | DWM_EP_PUSHED | DWM_EP_RANK_ORDER) &&
                    (phases & (DWM_EP_PUSH | DWM_EP_REDUCE)) != 0,
                "phases=%d", phases);
  DWM_CHECK_ARG(!(phases & DWM_EP_RANK_ORDER) || (c->topk <= 8 && !(phases & DWM_EP_PUSHED) &&
                                                  shared == nullptr),
                "the rank-order combine takes top_k <= 8, the pulled exchange and no shared "
                "expert");
  DWM_CHECK_ARG(!(phases & DWM_EP_PUSHED) || !(phases & DWM_EP_PUSH),
                "PUSH (announce) has no part in the pushed mode");
  DWM_CHECK_ARG(c->dispatched, "combine before any dispatch");
  DWM_CHECK_ARG(y_dtype == DWM_BF16 || y_dtype == DWM_F32, "y dtype must be bf16 or f32");
  DWM_CHECK_ARG(w_dtype == DWM_BF16 || w_dtype == DWM_F32, "weight dtype must be bf16 or f32");
  DWM_CHECK_ARG(out_dtype == DWM_BF16 || out_dtype == DWM_F32, "out dtype must be bf16 or f32");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const ep::Params P = make_params(c);
  const bool reduce = phases & DWM_EP_REDUCE;
  if ((phases & DWM_EP_PUSH) && !(phases & DWM_EP_PUSHED)) {
    DWM_CHECK_ARG(y && moe::aligned16(y), "y must be a 16-byte aligned device pointer");
    if (y != c->base + c->L.outb) {
      const int row_bytes = c->hidden * (y_dtype == DWM_F32 ? 4 : 2);
      const unsigned g = moe::grid_for(c->cap * (row_bytes / 16), 256, 4);
      ep::ep_stage_kernel<<<g, 256, 0, s>>>(P, static_cast<const uint4*>(y), row_bytes);
      rc = check_cuda(cudaGetLastError(), "ep stage launch");
      if (rc) return rc;
    }
  }
  if (reduce) {
    DWM_CHECK_ARG(P.T == 0 || (topk_weights && out), "NULL weights or out");
    DWM_CHECK_ARG(moe::aligned16(out), "out must be 16-byte aligned");
    DWM_CHECK_ARG(shared == nullptr || ((shared_dtype == DWM_BF16 || shared_dtype == DWM_F32) &&
                                        (mid_dtype == DWM_BF16 || mid_dtype == DWM_F32) &&
                                        moe::aligned16(shared)),
                  "shared partial: bf16/f32, 16-byte aligned; mid dtype bf16/f32");
  }
  const moe::SharedAdd sa{reduce ? shared : nullptr, shared_dtype == DWM_F32, routed_scale,
                          mid_dtype == DWM_BF16};
  // One thread per 8 elements of a token (no grid-stride loop).
  const int64_t threads = (int64_t)P.T * (c->hidden / 8);
  const unsigned grid =
      reduce && threads > 0 ? (unsigned)((threads + ep::COMBINE_THREADS - 1) / ep::COMBINE_THREADS)
                            : 1;
  int* st = status_ptr();
  const bool ro = phases & DWM_EP_RANK_ORDER;
#define DWM_EP_COMBINE_CASE(XD, WD, OD)                                                        \
  if (y_dtype == XD && w_dtype == WD && out_dtype == OD) {                                     \
    if (ro)                                                                                    \
      ep::ep_combine_kernel<XD, WD, OD, true>                                                  \
          <<<grid, ep::COMBINE_THREADS, 0, s>>>(P, topk_weights, out, sa, phases, st);         \
    else                                                                                       \
      ep::ep_combine_kernel<XD, WD, OD, false>                                                 \
          <<<grid, ep::COMBINE_THREADS, 0, s>>>(P, topk_weights, out, sa, phases, st);         \
    return check_cuda(cudaGetLastError(), "ep combine launch");                                \
  }
  DWM_EP_COMBINE_CASE(DWM_BF16, DWM_BF16, DWM_BF16)
  DWM_EP_COMBINE_CASE(DWM_BF16, DWM_F32, DWM_BF16)
  DWM_EP_COMBINE_CASE(DWM_F32, DWM_BF16, DWM_BF16)
  DWM_EP_COMBINE_CASE(DWM_F32, DWM_F32, DWM_BF16)
  DWM_EP_COMBINE_CASE(DWM_BF16, DWM_BF16, DWM_F32)
  DWM_EP_COMBINE_CASE(DWM_BF16, DWM_F32, DWM_F32)
  DWM_EP_COMBINE_CASE(DWM_F32, DWM_BF16, DWM_F32)
  DWM_EP_COMBINE_CASE(DWM_F32, DWM_F32, DWM_F32)
#undef DWM_EP_COMBINE_CASE
  return DWM_OK;
}

extern "C" int dwm_ep_combine(dwm_ep* c, const void* y, int y_dtype, const void* topk_weights,
                              int w_dtype, void* out, int out_dtype, int phases, void* stream) {
  return dwm_ep_combine_shared(c, y, y_dtype, topk_weights, w_dtype, nullptr, DWM_F32, 1.0f,
                               DWM_BF16, out, out_dtype, phases, stream);
}

namespace dwm {
int launch_gmm_pair(const void* lhs, const void* codes, const void* scales, int scale_dtype,
                    const int32_t* group_sizes, int num_groups, int m, int k, int n,
                    int group_offset, int n_local, int act, float limit, int out_dtype,
                    int zero_init, void* out, const EpHooks* hooks, cudaStream_t stream,
                    int tail_min, int wide, int grp_lo);
int launch_gmv(const void* lhs, const void* codes, const void* scales, int scale_dtype,
               const int32_t* group_sizes, int num_groups, int m, int k, int n, int group_offset,
               int n_local, int act, float limit, int out_dtype, int zero_init, void* out, int nt,
               cudaStream_t stream, int tail_min, int grp_lo, int grp_hi, const EpHooks* hooks);
int launch_gmm_single_ep(const void* lhs, const void* codes, const void* scales, int scale_dtype,
                         const int32_t* group_sizes, int num_groups, int m, int k, int n,
                         int act, float limit, int out_dtype, void* out, const EpHooks* hooks,
                         cudaStream_t stream);
}

extern "C" int dwm_ep_gmm_fp4(dwm_ep* c, const void* lhs, const void* codes, int codes_format,
                              const void* scales, int scale_dtype,
                              const int32_t* recv_group_sizes, int k, int n, int act,
                              float act_limit, int out_dtype, void* out, int mode, int variant,
                              void* stream) {
  int rc = check_ctx(c);
  if (rc) return rc;
  DWM_CHECK_ARG(mode == DWM_EP_GEMM_GATED || mode == DWM_EP_GEMM_PUSH, "mode=%d", mode);
  DWM_CHECK_ARG(variant == 1 || variant == 3 || variant == 4 || variant == 5 || variant == 7 ||
                    variant == 9,
                "the EP grouped matmul runs variant 1 (tcgen05, one CTA), 3 / 4 / 5 (mma.sync "
                "decode kernel, 8 / 16 / 32-row tiles), 7 (CTA pairs) or 9 (CTA pairs, 512-row "
                "tiles)");
  DWM_CHECK_ARG(codes_format == DWM_FP4_B200, "the EP grouped matmul takes the B200 layout");
  DWM_CHECK_ARG(scale_dtype == DWM_U8 || scale_dtype == DWM_BF16 || scale_dtype == DWM_F32,
                "scale dtype must be u8 (e8m0), bf16 or f32");
  DWM_CHECK_ARG(out_dtype == DWM_BF16 || out_dtype == DWM_F32, "out dtype must be bf16 or f32");
  DWM_CHECK_ARG(act == DWM_ACT_NONE || act == DWM_ACT_SWIGLU || act == DWM_ACT_SWIGLU_CLAMP,
                "unknown activation %d", act);
  DWM_CHECK_ARG(k > 0 && n > 0 && k % 64 == 0 && n % 256 == 0,
                "k=%d (multiple of 64) n=%d (multiple of 256)", k, n);
  DWM_CHECK_ARG(lhs && codes && scales && recv_group_sizes, "NULL pointer");
  DWM_CHECK_ARG(moe::aligned16(lhs) && moe::aligned16(codes) && moe::aligned16(scales),
                "pointers must be 16-byte aligned");
  EpHooks hk{};
  hk.wait_ns = c->wait_ns;
  hk.world = c->world;
  const ep::Params P = make_params(c);
  void* dst = out;
  if (mode == DWM_EP_GEMM_GATED) {
    DWM_CHECK_ARG(lhs == c->base + c->L.recv && k == c->hidden,
                  "the gated grouped matmul reads the receive buffer (k = hidden)");
    DWM_CHECK_ARG(out && moe::aligned16(out), "out must be a 16-byte aligned device pointer");
    hk.gate_arrive = reinterpret_cast<const uint64_t*>(c->base + c->L.exp_arrive);
    hk.gate_target = P.target;
  } else {
    DWM_CHECK_ARG(act == DWM_ACT_NONE && n == c->hidden,
                  "the pushing grouped matmul is the down projection (no activation, n = "
                  "hidden)");
    hk.push_tags = reinterpret_cast<const int32_t*>(c->base + c->L.tags);
    for (int p = 0; p < c->world; ++p) {
      hk.push_base[p] = c->peer[p] + c->L.outb;
      hk.push_done[p] = reinterpret_cast<uint64_t*>(c->peer[p] + c->L.delivered);
    }
    hk.ticket = P.ctl + ep::CTL_GEMM_TICKET;
    dst = c->base + c->L.outb;  // not written: every row goes to its token's owner
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (variant >= 3 && variant <= 5)
    return launch_gmv(lhs, codes, scales, scale_dtype, recv_group_sizes, c->local_experts,
                      (int)c->cap, k, n, 0, c->local_experts, act, act_limit, out_dtype, 0, dst,
                      variant == 3 ? 1 : variant == 4 ? 2 : 4, s, 0, 0, 1 << 30, &hk);
  if (variant == 1)
    return launch_gmm_single_ep(lhs, codes, scales, scale_dtype, recv_group_sizes,
                                c->local_experts, (int)c->cap, k, n, act, act_limit, out_dtype,
                                dst, &hk, s);
  return launch_gmm_pair(lhs, codes, scales, scale_dtype, recv_group_sizes, c->local_experts,
                         (int)c->cap, k, n, 0, c->local_experts, act, act_limit, out_dtype, 0, dst,
                         &hk, s, 0, variant == 9 ? 1 : 0, 0);
}

extern "C" int dwm_ep_link_probe(dwm_ep* c, int peer, int64_t bytes, void* stream) {
  int rc = check_ctx(c);
  if (rc) return rc;
  DWM_CHECK_ARG(peer >= 0 && peer < c->world && peer != c->rank, "peer=%d", peer);
  const int64_t cap = c->cap * c->hidden * 2;
  DWM_CHECK_ARG(bytes > 0 && bytes <= cap, "bytes=%lld out of (0, %lld]", (long long)bytes,
                (long long)cap);
  return check_cuda(cudaMemcpyAsync(c->peer[peer] + c->L.recv, c->base + c->L.recv, (size_t)bytes,
                                    cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)),
                    "ep link probe copy");
}

extern "C" int dwm_ep_set_wait_limit(dwm_ep* c, uint64_t limit_ns) {
  DWM_CHECK_ARG(c, "NULL ep context");
  DWM_CHECK_ARG(limit_ns >= 1000 && limit_ns <= 60000000000ull,
                "wait limit %llu ns out of [1 us, 60 s]", (unsigned long long)limit_ns);
  c->wait_ns = limit_ns;
  return DWM_OK;
}

extern "C" int dwm_ep_destroy(dwm_ep* c) {
  if (!c) return DWM_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  for (int p = 0; p < MAX_WORLD; ++p)
    if (c->peer_ipc[p]) cudaIpcCloseMemHandle(c->peer[p]);
  if (c->base) cudaFree(c->base);
  if (c->scratch) cudaFree(c->scratch);
  if (prev >= 0) cudaSetDevice(prev);
  delete c;
  return DWM_OK;
}
