// Expert-parallel token exchange for sm_100a over NVLink peer memory: the
// one-shot dispatch and combine that replace the reference's all-gather +
// per-shard sort (X0101:56-104, X0107:34-51) and its masked combine +
// reduce-scatter (X0107:15-29, KO:167-185).
//
// One process per GPU. Every rank owns one device allocation with the same
// layout (the "symmetric" buffer), exports it as a CUDA IPC handle, and maps
// every peer's; kernels then store straight into peer memory over NVLink.
//
//   dispatch  COUNTS  one CTA stably sorts the rank's (token, k) pairs by
//                     expert (the counting sort of the single-device permute),
//                     then stores its per-expert counts into every peer's count
//                     matrix and raises a per-source flag there.
//             ROWS    each CTA waits for all sources' counts, derives where
//                     each local pair lands in its owner's receive buffer, and
//                     copies the token row there (16-byte stores, a warp per
//                     row) with a (source rank, pair) tag; then it bumps every
//                     peer's arrival counter.
//             WAIT    one thread waits until all CTAs of all sources arrived.
//   combine   PUSH    each CTA copies expert-output rows back to the pair's
//                     source, into that rank's combine buffer at the pair's
//                     slot, then bumps every peer's arrival counter.
//             REDUCE  every CTA waits for all arrivals, then forms the k-order
//                     f32 weighted sum of each token (the single-device
//                     combine's arithmetic, bit for bit).
//
// Receive order: rank r's rows are expert-major over its experts
// [r*E/n, (r+1)*E/n), and inside an expert ordered by (source rank, source
// token, k slot): the rows the reference's global stable argsort over the
// rank-major gathered batch keeps on rank r (X0101:56-104). A pair's row is
//   sum of all ranks' counts of the owner's earlier experts
//   + sum of lower ranks' counts of its expert
//   + its rank among the source's own pairs of that expert (stable).
//
// Waits are bounded (2 s, then DWM_DEV_TIMEOUT in the status word and the
// kernel returns). Every wait depends only on kernels of other ranks (or of
// earlier launches), never on a CTA of the same grid, so a grid that is not
// fully resident cannot deadlock. Flags and counters are monotonic (epoch
// numbered), so nothing is reset between steps; the count matrix is double
// buffered by epoch parity.
#include <cstring>
#include <new>

#include "moe_common.cuh"

namespace dwm {
namespace ep {

constexpr int MAX_WORLD = 8;
constexpr int XFER_CTAS = 128;  // grid of the ROWS and PUSH kernels (the same on every rank)
constexpr int XFER_THREADS = 512;
constexpr int XFER_WARPS = XFER_THREADS / 32;

struct Layout {  // byte offsets inside every rank's symmetric buffer
  size_t flags;   // uint32 [MAX_WORLD]: epoch of the counts source s stored here
  size_t arrive;  // uint64 [2]: dispatch / combine CTA arrivals (monotonic)
  size_t counts;  // int32 [2][MAX_WORLD][E]: per-source expert counts, by epoch parity
  size_t meta;    // int32 [cap]: source rank * max_pairs + pair of each received row
  size_t recv;    // bf16 [cap][H]: received rows, expert-major
  size_t cbuf;    // [max_pairs][H] (4-byte capacity): combine buffer, one row per own pair
  size_t total;
};

struct Params {
  uint8_t* peer[MAX_WORLD];
  Layout L;
  int rank, world, E, LE, H, topk, T, max_pairs;
  int64_t cap;
  uint32_t epoch;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t ld_acquire_sys64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_sys_add(uint64_t* p, uint64_t v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Bounded spin until *p >= target (32-bit epoch flag).
__device__ __forceinline__ bool wait_flag(const uint32_t* p, uint32_t target, int* status) {
  if (ld_acquire_sys(p) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    __nanosleep(64);
    if (ld_acquire_sys(p) >= target) return true;
    if ((i & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
      report(status, DWM_DEV_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ bool wait_count(const uint64_t* p, uint64_t target, int* status) {
  if (ld_acquire_sys64(p) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    __nanosleep(64);
    if (ld_acquire_sys64(p) >= target) return true;
    if ((i & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
      report(status, DWM_DEV_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ int* counts_of(const Params& P, int rank_mem, int src) {
  return reinterpret_cast<int*>(P.peer[rank_mem] + P.L.counts) +
         ((size_t)(P.epoch & 1) * MAX_WORLD + src) * P.E;
}

// COUNTS: local stable sort + publish counts to every rank.
__global__ void __launch_bounds__(moe::SORT_THREADS, 1)
    ep_count_kernel(const __grid_constant__ Params P, const int32_t* __restrict__ ids, int32_t* revert,
                    int32_t* counts, int32_t* prefix, int* status) {
  extern __shared__ int sm[];
  moe::counting_sort_block(ids, P.T * P.topk, P.topk, P.E, nullptr, nullptr, revert, counts,
                           prefix, status, sm);
  __syncthreads();
  for (int i = threadIdx.x; i < P.world * P.E; i += blockDim.x) {
    const int p = i / P.E, x = i - p * P.E;
    counts_of(P, p, P.rank)[x] = counts[x];
  }
  __threadfence_system();
  __syncthreads();
  if ((int)threadIdx.x < P.world)
    st_release_sys(reinterpret_cast<uint32_t*>(P.peer[threadIdx.x] + P.L.flags) + P.rank,
                   P.epoch);
}

// ROWS: place every local pair in its owner's receive buffer.
// smem: colsum [E], before [E], dest [E] ints.
__global__ void __launch_bounds__(XFER_THREADS)
    ep_send_kernel(const __grid_constant__ Params P, const uint4* __restrict__ hidden,
                   const int32_t* __restrict__ ids, const int32_t* __restrict__ revert,
                   const int32_t* __restrict__ prefix, int32_t* recv_group_sizes, int* status) {
  extern __shared__ int sm[];
  int* colsum = sm;
  int* before = sm + P.E;
  int* dest = sm + 2 * P.E;
  __shared__ int s_fail;
  if (threadIdx.x == 0) s_fail = 0;
  __syncthreads();
  if ((int)threadIdx.x < P.world) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(P.peer[P.rank] + P.L.flags) + threadIdx.x;
    if (!wait_flag(f, P.epoch, status)) s_fail = 1;
  }
  __syncthreads();
  if (s_fail) return;
  for (int x = threadIdx.x; x < P.E; x += blockDim.x) {
    int col = 0, bef = 0;
    for (int s = 0; s < P.world; ++s) {
      const int v = __ldcg(counts_of(P, P.rank, s) + x);
      col += v;
      if (s < P.rank) bef += v;
    }
    colsum[x] = col;
    before[x] = bef;
  }
  __syncthreads();
  for (int x = threadIdx.x; x < P.E; x += blockDim.x) {
    const int owner = x / P.LE;
    int base = 0;
    for (int x2 = owner * P.LE; x2 < x; ++x2) base += colsum[x2];
    dest[x] = base + before[x] - prefix[x];  // + the pair's local sorted position
    if (blockIdx.x == 0 && owner == P.rank) recv_group_sizes[x - owner * P.LE] = colsum[x];
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h16 = P.H / 8;
  const int n = P.T * P.topk;
  for (int j = blockIdx.x * XFER_WARPS + warp; j < n; j += gridDim.x * XFER_WARPS) {
    const int pos = revert[j];
    if (pos < 0) continue;  // invalid id, reported by the sort
    const int e = ids[j];
    const int owner = e / P.LE;
    const int64_t row = (int64_t)dest[e] + pos;
    if (row < 0 || row >= P.cap) {
      if (lane == 0) report(status, DWM_DEV_OVERFLOW);
      continue;
    }
    const uint4* src = hidden + (int64_t)(j / P.topk) * h16;
    uint4* dst = reinterpret_cast<uint4*>(P.peer[owner] + P.L.recv) + row * h16;
    for (int c = lane; c < h16; c += 32) dst[c] = src[c];
    if (lane == 0)
      reinterpret_cast<int32_t*>(P.peer[owner] + P.L.meta)[row] = P.rank * P.max_pairs + j;
  }
  __threadfence_system();
  __syncthreads();
  if ((int)threadIdx.x < P.world)
    red_release_sys_add(reinterpret_cast<uint64_t*>(P.peer[threadIdx.x] + P.L.arrive), 1);
}

// WAIT (dispatch: which = 0) — one thread.
__global__ void ep_wait_kernel(const __grid_constant__ Params P, int which, uint64_t target, int* status) {
  if (threadIdx.x == 0)
    wait_count(reinterpret_cast<const uint64_t*>(P.peer[P.rank] + P.L.arrive) + which, target,
               status);
}

// PUSH: return every received row's expert output to the pair's source.
// y_es: bytes per element of y (2 or 4).
__global__ void __launch_bounds__(XFER_THREADS)
    ep_push_kernel(const __grid_constant__ Params P, const uint8_t* __restrict__ y, int y_es, int* status) {
  __shared__ int s_rows;
  if (threadIdx.x == 0) s_rows = 0;
  __syncthreads();
  int part = 0;
  for (int x = threadIdx.x; x < P.LE; x += blockDim.x)
    for (int s = 0; s < P.world; ++s) part += __ldcg(counts_of(P, P.rank, s) + P.rank * P.LE + x);
  if (part) atomicAdd(&s_rows, part);
  __syncthreads();
  const int rows = s_rows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row_bytes = (int64_t)P.H * y_es;
  const int n16 = (int)(row_bytes / 16);
  const int32_t* meta = reinterpret_cast<const int32_t*>(P.peer[P.rank] + P.L.meta);
  for (int r = blockIdx.x * XFER_WARPS + warp; r < rows && r < P.cap;
       r += gridDim.x * XFER_WARPS) {
    const int tag = __ldcg(meta + r);
    const int src = tag / P.max_pairs, pair = tag - src * P.max_pairs;
    if (src < 0 || src >= P.world) {
      if (lane == 0) report(status, DWM_DEV_BAD_INDEX);
      continue;
    }
    const uint4* from = reinterpret_cast<const uint4*>(y + r * row_bytes);
    uint4* to = reinterpret_cast<uint4*>(P.peer[src] + P.L.cbuf + pair * row_bytes);
    for (int c = lane; c < n16; c += 32) to[c] = from[c];
  }
  __threadfence_system();
  __syncthreads();
  if ((int)threadIdx.x < P.world)
    red_release_sys_add(reinterpret_cast<uint64_t*>(P.peer[threadIdx.x] + P.L.arrive) + 1, 1);
}

// REDUCE: out[t] = sum_k y(t, k) * w[t, k] in k order (f32, from +0.0).
template <int XD, int WD, int OD>
__global__ void ep_reduce_kernel(const __grid_constant__ Params P, const void* __restrict__ w,
                                 const int32_t* __restrict__ revert, void* __restrict__ out,
                                 uint64_t target, int* status) {
  __shared__ int s_ok;
  if (threadIdx.x == 0)
    s_ok = wait_count(reinterpret_cast<const uint64_t*>(P.peer[P.rank] + P.L.arrive) + 1, target,
                      status);
  __syncthreads();
  if (!s_ok) return;
  const void* cbuf = P.peer[P.rank] + P.L.cbuf;
  const int h8 = P.H / 8;
  const int64_t total = (int64_t)P.T * h8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / h8;
    const int c = (int)(i - t * h8);
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.0f;
    for (int k = 0; k < P.topk; ++k) {
      const int64_t j = t * P.topk + k;
      const float wk = moe::load_weight<WD>(w, j);
      if (revert[j] < 0) continue;  // invalid id (reported at dispatch)
      float v[8];
      moe::load8_cg<XD>(cbuf, j * P.H + (int64_t)c * 8, v);
      moe::mul_add8(acc, v, wk);
    }
    moe::store8<OD>(out, t * P.H + (int64_t)c * 8, acc);
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
  int32_t* scratch = nullptr;  // revert [max_pairs], counts [E], prefix [E]
  uint8_t* peer[MAX_WORLD] = {};
  bool peer_ipc[MAX_WORLD] = {};
  bool connected = false;
  uint32_t epoch = 0;  // dispatches started
  int last_t = -1;     // tokens of the current dispatch
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
  P.max_pairs = (int)c->max_pairs;
  P.cap = c->cap;
  P.epoch = c->epoch;
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
  DWM_CHECK_ARG(cap < (1LL << 31) / 2, "max_tokens * topk * world too large");
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
  L.flags = 0;
  L.arrive = 64;
  L.counts = 128;
  L.meta = align_up(L.counts + (size_t)2 * MAX_WORLD * num_experts * 4, 256);
  L.recv = align_up(L.meta + (size_t)cap * 4, 256);
  L.cbuf = align_up(L.recv + (size_t)cap * hidden * 2, 256);
  L.total = align_up(L.cbuf + (size_t)max_pairs * hidden * 4, 256);
  int rc = check_cuda(cudaMalloc(&c->base, L.total), "ep symmetric buffer");
  if (!rc) rc = check_cuda(cudaMemset(c->base, 0, L.meta), "ep header clear");
  if (!rc)
    rc = check_cuda(cudaMalloc(&c->scratch, (size_t)(max_pairs + 2 * num_experts) * 4),
                    "ep scratch");
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

extern "C" int dwm_ep_dispatch(dwm_ep* c, const void* hidden, const int32_t* topk_ids,
                               int num_tokens, int32_t* recv_group_sizes, int phases,
                               void* stream) {
  int rc = check_ctx(c);
  if (rc) return rc;
  DWM_CHECK_ARG(phases >= 1 && phases <= DWM_EP_ALL, "phases=%d", phases);
  DWM_CHECK_ARG(num_tokens >= 0 && num_tokens <= c->max_tokens,
                "num_tokens=%d out of [0, max_tokens=%d]", num_tokens, c->max_tokens);
  DWM_CHECK_ARG(num_tokens == 0 || (hidden && topk_ids), "NULL input");
  DWM_CHECK_ARG(moe::aligned16(hidden), "hidden must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* revert = c->scratch;
  int32_t* counts = c->scratch + c->max_pairs;
  int32_t* prefix = counts + c->num_experts;
  if (phases & DWM_EP_COUNTS) {
    ++c->epoch;
    c->last_t = num_tokens;
    const size_t smem = moe::sort_smem_bytes(c->num_experts);
    static bool attr_set[64] = {};
    if (c->device < 64 && !attr_set[c->device]) {
      rc = check_cuda(cudaFuncSetAttribute(ep::ep_count_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)moe::sort_smem_bytes(1024)),
                      "ep count smem attribute");
      if (rc) return rc;
      attr_set[c->device] = true;
    }
    ep::ep_count_kernel<<<1, moe::SORT_THREADS, smem, s>>>(make_params(c), topk_ids, revert,
                                                           counts, prefix, status_ptr());
    rc = check_cuda(cudaGetLastError(), "ep count launch");
    if (rc) return rc;
  }
  if (c->epoch == 0) return set_error(DWM_ERR_STATE, "dispatch phases before COUNTS");
  if (phases & DWM_EP_ROWS) {
    DWM_CHECK_ARG(num_tokens == c->last_t, "num_tokens=%d differs from the COUNTS phase (%d)",
                  num_tokens, c->last_t);
    DWM_CHECK_ARG(recv_group_sizes, "NULL recv_group_sizes");
    ep::ep_send_kernel<<<ep::XFER_CTAS, ep::XFER_THREADS, 3 * c->num_experts * sizeof(int), s>>>(
        make_params(c), static_cast<const uint4*>(hidden), topk_ids, revert, prefix,
        recv_group_sizes, status_ptr());
    rc = check_cuda(cudaGetLastError(), "ep send launch");
    if (rc) return rc;
  }
  if (phases & DWM_EP_WAIT) {
    const uint64_t target = (uint64_t)c->epoch * c->world * ep::XFER_CTAS;
    ep::ep_wait_kernel<<<1, 32, 0, s>>>(make_params(c), 0, target, status_ptr());
    rc = check_cuda(cudaGetLastError(), "ep wait launch");
    if (rc) return rc;
  }
  return DWM_OK;
}

extern "C" int dwm_ep_combine(dwm_ep* c, const void* y, int y_dtype, const void* topk_weights,
                              int w_dtype, void* out, int out_dtype, int phases, void* stream) {
  int rc = check_ctx(c);
  if (rc) return rc;
  DWM_CHECK_ARG(phases >= 1 && phases <= (DWM_EP_PUSH | DWM_EP_REDUCE), "phases=%d", phases);
  DWM_CHECK_ARG(c->epoch > 0, "combine before any dispatch");
  DWM_CHECK_ARG(y_dtype == DWM_BF16 || y_dtype == DWM_F32, "y dtype must be bf16 or f32");
  DWM_CHECK_ARG(w_dtype == DWM_BF16 || w_dtype == DWM_F32, "weight dtype must be bf16 or f32");
  DWM_CHECK_ARG(out_dtype == DWM_BF16 || out_dtype == DWM_F32, "out dtype must be bf16 or f32");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const ep::Params P = make_params(c);
  if (phases & DWM_EP_PUSH) {
    DWM_CHECK_ARG(y && moe::aligned16(y), "y must be a 16-byte aligned device pointer");
    ep::ep_push_kernel<<<ep::XFER_CTAS, ep::XFER_THREADS, 0, s>>>(
        P, static_cast<const uint8_t*>(y), y_dtype == DWM_F32 ? 4 : 2, status_ptr());
    rc = check_cuda(cudaGetLastError(), "ep push launch");
    if (rc) return rc;
  }
  if (phases & DWM_EP_REDUCE) {
    DWM_CHECK_ARG(P.T == 0 || (topk_weights && out), "NULL weights or out");
    DWM_CHECK_ARG(moe::aligned16(out), "out must be 16-byte aligned");
    const uint64_t target = (uint64_t)c->epoch * c->world * ep::XFER_CTAS;
    const unsigned grid = moe::grid_for((int64_t)P.T * (c->hidden / 8), 256, 4);
    int* st = status_ptr();
    const int32_t* revert = c->scratch;
#define DWM_EP_REDUCE_CASE(XD, WD, OD)                                                      \
  if (y_dtype == XD && w_dtype == WD && out_dtype == OD) {                                  \
    ep::ep_reduce_kernel<XD, WD, OD><<<grid, 256, 0, s>>>(P, topk_weights, revert, out,     \
                                                          target, st);                      \
    return check_cuda(cudaGetLastError(), "ep reduce launch");                              \
  }
    DWM_EP_REDUCE_CASE(DWM_BF16, DWM_BF16, DWM_BF16)
    DWM_EP_REDUCE_CASE(DWM_BF16, DWM_F32, DWM_BF16)
    DWM_EP_REDUCE_CASE(DWM_F32, DWM_BF16, DWM_BF16)
    DWM_EP_REDUCE_CASE(DWM_F32, DWM_F32, DWM_BF16)
    DWM_EP_REDUCE_CASE(DWM_BF16, DWM_BF16, DWM_F32)
    DWM_EP_REDUCE_CASE(DWM_BF16, DWM_F32, DWM_F32)
    DWM_EP_REDUCE_CASE(DWM_F32, DWM_BF16, DWM_F32)
    DWM_EP_REDUCE_CASE(DWM_F32, DWM_F32, DWM_F32)
#undef DWM_EP_REDUCE_CASE
  }
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
