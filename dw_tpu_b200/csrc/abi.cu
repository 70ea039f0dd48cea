// Library plumbing behind the C ABI: error messages, the per-device status
// word, tensor-map encoding and SM counts.
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <mutex>
#include <set>
#include <tuple>

#include "common.cuh"

namespace {

thread_local char g_last_error[512] = "";

// Device status word: kernels OR DWM_DEV_* bits into it.
__device__ int g_status;

constexpr int kMaxDevices = 64;
std::atomic<int*> g_status_addr[kMaxDevices] = {};
std::atomic<int> g_num_sms[kMaxDevices] = {};
std::mutex g_mu;
std::set<std::tuple<int, const void*, int>> g_smem_set;  // (device, kernel, bytes) done

std::atomic<PFN_cuTensorMapEncodeTiled_v12000> g_encode{nullptr};
std::atomic<PFN_cuCtxGetCurrent_v4000> g_ctx_current{nullptr};

}  // namespace

namespace dwm {

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return DWM_OK;
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s", what, cudaGetErrorString(e));
  return (int)e;
}

int* status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  if (int* p = g_status_addr[dev].load(std::memory_order_acquire)) return p;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_status_addr[dev].load(std::memory_order_relaxed)) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status) != cudaSuccess) return nullptr;
    g_status_addr[dev].store(static_cast<int*>(p), std::memory_order_release);
  }
  return g_status_addr[dev].load(std::memory_order_relaxed);
}

int num_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < kMaxDevices) {
    const int n = g_num_sms[dev].load(std::memory_order_relaxed);
    if (n) return n;
  }
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (n <= 0) n = 148;
  if (dev >= 0 && dev < kMaxDevices) g_num_sms[dev].store(n, std::memory_order_relaxed);
  return n;
}

int set_smem_limit(const void* kernel, int bytes, const char* what) {
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  const auto key = std::make_tuple(dev, kernel, bytes);
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_smem_set.count(key)) return DWM_OK;
  rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
                  what);
  if (!rc) g_smem_set.insert(key);
  return rc;
}

namespace {
// Resolves a driver entry point through the runtime (no -lcuda link), once.
template <typename PFN>
int resolve_driver_fn(std::atomic<PFN>& slot, const char* name) {
  if (slot.load(std::memory_order_acquire)) return DWM_OK;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!slot.load(std::memory_order_relaxed)) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint(name, &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
      return set_error(DWM_ERR_UNSUPPORTED, "%s unavailable", name);
    slot.store(reinterpret_cast<PFN>(fn), std::memory_order_release);
  }
  return DWM_OK;
}

int resolve_encode() { return resolve_driver_fn(g_encode, "cuTensorMapEncodeTiled"); }
}  // namespace

int current_context(void** ctx) {
  *ctx = nullptr;
  int rc = resolve_driver_fn(g_ctx_current, "cuCtxGetCurrent");
  if (rc) return rc;
  CUcontext c = nullptr;
  if (g_ctx_current.load(std::memory_order_acquire)(&c) != CUDA_SUCCESS || !c)
    return set_error(DWM_ERR_STATE, "no current CUDA context");
  *ctx = c;
  return DWM_OK;
}

int encode_tmap_nd(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                   const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                   CUtensorMapSwizzle swz) {
  if (rank < 1 || rank > 5) return set_error(DWM_ERR_INVALID, "tensor map rank %d", rank);
  int rc = resolve_encode();
  if (rc) return rc;
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], estr[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    estr[i] = 1;
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  CUresult r = g_encode.load(std::memory_order_acquire)(map, dtype, rank, const_cast<void*>(base), d, st, b, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(DWM_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d): rank %d", (int)r,
                     rank);
  return DWM_OK;
}

int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                   uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                   uint32_t box_outer, CUtensorMapSwizzle swz) {
  int rc = resolve_encode();
  if (rc) return rc;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode.load(std::memory_order_acquire)(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(DWM_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu",
                     (int)r, (unsigned long long)inner, (unsigned long long)outer);
  return DWM_OK;
}

}  // namespace dwm

extern "C" {

const char* dwm_version(void) { return "dw_moe 0.1.0 sm_100a"; }

const char* dwm_last_error(void) { return g_last_error; }

int dwm_device_status(void* stream, int* bits) {
  if (!bits) return dwm::set_error(DWM_ERR_INVALID, "bits is NULL");
  int* p = dwm::status_ptr();
  if (!p) return dwm::set_error(DWM_ERR_STATE, "no device status word");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int host = 0;
  int rc = dwm::check_cuda(cudaMemcpyAsync(&host, p, sizeof(int), cudaMemcpyDeviceToHost, s),
                           "status read");
  if (rc) return rc;
  rc = dwm::check_cuda(cudaMemsetAsync(p, 0, sizeof(int), s), "status clear");
  if (rc) return rc;
  rc = dwm::check_cuda(cudaStreamSynchronize(s), "status sync");
  if (rc) return rc;
  *bits = host;
  return DWM_OK;
}

}  // extern "C"
