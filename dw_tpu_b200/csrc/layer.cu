// The single-device FP4 MoE layer (fused_moe_func's GMM path, X0104:88-98)
// as one C call: route -> permute -> gather -> gmm1 (SwiGLU) -> gmm2 ->
// k-order combine, on a caller-provided workspace. Each stage is the same
// entry point the caller could make itself, so results are bit-identical to
// that sequence; the call only saves the host round trips (one call instead of
// six) and the intermediate bookkeeping.
#include <map>
#include <mutex>

#include "common.cuh"

namespace dwm {
namespace layer {

struct Plan {  // byte offsets inside the workspace
  size_t ids, w16, tok, revert, gs, x, h1, y, total;
};

inline size_t up(size_t v) { return (v + 255) / 256 * 256; }

Plan plan(int t, int h, int inter, int topk, int e, int y_f32) {
  const size_t rows = (size_t)t * topk;
  Plan p;
  p.ids = 0;
  p.w16 = up(p.ids + rows * 4);
  p.tok = up(p.w16 + rows * 2);
  p.revert = up(p.tok + rows * 4);
  p.gs = up(p.revert + rows * 4);
  p.x = up(p.gs + (size_t)e * 4);
  p.h1 = up(p.x + rows * h * 2);
  p.y = up(p.h1 + rows * inter * 2);
  p.total = up(p.y + rows * h * (y_f32 ? 4 : 2));
  return p;
}

}  // namespace layer
}  // namespace dwm

using namespace dwm;

extern "C" size_t dwm_moe_layer_workspace_bytes(int num_tokens, int hidden, int inter, int topk,
                                                int num_experts, int y_f32) {
  if (num_tokens < 0 || hidden <= 0 || inter <= 0 || topk <= 0 || num_experts <= 0) return 0;
  return layer::plan(num_tokens, hidden, inter, topk, num_experts, y_f32).total;
}

extern "C" int dwm_moe_layer_fp4(const void* hidden, const void* logits, int logits_dtype,
                                 int num_tokens, int hidden_size, int num_experts, int topk,
                                 int scoring, int renormalize, const void* w13, const void* s13,
                                 const void* w2, const void* s2, int codes_format,
                                 int scale_dtype, int inter, int act, float act_limit,
                                 int y_f32, void* workspace, size_t workspace_bytes, void* out,
                                 void* stream) {
  DWM_CHECK_ARG(num_tokens >= 0 && hidden_size > 0 && inter > 0 && topk >= 1 &&
                    num_experts >= 1,
                "bad shape t=%d h=%d i=%d topk=%d e=%d", num_tokens, hidden_size, inter, topk,
                num_experts);
  DWM_CHECK_ARG(act == DWM_ACT_SWIGLU || act == DWM_ACT_SWIGLU_CLAMP,
                "the layer's gmm1 activation must be SwiGLU (optionally clamped)");
  const layer::Plan p =
      layer::plan(num_tokens, hidden_size, inter, topk, num_experts, y_f32);
  DWM_CHECK_ARG(workspace && workspace_bytes >= p.total,
                "workspace of %zu bytes is smaller than the %zu bytes needed", workspace_bytes,
                p.total);
  DWM_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
                "workspace must be 256-byte aligned");
  if (num_tokens == 0) return DWM_OK;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* ids = reinterpret_cast<int32_t*>(ws + p.ids);
  void* w16 = ws + p.w16;
  int32_t* tok = reinterpret_cast<int32_t*>(ws + p.tok);
  int32_t* revert = reinterpret_cast<int32_t*>(ws + p.revert);
  int32_t* gs = reinterpret_cast<int32_t*>(ws + p.gs);
  void* x = ws + p.x;
  void* h1 = ws + p.h1;
  void* y = ws + p.y;
  const int rows = num_tokens * topk;
  int rc = dwm_route_topk(logits, logits_dtype, num_tokens, num_experts, topk, scoring,
                          renormalize, nullptr, -1, ids, nullptr, w16, stream);
  if (rc) return rc;
  rc = dwm_permute(ids, num_tokens, topk, num_experts, nullptr, tok, revert, gs, stream);
  if (rc) return rc;
  rc = dwm_dispatch_gather(hidden, num_tokens, hidden_size, tok, rows, x, stream);
  if (rc) return rc;
  rc = dwm_gmm_fp4(x, w13, codes_format, s13, scale_dtype, gs, num_experts, rows, hidden_size,
                   2 * inter, 0, num_experts, act, act_limit, DWM_BF16, 0, h1, stream);
  if (rc) return rc;
  rc = dwm_gmm_fp4(h1, w2, codes_format, s2, scale_dtype, gs, num_experts, rows, inter,
                   hidden_size, 0, num_experts, DWM_ACT_NONE, 0.0f, y_f32 ? DWM_F32 : DWM_BF16,
                   0, y, stream);
  if (rc) return rc;
  return dwm_combine(y, y_f32 ? DWM_F32 : DWM_BF16, rows, revert, w16, DWM_BF16, num_tokens,
                     hidden_size, topk, out, DWM_BF16, stream);
}

// ---------------------------------------------------------------------------
// The same layer for callers that cannot allocate device memory: the
// intermediates live in one file-scope device array of fixed size
// (DWM_LAYER_SCRATCH_BYTES) instead of a caller workspace.
// ---------------------------------------------------------------------------

namespace dwm {
namespace layer {

__device__ __align__(256) uint8_t g_scratch[DWM_LAYER_SCRATCH_BYTES];

// Address of g_scratch in the current context, resolved once per context
// (with its device current) and cached under the context handle, so that a
// new primary context (after cudaDeviceReset) resolves it afresh.
int scratch_address(void** out) {
  static std::mutex mu;
  static std::map<void*, void*> addr;  // CUDA context -> g_scratch's address in it
  void* ctx = nullptr;
  if (current_context(&ctx) != DWM_OK) {
    // No context current yet: resolving the symbol makes the runtime create
    // the device's primary context.
    void* p = nullptr;
    int rc = check_cuda(cudaGetSymbolAddress(&p, g_scratch), "cudaGetSymbolAddress(layer scratch)");
    if (rc) return rc;
    rc = current_context(&ctx);
    if (rc) return rc;
  }
  std::lock_guard<std::mutex> lock(mu);
  auto it = addr.find(ctx);
  if (it == addr.end()) {
    void* p = nullptr;
    const int rc =
        check_cuda(cudaGetSymbolAddress(&p, g_scratch), "cudaGetSymbolAddress(layer scratch)");
    if (rc) return rc;
    it = addr.emplace(ctx, p).first;
  }
  *out = it->second;
  return DWM_OK;
}

}  // namespace layer
}  // namespace dwm

extern "C" int dwm_moe_layer_fp4_noalloc(const void* hidden, const void* logits,
                                         int logits_dtype, int num_tokens, int hidden_size,
                                         int num_experts, int topk, int scoring, int renormalize,
                                         const void* w13, const void* s13, const void* w2,
                                         const void* s2, int codes_format, int scale_dtype,
                                         int inter, int act, float act_limit, int y_f32,
                                         void* out, void* stream) {
  DWM_CHECK_ARG(num_tokens >= 0 && hidden_size > 0 && inter > 0 && topk >= 1 &&
                    num_experts >= 1,
                "bad shape t=%d h=%d i=%d topk=%d e=%d", num_tokens, hidden_size, inter, topk,
                num_experts);
  const size_t need =
      layer::plan(num_tokens, hidden_size, inter, topk, num_experts, y_f32).total;
  DWM_CHECK_ARG(need <= (size_t)DWM_LAYER_SCRATCH_BYTES,
                "the layer needs %zu bytes of scratch, more than the %d bytes built in "
                "(DWM_LAYER_SCRATCH_BYTES)",
                need, DWM_LAYER_SCRATCH_BYTES);
  void* scratch = nullptr;
  int rc = layer::scratch_address(&scratch);  // a num_tokens = 0 call does only this setup
  if (rc) return rc;
  return dwm_moe_layer_fp4(hidden, logits, logits_dtype, num_tokens, hidden_size, num_experts,
                           topk, scoring, renormalize, w13, s13, w2, s2, codes_format,
                           scale_dtype, inter, act, act_limit, y_f32, scratch,
                           (size_t)DWM_LAYER_SCRATCH_BYTES, out, stream);
}
