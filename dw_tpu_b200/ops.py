"""Thin out-variant wrappers over the C ABI plus their torch.library custom ops.

Each ``*_out`` function validates torch tensors, then launches on the current
CUDA stream through libdw_moe.so. The ``dw_moe::*`` custom ops allocate their
outputs and call the same functions; they are what the reference-named shims
(``gmm_v2``, ``fast_dispatch_gather``, ``fast_combine`` ...) dispatch to.
"""

from __future__ import annotations

import torch

from . import _lib as L

_E8M0 = getattr(torch, "float8_e8m0fnu", None)
_FP4X2 = getattr(torch, "float4_e2m1fn_x2", None)


def _u8view(t: torch.Tensor) -> torch.Tensor:
    if t.dtype == torch.uint8:
        return t
    if t.dtype in (_E8M0, _FP4X2) or t.element_size() == 1:
        return t.view(torch.uint8)
    raise ValueError(f"expected a byte tensor, got {t.dtype}")


def _scale_view(s: torch.Tensor):
    """Scales [G, K/32, 1, N] or [G, K/32, N] -> (tensor, C dtype code)."""
    if s.dtype in (torch.uint8, _E8M0):
        return s.view(torch.uint8), L.U8
    if s.dtype == torch.bfloat16:
        return s, L.BF16
    if s.dtype == torch.float32:
        return s, L.F32
    raise ValueError(f"scale dtype {s.dtype} not supported (uint8 e8m0, bf16, f32)")


# ----------------------------------------------------------------------------
# FP4 grouped matmul
# ----------------------------------------------------------------------------

def fp4_dims(codes: torch.Tensor, layout: str):
    """(groups, k, n) of packed FP4 weights: "e2m1" [g, k, n/2]; "b200"
    [g, n, k/2]."""
    if codes.dim() != 3:
        raise ValueError("FP4 weights must be 3-D packed bytes")
    g, a, b = codes.shape
    if layout == "e2m1":
        return g, a, 2 * b
    if layout == "b200":
        return g, 2 * b, a
    raise ValueError(f"unknown FP4 layout {layout!r}")


def gmm_fp4_out(lhs, codes, scales, group_sizes, out, *, group_offset=0,
                num_local_groups=None, act=L.ACT_NONE, act_limit=0.0,
                zero_init=False, layout="e2m1", variant=0, stream=None):
    """out <- grouped matmul of lhs with the FP4 weights (see dwm_gmm_fp4).
    ``layout`` is "e2m1" (raw [g, k, n/2]) or "b200" (``fp4_to_b200_out``);
    ``variant`` 0 picks the kernel; 1 forces the tcgen05 kernel on one CTA,
    2-5 the mma.sync decode kernel (auto / 8 / 16 / 32-row token tiles), 7 the
    tcgen05 kernel on CTA pairs and 8 the pair kernel for each group's full
    256-row tiles with short remainders on the decode kernel, 9 the pair
    kernel with tiles of up to 512 rows, 10 each group on the kernel for its
    size; 1-5 and 7-10 need the B200 layout."""
    L.require_cuda(lhs, codes, scales, group_sizes, out)
    if lhs.dtype != torch.bfloat16 or lhs.dim() != 2:
        raise ValueError("lhs must be a 2-D bf16 tensor")
    codes = _u8view(codes)
    sc, sd = _scale_view(scales)
    g, k, n = fp4_dims(codes, layout)
    if sc.numel() != g * (k // 32) * n:
        raise ValueError(f"scales must hold [groups, k/32, n] = [{g}, {k // 32}, {n}]")
    m = lhs.shape[0]
    if lhs.shape[1] != k:
        raise ValueError(f"lhs has k={lhs.shape[1]}, weights k={k}")
    if group_sizes.dtype != torch.int32 or group_sizes.dim() != 1:
        raise ValueError("group_sizes must be a 1-D int32 tensor")
    nl = g if num_local_groups is None else int(num_local_groups)
    n_out = n if act == L.ACT_NONE else n // 2
    if out.shape != (m, n_out) or out.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"out must be [{m}, {n_out}] bf16/f32, got {tuple(out.shape)} "
                         f"{out.dtype}")
    for t in (lhs, codes, sc, group_sizes, out):
        if not t.is_contiguous():
            raise ValueError("tensors must be contiguous")
    rc = L.lib().dwm_gmm_fp4_variant(
        lhs.data_ptr(), codes.data_ptr(), L.LAYOUTS[layout], sc.data_ptr(), sd,
        group_sizes.data_ptr(), group_sizes.numel(), m, k, n, int(group_offset), nl, act,
        float(act_limit), L.dtype_code(out.dtype), int(bool(zero_init)), out.data_ptr(),
        int(variant), L.stream_ptr() if stream is None else stream)
    L.check(rc, "gmm_fp4")
    return out


def fp4_dequant_out(codes, scales, out, layout="e2m1", stream=None):
    L.require_cuda(codes, scales, out)
    codes = _u8view(codes)
    sc, sd = _scale_view(scales)
    g, k, n = fp4_dims(codes, layout)
    if out.shape != (g, k, n) or out.dtype != torch.bfloat16:
        raise ValueError("out must be bf16 [groups, k, n]")
    rc = L.lib().dwm_fp4_dequant(codes.data_ptr(), L.LAYOUTS[layout], sc.data_ptr(), sd, g, k,
                                 n, out.data_ptr(), L.stream_ptr() if stream is None else stream)
    L.check(rc, "fp4_dequant")
    return out


def fp4_to_b200_out(src, inverse=False, stream=None):
    """Raw e2m1 [g, k, n/2] -> the B200 layout (u32 words [g][n/16][k/16][32],
    returned as bytes shaped [g, n, k/2]), or back with ``inverse``; returns a
    new tensor."""
    L.require_cuda(src)
    src = _u8view(src).contiguous()
    if src.dim() != 3:
        raise ValueError("expected packed FP4 weights [g, k, n/2] (or [g, n, k/2])")
    if inverse:
        g, n, k2 = src.shape
        k = 2 * k2
        dst = torch.empty((g, k, n // 2), dtype=torch.uint8, device=src.device)
    else:
        g, k, n2 = src.shape
        n = 2 * n2
        dst = torch.empty((g, n, k // 2), dtype=torch.uint8, device=src.device)
    rc = L.lib().dwm_fp4_to_b200(src.data_ptr(), dst.data_ptr(), g, k, n, int(inverse),
                                 L.stream_ptr() if stream is None else stream)
    L.check(rc, "fp4_to_b200")
    return dst


def fp4_quantize_out(w, codes, scales, lossless=None, *, power_of_two_scale=True,
                     stream=None):
    """quantize_tensor(float4_e2m1fn, w, block 32, power_of_two_scale)
    (B01:319-347) of w [g, k, n] (bf16/f32) over blocks of 32 consecutive k:
    codes uint8 [g, k, n/2] (packed e2m1), scales [g, k/32, n] as uint8 E8M0
    codes (``lossless`` int32 [1] on the device is set to 1, cleared if a scale
    is not a normal power of two or +0) or f32 (dwm_fp4_quantize)."""
    L.require_cuda(w, codes, scales, lossless)
    if w.dim() != 3 or not w.is_contiguous():
        raise ValueError("w must be a contiguous [g, k, n] tensor")
    g, k, n = w.shape
    if codes.shape != (g, k, n // 2) or codes.dtype != torch.uint8:
        raise ValueError("codes must be uint8 [g, k, n/2]")
    if scales.shape != (g, k // 32, n):
        raise ValueError("scales must be [g, k/32, n]")
    rc = L.lib().dwm_fp4_quantize(w.data_ptr(), L.dtype_code(w.dtype), g, k, n,
                                  int(bool(power_of_two_scale)), codes.data_ptr(),
                                  scales.data_ptr(), L.dtype_code(scales.dtype), L.ptr(lossless),
                                  L.stream_ptr() if stream is None else stream)
    L.check(rc, "fp4_quantize")
    return codes, scales


def fp4_codes_convert_out(src, dst, from_format, to_format, stream=None):
    L.require_cuda(src, dst)
    src, dst = _u8view(src), _u8view(dst)
    if src.numel() != dst.numel():
        raise ValueError("size mismatch")
    rc = L.lib().dwm_fp4_codes_convert(src.data_ptr(), dst.data_ptr(), src.numel(),
                                       from_format, to_format,
                                       L.stream_ptr() if stream is None else stream)
    L.check(rc, "fp4_codes_convert")
    return dst


# ----------------------------------------------------------------------------
# Routing, permute, gather, combine, e8m0
# ----------------------------------------------------------------------------

_SCORING = {"softmax": L.SCORE_SOFTMAX, "sigmoid": L.SCORE_SIGMOID,
            "sqrtsoftplus": L.SCORE_SQRTSOFTPLUS}


def route_topk_out(logits, top_k, ids_out, w32_out=None, w16_out=None, *,
                   scoring_fn="sigmoid", renormalize=True, bias=None,
                   num_valid_tokens=None, stream=None):
    L.require_cuda(logits, ids_out, w32_out, w16_out, bias)
    if logits.dim() != 2 or not logits.is_contiguous():
        raise ValueError("logits must be a contiguous [t, e] tensor")
    t, e = logits.shape
    if scoring_fn not in _SCORING:
        raise ValueError(f"unknown scoring_fn {scoring_fn!r}")
    if bias is not None and (bias.dtype != torch.float32 or bias.numel() != e):
        raise ValueError("bias must be f32 [e]")
    rc = L.lib().dwm_route_topk(
        logits.data_ptr(), L.dtype_code(logits.dtype), t, e, int(top_k), _SCORING[scoring_fn],
        int(bool(renormalize)), L.ptr(bias),
        -1 if num_valid_tokens is None else int(num_valid_tokens), ids_out.data_ptr(),
        L.ptr(w32_out), L.ptr(w16_out), L.stream_ptr() if stream is None else stream)
    L.check(rc, "route_topk")


def route_hash_out(logits, hash_ids, ids_out, w32_out=None, w16_out=None, *,
                   scoring_fn="sigmoid", renormalize=True, num_valid_tokens=None, stream=None):
    L.require_cuda(logits, hash_ids, ids_out, w32_out, w16_out)
    if logits.dim() != 2 or not logits.is_contiguous():
        raise ValueError("logits must be a contiguous [t, e] tensor")
    t, e = logits.shape
    if hash_ids.dtype != torch.int32 or hash_ids.dim() != 2 or hash_ids.shape[0] != t:
        raise ValueError("hash_ids must be int32 [t, top_k]")
    if scoring_fn not in _SCORING:
        raise ValueError(f"unknown scoring_fn {scoring_fn!r}")
    rc = L.lib().dwm_route_hash(
        logits.data_ptr(), L.dtype_code(logits.dtype), t, e, hash_ids.shape[1],
        _SCORING[scoring_fn], int(bool(renormalize)), hash_ids.data_ptr(),
        -1 if num_valid_tokens is None else int(num_valid_tokens), ids_out.data_ptr(),
        L.ptr(w32_out), L.ptr(w16_out), L.stream_ptr() if stream is None else stream)
    L.check(rc, "route_hash")


def dedupe_topk_(w32, ids, num_experts, w16_out=None, stream=None):
    """In place on f32 weights and int32 ids [t, top_k] (dwm_dedupe_topk)."""
    L.require_cuda(w32, ids, w16_out)
    if w32.dtype != torch.float32 or ids.dtype != torch.int32 or w32.shape != ids.shape:
        raise ValueError("expected f32 weights and int32 ids of the same [t, top_k] shape")
    t, k = ids.shape
    rc = L.lib().dwm_dedupe_topk(w32.data_ptr(), ids.data_ptr(), t, k, int(num_experts),
                                 L.ptr(w16_out), L.stream_ptr() if stream is None else stream)
    L.check(rc, "dedupe_topk")


def permute_out(topk_ids, num_experts, group_sizes, argsort=None, token_indices_sorted=None,
                revert=None, stream=None):
    L.require_cuda(topk_ids, group_sizes, argsort, token_indices_sorted, revert)
    if topk_ids.dtype != torch.int32 or topk_ids.dim() != 2 or not topk_ids.is_contiguous():
        raise ValueError("topk_ids must be a contiguous int32 [t, topk] tensor")
    t, topk = topk_ids.shape
    rc = L.lib().dwm_permute(topk_ids.data_ptr(), t, topk, int(num_experts), L.ptr(argsort),
                             L.ptr(token_indices_sorted), L.ptr(revert), group_sizes.data_ptr(),
                             L.stream_ptr() if stream is None else stream)
    L.check(rc, "permute")


def sorted_token_indices_out(topk_argsort, topk, out, stream=None):
    L.require_cuda(topk_argsort, out)
    if topk_argsort.dtype != torch.int32:
        raise ValueError("argsort indices must be int32")
    rc = L.lib().dwm_sorted_token_indices(topk_argsort.data_ptr(), topk_argsort.numel(),
                                          int(topk), out.data_ptr(),
                                          L.stream_ptr() if stream is None else stream)
    L.check(rc, "sorted_token_indices")
    return out


def dispatch_gather_out(hidden, token_indices_sorted, out, stream=None):
    L.require_cuda(hidden, token_indices_sorted, out)
    if hidden.dtype != torch.bfloat16 or hidden.dim() != 2 or not hidden.is_contiguous():
        raise ValueError("hidden must be a contiguous bf16 [t, h] tensor")
    t, h = hidden.shape
    rows = token_indices_sorted.numel()
    if out.shape != (rows, h) or out.dtype != torch.bfloat16:
        raise ValueError("out must be bf16 [rows, h]")
    rc = L.lib().dwm_dispatch_gather(hidden.data_ptr(), t, h, token_indices_sorted.data_ptr(),
                                     rows, out.data_ptr(),
                                     L.stream_ptr() if stream is None else stream)
    L.check(rc, "dispatch_gather")
    return out


def combine_out(x, indices, topk_weights, topk, out, stream=None):
    L.require_cuda(x, indices, topk_weights, out)
    if x.dim() != 2 or not x.is_contiguous():
        raise ValueError("x must be a contiguous [rows, h] tensor")
    t = topk_weights.shape[0]
    h = x.shape[1]
    if topk_weights.shape != (t, topk) or not topk_weights.is_contiguous():
        raise ValueError("topk_weights must be contiguous [t, topk]")
    if indices.numel() != t * topk or indices.dtype != torch.int32:
        raise ValueError("indices must be int32 [t * topk]")
    if out.shape != (t, h):
        raise ValueError("out must be [t, h]")
    rc = L.lib().dwm_combine(x.data_ptr(), L.dtype_code(x.dtype), x.shape[0], indices.data_ptr(),
                             topk_weights.data_ptr(), L.dtype_code(topk_weights.dtype), t, h,
                             int(topk), out.data_ptr(), L.dtype_code(out.dtype),
                             L.stream_ptr() if stream is None else stream)
    L.check(rc, "combine")
    return out


def combine_shared_out(x, indices, topk_weights, topk, shared, out, *, routed_scale=1.0,
                       mid_dtype=torch.bfloat16, stream=None):
    """out <- combine (as ``combine_out``) with the shared expert summed in:
    out = round(f32(mid(routed)) * routed_scale + shared) (dwm_combine_shared,
    MOE_SHARED_EXPERT_TP X0104:80-87)."""
    L.require_cuda(x, indices, topk_weights, out, shared)
    if x.dim() != 2 or not x.is_contiguous():
        raise ValueError("x must be a contiguous [rows, h] tensor")
    t = topk_weights.shape[0]
    h = x.shape[1]
    if topk_weights.shape != (t, topk) or not topk_weights.is_contiguous():
        raise ValueError("topk_weights must be contiguous [t, topk]")
    if indices.numel() != t * topk or indices.dtype != torch.int32:
        raise ValueError("indices must be int32 [t * topk]")
    if out.shape != (t, h) or shared.shape != (t, h) or not shared.is_contiguous():
        raise ValueError("out and shared must be [t, h] (shared contiguous)")
    if mid_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("mid_dtype must be bf16 or f32")
    rc = L.lib().dwm_combine_shared(
        x.data_ptr(), L.dtype_code(x.dtype), x.shape[0], indices.data_ptr(),
        topk_weights.data_ptr(), L.dtype_code(topk_weights.dtype), t, h, int(topk),
        shared.data_ptr(), L.dtype_code(shared.dtype), float(routed_scale),
        L.dtype_code(mid_dtype), out.data_ptr(), L.dtype_code(out.dtype),
        L.stream_ptr() if stream is None else stream)
    L.check(rc, "combine_shared")
    return out


def _check_layer_args(hidden, logits, w13, s13, w2, s2, out, layout, scoring_fn):
    """Shape, dtype and layout checks of the one-call layer (the C layer builds
    its tensor maps and stores from these sizes alone): hidden bf16 [t, h],
    logits [t, e], w13 / s13 [e, h, 2I] and w2 / s2 [e, I, h] in ``layout``,
    out bf16 [t, h], all contiguous. Returns (t, h, e, I)."""
    if hidden.dtype != torch.bfloat16 or hidden.dim() != 2 or not hidden.is_contiguous():
        raise ValueError("hidden must be a contiguous bf16 [t, h] tensor")
    t, h = hidden.shape
    if logits.dim() != 2 or logits.shape[0] != t or not logits.is_contiguous():
        raise ValueError("logits must be a contiguous [t, e] tensor")
    if logits.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("logits must be bf16 or f32")
    e = logits.shape[1]
    if scoring_fn not in _SCORING:
        raise ValueError(f"unknown scoring_fn {scoring_fn!r}")
    if s2.dim() < 3 or s13.dim() < 3:
        raise ValueError("scales must be [e, k/32, n] (or [e, k/32, 1, n])")
    inter = s2.shape[1] * 32
    sc13, sd13 = _scale_view(s13)
    sc2, sd2 = _scale_view(s2)
    if sd13 != sd2:
        raise ValueError("s13 and s2 must have the same dtype")
    for name, codes, sc, k, n in (("w13", w13, sc13, h, 2 * inter), ("w2", w2, sc2, inter, h)):
        if fp4_dims(_u8view(codes), layout) != (e, k, n):
            raise ValueError(f"{name} must hold [{e}, {k}, {n}] FP4 weights in the {layout!r} "
                             f"layout, got {tuple(codes.shape)}")
        if sc.numel() != e * (k // 32) * n or sc.shape[0] != e:
            raise ValueError(f"{name} scales must be [{e}, {k // 32}, {n}]")
        if not codes.is_contiguous() or not sc.is_contiguous():
            raise ValueError(f"{name} and its scales must be contiguous")
    if h % 256 or inter % 128:
        raise ValueError(f"hidden={h} must be a multiple of 256 and intermediate={inter} of 128")
    if out.shape != (t, h) or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous bf16 [{t}, {h}] tensor")
    return t, h, e, inter


def moe_layer_workspace_bytes(num_tokens, hidden, inter, topk, num_experts, y_f32=False):
    return int(L.lib().dwm_moe_layer_workspace_bytes(int(num_tokens), int(hidden), int(inter),
                                                     int(topk), int(num_experts), int(y_f32)))


def moe_layer_fp4_out(hidden, logits, top_k, w13, s13, w2, s2, out, workspace, *,
                      layout="e2m1", scoring_fn="sigmoid", renormalize=True, act_limit=None,
                      f32_reduce=False, stream=None):
    """The whole single-device layer in one C call (dwm_moe_layer_fp4):
    route -> permute -> gather -> gmm1 (SwiGLU) -> gmm2 -> combine, with its
    intermediates in ``workspace`` (uint8, moe_layer_workspace_bytes)."""
    t, h, e, inter = _check_layer_args(hidden, logits, w13, s13, w2, s2, out, layout, scoring_fn)
    if workspace.dtype != torch.uint8 or workspace.dim() != 1:
        raise ValueError("workspace must be a 1-D uint8 tensor")
    L.require_cuda(hidden, logits, w13, s13, w2, s2, out, workspace)
    act = L.ACT_SWIGLU if act_limit is None else L.ACT_SWIGLU_CLAMP
    rc = L.lib().dwm_moe_layer_fp4(
        hidden.data_ptr(), logits.data_ptr(), L.dtype_code(logits.dtype), t, h, e, int(top_k),
        _SCORING[scoring_fn], int(bool(renormalize)), _u8view(w13).data_ptr(), s13.data_ptr(),
        _u8view(w2).data_ptr(), s2.data_ptr(), L.LAYOUTS[layout], L.dtype_code(s13.dtype),
        inter, act, 0.0 if act_limit is None else float(act_limit), int(bool(f32_reduce)),
        workspace.data_ptr(), workspace.numel() * workspace.element_size(), out.data_ptr(),
        L.stream_ptr() if stream is None else stream)
    L.check(rc, "moe_layer_fp4")
    return out


def moe_layer_fp4_noalloc_out(hidden, logits, top_k, w13, s13, w2, s2, out, *, layout="e2m1",
                              scoring_fn="sigmoid", renormalize=True, act_limit=None,
                              f32_reduce=False, stream=None):
    """``moe_layer_fp4_out`` without a workspace (dwm_moe_layer_fp4_noalloc):
    the intermediates live in the library's fixed device scratch
    (DWM_LAYER_SCRATCH_BYTES per device); larger inputs raise ValueError.
    Overlapping calls on one device race on that scratch."""
    t, h, e, inter = _check_layer_args(hidden, logits, w13, s13, w2, s2, out, layout, scoring_fn)
    L.require_cuda(hidden, logits, w13, s13, w2, s2, out)
    act = L.ACT_SWIGLU if act_limit is None else L.ACT_SWIGLU_CLAMP
    rc = L.lib().dwm_moe_layer_fp4_noalloc(
        hidden.data_ptr(), logits.data_ptr(), L.dtype_code(logits.dtype), t, h, e,
        int(top_k), _SCORING[scoring_fn], int(bool(renormalize)), _u8view(w13).data_ptr(),
        s13.data_ptr(), _u8view(w2).data_ptr(), s2.data_ptr(), L.LAYOUTS[layout],
        L.dtype_code(s13.dtype), inter, act,
        0.0 if act_limit is None else float(act_limit), int(bool(f32_reduce)), out.data_ptr(),
        L.stream_ptr() if stream is None else stream)
    L.check(rc, "moe_layer_fp4_noalloc")
    return out


def e8m0_encode_out(scale, codes, lossless, stream=None):
    L.require_cuda(scale, codes, lossless)
    if scale.dtype != torch.float32:
        raise ValueError("scale must be f32")
    rc = L.lib().dwm_e8m0_encode(scale.data_ptr(), scale.numel(), codes.data_ptr(),
                                 lossless.data_ptr(), L.stream_ptr() if stream is None else stream)
    L.check(rc, "e8m0_encode")


def e8m0_decode_out(codes, out, stream=None):
    L.require_cuda(codes, out)
    rc = L.lib().dwm_e8m0_decode(_u8view(codes).data_ptr(), codes.numel(), out.data_ptr(),
                                 L.stream_ptr() if stream is None else stream)
    L.check(rc, "e8m0_decode")
    return out


# ----------------------------------------------------------------------------
# torch.library custom ops (allocate outputs, call the out-variants)
# ----------------------------------------------------------------------------

@torch.library.custom_op("dw_moe::gmm_fp4", mutates_args=())
def gmm_fp4(lhs: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor,
            group_sizes: torch.Tensor, group_offset: int, num_local_groups: int, act: int,
            act_limit: float, out_f32: bool, zero_init: bool,
            layout: str = "e2m1") -> torch.Tensor:
    n = fp4_dims(codes, layout)[2]
    n_out = n if act == L.ACT_NONE else n // 2
    dt = torch.float32 if out_f32 else torch.bfloat16
    out = torch.empty((lhs.shape[0], n_out), dtype=dt, device=lhs.device)
    return gmm_fp4_out(lhs, codes, scales, group_sizes, out, group_offset=group_offset,
                       num_local_groups=num_local_groups, act=act, act_limit=act_limit,
                       zero_init=zero_init, layout=layout)


@gmm_fp4.register_fake
def _(lhs, codes, scales, group_sizes, group_offset, num_local_groups, act, act_limit, out_f32,
      zero_init, layout="e2m1"):
    n = fp4_dims(codes, layout)[2]
    n_out = n if act == L.ACT_NONE else n // 2
    return lhs.new_empty((lhs.shape[0], n_out),
                         dtype=torch.float32 if out_f32 else torch.bfloat16)


@torch.library.custom_op("dw_moe::permute", mutates_args=())
def permute(topk_ids: torch.Tensor, num_experts: int
            ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    n = topk_ids.numel()
    dev = topk_ids.device
    argsort = torch.empty(n, dtype=torch.int32, device=dev)
    tok = torch.empty(n, dtype=torch.int32, device=dev)
    revert = torch.empty(n, dtype=torch.int32, device=dev)
    gs = torch.empty(num_experts, dtype=torch.int32, device=dev)
    permute_out(topk_ids, num_experts, gs, argsort, tok, revert)
    return argsort, tok, revert, gs


@permute.register_fake
def _(topk_ids, num_experts):
    n = topk_ids.numel()
    e = topk_ids.new_empty(n)
    return e, e.clone(), e.clone(), topk_ids.new_empty(num_experts)


@torch.library.custom_op("dw_moe::dispatch_gather", mutates_args=())
def dispatch_gather(hidden: torch.Tensor, token_indices_sorted: torch.Tensor) -> torch.Tensor:
    out = hidden.new_empty((token_indices_sorted.numel(), hidden.shape[1]))
    return dispatch_gather_out(hidden, token_indices_sorted.contiguous(), out)


@dispatch_gather.register_fake
def _(hidden, token_indices_sorted):
    return hidden.new_empty((token_indices_sorted.numel(), hidden.shape[1]))


@torch.library.custom_op("dw_moe::combine", mutates_args=())
def combine(x: torch.Tensor, indices: torch.Tensor, topk_weights: torch.Tensor, topk: int,
            out_f32: bool) -> torch.Tensor:
    t = topk_weights.shape[0]
    out = x.new_empty((t, x.shape[1]), dtype=torch.float32 if out_f32 else torch.bfloat16)
    return combine_out(x, indices.contiguous(), topk_weights.contiguous(), topk, out)


@combine.register_fake
def _(x, indices, topk_weights, topk, out_f32):
    return x.new_empty((topk_weights.shape[0], x.shape[1]),
                       dtype=torch.float32 if out_f32 else torch.bfloat16)


@torch.library.custom_op("dw_moe::route_topk", mutates_args=())
def route_topk(logits: torch.Tensor, top_k: int, scoring_fn: str, renormalize: bool,
               num_valid_tokens: int) -> tuple[torch.Tensor, torch.Tensor]:
    t = logits.shape[0]
    ids = torch.empty((t, top_k), dtype=torch.int32, device=logits.device)
    w = torch.empty((t, top_k), dtype=torch.float32, device=logits.device)
    route_topk_out(logits.contiguous(), top_k, ids, w32_out=w, scoring_fn=scoring_fn,
                   renormalize=renormalize,
                   num_valid_tokens=None if num_valid_tokens < 0 else num_valid_tokens)
    return ids, w


@route_topk.register_fake
def _(logits, top_k, scoring_fn, renormalize, num_valid_tokens):
    t = logits.shape[0]
    return (logits.new_empty((t, top_k), dtype=torch.int32),
            logits.new_empty((t, top_k), dtype=torch.float32))
