"""MOE_FAST_COMBINE on B200 (KC, call sites X0404:81-113).

    out[t] = round(sum_k f32(x[idx[t * topk + k]]) * f32(w[t, k]))

f32 products, summed left to right from +0.0 (k = 0..topk-1), one rounding
(KC:14-21). Every mode runs the same CUDA kernel, bit-identical to that
sequence; unsupported shapes raise ValueError instead of falling back.
"""

from __future__ import annotations

import torch

from . import ops


def _combine(x, indices, topk_weights, topk, out_dtype):
    out_dtype = x.dtype if out_dtype is None else out_dtype
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"out_dtype {out_dtype} not supported")
    w = topk_weights
    if w.dtype not in (torch.bfloat16, torch.float32):
        w = w.to(torch.float32)
    return ops.combine(x.contiguous(), indices.to(torch.int32).reshape(-1), w.contiguous(),
                       int(topk), out_dtype == torch.float32)


def combine_xla(x: torch.Tensor, indices: torch.Tensor, topk_weights: torch.Tensor, topk: int,
                out_dtype=None) -> torch.Tensor:
    """KC:44-54 (mode 1)."""
    return _combine(x, indices, topk_weights, topk, out_dtype)


def pallas_supported(x: torch.Tensor, num_tokens: int, topk: int, tm: int = 64) -> bool:
    """KC:125-135 counterpart: bf16/f32 [N, H] with H % 8 == 0."""
    return (x.dim() == 2 and x.dtype in (torch.bfloat16, torch.float32)
            and x.shape[1] % 8 == 0)


def combine_pallas(x, indices, topk_weights, topk, out_dtype=None, tm: int = 64,
                   interpret: bool = False) -> torch.Tensor:
    """KC:140-198 (mode 2); same kernel as ``combine_xla``."""
    return _combine(x, indices, topk_weights, topk, out_dtype)


def fast_combine(x: torch.Tensor, indices: torch.Tensor, topk_weights: torch.Tensor, topk: int,
                 mode: int, out_dtype=None) -> torch.Tensor:
    """KC:201-207: dispatch on the MOE_FAST_COMBINE mode."""
    if mode not in (1, 2):
        raise ValueError(f"MOE_FAST_COMBINE mode must be 1 or 2, got {mode}")
    return _combine(x, indices, topk_weights, topk, out_dtype)


def combine_shared(x: torch.Tensor, indices: torch.Tensor, topk_weights: torch.Tensor, topk: int,
                   shared_partial: torch.Tensor, routed_scale: float = 1.0,
                   f32_reduce: bool = False, out_dtype=torch.bfloat16) -> torch.Tensor:
    """The combine with the shared expert's output (or this shard's partial
    of it) summed in, as MOE_SHARED_EXPERT_TP does before its reduce
    (X0104:80-87): out = dtype(f32(routed) * routed_scale + shared_partial),
    the routed k-order sum first rounded to bf16 unless ``f32_reduce``
    (MOE_F32_REDUCE keeps it f32)."""
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"out_dtype {out_dtype} not supported")
    w = topk_weights
    if w.dtype not in (torch.bfloat16, torch.float32):
        w = w.to(torch.float32)
    sh = shared_partial
    if sh.dtype not in (torch.bfloat16, torch.float32):
        sh = sh.to(torch.float32)
    t = w.shape[0]
    out = torch.empty((t, x.shape[1]), dtype=out_dtype, device=x.device)
    return ops.combine_shared_out(x.contiguous(), indices.to(torch.int32).reshape(-1),
                                  w.contiguous(), int(topk), sh.contiguous(), out,
                                  routed_scale=routed_scale,
                                  mid_dtype=torch.float32 if f32_reduce else torch.bfloat16)
