"""Top-k routing on B200, as fused_moe_func computes it for the GMM path
(E0901:656-687; weights cast to the activation dtype, X0101:131)."""

from __future__ import annotations

import torch

from . import ops


def route_topk(gating_output: torch.Tensor, top_k: int, renormalize: bool = True,
               scoring_fn: str = "sigmoid", dtype: torch.dtype = torch.bfloat16,
               bias: torch.Tensor | None = None, num_valid_tokens: int | None = None):
    """Returns (topk_weights in ``dtype``, topk_ids int32) like
    ``_fused_moe_fp4_routing``: scores in f32, ties to the lower expert index,
    bias for selection only, renormalised, rows >= num_valid_tokens -> expert
    0 with weight 0."""
    logits = gating_output.contiguous()
    if logits.dtype not in (torch.bfloat16, torch.float32):
        logits = logits.float()
    t = logits.shape[0]
    ids = torch.empty((t, top_k), dtype=torch.int32, device=logits.device)
    w32 = torch.empty((t, top_k), dtype=torch.float32, device=logits.device)
    w16 = (torch.empty((t, top_k), dtype=torch.bfloat16, device=logits.device)
           if dtype == torch.bfloat16 else None)
    ops.route_topk_out(logits, top_k, ids, w32_out=w32, w16_out=w16, scoring_fn=scoring_fn,
                       renormalize=renormalize,
                       bias=None if bias is None else bias.float().contiguous(),
                       num_valid_tokens=num_valid_tokens)
    if dtype == torch.bfloat16:
        return w16, ids
    return w32.to(dtype), ids


def route_hash(gating_output: torch.Tensor, hash_ids: torch.Tensor, renormalize: bool = True,
               scoring_fn: str = "sigmoid", dtype: torch.dtype = torch.bfloat16,
               num_valid_tokens: int | None = None):
    """Hash routing of ``_fused_moe_fp4_routing`` (E0901:667-671): the ids
    are ``hash_ids`` [t, top_k]; the weights are the scores at those ids,
    renormalised, padding rows -> expert 0 with weight 0."""
    logits = gating_output.contiguous()
    if logits.dtype not in (torch.bfloat16, torch.float32):
        logits = logits.float()
    t, top_k = hash_ids.shape
    ids = torch.empty((t, top_k), dtype=torch.int32, device=logits.device)
    w32 = torch.empty((t, top_k), dtype=torch.float32, device=logits.device)
    ops.route_hash_out(logits, hash_ids.to(torch.int32).contiguous(), ids, w32,
                       scoring_fn=scoring_fn, renormalize=renormalize,
                       num_valid_tokens=num_valid_tokens)
    return w32.to(dtype), ids


def dedupe_topk(topk_weights: torch.Tensor, topk_ids: torch.Tensor, num_experts: int):
    """E0901:98-121: makes each token's expert ids distinct. Returns new
    (f32 weights, int32 ids)."""
    w = topk_weights.float().contiguous().clone()
    ids = topk_ids.to(torch.int32).contiguous().clone()
    ops.dedupe_topk_(w, ids, num_experts)
    return w, ids
