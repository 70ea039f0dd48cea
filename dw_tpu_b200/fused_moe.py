"""The single-device MoE layer of the GMM path (fused_moe_func, call stack of
X0104:88-98 / X0405 / X0404 on one device), built from the CUDA ops:

    route (E0901:656-687) -> weights to bf16 (X0101:131)
    -> permute + gather (X0405:70-98, KD)
    -> gmm1 with fused SwiGLU (B01:218-232, TK)
    -> gmm2 (bf16, or f32 under MOE_F32_REDUCE, X0106:18-29)
    -> k-order combine (X0404:89-110, KC)

``MoELayer`` preallocates its workspace for a maximum token count so a whole
layer is 6 kernel launches with no allocation and can be captured in a CUDA
graph; ``fused_moe_func`` is the allocating functional form.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib as L
from . import ops


@dataclass
class FP4MoEWeights:
    """Expert weights in the stored layouts of X0103:240-245 / E0901:250-253
    (scale unit dim dropped): w13 [E, H, 2I] = [gate | up] as packed e2m1
    bytes [E, H, I]; s13 [E, H/32, 2I]; w2 bytes [E, I, H/2]; s2 [E, I/32, H].
    Scales are uint8 E8M0 codes, bf16 or f32. ``layout`` is "e2m1" (raw
    nibbles) or "b200" (re-laid once for the faster decode, ``to_b200``)."""

    w13: torch.Tensor
    s13: torch.Tensor
    w2: torch.Tensor
    s2: torch.Tensor
    layout: str = "e2m1"

    def to_b200(self) -> "FP4MoEWeights":
        """Load-time re-layout of both projections into the B200 decode layout
        (w13 [E, 2I, H/2], w2 [E, H, I/2]; B01:276-299 counterpart)."""
        if self.layout == "b200":
            return self
        return FP4MoEWeights(ops.fp4_to_b200_out(self.w13), self.s13,
                             ops.fp4_to_b200_out(self.w2), self.s2, "b200")

    @classmethod
    def from_dense(cls, w13: torch.Tensor, w2: torch.Tensor) -> "FP4MoEWeights":
        """Weight preparation on the device: dense (or dequantised MXFP4)
        expert weights w13 [E, H, 2I] and w2 [E, I, H] (bf16 / f32) re-quantised
        with quantize_tensor(float4_e2m1fn, block 32, power_of_two_scale=True)
        (B01:319-347) into packed e2m1 codes and E8M0 scales (KE:28-40), the
        layouts the grouped matmul reads. Raises if a scale does not fit E8M0
        (a block whose scale is not a normal power of two)."""
        out = []
        for w in (w13, w2):
            e, k, n = w.shape
            codes = torch.empty((e, k, n // 2), dtype=torch.uint8, device=w.device)
            scales = torch.empty((e, k // 32, n), dtype=torch.uint8, device=w.device)
            lossless = torch.empty(1, dtype=torch.int32, device=w.device)
            ops.fp4_quantize_out(w.contiguous(), codes, scales, lossless)
            if int(lossless.item()) != 1:
                raise ValueError("a block scale is not a normal power of two; keep f32 scales")
            out += [codes, scales]
        return cls(out[0], out[1], out[2], out[3])

    @property
    def num_experts(self) -> int:
        return self.s13.shape[0]

    @property
    def hidden_size(self) -> int:
        return self.s13.shape[1] * 32

    @property
    def intermediate_size(self) -> int:
        return self.s2.shape[1] * 32

    def weight_bytes_per_expert(self) -> int:
        per = lambda t: t.numel() * t.element_size() // t.shape[0]  # noqa: E731
        return per(self.w13) + per(self.s13) + per(self.w2) + per(self.s2)


class MoELayer:
    """Single-device FP4 MoE layer with a preallocated workspace."""

    def __init__(self, weights: FP4MoEWeights, top_k: int, max_tokens: int, *,
                 scoring_fn: str = "sigmoid", renormalize: bool = True,
                 act_limit: float | None = None, f32_reduce: bool = False,
                 device: torch.device | str = "cuda", gemm_variant: int = 0):
        self.w = weights
        self.top_k = int(top_k)
        self.max_tokens = int(max_tokens)
        self.scoring_fn = scoring_fn
        self.renormalize = renormalize
        self.act = L.ACT_SWIGLU if act_limit is None else L.ACT_SWIGLU_CLAMP
        self.act_limit = 0.0 if act_limit is None else float(act_limit)
        self.f32_reduce = f32_reduce
        self.gemm_variant = int(gemm_variant)  # 0: chosen per call (dwm_gmm_fp4_variant)
        e, h, i = weights.num_experts, weights.hidden_size, weights.intermediate_size
        rows = self.max_tokens * self.top_k
        dev = torch.device(device)
        self.ids = torch.empty((self.max_tokens, self.top_k), dtype=torch.int32, device=dev)
        self.w16 = torch.empty((self.max_tokens, self.top_k), dtype=torch.bfloat16, device=dev)
        self.tok = torch.empty(rows, dtype=torch.int32, device=dev)
        self.revert = torch.empty(rows, dtype=torch.int32, device=dev)
        self.group_sizes = torch.empty(e, dtype=torch.int32, device=dev)
        self.x = torch.empty((rows, h), dtype=torch.bfloat16, device=dev)
        self.h1 = torch.empty((rows, i), dtype=torch.bfloat16, device=dev)
        self.y = torch.empty((rows, h), dtype=torch.float32 if f32_reduce else torch.bfloat16,
                             device=dev)

    kernels_per_forward = 6

    def forward(self, hidden: torch.Tensor, logits: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
        t = hidden.shape[0]
        if t > self.max_tokens:
            raise ValueError(f"{t} tokens exceed max_tokens={self.max_tokens}")
        rows = t * self.top_k
        ids, w16 = self.ids[:t], self.w16[:t]
        ops.route_topk_out(logits, self.top_k, ids, w16_out=w16, scoring_fn=self.scoring_fn,
                           renormalize=self.renormalize)
        ops.permute_out(ids, self.w.num_experts, self.group_sizes,
                        token_indices_sorted=self.tok[:rows], revert=self.revert[:rows])
        x = self.x[:rows]
        ops.dispatch_gather_out(hidden, self.tok[:rows], x)
        h1 = self.h1[:rows]
        ops.gmm_fp4_out(x, self.w.w13, self.w.s13, self.group_sizes, h1, act=self.act,
                        act_limit=self.act_limit, layout=self.w.layout,
                        variant=self.gemm_variant)
        y = self.y[:rows]
        ops.gmm_fp4_out(h1, self.w.w2, self.w.s2, self.group_sizes, y, layout=self.w.layout,
                        variant=self.gemm_variant)
        if out is None:
            out = torch.empty((t, self.w.hidden_size), dtype=torch.bfloat16,
                              device=hidden.device)
        ops.combine_out(y, self.revert[:rows], w16, self.top_k, out)
        return out

    __call__ = forward


def fused_moe_func(hidden_states: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor,
                   w13_scale: torch.Tensor, w2_scale: torch.Tensor,
                   gating_output: torch.Tensor, topk: int, renormalize: bool = True,
                   scoring_fn: str = "sigmoid", act_limit: float | None = None,
                   f32_reduce: bool = False) -> torch.Tensor:
    """Functional single-device MoE layer (allocates its workspace)."""
    weights = FP4MoEWeights(w13, w13_scale, w2, w2_scale)
    layer = MoELayer(weights, topk, hidden_states.shape[0], scoring_fn=scoring_fn,
                     renormalize=renormalize, act_limit=act_limit, f32_reduce=f32_reduce,
                     device=hidden_states.device)
    return layer(hidden_states.contiguous(), gating_output.contiguous())
