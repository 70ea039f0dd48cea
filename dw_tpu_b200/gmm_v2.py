"""tokamax ``gmm_v2`` FP4 surface on B200 (TK:107-153) and ``gmm_wrapper``.

The reference decodes fp4 in-kernel from uint4 codes on TPUs without fp4
vectors (TK:9-14) and re-encodes stored weights once at load time into the
codes its kernel decodes fastest (B01:276-299). On B200 the e2m1 weights are
decoded on the SM, either from raw OCP nibbles packed two per byte along N
(element 2j in the low nibble, ``rhs_layout="e2m1"``; tcgen05 kernel) or,
faster, from the same nibbles re-laid once at load time into MMA-fragment
order with their bits permuted for a one-PRMT decode
(``fp4_weight_to_codes``, ``rhs_layout="b200"``; mma.sync kernel for
decode-sized groups, tcgen05 kernel for larger ones). tokamax codes (``rhs_fp4_codes=True``) are still
accepted and converted back to e2m1 per call, an extra pass over the weights,
like the reference's per-call re-encoding of float4 rhs (the docstring at
TK:107-125); convert them once with ``codes_to_e2m1`` instead.
"""

from __future__ import annotations

import torch

from . import _lib as L
from . import ops

_FP4X2 = getattr(torch, "float4_e2m1fn_x2", None)

_ACTS = {
    None: L.ACT_NONE,
    "silu": L.ACT_SWIGLU,
    "swiglu": L.ACT_SWIGLU,
    "silu_and_mul": L.ACT_SWIGLU,
    "silu_and_mul_with_clamp": L.ACT_SWIGLU_CLAMP,
    "swiglu_clamp": L.ACT_SWIGLU_CLAMP,
}


def needs_fp4_emulation(dtype) -> bool:
    """TK:9-14 counterpart: B200 never needs the uint4 code re-encoding."""
    return False


def e2m1_to_codes(rhs: torch.Tensor) -> torch.Tensor:
    """tokamax re-encoding (TK:17-30) of packed e2m1 nibbles, on the GPU."""
    out = torch.empty_like(ops._u8view(rhs))
    return ops.fp4_codes_convert_out(rhs, out, L.FP4_E2M1, L.FP4_TOKAMAX)


def codes_to_e2m1(codes: torch.Tensor) -> torch.Tensor:
    """Inverse of ``e2m1_to_codes`` (tokamax codes -> packed e2m1 nibbles)."""
    out = torch.empty_like(ops._u8view(codes))
    return ops.fp4_codes_convert_out(codes, out, L.FP4_TOKAMAX, L.FP4_E2M1)


def fp4_weight_to_codes(weight: torch.Tensor) -> torch.Tensor:
    """B01:276-299 counterpart: re-lay packed e2m1 weights [G, K, N/2] once, at
    load time, into the B200 decode layout (u32 words [G][N/16][K/16][32], one
    m16n8k16 A fragment per word, bits permuted for a one-PRMT decode; bytes
    shaped [G, N, K/2]; pass ``rhs_layout="b200"`` to ``gmm_v2``). Lossless: ``b200_to_e2m1`` undoes it."""
    return ops.fp4_to_b200_out(weight)


def b200_to_e2m1(codes: torch.Tensor) -> torch.Tensor:
    """Inverse of ``fp4_weight_to_codes``: [G, N, K/2] -> raw [G, K, N/2]."""
    return ops.fp4_to_b200_out(codes, inverse=True)


def decode_codes(codes: torch.Tensor, scales: torch.Tensor, layout: str = "e2m1") -> torch.Tensor:
    """Dequantise FP4 weights ([G, K, N/2] raw, or [G, N, K/2] "b200") with
    scales [G, K/32, (1,) N] to bf16 [G, K, N] in the reference order (TK:33-41
    decode, E0901:84-95 scale)."""
    c = ops._u8view(codes)
    g, k, n = ops.fp4_dims(c, layout)
    out = torch.empty((g, k, n), dtype=torch.bfloat16, device=c.device)
    return ops.fp4_dequant_out(c, scales.contiguous(), out, layout=layout)


def _act_code(fuse_act) -> int:
    if fuse_act not in _ACTS:
        raise ValueError(f"fuse_act {fuse_act!r} not supported "
                         f"(one of {sorted(k for k in _ACTS if k)})")
    return _ACTS[fuse_act]


def gmm_v2(lhs: torch.Tensor, rhs: torch.Tensor, group_sizes: torch.Tensor,
           rhs_scale: torch.Tensor | None = None, *, group_offset=None,
           zero_initialize: bool = True, fuse_act: str | None = None,
           preferred_element_type: torch.dtype | None = None, transpose_rhs: bool = False,
           rhs_fp4_codes: bool = False, act_limit: float | None = None,
           rhs_layout: str = "e2m1") -> torch.Tensor:
    """Grouped matmul ``out[rows_g] = lhs[rows_g] @ dequant(rhs[g])``.

    lhs bf16 [M, K] (rows sorted by group); rhs FP4 [G_local, K, N/2] (uint8 or
    float4_e2m1fn_x2); rhs_scale [G_local, K/32, (1,) N] as uint8 E8M0 /
    float8_e8m0fnu, bf16 or f32; group_sizes int32 [num_groups]; group_offset
    selects which groups the local rhs holds. fuse_act applies SwiGLU to the
    [gate | up] halves. Output [M, N or N/2] in preferred_element_type (bf16 by
    default). ``rhs_layout="b200"`` takes weights re-laid by
    ``fp4_weight_to_codes`` (faster decode, identical results). Raises
    ValueError on shapes the kernel does not take, like TK:132-134 does for a
    non-uint4 rhs with rhs_fp4_codes.
    """
    if rhs_fp4_codes and rhs_layout != "e2m1":
        raise ValueError("rhs_fp4_codes (tokamax codes) implies rhs_layout='e2m1'")
    if transpose_rhs:
        raise ValueError("transpose_rhs is not supported: store rhs as [G, K, N/2]")
    if rhs_scale is None:
        raise ValueError("FP4 rhs needs rhs_scale (per-32 block scales)")
    if lhs.dtype != torch.bfloat16:
        raise ValueError(f"lhs must be bf16, got {lhs.dtype}")
    if rhs.dtype not in (torch.uint8, _FP4X2):
        raise ValueError(f"rhs must hold packed fp4 (uint8 / float4_e2m1fn_x2), got {rhs.dtype}")
    codes = codes_to_e2m1(rhs) if rhs_fp4_codes else rhs
    out_dt = preferred_element_type or torch.bfloat16
    if out_dt not in (torch.bfloat16, torch.float32):
        raise ValueError(f"preferred_element_type {out_dt} not supported")
    act = _act_code(fuse_act)
    if act == L.ACT_SWIGLU_CLAMP and act_limit is None:
        raise ValueError("silu_and_mul_with_clamp needs act_limit")
    go = 0 if group_offset is None else int(group_offset)
    return ops.gmm_fp4(lhs.contiguous(), codes.contiguous(), rhs_scale.contiguous(),
                       group_sizes.to(torch.int32).contiguous(), go, codes.shape[0], act,
                       float(act_limit or 0.0), out_dt == torch.float32, bool(zero_initialize),
                       rhs_layout)


def gmm(lhs, rhs_codes, rhs_scales, group_sizes, **kw) -> torch.Tensor:
    """North-star surface ``gmm(lhs, rhs_codes, rhs_scales, group_sizes)``."""
    return gmm_v2(lhs, rhs_codes, group_sizes, rhs_scales, **kw)


def gmm_wrapper(lhs, rhs, rhs_scale, rhs_bias, group_sizes, group_offset, fuse_act=None,
                preferred_element_type=None, act_limit=None, rhs_layout="e2m1"):
    """B01:218-232 (+X0401:56-64, X0403:64-70): gmm_v2 with
    zero_initialize=False; uint8 / bf16 scales are consumed directly (the
    kernel casts every scale to bf16, which is what widening to f32 and the
    in-kernel cast produce for power-of-two scales)."""
    if rhs_bias is not None:
        raise ValueError("rhs_bias is not supported by the FP4 grouped GEMM")
    return gmm_v2(lhs, rhs, group_sizes, rhs_scale, group_offset=group_offset,
                  zero_initialize=False, fuse_act=fuse_act,
                  preferred_element_type=preferred_element_type, act_limit=act_limit,
                  rhs_layout=rhs_layout)
