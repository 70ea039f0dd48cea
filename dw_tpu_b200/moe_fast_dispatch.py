"""MOE_FAST_DISPATCH on B200 (KD, call site X0405:70-98).

Every mode runs the same CUDA kernels; the results are bitwise identical to
``hidden[arange(T).repeat(topk)[argsort]]`` as the reference's modes are.
Unlike the Pallas kernel there is no shape fallback: any bf16 [T, H] with
H % 8 == 0 is taken, anything else raises ValueError.
"""

from __future__ import annotations

import torch

from . import ops


def sorted_token_indices(topk_argsort_indices: torch.Tensor, topk: int) -> torch.Tensor:
    """KD:41-44: argsort // topk (int32)."""
    src = topk_argsort_indices.to(torch.int32).contiguous()
    out = torch.empty_like(src)
    return ops.sorted_token_indices_out(src, topk, out)


def moe_permute(topk_ids: torch.Tensor, num_experts: int):
    """The dispatch index work of X0405:73-88 in one kernel: stable argsort of
    the flattened ids, ``argsort // topk``, the revert (inverse) permutation
    used by the combine, and ``group_sizes = bincount(ids)``."""
    return ops.permute(topk_ids.to(torch.int32).contiguous(), int(num_experts))


def pallas_supported(hidden: torch.Tensor, num_rows: int, tm: int = 128) -> bool:
    """KD:127-131 counterpart: the CUDA gather takes every bf16 [T, H % 8]."""
    return hidden.dim() == 2 and hidden.dtype == torch.bfloat16 and hidden.shape[1] % 8 == 0


def dispatch_gather(hidden: torch.Tensor, token_indices_sorted: torch.Tensor) -> torch.Tensor:
    """KD:134-185: hidden[token_indices_sorted] (bitwise)."""
    return ops.dispatch_gather(hidden.contiguous(), token_indices_sorted.to(torch.int32))


def dispatch_gather_pallas(hidden, token_indices_sorted, tm: int = 128,
                           interpret: bool = False) -> torch.Tensor:
    """Name-compatible alias of ``dispatch_gather`` (KD:135)."""
    return dispatch_gather(hidden, token_indices_sorted)


def fast_dispatch_gather(hidden: torch.Tensor, topk_argsort_indices: torch.Tensor, topk: int,
                         mode: int) -> torch.Tensor:
    """KD:188-194: hidden[arange(T).repeat(topk)[argsort]], bitwise."""
    if mode not in (0, 1, 2):
        raise ValueError(f"MOE_FAST_DISPATCH mode must be 0, 1 or 2, got {mode}")
    tok = sorted_token_indices(topk_argsort_indices, topk)
    return dispatch_gather(hidden, tok)
