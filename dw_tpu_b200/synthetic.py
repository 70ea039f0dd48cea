"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (the reference measures this path on no public
dataset; BASELINE.json's configs fix shapes and distributions):

* cfg0  FP4 grouped matmul: lhs N(0,1) bf16 [256, 512], group sizes
        Multinomial(256, uniform over 8), e2m1 nibbles uniform over all 16
        codes [8, 512, 1024], E8M0 exponents uniform in [-4, 2].
* cfg1  decode layer: T=64 tokens N(0,1) of H=4096, router bf16 [4096, 256]
        N(0, 0.02), 256 experts with I=2048, sigmoid top-8 renormalised.
* cfg2  EP routing: per-rank tokens, ids uniform or Zipf(1.2) without repeats
        per token, Dirichlet(1) f32 weights.
"""

from __future__ import annotations

import numpy as np
import torch

from .fused_moe import FP4MoEWeights

E8M0_LO, E8M0_HI = 127 - 4, 127 + 2  # exponents -4..2


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def random_fp4(shape_bytes, seed: int, device="cpu") -> torch.Tensor:
    """Packed e2m1 bytes with every nibble uniform over the 16 codes."""
    g = _gen(seed, device)
    return torch.randint(0, 256, shape_bytes, dtype=torch.uint8, generator=g, device=device)


def random_e8m0(shape, seed: int, device="cpu", lo=E8M0_LO, hi=E8M0_HI) -> torch.Tensor:
    g = _gen(seed, device)
    return torch.randint(lo, hi + 1, shape, dtype=torch.uint8, generator=g, device=device)


def multinomial_group_sizes(total: int, groups: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.multinomial(total, [1.0 / groups] * groups).astype(np.int32)


def cfg0(seed: int = 0, device="cpu", m=256, k=512, n=1024, groups=8):
    """(lhs bf16 [m,k], codes u8 [g,k,n/2], scales u8 [g,k/32,n], group_sizes i32)."""
    g = _gen(seed, device)
    lhs = torch.randn((m, k), generator=g, device=device).to(torch.bfloat16)
    codes = random_fp4((groups, k, n // 2), seed + 1, device)
    scales = random_e8m0((groups, k // 32, n), seed + 2, device)
    gs = torch.from_numpy(multinomial_group_sizes(m, groups, seed + 3)).to(device)
    return lhs, codes, scales, gs


def moe_weights(num_experts: int, hidden: int, inter: int, seed: int = 0,
                device="cpu") -> FP4MoEWeights:
    """FP4 expert weights with E8M0 scales drawn as in cfg0."""
    return FP4MoEWeights(
        w13=random_fp4((num_experts, hidden, inter), seed + 11, device),
        s13=random_e8m0((num_experts, hidden // 32, 2 * inter), seed + 12, device),
        w2=random_fp4((num_experts, inter, hidden // 2), seed + 13, device),
        s2=random_e8m0((num_experts, inter // 32, hidden), seed + 14, device),
    )


def layer_inputs(tokens: int, hidden: int, num_experts: int, seed: int = 0, device="cpu"):
    """(hidden bf16 [T, H] ~N(0,1), router weight bf16 [H, E] ~N(0, 0.02))."""
    g = _gen(seed + 21, device)
    x = torch.randn((tokens, hidden), generator=g, device=device).to(torch.bfloat16)
    router = (torch.randn((hidden, num_experts), generator=g, device=device) * 0.02).to(
        torch.bfloat16)
    return x, router


def route_ids(tokens: int, num_experts: int, top_k: int, seed: int = 0,
              dist: str = "uniform", zipf_s: float = 1.2):
    """cfg2 routing: top_k distinct expert ids per token (uniform or Zipf(s)
    over a seeded random expert ranking) and Dirichlet(1) f32 weights."""
    rng = np.random.default_rng(seed)
    if dist == "uniform":
        p = np.full(num_experts, 1.0 / num_experts)
    elif dist == "zipf":
        ranks = np.arange(1, num_experts + 1, dtype=np.float64)
        p = ranks ** (-zipf_s)
        p /= p.sum()
        p = p[rng.permutation(num_experts)]
    else:
        raise ValueError(dist)
    ids = np.empty((tokens, top_k), np.int32)
    for t in range(tokens):
        ids[t] = rng.choice(num_experts, size=top_k, replace=False, p=p)
    w = rng.dirichlet(np.ones(top_k), size=tokens).astype(np.float32)
    return ids, w
