"""uint8 exponent storage for power-of-two f32 scales (KE:14-40), on the GPU.

Code c in 1..254 stands for 2**(c - 127), code 0 for +0.0; decoding is a
shift, so it reproduces the stored f32 bits for every scale ``e8m0_encode``
accepts.
"""

from __future__ import annotations

import torch

from . import ops


def e8m0_encode(scale: torch.Tensor):
    """KE:28-34: f32 scale -> (uint8 codes, lossless flag as a 0-d bool)."""
    s = scale.to(torch.float32).contiguous()
    codes = torch.empty(s.shape, dtype=torch.uint8, device=s.device)
    flag = torch.empty((), dtype=torch.int32, device=s.device)
    ops.e8m0_encode_out(s, codes, flag)
    return codes, flag.bool()


def e8m0_decode(codes: torch.Tensor) -> torch.Tensor:
    """KE:37-40: uint8 codes -> the exact f32 scales they encode."""
    c = codes.contiguous()
    out = torch.empty(c.shape, dtype=torch.float32, device=c.device)
    return ops.e8m0_decode_out(c, out)
