"""B200-native FP4 expert-parallel MoE hot path of dw-tpu.

CUDA kernels for sm_100a behind the C ABI in include/dw_moe.h
(libdw_moe.so, loaded through ctypes), exposed with the reference's operator
names:

* ``gmm_v2`` / ``gmm`` / ``gmm_wrapper``   tokamax FP4 grouped matmul
* ``fast_dispatch_gather``, ``sorted_token_indices``, ``moe_permute``
* ``fast_combine``, ``combine_xla``, ``combine_pallas``
* ``e8m0_encode`` / ``e8m0_decode``
* ``route_topk``, ``MoELayer`` / ``fused_moe_func``

Importing the package checks that the library has been built and raises if
it is missing; the library itself is mapped on the first op call. There is no
CPU or library fallback.
"""

from . import _lib

_lib.require_built()

from .e8m0_scale import e8m0_decode, e8m0_encode  # noqa: E402
from .fused_moe import FP4MoEWeights, MoELayer, fused_moe_func  # noqa: E402
from .gmm_v2 import (b200_to_e2m1, codes_to_e2m1, decode_codes, e2m1_to_codes,  # noqa: E402
                     fp4_weight_to_codes, gmm, gmm_v2, gmm_wrapper, needs_fp4_emulation)
from .moe_fast_combine import (combine_pallas, combine_shared, combine_xla,  # noqa: E402
                               fast_combine)
from .moe_fast_dispatch import (dispatch_gather, dispatch_gather_pallas,  # noqa: E402
                                fast_dispatch_gather, moe_permute, sorted_token_indices)
from .routing import dedupe_topk, route_hash, route_topk  # noqa: E402

__all__ = [
    "gmm_v2", "gmm", "gmm_wrapper", "e2m1_to_codes", "codes_to_e2m1", "decode_codes",
    "fp4_weight_to_codes", "b200_to_e2m1", "needs_fp4_emulation", "fast_dispatch_gather",
    "sorted_token_indices", "moe_permute", "dispatch_gather", "dispatch_gather_pallas",
    "fast_combine", "combine_xla", "combine_pallas", "combine_shared", "e8m0_encode", "e8m0_decode",
    "route_topk", "route_hash", "dedupe_topk", "MoELayer", "FP4MoEWeights", "fused_moe_func",
]
