"""CPU oracle for the FP4 expert-parallel MoE path (test infrastructure only).

This package is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it.
The CUDA library in ``dw_tpu_b200`` never calls into it and fails loudly when
its extension is missing.
"""

from .moe_oracle import *  # noqa: F401,F403
