"""The timed CPU baseline of the MoE layer (test and benchmark infrastructure).

The reference's own CPU path (JAX on CPU: ``decode_codes`` x scale,
``jax.lax.ragged_dot``, ``hidden[argsort // k]``, ``combine_xla``) cannot run
here: JAX, jaxlib and tokamax are not installed. This module restates the same
layer with the same arithmetic as ``moe_oracle.fused_moe`` and is organised
for speed so that a whole cfg1 layer fits a benchmark step:

* routing, permute, gather and the k-order combine are the oracle's own
  functions (E0901:656-687, KD:41-44, KC:44-54);
* the FP4 dequant (TK:33-41 table, E0901:84-95 order) reads each packed byte
  through a 256-entry table of its two e2m1 values, then multiplies by the
  E8M0 scale 2^(c-127) in f32; the product of an e2m1 value and a power of two
  is exact, and is rounded to bf16 as the reference's bf16 multiply does
  whenever a scale code could leave the exact range;
* each expert's two matmuls are f32 BLAS products (the reference's f32
  accumulation), SwiGLU in f32, gmm outputs rounded to bf16;
* experts run on a thread pool, one BLAS thread per worker, with per-thread
  buffers reused across experts.

``tests/test_oracle.py`` pins ``layer_forward`` against ``fused_moe``.
"""

from __future__ import annotations

import os
import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from . import moe_oracle as O

# The two e2m1 values of every packed byte: element 2j in the low nibble.
_E2M1 = O.e2m1_decode(np.arange(16, dtype=np.uint8)).astype(np.float32)
PAIR_LUT = np.stack([_E2M1[np.arange(256) & 15], _E2M1[np.arange(256) >> 4]], axis=1)


class _Buffers(threading.local):
    def get(self, name, shape):
        buf = getattr(self, name, None)
        if buf is None or buf.shape != shape:
            buf = np.empty(shape, np.float32)
            setattr(self, name, buf)
        return buf


_TLS = _Buffers()


def dequant_fp4_lut(packed: np.ndarray, scales: np.ndarray, tag: str = "w") -> np.ndarray:
    """bf16(e2m1 value x E8M0 scale) as f32 [K, N] from packed bytes [K, N/2]
    and E8M0 codes [K/32, N]; the same values as ``moe_oracle.dequant_fp4_block``.
    The result lives in a per-thread buffer (valid until the next call with
    the same tag on this thread)."""
    k, n2 = packed.shape
    n = 2 * n2
    v = _TLS.get(tag + "_v", (k, n2, 2))
    np.take(PAIR_LUT, packed, axis=0, out=v)
    s = (scales.astype(np.uint32) << np.uint32(23)).view(np.float32)  # 2^(c-127); 0 -> +0
    w = _TLS.get(tag, (k, n))
    np.multiply(v.reshape(k // 32, 32, n), s[:, None, :], out=w.reshape(k // 32, 32, n))
    lo, hi = int(scales.min()), int(scales.max())
    if lo < 3 or hi > 250:  # value * scale may be subnormal or overflow in bf16
        w[...] = O.round_bf16(w)
    return w


def layer_forward(hidden, logits, w13, s13, w2, s2, top_k: int, *, scoring_fn="sigmoid",
                  renormalize=True, pool: ThreadPoolExecutor | None = None):
    """The cfg1 layer on the host: hidden [T, H] and logits [T, E] (bf16
    values as f32), packed e2m1 w13 [E, H, I] / w2 [E, I, H/2] with E8M0
    scales s13 [E, H/32, 2I] / s2 [E, I/32, H] -> out [T, H] (bf16 values as
    f32). ``pool`` runs the experts (default: a pool over all host cores)."""
    ids, w = O.route_topk(logits, top_k, scoring_fn, renormalize)
    w_bf = O.round_bf16(w)
    e = w13.shape[0]
    inter = s2.shape[1] * 32
    _, tok, revert, gs = O.permute(ids, e)
    x = np.ascontiguousarray(O.dispatch_gather(O.round_bf16(np.asarray(hidden, np.float32)), tok),
                             dtype=np.float32)
    starts = np.concatenate([[0], np.cumsum(gs)[:-1]]).astype(np.int64)
    y = np.empty((x.shape[0], w2.shape[1] * 2), np.float32)

    def expert(ex):
        r0, r1 = int(starts[ex]), int(starts[ex] + gs[ex])
        h1 = x[r0:r1] @ dequant_fp4_lut(w13[ex], s13[ex], "w13")
        a = O.round_bf16(O.silu_and_mul(h1[:, :inter], h1[:, inter:]))
        y[r0:r1] = O.round_bf16(a @ dequant_fp4_lut(w2[ex], s2[ex], "w2"))

    active = [int(ex) for ex in np.nonzero(gs)[0]]
    if pool is None:
        with ThreadPoolExecutor(max_workers=os.cpu_count() or 1) as p:
            list(p.map(expert, active))
    else:
        list(pool.map(expert, active))
    return O.combine(y, revert, w_bf, top_k)


def make_pool(threads: int | None = None):
    """(executor, threads): a pool over the host cores whose workers each use
    one BLAS thread (the experts, not the BLAS calls, run in parallel)."""
    n = threads or os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(1)
    except ImportError:  # pragma: no cover
        pass
    return ThreadPoolExecutor(max_workers=n), n
