"""Regenerate the small golden fixtures in tests/golden/ (``python
tests/golden/make_golden.py``).

The reference's own path is JAX/Pallas on TPU and cannot run in this
environment (no jax, jaxlib, tokamax or libtpu), so fixtures come from the
NumPy oracle in ``oracle/``, whose decode table is cross-checked against
ml_dtypes' float4_e2m1fn here. Inputs are seeded and every file stays small.
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import moe_oracle as O  # noqa: E402


def _bf16_bits(x):
    return O.f32_to_bf16_bits(np.asarray(x, np.float32))


def e2m1_table():
    nib = np.arange(16, dtype=np.uint8)
    try:
        import ml_dtypes
        ref = nib.view(ml_dtypes.float4_e2m1fn).astype(np.float32)
        assert np.array_equal(ref, O.e2m1_decode(nib), equal_nan=True)
    except ImportError:
        pass
    codes = O.e2m1_to_codes(nib)
    return dict(nibbles=nib, values=O.e2m1_decode(nib), tokamax_codes=codes,
                tokamax_decoded=O.decode_codes(codes))


def gmm_small(seed=7, m=80, k=128, n=256, groups=4, scale_lo=123, scale_hi=129):
    rng = np.random.default_rng(seed)
    lhs = O.round_bf16(rng.standard_normal((m, k)).astype(np.float32))
    packed = rng.integers(0, 256, (groups, k, n // 2), dtype=np.uint8)
    scales = rng.integers(scale_lo, scale_hi + 1, (groups, k // 32, n), dtype=np.uint8)
    gs = rng.multinomial(m - 5, [1.0 / groups] * groups).astype(np.int32)  # 5 pad rows
    deq = O.dequant_fp4_block(packed, scales)
    out_ref, valid = O.gmm_ref(lhs, packed, scales, gs)
    out_f32, _ = O.gmm_f32(lhs, packed, scales, gs)
    act_ref, _ = O.gmm_ref(lhs, packed, scales, gs, act="swiglu")
    return dict(lhs_bits=_bf16_bits(lhs), packed=packed, scales=scales, group_sizes=gs,
                dequant_bits=_bf16_bits(deq), out_ref_bits=_bf16_bits(out_ref),
                out_f32=out_f32, valid=valid, swiglu_ref_bits=_bf16_bits(act_ref))


def permute_small(seed=11, t=37, topk=8, e=16):
    rng = np.random.default_rng(seed)
    ids = np.stack([rng.choice(e, topk, replace=False) for _ in range(t)]).astype(np.int32)
    argsort, tok, revert, gs = O.permute(ids, e)
    hidden = O.round_bf16(rng.standard_normal((t, 64)).astype(np.float32))
    x = O.dispatch_gather(hidden, tok)
    return dict(ids=ids, argsort=argsort, tok=tok, revert=revert, group_sizes=gs,
                hidden_bits=_bf16_bits(hidden), x_bits=_bf16_bits(x))


def combine_small(seed=13, t=19, topk=6, h=64):
    rng = np.random.default_rng(seed)
    rows = t * topk
    y = O.round_bf16(rng.standard_normal((rows, h)).astype(np.float32))
    idx = rng.permutation(rows).astype(np.int32)
    w = rng.dirichlet(np.ones(topk), size=t).astype(np.float32)
    out = O.combine(y, idx, w, topk)
    out_f32 = O.combine(y, idx, w, topk, out_dtype="f32")
    return dict(y_bits=_bf16_bits(y), idx=idx, w=w, out_bits=_bf16_bits(out), out_f32=out_f32)


def route_small(seed=17, t=24, e=64, topk=8):
    rng = np.random.default_rng(seed)
    logits = O.round_bf16((rng.standard_normal((t, e)) * 2).astype(np.float32))
    res = {"logits_bits": _bf16_bits(logits)}
    for fn in ("sigmoid", "softmax", "sqrtsoftplus"):
        ids, w = O.route_topk(logits, topk, fn, True)
        res[f"{fn}_ids"] = ids
        res[f"{fn}_w"] = w
    return res


def requant_kat(seed=0):
    """Inputs/outputs of the restated B01:131-157 known-answer test."""
    rng = np.random.default_rng(seed)
    shape = (4, 64, 256)
    nib = rng.integers(0, 16, shape, dtype=np.uint8)
    exps = rng.integers(-20, 5, shape[:-1] + (shape[-1] // 32,))
    scale = np.ldexp(np.ones(exps.shape, np.float32), exps).astype(np.float32)
    original = O.dequantize_fp4_block32(nib, scale)
    q, s = O.quantize_fp4_block32(original, power_of_two_scale=True)
    return dict(nibbles=nib, scale=scale, original=original, q_nibbles=q, q_scale=s)


FIXTURES = {
    "e2m1_table": e2m1_table,
    "gmm_small": gmm_small,
    "permute_small": permute_small,
    "combine_small": combine_small,
    "route_small": route_small,
    "requant_kat": requant_kat,
}


def main():
    for name, fn in FIXTURES.items():
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **fn())
        print(f"{path}: {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
