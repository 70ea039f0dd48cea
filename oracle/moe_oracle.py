"""NumPy restatement of the reference's FP4 MoE hot path (test infrastructure).

This module is the CPU oracle the CUDA path is checked against. It is not the
product: only tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline may call it.

Every function cites the reference line it restates. Aliases (all paths
relative to the dw-tpu project root):

* TK    patches/tokamax/0001-gmm_v2-fp4-emulation-v6e.patch
* B01   patches/tpu-inference/0001-dsv4-v6e-enablement.patch
* KD    kernels/tpu_inference/layers/common/moe_fast_dispatch.py
* KC    kernels/tpu_inference/layers/common/moe_fast_combine.py
* KO    kernels/tpu_inference/kernels/collectives/oneshot.py
* KE    kernels/tpu_inference/layers/common/quantization/e8m0_scale.py
* E0901 patches/tpu-inference-experimental/fused-moe-fp4/0901-*.patch
* X01NN, X04NN  patches/tpu-inference-ext/01NN-*.patch, 04NN-*.patch

Pinning (what fixes this restatement to the reference):

* e2m1 decode: the 16-entry table is checked against ml_dtypes'
  ``float4_e2m1fn`` (an independent OCP implementation) and against the TK:36
  table "0 .5 1 1.5 2 3 4 6"; the tokamax code round trip TK:17-41 is exact.
* Power-of-two requant: the reference's own known-answer test B01:131-157 is
  restated in ``tests/test_oracle.py``.
* Permute: the KD:16-22,43 identity ``argsort // topk ==
  arange(T).repeat(topk)[argsort]`` is checked.
* Combine order, EP order, GEMM accumulation: restated from docstrings
  (KC:14-21, X0107:15-29, KO:26-30); the reference ships no golden vectors for
  these and its JAX path cannot run here, so they are "parity unpinned"
  beyond those identities.
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "E2M1_MAGNITUDES", "f32_to_bf16_bits", "bf16_bits_to_f32", "round_bf16",
    "pack_nibbles", "unpack_nibbles", "e2m1_decode", "e2m1_to_codes",
    "codes_to_e2m1", "decode_codes", "round_to_e2m1", "b200_swizzle",
    "b200_unswizzle", "to_b200_layout", "from_b200_layout", "e8m0_encode",
    "e8m0_decode", "scales_to_f32", "dequant_fp4_block", "dequant_fp4_f32",
    "gmm_f32", "gmm_ref", "silu_and_mul", "combine_shared", "quantize_fp4_block32",
    "dequantize_fp4_block32", "apply_scoring_fn", "route_topk",
    "sorted_token_indices", "permute", "dispatch_gather", "combine",
    "fused_moe", "ep_dispatch", "ep_combine_korder", "ep_combine_rankorder",
    "all_gather", "reduce_scatter_rank_order", "dedupe_topk", "route_hash",
]

# e2m1 magnitudes by 3-bit magnitude code (exponent<<1 | mantissa), TK:35-36.
E2M1_MAGNITUDES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0],
                           dtype=np.float32)


# ----------------------------------------------------------------------------
# bf16 helpers (round-to-nearest-even, like XLA's f32 -> bf16 convert)
# ----------------------------------------------------------------------------

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bit patterns (uint16), round to nearest even, NaN kept."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(x)
    out = rounded.astype(np.uint16)
    if nan.any():
        out = np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), out)
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> exact f32 values."""
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round f32 values to bf16 and return them as f32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# ----------------------------------------------------------------------------
# FP4 (e2m1) storage
# ----------------------------------------------------------------------------

def pack_nibbles(nib: np.ndarray) -> np.ndarray:
    """[..., N] 4-bit values -> [..., N/2] uint8, element 2j in the LOW nibble.

    This is the packing the C ABI consumes (two e2m1 values per byte along the
    last, N, dimension: XLA's uint4 pairing along the minor dim, X0103:210-220).
    """
    nib = np.asarray(nib, dtype=np.uint8)
    assert nib.shape[-1] % 2 == 0
    return (nib[..., 0::2] & 0xF) | ((nib[..., 1::2] & 0xF) << 4)


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    """Inverse of ``pack_nibbles``."""
    packed = np.asarray(packed, dtype=np.uint8)
    out = np.empty(packed.shape[:-1] + (packed.shape[-1] * 2,), np.uint8)
    out[..., 0::2] = packed & 0xF
    out[..., 1::2] = packed >> 4
    return out


def e2m1_decode(nib: np.ndarray) -> np.ndarray:
    """OCP e2m1 nibble (sign | exponent(2) | mantissa(1)) -> exact f32 value."""
    nib = np.asarray(nib, dtype=np.uint8)
    mag = E2M1_MAGNITUDES[nib & 7]
    return np.where(nib & 8, -mag, mag).astype(np.float32)


def e2m1_to_codes(nib: np.ndarray) -> np.ndarray:
    """tokamax re-encoding (TK:17-30): q = sign*(2e+m) as two's complement int4.

    -0 becomes +0. Returned as uint8 holding the 4-bit two's complement code.
    """
    c = np.asarray(nib, dtype=np.int16)
    q = np.where(c >= 8, -(c & 7), c & 7)
    return (q & 0xF).astype(np.uint8)


def codes_to_e2m1(codes: np.ndarray) -> np.ndarray:
    """Inverse of ``e2m1_to_codes`` (code 0 -> +0; code 8, i.e. -8, is not
    produced by the encoder and maps to -0)."""
    c = np.asarray(codes, dtype=np.int16) & 0xF
    q = np.where(c >= 8, c - 16, c)
    return np.where(q < 0, 8 | (-q & 7), q & 7).astype(np.uint8)


def decode_codes(codes: np.ndarray) -> np.ndarray:
    """TK:33-41: v = 2q - (clip(q,-6,6) + 0.5*clip(q,-4,4)), exact in bf16."""
    c = np.asarray(codes, dtype=np.int16) & 0xF
    q = np.where(c >= 8, c - 16, c).astype(np.float32)
    v = (q + q) - (np.clip(q, -6, 6) + np.float32(0.5) * np.clip(q, -4, 4))
    return v.astype(np.float32)


def round_to_e2m1(x: np.ndarray) -> np.ndarray:
    """f32 -> nearest e2m1 nibble, ties to even mantissa, saturating at 6.

    The float4_e2m1fn cast used by quantize_tensor (B01:319-347).
    """
    x = np.asarray(x, dtype=np.float32)
    mag = np.minimum(np.abs(x), np.float32(6.0))
    # Candidate codes below/above and the tie rule on the e2m1 grid.
    grid = E2M1_MAGNITUDES
    hi = np.searchsorted(grid, mag, side="left").clip(0, 7)
    lo = np.clip(hi - 1, 0, 7)
    d_lo = mag - grid[lo]
    d_hi = grid[hi] - mag
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & ((hi & 1) == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    code = np.where(mag == grid[hi], hi, code).astype(np.uint8)
    sign = (np.signbit(x) & (code != 0)).astype(np.uint8) << 3
    return (code | sign).astype(np.uint8)


def b200_swizzle(packed: np.ndarray) -> np.ndarray:
    """The B200 decode layout of packed e2m1 bytes: inside every 32-bit word
    (little-endian, 8 columns), output pair p = raw byte p moves its 2-bit
    fields (bits 1:0, 3:2 of the low nibble, 1:0, 3:2 of the high nibble) to
    bits B, B+4, B+8, B+12 with B = 0, 2, 16, 18 for p = 0..3. Not part of
    the reference: a lossless storage permutation (tests pin it as such)."""
    w = np.ascontiguousarray(packed, dtype=np.uint8).view(np.uint32)
    out = np.zeros_like(w)
    for p in range(4):
        byte = (w >> np.uint32(8 * p)) & np.uint32(0xFF)
        base = (p & 1) * 2 + (p >> 1) * 16
        for f in range(4):
            out |= ((byte >> np.uint32(2 * f)) & np.uint32(3)) << np.uint32(base + 4 * f)
    return out.view(np.uint8).reshape(np.asarray(packed).shape)


def b200_fragment_coords():
    """(dk, dc) of nibble j of word l inside a 16x16 (k, column) block: the
    A fragment of an m16n8k16 MMA for W^T (gid = l // 4, t = l % 4; columns
    gid, gid + 8; k pairs 2t, 2t + 8), nibble order
    (2t,gid) (2t+1,gid) (2t,gid+8) (2t+1,gid+8) then the same at k + 8."""
    l = np.arange(32)[:, None]
    j = np.arange(8)[None, :]
    gid, t = l >> 2, l & 3
    dk = 2 * t + (j & 1) + ((j >> 2) << 3)
    dc = gid + (((j >> 1) & 1) << 3)
    return dk, dc


def to_b200_layout(packed: np.ndarray) -> np.ndarray:
    """Raw e2m1 weights [g, k, n/2] -> the B200 layout, returned as uint8
    [g, n, k/2] (same byte count): u32 words [g][n/16][k/16][32], word l of
    block (cb, kb) holding the 8 nibbles ``b200_fragment_coords`` lists
    (nibble j in bits 4j..4j+3), then ``b200_swizzle`` on every word. Not part
    of the reference: a lossless load-time re-layout."""
    packed = np.asarray(packed, np.uint8)
    g, k, n2 = packed.shape
    n = 2 * n2
    nib = unpack_nibbles(packed).astype(np.uint32)          # [g, k, n]
    blocks = nib.reshape(g, k // 16, 16, n // 16, 16).transpose(0, 3, 1, 2, 4)
    dk, dc = b200_fragment_coords()
    sel = blocks[:, :, :, dk, dc]                            # [g, n/16, k/16, 32, 8]
    words = np.zeros(sel.shape[:-1], np.uint32)
    for j in range(8):
        words |= sel[..., j] << np.uint32(4 * j)
    raw = np.ascontiguousarray(words).view(np.uint8).reshape(g, n, k // 2)
    return b200_swizzle(raw)


def from_b200_layout(b200: np.ndarray) -> np.ndarray:
    """Inverse of ``to_b200_layout``."""
    b200 = np.asarray(b200, np.uint8)
    g, n, k2 = b200.shape
    k = 2 * k2
    words = np.ascontiguousarray(b200_unswizzle(b200)).view(np.uint32).reshape(
        g, n // 16, k // 16, 32)
    dk, dc = b200_fragment_coords()
    blocks = np.zeros((g, n // 16, k // 16, 16, 16), np.uint8)
    for j in range(8):
        blocks[:, :, :, dk[:, j], dc[:, j]] = (words >> np.uint32(4 * j)) & np.uint32(0xF)
    nib = blocks.transpose(0, 2, 3, 1, 4).reshape(g, k, n)
    return pack_nibbles(nib)


def b200_unswizzle(packed: np.ndarray) -> np.ndarray:
    """Inverse of ``b200_swizzle``."""
    o = np.ascontiguousarray(packed, dtype=np.uint8).view(np.uint32)
    w = np.zeros_like(o)
    for p in range(4):
        base = (p & 1) * 2 + (p >> 1) * 16
        byte = np.zeros_like(o)
        for f in range(4):
            byte |= ((o >> np.uint32(base + 4 * f)) & np.uint32(3)) << np.uint32(2 * f)
        w |= byte << np.uint32(8 * p)
    return w.view(np.uint8).reshape(np.asarray(packed).shape)


# ----------------------------------------------------------------------------
# E8M0 scales (KE:14-40)
# ----------------------------------------------------------------------------

_NON_E8M0_BITS = np.uint32(0x807FFFFF)


def e8m0_encode(scale: np.ndarray):
    """KE:28-34: f32 -> (uint8 exponent codes, lossless flag)."""
    bits = np.ascontiguousarray(scale, dtype=np.float32).view(np.uint32)
    exp = bits >> 23
    lossless = bool(np.all(((bits & _NON_E8M0_BITS) == 0) & (exp != 255)))
    return exp.astype(np.uint8), lossless


def e8m0_decode(codes: np.ndarray) -> np.ndarray:
    """KE:37-40: code c -> f32 with bits c << 23 (c = 0 -> +0)."""
    c = np.asarray(codes, dtype=np.uint32)
    return (c << 23).view(np.float32)


def scales_to_f32(scales: np.ndarray) -> np.ndarray:
    """gmm_wrapper's widening (X0401:56-64, X0403:64-70): u8 e8m0 / bf16 / f32
    scales -> exact f32. bf16 scales are passed as uint16 bit patterns."""
    s = np.asarray(scales)
    if s.dtype == np.uint8:
        return e8m0_decode(s)
    if s.dtype == np.uint16:
        return bf16_bits_to_f32(s)
    return s.astype(np.float32)


# ----------------------------------------------------------------------------
# Dequantisation and the grouped matmul (TK, E0901:84-95)
# ----------------------------------------------------------------------------

def dequant_fp4_block(packed: np.ndarray, scales: np.ndarray,
                      block: int = 32) -> np.ndarray:
    """E0901:84-95 order: decode to bf16, cast the scale to bf16, multiply in
    bf16 (one rounding). packed [..., K, N/2] uint8 e2m1; scales [..., K/32, N]
    (u8 e8m0, bf16 bits as uint16, or f32). Returns bf16 values as f32."""
    nib = unpack_nibbles(packed)
    v = e2m1_decode(nib)                       # exact, also exact in bf16
    s = round_bf16(scales_to_f32(scales))      # scale.astype(bf16)
    k = v.shape[-2]
    s = np.repeat(s, block, axis=-2)[..., :k, :]
    return round_bf16(v * s)                   # bf16 multiply = RN(exact)


def dequant_fp4_f32(packed: np.ndarray, scales: np.ndarray,
                    block: int = 32) -> np.ndarray:
    """The fp32 decode of the BASELINE oracle: e2m1 value * f32 scale."""
    v = e2m1_decode(unpack_nibbles(packed))
    s = scales_to_f32(scales)
    k = v.shape[-2]
    s = np.repeat(s, block, axis=-2)[..., :k, :]
    return (v * s).astype(np.float32)


def _group_rows(group_sizes):
    gs = np.asarray(group_sizes, dtype=np.int64)
    starts = np.concatenate([[0], np.cumsum(gs)[:-1]])
    return starts, gs


def silu_and_mul(gate: np.ndarray, up: np.ndarray,
                 limit: float | None = None) -> np.ndarray:
    """SwiGLU on f32 values: silu(gate) * up (X0104:286-296 op order; the clamp
    variant min(gate, limit), clip(up, -limit, limit))."""
    g = np.asarray(gate, dtype=np.float32)
    u = np.asarray(up, dtype=np.float32)
    if limit is not None:
        g = np.minimum(g, np.float32(limit))
        u = np.clip(u, -np.float32(limit), np.float32(limit))
    with np.errstate(over="ignore"):
        sig = (np.float32(1.0) / (np.float32(1.0) + np.exp(-g))).astype(np.float32)
    return (g * sig * u).astype(np.float32)


def _gmm_core(lhs_f32, w_f32, group_sizes, group_offset, act, limit):
    m, _ = lhs_f32.shape
    n_local, _, n = w_f32.shape
    n_out = n // 2 if act else n
    out = np.zeros((m, n_out), np.float64)
    valid = np.zeros(m, bool)
    starts, gs = _group_rows(group_sizes)
    for gl in range(n_local):
        g = group_offset + gl
        if g >= len(gs) or gs[g] == 0:
            continue
        r0, r1 = int(starts[g]), int(starts[g] + gs[g])
        acc = lhs_f32[r0:r1].astype(np.float64) @ w_f32[gl].astype(np.float64)
        if act:
            acc32 = acc.astype(np.float32)
            acc = silu_and_mul(acc32[:, :n_out], acc32[:, n_out:], limit)
        out[r0:r1] = acc
        valid[r0:r1] = True
    return out.astype(np.float32), valid


def gmm_f32(lhs, packed, scales, group_sizes, group_offset=0, act=None,
            limit=None):
    """The BASELINE fp32 oracle: fp32 decode*scale, f64-accumulated ragged dot
    (jax.lax.ragged_dot semantics, rows sorted by group), optional SwiGLU.

    lhs: f32 values (already bf16-representable) [M, K]. Returns (out f32
    [M, N_out], valid-row mask); rows outside the local groups are 0.
    """
    w = dequant_fp4_f32(packed, scales)
    return _gmm_core(np.asarray(lhs, np.float32), w, group_sizes,
                     group_offset, act, limit)


def gmm_ref(lhs, packed, scales, group_sizes, group_offset=0, act=None,
            limit=None, out_dtype="bf16"):
    """Reference numerics of gmm_v2 with rhs_fp4_codes (TK:62-63, TK:93-96,
    E0901:84-95): bf16 lhs (no lhs quantisation), bf16-dequantised weights,
    f32 accumulation (here f64 then one rounding), output rounded once to
    ``out_dtype``. Returns (out as f32 values, valid-row mask)."""
    w = dequant_fp4_block(packed, scales)
    out, valid = _gmm_core(round_bf16(np.asarray(lhs, np.float32)), w,
                           group_sizes, group_offset, act, limit)
    if out_dtype == "bf16":
        out = round_bf16(out)
    return out, valid


# ----------------------------------------------------------------------------
# Load-time power-of-two requant (B01:276-347)
# ----------------------------------------------------------------------------

def quantize_fp4_block32(tensor: np.ndarray, power_of_two_scale: bool):
    """quantize_tensor(float4_e2m1fn, t, axis=-1, block_size=32,
    power_of_two_scale) restated (B01:319-347): per-32 absmax / 6, optionally
    rounded up to 2^ceil(log2) exactly via frexp; values / scale rounded to
    e2m1. Returns (nibbles [..., N], f32 scales [..., N/32])."""
    t = np.asarray(tensor, dtype=np.float32)
    shp = t.shape
    blocks = t.reshape(shp[:-1] + (shp[-1] // 32, 32))
    abs_max = np.max(np.abs(blocks), axis=-1, keepdims=True)
    scale = (abs_max / np.float32(6.0)).astype(np.float32)
    if power_of_two_scale:
        mant, exp = np.frexp(scale)
        scale = np.where(
            scale > 0,
            np.ldexp(np.ones_like(scale), np.where(mant == 0.5, exp - 1, exp)),
            scale).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(scale > 0, blocks / scale, 0.0).astype(np.float32)
    nib = round_to_e2m1(q).reshape(shp)
    return nib, scale[..., 0]


def dequantize_fp4_block32(nib: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """dequantize_tensor(q, scale, -1, f32, (32,)): value * per-block scale."""
    v = e2m1_decode(nib)
    shp = v.shape
    out = v.reshape(shp[:-1] + (shp[-1] // 32, 32)) * scale[..., None]
    return out.reshape(shp).astype(np.float32)


# ----------------------------------------------------------------------------
# Routing (E0901:656-687, X0101:131)
# ----------------------------------------------------------------------------

def apply_scoring_fn(scoring_fn: str, logits: np.ndarray) -> np.ndarray:
    """Scores in f32 from f32-widened logits: softmax / sigmoid /
    sqrtsoftplus (upstream apply_scoring_fn, used at E0901:668).

    Assumption: upstream apply_scoring_fn lives in the tpu-inference
    submodule, which the reference does not vendor, so its compute dtype is
    not visible. This restatement (and the CUDA routing) scores in f32."""
    x = np.asarray(logits, dtype=np.float32)
    if scoring_fn == "softmax":
        m = x.max(axis=-1, keepdims=True)
        e = np.exp(x - m).astype(np.float32)
        return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)
    if scoring_fn == "sigmoid":
        with np.errstate(over="ignore"):
            return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))).astype(
                np.float32)
    if scoring_fn == "sqrtsoftplus":
        sp = np.logaddexp(np.float32(0.0), x).astype(np.float32)
        return np.sqrt(sp).astype(np.float32)
    raise ValueError(f"unknown scoring_fn {scoring_fn}")


def route_topk(logits, top_k: int, scoring_fn: str = "sigmoid",
               renormalize: bool = True, bias=None, num_valid_tokens=None):
    """E0901:656-687: scores, top-k (ties -> lower expert index, lax.top_k),
    optional correction bias for selection only, renormalise w / sum(w),
    padding rows -> expert 0 with weight 0. Returns (ids int32, w f32); the
    caller casts w to the activation dtype (X0101:131)."""
    s = apply_scoring_fn(scoring_fn, logits)
    sel = s if bias is None else (s + np.asarray(bias, np.float32)[None, :])
    order = np.argsort(-sel, axis=-1, kind="stable")[:, :top_k]
    ids = order.astype(np.int32)
    w = np.take_along_axis(s, order, axis=-1).astype(np.float32)
    if renormalize:
        w = (w / w.sum(axis=-1, keepdims=True)).astype(np.float32)
    if num_valid_tokens is not None:
        valid = (np.arange(s.shape[0]) < num_valid_tokens)[:, None]
        ids = np.where(valid, ids, 0).astype(np.int32)
        w = np.where(valid, w, 0.0).astype(np.float32)
    return ids, w


def route_hash(logits, hash_ids, scoring_fn: str = "sigmoid", renormalize: bool = True,
               num_valid_tokens=None):
    """E0901:667-671 (hash routing): ids = hash_ids, weights = the scores at
    those ids; then renormalise and pad like ``route_topk``."""
    s = apply_scoring_fn(scoring_fn, logits)
    ids = np.asarray(hash_ids, np.int32)
    w = np.take_along_axis(s, ids, axis=-1).astype(np.float32)
    if renormalize:
        w = (w / w.sum(axis=-1, keepdims=True)).astype(np.float32)
    if num_valid_tokens is not None:
        valid = (np.arange(s.shape[0]) < num_valid_tokens)[:, None]
        ids = np.where(valid, ids, 0).astype(np.int32)
        w = np.where(valid, w, 0.0).astype(np.float32)
    return ids, w


def dedupe_topk(weights, ids, num_experts: int):
    """E0901:98-121: a repeated expert id adds its weight (f32) to the first
    occurrence and is re-pointed at the lowest unused expert with weight 0."""
    w = np.asarray(weights, np.float32).copy()
    ids = np.asarray(ids, np.int32).copy()
    top_k = ids.shape[-1]
    cand = np.arange(min(2 * top_k, num_experts), dtype=np.int32)
    rows = np.arange(w.shape[0])
    for j in range(1, top_k):
        same = ids[:, :j] == ids[:, j:j + 1]
        dup = same.any(axis=-1)
        first = same.argmax(axis=-1)
        add = np.where(dup, w[:, j], 0.0).astype(np.float32)
        np.add.at(w, (rows, first), add)
        used = (ids[:, :, None] == cand[None, None, :]).any(axis=1)
        free = cand[np.argmin(used, axis=-1)]
        ids[:, j] = np.where(dup, free, ids[:, j])
        w[:, j] = np.where(dup, 0.0, w[:, j])
    return w, ids


# ----------------------------------------------------------------------------
# Permute / dispatch (KD, X0405:70-98)
# ----------------------------------------------------------------------------

def sorted_token_indices(topk_argsort_indices, topk: int) -> np.ndarray:
    """KD:41-44: argsort // topk (== arange(T).repeat(topk)[argsort])."""
    return (np.asarray(topk_argsort_indices, np.int64) // topk).astype(
        np.int32)


def permute(topk_ids: np.ndarray, num_experts: int):
    """X0405:73-88: stable argsort of the flattened ids, the expert-sorted
    token indices, group sizes (bincount) and the revert (inverse) map used by
    the combine. Returns (argsort, token_indices_sorted, revert, group_sizes),
    all int32."""
    flat = np.asarray(topk_ids, np.int64).reshape(-1)
    topk = topk_ids.shape[-1]
    order = np.argsort(flat, kind="stable")
    tok = sorted_token_indices(order, topk)
    revert = np.empty_like(order)
    revert[order] = np.arange(order.size)
    gs = np.bincount(flat, minlength=num_experts)[:num_experts]
    return (order.astype(np.int32), tok, revert.astype(np.int32),
            gs.astype(np.int32))


def dispatch_gather(hidden: np.ndarray, token_indices_sorted) -> np.ndarray:
    """KD:188-194: hidden[token_indices_sorted] (pure data movement)."""
    return np.asarray(hidden)[np.asarray(token_indices_sorted, np.int64)]


# ----------------------------------------------------------------------------
# Combine (KC:44-54, the k-order contract of KC:14-21)
# ----------------------------------------------------------------------------

def combine(x: np.ndarray, indices, topk_weights, topk: int,
            out_dtype: str = "bf16") -> np.ndarray:
    """out[t] = round(sum_k f32(x[idx[t*topk+k]]) * f32(w[t,k])), products
    rounded to f32, summed left to right from +0.0, one final rounding."""
    xf = np.asarray(x, np.float32)
    w = np.asarray(topk_weights, np.float32)
    t = w.shape[0]
    idx = np.asarray(indices, np.int64).reshape(t, topk)
    acc = np.zeros((t, xf.shape[-1]), np.float32)
    for k in range(topk):
        prod = (xf[idx[:, k]] * w[:, k:k + 1]).astype(np.float32)
        acc = (acc + prod).astype(np.float32)
    return round_bf16(acc) if out_dtype == "bf16" else acc


def combine_shared(x, indices, topk_weights, topk: int, shared, routed_scale: float = 1.0,
                   mid_dtype: str = "bf16", out_dtype: str = "bf16") -> np.ndarray:
    """The routed combine with the shared expert's partial summed in
    (MOE_SHARED_EXPERT_TP, X0104:80-87 of the patch): the routed k-order sum
    in the combine's dtype (bf16, or f32 under MOE_F32_REDUCE), widened to
    f32, times routed_scale, plus the f32 shared partial, each step rounded
    to f32, then one rounding to the output dtype:
        out = dtype(f32(combine_out) * routed_scale + shared_partial)."""
    routed = combine(x, indices, topk_weights, topk, out_dtype=mid_dtype)
    sh = np.asarray(shared, np.float32)
    v = (np.asarray(routed, np.float32) * np.float32(routed_scale)).astype(np.float32)
    v = (v + sh).astype(np.float32)
    return round_bf16(v) if out_dtype == "bf16" else v


# ----------------------------------------------------------------------------
# Single-device MoE layer (the fused_moe_func GMM path, X0104:88-98)
# ----------------------------------------------------------------------------

def fused_moe(hidden, logits, w13_packed, w13_scales, w2_packed, w2_scales,
              top_k, scoring_fn="sigmoid", renormalize=True, limit=None,
              f32_reduce=False):
    """route -> permute -> gather -> gmm1(SwiGLU) -> gmm2 -> combine, with the
    reference numerics (bf16 activations, weights cast to bf16 before the
    combine per X0101:131). Returns bf16 values as f32 [T, H]."""
    ids, w = route_topk(logits, top_k, scoring_fn, renormalize)
    w_bf = round_bf16(w)
    e = w13_packed.shape[0]
    _, tok, revert, gs = permute(ids, e)
    x = dispatch_gather(round_bf16(np.asarray(hidden, np.float32)), tok)
    h1, _ = gmm_ref(x, w13_packed, w13_scales, gs, act="swiglu", limit=limit)
    y, _ = gmm_ref(h1, w2_packed, w2_scales, gs,
                   out_dtype="f32" if f32_reduce else "bf16")
    return combine(y, revert, w_bf, top_k)


# ----------------------------------------------------------------------------
# Expert-parallel exchange (X0101:56-104, X0107:15-51, KO:152-185)
# ----------------------------------------------------------------------------

def all_gather(blocks):
    """KO:152-164: rank-major concatenation (bitwise lax.all_gather)."""
    return np.concatenate([np.asarray(b) for b in blocks], axis=0)


def reduce_scatter_rank_order(partials, n: int, out_dtype="bf16"):
    """KO:167-185 and KO:236-239: rank r receives block r of every rank's
    partial and sums them in f32 in rank order 0..n-1, then rounds once."""
    outs = []
    for r in range(n):
        blocks = [np.asarray(p, np.float32).reshape(n, -1, p.shape[-1])[r]
                  for p in partials]
        acc = blocks[0].astype(np.float32)
        for b in blocks[1:]:
            acc = (acc + b).astype(np.float32)
        outs.append(round_bf16(acc) if out_dtype == "bf16" else acc)
    return outs


def ep_dispatch(hidden_per_rank, ids_per_rank, num_experts: int):
    """EP receive order (X0101:56-104 + X0107:34-51): tokens are gathered rank
    major, the flattened ids of the gathered batch are stably argsorted, and
    rank r keeps the sorted rows whose expert is in [r*E/n, (r+1)*E/n).

    Within an expert the order is (source rank, local token, k slot).
    Returns per rank: (recv rows [R_r, H], local group_sizes [E/n], source
    (rank, token, k) triples [R_r, 3] int32)."""
    n = len(hidden_per_rank)
    hid = all_gather(hidden_per_rank)
    ids = all_gather(ids_per_rank)
    topk = ids.shape[-1]
    t_counts = [np.asarray(h).shape[0] for h in hidden_per_rank]
    t_start = np.concatenate([[0], np.cumsum(t_counts)[:-1]])
    order, tok, _, gs = permute(ids, num_experts)
    flat = ids.reshape(-1)
    e_loc = num_experts // n
    src_rank = np.searchsorted(np.cumsum(t_counts), tok, side="right")
    out = []
    for r in range(n):
        lo, hi = r * e_loc, (r + 1) * e_loc
        sel = (flat[order] >= lo) & (flat[order] < hi)
        rows = tok[sel]
        srank = src_rank[sel]
        src = np.stack([srank, rows - t_start[srank], order[sel] % topk],
                       axis=1).astype(np.int32)
        out.append((hid[rows], gs[lo:hi].copy(), src))
    return out


def ep_combine_korder(y_per_rank, src_per_rank, w_per_rank, out_dtype="bf16"):
    """The BASELINE config-2 combine contract: each token owner receives the
    expert-output row of each of its (token, k) pairs and forms
    round(sum_k f32(y) * f32(w[t, k])) in k order from +0.0."""
    n = len(w_per_rank)
    h = np.asarray(y_per_rank[0]).shape[-1] if len(y_per_rank[0]) else None
    if h is None:
        h = next(np.asarray(y).shape[-1] for y in y_per_rank if len(y))
    outs = []
    for r in range(n):
        w = np.asarray(w_per_rank[r], np.float32)
        t, topk = w.shape
        rows = np.zeros((t, topk, h), np.float32)
        for rr in range(n):
            src = np.asarray(src_per_rank[rr])
            if src.size == 0:
                continue
            mine = src[:, 0] == r
            yv = np.asarray(y_per_rank[rr], np.float32)[mine]
            rows[src[mine, 1], src[mine, 2]] = yv
        acc = np.zeros((t, h), np.float32)
        for k in range(topk):
            acc = (acc + (rows[:, k] * w[:, k:k + 1]).astype(np.float32)
                   ).astype(np.float32)
        outs.append(round_bf16(acc) if out_dtype == "bf16" else acc)
    return outs


def ep_combine_rankorder(y_per_rank, src_per_rank, w_per_rank,
                         num_experts: int, ids_per_rank):
    """The reference GMM_EP order (X0107:15-29 then KO:167-185): every rank
    forms an f32 partial over the k slots of its own experts (others masked),
    then partials are summed over ranks 0..n-1 in f32 and rounded once."""
    n = len(w_per_rank)
    h = next(np.asarray(y).shape[-1] for y in y_per_rank if len(y))
    t_counts = [np.asarray(w).shape[0] for w in w_per_rank]
    partials = []
    for rr in range(n):
        src = np.asarray(src_per_rank[rr])
        yv = np.asarray(y_per_rank[rr], np.float32)
        part = []
        for r in range(n):
            w = np.asarray(w_per_rank[r], np.float32)
            t, topk = w.shape
            rows = np.zeros((t, topk, h), np.float32)
            mask = np.zeros((t, topk), bool)
            if src.size:
                mine = src[:, 0] == r
                rows[src[mine, 1], src[mine, 2]] = yv[mine]
                mask[src[mine, 1], src[mine, 2]] = True
            prod = (rows * w[:, :, None]).astype(np.float32)
            acc = np.zeros((t, h), np.float32)
            for k in range(topk):
                acc = (acc + np.where(mask[:, k:k + 1], prod[:, k], 0.0)
                       ).astype(np.float32)
            part.append(acc)
        partials.append(part)
    outs = []
    for r in range(n):
        acc = partials[0][r].astype(np.float32)
        for rr in range(1, n):
            acc = (acc + partials[rr][r]).astype(np.float32)
        outs.append(round_bf16(acc))
    return outs
