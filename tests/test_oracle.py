"""Pins the CPU oracle to the reference (no GPU needed).

* e2m1 decode vs ml_dtypes float4_e2m1fn and the TK:35-36 table;
* tokamax codes round trip (TK:17-41);
* e8m0 encode/decode (KE:14-40);
* the reference's known-answer test for power-of-two requant (B01:131-157);
* the permute identity of KD:16-22,43 and the combine order of KC:44-54;
* the EP receive order and the one-shot collectives (X0107, KO);
* the committed golden fixtures are reproduced bit for bit.
"""

import numpy as np
import pytest

from oracle import moe_oracle as O
from tests.golden import make_golden


def test_e2m1_table_matches_ml_dtypes_and_tk_table():
    ml_dtypes = pytest.importorskip("ml_dtypes")
    nib = np.arange(16, dtype=np.uint8)
    ref = nib.view(ml_dtypes.float4_e2m1fn).astype(np.float32)
    assert np.array_equal(O.e2m1_decode(nib), ref)
    # TK:35-36: "e2m1 magnitudes by code: 0 .5 1 1.5 2 3 4 6"
    assert O.E2M1_MAGNITUDES.tolist() == [0, .5, 1, 1.5, 2, 3, 4, 6]


def test_tokamax_codes_decode_exactly():
    nib = np.arange(16, dtype=np.uint8)
    codes = O.e2m1_to_codes(nib)
    dec = O.decode_codes(codes)
    val = O.e2m1_decode(nib)
    assert np.array_equal(dec, val)           # -0 -> +0 compares equal
    assert codes[8] == 0                      # TK:27: -0 becomes +0
    back = O.codes_to_e2m1(codes)
    assert np.array_equal(O.e2m1_decode(back), val)
    # decode is exact in bf16 (TK:38-39)
    assert np.array_equal(O.round_bf16(dec), dec)


def test_pack_unpack_low_nibble_first():
    nib = np.array([[1, 2, 3, 4]], np.uint8)
    packed = O.pack_nibbles(nib)
    assert packed.tolist() == [[0x21, 0x43]]
    assert np.array_equal(O.unpack_nibbles(packed), nib)


def test_b200_swizzle_is_a_lossless_bit_permutation():
    rng = np.random.default_rng(8)
    packed = rng.integers(0, 256, (2, 16, 64), dtype=np.uint8)
    sw = O.b200_swizzle(packed)
    assert np.array_equal(O.b200_unswizzle(sw), packed)
    # every bit lands on a distinct position: popcounts are preserved
    assert np.array_equal(np.unpackbits(sw).sum(), np.unpackbits(packed).sum())
    one = np.zeros(4, np.uint8)
    seen = set()
    for bit in range(32):
        w = np.array([1 << bit], np.uint32).view(np.uint8)
        s = int(O.b200_swizzle(w).view(np.uint32)[0])
        assert bin(s).count("1") == 1 and s not in seen
        seen.add(s)
    assert one.sum() == 0
    raw = rng.integers(0, 256, (2, 64, 16), dtype=np.uint8)   # [g, k, n/2]
    b = O.to_b200_layout(raw)
    assert b.shape == (2, 32, 32)                             # [g, n, k/2]
    assert np.array_equal(O.from_b200_layout(b), raw)
    # element check of the fragment order against a direct formula
    nib = O.unpack_nibbles(raw)                               # [g, k, n]
    words = O.b200_unswizzle(b).view(np.uint32).reshape(2, 32 // 16, 64 // 16, 32)
    for (g, kk, c) in [(0, 0, 0), (1, 63, 31), (0, 9, 17), (1, 22, 5), (0, 40, 30)]:
        kb, dk, cb, dc = kk // 16, kk % 16, c // 16, c % 16
        gid, j_hi = dc % 8, dc // 8
        t, j_lo, j_k8 = (dk % 8) // 2, dk % 2, dk // 8
        j = j_lo | (j_hi << 1) | (j_k8 << 2)
        got = (int(words[g, cb, kb, gid * 4 + t]) >> (4 * j)) & 0xF
        assert got == nib[g, kk, c], (g, kk, c)


def test_e8m0_roundtrip_and_lossless_flag():
    e = np.arange(-126, 128)
    s = np.ldexp(np.ones(e.shape, np.float32), e).astype(np.float32)
    s = np.concatenate([s, [0.0]]).astype(np.float32)
    codes, lossless = O.e8m0_encode(s)
    assert lossless
    assert np.array_equal(O.e8m0_decode(codes).view(np.uint32), s.view(np.uint32))
    assert O.e8m0_decode(np.array([0], np.uint8))[0] == 0.0
    _, lossless = O.e8m0_encode(np.array([1.5], np.float32))
    assert not lossless
    _, lossless = O.e8m0_encode(np.array([-2.0], np.float32))
    assert not lossless
    _, lossless = O.e8m0_encode(np.array([np.inf], np.float32))
    assert not lossless


def test_round_to_e2m1_matches_ml_dtypes():
    ml_dtypes = pytest.importorskip("ml_dtypes")
    x = np.concatenate([np.linspace(-7, 7, 2801, dtype=np.float32),
                        np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25, -5.0],
                                 np.float32)])
    ours = O.e2m1_decode(O.round_to_e2m1(x))
    ref = x.astype(ml_dtypes.float4_e2m1fn).astype(np.float32)
    assert np.array_equal(ours, ref)


def test_requant_known_answer_b01():
    """B01:131-157 restated: power-of-two requant of MXFP4 data is exact; the
    absmax default is not."""
    d = make_golden.requant_kat(seed=0)
    original = d["original"]
    q, s = O.quantize_fp4_block32(original, power_of_two_scale=True)
    assert np.array_equal(O.dequantize_fp4_block32(q, s), original)
    q2, s2 = O.quantize_fp4_block32(original, power_of_two_scale=False)
    assert not np.array_equal(O.dequantize_fp4_block32(q2, s2), original)


def test_sorted_token_indices_identity_kd():
    rng = np.random.default_rng(3)
    t, k = 50, 8
    ids = rng.integers(0, 32, (t, k))
    argsort = np.argsort(ids.reshape(-1), kind="stable")
    # KD:16-22: bitwise identical to arange(T).repeat(topk)[argsort]
    assert np.array_equal(O.sorted_token_indices(argsort, k),
                          np.repeat(np.arange(t), k)[argsort])


def test_permute_is_stable_and_revert_inverts():
    rng = np.random.default_rng(4)
    ids = rng.integers(0, 16, (33, 4)).astype(np.int32)
    argsort, tok, revert, gs = O.permute(ids, 16)
    flat = ids.reshape(-1)
    assert np.all(np.diff(flat[argsort]) >= 0)
    for e in range(16):  # stability: within an expert, flat order
        pos = argsort[flat[argsort] == e]
        assert np.all(np.diff(pos) > 0)
    assert np.array_equal(argsort[revert], np.arange(flat.size))
    assert np.array_equal(gs, np.bincount(flat, minlength=16))


def test_combine_matches_explicit_k_loop():
    rng = np.random.default_rng(5)
    t, k, h = 7, 6, 16
    x = O.round_bf16(rng.standard_normal((t * k, h)).astype(np.float32))
    idx = rng.permutation(t * k).astype(np.int32)
    w = rng.random((t, k)).astype(np.float32)
    got = O.combine(x, idx, w, k, out_dtype="f32")
    for tt in range(t):
        acc = np.zeros(h, np.float32)
        for kk in range(k):
            acc = np.float32(acc + np.float32(x[idx[tt * k + kk]] * w[tt, kk]))
        assert np.array_equal(got[tt], acc)


def test_combine_shared_follows_x0104_order():
    rng = np.random.default_rng(12)
    t, k, h = 5, 3, 8
    x = O.round_bf16(rng.standard_normal((t * k, h)).astype(np.float32))
    idx = rng.permutation(t * k).astype(np.int32)
    w = rng.random((t, k)).astype(np.float32)
    sh = rng.standard_normal((t, h)).astype(np.float32)
    got = O.combine_shared(x, idx, w, k, sh, 0.75, mid_dtype="bf16", out_dtype="f32")
    routed = O.round_bf16(O.combine(x, idx, w, k, out_dtype="f32"))
    for tt in range(t):
        for c in range(h):
            v = np.float32(np.float32(routed[tt, c]) * np.float32(0.75))
            assert got[tt, c] == np.float32(v + sh[tt, c])


def test_gmm_ref_close_to_f32_oracle():
    d = make_golden.gmm_small(seed=1)
    lhs = O.bf16_bits_to_f32(d["lhs_bits"])
    ref = O.bf16_bits_to_f32(d["out_ref_bits"])
    f32 = d["out_f32"]
    v = d["valid"]
    rel = np.linalg.norm(ref[v] - f32[v]) / np.linalg.norm(f32[v])
    assert rel < 4e-3
    assert lhs.shape[0] == ref.shape[0]


def test_ep_dispatch_matches_global_sort_and_combines():
    rng = np.random.default_rng(6)
    n, e, k, h = 4, 16, 3, 8
    t_counts = [5, 0, 7, 3]
    hid = [O.round_bf16(rng.standard_normal((t, h)).astype(np.float32)) for t in t_counts]
    ids = [np.stack([rng.choice(e, k, replace=False) for _ in range(t)]).astype(np.int32)
           if t else np.zeros((0, k), np.int32) for t in t_counts]
    ws = [rng.dirichlet(np.ones(k), size=t).astype(np.float32) for t in t_counts]
    per_rank = O.ep_dispatch(hid, ids, e)
    allhid = np.concatenate(hid)
    allids = np.concatenate(ids)
    _, tok, _, gs = O.permute(allids, e)
    recv = np.concatenate([p[0] for p in per_rank])
    assert np.array_equal(recv, allhid[tok])
    assert np.array_equal(np.concatenate([p[1] for p in per_rank]), gs)
    # identity expert (y = x) then combine == weighted sum of the token itself
    ys = [p[0] for p in per_rank]
    srcs = [p[2] for p in per_rank]
    outs = O.ep_combine_korder(ys, srcs, ws)
    for r in range(n):
        if t_counts[r] == 0:
            continue
        exp = O.combine(np.repeat(hid[r], k, axis=0), np.arange(t_counts[r] * k), ws[r], k)
        assert np.array_equal(outs[r], exp)
    ro = O.ep_combine_rankorder(ys, srcs, ws, e, ids)
    for r in range(n):
        if t_counts[r]:
            assert np.allclose(ro[r], outs[r], rtol=1e-2, atol=1e-2)


def test_oneshot_collectives():
    blocks = [np.full((2, 3), r, np.float32) for r in range(3)]
    assert np.array_equal(O.all_gather(blocks), np.concatenate(blocks))
    parts = [np.arange(3 * 2 * 4, dtype=np.float32).reshape(6, 4) * (r + 1) for r in range(3)]
    outs = O.reduce_scatter_rank_order(parts, 3, out_dtype="f32")
    for r in range(3):
        exp = sum(p.reshape(3, 2, 4)[r] for p in parts)
        assert np.array_equal(outs[r], exp)


def test_route_hash_matches_take_along_scores():
    rng = np.random.default_rng(6)
    logits = rng.standard_normal((5, 16)).astype(np.float32)
    hid = rng.integers(0, 16, (5, 4)).astype(np.int32)
    ids, w = O.route_hash(logits, hid, "sigmoid", renormalize=False)
    s = 1.0 / (1.0 + np.exp(-logits.astype(np.float64)))
    assert np.array_equal(ids, hid)
    np.testing.assert_allclose(w, np.take_along_axis(s, hid, axis=-1), rtol=1e-6)
    ids2, w2 = O.route_hash(logits, hid, "sigmoid", num_valid_tokens=3)
    assert np.all(ids2[3:] == 0) and np.all(w2[3:] == 0)
    np.testing.assert_allclose(w2[:3].sum(-1), 1.0, rtol=1e-6)


def test_dedupe_topk():
    w = np.array([[0.5, 0.3, 0.2]], np.float32)
    ids = np.array([[3, 3, 1]], np.int32)
    w2, ids2 = O.dedupe_topk(w, ids, 8)
    assert ids2.tolist() == [[3, 0, 1]]
    assert np.allclose(w2, [[0.8, 0.0, 0.2]])


@pytest.mark.parametrize("name", sorted(make_golden.FIXTURES))
def test_golden_fixtures_reproduce(name, golden):
    fresh = make_golden.FIXTURES[name]()
    stored = golden(name)
    assert set(fresh) == set(stored)
    for key in fresh:
        a, b = np.asarray(fresh[key]), stored[key]
        assert a.dtype == b.dtype and a.shape == b.shape, key
        assert np.array_equal(a, b, equal_nan=True), key


def test_cpu_baseline_layer_matches_the_oracle():
    """oracle/layer_cpu.py (the timed CPU baseline) is the oracle's layer
    arithmetic: its table dequant equals dequant_fp4_block bit for bit (also
    for E8M0 codes that underflow or overflow bf16), and its layer output
    equals fused_moe's up to f32-vs-f64 summation order."""
    from oracle import layer_cpu as C
    rng = np.random.default_rng(21)
    packed = rng.integers(0, 256, (64, 48), dtype=np.uint8)
    for lo, hi in ((123, 129), (0, 255)):
        sc = rng.integers(lo, hi + 1, (2, 96), dtype=np.uint8)
        got = C.dequant_fp4_lut(packed, sc).copy()
        assert np.array_equal(got, O.dequant_fp4_block(packed, sc), equal_nan=True), (lo, hi)
    t, e, h, i, k = 12, 8, 256, 128, 4
    hid = O.round_bf16(rng.standard_normal((t, h)).astype(np.float32))
    logits = O.round_bf16(rng.standard_normal((t, e)).astype(np.float32))
    w13 = rng.integers(0, 256, (e, h, i), dtype=np.uint8)
    s13 = rng.integers(118, 122, (e, h // 32, 2 * i), dtype=np.uint8)
    w2 = rng.integers(0, 256, (e, i, h // 2), dtype=np.uint8)
    s2 = rng.integers(118, 122, (e, i // 32, h), dtype=np.uint8)
    pool, _ = C.make_pool(2)
    with pool:
        got = C.layer_forward(hid, logits, w13, s13, w2, s2, k, pool=pool)
    ref = O.fused_moe(hid, logits, w13, s13, w2, s2, k)
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert rel < 1e-3, rel
