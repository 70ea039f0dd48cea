"""FP4 grouped matmul on the GPU vs the oracle (through the C ABI)."""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from tests.gpu_util import assert_gemm_close, bf16_to_np, np_to_bf16, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dw():
    import dw_tpu_b200
    return dw_tpu_b200


def _run_gmm(dw, lhs_np, packed, scales, gs, **kw):
    lhs = np_to_bf16(lhs_np)
    codes = torch.from_numpy(packed).cuda()
    sc = scales if isinstance(scales, torch.Tensor) else torch.from_numpy(scales)
    out = dw.gmm_v2(lhs, codes, torch.from_numpy(gs).cuda(), sc.cuda(), **kw)
    torch.cuda.synchronize()
    from dw_tpu_b200 import _lib
    _lib.raise_on_device_error()
    return out


def _case(seed, m, k, n, groups, gs=None, lo=123, hi=129):
    rng = np.random.default_rng(seed)
    lhs = O.round_bf16(rng.standard_normal((m, k)).astype(np.float32))
    packed = rng.integers(0, 256, (groups, k, n // 2), dtype=np.uint8)
    scales = rng.integers(lo, hi + 1, (groups, k // 32, n), dtype=np.uint8)
    if gs is None:
        gs = rng.multinomial(m, [1.0 / groups] * groups)
    return lhs, packed, scales, np.asarray(gs, np.int32)


def test_dequant_bit_exact_golden(dw, golden):
    d = golden("gmm_small")
    out = dw.decode_codes(torch.from_numpy(d["packed"]).cuda(),
                          torch.from_numpy(d["scales"]).cuda())
    got = out.cpu().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, d["dequant_bits"])


@pytest.mark.parametrize("scale_kind", ["e8m0_wide", "bf16", "f32"])
def test_dequant_bit_exact_scale_types(dw, scale_kind):
    rng = np.random.default_rng(5)
    g, k, n = 2, 64, 256
    packed = rng.integers(0, 256, (g, k, n // 2), dtype=np.uint8)
    if scale_kind == "e8m0_wide":
        sc_np = rng.integers(0, 256, (g, k // 32, n), dtype=np.uint8)  # incl. 0, >128, 255
        sc = torch.from_numpy(sc_np)
    elif scale_kind == "bf16":
        sc_f = (rng.random((g, k // 32, n)) * 3).astype(np.float32)
        sc_np = O.f32_to_bf16_bits(sc_f)
        sc = torch.from_numpy(sc_np.view(np.int16).copy()).view(torch.bfloat16)
    else:
        sc_np = (rng.random((g, k // 32, n)) * 3).astype(np.float32)
        sc = torch.from_numpy(sc_np)
    out = dw.decode_codes(torch.from_numpy(packed).cuda(), sc.cuda())
    ref = O.dequant_fp4_block(packed, sc_np)
    got = bf16_to_np(out)
    assert np.array_equal(got, ref, equal_nan=True)


def test_gmm_golden_fixture(dw, golden):
    d = golden("gmm_small")
    lhs = O.bf16_bits_to_f32(d["lhs_bits"])
    out = _run_gmm(dw, lhs, d["packed"], d["scales"], d["group_sizes"])
    got = bf16_to_np(out)
    ref = O.bf16_bits_to_f32(d["out_ref_bits"])
    v = d["valid"]
    assert_gemm_close(got, ref, d["out_f32"], lhs.shape[1], rows=v)
    assert np.all(got[~v] == 0)  # zero_initialize=True (gmm_v2 default)


def test_gmm_cfg0_full_size(dw):
    from dw_tpu_b200 import synthetic
    lhs, codes, scales, gs = synthetic.cfg0(seed=0)
    lhs_np = bf16_to_np(lhs)
    out = _run_gmm(dw, lhs_np, codes.numpy(), scales.numpy(), gs.numpy())
    ref, v = O.gmm_ref(lhs_np, codes.numpy(), scales.numpy(), gs.numpy())
    ref32, _ = O.gmm_f32(lhs_np, codes.numpy(), scales.numpy(), gs.numpy())
    assert_gemm_close(bf16_to_np(out), ref, ref32, 512, rows=v)


@pytest.mark.parametrize("gs", [
    [1, 0, 2, 3],            # decode-sized groups, one empty
    [0, 0, 0, 37],           # one group only, rows not a multiple of 16
    [129, 1, 0, 300],        # multiple row tiles per group
    [0, 0, 0, 0],            # nothing to do
])
def test_gmm_ragged_groups(dw, gs):
    m = max(1, sum(gs) + 3)
    lhs, packed, scales, gs = _case(2, m, 128, 256, 4, gs=gs)
    out = _run_gmm(dw, lhs, packed, scales, gs)
    ref, v = O.gmm_ref(lhs, packed, scales, gs)
    ref32, _ = O.gmm_f32(lhs, packed, scales, gs)
    got = bf16_to_np(out)
    assert_gemm_close(got, ref, ref32, 128, rows=v)
    assert np.all(got[~v] == 0)


def test_gmm_group_offset_and_untouched_rows(dw):
    """EP shard: only groups [2, 4) are local; other rows keep their bits
    with zero_initialize=False and are zeroed with True."""
    lhs, packed, scales, gs = _case(3, 96, 128, 512, 6)
    loc = slice(2, 4)
    for zero_init in (False, True):
        lhs_t = np_to_bf16(lhs)
        out = dw.gmm_v2(lhs_t, torch.from_numpy(packed[loc]).cuda(),
                        torch.from_numpy(gs).cuda(), torch.from_numpy(scales[loc]).cuda(),
                        group_offset=2, zero_initialize=zero_init)
        torch.cuda.synchronize()
        ref, v = O.gmm_ref(lhs, packed[loc], scales[loc], gs, group_offset=2)
        ref32, _ = O.gmm_f32(lhs, packed[loc], scales[loc], gs, group_offset=2)
        got = bf16_to_np(out)
        assert_gemm_close(got, ref, ref32, 128, rows=v)
        if zero_init:
            assert np.all(got[~v] == 0)


@pytest.mark.parametrize("act,limit", [("silu", None), ("silu_and_mul_with_clamp", 10.0)])
def test_gmm_fused_swiglu(dw, act, limit):
    lhs, packed, scales, gs = _case(4, 70, 256, 512, 3, lo=118, hi=121)
    out = _run_gmm(dw, lhs, packed, scales, gs, fuse_act=act, act_limit=limit)
    ref, v = O.gmm_ref(lhs, packed, scales, gs, act="swiglu", limit=limit)
    ref32, _ = O.gmm_f32(lhs, packed, scales, gs, act="swiglu", limit=limit)
    assert out.shape == (70, 256)
    assert_gemm_close(bf16_to_np(out), ref, ref32, 256, rows=v)


def test_gmm_f32_output_and_float_scales(dw):
    lhs, packed, scales, gs = _case(5, 50, 192, 256, 2)
    sc_f32 = O.e8m0_decode(scales)
    out = _run_gmm(dw, lhs, packed, torch.from_numpy(sc_f32), gs,
                   preferred_element_type=torch.float32)
    assert out.dtype == torch.float32
    ref, v = O.gmm_ref(lhs, packed, scales, gs, out_dtype="f32")
    ref32, _ = O.gmm_f32(lhs, packed, scales, gs)
    got = out.cpu().numpy()
    assert_gemm_close(got, O.round_bf16(ref), ref32, 192, rows=v)
    # bf16 scales give the same bits as e8m0 codes (power-of-two scales)
    out_bf = _run_gmm(dw, lhs, packed, torch.from_numpy(sc_f32).to(torch.bfloat16), gs)
    out_u8 = _run_gmm(dw, lhs, packed, scales, gs)
    assert torch.equal(out_bf.view(torch.int16), out_u8.view(torch.int16))


def test_gmm_tokamax_codes_equal_e2m1(dw):
    lhs, packed, scales, gs = _case(6, 40, 128, 256, 2)
    a = _run_gmm(dw, lhs, packed, scales, gs)
    nib = O.unpack_nibbles(packed)
    tok = O.pack_nibbles(O.e2m1_to_codes(nib))
    b = _run_gmm(dw, lhs, tok, scales, gs, rhs_fp4_codes=True)
    # tokamax maps -0 to +0; products with +-0 sum to the same values
    assert np.array_equal(bf16_to_np(a), bf16_to_np(b))
    conv = dw.e2m1_to_codes(torch.from_numpy(packed).cuda())
    assert np.array_equal(conv.cpu().numpy(), tok)


@pytest.mark.parametrize("sd", ["u8", "bf16", "f32"])
def test_b200_layout_dequant_and_gmm_match_e2m1(dw, sd):
    """The load-time B200 re-layout decodes to the same bf16 weights; the
    tcgen05 kernel on it gives the same bits as the raw e2m1 path, and the
    mma.sync kernel (another f32 summation order) stays within the GEMM
    tolerance of the oracle, for plain, SwiGLU and f32 outputs."""
    from dw_tpu_b200 import ops
    from dw_tpu_b200 import _lib as L
    lhs, packed, scales, gs = _case(9, 400, 128, 512, 4, gs=[3, 0, 70, 300], lo=120, hi=140)
    if sd == "u8":
        sc = torch.from_numpy(scales)
    elif sd == "bf16":
        sc = torch.from_numpy(O.e8m0_decode(scales)).to(torch.bfloat16)
    else:
        sc = torch.from_numpy(O.e8m0_decode(scales))
    sc = sc.cuda()
    raw = torch.from_numpy(packed).cuda()
    b200 = dw.fp4_weight_to_codes(raw)
    assert np.array_equal(b200.cpu().numpy(), O.to_b200_layout(packed))
    assert torch.equal(dw.b200_to_e2m1(b200), raw)
    d0 = dw.decode_codes(raw, sc)
    d1 = dw.decode_codes(b200, sc, layout="b200")
    assert torch.equal(d0.view(torch.int16), d1.view(torch.int16))
    assert np.array_equal(bf16_to_np(d0), O.dequant_fp4_block(packed, O.e8m0_decode(scales)))
    x = np_to_bf16(lhs)
    g = torch.from_numpy(gs).cuda()
    for act, n_out, dt in ((L.ACT_NONE, 512, torch.bfloat16), (L.ACT_SWIGLU, 256, torch.bfloat16),
                           (L.ACT_NONE, 512, torch.float32)):
        ref = ops.gmm_fp4_out(x, raw, sc, g, torch.empty((400, n_out), dtype=dt, device="cuda"),
                              act=act, zero_init=True)
        kind = "swiglu" if act == L.ACT_SWIGLU else None
        r, v = O.gmm_ref(lhs, packed, scales, gs, act=kind,
                         out_dtype="f32" if dt == torch.float32 else "bf16")
        r32, _ = O.gmm_f32(lhs, packed, scales, gs, act=kind)
        for variant in (0, 1, 2):
            got = ops.gmm_fp4_out(x, b200, sc, g,
                                  torch.empty((400, n_out), dtype=dt, device="cuda"), act=act,
                                  zero_init=True, layout="b200", variant=variant)
            torch.cuda.synchronize()
            L.raise_on_device_error()
            if variant in (0, 1):  # 100 rows per group on average: tcgen05, 128-row tiles
                assert torch.equal(ref.view(torch.int16), got.view(torch.int16)), (act, variant)
            else:
                assert_gemm_close(to_np(got), O.round_bf16(r), r32, 128, rows=v)
                assert np.all(to_np(got)[~v] == 0)
    r, v = O.gmm_ref(lhs, packed, scales, gs)
    r32, _ = O.gmm_f32(lhs, packed, scales, gs)
    out = dw.gmm_v2(x, b200, g, sc, rhs_layout="b200")
    assert_gemm_close(bf16_to_np(out), r, r32, 128, rows=v)


@pytest.mark.parametrize("sd", ["u8", "bf16", "f32", "u8_wide"])
def test_pair_kernel_matches_single_cta(dw, sd):
    """The CTA-pair tcgen05 kernel (variant 7: M = 256 UMMAs over two SMs,
    double-buffered accumulators, groups above 256 rows split into equal
    tiles; variant 9: tiles of up to 512 rows as two UMMAs per k-step) gives
    the single-CTA kernel's bits (the same decoded bf16 weights and UMMA k
    order) for plain, SwiGLU, clamped SwiGLU and f32 outputs, on ragged
    groups: empty, 1 row, below and above 128, exactly 256, 257 and 600 rows
    (2 and 3 tiles; 1 and 2 wide tiles); also on a window of local groups
    with zero_init."""
    from dw_tpu_b200 import ops
    from dw_tpu_b200 import _lib as L
    lo, hi = (0, 140) if sd == "u8_wide" else (120, 140)
    sizes = [0, 1, 17, 129, 256, 257, 600, 31]
    m = sum(sizes)
    lhs, packed, scales, gs = _case(21, m, 256, 512, len(sizes), gs=sizes, lo=lo, hi=hi)
    if sd in ("u8", "u8_wide"):
        sc = torch.from_numpy(scales)
    elif sd == "bf16":
        sc = torch.from_numpy(O.e8m0_decode(scales)).to(torch.bfloat16)
    else:
        sc = torch.from_numpy(O.e8m0_decode(scales))
    sc = sc.cuda()
    b200 = ops.fp4_to_b200_out(torch.from_numpy(packed).cuda())
    x = np_to_bf16(lhs)
    g = torch.from_numpy(gs).cuda()

    def bits(t):
        return t.view(torch.int16 if t.dtype == torch.bfloat16 else torch.int32)

    for act, n_out, dt, limit in ((L.ACT_NONE, 512, torch.bfloat16, 0.0),
                                  (L.ACT_SWIGLU, 256, torch.bfloat16, 0.0),
                                  (L.ACT_SWIGLU_CLAMP, 256, torch.float32, 0.5),
                                  (L.ACT_NONE, 512, torch.float32, 0.0)):
        outs = []
        for variant in (1, 7, 9):
            o = torch.full((m, n_out), float("nan"), dtype=dt, device="cuda")
            ops.gmm_fp4_out(x, b200, sc, g, o, act=act, act_limit=limit, layout="b200",
                            variant=variant)
            outs.append(o)
        torch.cuda.synchronize()
        L.raise_on_device_error()
        assert torch.equal(bits(outs[0]), bits(outs[1])), (act, dt)
        assert torch.equal(bits(outs[0]), bits(outs[2])), (act, dt, "wide")
        if act != L.ACT_SWIGLU_CLAMP:
            kind = "swiglu" if act == L.ACT_SWIGLU else None
            r, v = O.gmm_ref(lhs, packed, scales, gs, act=kind,
                             out_dtype="f32" if dt == torch.float32 else "bf16")
            r32, _ = O.gmm_f32(lhs, packed, scales, gs, act=kind)
            assert_gemm_close(to_np(outs[1]), O.round_bf16(r) if dt == torch.bfloat16 else r,
                              r32, 256, rows=v)
    # Local groups 2..5 of 8 (rows 1..659), rows outside zeroed.
    wins = []
    for variant in (1, 7, 9):
        o = torch.full((m, 256), float("nan"), dtype=torch.bfloat16, device="cuda")
        ops.gmm_fp4_out(x, b200[2:6], sc[2:6], g, o, group_offset=2, num_local_groups=4,
                        act=L.ACT_SWIGLU, zero_init=True, layout="b200", variant=variant)
        wins.append(o)
    torch.cuda.synchronize()
    L.raise_on_device_error()
    assert torch.equal(bits(wins[0]), bits(wins[1]))
    assert torch.equal(bits(wins[0]), bits(wins[2]))
    w = to_np(wins[1])
    assert np.all(w[:1] == 0) and np.all(w[660:] == 0)


def test_pair_kernel_many_short_tiles(dw):
    """Many short pair tiles per cluster (128 groups of 17-48 rows, 32 k-steps
    each): every role of the pipeline keeps pace with every stage barrier's
    phases (a waiter that falls a phase behind would time out), three
    launches in a row, with the single-CTA kernel's bits."""
    from dw_tpu_b200 import ops
    from dw_tpu_b200 import _lib as L
    rng = np.random.default_rng(33)
    sizes = rng.integers(17, 49, 128)
    m = int(sizes.sum())
    lhs, packed, scales, gs = _case(34, m, 2048, 1024, len(sizes), gs=sizes)
    b200 = ops.fp4_to_b200_out(torch.from_numpy(packed).cuda())
    sc = torch.from_numpy(scales).cuda()
    x = np_to_bf16(lhs)
    g = torch.from_numpy(gs).cuda()
    ref = torch.empty((m, 1024), dtype=torch.bfloat16, device="cuda")
    ops.gmm_fp4_out(x, b200, sc, g, ref, layout="b200", variant=1)
    for variant in (7, 9):
        for _ in range(3):
            o = torch.full((m, 1024), float("nan"), dtype=torch.bfloat16, device="cuda")
            ops.gmm_fp4_out(x, b200, sc, g, o, layout="b200", variant=variant)
            torch.cuda.synchronize()
            L.raise_on_device_error()
            assert torch.equal(o.view(torch.int16), ref.view(torch.int16)), variant


@pytest.mark.parametrize("gs,k,act,limit,sd,out_dt", [
    ([1, 0, 2, 3, 5, 8, 0, 7], 192, None, None, "u8", "bf16"),        # <= 8 rows: one n8 tile
    ([9, 16, 11, 0, 14, 3, 12, 15], 256, None, None, "u8", "f32"),    # 9-16 rows: two n8 tiles
    ([4, 6, 0, 2, 8, 1, 3, 5], 128, "swiglu", None, "u8", "bf16"),
    ([4, 6, 0, 2, 8, 1, 3, 5], 320, "swiglu", 7.0, "bf16", "bf16"),
    ([13, 2, 16, 7, 0, 10, 1, 9], 64, None, None, "f32", "bf16"),
    ([3, 1, 4, 1, 5, 9, 2, 6], 448, None, None, "u8_wide", "bf16"),   # e8m0 codes 0 and > 132
    ([12, 9, 16, 0, 14, 7, 11, 15], 256, "swiglu", None, "u8", "bf16"),  # two tiles, 128-k stages
    ([10, 16, 8, 0, 13, 9, 12, 7], 384, None, None, "u8_wide", "f32"),
    ([15, 8, 11, 16, 0, 9, 10, 14], 320, "swiglu", 7.0, "f32", "bf16"),  # two tiles, 64-k stages
])
def test_gmm_decode_regime_b200(dw, gs, k, act, limit, sd, out_dt):
    """Decode-sized groups on the B200 layout take the mma.sync kernel."""
    _decode_case(dw, gs, k, act, limit, sd, out_dt, 0)


@pytest.mark.parametrize("gs,k,act,limit,sd,out_dt", [
    ([17, 32, 0, 25, 40, 1, 33, 31], 256, None, None, "u8", "bf16"),
    ([20, 64, 18, 0, 35, 30, 29, 24], 128, "swiglu", None, "u8", "bf16"),   # 64 rows: two tasks
    ([26, 19, 31, 8, 0, 40, 22, 17], 448, None, None, "u8_wide", "f32"),    # codes 0 and > 132
    ([32, 17, 25, 30, 21, 0, 28, 19], 320, "swiglu", 7.0, "bf16", "bf16"),
    ([23, 29, 18, 32, 27, 0, 20, 31], 192, None, None, "f32", "bf16"),
])
def test_gmm_32row_tiles(dw, gs, k, act, limit, sd, out_dt):
    """Variant 5: the mma.sync decode kernel with 32-row token tiles (four n8
    tiles per decoded weight fragment, weights scaled in bf16 before the
    MMA) on groups of 17-64 rows, every scale type, against the oracle."""
    _decode_case(dw, gs, k, act, limit, sd, out_dt, 5)


def _decode_case(dw, gs, k, act, limit, sd, out_dt, variant):
    from dw_tpu_b200 import ops
    from dw_tpu_b200 import _lib as L
    m = sum(gs) + 5
    n = 512
    lo, hi = (0, 140) if sd == "u8_wide" else (118, 132)
    lhs, packed, scales, gs = _case(11, m, k, n, len(gs), gs=gs, lo=lo, hi=hi)
    if sd in ("u8", "u8_wide"):
        sc = torch.from_numpy(scales)
    elif sd == "bf16":
        sc = torch.from_numpy(O.e8m0_decode(scales)).to(torch.bfloat16)
    else:
        sc = torch.from_numpy(O.e8m0_decode(scales))
    b200 = dw.fp4_weight_to_codes(torch.from_numpy(packed).cuda())
    kind = "swiglu" if act else None
    a = {None: L.ACT_NONE, "swiglu": L.ACT_SWIGLU}[act]
    if limit is not None:
        a = L.ACT_SWIGLU_CLAMP
    dt = torch.float32 if out_dt == "f32" else torch.bfloat16
    n_out = n // 2 if act else n
    out = torch.full((m, n_out), 3.0, dtype=dt, device="cuda")
    ops.gmm_fp4_out(np_to_bf16(lhs), b200, sc.cuda(), torch.from_numpy(gs).cuda(), out, act=a,
                    act_limit=limit or 0.0, zero_init=True, layout="b200", variant=variant)
    torch.cuda.synchronize()
    L.raise_on_device_error()
    r, v = O.gmm_ref(lhs, packed, scales, gs, act=kind, limit=limit, out_dtype=out_dt)
    r32, _ = O.gmm_f32(lhs, packed, scales, gs, act=kind, limit=limit)
    got = to_np(out)
    assert_gemm_close(got, O.round_bf16(r), r32, k, rows=v)
    assert np.all(got[m - 5:] == 0)


def test_gmm_decode_regime_group_offset(dw):
    """EP shard through the mma.sync kernel: groups [3, 6) local, other rows
    untouched without zero_init."""
    from dw_tpu_b200 import ops
    lhs, packed, scales, gs = _case(12, 60, 128, 256, 8, gs=[5, 9, 2, 7, 0, 4, 11, 6])
    loc = slice(3, 6)
    b200 = dw.fp4_weight_to_codes(torch.from_numpy(packed[loc]).cuda())
    out = torch.full((60, 256), 3.0, dtype=torch.bfloat16, device="cuda")
    ops.gmm_fp4_out(np_to_bf16(lhs), b200, torch.from_numpy(scales[loc]).cuda(),
                    torch.from_numpy(gs).cuda(), out, group_offset=3, num_local_groups=3,
                    layout="b200")
    torch.cuda.synchronize()
    r, v = O.gmm_ref(lhs, packed[loc], scales[loc], gs, group_offset=3)
    r32, _ = O.gmm_f32(lhs, packed[loc], scales[loc], gs, group_offset=3)
    got = bf16_to_np(out)
    assert_gemm_close(got, r, r32, 128, rows=v)
    assert np.all(got[~v] == 3.0)


@pytest.mark.parametrize("layout", ["b200", "e2m1"])
def test_gmm_prefill_tiles(dw, layout):
    """Groups of 129-300 rows: 128-row tcgen05 tiles on one CTA and on CTA
    pairs, partial tiles, SwiGLU, against the oracle."""
    from dw_tpu_b200 import ops
    from dw_tpu_b200 import _lib as L
    gs = [300, 0, 200, 170, 129]
    m = sum(gs) + 7
    lhs, packed, scales, gs = _case(13, m, 256, 512, 5, gs=gs, lo=118, hi=121)
    raw = torch.from_numpy(packed).cuda()
    codes = dw.fp4_weight_to_codes(raw) if layout == "b200" else raw
    sc = torch.from_numpy(scales).cuda()
    g = torch.from_numpy(gs).cuda()
    for act, kind, n_out in ((L.ACT_NONE, None, 512), (L.ACT_SWIGLU, "swiglu", 256)):
        r, v = O.gmm_ref(lhs, packed, scales, gs, act=kind)
        r32, _ = O.gmm_f32(lhs, packed, scales, gs, act=kind)
        for variant in ((0, 1, 7, 8, 9) if layout == "b200" else (0,)):
            out = torch.full((m, n_out), 5.0, dtype=torch.bfloat16, device="cuda")
            ops.gmm_fp4_out(np_to_bf16(lhs), codes, sc, g, out, act=act, zero_init=True,
                            layout=layout, variant=variant)
            torch.cuda.synchronize()
            L.raise_on_device_error()
            got = bf16_to_np(out)
            assert_gemm_close(got, r, r32, 256, rows=v)
            assert np.all(got[~v] == 0), variant


@pytest.mark.parametrize("act", [None, "swiglu"])
def test_gmm_size_classes(dw, act):
    """Variant 10: each group on the kernel for its size (1-16 rows on the
    decode kernel's 16-row tiles, 17-32 on its 32-row tiles, larger groups on
    CTA pairs with 512-row tiles), on a skewed mix of groups, with
    zero_init, against the oracle."""
    from dw_tpu_b200 import ops
    from dw_tpu_b200 import _lib as L
    gs = [1, 5, 16, 0, 17, 32, 33, 64, 300, 2, 520, 8]
    m = sum(gs) + 9
    lhs, packed, scales, gs = _case(17, m, 256, 512, len(gs), gs=gs, lo=118, hi=132)
    codes = dw.fp4_weight_to_codes(torch.from_numpy(packed).cuda())
    sc = torch.from_numpy(scales).cuda()
    g = torch.from_numpy(gs).cuda()
    kind = act
    a = L.ACT_SWIGLU if act else L.ACT_NONE
    n_out = 256 if act else 512
    r, v = O.gmm_ref(lhs, packed, scales, gs, act=kind)
    r32, _ = O.gmm_f32(lhs, packed, scales, gs, act=kind)
    out = torch.full((m, n_out), 5.0, dtype=torch.bfloat16, device="cuda")
    ops.gmm_fp4_out(np_to_bf16(lhs), codes, sc, g, out, act=a, zero_init=True, layout="b200",
                    variant=10)
    torch.cuda.synchronize()
    L.raise_on_device_error()
    got = bf16_to_np(out)
    assert_gemm_close(got, r, r32, 256, rows=v)
    assert np.all(got[~v] == 0)


def test_gmm_deterministic(dw):
    lhs, packed, scales, gs = _case(7, 300, 256, 512, 4)
    a = _run_gmm(dw, lhs, packed, scales, gs)
    b = _run_gmm(dw, lhs, packed, scales, gs)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_gmm_bad_group_sizes_reported(dw):
    """Group sizes summing past M are clamped and flagged in the status word."""
    from dw_tpu_b200 import _lib
    lhs, packed, scales, _ = _case(8, 32, 64, 256, 2)
    gs = np.array([30, 30], np.int32)
    out = dw.gmm_v2(np_to_bf16(lhs), torch.from_numpy(packed).cuda(),
                    torch.from_numpy(gs).cuda(), torch.from_numpy(scales).cuda())
    bits = _lib.device_status()
    assert bits & _lib.DEV_BAD_INDEX
    assert out.shape == (32, 256)


@pytest.mark.parametrize("scale_exp", [-70, 0, 40])
@pytest.mark.parametrize("variant", [3, 4])
def test_decode_kernel_token_magnitudes(dw, scale_exp, variant):
    """The mma.sync decode kernel keeps the reference's products for tokens
    far from 1: whole token rows of magnitude ~2^-70 (which a fixed 2^64
    token pre-scale used to flush) and ~2^40, with E8M0 codes that take both
    the post-MMA path and the exact path (code 0 and codes above its range)."""
    from dw_tpu_b200 import ops
    from dw_tpu_b200 import _lib as L
    wide_hi = 215 if scale_exp <= 0 else 160  # keep the reference's f32 sums finite
    for lo, hi in ((118, 130), (0, wide_hi)):
        lhs, packed, scales, gs = _case(21, 96, 256, 512, 8, lo=lo, hi=hi)
        lhs = (lhs * np.float32(2.0) ** scale_exp).astype(np.float32)  # exact power-of-two scaling
        b200 = dw.fp4_weight_to_codes(torch.from_numpy(packed).cuda())
        out = torch.full((96, 512), 3.0, dtype=torch.bfloat16, device="cuda")
        ops.gmm_fp4_out(np_to_bf16(lhs), b200, torch.from_numpy(scales).cuda(),
                        torch.from_numpy(gs).cuda(), out, zero_init=True, layout="b200",
                        variant=variant)
        torch.cuda.synchronize()
        L.raise_on_device_error()
        r, v = O.gmm_ref(lhs, packed, scales, gs)
        r32, _ = O.gmm_f32(lhs, packed, scales, gs)
        got = bf16_to_np(out)
        assert np.all(np.isfinite(r32[v])), "the case must stay in range for the reference"
        assert_gemm_close(got, r, r32, 256, rows=v)
