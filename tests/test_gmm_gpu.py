"""FP4 grouped matmul on the GPU vs the oracle (through the C ABI)."""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from tests.gpu_util import assert_gemm_close, bf16_to_np, np_to_bf16

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
