"""On-device FP4 weight preparation (dwm_fp4_quantize) vs the oracle's
quantize_tensor restatement (B01:319-347): bit-exact codes and scales."""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from tests.golden import make_golden

pytestmark = pytest.mark.gpu


def _oracle(w, pow2):
    """Blocks of 32 along k of w [g, k, n]: the oracle quantises the last
    axis, so quantise w^T and transpose back."""
    nib, sc = O.quantize_fp4_block32(np.swapaxes(w, -1, -2), power_of_two_scale=pow2)
    return (O.pack_nibbles(np.ascontiguousarray(np.swapaxes(nib, -1, -2))),
            np.ascontiguousarray(np.swapaxes(sc, -1, -2)))


@pytest.mark.parametrize("dtype,pow2", [("f32", True), ("f32", False), ("bf16", True)])
def test_quantize_matches_oracle(dtype, pow2):
    from dw_tpu_b200 import ops
    rng = np.random.default_rng(3)
    g, k, n = 3, 256, 96
    w = (rng.standard_normal((g, k, n)) * np.exp(rng.uniform(-6, 3, (g, 1, n)))).astype(
        np.float32)
    w[0, :32, 5] = 0.0               # an all-zero block: scale 0, codes 0
    w[1, 40, 7] = -1e-30             # tiny negative rounds to +0
    if dtype == "bf16":
        w = O.round_bf16(w)
        wt = torch.from_numpy(O.f32_to_bf16_bits(w).view(np.int16)).view(torch.bfloat16)
    else:
        wt = torch.from_numpy(w)
    codes = torch.empty((g, k, n // 2), dtype=torch.uint8, device="cuda")
    scales = torch.empty((g, k // 32, n), dtype=torch.float32, device="cuda")
    ops.fp4_quantize_out(wt.cuda(), codes, scales, power_of_two_scale=pow2)
    ref_codes, ref_scales = _oracle(w, pow2)
    assert np.array_equal(scales.cpu().numpy(), ref_scales)
    assert np.array_equal(codes.cpu().numpy(), ref_codes)


def test_requant_known_answer_on_device():
    """B01:131-157: re-quantising MXFP4 data with power-of-two scales gives
    back the same values; E8M0 scales come out lossless."""
    from dw_tpu_b200 import ops
    d = make_golden.requant_kat(seed=0)
    original = np.ascontiguousarray(np.swapaxes(d["original"], -1, -2))  # blocks along k
    g, k, n = original.shape
    codes = torch.empty((g, k, n // 2), dtype=torch.uint8, device="cuda")
    scales = torch.empty((g, k // 32, n), dtype=torch.uint8, device="cuda")
    lossless = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.fp4_quantize_out(torch.from_numpy(original).cuda(), codes, scales, lossless)
    assert int(lossless.item()) == 1
    back = O.dequant_fp4_f32(codes.cpu().numpy(), scales.cpu().numpy())
    assert np.array_equal(back, original)


def test_from_dense_weights_run_the_layer():
    """FP4MoEWeights.from_dense on dequantised MXFP4 experts gives back the
    same weight values (codes may shift with the scale), so the layer gives
    the same bits."""
    import dw_tpu_b200 as dw
    from dw_tpu_b200 import synthetic
    e, h, i, t, k = 8, 256, 128, 16, 4
    w = synthetic.moe_weights(e, h, i, seed=8, device="cuda")
    dense13 = O.dequant_fp4_f32(w.w13.cpu().numpy(), w.s13.cpu().numpy())
    dense2 = O.dequant_fp4_f32(w.w2.cpu().numpy(), w.s2.cpu().numpy())
    w2 = dw.FP4MoEWeights.from_dense(torch.from_numpy(dense13).cuda(),
                                     torch.from_numpy(dense2).cuda())
    assert np.array_equal(O.dequant_fp4_f32(w2.w13.cpu().numpy(), w2.s13.cpu().numpy()), dense13)
    assert np.array_equal(O.dequant_fp4_f32(w2.w2.cpu().numpy(), w2.s2.cpu().numpy()), dense2)
    x, router = synthetic.layer_inputs(t, h, e, seed=9)
    x = x.cuda()
    lg = (x.float() @ router.cuda().float()).to(torch.bfloat16)
    a = dw.MoELayer(w, k, t)(x, lg)
    b = dw.MoELayer(w2, k, t)(x, lg)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
