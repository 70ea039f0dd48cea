"""The single-device MoE layer on the GPU vs the oracle: a reduced layer in
full, and the BASELINE config-1 layer (T=64, H=4096, I=2048, E=256, top-8) on
all of its tokens."""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from tests.gpu_util import (assert_layer_close, bf16_to_np, gemm_rel_tol, rel_fro,
                             torch_dequant, torch_layer_reference)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dw():
    import dw_tpu_b200
    return dw_tpu_b200


def _layer(dw, t, e, h, i, k, seed, lo=118, hi=121, f32_reduce=False):
    from dw_tpu_b200 import synthetic
    w = synthetic.moe_weights(e, h, i, seed=seed, device="cuda")
    for name in ("s13", "s2"):  # keep activations O(1): scales 2^-9..2^-6
        setattr(w, name, synthetic.random_e8m0(getattr(w, name).shape, seed + 5, "cuda",
                                               lo=lo, hi=hi))
    x, router = synthetic.layer_inputs(t, h, e, seed=seed)
    logits = (x.float() @ router.float()).to(torch.bfloat16)
    layer = dw.MoELayer(w, k, t, f32_reduce=f32_reduce)
    out = layer(x.cuda(), logits.cuda())
    torch.cuda.synchronize()
    from dw_tpu_b200 import _lib
    _lib.raise_on_device_error()
    return w, x, logits, layer, out


@pytest.mark.parametrize("f32_reduce", [False, True])
def test_layer_small_matches_oracle(dw, f32_reduce):
    t, e, h, i, k = 24, 16, 512, 256, 4
    w, x, logits, layer, out = _layer(dw, t, e, h, i, k, seed=1, f32_reduce=f32_reduce)
    ref = O.fused_moe(bf16_to_np(x), bf16_to_np(logits), w.w13.cpu().numpy(),
                      w.s13.cpu().numpy(), w.w2.cpu().numpy(), w.s2.cpu().numpy(), k,
                      f32_reduce=f32_reduce)
    ids, _ = O.route_topk(bf16_to_np(logits), k, "sigmoid", True)
    assert np.array_equal(layer.ids[:t].cpu().numpy(), ids)
    got = bf16_to_np(out)
    rf = rel_fro(got, ref)
    assert rf < 2 * gemm_rel_tol(i), rf


def test_layer_cfg1_all_tokens(dw):
    """The full BASELINE config-1 decode layer (T=64, H=4096, I=2048, E=256
    FP4 experts, top-8 sigmoid, the bench's E8M0 exponents -4..2) on the
    B200 layout, i.e. the decode kernel at K=4096 and 2048 over ~224 experts:
    routing bit-exact against the oracle, and every one of the 64 output rows
    against a plain-PyTorch fp32 restatement of the reference numerics whose
    dequant is pinned to the oracle's."""
    from dw_tpu_b200 import _lib, synthetic
    t, e, h, i, k = 64, 256, 4096, 2048, 8
    w = synthetic.moe_weights(e, h, i, seed=2, device="cuda")
    x, router = synthetic.layer_inputs(t, h, e, seed=2)
    logits = (x.float() @ router.float()).to(torch.bfloat16)
    layer = dw.MoELayer(w.to_b200(), k, t)
    out = layer(x.cuda(), logits.cuda())
    torch.cuda.synchronize()
    _lib.raise_on_device_error()
    ids, wts = O.route_topk(bf16_to_np(logits), k, "sigmoid", True)
    assert np.array_equal(layer.ids.cpu().numpy(), ids)
    assert np.array_equal(bf16_to_np(layer.w16), O.round_bf16(wts))
    for ex in (int(ids[0, 0]), int(ids[37, 5])):
        for wq, sq in ((w.w13, w.s13), (w.w2, w.s2)):
            assert np.array_equal(torch_dequant(wq[ex], sq[ex]).cpu().numpy(),
                                  O.dequant_fp4_block(wq[ex].cpu().numpy(), sq[ex].cpu().numpy()))
    ref = torch_layer_reference(x.cuda(), layer.ids, layer.w16, w.w13, w.s13, w.w2, w.s2)
    assert_layer_close(out, ref, i, "cfg1 layer")


def test_layer_graph_capture_replays_bitwise(dw):
    t, e, h, i, k = 32, 16, 512, 256, 4
    w, x, logits, layer, out = _layer(dw, t, e, h, i, k, seed=3)
    xc, lc = x.cuda(), logits.cuda()
    res = torch.empty_like(out)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        layer(xc, lc, out=res)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        layer(xc, lc, out=res)
    res.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(res.view(torch.int16), out.view(torch.int16))


def test_layer_prefill_pair_kernel(dw):
    """A prefill-sized layer (512 tokens, top-8 over 16 experts: ~256 rows
    per expert) takes the GEMM on CTA pairs with 512-row tiles automatically
    (variant 9): it replays bitwise from a CUDA graph, matches the oracle
    layer and has the single-CTA kernel's bits, as does the pair kernel with
    256-row tiles (variant 7); variant 8 (256-row pair tiles, short group
    remainders on the decode kernel) matches the oracle layer."""
    from dw_tpu_b200 import synthetic
    t, e, h, i, k = 512, 16, 512, 256, 8
    w = synthetic.moe_weights(e, h, i, seed=8, device="cuda")
    for name in ("s13", "s2"):
        setattr(w, name, synthetic.random_e8m0(getattr(w, name).shape, 13, "cuda", lo=118,
                                               hi=121))
    raw, w = w, w.to_b200()
    x, router = synthetic.layer_inputs(t, h, e, seed=8)
    xc = x.cuda()
    lc = (x.float() @ router.float()).to(torch.bfloat16).cuda()
    auto = dw.MoELayer(w, k, t)
    pair = dw.MoELayer(w, k, t, gemm_variant=7)
    tails = dw.MoELayer(w, k, t, gemm_variant=8)
    single = dw.MoELayer(w, k, t, gemm_variant=1)
    out = auto(xc, lc)
    out_pair = pair(xc, lc)
    out_tails = tails(xc, lc)
    ref_bits = single(xc, lc)
    torch.cuda.synchronize()
    from dw_tpu_b200 import _lib
    _lib.raise_on_device_error()
    assert int(auto.group_sizes.float().mean().item()) >= 128
    assert int(auto.group_sizes.max().item()) > 256  # two UMMAs per k-step / a remainder
    assert torch.equal(out_pair.view(torch.int16), ref_bits.view(torch.int16))
    assert torch.equal(out.view(torch.int16), ref_bits.view(torch.int16))
    res = torch.empty_like(out)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        auto(xc, lc, out=res)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        auto(xc, lc, out=res)
    res.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(res.view(torch.int16), out.view(torch.int16))
    ref = O.fused_moe(bf16_to_np(x), bf16_to_np(lc.cpu()), raw.w13.cpu().numpy(),
                      raw.s13.cpu().numpy(), raw.w2.cpu().numpy(), raw.s2.cpu().numpy(), k)
    assert rel_fro(bf16_to_np(out), ref) < 2 * gemm_rel_tol(h)
    assert rel_fro(bf16_to_np(out_tails), ref) < 2 * gemm_rel_tol(h)


@pytest.mark.parametrize("layout,f32_reduce,limit", [("e2m1", False, None), ("b200", True, None),
                                                      ("b200", False, 7.0)])
def test_one_call_layer_matches_layer_object(dw, layout, f32_reduce, limit):
    """dwm_moe_layer_fp4 (one C call, caller workspace) gives the bits of the
    six-call MoELayer, on two calls in a row with new tokens."""
    from dw_tpu_b200 import ops, synthetic
    t, e, h, i, k = 40, 16, 512, 256, 4
    w = synthetic.moe_weights(e, h, i, seed=6, device="cuda")
    for name in ("s13", "s2"):
        setattr(w, name, synthetic.random_e8m0(getattr(w, name).shape, 11, "cuda", lo=118,
                                               hi=121))
    if layout == "b200":
        w = w.to_b200()
    layer = dw.MoELayer(w, k, t, f32_reduce=f32_reduce, act_limit=limit)
    nbytes = ops.moe_layer_workspace_bytes(t, h, i, k, e, f32_reduce)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    for seed in (30, 31):
        x, router = synthetic.layer_inputs(t, h, e, seed=seed)
        x = x.cuda()
        lg = (x.float() @ router.cuda().float()).to(torch.bfloat16)
        ref = layer(x, lg)
        got = torch.empty_like(ref)
        ops.moe_layer_fp4_out(x, lg, k, w.w13, w.s13, w.w2, w.s2, got, ws, layout=layout,
                              f32_reduce=f32_reduce, act_limit=limit)
        torch.cuda.synchronize()
        from dw_tpu_b200 import _lib
        _lib.raise_on_device_error()
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), seed
    with pytest.raises(ValueError):
        ops.moe_layer_fp4_out(x, lg, k, w.w13, w.s13, w.w2, w.s2, got, ws[:nbytes // 2],
                              layout=layout, f32_reduce=f32_reduce, act_limit=limit)
