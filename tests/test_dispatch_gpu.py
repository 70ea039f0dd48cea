"""Routing, permute, gather, combine and e8m0 on the GPU vs the oracle:
bit-exact for the integer/data-movement ops and the k-order combine."""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from tests.gpu_util import bf16_to_np, np_to_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dw():
    import dw_tpu_b200
    return dw_tpu_b200


def _ids(t, e, k, seed, dist="uniform"):
    from dw_tpu_b200 import synthetic
    ids, w = synthetic.route_ids(t, e, k, seed=seed, dist=dist)
    return ids, w


def test_permute_golden(dw, golden):
    d = golden("permute_small")
    argsort, tok, revert, gs = dw.moe_permute(torch.from_numpy(d["ids"]).cuda(), 16)
    assert np.array_equal(argsort.cpu().numpy(), d["argsort"])
    assert np.array_equal(tok.cpu().numpy(), d["tok"])
    assert np.array_equal(revert.cpu().numpy(), d["revert"])
    assert np.array_equal(gs.cpu().numpy(), d["group_sizes"])
    x = dw.dispatch_gather(np_to_bf16(O.bf16_bits_to_f32(d["hidden_bits"])), tok)
    assert np.array_equal(x.cpu().view(torch.int16).numpy().view(np.uint16), d["x_bits"])


@pytest.mark.parametrize("t,e,k,dist", [
    (1, 256, 8, "uniform"), (64, 256, 8, "uniform"), (512, 256, 8, "zipf"),
    (8192, 256, 8, "uniform"), (3000, 32, 6, "zipf"), (0, 16, 4, "uniform"),
    (100, 1024, 8, "uniform"),
])
def test_permute_bit_exact(dw, t, e, k, dist):
    if t:
        ids, _ = _ids(t, e, k, seed=t + e, dist=dist)
    else:
        ids = np.zeros((0, k), np.int32)
    argsort, tok, revert, gs = dw.moe_permute(torch.from_numpy(ids).cuda(), e)
    ra, rt, rr, rg = O.permute(ids, e)
    assert np.array_equal(argsort.cpu().numpy(), ra)
    assert np.array_equal(tok.cpu().numpy(), rt)
    assert np.array_equal(revert.cpu().numpy(), rr)
    assert np.array_equal(gs.cpu().numpy(), rg)


def test_permute_repeated_ids_stable(dw):
    """Repeated expert ids inside a token (no dedupe) keep flat order."""
    rng = np.random.default_rng(9)
    ids = rng.integers(0, 4, (700, 8)).astype(np.int32)
    argsort, tok, revert, gs = dw.moe_permute(torch.from_numpy(ids).cuda(), 4)
    ra, rt, rr, rg = O.permute(ids, 4)
    assert np.array_equal(argsort.cpu().numpy(), ra)
    assert np.array_equal(gs.cpu().numpy(), rg)


def test_permute_bad_id_reported(dw):
    from dw_tpu_b200 import _lib
    ids = np.array([[0, 1], [2, 99]], np.int32)
    _, _, _, gs = dw.moe_permute(torch.from_numpy(ids).cuda(), 4)
    assert _lib.device_status() & _lib.DEV_BAD_INDEX
    assert gs.cpu().tolist() == [1, 1, 1, 0]


def test_sorted_token_indices_and_fast_dispatch(dw):
    rng = np.random.default_rng(1)
    ids = rng.integers(0, 64, (333, 8)).astype(np.int32)
    argsort = np.argsort(ids.reshape(-1), kind="stable").astype(np.int32)
    got = dw.sorted_token_indices(torch.from_numpy(argsort).cuda(), 8)
    assert np.array_equal(got.cpu().numpy(), np.repeat(np.arange(333), 8)[argsort])
    hidden = O.round_bf16(rng.standard_normal((333, 4096)).astype(np.float32))
    for mode in (0, 1, 2):
        x = dw.fast_dispatch_gather(np_to_bf16(hidden), torch.from_numpy(argsort).cuda(), 8,
                                    mode)
        assert np.array_equal(bf16_to_np(x), hidden[np.repeat(np.arange(333), 8)[argsort]])


def test_combine_golden(dw, golden):
    d = golden("combine_small")
    y = np_to_bf16(O.bf16_bits_to_f32(d["y_bits"]))
    idx = torch.from_numpy(d["idx"]).cuda()
    w = torch.from_numpy(d["w"]).cuda()
    out = dw.fast_combine(y, idx, w, 6, mode=2, out_dtype=torch.bfloat16)
    assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), d["out_bits"])
    out32 = dw.combine_xla(y, idx, w, 6, out_dtype=torch.float32)
    assert np.array_equal(out32.cpu().numpy(), d["out_f32"])


@pytest.mark.parametrize("xdt", ["bf16", "f32"])
@pytest.mark.parametrize("wdt", ["bf16", "f32"])
def test_combine_bit_exact(dw, xdt, wdt):
    rng = np.random.default_rng(2)
    t, k, h = 257, 8, 4096
    y = rng.standard_normal((t * k, h)).astype(np.float32)
    if xdt == "bf16":
        y = O.round_bf16(y)
        y_t = np_to_bf16(y)
    else:
        y_t = torch.from_numpy(y).cuda()
    w = rng.dirichlet(np.ones(k), size=t).astype(np.float32)
    if wdt == "bf16":
        w = O.round_bf16(w)
        w_t = np_to_bf16(w)
    else:
        w_t = torch.from_numpy(w).cuda()
    idx = rng.permutation(t * k).astype(np.int32)
    out = dw.fast_combine(y_t, torch.from_numpy(idx).cuda(), w_t, k, mode=1,
                          out_dtype=torch.bfloat16)
    assert np.array_equal(bf16_to_np(out), O.combine(y, idx, w, k))


@pytest.mark.parametrize("f32_reduce", [False, True])
@pytest.mark.parametrize("shdt,odt", [("f32", "bf16"), ("bf16", "bf16"), ("f32", "f32")])
def test_combine_shared_bit_exact(dw, f32_reduce, shdt, odt):
    """The shared expert summed into the combine (X0104:80-87): bit-exact
    against the oracle's f32(mid(routed)) * routed_scale + shared."""
    rng = np.random.default_rng(9)
    t, k, h = 129, 6, 1024
    y = O.round_bf16(rng.standard_normal((t * k, h)).astype(np.float32))
    w = rng.dirichlet(np.ones(k), size=t).astype(np.float32)
    idx = rng.permutation(t * k).astype(np.int32)
    sh = (rng.standard_normal((t, h)) * 0.5).astype(np.float32)
    if shdt == "bf16":
        sh = O.round_bf16(sh)
        sh_t = np_to_bf16(sh)
    else:
        sh_t = torch.from_numpy(sh).cuda()
    odtype = torch.bfloat16 if odt == "bf16" else torch.float32
    out = dw.combine_shared(np_to_bf16(y), torch.from_numpy(idx).cuda(),
                            torch.from_numpy(w).cuda(), k, sh_t, routed_scale=2.5,
                            f32_reduce=f32_reduce, out_dtype=odtype)
    want = O.combine_shared(y, idx, w, k, sh, 2.5, mid_dtype="f32" if f32_reduce else "bf16",
                            out_dtype=odt)
    got = bf16_to_np(out) if odt == "bf16" else out.cpu().numpy()
    assert np.array_equal(got, want)
    # routed_scale 1 and a zero shared partial give back the plain combine
    # (up to the mid rounding, which the bf16 output repeats).
    zero = torch.zeros((t, h), dtype=torch.float32, device="cuda")
    out0 = dw.combine_shared(np_to_bf16(y), torch.from_numpy(idx).cuda(),
                             torch.from_numpy(w).cuda(), k, zero)
    assert np.array_equal(bf16_to_np(out0), O.combine(y, idx, w, k))


@pytest.mark.parametrize("fn", ["sigmoid", "softmax", "sqrtsoftplus"])
def test_route_topk_golden(dw, golden, fn):
    d = golden("route_small")
    logits = np_to_bf16(O.bf16_bits_to_f32(d["logits_bits"]))
    w, ids = dw.route_topk(logits, 8, renormalize=True, scoring_fn=fn, dtype=torch.float32)
    assert np.array_equal(ids.cpu().numpy(), d[f"{fn}_ids"])
    np.testing.assert_allclose(w.cpu().numpy(), d[f"{fn}_w"], rtol=2e-6, atol=1e-7)


def test_route_topk_bias_and_padding(dw):
    rng = np.random.default_rng(3)
    logits = O.round_bf16(rng.standard_normal((40, 256)).astype(np.float32))
    bias = (rng.standard_normal(256) * 0.1).astype(np.float32)
    w, ids = dw.route_topk(np_to_bf16(logits), 8, scoring_fn="sigmoid",
                           bias=torch.from_numpy(bias).cuda(), num_valid_tokens=33,
                           dtype=torch.float32)
    rid, rw = O.route_topk(logits, 8, "sigmoid", True, bias=bias, num_valid_tokens=33)
    assert np.array_equal(ids.cpu().numpy(), rid)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)
    assert np.all(ids.cpu().numpy()[33:] == 0) and np.all(w.cpu().numpy()[33:] == 0)


@pytest.mark.parametrize("fn", ["sigmoid", "sqrtsoftplus", "softmax"])
def test_route_hash(dw, fn):
    """Hash routing (E0901:667-671): given ids, weights = scores at them."""
    rng = np.random.default_rng(4)
    t, e, k = 37, 64, 6
    logits = O.round_bf16(rng.standard_normal((t, e)).astype(np.float32))
    hid = rng.integers(0, e, (t, k)).astype(np.int32)   # repeats allowed
    w, ids = dw.route_hash(np_to_bf16(logits), torch.from_numpy(hid).cuda(), scoring_fn=fn,
                           num_valid_tokens=30, dtype=torch.float32)
    rid, rw = O.route_hash(logits, hid, fn, True, num_valid_tokens=30)
    assert np.array_equal(ids.cpu().numpy(), rid)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)


def test_dedupe_topk_bit_exact(dw):
    """E0901:98-121: repeated ids fold their weight into the first occurrence
    and move to the lowest unused expert with weight 0."""
    rng = np.random.default_rng(5)
    t, e, k = 200, 16, 8
    ids = rng.integers(0, 6, (t, k)).astype(np.int32)   # many repeats
    ids[0] = [3, 3, 3, 3, 3, 3, 3, 3]
    ids[1] = np.arange(8)                                 # already distinct
    w = rng.random((t, k)).astype(np.float32)
    gw, gi = dw.dedupe_topk(torch.from_numpy(w).cuda(), torch.from_numpy(ids).cuda(), e)
    rw, ri = O.dedupe_topk(w, ids, e)
    assert np.array_equal(gi.cpu().numpy(), ri)
    assert np.array_equal(gw.cpu().numpy(), rw)
    assert all(len(set(r)) == k for r in gi.cpu().numpy().tolist())


def test_route_ties_go_to_lower_index(dw):
    logits = torch.zeros((2, 64), dtype=torch.float32, device="cuda")
    w, ids = dw.route_topk(logits, 4, scoring_fn="softmax", dtype=torch.float32)
    assert ids.cpu().tolist() == [[0, 1, 2, 3], [0, 1, 2, 3]]


def test_e8m0_roundtrip(dw):
    e = np.arange(-126, 128)
    s = np.ldexp(np.ones(e.shape, np.float32), e).astype(np.float32)
    codes, lossless = dw.e8m0_encode(torch.from_numpy(s).cuda())
    assert bool(lossless)
    rc, _ = O.e8m0_encode(s)
    assert np.array_equal(codes.cpu().numpy(), rc)
    back = dw.e8m0_decode(codes)
    assert np.array_equal(back.cpu().numpy().view(np.uint32), s.view(np.uint32))
    _, lossless = dw.e8m0_encode(torch.tensor([1.0, 3.0], device="cuda"))
    assert not bool(lossless)
