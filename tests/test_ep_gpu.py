"""Expert-parallel one-shot dispatch / combine on the GPU vs the oracle,
bit-exact: the exchange of ``world`` ranks emulated on one device (all
contexts in this process, phases issued rank by rank so that every wait is
already satisfied when it runs)."""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from tests.gpu_util import bf16_to_np, np_to_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ep():
    from dw_tpu_b200 import ep as E
    return E


def _inputs(world, t_per_rank, e, k, h, seed, dist="uniform"):
    from dw_tpu_b200 import synthetic
    rng = np.random.default_rng(seed)
    hid, ids, w = [], [], []
    for r in range(world):
        t = t_per_rank[r] if isinstance(t_per_rank, (list, tuple)) else t_per_rank
        hid.append(O.round_bf16(rng.standard_normal((t, h)).astype(np.float32)))
        if t:
            i, ww = synthetic.route_ids(t, e, k, seed=seed * 31 + r, dist=dist)
        else:
            i, ww = np.zeros((0, k), np.int32), np.zeros((0, k), np.float32)
        ids.append(i)
        w.append(ww)
    return hid, ids, w


def _bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def _exchange_bit_exact(ep, world, t, e, k, h, dist, seed):
    """One dispatch + combine of `world` emulated ranks against the oracle:
    receive rows, group sizes and combine output bit for bit."""
    hid, ids, w = _inputs(world, t, e, k, h, seed=seed, dist=dist)
    tmax = max(x.shape[0] for x in hid) or 1
    ctxs = ep.create_local_contexts(world, max_tokens=tmax, hidden=h, topk=k, num_experts=e)
    try:
        res = ep.emulated_dispatch(ctxs, [np_to_bf16(x) for x in hid],
                                   [torch.from_numpy(i).cuda() for i in ids])
        torch.cuda.synchronize()
        from dw_tpu_b200 import _lib as L
        L.raise_on_device_error()
        ref = O.ep_dispatch(hid, ids, e)
        ys = []
        for r, ((recv, gs), (rrows, rgs, rsrc)) in enumerate(zip(res, ref)):
            n = int(rgs.sum())
            assert np.array_equal(gs.cpu().numpy(), rgs), r
            assert np.array_equal(_bits(recv[:n]), O.f32_to_bf16_bits(rrows)), r
            # expert outputs: any values, in receive order (the received rows only)
            y = O.round_bf16(np.random.default_rng(r).standard_normal(
                (max(n, 1), h)).astype(np.float32))
            ys.append(y)
        outs = ep.emulated_combine(ctxs, [np_to_bf16(y) for y in ys],
                                   [torch.from_numpy(x).cuda() for x in w])
        torch.cuda.synchronize()
        L.raise_on_device_error()
        want = O.ep_combine_korder([y[:int(g[1].sum())] for y, g in zip(ys, ref)],
                                   [g[2] for g in ref], w)
        for r in range(world):
            assert np.array_equal(bf16_to_np(outs[r]), want[r]), r
    finally:
        for c in ctxs:
            c.close()


@pytest.mark.parametrize("world,t,e,k,h,dist", [
    (2, 16, 256, 8, 4096, "uniform"),
    (4, 128, 256, 8, 512, "zipf"),
    (8, 64, 256, 8, 256, "uniform"),
    (8, [5, 0, 17, 64, 1, 33, 2, 9], 64, 6, 128, "zipf"),   # ragged, one empty rank
    (1, 40, 16, 4, 64, "uniform"),                           # degenerate: no exchange
])
def test_ep_dispatch_combine_bit_exact(ep, world, t, e, k, h, dist):
    _exchange_bit_exact(ep, world, t, e, k, h, dist, seed=world + e)


@pytest.mark.parametrize("world", [4, 8])
@pytest.mark.parametrize("dist", ["uniform", "zipf"])
def test_ep_cfg2_full_size_bit_exact(ep, world, dist):
    """BASELINE config 2 at its largest size: 512 tokens per rank of H=4096,
    top-8 over 256 experts, uniform or Zipf(1.2) routing, 4 and 8 ranks."""
    _exchange_bit_exact(ep, world, 512, 256, 8, 4096, dist, seed=40 + world)


@pytest.mark.parametrize("t", [2, 16, 64, 128, 256, 512])
def test_ep_cfg4_token_counts_bit_exact(ep, t):
    """BASELINE config 4's per-rank token counts ({1, 8, 32, 64, 128, 256}
    doubled) on 8 ranks with Zipf(1.2) routing, which leaves some experts
    empty and others hot."""
    _exchange_bit_exact(ep, 8, t, 256, 8, 4096, "zipf", seed=60 + t)


def test_ep_wait_runs_out_and_recovers(ep):
    """A rank that never publishes its counts: the other rank's dispatch waits
    on a count word that nothing writes, gives up after the shortened limit
    (10 ms) with DWM_DEV_TIMEOUT and returns; after every rank's context is
    created again, the next exchange is bit-exact."""
    import time
    from dw_tpu_b200 import _lib as L
    world, t, e, k, h = 2, 16, 32, 4, 256
    hid, ids, _ = _inputs(world, t, e, k, h, seed=91)
    ctxs = ep.create_local_contexts(world, max_tokens=t, hidden=h, topk=k, num_experts=e)
    try:
        for c in ctxs:
            c.set_wait_limit(0.01)
        assert L.device_status() == 0
        x0, i0 = np_to_bf16(hid[0]), torch.from_numpy(ids[0]).cuda()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for phase in (L.EP_COUNTS, L.EP_ROWS, L.EP_WAIT):  # rank 1 never runs COUNTS
            ctxs[0].dispatch(x0, i0, phases=phase)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        bits = L.device_status()
        assert bits & L.DEV_TIMEOUT, bits
        assert elapsed < 5.0, elapsed  # two bounded waits of 10 ms, not the 2 s default
        with pytest.raises(ValueError):
            ctxs[0].set_wait_limit(0.0)
    finally:
        for c in ctxs:
            c.close()
    _exchange_bit_exact(ep, world, t, e, k, h, "uniform", seed=92)
    assert L.device_status() == 0


def test_ep_repeated_steps_and_f32_outputs(ep):
    """Monotonic epochs: several steps in a row with new inputs each time; f32
    expert outputs and f32 combine output."""
    world, e, k, h = 4, 32, 4, 256
    ctxs = ep.create_local_contexts(world, max_tokens=48, hidden=h, topk=k, num_experts=e)
    from dw_tpu_b200 import _lib as L
    try:
        for step in range(5):
            t = [48, 7, 30, 0][step % 4:] + [48, 7, 30, 0][:step % 4]
            hid, ids, w = _inputs(world, t, e, k, h, seed=100 + step, dist="zipf")
            ep.emulated_dispatch(ctxs, [np_to_bf16(x) for x in hid],
                                 [torch.from_numpy(i).cuda() for i in ids])
            ref = O.ep_dispatch(hid, ids, e)
            ys = [np.random.default_rng(step * 8 + r).standard_normal(
                (ctxs[r].capacity, h)).astype(np.float32) for r in range(world)]
            outs = [torch.empty((hid[r].shape[0], h), dtype=torch.float32, device="cuda")
                    for r in range(world)]
            ep.emulated_combine(ctxs, [torch.from_numpy(y).cuda() for y in ys],
                                [torch.from_numpy(x).cuda() for x in w], outs)
            torch.cuda.synchronize()
            L.raise_on_device_error()
            for r in range(world):
                n = int(ref[r][1].sum())
                assert np.array_equal(ctxs[r].recv_group_sizes.cpu().numpy(), ref[r][1])
                assert np.array_equal(_bits(ctxs[r].recv[:n]), O.f32_to_bf16_bits(ref[r][0]))
            want = O.ep_combine_korder([y[:int(g[1].sum())] for y, g in zip(ys, ref)],
                                       [g[2] for g in ref], w, out_dtype="f32")
            for r in range(world):
                assert np.array_equal(outs[r].cpu().numpy(), want[r]), (step, r)
    finally:
        for c in ctxs:
            c.close()


def test_ep_graph_replay_advances_epoch(ep):
    """The exchange captured once in a CUDA graph and replayed with new inputs
    copied into the captured tensors: the epoch advances on the device, so
    every replay matches the oracle (the count parity alternates too)."""
    world, e, k, h, t = 4, 32, 4, 256, 24
    from dw_tpu_b200 import _lib as L
    ctxs = ep.create_local_contexts(world, max_tokens=t, hidden=h, topk=k, num_experts=e)
    try:
        hs = [torch.empty((t, h), dtype=torch.bfloat16, device="cuda") for _ in range(world)]
        ids = [torch.empty((t, k), dtype=torch.int32, device="cuda") for _ in range(world)]
        ws = [torch.empty((t, k), dtype=torch.float32, device="cuda") for _ in range(world)]
        ys = [torch.empty((c.capacity, h), dtype=torch.bfloat16, device="cuda") for c in ctxs]
        outs = [torch.empty((t, h), dtype=torch.float32, device="cuda") for _ in range(world)]

        def load(step):
            hid, i, w = _inputs(world, t, e, k, h, seed=300 + step, dist="zipf")
            for r in range(world):
                hs[r].copy_(np_to_bf16(hid[r]))
                ids[r].copy_(torch.from_numpy(i[r]))
                ws[r].copy_(torch.from_numpy(w[r]))
                ys[r].copy_(np_to_bf16(O.round_bf16(np.random.default_rng(step * 8 + r)
                                                    .standard_normal((ctxs[r].capacity, h))
                                                    .astype(np.float32))))
            return hid, i, w

        def step():
            ep.emulated_dispatch(ctxs, hs, ids)
            ep.emulated_combine(ctxs, ys, ws, outs)

        def check(hid, i, w):
            torch.cuda.synchronize()
            L.raise_on_device_error()
            ref = O.ep_dispatch(hid, i, e)
            yn = [bf16_to_np(y) for y in ys]
            for r in range(world):
                n = int(ref[r][1].sum())
                assert np.array_equal(ctxs[r].recv_group_sizes.cpu().numpy(), ref[r][1])
                assert np.array_equal(_bits(ctxs[r].recv[:n]), O.f32_to_bf16_bits(ref[r][0]))
            want = O.ep_combine_korder([y[:int(g[1].sum())] for y, g in zip(yn, ref)],
                                       [g[2] for g in ref], w, out_dtype="f32")
            for r in range(world):
                assert np.array_equal(outs[r].cpu().numpy(), want[r]), r

        inputs = load(0)
        step()                                             # eager step: epoch 1
        check(*inputs)
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side), torch.cuda.graph(g, stream=side):
            step()
        torch.cuda.current_stream().wait_stream(side)
        for s in range(1, 5):                              # replays: epochs 2..5
            inputs = load(s)
            g.replay()
            check(*inputs)
        del g
    finally:
        for c in ctxs:
            c.close()


def test_ep_combine_with_shared_expert(ep):
    """The EP combine with a shared expert summed in (X0104:80-87): each
    rank's k-order routed sum, rounded to bf16, times routed_scale, plus its
    shared partial, bit-exact."""
    world, e, k, h = 4, 32, 4, 256
    from dw_tpu_b200 import _lib as L
    t = [24, 3, 17, 0]
    hid, ids, w = _inputs(world, t, e, k, h, seed=41, dist="zipf")
    ctxs = ep.create_local_contexts(world, max_tokens=24, hidden=h, topk=k, num_experts=e)
    try:
        ep.emulated_dispatch(ctxs, [np_to_bf16(x) for x in hid],
                             [torch.from_numpy(i).cuda() for i in ids])
        ref = O.ep_dispatch(hid, ids, e)
        ys = [O.round_bf16(np.random.default_rng(r).standard_normal(
            (ctxs[r].capacity, h)).astype(np.float32)) for r in range(world)]
        shs = [np.random.default_rng(50 + r).standard_normal((t[r], h)).astype(np.float32)
               for r in range(world)]
        for c, y in zip(ctxs, ys):
            c.combine(np_to_bf16(y), torch.zeros((c.num_tokens, k), device="cuda"),
                      phases=L.EP_PUSH)
        outs = [c.combine(np_to_bf16(y), torch.from_numpy(ww).cuda(), phases=L.EP_REDUCE,
                          shared=torch.from_numpy(sh).cuda(), routed_scale=1.5)
                for c, y, ww, sh in zip(ctxs, ys, w, shs)]
        torch.cuda.synchronize()
        L.raise_on_device_error()
        routed = O.ep_combine_korder([y[:int(g[1].sum())] for y, g in zip(ys, ref)],
                                     [g[2] for g in ref], w, out_dtype="bf16")
        for r in range(world):
            want = O.round_bf16((np.asarray(routed[r], np.float32) * np.float32(1.5)
                                 ).astype(np.float32) + shs[r])
            assert np.array_equal(bf16_to_np(outs[r]), want), r
    finally:
        for c in ctxs:
            c.close()


@pytest.mark.parametrize("world,t,k,ydt", [(4, [24, 3, 17, 0], 8, "bf16"),
                                           (8, [9, 16, 1, 30, 5, 12, 0, 7], 6, "f32")])
def test_ep_rank_order_combine_bit_exact(ep, world, t, k, ydt):
    """The reference GMM_EP numerics as a combine mode: each rank's masked f32
    partial over the k slots of its experts, summed over ranks in rank order
    (X0107:15-29, KO:181-184), bit-exact against oracle.ep_combine_rankorder."""
    from dw_tpu_b200 import _lib as L
    e, h = 32, 256
    hid, ids, w = _inputs(world, t, e, k, h, seed=81 + world, dist="zipf")
    ctxs = ep.create_local_contexts(world, max_tokens=max(t), hidden=h, topk=k, num_experts=e)
    try:
        ep.emulated_dispatch(ctxs, [np_to_bf16(x) for x in hid],
                             [torch.from_numpy(i).cuda() for i in ids])
        ref = O.ep_dispatch(hid, ids, e)
        ys = []
        for r in range(world):
            n = int(ref[r][1].sum())
            y = np.random.default_rng(90 + r).standard_normal((max(n, 1), h)).astype(np.float32)
            ys.append(O.round_bf16(y) if ydt == "bf16" else y)
        yt = [np_to_bf16(y) if ydt == "bf16" else torch.from_numpy(y).cuda() for y in ys]
        for c, y in zip(ctxs, yt):
            c.combine(y, torch.zeros((c.num_tokens, k), device="cuda"), phases=L.EP_PUSH)
        outs = [c.combine(y, torch.from_numpy(ww).cuda(), phases=L.EP_REDUCE, rank_order=True)
                for c, y, ww in zip(ctxs, yt, w)]
        torch.cuda.synchronize()
        L.raise_on_device_error()
        want = O.ep_combine_rankorder([y[:int(g[1].sum())] for y, g in zip(ys, ref)],
                                      [g[2] for g in ref], w, e, ids)
        for r in range(world):
            assert np.array_equal(bf16_to_np(outs[r]), want[r]), r
    finally:
        for c in ctxs:
            c.close()


def test_ep_invalid_ids_reported_and_dropped(ep):
    world, e, k, h = 2, 16, 2, 64
    ctxs = ep.create_local_contexts(world, max_tokens=8, hidden=h, topk=k, num_experts=e)
    from dw_tpu_b200 import _lib as L
    try:
        hid, ids, w = _inputs(world, 8, e, k, h, seed=5)
        ids[0][3, 1] = 99   # out of range: dropped, reported
        ep.emulated_dispatch(ctxs, [np_to_bf16(x) for x in hid],
                             [torch.from_numpy(i).cuda() for i in ids])
        assert L.device_status() & L.DEV_BAD_INDEX
        gs = [c.recv_group_sizes.cpu().numpy() for c in ctxs]
        assert sum(int(g.sum()) for g in gs) == 2 * 8 * k - 1
    finally:
        for c in ctxs:
            c.close()


def test_ep_rejects_bad_arguments(ep):
    from dw_tpu_b200 import _lib as L
    with pytest.raises(ValueError):
        ep.EPContext(0, 3, max_tokens=4, hidden=64, topk=2, num_experts=16)  # 16 % 3
    with pytest.raises(ValueError):
        ep.EPContext(0, 2, max_tokens=4, hidden=60, topk=2, num_experts=16)  # h % 8
    ctxs = ep.create_local_contexts(2, max_tokens=4, hidden=64, topk=2, num_experts=16)
    try:
        x = torch.zeros((5, 64), dtype=torch.bfloat16, device="cuda")
        i = torch.zeros((5, 2), dtype=torch.int32, device="cuda")
        with pytest.raises(ValueError):
            ctxs[0].dispatch(x, i)  # 5 tokens > max_tokens
        assert L.OK == 0
    finally:
        for c in ctxs:
            c.close()


@pytest.mark.parametrize("layout,t", [("b200", 24), ("b200", 3), ("e2m1", 10)])
def test_ep_layer_matches_single_device_layer(ep, layout, t):
    """The EP layer of 4 emulated ranks gives every rank the output of the
    single-device layer (all experts) on that rank's tokens, within the GEMM
    tolerance (the grouped matmuls see the rows in another order)."""
    import dw_tpu_b200 as dw
    from dw_tpu_b200 import synthetic
    from tests.gpu_util import gemm_rel_tol, rel_fro
    world, e, h, i, k = 4, 16, 512, 256, 4
    w = synthetic.moe_weights(e, h, i, seed=4, device="cuda")
    for name in ("s13", "s2"):
        setattr(w, name, synthetic.random_e8m0(getattr(w, name).shape, 9, "cuda", lo=118,
                                               hi=121))
    if layout == "b200":
        w = w.to_b200()
    le = e // world
    ctxs = ep.create_local_contexts(world, max_tokens=t, hidden=h, topk=k, num_experts=e)
    try:
        layers = []
        for r in range(world):
            lw = dw.FP4MoEWeights(w.w13[r * le:(r + 1) * le], w.s13[r * le:(r + 1) * le],
                                  w.w2[r * le:(r + 1) * le], w.s2[r * le:(r + 1) * le],
                                  w.layout)
            layers.append(ep.EPMoELayer(lw, ctxs[r], k))
        xs, lgs = [], []
        for r in range(world):
            x, router = synthetic.layer_inputs(t, h, e, seed=20 + r)
            xs.append(x.cuda())
            lgs.append((x.float() @ router.float()).to(torch.bfloat16).cuda())
        outs = ep.EPMoELayer.forward_emulated(layers, xs, lgs)
        torch.cuda.synchronize()
        from dw_tpu_b200 import _lib as L
        L.raise_on_device_error()
        single = dw.MoELayer(w, k, t)
        for r in range(world):
            ref = single(xs[r], lgs[r])
            torch.cuda.synchronize()
            rf = rel_fro(bf16_to_np(outs[r]), bf16_to_np(ref))
            assert rf < gemm_rel_tol(i), (r, rf)
    finally:
        for c in ctxs:
            c.close()


def test_ep_layer_rank_order_combine(ep):
    """EPMoELayer(rank_order=True) sums each token's expert outputs in the
    reference GMM_EP order: its output has the bits of
    oracle.ep_combine_rankorder on the layer's own expert outputs, routing and
    weights, and stays within the GEMM tolerance of the k-order layer."""
    import dw_tpu_b200 as dw
    from dw_tpu_b200 import _lib as L
    from dw_tpu_b200 import synthetic
    from tests.gpu_util import gemm_rel_tol, rel_fro
    world, e, h, i, k, t = 4, 16, 512, 256, 4, 24
    w = synthetic.moe_weights(e, h, i, seed=41, device="cuda")
    for name in ("s13", "s2"):
        setattr(w, name, synthetic.random_e8m0(getattr(w, name).shape, 42, "cuda", lo=118,
                                               hi=121))
    w = w.to_b200()
    le = e // world
    ctx_r = ep.create_local_contexts(world, max_tokens=t, hidden=h, topk=k, num_experts=e)
    ctx_k = ep.create_local_contexts(world, max_tokens=t, hidden=h, topk=k, num_experts=e)
    try:
        def shard(r):
            return dw.FP4MoEWeights(w.w13[r * le:(r + 1) * le], w.s13[r * le:(r + 1) * le],
                                    w.w2[r * le:(r + 1) * le], w.s2[r * le:(r + 1) * le], "b200")
        lro = [ep.EPMoELayer(shard(r), ctx_r[r], k, rank_order=True) for r in range(world)]
        lko = [ep.EPMoELayer(shard(r), ctx_k[r], k) for r in range(world)]
        xs, lgs = [], []
        for r in range(world):
            x, router = synthetic.layer_inputs(t, h, e, seed=60 + r)
            xs.append(x.cuda())
            lgs.append((x.float() @ router.float()).to(torch.bfloat16).cuda())
        a = ep.EPMoELayer.forward_emulated(lro, xs, lgs)
        b = ep.EPMoELayer.forward_emulated(lko, xs, lgs)
        torch.cuda.synchronize()
        L.raise_on_device_error()
        ids = [ly.ids[:t].cpu().numpy() for ly in lro]
        wts = [ly.w16[:t].float().cpu().numpy() for ly in lro]
        ref = O.ep_dispatch([bf16_to_np(x.cpu()) for x in xs], ids, e)
        ys = [bf16_to_np(ly.y[:int(g[1].sum())].cpu()) for ly, g in zip(lro, ref)]
        want = O.ep_combine_rankorder(ys, [g[2] for g in ref], wts, e, ids)
        for r in range(world):
            assert np.array_equal(bf16_to_np(a[r]), want[r]), r
            assert rel_fro(bf16_to_np(a[r]), bf16_to_np(b[r])) < gemm_rel_tol(i), r
        with pytest.raises(ValueError):
            ep.EPMoELayer(shard(0), ctx_r[0], k, rank_order=True, overlap=True)
    finally:
        for c in ctx_r + ctx_k:
            c.close()


def test_ep_layer_full_size_matches_single_device(ep):
    """The cfg1 architecture (H=4096, I=2048, 256 FP4 experts, top-8 sigmoid)
    as an EP layer of 8 emulated ranks with 32 tokens each: every rank's output
    matches the single-device layer over all 256 experts on its tokens, and the
    plain-PyTorch fp32 reference."""
    import dw_tpu_b200 as dw
    from dw_tpu_b200 import _lib as L
    from dw_tpu_b200 import synthetic
    from tests.gpu_util import assert_layer_close, torch_layer_reference
    world, t, e, h, i, k = 8, 32, 256, 4096, 2048, 8
    raw = synthetic.moe_weights(e, h, i, seed=7, device="cuda")
    w = raw.to_b200()
    le = e // world
    ctxs = ep.create_local_contexts(world, max_tokens=t, hidden=h, topk=k, num_experts=e)
    try:
        layers = [ep.EPMoELayer(dw.FP4MoEWeights(w.w13[r * le:(r + 1) * le],
                                                 w.s13[r * le:(r + 1) * le],
                                                 w.w2[r * le:(r + 1) * le],
                                                 w.s2[r * le:(r + 1) * le], w.layout),
                                ctxs[r], k) for r in range(world)]
        xs, lgs = [], []
        for r in range(world):
            x, router = synthetic.layer_inputs(t, h, e, seed=70 + r)
            xs.append(x.cuda())
            lgs.append((x.float() @ router.float()).to(torch.bfloat16).cuda())
        outs = ep.EPMoELayer.forward_emulated(layers, xs, lgs)
        torch.cuda.synchronize()
        L.raise_on_device_error()
        single = dw.MoELayer(w, k, t)
        for r in range(world):
            ref = single(xs[r], lgs[r])
            torch.cuda.synchronize()
            assert_layer_close(outs[r], ref, i, f"rank {r} vs single device")
            ref32 = torch_layer_reference(xs[r], single.ids[:t], single.w16[:t], raw.w13,
                                          raw.s13, raw.w2, raw.s2)
            assert_layer_close(outs[r], ref32, i, f"rank {r} vs fp32 reference")
    finally:
        for c in ctxs:
            c.close()


@pytest.mark.parametrize("f32_reduce,t,variant", [(False, 128, 9), (True, 128, 9),
                                                  (False, 96, 7), (False, 32, 1), (False, 16, 5),
                                                  (True, 8, 4), (False, 2, 3)])
def test_ep_overlapped_layer_matches_serial_bitwise(ep, f32_reduce, t, variant):
    """The overlapped exchange (rows gated per expert into gmm1, gmm2 pushing
    its rows to the token owners, local combine) gives the serial EP layer's
    bits, three steps in a row, on 4 emulated ranks with prefill-sized groups
    (~256 rows per expert: the CTA-pair kernel with 512-row tiles; ~192: the
    CTA-pair kernel; ~64: the one-CTA kernel) and decode-sized ones (~32, 16
    and 4 rows: the mma.sync decode kernel with 32, 16 and 8-row tiles)."""
    import dw_tpu_b200 as dw
    from dw_tpu_b200 import _lib as L
    from dw_tpu_b200 import synthetic
    world, e, h, i, k = 4, 16, 512, 256, 8
    w = synthetic.moe_weights(e, h, i, seed=17, device="cuda")
    for name in ("s13", "s2"):
        setattr(w, name, synthetic.random_e8m0(getattr(w, name).shape, 18, "cuda", lo=118,
                                               hi=121))
    w = w.to_b200()
    le = e // world
    ctx_s = ep.create_local_contexts(world, max_tokens=t, hidden=h, topk=k, num_experts=e)
    ctx_o = ep.create_local_contexts(world, max_tokens=t, hidden=h, topk=k, num_experts=e)
    try:
        def shard(r):
            return dw.FP4MoEWeights(w.w13[r * le:(r + 1) * le], w.s13[r * le:(r + 1) * le],
                                    w.w2[r * le:(r + 1) * le], w.s2[r * le:(r + 1) * le], "b200")
        serial = [ep.EPMoELayer(shard(r), ctx_s[r], k, f32_reduce=f32_reduce,
                                gemm_variant=variant) for r in range(world)]
        over = [ep.EPMoELayer(shard(r), ctx_o[r], k, f32_reduce=f32_reduce, overlap=True)
                for r in range(world)]
        assert all(ly.variant == variant for ly in serial + over)
        for step in range(3):
            xs, lgs = [], []
            for r in range(world):
                x, router = synthetic.layer_inputs(t, h, e, seed=200 + 10 * step + r)
                xs.append(x.cuda())
                lgs.append((x.float() @ router.float()).to(torch.bfloat16).cuda())
            a = ep.EPMoELayer.forward_emulated(serial, xs, lgs)
            b = ep.EPMoELayer.forward_emulated(over, xs, lgs)
            torch.cuda.synchronize()
            L.raise_on_device_error()
            for r in range(world):
                assert torch.equal(a[r].view(torch.int16), b[r].view(torch.int16)), (step, r)
    finally:
        for c in ctx_s + ctx_o:
            c.close()
