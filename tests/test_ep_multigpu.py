"""Expert-parallel exchange across real GPUs: one process per GPU over NCCL
plumbing, peer buffers mapped with CUDA IPC, dispatch/combine bit-exact
against the oracle, the EP layer against the single-device layer, the
one-shot exchange against the NCCL all_to_all_single path at cfg2's size,
and the overlapped layer against the serial one. Skipped with fewer than 2
GPUs."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(world, t, e, k, h, seed):
    from oracle import moe_oracle as O
    from dw_tpu_b200 import synthetic
    rng = np.random.default_rng(seed)
    hid, ids, w = [], [], []
    for r in range(world):
        hid.append(O.round_bf16(rng.standard_normal((t[r], h)).astype(np.float32)))
        i, ww = synthetic.route_ids(t[r], e, k, seed=seed * 31 + r, dist="zipf")
        ids.append(i)
        w.append(ww)
    return hid, ids, w


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import torch.distributed as dist
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    msgs = []
    try:
        from oracle import moe_oracle as O
        from tests.gpu_util import bf16_to_np, np_to_bf16
        import dw_tpu_b200 as dw
        from dw_tpu_b200 import _lib as L
        from dw_tpu_b200 import ep, synthetic
        e, k, h = 64, 8, 1024
        t = [40, 3, 17, 64, 1, 29, 8, 50][:world]
        ctx = ep.create_context(max_tokens=64, hidden=h, topk=k, num_experts=e)
        for step in range(3):
            hid, ids, w = _inputs(world, t[step % world:] + t[:step % world], e, k, h, step)
            recv, gs = ctx.dispatch(np_to_bf16(hid[rank]), torch.from_numpy(ids[rank]).cuda())
            ys = [O.round_bf16(np.random.default_rng(100 * step + r).standard_normal(
                (ctx.capacity, h)).astype(np.float32)) for r in range(world)]
            out = ctx.combine(np_to_bf16(ys[rank]), torch.from_numpy(w[rank]).cuda())
            torch.cuda.synchronize()
            bits = L.device_status()
            ref = O.ep_dispatch(hid, ids, e)
            n = int(ref[rank][1].sum())
            ok_gs = np.array_equal(gs.cpu().numpy(), ref[rank][1])
            ok_rows = np.array_equal(bf16_to_np(recv[:n]), ref[rank][0])
            want = O.ep_combine_korder([y[:int(g[1].sum())] for y, g in zip(ys, ref)],
                                       [g[2] for g in ref], w)[rank]
            ok_out = np.array_equal(bf16_to_np(out), want)
            if not (ok_gs and ok_rows and ok_out and bits == 0):
                msgs.append(f"step {step}: gs={ok_gs} rows={ok_rows} out={ok_out} "
                            f"status={bits:#x}")
        # EP layer vs the single-device layer on this rank's tokens.
        e2, hh, ii, kk, tt = 16, 512, 256, 4, 12
        wts = synthetic.moe_weights(e2, hh, ii, seed=4, device="cuda")
        for name in ("s13", "s2"):
            setattr(wts, name, synthetic.random_e8m0(getattr(wts, name).shape, 9, "cuda",
                                                     lo=118, hi=121))
        wts = wts.to_b200()
        le = e2 // world
        sl = slice(rank * le, (rank + 1) * le)
        lw = dw.FP4MoEWeights(wts.w13[sl], wts.s13[sl], wts.w2[sl], wts.s2[sl], "b200")
        ctx2 = ep.create_context(max_tokens=tt, hidden=hh, topk=kk, num_experts=e2)
        layer = ep.EPMoELayer(lw, ctx2, kk)
        x, router = synthetic.layer_inputs(tt, hh, e2, seed=20 + rank)
        x = x.cuda()
        lg = (x.float() @ router.cuda().float()).to(torch.bfloat16)
        out = layer(x, lg)
        ref = dw.MoELayer(wts, kk, tt)(x, lg)
        torch.cuda.synchronize()
        from tests.gpu_util import gemm_rel_tol, rel_fro
        rf = rel_fro(bf16_to_np(out), bf16_to_np(ref))
        if not rf < gemm_rel_tol(ii) or L.device_status():
            msgs.append(f"layer rel_fro {rf:.3e}")
        # cfg2 size (512 tokens per rank, H=4096, top-8 over 256 experts):
        # the one-shot exchange and the NCCL all_to_all_single path give the
        # same receive buffer and combine output, bit for bit.
        ctx3 = ep.create_context(max_tokens=512, hidden=4096, topk=8, num_experts=256)
        nccl = ep.NcclExchange(256, 4096, 8)
        ids3, w3 = synthetic.route_ids(512, 256, 8, seed=70 + rank, dist="zipf")
        ids3 = torch.from_numpy(ids3).cuda()
        w3 = torch.from_numpy(w3).cuda()
        x3 = torch.randn((512, 4096), generator=torch.Generator().manual_seed(rank)).to(
            torch.bfloat16).cuda()
        recv3, gs3 = ctx3.dispatch(x3, ids3)
        n3 = int(gs3.sum())
        y3 = ctx3.output(torch.bfloat16)
        y3[:n3].copy_(recv3[:n3])
        o1 = ctx3.combine(y3, w3)
        r2, g2 = nccl.dispatch(x3, ids3)
        o2 = nccl.combine(r2, w3)
        torch.cuda.synchronize()
        if not (torch.equal(gs3, g2) and torch.equal(recv3[:n3].view(torch.int16),
                                                     r2.view(torch.int16))
                and torch.equal(o1.view(torch.int16), o2.view(torch.int16))):
            msgs.append("one-shot and NCCL all_to_all exchanges differ")
        # The overlapped exchange (gated gmm1, gmm2 pushing to the owners)
        # against the serial EP layer, prefill-sized groups, two steps.
        e4, h4, i4, k4, t4 = 8 * world, 512, 256, 8, 128
        w4 = synthetic.moe_weights(e4, h4, i4, seed=5, device="cuda")
        for name in ("s13", "s2"):
            setattr(w4, name, synthetic.random_e8m0(getattr(w4, name).shape, 6, "cuda",
                                                    lo=118, hi=121))
        w4 = w4.to_b200()
        sl4 = slice(rank * 8, (rank + 1) * 8)
        lw4 = dw.FP4MoEWeights(w4.w13[sl4], w4.s13[sl4], w4.w2[sl4], w4.s2[sl4], "b200")
        ctx4 = ep.create_context(max_tokens=t4, hidden=h4, topk=k4, num_experts=e4)
        ctx5 = ep.create_context(max_tokens=t4, hidden=h4, topk=k4, num_experts=e4)
        ser = ep.EPMoELayer(lw4, ctx4, k4, gemm_variant=7)
        ovl = ep.EPMoELayer(lw4, ctx5, k4, overlap=True)
        for step in range(2):
            x4, r4 = synthetic.layer_inputs(t4, h4, e4, seed=90 + 10 * step + rank)
            x4 = x4.cuda()
            lg4 = (x4.float() @ r4.cuda().float()).to(torch.bfloat16)
            a4 = ser(x4, lg4)
            b4 = ovl(x4, lg4)
            torch.cuda.synchronize()
            if not torch.equal(a4.view(torch.int16), b4.view(torch.int16)):
                msgs.append(f"overlapped layer differs from the serial one at step {step}")
        if L.device_status():
            msgs.append("device status set")
        dist.barrier()
        for c in (ctx, ctx2, ctx3, ctx4, ctx5):
            c.close()
        q.put((rank, msgs))
    except Exception as ex:  # report, then leave the group
        q.put((rank, msgs + [f"{type(ex).__name__}: {ex}"]))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 or more GPUs")
def test_ep_exchange_across_gpus():
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        assert res[r] == [], (r, res[r])
    for p in procs:
        assert p.exitcode == 0
