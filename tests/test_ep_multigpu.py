"""Expert-parallel exchange across real GPUs: one process per GPU over NCCL
plumbing, peer buffers mapped with CUDA IPC, dispatch/combine bit-exact
against the oracle and the EP layer against the single-device layer. Skipped
with fewer than 2 GPUs."""

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
        dist.barrier()
        ctx.close()
        ctx2.close()
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
