"""Host side of the expert-parallel exchange, no GPU: the receive-placement
arithmetic the dispatch kernel uses (restated here in NumPy) against the
oracle's EP order, and the multi-rank plumbing (IPC handle exchange, the NCCL
comparison collectives) on world-size-2 gloo process groups."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe_oracle as O


def _placement(ids_per_rank, num_experts):
    """The dispatch kernel's arithmetic: a pair (rank r, token t, slot k) with
    expert e lands on owner e // LE at row
        sum over the owner's earlier experts of all ranks' counts
      + sum over ranks < r of counts[., e]
      + the pair's stable rank among r's own pairs of expert e.
    Returns per owner a list of (row, r, t, k)."""
    world = len(ids_per_rank)
    le = num_experts // world
    counts = np.stack([np.bincount(np.asarray(i).reshape(-1), minlength=num_experts)
                       for i in ids_per_rank])                     # [world, E]
    colsum = counts.sum(0)
    out = [[] for _ in range(world)]
    for r, ids in enumerate(ids_per_rank):
        flat = np.asarray(ids).reshape(-1)
        k = np.asarray(ids).shape[-1] if np.asarray(ids).ndim == 2 else 1
        seen = np.zeros(num_experts, np.int64)
        for j, e in enumerate(flat):
            owner = e // le
            base = colsum[owner * le:e].sum()
            before = counts[:r, e].sum()
            row = base + before + seen[e]
            seen[e] += 1
            out[owner].append((int(row), r, j // k, j % k))
    return out


@pytest.mark.parametrize("world,t,e,k,dist_", [
    (2, 16, 32, 4, "uniform"), (4, 24, 64, 8, "zipf"), (8, [3, 0, 9, 1, 12, 5, 0, 7], 64, 6,
                                                         "zipf"),
])
def test_placement_formula_matches_oracle_ep_order(world, t, e, k, dist_):
    from dw_tpu_b200 import synthetic
    ids = []
    for r in range(world):
        tr = t[r] if isinstance(t, list) else t
        ids.append(synthetic.route_ids(tr, e, k, seed=r + 7, dist=dist_)[0] if tr
                   else np.zeros((0, k), np.int32))
    hid = [np.zeros((i.shape[0], 8), np.float32) for i in ids]
    ref = O.ep_dispatch(hid, ids, e)
    got = _placement(ids, e)
    for owner in range(world):
        rows = sorted(got[owner])
        assert [r[0] for r in rows] == list(range(len(rows)))      # dense, no collisions
        src = np.array([r[1:] for r in rows], np.int32).reshape(-1, 3)
        assert np.array_equal(src, ref[owner][2]), owner


def test_gemm_variant_choice():
    from dw_tpu_b200.ep import gemm_variant
    assert gemm_variant("e2m1", 4) == 0
    assert gemm_variant("b200", 2) == 3
    assert gemm_variant("b200", 8) == 4
    assert gemm_variant("b200", 16) == 4
    assert gemm_variant("b200", 32) == 10
    assert gemm_variant("b200", 64) == 1
    assert gemm_variant("b200", 96) == 7
    assert gemm_variant("b200", 128) == 7
    assert gemm_variant("b200", 256) == 9
    from dw_tpu_b200.ep import overlap_variant
    assert [overlap_variant(r) for r in (4, 16, 32, 64, 128, 256)] == [3, 4, 5, 1, 7, 9]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from dw_tpu_b200 import _lib as L
        from dw_tpu_b200 import ep
        handle = bytes([rank + 1]) * L.EP_HANDLE_BYTES
        hs = ep.exchange_handles(handle, None)
        ok_handles = hs == [bytes([r + 1]) * L.EP_HANDLE_BYTES for r in range(world)]
        try:
            ep.exchange_handles(b"short", None)
            bad_rejected = False
        except ValueError:
            bad_rejected = True
        rng = np.random.default_rng(rank)
        x = torch.from_numpy(O.round_bf16(rng.standard_normal((3, 16)).astype(np.float32)))
        xb = x.to(torch.bfloat16)
        g = ep.all_gather_local(xb)
        parts = [torch.from_numpy(O.round_bf16(np.random.default_rng(r).standard_normal(
            (3, 16)).astype(np.float32))).to(torch.bfloat16) for r in range(world)]
        ok_ag = torch.equal(g.view(torch.int16), torch.cat(parts).view(torch.int16))
        p = torch.from_numpy(np.random.default_rng(10 + rank).standard_normal(
            (world * 2, 16)).astype(np.float32))
        rs = ep.reduce_scatter_local(p, None, torch.float32)
        allp = [np.random.default_rng(10 + r).standard_normal((world * 2, 16)).astype(np.float32)
                for r in range(world)]
        want = O.reduce_scatter_rank_order(allp, world, out_dtype="f32")[rank]
        ok_rs = np.array_equal(rs.numpy(), want)   # two ranks: a + b is order-free
        q.put((rank, ok_handles, bad_rejected, ok_ag, ok_rs))
    finally:
        dist.destroy_process_group()


def test_gloo_world2_exchange_and_comparison_collectives():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok_h, bad, ok_ag, ok_rs in res:
        assert ok_h and bad and ok_ag and ok_rs, (rank, ok_h, bad, ok_ag, ok_rs)


def _a2a_worker(rank, world, port, q, t_per_rank, e, k, h, dist_):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from dw_tpu_b200 import ep, synthetic
        hid, ids, w = [], [], []
        for r in range(world):
            rng = np.random.default_rng(100 + r)
            hid.append(O.round_bf16(rng.standard_normal((t_per_rank[r], h)).astype(np.float32)))
            i, ww = synthetic.route_ids(t_per_rank[r], e, k, seed=200 + r, dist=dist_)
            ids.append(i)
            w.append(ww)
        xch = ep.NcclExchange(e, h, k)
        recv, gs = xch.dispatch(torch.from_numpy(hid[rank]), torch.from_numpy(ids[rank]))
        ref = O.ep_dispatch(hid, ids, e)
        ok_gs = np.array_equal(gs.numpy(), ref[rank][1])
        ok_rows = np.array_equal(recv.numpy(), ref[rank][0])
        # expert outputs: the received rows scaled by 1 + rank, returned to the owners
        y = recv * (1.0 + rank)
        rows = xch.return_rows(y).numpy()
        want = np.zeros_like(rows)
        for owner in range(world):
            src = ref[owner][2]
            mine = src[:, 0] == rank
            want[src[mine, 1] * k + src[mine, 2]] = ref[owner][0][mine] * (1.0 + owner)
        ok_back = np.array_equal(rows, want)
        q.put((rank, ok_gs, ok_rows, ok_back))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,t,dist_", [(2, [16, 16], "uniform"), (4, [9, 0, 24, 5], "zipf")])
def test_gloo_nccl_exchange_path_receive_order(world, t, dist_):
    """The all_to_all_single comparison path (NcclExchange) delivers the
    oracle's EP receive order and group sizes, and returns each pair's expert
    output to its owner, on gloo process groups."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_a2a_worker, args=(r, world, port, q, t, 32, 4, 16, dist_))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok_gs, ok_rows, ok_back in res:
        assert ok_gs and ok_rows and ok_back, (rank, ok_gs, ok_rows, ok_back)
