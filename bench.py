"""Benchmark: FP4 MoE layer tokens/s (dispatch + FP4 GMM + combine) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --case layer|gemm [...]      (small single-GPU cases for ncu)

One step = one MoE layer forward over one batch of synthetic tokens:
route (top-8 sigmoid) -> permute -> gather -> gmm1 (SwiGLU) -> gmm2 ->
combine. At N=1 the workload is BASELINE config 1 (T=64 tokens, H=4096,
I=2048, E=256 FP4 experts with E8M0 scales). N>1 runs the expert-parallel
layer (weak scaling): every rank routes its own 64 tokens over all 256
experts, holds experts [r*E/N, (r+1)*E/N), and exchanges rows with the
one-shot NVLink dispatch/combine. The weights (3.3 GB, or 3.3/N GB per rank)
exceed L2, so every step streams them from HBM.

Printed (rank 0, one JSON line):
  value         device-timed tokens/s with inputs resident (max over ranks)
  e2e           the same layer through the public API with pinned host
                buffers, host<->device copies inside the timed region
  roofline      the decode GEMM (dw_moe gmm_fp4, CUDA events on its stream)
  parity        all output rows against a plain-PyTorch fp32 restatement of
                the reference numerics; at N>1 also against the single-device
                layer over all 256 experts on the same rank's tokens
  cpu_baseline  the CPU restatement of the layer on the host cores (N=1)
  clocks, gpu_launches
and, unless --no-extras:
  N=1  prefill (cfg3-rank grouped matmuls vs the tensor roofline) and
       prefill_layer (cfg3 at n=1: T=1024)
  N>1  link (measured NCCL send/recv peer bandwidth), exchange_sweep
       (cfg2: one-shot vs NCCL all_to_all_single, bit-compared),
       prefill_layer (cfg3: T=1024 per rank), decode_sweep (cfg4, N=8)

``--impl reference`` times the reference's layer arithmetic on the host
cores instead (the reference's JAX path cannot run here; its CPU restatement
under oracle/ stands in) on the same config and prints the same metric; it
imports nothing that maps this repository's CUDA library.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MoE layer tokens/s (dispatch+FP4 GMM+combine)"
UNIT = "tokens/s"
T_RANK, H, I, E, TOPK = 64, 4096, 2048, 256, 8
WORKLOAD = "cfg1 decode MoE layer: T=64/rank, H=4096, I=2048, E=256 FP4 experts, top-8 sigmoid"
# Per-launch DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum, mean of
# the gmm1 and gmm2 launches) of the decode GEMM on the N=1 cfg1 layer of
# this bench (seed 0), from one ncu capture of `bench.py --case layer`.
GMM_TRAFFIC_PER_LAUNCH_N1 = 1504650000.0
# Parity tolerance of the layer output (relative Frobenius error against the
# fp32 restatement): the reference's GMM_EP error level, 4e-3 at K=4096,
# scaled by sqrt(K/4096) with K = I for the last projection.
PARITY_REL_TOL = 4e-3 * (I / 4096) ** 0.5
# A device-side sleep (cycles, ~10 ms at 1.9 GHz) before a loop of short
# launches, so that the launches queue up and CUDA events time the device.
PREROLL_CYCLES = 20_000_000
E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
               -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extras", action="store_true",
                   help="skip the prefill / exchange / sweep measurements")
    p.add_argument("--case", default="bench", choices=["bench", "layer", "gemm"],
                   help="layer / gemm: a small single-GPU case for ncu captures")
    p.add_argument("--experts", type=int, default=E)
    p.add_argument("--tokens", type=int, default=T_RANK)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--variant", type=int, default=0)
    p.add_argument("--groups", choices=["uniform", "multinomial", "zipf"], default="uniform")
    p.add_argument("--overlap", action="store_true",
                   help="N > 1: the cfg1 step with the overlapped exchange (gated gmm1, "
                        "pushing gmm2)")
    p.add_argument("--decode-sweep", action="store_true",
                   help="run the cfg4 decode sweep at any N > 1 (by default at N = 8 only)")
    return p.parse_args()


# ----------------------------------------------------------------------------
# clocks
# ----------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.idx)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        return None


# ----------------------------------------------------------------------------
# CPU arm: the reference's layer arithmetic on the host cores
# ----------------------------------------------------------------------------

def cpu_inputs(tokens: int, seed: int):
    """The cfg1 inputs as host arrays, drawn with the GPU arm's distributions
    (tokens and router from the same generator; FP4 bytes uniform over all
    256 values, E8M0 codes uniform in 123..129, from NumPy's generator):
    hidden and logits (bf16 values as f32), packed e2m1 weights, scales."""
    import torch
    from dw_tpu_b200 import synthetic  # no op call: the CUDA library stays unmapped
    rng = np.random.default_rng(seed)
    lo, hi = synthetic.E8M0_LO, synthetic.E8M0_HI
    w13 = rng.integers(0, 256, (E, H, I), dtype=np.uint8)
    s13 = rng.integers(lo, hi + 1, (E, H // 32, 2 * I), dtype=np.uint8)
    w2 = rng.integers(0, 256, (E, I, H // 2), dtype=np.uint8)
    s2 = rng.integers(lo, hi + 1, (E, I // 32, H), dtype=np.uint8)
    x, router = synthetic.layer_inputs(tokens, H, E, seed=seed)
    logits = (x.float() @ router.float()).to(torch.bfloat16)
    return x.float().numpy(), logits.float().numpy(), w13, s13, w2, s2


def jax_probe() -> str:
    try:
        import jax  # noqa: F401
        return "importable (not used: the reference's JAX path needs tokamax and TPU patches)"
    except Exception as e:  # noqa: BLE001
        return f"absent ({type(e).__name__})"


def cpu_layer_runner(tokens: int, seed: int):
    """(run, threads, sample): run() does one full layer step on the host and
    returns its seconds."""
    from oracle import layer_cpu
    inputs = cpu_inputs(tokens, seed)
    pool, threads = layer_cpu.make_pool()

    def run():
        t0 = time.perf_counter()
        layer_cpu.layer_forward(*inputs, TOPK, pool=pool)
        return time.perf_counter() - t0

    sample = (f"the whole layer on all {tokens} tokens per step (routing, permute, gather, "
              f"table-decoded FP4 dequant and f32 BLAS GEMMs of every active expert, k-order "
              f"combine): the reference's arithmetic restated in NumPy (oracle/layer_cpu.py; "
              f"the reference's JAX path is unavailable)")
    return run, threads, sample, pool


def cpu_baseline(seed: int):
    """One bounded sample of the reference arm (one full layer step after one
    untimed warm-up), for the N=1 line."""
    run, threads, sample, pool = cpu_layer_runner(T_RANK, seed)
    with pool:
        run()
        secs = run()
    return {"value": round(T_RANK / secs, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": "one step: " + sample, "seconds_per_step": secs}


def run_reference(args, rank, world):
    """The reference arm: rank 0 times the CPU restatement of the layer on the
    whole job's tokens (64 per rank) with every host thread; other ranks exit."""
    if rank != 0:
        return
    tokens = T_RANK * world
    run, threads, sample, pool = cpu_layer_runner(tokens, args.seed)
    with pool:
        for _ in range(args.warmup):
            run()
        t0 = time.perf_counter()
        per = [run() for _ in range(args.steps)]
        total = time.perf_counter() - t0
    value = tokens * args.steps / total
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / args.steps * 1e3, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config_of(world),
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "step_seconds": {"min": round(min(per), 3), "max": round(max(per), 3)},
        "jax": jax_probe(),
    }), flush=True)


def config_of(world):
    return {"workload": WORKLOAD, "tokens_per_rank": T_RANK, "hidden": H, "intermediate": I,
            "experts": E, "top_k": TOPK, "global_batch": T_RANK * world,
            "parallelism": f"ep{world}" if world > 1 else "single",
            "l2": "inputs larger than L2 (3.3 GB of FP4 weights streamed per step)"}


# ----------------------------------------------------------------------------
# GPU helpers
# ----------------------------------------------------------------------------

def torch_dequant(codes, scales):
    """bf16(e2m1 value x 2^(c-127)) as f32 [k, n] from raw packed e2m1 [k, n/2]
    (element 2j in the low nibble) and E8M0 codes [k/32, n] (code 0 -> +0)."""
    import torch
    lut = torch.tensor(E2M1_VALUES, dtype=torch.float32, device=codes.device)
    c = codes.to(torch.int64)
    k, n2 = codes.shape
    v = torch.stack([lut[c & 0xF], lut[c >> 4]], dim=-1).reshape(k, 2 * n2)
    s = (scales.to(torch.int32) << 23).view(torch.float32)
    return (v * s.repeat_interleave(32, dim=0)).to(torch.bfloat16).float()


def torch_layer_reference(x, ids, w16, raw, expert_offset=0):
    """A plain-PyTorch fp32 restatement of the layer's reference numerics
    (E0901:84-95 dequant, f32 products and sums, bf16 gmm outputs, k-order
    f32 combine KC:44-54) on x's device, for the experts held in ``raw`` (raw
    e2m1 layout) starting at global expert ``expert_offset``."""
    import torch
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        t = x.shape[0]
        y = torch.zeros((t, TOPK, H), dtype=torch.float32, device=x.device)
        xf = x.float()
        for ex in torch.unique(ids).tolist():
            le = ex - expert_offset
            tok, slot = (ids == ex).nonzero(as_tuple=True)
            a = xf[tok] @ torch_dequant(raw.w13[le], raw.s13[le])
            g, u = a[:, :I], a[:, I:]
            hdn = (g * torch.sigmoid(g) * u).to(torch.bfloat16).float()
            y[tok, slot] = (hdn @ torch_dequant(raw.w2[le], raw.s2[le])).to(torch.bfloat16).float()
        acc = torch.zeros((t, H), dtype=torch.float32, device=x.device)
        wf = w16.float()
        for kk in range(TOPK):
            acc = acc + y[:, kk] * wf[:, kk:kk + 1]
        return acc.to(torch.bfloat16)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def compare(got, ref):
    """(relative Frobenius error, max-abs error in bf16 ulps of max|ref|)."""
    g = got.float()
    r = ref.float()
    den = float(r.norm())
    rel = float((g - r).norm()) / den if den else float(g.norm())
    amax = float(r.abs().max())
    ulp = 2.0 ** (np.floor(np.log2(amax)) - 7) if amax > 0 else 1.0
    return rel, float((g - r).abs().max()) / ulp


def events():
    import torch
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def max_over_ranks(vals, world, dev):
    import torch
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


class GmmTimer:
    """Records CUDA events around every dw_moe gmm_fp4 launch (on the current
    stream) while active, tagged gmm1 (SwiGLU) or gmm2; with `ctx`, also
    around the overlapped exchange's grouped matmuls (EPContext.gmm)."""

    def __init__(self, ctx=None):
        from dw_tpu_b200 import ops
        self.ops = ops
        self.orig = ops.gmm_fp4_out
        self.ctx = ctx
        self.ev = []

    def __enter__(self):
        import torch
        from dw_tpu_b200 import _lib as L

        def timed(*a, **kw):
            e0, e1 = events()
            s = torch.cuda.current_stream()
            e0.record(s)
            r = self.orig(*a, **kw)
            e1.record(s)
            self.ev.append((e0, e1, kw.get("act", L.ACT_NONE) != L.ACT_NONE))
            return r
        self.ops.gmm_fp4_out = timed
        if self.ctx is not None:
            orig_gmm = self.ctx.gmm

            def timed_ep(*a, **kw):
                e0, e1 = events()
                s = torch.cuda.current_stream()
                e0.record(s)
                r = orig_gmm(*a, **kw)
                e1.record(s)
                self.ev.append((e0, e1, kw.get("mode") == L.EP_GEMM_GATED))
                return r
            self.ctx.gmm = timed_ep
        return self

    def __exit__(self, *exc):
        self.ops.gmm_fp4_out = self.orig
        if self.ctx is not None:
            del self.ctx.gmm  # back to the class method

    def ms(self):
        g1 = [a.elapsed_time(b) for a, b, act in self.ev if act]
        g2 = [a.elapsed_time(b) for a, b, act in self.ev if not act]
        return g1, g2


def gemm_bytes(gs_np):
    """Algorithmic bytes of gmm1 and gmm2 for group sizes gs_np: FP4 codes and
    E8M0 scales of every active expert, lhs rows read and output rows written."""
    active = int((gs_np > 0).sum())
    rows = int(gs_np.sum())
    w13 = H * I + (H // 32) * 2 * I
    w2 = I * (H // 2) + (I // 32) * H
    return (active * w13 + rows * H * 2 + rows * I * 2,
            active * w2 + rows * I * 2 + rows * H * 2, active, rows)


# ----------------------------------------------------------------------------
# GPU arm: the cfg1 layer
# ----------------------------------------------------------------------------

def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import dw_tpu_b200 as dw
    from dw_tpu_b200 import _lib as L
    from dw_tpu_b200 import synthetic

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    le = E // world
    raw = synthetic.moe_weights(E, H, I, seed=args.seed, device=dev)  # all experts, raw e2m1
    if world > 1:
        sl = slice(rank * le, (rank + 1) * le)
        local = dw.FP4MoEWeights(raw.w13[sl], raw.s13[sl], raw.w2[sl], raw.s2[sl]).to_b200()
    else:
        local = raw.to_b200()  # load-time re-layout for the B200 decode (untimed)
    x_cpu, router = synthetic.layer_inputs(T_RANK, H, E, seed=args.seed + 100 * rank)
    x = x_cpu.to(dev)
    router = router.to(dev)
    logits = (x.float() @ router.float()).to(torch.bfloat16)
    ctx = None
    if world > 1:
        from dw_tpu_b200 import ep as ep_mod
        ctx = ep_mod.create_context(max_tokens=T_RANK, hidden=H, topk=TOPK, num_experts=E)
        layer = ep_mod.EPMoELayer(local, ctx, TOPK, overlap=args.overlap)
    else:
        layer = dw.MoELayer(local, TOPK, T_RANK)
    out = torch.empty((T_RANK, H), dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(3, args.warmup)):
        layer(x, logits, out=out)
    torch.cuda.synchronize(dev)
    L.raise_on_device_error()

    # Timed region: K steps; events around every gmm launch and exchange call.
    xchg = {"dispatch": [], "combine": []}
    if ctx is not None:
        orig_d, orig_c = ctx.dispatch, ctx.combine

        def timed(fn, tag):
            def run(*a, **kw):
                e0, e1 = events()
                e0.record(stream)
                r = fn(*a, **kw)
                e1.record(stream)
                xchg[tag].append((e0, e1))
                return r
            return run
        ctx.dispatch, ctx.combine = timed(orig_d, "dispatch"), timed(orig_c, "combine")
    start, end = events()
    with GmmTimer(ctx) as gt, ClockSampler(local_rank) as clk:
        barrier()
        torch.cuda.synchronize(dev)
        torch.cuda._sleep(PREROLL_CYCLES)  # the steps queue up: the events time the device
        start.record(stream)
        for _ in range(args.steps):
            layer(x, logits, out=out)
        end.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
    if ctx is not None:
        ctx.dispatch, ctx.combine = orig_d, orig_c
    ms = start.elapsed_time(end)
    g1, g2 = gt.ms()
    L.raise_on_device_error()

    # e2e through the public API with pinned host buffers: every step copies
    # its inputs host -> device and its output device -> host. The copies run
    # on a second stream, double-buffered, so step i's copies overlap the
    # compute of its neighbours (a serving loop's pipelining); the timed
    # region holds all of them.
    hx = x.cpu().pin_memory()
    hl = logits.cpu().pin_memory()
    hout = torch.empty((T_RANK, H), dtype=torch.bfloat16).pin_memory()
    dxs = [torch.empty_like(x) for _ in range(2)]
    dls = [torch.empty_like(logits) for _ in range(2)]
    outs = [torch.empty_like(out) for _ in range(2)]
    cs = torch.cuda.Stream(dev)
    copied = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]

    def pipelined(n):
        with torch.cuda.stream(cs):
            cs.wait_stream(stream)
            dxs[0].copy_(hx, non_blocking=True)
            dls[0].copy_(hl, non_blocking=True)
            copied[0].record(cs)
        for i in range(n):
            sl = i & 1
            stream.wait_event(copied[sl])
            layer(dxs[sl], dls[sl], out=outs[sl])
            computed[sl].record(stream)
            with torch.cuda.stream(cs):
                if i + 1 < n:  # the next step's inputs, once step i-1 is done with the slot
                    if i >= 1:
                        cs.wait_event(computed[1 - sl])
                    dxs[1 - sl].copy_(hx, non_blocking=True)
                    dls[1 - sl].copy_(hl, non_blocking=True)
                    copied[1 - sl].record(cs)
                cs.wait_event(computed[sl])
                hout.copy_(outs[sl], non_blocking=True)
        stream.wait_stream(cs)

    pipelined(3)
    torch.cuda.synchronize(dev)
    barrier()
    e0, e1 = events()
    e0.record(stream)
    pipelined(args.steps)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    L.raise_on_device_error()
    ms, e2e_ms = max_over_ranks([ms, e2e_ms], world, dev)

    # Roofline of the dominant kernel (gmm_fp4): algorithmic bytes per launch.
    gs = (ctx.recv_group_sizes if ctx is not None else layer.group_sizes).cpu().numpy()
    b1, b2, active, rows = gemm_bytes(gs)
    avg_ms = (sum(g1) + sum(g2)) / max(1, len(g1) + len(g2))
    per_launch = (b1 + b2) / 2
    achieved = per_launch / (avg_ms * 1e-3) / 1e9
    peaks = measured_peaks()
    peak = peaks["hbm_gbs"] if peaks else 6650.0
    m1, m2 = statistics.mean(g1), statistics.mean(g2)
    res = {
        "ms": ms, "e2e_ms": e2e_ms, "active": active,
        "roofline": {
            "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "traffic": GMM_TRAFFIC_PER_LAUNCH_N1 if world == 1 else None,
            "kernel": "dw_moe gmm_fp4 (gmm1+gmm2 average, rank 0)",
            "peak_source": "measured" if peaks else "fallback",
            "algorithmic_bytes_per_launch": per_launch,
            "gmm1_ms": round(m1, 4), "gmm2_ms": round(m2, 4),
            "gmm1_GBps": round(b1 / (m1 * 1e-3) / 1e9, 1),
            "gmm2_GBps": round(b2 / (m2 * 1e-3) / 1e9, 1),
            "gmm_share_of_step": round((sum(g1) + sum(g2)) / ms, 3),
        },
        "clocks": clk.summary(),
        "h2d": hx.numel() * 2 + hl.numel() * 2,
        "d2h": hout.numel() * 2,
        "launches_per_step": layer.kernels_per_forward,
    }
    if world > 1:
        # per-rank GEMM fraction of HBM (max and min over ranks)
        frac = achieved / peak
        lo_hi = max_over_ranks([frac, -frac], world, dev)
        res["roofline"]["frac_max_over_ranks"] = round(lo_hi[0], 4)
        res["roofline"]["frac_min_over_ranks"] = round(-lo_hi[1], 4)
        ids = layer.ids.cpu().numpy()
        owners = ids // le
        remote = int((owners != rank).sum())
        remote_dedup = sum(len(set(int(o) for o in row) - {rank}) for row in owners)
        recv_remote = rows - int((owners == rank).sum())
        d_ms = statistics.median(a.elapsed_time(b) for a, b in xchg["dispatch"])
        c_ms = statistics.median(a.elapsed_time(b) for a, b in xchg["combine"])
        d_ms, c_ms = max_over_ranks([d_ms, c_ms], world, dev)
        res["exchange"] = {
            "dispatch_ms": round(d_ms, 4), "combine_ms": round(c_ms, 4),
            "includes": "waiting for the slowest peer inside the layer step",
            "remote_pairs_sent": remote, "remote_token_rank_pairs_sent": remote_dedup,
            "remote_pairs_received": recv_remote,
            # each direction: rows stored to peers by the dispatch plus rows
            # the peers load back in their combine (and the mirror image in)
            "nvlink_bytes_each_way_per_step": (remote + recv_remote) * H * 2,
        }

    # Parity: every output row against the fp32 restatement (and, with EP,
    # against the single-device layer over all experts on the same tokens).
    layer(x, logits, out=out)
    torch.cuda.synchronize(dev)
    ids_now = layer.ids[:T_RANK].clone()
    w16_now = layer.w16[:T_RANK].clone()
    ref32 = torch_layer_reference(x, ids_now, w16_now, raw)
    rel, ulps = compare(out, ref32)
    vals = [rel, ulps]
    if world > 1:
        single = dw.MoELayer(raw.to_b200(), TOPK, T_RANK)
        ref_single = single(x, logits)
        torch.cuda.synchronize(dev)
        rel_s, ulps_s = compare(out, ref_single)
        vals += [rel_s, ulps_s, 0.0 if torch.equal(out.view(torch.int16),
                                                   ref_single.view(torch.int16)) else 1.0,
                 0.0 if torch.equal(ids_now, single.ids[:T_RANK]) else 1.0]
        del single
    L.raise_on_device_error()
    vals = max_over_ranks(vals, world, dev)
    res["parity"] = {
        "reference": "plain-PyTorch fp32 restatement of the reference numerics, all rows",
        "rel_fro": float(f"{vals[0]:.3e}"), "max_abs_bf16_ulps": round(vals[1], 2),
        "tol_rel_fro": round(PARITY_REL_TOL, 6), "pass": vals[0] <= PARITY_REL_TOL,
        "ranks": world,
    }
    if world > 1:
        res["parity"].update({
            "vs_single_device_rel_fro": float(f"{vals[2]:.3e}"),
            "vs_single_device_max_abs_bf16_ulps": round(vals[3], 2),
            "vs_single_device_bitwise": vals[4] == 0.0,
            "routing_ids_equal": vals[5] == 0.0,
        })
    torch.cuda.empty_cache()

    if not args.no_extras:
        if world == 1:
            res["prefill"] = prefill_gemm(local, dev, args.seed)
            res["prefill_layer"] = prefill_layer_single(local, dev, args.seed)
        else:
            res.update(ep_extras(args, local, dev, world, rank))
    if ctx is not None:
        ctx.close()
    return res


# ----------------------------------------------------------------------------
# Extras at N=1: the grouped matmuls at a cfg3 rank's shape, cfg3 at n=1
# ----------------------------------------------------------------------------

def prefill_gemm(weights, dev, seed, iters=10):
    """The grouped matmuls at one cfg3 rank's shape at n=8 (32 local experts,
    T=1024 tokens x top-8 = 8192 rows, 256 per expert on average): gmm1 with
    SwiGLU and gmm2 on the first 32 experts, with groups of exactly 256 rows
    and with one seeded multinomial draw (uniform routing). Median of `iters`
    launches (CUDA events) after 3 warm-ups; the weights (0.43 GB) exceed L2.
    TFLOP/s against the measured bf16 peak."""
    import torch
    import dw_tpu_b200 as dw
    from dw_tpu_b200 import ops
    from dw_tpu_b200 import _lib as L
    e, rows = 32, 1024 * TOPK
    w = dw.FP4MoEWeights(weights.w13[:e], weights.s13[:e], weights.w2[:e], weights.s2[:e],
                         weights.layout)
    x = torch.randn((rows, H), generator=torch.Generator().manual_seed(seed)).to(
        torch.bfloat16).to(dev)
    h1 = torch.empty((rows, I), dtype=torch.bfloat16, device=dev)
    y = torch.empty((rows, H), dtype=torch.bfloat16, device=dev)
    peaks = measured_peaks()
    peak = peaks["bf16_tflops"] if peaks else 1590.0
    out = {"workload": "cfg3 rank at n=8: 32 experts, 8192 rows, H=4096, I=2048",
           "bound": "tensor", "peak": peak, "unit": "TFLOP/s",
           "peak_source": "measured burst" if peaks else "fallback",
           "kernel": "dw_moe gmm_fp4 (automatic choice, variant 9: tcgen05 on CTA pairs, "
                     "tiles of up to 512 rows)"}
    for kind in ("uniform", "multinomial"):
        if kind == "uniform":
            gs_np = np.full(e, rows // e, np.int32)
        else:
            gs_np = np.random.default_rng(seed).multinomial(rows, [1.0 / e] * e).astype(np.int32)
        gs = torch.from_numpy(gs_np).to(dev)
        for name, fn, flops in (
                ("gmm1", lambda: ops.gmm_fp4_out(x, w.w13, w.s13, gs, h1, act=L.ACT_SWIGLU,
                                                 layout=w.layout), 2.0 * rows * H * 2 * I),
                ("gmm2", lambda: ops.gmm_fp4_out(h1, w.w2, w.s2, gs, y, layout=w.layout),
                 2.0 * rows * I * H)):
            for _ in range(3):
                fn()
            torch.cuda.synchronize(dev)
            ts = []
            for _ in range(iters):
                e0, e1 = events()
                e0.record()
                fn()
                e1.record()
                torch.cuda.synchronize(dev)
                ts.append(e0.elapsed_time(e1))
            tf = flops / statistics.median(ts) / 1e9
            out[f"{kind}_{name}_tflops"] = round(tf, 1)
            out[f"{kind}_{name}_frac"] = round(tf / peak, 4)
        if kind == "multinomial":  # the pair kernel with 256-row tiles (variant 7)
            for name, fn, flops in (
                    ("gmm1", lambda: ops.gmm_fp4_out(x, w.w13, w.s13, gs, h1, act=L.ACT_SWIGLU,
                                                     layout=w.layout, variant=7),
                     2.0 * rows * H * 2 * I),
                    ("gmm2", lambda: ops.gmm_fp4_out(h1, w.w2, w.s2, gs, y, layout=w.layout,
                                                     variant=7), 2.0 * rows * I * H)):
                fn()
                torch.cuda.synchronize(dev)
                ts = []
                for _ in range(iters):
                    e0, e1 = events()
                    e0.record()
                    fn()
                    e1.record()
                    torch.cuda.synchronize(dev)
                    ts.append(e0.elapsed_time(e1))
                out[f"multinomial_pair_only_{name}_tflops"] = round(
                    flops / statistics.median(ts) / 1e9, 1)
    L.raise_on_device_error()
    return out


def prefill_layer_single(weights, dev, seed, iters=10):
    """cfg3 at n=1: the single-device layer on T=1024 tokens (8192 rows over
    256 experts, ~32 rows per expert: the one-CTA tcgen05 kernel)."""
    import torch
    import dw_tpu_b200 as dw
    from dw_tpu_b200 import _lib as L
    from dw_tpu_b200 import synthetic
    t = 1024
    x, router = synthetic.layer_inputs(t, H, E, seed=seed + 7)
    x = x.to(dev)
    logits = (x.float() @ router.to(dev).float()).to(torch.bfloat16)
    layer = dw.MoELayer(weights, TOPK, t)
    out = torch.empty((t, H), dtype=torch.bfloat16, device=dev)
    for _ in range(3):
        layer(x, logits, out=out)
    torch.cuda.synchronize(dev)
    ts = []
    with GmmTimer() as gt:
        for _ in range(iters):
            e0, e1 = events()
            e0.record()
            layer(x, logits, out=out)
            e1.record()
            torch.cuda.synchronize(dev)
            ts.append(e0.elapsed_time(e1))
    L.raise_on_device_error()
    g1, g2 = gt.ms()
    ms = statistics.median(ts)
    flops = 2.0 * t * TOPK * (H * 2 * I + I * H)
    gs = layer.group_sizes.cpu().numpy()
    b1, b2, active, _ = gemm_bytes(gs)
    gmm_ms = statistics.median(g1) + statistics.median(g2)
    peaks = measured_peaks()
    return {"workload": "cfg3 at n=1: T=1024 tokens, 256 experts (one GPU)",
            "tokens_per_s": round(t / ms * 1e3, 1), "ms_per_step": round(ms, 4),
            "gmm_ms": round(gmm_ms, 4), "gmm_tflops": round(flops / gmm_ms / 1e9, 1),
            "gmm_GBps": round((b1 + b2) / (gmm_ms * 1e-3) / 1e9, 1),
            "gmm_frac_of_hbm": round((b1 + b2) / (gmm_ms * 1e-3) / 1e9 /
                                     (peaks["hbm_gbs"] if peaks else 6650.0), 4),
            "bound": "hbm (32 rows per expert: 3.4 GB of weights vs 412 GFLOP)",
            "active_experts": active, "rows_per_expert_max": int(gs.max())}


# ----------------------------------------------------------------------------
# Extras at N>1: link peak, exchange sweep (cfg2), prefill layer (cfg3),
# decode sweep (cfg4)
# ----------------------------------------------------------------------------

def link_peak(dev, world, rank, ctx, mib=256, iters=5):
    """Per-rank NVLink bandwidth measured here, each rank sending `mib` MiB to
    the next rank while receiving as much from the previous one (a ring):
    with NCCL send/recv, and with one copy-engine copy into the peer's mapped
    receive buffer (dwm_ep_link_probe). The larger is the link peak."""
    import torch
    import torch.distributed as dist
    n = mib * 2**20
    cn = min(n, ctx.capacity * ctx.hidden * 2)  # the peer copy stays inside the receive buffer
    src = torch.empty(n, dtype=torch.uint8, device=dev).fill_(1)
    dst = torch.empty(n, dtype=torch.uint8, device=dev)
    nxt, prv = (rank + 1) % world, (rank - 1) % world

    def ring():
        ops_ = [dist.P2POp(dist.isend, src, nxt), dist.P2POp(dist.irecv, dst, prv)]
        for r in dist.batch_isend_irecv(ops_):
            r.wait()
    for _ in range(2):
        ring()
    torch.cuda.synchronize(dev)
    ts = []
    for _ in range(iters):
        dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = events()
        e0.record()
        ring()
        e1.record()
        torch.cuda.synchronize(dev)
        ts.append(e0.elapsed_time(e1))
    cts = []
    for i in range(iters + 2):
        dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = events()
        e0.record()
        ctx.link_probe(nxt, cn)
        e1.record()
        torch.cuda.synchronize(dev)
        if i >= 2:
            cts.append(e0.elapsed_time(e1))
    dist.barrier()
    ms, cms = max_over_ranks([statistics.median(ts), statistics.median(cts)], world, dev)
    nccl_gbps = n / (ms * 1e-3) / 1e9
    copy_gbps = cn / (cms * 1e-3) / 1e9
    return {"GBps": round(max(nccl_gbps, copy_gbps), 1), "nccl_sendrecv_GBps": round(nccl_gbps, 1),
            "peer_copy_GBps": round(copy_gbps, 1),
            "how": f"ring of {mib} MiB per rank each way with NCCL send/recv, and a "
                   f"copy-engine copy of {cn // 2**20} MiB into the peer's mapped receive "
                   "buffer, median of 5, max over ranks; GBps = the larger"}


def zipf_logits(ids, dev):
    """Router logits whose sigmoid top-k are exactly `ids` (distinct per token)."""
    import torch
    t, k = ids.shape
    lg = torch.full((t, E), -16.0, dtype=torch.float32)
    lg.scatter_(1, torch.from_numpy(ids).long(),
                (8.0 - 0.25 * torch.arange(k, dtype=torch.float32)).expand(t, k).contiguous())
    return lg.to(torch.bfloat16).to(dev)


def ep_extras(args, local, dev, world, rank):
    import torch
    import torch.distributed as dist
    from dw_tpu_b200 import _lib as L
    from dw_tpu_b200 import ep as ep_mod
    from dw_tpu_b200 import synthetic
    le = E // world
    out = {}
    ctx = ep_mod.create_context(max_tokens=1024, hidden=H, topk=TOPK, num_experts=E)
    nccl = ep_mod.NcclExchange(E, H, TOPK)
    try:
        out["link"] = link_peak(dev, world, rank, ctx)
        link_gbps = out["link"]["GBps"]
        # ---- cfg2: the exchange alone, one-shot vs NCCL all_to_all_single ----
        sweep = []
        for t in (16, 128, 512):
            for dist_ in ("uniform", "zipf"):
                ids_np, w_np = synthetic.route_ids(t, E, TOPK, seed=1000 + 31 * t + rank,
                                                   dist=dist_)
                ids = torch.from_numpy(ids_np).to(dev)
                wts = torch.from_numpy(w_np).to(dev)
                hid = torch.randn((t, H), generator=torch.Generator().manual_seed(rank + t),
                                  ).to(torch.bfloat16).to(dev)
                y = ctx.output(torch.bfloat16)
                o1 = torch.empty((t, H), dtype=torch.bfloat16, device=dev)
                o2 = torch.empty_like(o1)

                def oneshot():
                    recv, gs = ctx.dispatch(hid, ids)
                    return recv, gs

                def oneshot_combine():
                    ctx.combine(y, wts, o1)

                # correctness on the real GPUs: both paths, identity experts
                recv, gs = oneshot()
                n = int(gs.sum())
                y[:n].copy_(recv[:n])
                oneshot_combine()
                r2, gs2 = nccl.dispatch(hid, ids)
                nccl.combine(r2, wts, o2)
                torch.cuda.synchronize(dev)
                same = (torch.equal(gs, gs2) and torch.equal(recv[:n].view(torch.int16),
                                                              r2.view(torch.int16))
                        and torch.equal(o1.view(torch.int16), o2.view(torch.int16)))
                times = {}
                for name, d_fn, c_fn in (
                        ("oneshot", oneshot, oneshot_combine),
                        ("nccl", lambda: nccl.dispatch(hid, ids),
                         lambda: nccl.combine(r2, wts, o2))):
                    for _ in range(3):
                        d_fn()
                        c_fn()
                    torch.cuda.synchronize(dev)
                    dist.barrier()
                    evs = []
                    # The one-shot kernels are shorter than the host's launch
                    # path: queue all iterations behind a device-side sleep so
                    # that the events time the device, not the host. (The NCCL
                    # path syncs on the host every dispatch; it runs as is.)
                    if name == "oneshot":
                        torch.cuda._sleep(PREROLL_CYCLES)
                    for _ in range(20):
                        a0, a1 = events()
                        b0, b1 = events()
                        a0.record()
                        d_fn()
                        a1.record()
                        b0.record()
                        c_fn()
                        b1.record()
                        evs.append((a0, a1, b0, b1))
                    torch.cuda.synchronize(dev)
                    dts = [a0.elapsed_time(a1) for a0, a1, _, _ in evs]
                    cts = [b0.elapsed_time(b1) for _, _, b0, b1 in evs]
                    times[name] = (statistics.median(dts), statistics.median(cts))
                owners = ids_np // le
                out_pairs = int((owners != rank).sum())
                out_dedup = sum(len(set(int(o) for o in row) - {rank}) for row in owners)
                in_pairs = n - int((owners == rank).sum())
                m = max_over_ranks([times["oneshot"][0], times["oneshot"][1], times["nccl"][0],
                                    times["nccl"][1], out_pairs, out_dedup, in_pairs,
                                    0.0 if same else 1.0], world, dev)
                pair_bytes = H * 2
                d_b, dd_b, c_b = m[4] * pair_bytes, m[5] * pair_bytes, m[6] * pair_bytes
                xch_ms = m[0] + m[1]
                sweep.append({
                    "tokens_per_rank": t, "routing": dist_,
                    "oneshot_dispatch_us": round(m[0] * 1e3, 1),
                    "oneshot_combine_us": round(m[1] * 1e3, 1),
                    "nccl_a2a_dispatch_us": round(m[2] * 1e3, 1),
                    "nccl_a2a_combine_us": round(m[3] * 1e3, 1),
                    "bytes_out_max_rank": int(d_b), "bytes_out_dedup_max_rank": int(dd_b),
                    "bytes_in_max_rank": int(c_b),
                    "nvlink_frac_dedup": round((dd_b + c_b) / (xch_ms * 1e-3) / 1e9 / link_gbps, 4),
                    "nvlink_frac_pairs": round((d_b + c_b) / (xch_ms * 1e-3) / 1e9 / link_gbps, 4),
                    "bit_equal_to_nccl_path": m[7] == 0.0,
                })
        out["exchange_sweep"] = {
            "workload": "cfg2: H=4096, top-8 over 256 experts, Dirichlet(1) weights; "
                        "dispatch then combine back to back, median of 20 per rank, max over "
                        "ranks",
            "link_GBps": link_gbps, "cases": sweep}
        L.raise_on_device_error()

        # ---- cfg3: the prefill EP layer, T=1024 per rank ----
        serial, o_s = ep_layer_case(ctx, local, dev, world, rank, 1024, "router", args.seed,
                                    link_gbps)
        over, o_o = ep_layer_case(ctx, local, dev, world, rank, 1024, "router", args.seed,
                                  link_gbps, compact=True, overlap=True)
        if over["variant"] != serial["variant"]:  # the bits check on the same GEMM kernel
            _, o_s = ep_layer_case(ctx, local, dev, world, rank, 1024, "router", args.seed,
                                   link_gbps, compact=True, iters=1,
                                   gemm_variant=over["variant"])
        differ = max_over_ranks([0.0 if torch.equal(o_s.view(torch.int16),
                                                    o_o.view(torch.int16)) else 1.0],
                                world, dev)[0]
        out["prefill_layer"] = {
            "workload": serial.pop("workload"), "serial": serial, "overlapped": over,
            "overlap_speedup": round(serial["ms_per_step"] / over["ms_per_step"], 3),
            "overlapped_bitwise_equal_serial_same_kernel": differ == 0.0}
        # ---- cfg4: the decode sweep on 8 GPUs, Zipf(1.2) ----
        if world == 8 or (world > 1 and args.decode_sweep):
            cases = [ep_layer_case(ctx, local, dev, world, rank, t, "zipf", args.seed,
                                   link_gbps, compact=True)[0]
                     for t in (2, 16, 64, 128, 256, 512)]
            out["decode_sweep"] = {"workload": "cfg4: T_rank in {1,8,32,64,128,256}x2, "
                                               f"Zipf(1.2) routing, {world} GPUs", "cases": cases}
    finally:
        ctx.close()
    return out


def ep_layer_case(ctx, local, dev, world, rank, t, routing, seed, link_gbps, compact=False,
                  iters=10, overlap=False, gemm_variant=None):
    """The EP layer on t tokens per rank: routing from a random router
    ("router", near-uniform) or Zipf(1.2)-skewed ids; median step time (max
    over ranks) and, for the serial layer, the GEMM's time and rate. With
    `overlap` the exchange is folded into the CTA-pair GEMMs. Returns (the
    record, this rank's output)."""
    import torch
    import torch.distributed as dist
    from dw_tpu_b200 import _lib as L
    from dw_tpu_b200 import ep as ep_mod
    from dw_tpu_b200 import synthetic
    x, router = synthetic.layer_inputs(t, H, E, seed=seed + 500 + rank)
    x = x.to(dev)
    if routing == "router":
        logits = (x.float() @ router.to(dev).float()).to(torch.bfloat16)
    else:
        ids_np, _ = synthetic.route_ids(t, E, TOPK, seed=2000 + 7 * t + rank, dist="zipf")
        logits = zipf_logits(ids_np, dev)
    expected = t * TOPK / E * world
    if gemm_variant is None and routing == "zipf" and expected > 16 and not overlap:
        gemm_variant = 10  # skewed groups: each on the kernel for its size
    layer = ep_mod.EPMoELayer(local, ctx, TOPK, expected_rows=expected, overlap=overlap,
                              gemm_variant=gemm_variant)
    out = torch.empty((t, H), dtype=torch.bfloat16, device=dev)
    for _ in range(3):
        layer(x, logits, out=out)
    torch.cuda.synchronize(dev)
    dist.barrier()
    evs = []
    with GmmTimer() as gt:
        torch.cuda._sleep(PREROLL_CYCLES)  # queue the steps: the events time the device
        for _ in range(iters):
            e0, e1 = events()
            e0.record()
            layer(x, logits, out=out)
            e1.record()
            evs.append((e0, e1))
        torch.cuda.synchronize(dev)
    ts = [a.elapsed_time(b) for a, b in evs]
    L.raise_on_device_error()
    g1, g2 = gt.ms()
    gs = ctx.recv_group_sizes.cpu().numpy()
    b1, b2, active, rows = gemm_bytes(gs)
    gmm_ms = statistics.median(g1) + statistics.median(g2) if g1 and g2 else 0.0
    flops = 2.0 * rows * (H * 2 * I + I * H)
    m = max_over_ranks([statistics.median(ts), gmm_ms, float(gs.max()), -float(gs.min())],
                       world, dev)
    peaks = measured_peaks()
    res = {"tokens_per_rank": t, "routing": routing,
           "variant": layer.variant, "overlap": overlap,
           "tokens_per_s": round(t * world / m[0] * 1e3, 1), "ms_per_step": round(m[0], 4),
           "rows_per_expert_max": int(m[2]), "rows_per_expert_min": int(-m[3])}
    if gmm_ms > 0:
        res.update({"gmm_ms_rank0": round(gmm_ms, 4), "gmm_ms_max": round(m[1], 4)})
        if flops / max(1, b1 + b2) > 300:  # tensor-bound (cfg3 at n >= 4)
            peak = peaks["bf16_tflops"] if peaks else 1590.0
            res["gmm_tflops_rank0"] = round(flops / gmm_ms / 1e9, 1)
            res["gmm_frac_of_tensor_rank0"] = round(flops / gmm_ms / 1e9 / peak, 4)
        else:
            peak = peaks["hbm_gbs"] if peaks else 6650.0
            res["gmm_GBps_rank0"] = round((b1 + b2) / (gmm_ms * 1e-3) / 1e9, 1)
            res["gmm_frac_of_hbm_rank0"] = round((b1 + b2) / (gmm_ms * 1e-3) / 1e9 / peak, 4)
    if not compact:
        res["workload"] = f"cfg3: T={t} tokens per rank, {world} ranks, router-drawn routing"
    return res, out


# ----------------------------------------------------------------------------
# Small single-GPU cases for ncu captures (``--case layer`` / ``--case gemm``)
# ----------------------------------------------------------------------------

def run_case(a):
    """layer: the cfg1 layer shapes with --experts experts and --tokens tokens
    (so an ncu capture stays at a few hundred MB); gemm: the two grouped
    matmuls alone on tokens*8 rows over the experts, --groups uniform (equal)
    or multinomial. Prints CUDA-event times and rates as one JSON line."""
    import torch
    import dw_tpu_b200 as dw
    from dw_tpu_b200 import _lib as L
    from dw_tpu_b200 import ops, synthetic
    dev = torch.device("cuda", 0)
    e, t = a.experts, a.tokens
    w = synthetic.moe_weights(e, H, I, seed=a.seed, device=dev).to_b200()
    res = {"case": a.case, "experts": e, "tokens": t}
    if a.case == "layer":
        x, router = synthetic.layer_inputs(t, H, e, seed=a.seed)
        x = x.to(dev)
        logits = (x.float() @ router.to(dev).float()).to(torch.bfloat16)
        layer = dw.MoELayer(w, TOPK, t, gemm_variant=a.variant)
        out = torch.empty((t, H), dtype=torch.bfloat16, device=dev)
        for _ in range(a.warmup):
            layer(x, logits, out=out)
        torch.cuda.synchronize(dev)
        s0, s1 = events()
        with GmmTimer() as gt:
            s0.record()
            for _ in range(a.iters):
                layer(x, logits, out=out)
            s1.record()
            torch.cuda.synchronize(dev)
        g1, g2 = gt.ms()
        b1, b2, active, rows = gemm_bytes(layer.group_sizes.cpu().numpy())
        m1, m2 = statistics.mean(g1), statistics.mean(g2)
        res.update({"active": active, "step_ms": round(s0.elapsed_time(s1) / a.iters, 4),
                    "gmm1_ms": round(m1, 4), "gmm1_GBps": round(b1 / m1 / 1e6, 1),
                    "gmm2_ms": round(m2, 4), "gmm2_GBps": round(b2 / m2 / 1e6, 1)})
    else:
        rows = t * TOPK
        if a.groups == "uniform":
            gs_np = np.full(e, rows // e, np.int32)
            gs_np[: rows - int(gs_np.sum())] += 1
        elif a.groups == "zipf":  # the experts of top-k Zipf(1.2) routing (cfg2/cfg4)
            ids_np, _ = synthetic.route_ids(t, e, TOPK, seed=a.seed, dist="zipf")
            gs_np = np.bincount(ids_np.ravel(), minlength=e).astype(np.int32)
        else:
            gs_np = np.random.default_rng(a.seed).multinomial(rows, [1.0 / e] * e).astype(
                np.int32)
        gs = torch.from_numpy(gs_np).to(dev)
        x = torch.randn((rows, H), generator=torch.Generator().manual_seed(a.seed)).to(
            torch.bfloat16).to(dev)
        h1 = torch.empty((rows, I), dtype=torch.bfloat16, device=dev)
        y = torch.empty((rows, H), dtype=torch.bfloat16, device=dev)
        res.update({"rows": rows, "groups": a.groups, "max_group": int(gs_np.max()),
                    "min_group": int(gs_np.min())})
        for name, fn, flops in (
                ("gmm1", lambda: ops.gmm_fp4_out(x, w.w13, w.s13, gs, h1, act=L.ACT_SWIGLU,
                                                 layout="b200", variant=a.variant),
                 2.0 * rows * H * 2 * I),
                ("gmm2", lambda: ops.gmm_fp4_out(h1, w.w2, w.s2, gs, y, layout="b200",
                                                 variant=a.variant), 2.0 * rows * I * H)):
            for _ in range(a.warmup):
                fn()
            torch.cuda.synchronize(dev)
            ts = []
            for _ in range(a.iters):
                e0, e1 = events()
                e0.record()
                fn()
                e1.record()
                torch.cuda.synchronize(dev)
                ts.append(e0.elapsed_time(e1))
            ms = statistics.median(ts)
            res[f"{name}_ms"] = round(ms, 4)
            res[f"{name}_TFLOPs"] = round(flops / ms / 1e9, 1)
    L.raise_on_device_error()
    print(json.dumps(res), flush=True)


# ----------------------------------------------------------------------------

def main():
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.gpus != world and world > 1:
        print(f"--gpus {args.gpus} != WORLD_SIZE {world}", file=sys.stderr)

    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.case != "bench":
        run_case(args)
        return

    import torch
    import torch.distributed as dist
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank),
                                timeout=datetime.timedelta(seconds=120))
    res = run_ours(args, rank, world, local_rank)
    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline(args.seed)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    tokens = T_RANK * world * args.steps
    line = {
        "metric": METRIC, "value": round(tokens / (res["ms"] * 1e-3), 1), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(res["ms"] / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; FP4 weights and E8M0 scales as BASELINE config 0/1)",
        "config": dict(config_of(world), **({"exchange": "one-shot, overlapped with the GEMMs"}
                                             if world > 1 and args.overlap else {})),
        "e2e": {"value": round(tokens / (res["e2e_ms"] * 1e-3), 1), "unit": UNIT,
                "h2d_bytes_per_step": res["h2d"], "d2h_bytes_per_step": res["d2h"]},
        "roofline": res["roofline"],
        "parity": res["parity"],
        "cpu_baseline": None if cb is None else
        {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "clocks": res["clocks"],
        "gpu_launches": res["launches_per_step"] * args.steps,
        "active_experts": res["active"],
    }
    for key in ("exchange", "link", "prefill", "prefill_layer", "exchange_sweep",
                "decode_sweep"):
        if key in res:
            line[key] = res[key]
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
