"""Small, self-contained MoE layer run for timing and for ncu captures.

    python -m dw_tpu_b200.profile_case [--experts E] [--tokens T] [--iters N]
    python -m dw_tpu_b200.profile_case --groups uniform|multinomial ...

Runs the config-1 layer shapes (H=4096, I=2048, top-8, sigmoid routing) with
a configurable expert count, so an ncu capture of the FP4 GEMM can stay at a
few hundred MB on the device, and prints per-kernel CUDA-event times and the
algorithmic HBM bandwidth of each gmm launch.

With --groups the two grouped matmuls run alone on tokens * topk rows spread
over the experts either exactly evenly or as one seeded multinomial draw
(what uniform routing gives), and the median of --iters launches is
reported.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import MoELayer, ops, synthetic
from . import _lib as L
from . import fused_moe as fm


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--experts", type=int, default=256)
    p.add_argument("--tokens", type=int, default=64)
    p.add_argument("--hidden", type=int, default=4096)
    p.add_argument("--inter", type=int, default=2048)
    p.add_argument("--topk", type=int, default=8)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--layout", default="b200", choices=["b200", "e2m1", "cm"])
    p.add_argument("--variant", type=int, default=0,
                   help="dwm_gmm_fp4_variant kernel choice (0 = automatic)")
    p.add_argument("--groups", choices=["uniform", "multinomial"], default=None,
                   help="time gmm1/gmm2 alone on these group sizes")
    a = p.parse_args()
    if a.groups:
        return gemm_only(a)
    e, h, i, t, k = a.experts, a.hidden, a.inter, a.tokens, a.topk
    w = synthetic.moe_weights(e, h, i, seed=a.seed, device="cuda")
    if a.layout == "b200":
        w = w.to_b200()
    elif a.layout == "cm":
        w = w.to_cm()
    x, router = synthetic.layer_inputs(t, h, e, seed=a.seed)
    x = x.cuda()
    logits = (x.float() @ router.cuda().float()).to(torch.bfloat16)
    layer = MoELayer(w, k, t, gemm_variant=a.variant)
    out = torch.empty((t, h), dtype=torch.bfloat16, device="cuda")
    for _ in range(a.warmup):
        layer(x, logits, out=out)
    torch.cuda.synchronize()
    L.raise_on_device_error()

    events = []
    orig = ops.gmm_fp4_out

    def timed(*args, **kw):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        r = orig(*args, **kw)
        e1.record()
        events.append((kw.get("act", L.ACT_NONE), e0, e1))
        return r

    fm.ops.gmm_fp4_out = timed
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(a.iters):
        layer(x, logits, out=out)
    s1.record()
    torch.cuda.synchronize()
    fm.ops.gmm_fp4_out = orig
    L.raise_on_device_error()

    gs = layer.group_sizes.cpu()
    active = int((gs > 0).sum())
    rows = t * k
    b1 = active * (h * i + (h // 32) * 2 * i) + rows * h * 2 + rows * i * 2
    b2 = active * (i * h // 2 + (i // 32) * h) + rows * i * 2 + rows * h * 2
    g1 = [a_.elapsed_time(b_) for act, a_, b_ in events if act != L.ACT_NONE]
    g2 = [a_.elapsed_time(b_) for act, a_, b_ in events if act == L.ACT_NONE]
    m1, m2 = sum(g1) / len(g1), sum(g2) / len(g2)
    step = s0.elapsed_time(s1) / a.iters
    print(json.dumps({
        "experts": e, "active": active, "tokens": t, "step_ms": round(step, 4),
        "gmm1_ms": round(m1, 4), "gmm1_GBps": round(b1 / m1 / 1e6, 1),
        "gmm2_ms": round(m2, 4), "gmm2_GBps": round(b2 / m2 / 1e6, 1),
        "gmm1_TFLOPs": round(2 * rows * h * 2 * i / m1 / 1e9, 1),
        "gmm2_TFLOPs": round(2 * rows * i * h / m2 / 1e9, 1),
        "tokens_per_s": round(t / step * 1e3, 1),
    }))


def gemm_only(a):
    import numpy as np
    e, h, i = a.experts, a.hidden, a.inter
    rows = a.tokens * a.topk
    w = synthetic.moe_weights(e, h, i, seed=a.seed, device="cuda")
    w = w.to_b200() if a.layout == "b200" else w.to_cm() if a.layout == "cm" else w
    if a.groups == "uniform":
        gs_np = np.full(e, rows // e, np.int32)
        gs_np[: rows - int(gs_np.sum())] += 1
    else:
        gs_np = np.random.default_rng(a.seed).multinomial(rows, [1.0 / e] * e).astype(np.int32)
    gs = torch.from_numpy(gs_np).cuda()
    x = torch.randn((rows, h), generator=torch.Generator().manual_seed(a.seed)).to(torch.bfloat16).cuda()
    h1 = torch.empty((rows, i), dtype=torch.bfloat16, device="cuda")
    y = torch.empty((rows, h), dtype=torch.bfloat16, device="cuda")

    def g1():
        ops.gmm_fp4_out(x, w.w13, w.s13, gs, h1, act=L.ACT_SWIGLU, layout=w.layout,
                        variant=a.variant)

    def g2():
        ops.gmm_fp4_out(h1, w.w2, w.s2, gs, y, layout=w.layout, variant=a.variant)

    res = {"experts": e, "rows": rows, "groups": a.groups, "max_group": int(gs_np.max()),
           "min_group": int(gs_np.min())}
    for f, name, flops in ((g1, "gmm1", 2.0 * rows * h * 2 * i), (g2, "gmm2", 2.0 * rows * i * h)):
        for _ in range(a.warmup):
            f()
        torch.cuda.synchronize()
        ts = []
        for _ in range(a.iters):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            f()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        ms = float(np.median(ts))
        res[f"{name}_ms"] = round(ms, 4)
        res[f"{name}_TFLOPs"] = round(flops / ms / 1e9, 1)
    L.raise_on_device_error()
    print(json.dumps(res))


if __name__ == "__main__":
    main()
