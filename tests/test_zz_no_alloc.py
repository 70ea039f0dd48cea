"""dwm_moe_layer_fp4_noalloc (the layer on the library's fixed device scratch)
against dwm_moe_layer_fp4 (the same layer on a caller workspace): identical
bits on two calls in a row, and no device memory taken by a call. This file
sorts last so that it also runs after every other GPU test in the same
process."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("layout,f32_reduce", [("b200", False), ("e2m1", True)])
def test_noalloc_layer_matches_workspace_layer_twice(layout, f32_reduce):
    from dw_tpu_b200 import _lib as L
    from dw_tpu_b200 import ops, synthetic
    t, e, h, i, k = 48, 16, 512, 256, 4
    w = synthetic.moe_weights(e, h, i, seed=12, device="cuda")
    for name in ("s13", "s2"):
        setattr(w, name, synthetic.random_e8m0(getattr(w, name).shape, 13, "cuda", lo=118,
                                               hi=121))
    if layout == "b200":
        w = w.to_b200()
    ws = torch.empty(ops.moe_layer_workspace_bytes(t, h, i, k, e, f32_reduce),
                     dtype=torch.uint8, device="cuda")
    for seed in (40, 41):  # two calls in a row, new tokens each time
        x, router = synthetic.layer_inputs(t, h, e, seed=seed)
        x = x.cuda()
        lg = (x.float() @ router.cuda().float()).to(torch.bfloat16)
        ref = torch.empty((t, h), dtype=torch.bfloat16, device="cuda")
        ops.moe_layer_fp4_out(x, lg, k, w.w13, w.s13, w.w2, w.s2, ref, ws, layout=layout,
                              f32_reduce=f32_reduce)
        got = torch.full((t, h), 7.0, dtype=torch.bfloat16, device="cuda")
        ops.moe_layer_fp4_noalloc_out(x, lg, k, w.w13, w.s13, w.w2, w.s2, got, layout=layout,
                                      f32_reduce=f32_reduce)
        torch.cuda.synchronize()
        L.raise_on_device_error()
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), seed


def test_noalloc_layer_rejects_oversize_inputs():
    from dw_tpu_b200 import _lib as L
    from dw_tpu_b200 import ops
    e, h, i, k = 16, 4096, 2048, 8
    t = 1024  # 8192 rows: about 200 MiB of intermediates
    assert ops.moe_layer_workspace_bytes(t, h, i, k, e) > L.LAYER_SCRATCH_BYTES
    x = torch.zeros((t, h), dtype=torch.bfloat16, device="cuda")
    lg = torch.zeros((t, e), dtype=torch.bfloat16, device="cuda")
    w13 = torch.zeros((e, h, i), dtype=torch.uint8, device="cuda")
    s13 = torch.zeros((e, h // 32, 2 * i), dtype=torch.uint8, device="cuda")
    w2 = torch.zeros((e, i, h // 2), dtype=torch.uint8, device="cuda")
    s2 = torch.zeros((e, i // 32, h), dtype=torch.uint8, device="cuda")
    out = torch.empty((t, h), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="scratch"):
        ops.moe_layer_fp4_noalloc_out(x, lg, k, w13, s13, w2, s2, out)


def test_noalloc_layer_setup_call_and_no_device_allocation():
    """A num_tokens = 0 call does only the per-device set-up; later calls take
    no device memory: PyTorch's allocator and the device's free bytes are
    unchanged across a call (the first real call may still load kernels)."""
    from dw_tpu_b200 import _lib as L
    from dw_tpu_b200 import ops, synthetic
    t, e, h, i, k = 32, 16, 512, 256, 4
    w = synthetic.moe_weights(e, h, i, seed=14, device="cuda").to_b200()
    for name in ("s13", "s2"):
        setattr(w, name, synthetic.random_e8m0(getattr(w, name).shape, 15, "cuda", lo=118,
                                               hi=121))
    x, router = synthetic.layer_inputs(t, h, e, seed=16)
    x = x.cuda()
    lg = (x.float() @ router.cuda().float()).to(torch.bfloat16)
    out = torch.empty((t, h), dtype=torch.bfloat16, device="cuda")
    ops.moe_layer_fp4_noalloc_out(x[:0], lg[:0], k, w.w13, w.s13, w.w2, w.s2, out[:0],
                                  layout="b200")                     # set-up only
    ops.moe_layer_fp4_noalloc_out(x, lg, k, w.w13, w.s13, w.w2, w.s2, out, layout="b200")
    torch.cuda.synchronize()
    L.raise_on_device_error()
    first = out.clone()
    alloc0 = torch.cuda.memory_allocated()
    free0, _ = torch.cuda.mem_get_info()
    ops.moe_layer_fp4_noalloc_out(x, lg, k, w.w13, w.s13, w.w2, w.s2, out, layout="b200")
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert torch.cuda.memory_allocated() == alloc0
    assert free1 >= free0, (free0, free1)
    assert torch.equal(out.view(torch.int16), first.view(torch.int16))
