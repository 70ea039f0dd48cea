"""The C ABI library loads and exports every symbol include/*.h declares, and
argument validation runs on the host (no GPU compute in this file)."""

import ctypes
import glob
import os
import re

import pytest

from tests.conftest import ROOT

HEADERS = sorted(glob.glob(os.path.join(ROOT, "include", "*.h")))


def declared_symbols():
    names = set()
    for h in HEADERS:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"\b(dwm_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    from dw_tpu_b200 import _lib
    return _lib.load()


def test_headers_declare_entry_points():
    syms = declared_symbols()
    assert "dwm_gmm_fp4" in syms and "dwm_combine" in syms and "dwm_permute" in syms


def test_library_exports_every_declared_symbol(lib):
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_python_signatures_cover_header():
    from dw_tpu_b200 import _lib
    missing = [s for s in declared_symbols() if s not in _lib.SIGNATURES]
    assert not missing, missing


def test_version(lib):
    assert b"sm_100a" in lib.dwm_version()


def _gmm(lib, **kw):
    args = dict(lhs=None, codes=None, fmt=0, scales=None, sd=2, gs=None, ng=8, m=16, k=64,
                n=256, go=0, nl=8, act=0, lim=0.0, od=0, zi=0, out=None, stream=None)
    args.update(kw)
    return lib.dwm_gmm_fp4(*args.values())


def test_gmm_rejects_bad_shapes_on_host(lib):
    from dw_tpu_b200 import _lib
    fake = 1 << 20  # never dereferenced: validation fails first
    assert _gmm(lib, k=63, lhs=fake, codes=fake, scales=fake, gs=fake, out=fake) == -1
    assert "multiple of 64" in _lib.last_error()
    assert _gmm(lib, n=128, lhs=fake, codes=fake, scales=fake, gs=fake, out=fake) == -1
    assert _gmm(lib, fmt=1, lhs=fake, codes=fake, scales=fake, gs=fake, out=fake) == -1
    assert "tokamax" in _lib.last_error()
    assert _gmm(lib, go=4, nl=8, lhs=fake, codes=fake, scales=fake, gs=fake, out=fake) == -1
    assert _gmm(lib, sd=7, lhs=fake, codes=fake, scales=fake, gs=fake, out=fake) == -1
    assert _gmm(lib, lhs=fake + 8, codes=fake, scales=fake, gs=fake, out=fake) == -1
    assert "aligned" in _lib.last_error()


def test_other_entry_points_validate(lib):
    fake = 1 << 20
    assert lib.dwm_permute(fake, 4, 0, 8, None, None, None, fake, None) == -1
    assert lib.dwm_permute(fake, 4, 2, 2000, None, None, None, fake, None) == -1
    assert lib.dwm_combine(fake, 5, 4, fake, fake, 0, 1, 64, 2, fake, 0, None) == -1
    assert lib.dwm_combine(fake, 0, 4, fake, fake, 0, 1, 60, 2, fake, 0, None) == -1
    assert lib.dwm_dispatch_gather(fake, 4, 12, fake, 4, fake, None) == -1
    assert lib.dwm_route_topk(fake, 0, 4, 8, 9, 1, 1, None, -1, fake, None, None, None) == -1
    assert lib.dwm_route_topk(fake, 0, 4, 8, 2, 7, 1, None, -1, fake, None, None, None) == -1
    assert lib.dwm_fp4_codes_convert(fake, fake, 16, 0, 5, None) == -1
    assert lib.dwm_fp4_dequant(fake, 0, fake, 2, 1, 48, 64, fake, None) == -1
    assert lib.dwm_fp4_dequant(fake, 1, fake, 2, 1, 64, 64, fake, None) == -1
    assert lib.dwm_fp4_to_b200(fake, fake + 64, 1, 12, 8, 0, None) == -1
    assert lib.dwm_fp4_to_b200(fake, fake, 1, 16, 8, 0, None) == -1
    assert lib.dwm_gmm_fp4_variant(fake, fake, 0, fake, 2, fake, 8, 16, 64, 256, 0, 8, 0, 0.0,
                                   0, 0, fake, 2, None) == -1  # explicit variant needs B200
    assert lib.dwm_device_status(None, None) == -1
    import ctypes
    ctx = ctypes.c_void_p()
    assert lib.dwm_ep_create(0, 9, 4, 64, 2, 16, ctypes.byref(ctx)) == -1   # world > 8
    assert lib.dwm_ep_create(2, 2, 4, 64, 2, 16, ctypes.byref(ctx)) == -1   # rank >= world
    assert lib.dwm_ep_create(0, 3, 4, 64, 2, 16, ctypes.byref(ctx)) == -1   # 16 % 3
    assert lib.dwm_ep_create(0, 2, 4, 60, 2, 16, ctypes.byref(ctx)) == -1   # hidden % 8
    assert ctx.value is None
    assert lib.dwm_ep_dispatch(None, fake, fake, 4, fake, 7, None) == -1
    assert lib.dwm_ep_combine(None, fake, 0, fake, 0, fake, 0, 3, None) == -1
    assert lib.dwm_ep_ipc_handle(None, None) == -1
    assert lib.dwm_ep_destroy(None) == 0
    # the no-alloc layer rejects inputs larger than its built-in scratch on the host
    assert lib.dwm_moe_layer_fp4_noalloc(fake, fake, 0, 1024, 4096, 16, 8, 1, 1, fake, fake, fake,
                                         fake, 2, 2, 2048, 1, 0.0, 0, fake, None) == -1
    from dw_tpu_b200 import _lib
    assert "scratch" in _lib.last_error()
    assert lib.dwm_moe_layer_fp4(fake, fake, 0, 8, 512, 16, 4, 1, 1, fake, fake, fake, fake, 2, 2,
                                 256, 1, 0.0, 0, fake, 16, fake, None) == -1  # workspace too small


def test_python_shims_raise_value_error_without_gpu():
    import torch
    import dw_tpu_b200 as dw
    lhs = torch.zeros((4, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        dw.gmm_v2(lhs, torch.zeros((1, 64, 128), dtype=torch.uint8),
                  torch.zeros(1, dtype=torch.int32),
                  torch.zeros((1, 2, 256), dtype=torch.uint8))
    with pytest.raises(ValueError):
        dw.fast_combine(torch.zeros((4, 8)), torch.zeros(4, dtype=torch.int32),
                        torch.zeros((2, 2)), 2, mode=3)
    with pytest.raises(ValueError):
        dw.gmm_v2(lhs.float(), torch.zeros((1, 64, 128), dtype=torch.uint8),
                  torch.zeros(1, dtype=torch.int32), torch.zeros((1, 2, 256), dtype=torch.uint8))


def test_build_writes_library_in_tree():
    from dw_tpu_b200 import _lib
    assert os.path.dirname(_lib.LIB_PATH) == os.path.join(ROOT, "dw_tpu_b200")
    assert os.path.exists(_lib.LIB_PATH)


def _layer_tensors(t=8, e=4, h=256, i=128, layout="e2m1"):
    import torch
    x = torch.zeros((t, h), dtype=torch.bfloat16)
    lg = torch.zeros((t, e), dtype=torch.bfloat16)
    if layout == "e2m1":
        w13 = torch.zeros((e, h, i), dtype=torch.uint8)
        w2 = torch.zeros((e, i, h // 2), dtype=torch.uint8)
    else:
        w13 = torch.zeros((e, 2 * i, h // 2), dtype=torch.uint8)
        w2 = torch.zeros((e, h, i // 2), dtype=torch.uint8)
    s13 = torch.zeros((e, h // 32, 2 * i), dtype=torch.uint8)
    s2 = torch.zeros((e, i // 32, h), dtype=torch.uint8)
    out = torch.zeros((t, h), dtype=torch.bfloat16)
    return x, lg, w13, s13, w2, s2, out


@pytest.mark.parametrize("layout", ["e2m1", "b200"])
def test_layer_wrappers_check_shapes_before_any_launch(layout):
    """The one-call layer wrappers reject a wrong-sized out or weight tensor
    (the C layer sizes its tensor maps and stores from the shapes alone)."""
    import torch
    from dw_tpu_b200 import ops
    x, lg, w13, s13, w2, s2, out = _layer_tensors(layout=layout)
    ws = torch.zeros(1 << 16, dtype=torch.uint8)
    bad = {
        "out_rows": dict(out=out[:4]),
        "out_dtype": dict(out=out.float()),
        "w13": dict(w13=w13[:, :, : w13.shape[2] // 2]),
        "w2": dict(w2=w2[:2]),
        "s13": dict(s13=s13[:, :4]),
        "s2_dtype": dict(s2=s2.float()),
    }
    for name, kw in bad.items():
        args = dict(hidden=x, logits=lg, w13=w13, s13=s13, w2=w2, s2=s2, out=out)
        args.update(kw)
        with pytest.raises(ValueError):
            ops.moe_layer_fp4_out(args["hidden"], args["logits"], 2, args["w13"], args["s13"],
                                  args["w2"], args["s2"], args["out"], ws, layout=layout)
        with pytest.raises(ValueError):
            ops.moe_layer_fp4_noalloc_out(args["hidden"], args["logits"], 2, args["w13"],
                                          args["s13"], args["w2"], args["s2"], args["out"],
                                          layout=layout)
    # well-formed host tensors get past the shape checks and stop at the CUDA check
    with pytest.raises(ValueError, match="CUDA"):
        ops.moe_layer_fp4_out(x, lg, 2, w13, s13, w2, s2, out, ws, layout=layout)


def test_package_import_does_not_map_the_library():
    """Importing the package (e.g. for its input generators) maps no library;
    the first op call does."""
    import subprocess
    import sys
    code = ("import dw_tpu_b200, dw_tpu_b200.synthetic, sys\n"
            "maps = open('/proc/self/maps').read()\n"
            "sys.exit(3 if 'libdw_moe.so' in maps else 0)\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
