"""Loader for libdw_moe.so, the C ABI declared in include/dw_moe.h.

The library is built in-tree (``dw_tpu_b200/libdw_moe.so``, see
``dw_tpu_b200/build.py``). There is no fallback: if the library is missing or
does not load, every op raises instead of computing anything elsewhere.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
# DWM_LIB_PATH selects another build of the same C ABI (e.g. one compiled with
# different pipeline depths); default: the in-tree library.
LIB_PATH = os.environ.get("DWM_LIB_PATH") or os.path.join(_HERE, "libdw_moe.so")

# include/dw_moe.h constants
OK = 0
ERR_INVALID = -1
ERR_UNSUPPORTED = -2
ERR_STATE = -3
DEV_TIMEOUT = 1
DEV_BAD_INDEX = 2
DEV_OVERFLOW = 4
BF16 = 0
F32 = 1
U8 = 2
ACT_NONE = 0
ACT_SWIGLU = 1
ACT_SWIGLU_CLAMP = 2
FP4_E2M1 = 0
FP4_TOKAMAX = 1
FP4_B200 = 2
LAYOUTS = {"e2m1": FP4_E2M1, "b200": FP4_B200}
SCORE_SOFTMAX = 0
SCORE_SIGMOID = 1
SCORE_SQRTSOFTPLUS = 2
LAYER_SCRATCH_BYTES = 33554432  # DWM_LAYER_SCRATCH_BYTES
EP_HANDLE_BYTES = 64
EP_COUNTS = 1
EP_ROWS = 2
EP_WAIT = 4
EP_ALL = 7
EP_PUSH = 1
EP_REDUCE = 2
EP_GATED = 8
EP_PUSHED = 4
EP_RANK_ORDER = 16
EP_GEMM_GATED = 1
EP_GEMM_PUSH = 2

_c = ctypes
_P = _c.c_void_p
_I = _c.c_int
_I64 = _c.c_int64
_SZ = _c.c_size_t
_F = _c.c_float

# name -> argtypes (restype is always int unless noted)
SIGNATURES = {
    "dwm_version": ([], _c.c_char_p),
    "dwm_last_error": ([], _c.c_char_p),
    "dwm_device_status": ([_P, _c.POINTER(_I)], _I),
    "dwm_gmm_fp4": ([_P, _P, _I, _P, _I, _P, _I, _I, _I, _I, _I, _I, _I, _F, _I, _I, _P, _P],
                    _I),
    "dwm_fp4_dequant": ([_P, _I, _P, _I, _I, _I, _I, _P, _P], _I),
    "dwm_fp4_to_b200": ([_P, _P, _I, _I, _I, _I, _P], _I),
    "dwm_gmm_fp4_variant": ([_P, _P, _I, _P, _I, _P, _I, _I, _I, _I, _I, _I, _I, _F, _I, _I, _P,
                             _I, _P], _I),
    "dwm_fp4_codes_convert": ([_P, _P, _SZ, _I, _I, _P], _I),
    "dwm_fp4_quantize": ([_P, _I, _I, _I, _I, _I, _P, _P, _I, _P, _P], _I),
    "dwm_e8m0_encode": ([_P, _SZ, _P, _P, _P], _I),
    "dwm_e8m0_decode": ([_P, _SZ, _P, _P], _I),
    "dwm_route_topk": ([_P, _I, _I, _I, _I, _I, _I, _P, _I, _P, _P, _P, _P], _I),
    "dwm_route_hash": ([_P, _I, _I, _I, _I, _I, _I, _P, _I, _P, _P, _P, _P], _I),
    "dwm_dedupe_topk": ([_P, _P, _I, _I, _I, _P, _P], _I),
    "dwm_sorted_token_indices": ([_P, _I64, _I, _P, _P], _I),
    "dwm_permute": ([_P, _I, _I, _I, _P, _P, _P, _P, _P], _I),
    "dwm_dispatch_gather": ([_P, _I, _I, _P, _I64, _P, _P], _I),
    "dwm_combine": ([_P, _I, _I64, _P, _P, _I, _I, _I, _I, _P, _I, _P], _I),
    "dwm_combine_shared": ([_P, _I, _I64, _P, _P, _I, _I, _I, _I, _P, _I, _F, _I, _P, _I, _P], _I),
    "dwm_moe_layer_workspace_bytes": ([_I, _I, _I, _I, _I, _I], _SZ),
    "dwm_moe_layer_fp4": ([_P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _I, _I, _I, _I,
                           _F, _I, _P, _SZ, _P, _P], _I),
    "dwm_moe_layer_fp4_noalloc": ([_P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _I, _I,
                                   _I, _I, _F, _I, _P, _P], _I),
    "dwm_ep_create": ([_I, _I, _I, _I, _I, _I, _c.POINTER(_P)], _I),
    "dwm_ep_ipc_handle": ([_P, _P], _I),
    "dwm_ep_connect": ([_P, _P], _I),
    "dwm_ep_connect_local": ([_P, _c.POINTER(_P)], _I),
    "dwm_ep_recv_buffer": ([_P, _c.POINTER(_P), _c.POINTER(_I64)], _I),
    "dwm_ep_output_buffer": ([_P, _c.POINTER(_P), _c.POINTER(_I64)], _I),
    "dwm_ep_dispatch": ([_P, _P, _P, _I, _P, _I, _P], _I),
    "dwm_ep_combine": ([_P, _P, _I, _P, _I, _P, _I, _I, _P], _I),
    "dwm_ep_combine_shared": ([_P, _P, _I, _P, _I, _P, _I, _F, _I, _P, _I, _I, _P], _I),
    "dwm_ep_set_wait_limit": ([_P, _c.c_uint64], _I),
    "dwm_ep_link_probe": ([_P, _I, _I64, _P], _I),
    "dwm_ep_gmm_fp4": ([_P, _P, _P, _I, _P, _I, _P, _I, _I, _I, _F, _I, _P, _I, _I, _P], _I),
    "dwm_ep_destroy": ([_P], _I),
}

_lib = None
_lock = threading.Lock()


class DeviceError(RuntimeError):
    """A kernel reported a device-side fault through the status word."""


def require_built() -> None:
    """Raise ImportError if libdw_moe.so has not been built (without mapping it)."""
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} not found: build it with `python __graft_entry__.py` (nvcc, sm_100a)")


def load():
    """Map libdw_moe.so once (on the first op call); raise ImportError if it
    is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            require_built()
            lib = _c.CDLL(LIB_PATH)
            for name, (args, res) in SIGNATURES.items():
                fn = getattr(lib, name, None)
                if fn is None:
                    continue  # reported by exported_symbols() checks
                fn.argtypes = args
                fn.restype = res
            _lib = lib
    return _lib


def lib():
    return load()


def last_error() -> str:
    msg = lib().dwm_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    """Map a C ABI return code to a Python exception."""
    if rc == OK:
        return
    if rc in (ERR_INVALID, ERR_UNSUPPORTED):
        raise ValueError(f"{what}: {last_error()}")
    if rc < 0:
        raise RuntimeError(f"{what}: {last_error()}")
    raise RuntimeError(f"{what}: CUDA error {rc}: {last_error()}")


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def device_status(stream: int | None = None) -> int:
    """Synchronise the stream, return and clear the device status bits."""
    bits = _I(0)
    s = stream_ptr() if stream is None else stream
    check(lib().dwm_device_status(s, _c.byref(bits)), "dwm_device_status")
    return bits.value


def raise_on_device_error(stream: int | None = None) -> None:
    bits = device_status(stream)
    if bits:
        names = [n for b, n in ((DEV_TIMEOUT, "timeout"), (DEV_BAD_INDEX, "bad index"),
                                (DEV_OVERFLOW, "overflow")) if bits & b]
        raise DeviceError(f"device status {bits:#x}: {', '.join(names)}")


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return BF16
    if dt == torch.float32:
        return F32
    if dt == torch.uint8 or dt == getattr(torch, "float8_e8m0fnu", None):
        return U8
    raise ValueError(f"unsupported dtype {dt}")


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("dw_tpu_b200 ops take CUDA tensors (no CPU path)")
