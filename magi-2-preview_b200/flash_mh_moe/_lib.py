"""ctypes binding of libmhmoe (the C ABI in include/mhmoe.h).

There is exactly one backend: the sm_100a CUDA library.  If it is missing, or the
current device is not a B200 (sm_100), every call raises — there is no CPU or
Triton fallback.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import torch

_PKG_ROOT = Path(__file__).resolve().parent.parent
LIB_PATH = Path(os.environ.get("MHMOE_LIB", _PKG_ROOT / "lib" / "libmhmoe.so"))

MHMOE_OK = 0
MHMOE_ERR_ARGS = 1
MHMOE_ERR_TIMEOUT = 4

vp, i32, i64, f32, u64, sz = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_uint64, C.c_size_t

# name -> (restype, argtypes); mirrors include/mhmoe.h
SIGNATURES: dict[str, tuple] = {
    "mhmoe_version": (i32, []),
    "mhmoe_status_string": (C.c_char_p, [i32]),
    "mhmoe_last_error": (C.c_char_p, []),
    "mhmoe_router_logits": (i32, [vp, i64, i64, vp, i32, i32, i32, i32, vp, vp]),
    "mhmoe_router_prepare": (i32, [vp, i32, i32, i32, vp, vp, vp]),
    "mhmoe_route": (i32, [vp, i64, i64, vp, i32, i32, i32, i32, i32, i32, i32, vp, vp, i32, f32, f32, vp, vp, vp,
                          vp, vp]),
    "mhmoe_topk": (i32, [vp, vp, i32, i32, i32, i32, i32, i32, i32, i32, f32, f32, vp, vp, vp]),
    "mhmoe_global_sort_workspace_bytes": (sz, [i32, i32, i32, i32]),
    "mhmoe_global_sort": (i32, [vp, vp, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp]),
    "mhmoe_global_sort_noalloc": (i32, [vp, vp, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp]),
    "mhmoe_max_mtiles": (i64, [i64, i32]),
    "mhmoe_ffn_workspace_bytes": (sz, [i64, i32, i32, i32, i32, i32]),
    "mhmoe_pack_weights_nvfp4": (i32, [i32, vp, vp, i32, i32, i32, vp, vp, vp, vp, vp]),
    "mhmoe_ffn_nvfp4": (i32, [vp, i64, i64, i32, i32, i32, i32, i32, i64, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                              vp, vp, i32, vp, vp, i64, i64, vp, u64, vp, vp]),
    "mhmoe_ffn_nvfp4_quantized": (i32, [vp, i64, vp, i64, vp, i64, i32, i32, i32, i32, i64, vp, vp, vp, vp, vp, vp,
                                        vp, vp, vp, vp, vp, i32, vp, vp, i64, vp, u64, vp, vp]),
    "mhmoe_quant_tokens": (i32, [vp, i64, i64, i32, i32, i32, vp, vp, vp, vp]),
    "mhmoe_combine": (i32, [vp, i64, vp, i32, i32, i32, vp, vp, i32, i64, vp, i64, i64, vp]),
    "mhmoe_ep_row_bytes": (i64, [i32, i32]),
    "mhmoe_ep_dest": (i32, [vp, i32, i32, i32, i32, i32, vp, vp, vp]),
    "mhmoe_ep_pack": (i32, [vp, vp, vp, i32, i32, i32, vp, vp, i32, i32, i32, vp, vp, i64, vp, vp]),
    "mhmoe_ep_unpack": (i32, [vp, i64, i32, i32, i32, vp, vp, vp, vp]),
    "mhmoe_quantize_rows_nvfp4": (i32, [vp, i64, i64, i32, vp, vp, vp, vp]),
    "mhmoe_gemm_nvfp4_raw": (i32, [vp, vp, i32, vp, vp, vp, i32, i32, i32, vp, vp, u64, vp]),
    "mhmoe_wait_selftest": (i32, [vp, i32, i32, u64, vp, vp, vp]),
    "mhmoe_rmsnorm": (i32, [vp, i64, vp, vp, i32, i64, i32, f32, f32, vp, i64, vp]),
    "mhmoe_ffn_nvfp4_atomic": (i32, [vp, i64, i64, i32, i32, i32, i32, i32, i64, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                     vp, vp, i64, i64, vp, u64, vp, vp]),
    "mhmoe_ep_stage_records": (i32, [vp, vp, vp, i32, i32, i32, vp, vp, i32, i32, vp, vp, i32, i32, i64, vp, vp,
                                      vp]),
    "mhmoe_ep_push": (i32, [vp, i32, i32, i32, i64, i32, i32, vp, vp]),
    "mhmoe_ep_sym_bytes": (sz, [i32, i64, i32, i32]),
    "mhmoe_ep_sym_offsets": (i32, [i32, i64, i32, i32, vp]),
    "mhmoe_ep_sym_alloc": (i32, [sz, vp, vp]),
    "mhmoe_ep_sym_open": (i32, [vp, vp]),
    "mhmoe_ep_sym_close": (i32, [vp]),
    "mhmoe_ep_sym_free": (i32, [vp]),
    "mhmoe_ep_send_records": (i32, [vp, vp, vp, i32, i32, i32, vp, vp, i32, i32, vp, vp, i32, i32, i64, vp, vp, vp]),
    "mhmoe_ep_wait": (i32, [vp, i32, i32, i32, u64, vp, vp]),
    "mhmoe_ep_unpack_slots": (i32, [vp, i32, i64, i32, i32, i32, vp, vp, vp, vp]),
    "mhmoe_ep_ffn_return": (i32, [vp, i32, i32, i64, i32, i32, i32, i32, i64, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                  vp, vp, vp, vp, u64, vp, vp]),
    "mhmoe_ep_ffn_stage": (i32, [vp, i32, i32, i64, i32, i32, i32, i32, i64, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                 vp, vp, vp, vp, u64, vp, vp]),
}

_lib = None


def lib() -> C.CDLL:
    """Load libmhmoe.so once; raise loudly if it is not built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"libmhmoe.so not found at {LIB_PATH}; build it with "
                f"`python {_PKG_ROOT / 'build.py'}` (nvcc, sm_100a)")
        h = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


class MHMoEError(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc == MHMOE_OK:
        return
    L = lib()
    msg = f"{what}: {L.mhmoe_status_string(rc).decode()} ({L.mhmoe_last_error().decode()})"
    if rc == MHMOE_ERR_ARGS:
        raise ValueError(msg)
    raise MHMoEError(msg)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("flash_mh_moe (B200) needs CUDA tensors; there is no CPU path")


_status: dict[int, torch.Tensor] = {}


def device_status(device: torch.device) -> torch.Tensor:
    """Per-device int32 word the kernels record device-side failures in."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = t
    return t


def check_device_status(device: torch.device | None = None, reset: bool = True) -> None:
    """Synchronise and raise if a kernel recorded a device-side failure."""
    devs = [device] if device is not None else [torch.device("cuda", i) for i in list(_status)]
    for d in devs:
        t = device_status(d)
        v = int(t.item())
        if v != 0:
            if reset:
                t.zero_()
            check(v, f"device status on {d}")
