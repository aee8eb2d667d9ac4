"""ctypes binding of ``libexq_b200.so`` (the C ABI declared in include/exq_b200.h).

There is no fallback: if the library is missing or fails to load, every entry
point raises.  Tensors cross the boundary as raw device pointers plus dtype
tags; the stream is torch's current CUDA stream.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libexq_b200.so"

# include/exq_b200.h constants
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_WORKSPACE = 0, -1, -2, -3, -4
F16, BF16, F32, I32, I64, U8, I8 = 0, 1, 2, 3, 4, 5, 6
TIER_BF16, TIER_INT8, TIER_INT4, TIER_NONE = 0, 1, 2, -1
DEV_BAD_EXPERT_ID, DEV_BAD_SLOT, DEV_BAD_TIER, DEV_TIMEOUT = 1, 2, 4, 8

_DTYPE_TAG = {
    torch.float16: F16,
    torch.bfloat16: BF16,
    torch.float32: F32,
    torch.int32: I32,
    torch.int64: I64,
    torch.uint8: U8,
    torch.int8: I8,
}

vp, i32, i64, sz = C.c_void_p, C.c_int32, C.c_int64, C.c_size_t

# name -> (restype, argtypes)
SIGNATURES = {
    "exq_abi_version": (C.c_int, []),
    "exq_last_error": (C.c_char_p, []),
    "exq_status_string": (C.c_char_p, [C.c_int]),
    "exq_read_device_status": (C.c_int, [C.POINTER(C.c_uint32), C.c_int, vp]),
    "exq_moe_align_block_size": (C.c_int, [vp, C.c_int, i64, i32, i32, vp, i64, vp, i64, vp, vp,
                                           i32, vp]),
    "exq_build_ends_from_slots": (C.c_int, [vp, i64, vp, i64, i32, vp, vp, vp]),
    "exq_dispatch": (C.c_int, [vp, C.c_int, i64, i32, vp, vp, vp, vp]),
    "exq_gather_hidden": (C.c_int, [vp, C.c_int, i64, i64, i64, vp, i64, i32, vp, vp]),
    "exq_combine_workspace_bytes": (sz, [i64]),
    "exq_combine": (C.c_int, [vp, C.c_int, i64, i64, vp, vp, C.c_int, i64, i32, vp, C.c_int, vp,
                              sz, vp]),
    "exq_ep_pack": (C.c_int, [vp, C.c_int, i64, i32, i32, i32, vp, C.c_int, i64, vp, vp, vp, vp,
                              vp]),
    "exq_ep_combine": (C.c_int, [vp, C.c_int, vp, vp, C.c_int, i64, i32, i64, vp, vp, vp]),
    "exq_ep_buffer_bytes": (sz, [i32, i64, i64]),
    "exq_ep_set_wait_timeout": (C.c_int, [C.c_uint64]),
    "exq_ep_buffer_init": (C.c_int, [vp, i32, i64, i64, vp]),
    "exq_ep_ipc_alloc": (C.c_int, [sz, C.POINTER(C.c_void_p), vp]),
    "exq_ep_ipc_free": (C.c_int, [vp]),
    "exq_ep_ipc_open": (C.c_int, [vp, C.POINTER(C.c_void_p)]),
    "exq_ep_ipc_close": (C.c_int, [vp]),
    "exq_ep_dispatch": (C.c_int, [vp, C.c_int, i64, i32, i32, i32, i32, vp, C.c_int, i64, i64, vp,
                                  vp, vp]),
    "exq_ep_expert_forward": (C.c_int, [vp, C.c_int, i32, i32, i64, vp, vp, vp, sz, vp]),
    "exq_ep_expert_forward_shared": (C.c_int, [vp, C.c_int, i32, i32, i64, vp, vp, vp, i64, i32,
                                               vp, vp, sz, vp]),
    "exq_ep_combine_peer": (C.c_int, [vp, i32, i64, i64, C.c_int, vp, vp, C.c_int, i64, i32, vp,
                                      vp, vp]),
    "exq_combine_noalloc": (C.c_int, [vp, C.c_int, i64, i64, vp, vp, C.c_int, i64, i32, vp,
                                      C.c_int, vp]),
    "exq_silu_and_mul": (C.c_int, [vp, vp, C.c_int, i64, i64, vp]),
    "exq_router_topk": (C.c_int, [vp, C.c_int, i64, i32, i32, i32, vp, vp, vp]),
    "exq_pack_int4": (C.c_int, [vp, C.c_int, i64, i64, i32, vp, vp, vp]),
    "exq_quant_int8": (C.c_int, [vp, C.c_int, i64, i64, vp, vp, vp]),
    "exq_moe_gemm_workspace_bytes": (sz, [i64, i32, i32]),
    "exq_moe_gemm": (C.c_int, [vp, i32, i64, i64, vp, C.c_int, i64, vp, C.c_int, i32, vp, C.c_int,
                               vp, vp, vp, sz, vp]),
    "exq_moe_layer_workspace_bytes": (sz, [i64, i32, i32, i32, i64, i64]),
    "exq_moe_layer_forward": (C.c_int, [vp, vp, C.c_int, i64, vp, C.c_int, vp, C.c_int, i32, vp,
                                        vp, sz, vp]),
    "exq_moe_layer_forward_range": (C.c_int, [vp, vp, C.c_int, i64, vp, C.c_int, vp, C.c_int, i32,
                                              vp, vp, sz, vp, i32, i32]),
    "exq_moe_layer_from_logits_workspace_bytes": (sz, [i64, i32, i32, i32, i64, i64]),
    "exq_moe_layer_forward_from_logits": (C.c_int, [vp, vp, C.c_int, i64, vp, C.c_int, i32, i32,
                                                    vp, vp, sz, vp]),
}

_lock = threading.Lock()
_lib = None


class ExqError(RuntimeError):
    """A nonzero status from the C ABI."""

    def __init__(self, what: str, status: int, msg: str):
        super().__init__(f"{what}: {msg} (status {status})")
        self.status = status


def lib() -> C.CDLL:
    """Load the library once; raises if it is missing (no fallback path)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m exq_b200.build` "
                    "(exq_b200 has no CPU fallback)")
            handle = C.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    if status != OK:
        msg = lib().exq_last_error().decode(errors="replace")
        if status == ERR_INVALID:
            raise ValueError(f"{what}: {msg}")
        if status == ERR_UNSUPPORTED:
            raise NotImplementedError(f"{what}: {msg}")
        raise ExqError(what, status, msg)


def tag(t: torch.Tensor) -> int:
    try:
        return _DTYPE_TAG[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("exq_b200 runs on CUDA tensors only (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all tensors must be on the same CUDA device")
    return dev


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Scratch from torch's caching allocator (never on the library's side)."""
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def read_device_status(device: torch.device | None = None, clear: bool = True) -> int:
    """Synchronously read (and clear) the device status word (EXQ_DEV_* bits)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    out = C.c_uint32(0)
    with torch.cuda.device(device):
        check(lib().exq_read_device_status(C.byref(out), int(clear), stream_of(device)),
              "read_device_status")
    return int(out.value)


def set_ep_wait_timeout(ns: int = 0) -> None:
    """Limit of the expert-parallel kernels' waits on other ranks, in
    nanoseconds, for launches made after this call (0: the 5 s default)."""
    check(lib().exq_ep_set_wait_timeout(int(ns)), "ep_set_wait_timeout")


def exported_symbols() -> list[str]:
    return sorted(SIGNATURES)


def header_declarations(header: str | os.PathLike | None = None) -> list[str]:
    """Names of the functions ``include/exq_b200.h`` declares."""
    import re
    path = Path(header) if header else Path(__file__).resolve().parent.parent / "include" / "exq_b200.h"
    return sorted(set(re.findall(r"EXQ_API\s+[\w\s\*]*?\b(exq_\w+)\s*\(", path.read_text())))
