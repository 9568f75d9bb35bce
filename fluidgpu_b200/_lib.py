"""ctypes binding of libfgb200.so (declared in include/fgb200.h).

This is the reference-facing C ABI: plain pointers, sizes and a CUDA stream
handle. There is no fallback: if the library is missing or fails to load,
`lib()` raises, and every GPU op in this package fails with it.
"""
from __future__ import annotations

import ctypes
import os
import threading
from ctypes import c_float, c_int, c_size_t, c_uint, c_void_p
from pathlib import Path

from .build import LIB_PATH

_P = c_void_p
_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

FG_OK = 0
FG_ERR_ARG = 1
FG_ERR_CUDA = 2
FG_ERR_TIMEOUT = 3
FG_ERR_PEER = 4

FG_EPI_STORE = 0
FG_EPI_RESIDUAL = 1
FG_EPI_SWIGLU = 2
FG_EPI_SWIGLU_OAI = 3
FG_EPI_F32 = 4

FG_NORM_LLAMA = 0
FG_NORM_FP32MUL = 1

FG_ROUTE_SPLIT = 1
FG_ROUTE_BROADCAST = 2

# name -> (restype, argtypes); every symbol include/fgb200.h declares
SIGNATURES: dict[str, tuple] = {
    "fg_last_error": (ctypes.c_char_p, []),
    "fg_version": (c_int, []),
    "fg_launch_count": (ctypes.c_ulonglong, []),
    "fg_device_status": (c_int, [ctypes.POINTER(c_uint), c_int, _P]),
    "fg_embed": (c_int, [_P, _P, _P, c_int, c_int, c_int, _P]),
    "fg_rmsnorm": (c_int, [_P, _P, _P, c_int, c_int, c_float, c_int, _P]),
    "fg_gemm_bf16": (c_int, [_P, _P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, _P, c_size_t, _P]),
    "fg_gemm_bf16_packed": (c_int, [_P, _P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, _P, c_size_t, _P]),
    "fg_gemm_bf16_packed_routed": (
        c_int,
        [_P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, _P, c_int, c_int, c_int, _P, c_int, _P, c_uint,
         c_uint, _P, _P],
    ),
    "fg_pack_weight_bf16": (c_int, [_P, _P, c_int, c_int, _P]),
    "fg_packed_weight_bytes": (c_size_t, [c_int, c_int]),
    "fg_gemm_grid": (c_int, [c_int, c_int, c_int, c_int]),
    "fg_gemm_split": (c_int, [c_int, c_int, c_int, c_int]),
    "fg_gemm_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "fg_rope_kv_append": (
        c_int,
        [_P, _P, _P, c_float, _P, c_int, c_int, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, _P],
    ),
    "fg_rope_kv_append_tokens": (
        c_int,
        [_P, _P, _P, _P, c_float, _P, c_int, c_int, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, _P],
    ),
    "fg_prefill_attn": (
        c_int,
        [_P, _P, _P, _P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
         c_float, _P],
    ),
    "fg_kv_append": (
        c_int, [_P, _P, _P, _P, _P, c_int, c_int, _P, _P, c_int, c_int, c_int, c_int, _P],
    ),
    "fg_paged_decode_attn": (
        c_int,
        [_P, _P, _P, _P, _P, _P, _P, _P, c_size_t, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
         c_int, c_int, c_float, _P],
    ),
    "fg_paged_decode_attn_noalloc": (
        c_int,
        [_P, _P, _P, _P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
         c_float, _P],
    ),
    "fg_attn_splits": (c_int, [c_int, c_int, c_int, c_int, c_int]),
    "fg_attn_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "fg_argmax": (c_int, [_P, _P, c_int, c_int, _P]),
    "fg_moe_router_topk": (c_int, [_P, _P, _P, c_int, c_int, c_int, c_int, _P, _P, _P, _P]),
    "fg_moe_topk_softmax": (c_int, [_P, c_int, c_int, c_int, _P, _P, _P]),
    "fg_moe_tile_tokens": (c_int, [c_int, c_int, c_int]),
    "fg_moe_max_items": (c_int, [c_int, c_int, c_int, c_int]),
    "fg_moe_permute": (c_int, [_P, c_int, c_int, c_int, c_int, c_int, c_int, _P, _P, _P, _P, _P, _P]),
    "fg_moe_gather": (c_int, [_P, _P, c_int, c_int, c_int, _P, _P]),
    "fg_pack_mxfp4": (c_int, [_P, _P, _P, c_int, c_int, c_int, _P]),
    "fg_mxfp4_packed_bytes": (c_size_t, [c_int, c_int, c_int]),
    "fg_moe_gemm_mxfp4": (
        c_int, [_P, _P, _P, _P, _P, _P, c_int, _P, c_int, c_int, c_int, c_int, c_int, c_int, _P],
    ),
    "fg_moe_unpermute": (c_int, [_P, _P, _P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, c_int, _P]),
    "fg_advance": (c_int, [_P, _P, c_int, _P]),
    "fg_add_bf16": (c_int, [_P, _P, _P, ctypes.c_longlong, _P]),
    "fg_sum_partials": (c_int, [_P, c_int, ctypes.c_longlong, _P, _P]),
    "fg_mailbox_bytes": (c_size_t, [c_int, c_int, c_size_t]),
    "fg_ipc_export": (c_int, [_P, _P, ctypes.POINTER(c_size_t)]),
    "fg_ipc_import": (c_int, [_P, c_size_t, ctypes.POINTER(c_void_p)]),
    "fg_ipc_close": (c_int, [_P, c_size_t]),
    "fg_handoff_put": (c_int, [_P, c_size_t, _P, _P, c_int, c_int, c_int, c_int, c_size_t, c_int, _P]),
    "fg_handoff_recv": (c_int, [_P, c_size_t, _P, _P, c_int, c_int, c_int, c_int, c_size_t, c_int, _P]),
    "fg_mailbox_slot": (_P, [_P, c_int, c_int, c_size_t, c_int, c_int]),
    "fg_handoff_signal": (c_int, [_P, _P, c_int, c_int, c_int, c_size_t, _P]),
    "fg_handoff_wait": (c_int, [_P, c_int, c_int, c_int, c_size_t, c_int, _P]),
    "fg_rmsnorm_wait": (
        c_int, [_P, _P, _P, c_int, c_int, c_float, c_int, _P, c_int, c_int, _P, c_uint, c_uint, c_int, _P],
    ),
    "fg_rmsnorm_gather_wait": (
        c_int,
        [_P, c_int, c_int, _P, _P, _P, c_int, c_int, c_float, c_int, _P, c_int, c_int, _P, c_uint, c_uint, c_int,
         _P],
    ),
    "fg_sum_rmsnorm_wait": (
        c_int,
        [_P, c_int, _P, _P, _P, c_int, c_int, c_float, c_int, _P, c_int, _P, c_uint, c_uint, c_int, _P],
    ),
    "fg_counter_add": (c_int, [_P, c_uint, _P]),
    "fg_preload": (c_int, []),
}


def ptr_array(ptrs) -> ctypes.Array:
    """A C array of void* (the pointer-array arguments of the routed hand-off
    entry points); keep it alive for the duration of the call."""
    arr = (c_void_p * max(len(ptrs), 1))()
    for i, p in enumerate(ptrs):
        arr[i] = p
    return arr


def lib_path() -> Path:
    override = os.environ.get("FGB200_LIB")
    return Path(override) if override else LIB_PATH


def lib() -> ctypes.CDLL:
    """Load (once) and return the C library with typed entry points."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if not path.exists():
            raise RuntimeError(
                f"fgb200 CUDA library not found at {path}; build it with "
                "`python -m fluidgpu_b200.build` (nvcc, sm_100a)"
            )
        handle = ctypes.CDLL(str(path))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
    return _lib


class FgError(RuntimeError):
    """A C entry point returned a nonzero status."""

    def __init__(self, name: str, code: int, text: str) -> None:
        super().__init__(f"{name} failed with status {code}: {text}")
        self.code = code


def call(name: str, *args) -> int:
    """Call `name` and raise FgError on a nonzero status."""
    handle = lib()
    rc = getattr(handle, name)(*args)
    if rc != FG_OK:
        text = handle.fg_last_error()
        raise FgError(name, rc, text.decode() if text else "")
    return rc
