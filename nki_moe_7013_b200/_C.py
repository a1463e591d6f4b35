"""ctypes binding of the C ABI in include/qmoe.h (library ``_lib/libqmoe.so``).

The library must have been built (``python -m nki_moe_7013_b200.build`` or
``__graft_entry__.build()``); if it is missing this module raises -- there is
no fallback implementation.
"""
from __future__ import annotations

import ctypes
import os
import re
import threading

from .build import HEADER, LIB_PATH

_lock = threading.Lock()
_lib = None

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int
SZ = ctypes.c_size_t

# name -> (restype, argtypes)
_SIGNATURES = {
    "qmoe_version": (I32, []),
    "qmoe_status_string": (ctypes.c_char_p, [I32]),
    "qmoe_last_error": (ctypes.c_char_p, []),
    "qmoe_device_error": (I32, [I32, ctypes.POINTER(ctypes.c_uint)]),
    "qmoe_router_topk": (I32, [P, P, P, I64, I64, I64, I64, I32, P, P, P, P, P]),
    "qmoe_max_tiles": (I64, [I64, I64]),
    "qmoe_moe_permute": (I32, [P, P, P, P, I64, I64, I64, I64, P, P, P, P, P, P, P, P, P, I64, P]),
    "qmoe_route_permute": (I32, [P, P, P, I64, I64, I64, I64, I32, P, P, P, P, P, P, P, P, P, P, P, P, I64, P, P]),
    "qmoe_moe_experts": (I32, [P, I64, P, P, P, P, I64, P, P, I64, I64, I64, I64, P, P, I64, P, P]),
    "qmoe_grouped_gemm_gateup_split_workspace_size": (SZ, []),
    "qmoe_route_small": (I32, [P, P, P, I64, I64, I64, I64, I32, P, P, P, P, P, P, P, P, P, P, P]),
    "qmoe_grouped_gemm_gateup_swiglu": (I32, [P, I64, P, P, P, I64, I64, I64, I64, I64, I64, P, P, SZ, P]),
    "qmoe_grouped_gemm_down_combine": (I32, [P, P, P, I64, I64, I64, P, P, I64, I64, I64, I64, P, I64, P]),
    "qmoe_blockwise_max_tiles": (I64, [I64, I64]),
    "qmoe_blockwise_prepare": (I32, [P, P, I64, P, P, I64, I64, I64, I64, I64, P, P, P, P, P]),
    "qmoe_combine_finalize": (I32, [P, P, I64, I64, P, P]),
    "qmoe_embedding_gather": (I32, [P, I64, I64, P, I64, P, P]),
    "qmoe_masked_residual_add": (I32, [P, P, P, I64, I64, P, P]),
    "qmoe_greedy_pick": (I32, [P, I64, I64, P, P, P, P]),
    "qmoe_select_affinities": (I32, [P, P, I64, I64, I64, I64, P, P]),
    "qmoe_moe_forward_workspace_size": (SZ, [I64, I64, I64, I64, I64]),
    "qmoe_moe_forward": (I32, [P, P, P, P, P, P, I64, I64, I64, I64, I64, I32, P, P, P, P, SZ, P]),
    "qmoe_moe_block_forward_workspace_size": (SZ, [I64, I64, I64, I64, I64]),
    "qmoe_moe_block_forward": (I32, [P, P, P, ctypes.c_float, P, P, P, P, I64, I64, I64, I64, I64, I32, P, P, P,
                                     P, P, P, SZ, P]),
    "qmoe_linear": (I32, [P, P, I64, I64, I64, P, P, SZ, P]),
    "qmoe_rmsnorm": (I32, [P, I32, P, P, I64, I64, ctypes.c_float, P, I32, P, P]),
    "qmoe_qk_norm_rope": (I32, [P, P, P, P, P, P, I64, I64, I64, I64, ctypes.c_float, P, P, P, I64,
                                I64, P]),
    "qmoe_attention_prefill": (I32, [P, P, P, P, P, P, I64, I64, I64, I64, I64, I64, I64,
                                     ctypes.c_float, P, P]),
    "qmoe_attention_decode_splits": (I64, [I64, I64, I64]),
    "qmoe_attention_decode_workspace_size": (SZ, [I64, I64, I64]),
    "qmoe_attention_decode": (I32, [P, P, P, P, P, P, I64, I64, I64, I64, I64, I64, I64, I64,
                                    ctypes.c_float, P, P, SZ, P]),
    "qmoe_routing_histogram": (I32, [P, I64, I64, I64, P, P]),
    "qmoe_ep_pack": (I32, [P, P, P, I64, I64, I64, I64, I64, P, P, P, P, P, P, P]),
    "qmoe_ep_unpack": (I32, [P, P, P, I64, I64, I64, I64, P, P]),
    "qmoe_ipc_export": (I32, [P, P, ctypes.POINTER(ctypes.c_int64)]),
    "qmoe_ipc_import": (I32, [P, I64, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p)]),
    "qmoe_ipc_close": (I32, [P]),
    "qmoe_ep_ctrl_words": (I64, [I64, I64]),
    "qmoe_ep_exchange_counts": (I32, [P, P, P, I64, I64, I64, I64, I64, I64, P, P, I64, P, I64, P, I64, P]),
    "qmoe_moe_experts_return": (I32, [P, P, P, P, I64, P, P, I64, I64, I64, I64, I64, I64, I64, P, P, P]),
    "qmoe_ep_dispatch": (I32, [P, P, P, P, P, P, P, P, I64, I64, I64, I64, I64, I64, I64, I64, I64, P]),
    "qmoe_ep_wait_expand": (I32, [P, P, I64, I64, I64, I64, I64, P, I64, P, P, P, I64, I64, P]),
    "qmoe_ep_wait_unpack": (I32, [P, P, I64, I64, I64, I64, I64, P, P, I64, I64, I64, P, P]),
    "qmoe_ep_signal_wait": (I32, [P, P, I64, I64, I64, I64, I64, I64, P]),
    "qmoe_grouped_gemm_down_return": (I32, [P, P, P, I64, P, P, I64, I64, I64, I64, I64, I64, I64, P]),
    "qmoe_moe_forward_noalloc": (I32, [P, P, P, P, P, P, I64, I64, I64, I64, I64, I32, P, P, P, P]),
}


class QmoeError(RuntimeError):
    """A qmoe C-ABI call returned a non-zero status."""

    def __init__(self, what: str, status: int, detail: str):
        super().__init__(f"{what}: {detail or 'status ' + str(status)} (status {status})")
        self.status = status
        self.detail = detail


def header_symbols(header: str = HEADER):
    """Every function the public header declares."""
    text = open(header).read()
    return sorted(set(re.findall(r"QMOE_API\s+[\w\s\*]+?\b(qmoe_\w+)\s*\(", text)))


def lib():
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"qmoe CUDA library not built ({LIB_PATH} missing); run "
                    "`python -m nki_moe_7013_b200.build` -- there is no CPU fallback")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                f = getattr(handle, name)
                f.restype = res
                f.argtypes = args
            _lib = handle
    return _lib


def last_error() -> str:
    return (lib().qmoe_last_error() or b"").decode()


def check(status: int, what: str) -> None:
    if status != 0:
        raise QmoeError(what, status, last_error())


def device_error(clear: bool = True) -> int:
    code = ctypes.c_uint(0)
    check(lib().qmoe_device_error(1 if clear else 0, ctypes.byref(code)), "qmoe_device_error")
    return int(code.value)
