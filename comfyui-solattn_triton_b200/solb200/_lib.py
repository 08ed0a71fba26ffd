"""ctypes binding of libsolb200.so (the C ABI in include/solb200.h).

The library is loaded from this package's folder. There is no fallback: if it is
missing or the process has no sm_100 device, the ops raise.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_float, c_int32, c_int64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libsolb200.so"

OK = 0
STATUS = {
    0: "ok", 1: "invalid argument", 2: "alignment", 3: "workspace", 4: "cuda error",
    5: "unsupported device", 6: "device-side wait timed out",
}

# enum solb200_buffer
BUF = dict(error=0, kc=1, vc=2, centroid=3, kmean=4, kvar=5, thr=6, mask=7, count=8, vamax=9,
           vscale=10, qi=11, qs=12, ki=13, ks=14, vi=15, order=16)
STAGES_ALL, STAGES_PREPARE, STAGES_FORWARD = 0, 1, 2
STAGES_POOL, STAGES_QUANT, STAGES_ROUTE = 3, 4, 5   # PREPARE in parts (per-stage timing)

_lib = None

I64x3 = c_int64 * 3
I64x2 = c_int64 * 2

_SIGS = {
    "solb200_last_error": (ctypes.c_char_p, []),
    "solb200_abi_version": (c_int32, []),
    "solb200_workspace_bytes": (c_int32, [c_int64, c_int64, c_int64, c_int64, c_int32, c_int32,
                                          POINTER(c_int64)]),
    "solb200_workspace_offset": (c_int32, [c_int64, c_int64, c_int64, c_int64, c_int32, c_int32, c_int32,
                                           POINTER(c_int64)]),
    "solb200_sol_attn_bf16": (c_int32, [c_void_p, POINTER(c_int64), c_void_p, POINTER(c_int64), c_void_p,
                                        POINTER(c_int64), c_void_p, c_int64, c_int64, c_int64, c_int64,
                                        c_int32, c_float, c_float, POINTER(c_int64), POINTER(c_int64),
                                        c_int32, c_void_p, c_int64, c_void_p, c_void_p, c_void_p]),
    "solb200_sol_attn_int8": (c_int32, [c_void_p, POINTER(c_int64), c_void_p, POINTER(c_int64), c_void_p,
                                        POINTER(c_int64), c_void_p, c_int64, c_int64, c_int64, c_int64,
                                        c_int32, c_float, c_float, POINTER(c_int64), POINTER(c_int64),
                                        c_int32, c_int32, c_void_p, c_int64, c_void_p, c_void_p, c_void_p]),
    "solb200_sol_attn_bf16_noalloc": (c_int32, [c_void_p, POINTER(c_int64), c_void_p, POINTER(c_int64),
                                                c_void_p, POINTER(c_int64), c_void_p, c_int64, c_int64,
                                                c_int64, c_int64, c_int32, c_float, c_float,
                                                POINTER(c_int64), POINTER(c_int64), c_void_p]),
    "solb200_read_device_error": (c_int32, [c_void_p, POINTER(c_int32), c_void_p]),
    "solb200_noalloc_read_device_error": (c_int32, [POINTER(c_int32), c_void_p]),
    "solb200_debug_set_wait": (c_int32, [c_int64, c_int32]),
    "solb200_attn_dense": (c_int32, [c_void_p, POINTER(c_int64), c_void_p, POINTER(c_int64), c_void_p,
                                     POINTER(c_int64), c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64,
                                     c_float, c_void_p, c_int64, c_void_p]),
    "solb200_attn_dense_masked": (c_int32, [c_void_p, POINTER(c_int64), c_void_p, POINTER(c_int64), c_void_p,
                                            POINTER(c_int64), c_void_p, c_int32, POINTER(c_int64), c_void_p,
                                            c_int64, c_int64, c_int64, c_int64, c_int64, c_float, c_void_p,
                                            c_int64, c_void_p]),
    "solb200_workspace_bytes_reordered": (c_int32, [c_int64, c_int64, c_int64, c_int64, c_int32, c_int32,
                                                    c_int32, POINTER(c_int64)]),
    "solb200_sol_attn_reordered": (c_int32, [c_void_p, POINTER(c_int64), c_void_p, POINTER(c_int64), c_void_p,
                                             POINTER(c_int64), c_void_p, c_int64, c_int64, c_int64, c_int64,
                                             c_int32, c_float, c_float, POINTER(c_int64), POINTER(c_int64),
                                             c_void_p, c_int32, c_int32, c_void_p, c_int64, c_void_p]),
    "solb200_morton_perm": (c_int32, [c_int64, c_int64, c_int64, c_int32, c_int64, c_void_p, c_void_p,
                                      c_void_p]),
    "solb200_copy_heads": (c_int32, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64,
                                     c_int32, c_void_p]),
    "solb200_selftest_quotient": (c_int32, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p]),
    "solb200_gather_rows": (c_int32, [POINTER(c_void_p), POINTER(c_void_p), c_int32, c_void_p, c_int64,
                                      c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p]),
}


def lib():
    """The loaded library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"solb200: {LIB_PATH} is missing; build it with "
                "`python comfyui-solattn_triton_b200/csrc/build.py`")
        handle = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_LOCAL if hasattr(os, "RTLD_LOCAL") else 0)
        for name, (res, args) in _SIGS.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def exported_symbols():
    return list(_SIGS)


def last_error() -> str:
    msg = lib().solb200_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str):
    if rc != OK:
        raise RuntimeError(f"solb200 {what} failed ({STATUS.get(rc, rc)}): {last_error()}")
