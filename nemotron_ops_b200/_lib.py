"""ctypes binding of libbolt_b200.so (the C ABI declared in include/bolt_b200.h)."""
from __future__ import annotations

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libbolt_b200.so")

_P = ctypes.c_void_p
_S = ctypes.POINTER(ctypes.c_int64)
_I = ctypes.c_int
_L = ctypes.c_int64
_F = ctypes.c_float

# name -> (restype, argtypes); kept in the order of include/bolt_b200.h
SIGNATURES = {
    "bolt_last_error": (ctypes.c_char_p, []),
    "bolt_abi_version": (_I, []),
    "bolt_set_launch_options": (_I, [_I, _I, _L]),
    "bolt_get_device_status": (_I, [ctypes.POINTER(ctypes.c_uint)]),
    "bolt_nvfp4_gemv": (_I, [_P, _S, _I, _P, _S, _I, _P, _P, _P, _P]),
    "bolt_q8_gemv": (_I, [_P, _S, _I, _P, _S, _I, _P, _P, _P]),
    "bolt_q4_gemv": (_I, [_P, _S, _I, _P, _S, _I, _P, _L, _P, _P]),
    "bolt_moe_route": (_I, [_P, _S, _I, _P, _S, _I, _P, _L, ctypes.c_float, _P, _P, _P, _P]),
    "bolt_moe_decode": (_I, [_P, _S, _I, _P, _P, _P, _S, _I, _P, _P, _P, _L, _P, _P, _P, _P]),
    "bolt_moe_verify": (_I, [_P, _S, _I, _P, _P, _P, _S, _I, _P, _P, _P, _L, _L, _P, _P, _P, _P, _P]),
    "bolt_moe_verify_noalloc": (_I, [_P, _S, _I, _P, _P, _P, _S, _I, _P, _P, _P, _L, _L, _P, _P]),
    "bolt_moe_verify_shard": (_I, [_P, _S, _I, _P, _P, _P, _S, _I, _P, _P, _P, _L, _L, _L, _L, _P, _P, _P, _P, _P,
                                   _P]),
    "bolt_moe_verify_shard_allreduce": (_I, [_P, _S, _I, _P, _P, _P, _S, _I, _P, _P, _P, _L, _L, _L, _L, _P, _P, _P,
                                             _P, _P, _L, _L, _L, _P, _P]),
    "bolt_moe_decode_shard": (_I, [_P, _S, _I, _P, _P, _P, _S, _I, _P, _P, _P, _L, _L, _L, _P, _P, _P, _P, _P]),
    "bolt_mamba_step": (_I, [_P, _S, _I, _P, _S, _I, _P, _S, _I, _P, _P, _P, _P, _P, _P, _L, _L, _L, _L, _F, _F,
                             _P, _P, _P, _P, _P, _P]),
    "bolt_mamba_verify": (_I, [_P, _S, _I, _P, _S, _I, _P, _S, _I, _P, _P, _P, _P, _P, _P, _P, _L, _L, _L, _L, _F,
                               _F, _P, _P, _P, _P, _P, _P]),
    "bolt_relu2": (_I, [_P, _S, _I, _P, _P]),
    "bolt_f32_to_bf16": (_I, [_P, _P, _L, _P]),
    "bolt_memcpy_async": (_I, [_P, _P, _L, _P]),
    "bolt_dequant": (_I, [_I, _I, _P, _P, _L, _L, _P, _P]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load libbolt_b200.so (built in-tree by ``python -m nemotron_ops_b200.build``)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m nemotron_ops_b200.build`")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().bolt_last_error()
    return msg.decode() if msg else ""


_SHAPES: dict = {}


def shape_arg(shape):
    """(int64_t* view, owning array) for a shape.  Shapes repeat from call to call, so the
    read-only arrays are cached (building one costs several microseconds per call)."""
    key = tuple(int(s) for s in shape)
    hit = _SHAPES.get(key)
    if hit is None:
        arr = (ctypes.c_int64 * max(1, len(key)))(*key)
        hit = (ctypes.cast(arr, _S), arr)
        if len(_SHAPES) < 4096:
            _SHAPES[key] = hit
    return hit
