"""ctypes binding of the C ABI in include/nibble_cuda.h (libnibble_cuda.so, built in-tree).

This module is plumbing for Python callers (tests, bench, smoke): every call goes through the C ABI into the
sm_100a kernels. There is no CPU fallback: the library is loaded on first use, and a missing or unloadable
library raises ImportError there.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libnibble_cuda.so")

NBL_OK, NBL_E_INVALID, NBL_E_CUDA, NBL_E_NOMEM, NBL_E_UNSUPPORTED, NBL_E_DEVICE = range(6)
F32, F16, BF16, Q4_0, Q5_0, Q8_0, Q5_1, Q4_K, Q5_K, Q6_K = 0, 1, 2, 3, 4, 5, 6, 7, 8, 9
STATUS_NAMES = {0: "NBL_OK", 1: "NBL_E_INVALID", 2: "NBL_E_CUDA", 3: "NBL_E_NOMEM", 4: "NBL_E_UNSUPPORTED",
                5: "NBL_E_DEVICE"}


class NibbleError(RuntimeError):
    """A non-zero nbl_status, carrying nbl_last_error()'s message (the C-side nibble::Error)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class RopeParams(C.Structure):
    _fields_ = [("freq_base", C.c_float), ("neox", C.c_int32), ("freq_factors", C.c_void_p)]


class KvConfig(C.Structure):
    _fields_ = [("n_pages", C.c_int64), ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32),
                ("page_size", C.c_int32), ("dtype", C.c_int32)]


_P = C.c_void_p
_I32 = C.c_int32
_I64 = C.c_int64

# name -> argtypes (all return int status unless listed in _RESTYPES)
SIGNATURES = {
    "nbl_abi_version": [],
    "nbl_last_error": [C.c_char_p, C.c_size_t],
    "nbl_ctx_create": [C.c_int, C.POINTER(_P)],
    "nbl_ctx_destroy": [_P],
    "nbl_ctx_set_stream": [_P, _P],
    "nbl_ctx_use_own_stream": [_P],
    "nbl_ctx_stream": [_P],
    "nbl_ctx_sync": [_P],
    "nbl_ctx_check": [_P],
    "nbl_ctx_set_paged_kv": [_P, _I32],
    "nbl_reserve": [_P, _I64, _I64, _I64, _I64],
    "nbl_alloc": [_P, _I64, C.POINTER(_P)],
    "nbl_free": [_P, _P],
    "nbl_read": [_P, _P, _P, _I64],
    "nbl_write": [_P, _P, _P, _I64],
    "nbl_add_bias": [_P, _P, _P, _I64, _I64],
    "nbl_rope": [_P, _P, _I64, _I64, _I64, _I64, C.POINTER(RopeParams)],
    "nbl_attention": [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64],
    "nbl_kv_create": [_P, C.POINTER(KvConfig), C.POINTER(_P)],
    "nbl_kv_destroy": [_P],
    "nbl_kv_pool": [_P, C.POINTER(_P), C.POINTER(_I64)],
    "nbl_rope_kv_append": [_P, _P, _P, _P, _P, _I32, _P, _P, _P, _P, _I32, _P, _P, _P, _I32, _I64, _I32,
                           C.POINTER(RopeParams)],
    "nbl_attn_decode": [_P, _P, _P, _P, _I32, _P, _I32, _I32, _I32, _P, _P, _I32],
    "nbl_attn_decode_static": [_P, _P, _P, _P, _I32, _P, _I32, _I32, _I32, _P, _P, _I32],
    "nbl_decode_step_host": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I32, _P, _I32, _I32, _I32, C.POINTER(RopeParams),
                             _P, _I32],
    "nbl_attn_prefill": [_P, _P, _P, _I32, _I64, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _P, _I32],
    "nbl_lse_merge": [_P, _P, _P, _I32, _I64, _I32, _P, _P],
    "nbl_lse_merge_packed": [_P, _P, _I32, _I64, _I32, _P, _P],
    "nbl_weight_create": [_P, _P, _I32, _I64, _I64, C.POINTER(_P)],
    "nbl_weight_destroy": [_P],
    "nbl_weight_data": [_P, C.POINTER(_P), C.POINTER(_I32), C.POINTER(_I64), C.POINTER(_I64)],
    "nbl_embed": [_P, _P, _P, _I64, _P],
    "nbl_matmul": [_P, _P, _P, _P, _I64],
    "nbl_matmul_multi": [_P, _P, _I32, _P, _P, _I64],
    "nbl_rmsnorm": [_P, _P, _P, _P, _I64, C.c_float],
    "nbl_add": [_P, _P, _P, _I64],
    "nbl_copy": [_P, _P, _P, _I64],
    "nbl_silu_mul": [_P, _P, _P, _I64],
    "nbl_selftest_bounded_wait": [_P, _I64],
    "nbl_lse_exchange_peers": [_P, _P, _I64, _I32, _I32, _I32, _P, _P, _P, _P, _P],
    "nbl_attn_decode_peers": [_P, _P, _P, _P, _I32, _P, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _P],
}
_RESTYPES = {"nbl_last_error": C.c_size_t, "nbl_ctx_stream": _P}


def _load() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m nibble_b200.build` (nvcc, sm_100a)")
    lib = C.CDLL(LIB_PATH)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, C.c_int)
    return lib


_lib = None


def get_lib() -> C.CDLL:
    """The loaded library (loaded on first use, so the build step can import this package without it)."""
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


def __getattr__(name):
    if name == "lib":
        return get_lib()
    raise AttributeError(name)


def last_error() -> str:
    lib = get_lib()
    n = lib.nbl_last_error(None, 0)
    buf = C.create_string_buffer(n + 1)
    lib.nbl_last_error(buf, n + 1)
    return buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status != NBL_OK:
        raise NibbleError(status, last_error())
