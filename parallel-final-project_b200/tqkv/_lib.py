"""ctypes binding of libtqkv_b200.so (the C ABI in include/tqkv.h).

This module is the Python face of the library for tests and the benchmark.
It loads the in-tree shared library and fails loudly if it is missing: there
is no fallback implementation.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int, c_size_t, c_uint32, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "lib", "libtqkv_b200.so")

TQKV_OK = 0
STATUS_NAMES = {
    0: "TQKV_OK",
    1: "TQKV_ERR_UNSUPPORTED",
    2: "TQKV_ERR_INVALID_SIZE",
    3: "TQKV_ERR_MISALIGNED",
    4: "TQKV_ERR_WORKSPACE",
    5: "TQKV_ERR_CUDA",
    6: "TQKV_ERR_NULL",
}

# C ABI: name -> (restype, argtypes)
C_ABI = {
    "tqkv_status_string": (ctypes.c_char_p, [c_int]),
    "tqkv_last_cuda_error": (c_int, []),
    "tqkv_version": (ctypes.c_char_p, []),
    "tqkv_kv_compress": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "tqkv_kv_reconstruct": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "tqkv_decode_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "tqkv_workspace_init": (c_int, [c_void_p, c_size_t, c_void_p]),
    "tqkv_decode_int8": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                 c_int, c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "tqkv_decode_fp16": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p,
                                 c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "tqkv_decode_int8_partial": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_int, c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "tqkv_lse_combine": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "tqkv_read_device_error": (c_int, [ctypes.POINTER(c_uint32)]),
    "tqkv_decode_int8_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "tqkv_kv_append": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                               c_int, c_int, c_void_p]),
    "tqkv_decode_int8_cache": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_int, c_int, c_int, c_int, c_int, c_int, c_void_p,
                                       c_size_t, c_void_p]),
    "tqkv_exchange_bytes": (c_size_t, [c_int, c_int, c_int]),
    "tqkv_exchange_alloc": (c_int, [c_size_t, ctypes.POINTER(c_void_p)]),
    "tqkv_exchange_free": (c_int, [c_void_p]),
    "tqkv_ipc_get_handle": (c_int, [c_void_p, c_void_p]),
    "tqkv_ipc_open_handle": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "tqkv_ipc_close_handle": (c_int, [c_void_p]),
    "tqkv_decode_int8_publish": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_int, c_int, c_int, c_int, c_int, c_void_p, c_size_t,
                                         ctypes.POINTER(c_void_p), c_int, c_int, c_void_p]),
    "tqkv_exchange_combine": (c_int, [ctypes.POINTER(c_void_p), c_void_p, c_int, c_int, c_int,
                                      c_int, c_void_p]),
    "tqkv_decode_plan": (c_int, [ctypes.c_longlong, c_int, c_int] +
                         [ctypes.POINTER(ctypes.c_longlong)] * 4),
    "tqkv_decode_int8_gqa": (c_int, [c_void_p] * 6 + [c_int] * 6 + [c_void_p, c_size_t,
                                                                     c_void_p]),
    "tqkv_decode_int8_append": (c_int, [c_void_p] * 8 + [c_int] * 7 + [c_void_p, c_size_t,
                                                                        c_void_p]),
    "tqkv_decode_int8_append_publish": (c_int, [c_void_p] * 7 + [c_int] * 7 +
                                        [c_void_p, c_size_t, ctypes.POINTER(c_void_p), c_int,
                                         c_int, c_void_p]),
    "tqkv_decode_int8_exchange": (c_int, [c_void_p] * 6 + [c_int] * 5 +
                                  [c_void_p, c_size_t, ctypes.POINTER(c_void_p), c_int, c_int,
                                   c_void_p]),
    "tqkv_decode_int8_append_exchange": (c_int, [c_void_p] * 8 + [c_int] * 7 +
                                         [c_void_p, c_size_t, ctypes.POINTER(c_void_p), c_int,
                                          c_int, c_void_p]),
}

# The reference's C++ launchers (include/attention.h, include/quantization.h),
# exported with their Itanium-mangled names.
REF_LAUNCHERS = {
    "launch_kv_compress": "_Z18launch_kv_compressPK6__halfPaPS_iiiiiP11CUstream_st",
    "launch_kv_reconstruct": "_Z21launch_kv_reconstructPKaPK6__halfPS1_iiiiiP11CUstream_st",
    "launch_decode_attn_baseline": "_Z27launch_decode_attn_baselinePK6__halfS1_S1_PS_iiiiP11CUstream_st",
    "launch_decode_attn_int8_fused": "_Z29launch_decode_attn_int8_fusedPK6__halfPKaS1_S3_S1_PS_iiiiiP11CUstream_st",
    "launch_decode_attn_int8_fused_online":
        "_Z36launch_decode_attn_int8_fused_onlinePK6__halfPKaS1_S3_S1_PS_iiiiiiiP11CUstream_st",
}
REF_ARGTYPES = {
    "launch_kv_compress": [c_void_p, c_void_p, c_void_p] + [c_int] * 5 + [c_void_p],
    "launch_kv_reconstruct": [c_void_p, c_void_p, c_void_p] + [c_int] * 5 + [c_void_p],
    "launch_decode_attn_baseline": [c_void_p] * 4 + [c_int] * 4 + [c_void_p],
    "launch_decode_attn_int8_fused": [c_void_p] * 6 + [c_int] * 5 + [c_void_p],
    "launch_decode_attn_int8_fused_online": [c_void_p] * 6 + [c_int] * 7 + [c_void_p],
}

_lib = None


class TqkvError(RuntimeError):
    def __init__(self, fn: str, status: int):
        lib = load()
        detail = lib.tqkv_status_string(status).decode()
        extra = ""
        if status == 5:
            extra = f" (cudaError {lib.tqkv_last_cuda_error()})"
        super().__init__(f"{fn}: {STATUS_NAMES.get(status, status)}: {detail}{extra}")
        self.status = status


def load() -> ctypes.CDLL:
    """Load libtqkv_b200.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `make -C parallel-final-project_b200` "
            "(or __graft_entry__.build()); there is no fallback implementation")
    lib = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_LOCAL)
    for name, (res, args) in C_ABI.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    for name, mangled in REF_LAUNCHERS.items():
        fn = getattr(lib, mangled)
        fn.restype = None
        fn.argtypes = REF_ARGTYPES[name]
    _lib = lib
    return lib


def check(fn: str, status: int) -> None:
    if status != TQKV_OK:
        raise TqkvError(fn, status)


def ref_launcher(name: str):
    """The C++ launcher `name` (reference signature) as a ctypes function."""
    return getattr(load(), REF_LAUNCHERS[name])


__all__ = ["load", "check", "ref_launcher", "TqkvError", "LIB_PATH", "C_ABI", "REF_LAUNCHERS",
           "c_float"]
