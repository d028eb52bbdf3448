"""tqkv — B200 (sm_100a) INT8 KV-cache compression and fused decode attention.

Python front end of libtqkv_b200.so.  The compute is the library's CUDA
kernels; this package loads the library (failing loudly if it has not been
built), wraps the C ABI for torch CUDA tensors, defines the synthetic
benchmark workloads, and orchestrates multi-GPU decode.
"""
from ._lib import LIB_PATH, TqkvError, load
from .ops import (Workspace, decode_fp16, decode_int8, decode_int8_append, decode_int8_cache,
                  decode_int8_gqa, decode_int8_partial, kv_append, kv_compress, kv_reconstruct, lse_combine,
                  read_device_error, workspace_bytes)
from .health import PeerFailure, StepMonitor
from .peer import LocalExchange, PeerExchange

__all__ = [
    "LIB_PATH", "TqkvError", "load", "Workspace", "decode_fp16", "decode_int8",
    "decode_int8_partial", "kv_compress", "kv_reconstruct", "lse_combine",
    "read_device_error", "workspace_bytes", "PeerExchange", "LocalExchange", "kv_append",
    "decode_int8_cache", "decode_int8_append", "decode_int8_gqa", "PeerFailure", "StepMonitor",
]
