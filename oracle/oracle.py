"""TEST INFRASTRUCTURE ONLY — numpy front end of liboracle_tqkv.so, the plain
C restatement of the reference's decode path (oracle/tqkv_oracle.c).

Functions take and return numpy arrays in the reference's layouts
(binary16 as np.float16, codes as np.int8).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liboracle_tqkv.so")
_lib = None

_P = ctypes.c_void_p
_LL = ctypes.c_longlong
_I = ctypes.c_int


def build() -> None:
    subprocess.run(["make", "-s", "-C", _HERE, "all"], check=True)


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        build()
    lib = ctypes.CDLL(LIB_PATH)
    sig = {
        "oracle_kv_compress": [_P, _P, _P, _LL, _I, _I],
        "oracle_kv_tie_mask": [_P, _P, _LL, _I, _I],
        "oracle_kv_reconstruct": [_P, _P, _P, _LL, _I, _I],
        "oracle_dequantize_f32": [_P, _P, _P, _LL, _I, _I],
        "oracle_half_array_to_float": [_P, _P, _LL],
        "oracle_float_array_to_half": [_P, _P, _LL],
        "oracle_attention": [_P, _P, _P, _P, _LL, _I, _I],
        "oracle_attention_partial": [_P, _P, _P, _P, _LL, _I, _I],
    }
    for name, args in sig.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = _LL if name == "oracle_kv_tie_mask" else None
    _lib = lib
    return lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def kv_compress(x: np.ndarray, block_size: int):
    """x fp16 [..., D] -> (int8 codes, fp16 scales [..., D/bs]), IEEE rule."""
    x = np.ascontiguousarray(x, dtype=np.float16)
    D = x.shape[-1]
    rows = x.size // D
    q = np.empty(x.shape, dtype=np.int8)
    s = np.empty(x.shape[:-1] + (D // block_size,), dtype=np.float16)
    load().oracle_kv_compress(_p(x), _p(q), _p(s), rows, D, block_size)
    return q, s


def tie_mask(x: np.ndarray, block_size: int):
    """uint8 mask of the elements whose code depends on the division
    implementation (exact quotient 127 x / m is a half-integer), and its count."""
    x = np.ascontiguousarray(x, dtype=np.float16)
    D = x.shape[-1]
    m = np.empty(x.shape, dtype=np.uint8)
    n = load().oracle_kv_tie_mask(_p(x), _p(m), x.size // D, D, block_size)
    return m, int(n)


def kv_reconstruct(q: np.ndarray, scales: np.ndarray, block_size: int) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.int8)
    scales = np.ascontiguousarray(scales, dtype=np.float16)
    D = q.shape[-1]
    y = np.empty(q.shape, dtype=np.float16)
    load().oracle_kv_reconstruct(_p(q), _p(scales), _p(y), q.size // D, D, block_size)
    return y


def dequantize(q: np.ndarray, scales: np.ndarray, block_size: int,
               exact: bool = False) -> np.ndarray:
    """float32 K/V from codes and scales.  Default: fp16(code * scale), the
    K/V the reference's Python check feeds its attention
    (python/check_correctness.py:47-56).  exact=True: code * scale in fp32
    (exact: a 7-bit code times an 11-bit scale), what the reference kernels
    use in registers (src/attention_int8_fused_online.cu:94-97)."""
    q = np.ascontiguousarray(q, dtype=np.int8)
    scales = np.ascontiguousarray(scales, dtype=np.float16)
    D = q.shape[-1]
    if exact:
        s = np.repeat(scales.astype(np.float32), block_size, axis=-1)
        return q.astype(np.float32) * s
    out = np.empty(q.shape, dtype=np.float32)
    load().oracle_dequantize_f32(_p(q), _p(scales), _p(out), q.size // D, D, block_size)
    return out


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """softmax(q.K^T/sqrt(D)).V in binary64; q [B,H,D], k/v [B,H,S,D] (any float
    dtype) -> float32 [B,H,D]."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    B, H, S, D = k.shape
    out = np.empty((B, H, D), dtype=np.float32)
    load().oracle_attention(_p(q), _p(k), _p(v), _p(out), B * H, S, D)
    return out


def attention_partial(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """Split-S partial records float64 [B*H, D+2] = (acc, m, l) over the given slice."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    B, H, S, D = k.shape
    rec = np.empty((B * H, D + 2), dtype=np.float64)
    load().oracle_attention_partial(_p(q), _p(k), _p(v), _p(rec), B * H, S, D)
    return rec


def lse_combine(records: np.ndarray) -> np.ndarray:
    """Merge partial records [R, BH, D+2] (natural-log units) -> float64 [BH, D]."""
    D = records.shape[-1] - 2
    m = records[..., D]
    M = np.max(m, axis=0)
    f = np.where(np.isneginf(m), 0.0, np.exp(m - np.where(np.isneginf(M), 0.0, M)))
    L = np.sum(records[..., D + 1] * f, axis=0)
    A = np.sum(records[..., :D] * f[..., None], axis=0)
    return A / L[:, None]


def float_to_half_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    h = np.empty(x.shape, dtype=np.uint16)
    load().oracle_float_array_to_half(_p(x), _p(h), x.size)
    return h


def half_bits_to_float(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    f = np.empty(h.shape, dtype=np.float32)
    load().oracle_half_array_to_float(_p(h), _p(f), h.size)
    return f
