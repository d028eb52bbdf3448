"""Torch-tensor front end of the C ABI (include/tqkv.h).

Every function takes CUDA tensors in the reference's layouts
(reference include/quantization.h:5-12, include/attention.h):

    q, o     fp16 [B, H, D]
    k, v     fp16 [B, H, S, D]
    kq, vq   int8 [B, H, S, D]
    ks, vs   fp16 [B, H, S, D // block_size]

and launches on the current torch stream (or `stream=`).  Torch only
allocates memory and provides streams here; all compute is the library's
sm_100a kernels.  Errors raise TqkvError.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from ._lib import check, load

_F16 = torch.float16


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream_handle(stream: Optional[torch.cuda.Stream]) -> int:
    s = torch.cuda.current_stream() if stream is None else stream
    return s.cuda_stream


def _bhsd(t: torch.Tensor, name: str) -> Tuple[int, int, int, int]:
    if t.dim() != 4 or not t.is_contiguous() or not t.is_cuda:
        raise ValueError(f"{name} must be a contiguous CUDA tensor [B, H, S, D]")
    return tuple(t.shape)  # type: ignore[return-value]


# Memory safety at the boundary: the library gets raw pointers and sizes, so
# these checks make sure every buffer holds exactly what the kernels will read
# or write there (element count, element size, contiguity, device).
def _need(t: Optional[torch.Tensor], name: str, numel: int, esize: int,
          like: torch.Tensor) -> None:
    if t is None:
        raise ValueError(f"{name} is required")
    if not t.is_contiguous() or t.device != like.device:
        raise ValueError(f"{name} must be a contiguous tensor on {like.device}")
    if t.element_size() != esize or t.numel() != numel:
        raise ValueError(f"{name}: need {numel} elements of {esize} bytes, got shape "
                         f"{tuple(t.shape)} of {t.dtype}")


def _nsub(D: int, block_size: int) -> Optional[int]:
    """Scales per row, or None for a block size the library rejects anyway."""
    return D // block_size if block_size > 0 and D % block_size == 0 else None


def _check_scales(ks: torch.Tensor, name: str, rows: int, D: int, block_size: int,
                  like: torch.Tensor) -> None:
    nsub = _nsub(D, block_size)
    if nsub is not None:
        _need(ks, name, rows * nsub, 2, like)


def _check_int8_kv(kq, ks, vq, vs, block_size: int) -> Tuple[int, int, int, int]:
    """kq/vq int8 [B,H,S,D] and ks/vs fp16 [B,H,S,D/bs]; returns (B, H, S, D)."""
    B, H, S, D = _bhsd(kq, "kq")
    for t, n in ((kq, "kq"), (vq, "vq")):
        _need(t, n, B * H * S * D, 1, kq)
    for t, n in ((ks, "ks"), (vs, "vs")):
        _check_scales(t, n, B * H * S, D, block_size, kq)
    return B, H, S, D


def kv_compress(x: torch.Tensor, block_size: int, xq: Optional[torch.Tensor] = None,
                scales: Optional[torch.Tensor] = None, stream=None):
    """Kernel A: fp16 [B,H,S,D] -> (int8 codes [B,H,S,D], fp16 scales [B,H,S,D/bs])."""
    if x.dtype != _F16:
        raise ValueError("x must be fp16")
    B, H, S, D = _bhsd(x, "x")
    if xq is None:
        xq = torch.empty((B, H, S, D), dtype=torch.int8, device=x.device)
    if scales is None:
        scales = torch.empty((B, H, S, max(D // block_size, 1)), dtype=_F16, device=x.device)
    _need(xq, "xq", x.numel(), 1, x)
    _check_scales(scales, "scales", B * H * S, D, block_size, x)
    lib = load()
    check("tqkv_kv_compress", lib.tqkv_kv_compress(
        _ptr(x), _ptr(xq), _ptr(scales), B, H, S, D, block_size, _stream_handle(stream)))
    return xq, scales


def kv_reconstruct(xq: torch.Tensor, scales: torch.Tensor, block_size: int,
                   y: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Kernel B: codes + scales -> fp16 [B,H,S,D]."""
    B, H, S, D = _bhsd(xq, "xq")
    _need(xq, "xq", B * H * S * D, 1, xq)
    _check_scales(scales, "scales", B * H * S, D, block_size, xq)
    if y is None:
        y = torch.empty((B, H, S, D), dtype=_F16, device=xq.device)
    _need(y, "y", B * H * S * D, 2, xq)
    lib = load()
    check("tqkv_kv_reconstruct", lib.tqkv_kv_reconstruct(
        _ptr(xq), _ptr(scales), _ptr(y), B, H, S, D, block_size, _stream_handle(stream)))
    return y


def kv_append(x: torch.Tensor, cache_q: torch.Tensor, cache_s: torch.Tensor, t0: int,
              block_size: int, stream=None) -> None:
    """Quantise T new tokens per head, x fp16 [B,H,T,D], into rows [t0, t0+T) of
    the INT8 cache (cache_q int8 [B,H,S_cap,D], cache_s fp16 [B,H,S_cap,D/bs])."""
    B, H, T, D = _bhsd(x, "x")
    _need(x, "x", B * H * T * D, 2, x)
    Bc, Hc, S_cap, Dc = _bhsd(cache_q, "cache_q")
    if (Bc, Hc, Dc) != (B, H, D):
        raise ValueError(f"cache_q {tuple(cache_q.shape)} does not match x {tuple(x.shape)}")
    _need(cache_q, "cache_q", B * H * S_cap * D, 1, x)
    _check_scales(cache_s, "cache_s", B * H * S_cap, D, block_size, x)
    lib = load()
    check("tqkv_kv_append", lib.tqkv_kv_append(
        _ptr(x), _ptr(cache_q), _ptr(cache_s), B, H, T, D, block_size, S_cap, t0,
        _stream_handle(stream)))


def decode_int8_cache(q: torch.Tensor, kq: torch.Tensor, ks: torch.Tensor, vq: torch.Tensor,
                      vs: torch.Tensor, S: int, block_size: int,
                      out: Optional[torch.Tensor] = None, workspace: Optional["Workspace"] = None,
                      stream=None) -> torch.Tensor:
    """Decode over the first S rows of caches holding S_cap >= S rows per head."""
    B, H, S_cap, D = _check_int8_kv(kq, ks, vq, vs, block_size)
    _need(q, "q", B * H * D, 2, kq)
    if out is None:
        out = torch.empty((B, H, D), dtype=_F16, device=q.device)
    _need(out, "out", B * H * D, 2, kq)
    ws = _workspace(workspace, q.device)
    wptr, wbytes = ws.get(workspace_bytes(B, H, S, D) if S > 0 else 0, stream)
    lib = load()
    check("tqkv_decode_int8_cache", lib.tqkv_decode_int8_cache(
        _ptr(q), _ptr(kq), _ptr(ks), _ptr(vq), _ptr(vs), _ptr(out), B, H, S, S_cap, D,
        block_size, wptr, wbytes, _stream_handle(stream)))
    return out


def decode_int8_append(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                       kq: torch.Tensor, ks: torch.Tensor, vq: torch.Tensor, vs: torch.Tensor,
                       S: int, block_size: int, out: Optional[torch.Tensor] = None,
                       workspace: Optional["Workspace"] = None, stream=None) -> torch.Tensor:
    """Append fused into decode: quantise the T newest tokens (k_new / v_new fp16
    [B,H,T,D]) into rows [S-T, S) of the caches (kq/vq int8 [B,H,S_cap,D], ks/vs
    fp16 [B,H,S_cap,D/bs]) and attend over rows [0, S), in one launch."""
    B, H, S_cap, D = _check_int8_kv(kq, ks, vq, vs, block_size)
    Bn, Hn, T, Dn = _bhsd(k_new, "k_new")
    if (Bn, Hn, Dn) != (B, H, D) or k_new.dtype != _F16 or v_new.dtype != _F16 or \
            v_new.shape != k_new.shape:
        raise ValueError("k_new and v_new must be fp16 [B, H, T, D] matching the caches")
    _need(v_new, "v_new", k_new.numel(), 2, kq)
    _need(q, "q", B * H * D, 2, kq)
    if out is None:
        out = torch.empty((B, H, D), dtype=_F16, device=q.device)
    _need(out, "out", B * H * D, 2, kq)
    ws = _workspace(workspace, q.device)
    wptr, wbytes = ws.get(workspace_bytes(B, H, S, D) if S > 0 else 0, stream)
    lib = load()
    check("tqkv_decode_int8_append", lib.tqkv_decode_int8_append(
        _ptr(q), _ptr(k_new), _ptr(v_new), _ptr(kq), _ptr(ks), _ptr(vq), _ptr(vs), _ptr(out),
        B, H, T, S, S_cap, D, block_size, wptr, wbytes, _stream_handle(stream)))
    return out


def workspace_bytes(B: int, H: int, S: int, D: int) -> int:
    """Scratch the decode kernels need for this shape on the current device."""
    return int(load().tqkv_decode_workspace_bytes(B, H, S, D))


class Workspace:
    """A zero-initialised decode workspace on one device, grown on demand.

    The kernels leave it zeroed after every call, so one Workspace can serve
    any number of calls that are ordered on the same stream.  A buffer once
    handed out is never freed while the Workspace lives: when a larger shape
    needs more, the old buffer is retired and kept, so a CUDA graph captured
    with it stays valid (torch.cuda.graph empties the allocator's cache when a
    capture begins, which would otherwise unmap a freed workspace under an
    earlier graph).  Growth at least doubles, so retired buffers add up to
    less than the live one.
    """

    def __init__(self, device=None):
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        self.buf: Optional[torch.Tensor] = None
        self._retired: list = []

    def get(self, nbytes: int, stream=None) -> Tuple[Optional[int], int]:
        if nbytes == 0:
            return None, 0
        if self.buf is None or self.buf.numel() < nbytes:
            size = nbytes if self.buf is None else max(nbytes, 2 * self.buf.numel())
            if self.buf is not None:
                self._retired.append(self.buf)
            self.buf = torch.empty(size, dtype=torch.uint8, device=self.device)
            lib = load()
            check("tqkv_workspace_init", lib.tqkv_workspace_init(
                self.buf.data_ptr(), size, _stream_handle(stream)))
        return self.buf.data_ptr(), self.buf.numel()


_default_ws: dict = {}


def _workspace(ws: Optional[Workspace], device: torch.device) -> Workspace:
    if ws is not None:
        return ws
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    if key not in _default_ws:
        _default_ws[key] = Workspace(device)
    return _default_ws[key]


def decode_int8(q: torch.Tensor, kq: torch.Tensor, ks: torch.Tensor, vq: torch.Tensor,
                vs: torch.Tensor, block_size: int, out: Optional[torch.Tensor] = None,
                workspace: Optional[Workspace] = None, stream=None) -> torch.Tensor:
    """Kernel D: fused INT8 decode attention -> O fp16 [B,H,D]."""
    B, H, S, D = _check_int8_kv(kq, ks, vq, vs, block_size)
    _need(q, "q", B * H * D, 2, kq)
    if out is None:
        out = torch.empty((B, H, D), dtype=_F16, device=q.device)
    _need(out, "out", B * H * D, 2, kq)
    ws = _workspace(workspace, q.device)
    wptr, wbytes = ws.get(workspace_bytes(B, H, S, D), stream)
    lib = load()
    check("tqkv_decode_int8", lib.tqkv_decode_int8(
        _ptr(q), _ptr(kq), _ptr(ks), _ptr(vq), _ptr(vs), _ptr(out), B, H, S, D, block_size,
        wptr, wbytes, _stream_handle(stream)))
    return out


def decode_int8_gqa(q: torch.Tensor, kq: torch.Tensor, ks: torch.Tensor, vq: torch.Tensor,
                    vs: torch.Tensor, block_size: int, out: Optional[torch.Tensor] = None,
                    workspace: Optional[Workspace] = None, stream=None) -> torch.Tensor:
    """Grouped-query decode: q [B,H_q,D] over K/V with H_kv heads ([B,H_kv,S,D]),
    H_q a multiple of H_kv; query head h uses K/V head h // (H_q // H_kv)."""
    B, H_kv, S, D = _check_int8_kv(kq, ks, vq, vs, block_size)
    if q.dim() != 3 or q.shape[0] != B or q.shape[2] != D:
        raise ValueError("q must be [B, H_q, D]")
    H_q = q.shape[1]
    _need(q, "q", B * H_q * D, 2, kq)
    if out is None:
        out = torch.empty((B, H_q, D), dtype=_F16, device=q.device)
    _need(out, "out", B * H_q * D, 2, kq)
    ws = _workspace(workspace, q.device)
    wptr, wbytes = ws.get(workspace_bytes(B, H_q, S, D) if S > 0 else 0, stream)
    check("tqkv_decode_int8_gqa", load().tqkv_decode_int8_gqa(
        _ptr(q), _ptr(kq), _ptr(ks), _ptr(vq), _ptr(vs), _ptr(out), B, H_q, H_kv, S, D,
        block_size, wptr, wbytes, _stream_handle(stream)))
    return out


def decode_fp16(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                out: Optional[torch.Tensor] = None, workspace: Optional[Workspace] = None,
                stream=None) -> torch.Tensor:
    """FP16 decode attention (the reference's baseline) -> O fp16 [B,H,D]."""
    B, H, S, D = _bhsd(k, "k")
    for t, n in ((k, "k"), (v, "v")):
        _need(t, n, B * H * S * D, 2, k)
    _need(q, "q", B * H * D, 2, k)
    if out is None:
        out = torch.empty((B, H, D), dtype=_F16, device=q.device)
    _need(out, "out", B * H * D, 2, k)
    ws = _workspace(workspace, q.device)
    wptr, wbytes = ws.get(workspace_bytes(B, H, S, D), stream)
    lib = load()
    check("tqkv_decode_fp16", lib.tqkv_decode_fp16(
        _ptr(q), _ptr(k), _ptr(v), _ptr(out), B, H, S, D, wptr, wbytes,
        _stream_handle(stream)))
    return out


def decode_int8_partial(q: torch.Tensor, kq: torch.Tensor, ks: torch.Tensor, vq: torch.Tensor,
                        vs: torch.Tensor, block_size: int, out: Optional[torch.Tensor] = None,
                        workspace: Optional[Workspace] = None, stream=None) -> torch.Tensor:
    """Per-head split-S partial records over this device's token slice:
    float32 [B*H, D+2] = (acc[0..D-1], m, l), natural-log units."""
    B, H, S, D = _check_int8_kv(kq, ks, vq, vs, block_size)
    _need(q, "q", B * H * D, 2, kq)
    if out is None:
        out = torch.empty((B * H, D + 2), dtype=torch.float32, device=q.device)
    _need(out, "out", B * H * (D + 2), 4, kq)
    ws = _workspace(workspace, q.device)
    wptr, wbytes = ws.get(workspace_bytes(B, H, S, D) if S > 0 else 0, stream)
    lib = load()
    check("tqkv_decode_int8_partial", lib.tqkv_decode_int8_partial(
        _ptr(q), _ptr(kq), _ptr(ks), _ptr(vq), _ptr(vs), _ptr(out), B, H, S, D, block_size,
        wptr, wbytes, _stream_handle(stream)))
    return out


def lse_combine(partials: torch.Tensor, D: int, out: Optional[torch.Tensor] = None,
                stream=None) -> torch.Tensor:
    """Merge R partial-record sets [R, BH, D+2] into O fp16 [BH, D]."""
    if partials.dim() != 3 or partials.shape[2] != D + 2 or partials.dtype != torch.float32:
        raise ValueError("partials must be float32 [R, BH, D + 2]")
    R, BH = partials.shape[0], partials.shape[1]
    if out is None:
        out = torch.empty((BH, D), dtype=_F16, device=partials.device)
    lib = load()
    check("tqkv_lse_combine", lib.tqkv_lse_combine(
        _ptr(partials), _ptr(out), R, BH, D, _stream_handle(stream)))
    return out


def read_device_error() -> int:
    """Read and clear the device-side bounded-wait failure flag (0 = none)."""
    code = ctypes.c_uint32(0)
    check("tqkv_read_device_error", load().tqkv_read_device_error(ctypes.byref(code)))
    return int(code.value)
