"""Split-S decode across the GPUs of one node over NVLink peer mappings.

Each rank owns one exchange buffer (a step counter and double-buffered
per-head records, see include/tqkv.h).  The buffers are shared with CUDA IPC
handles, exchanged once through torch.distributed, so every rank can write
into every other rank's buffer.  Per decode step:

    publish(...)   decode kernel over this rank's token slice; each finished
                   head's (acc, m, l) goes into every rank's buffer, every
                   value stored together with the step number (64-bit stores)
    combine(out)   bounded wait until this rank's buffer holds every rank's
                   entries of this step, merge into O, advance the step

or both in one launch, step(..., out) (step_append with the
newest tokens appended): after its share of the slice, each CTA of the decode
launch merges heads whose records have arrived from every rank, so the
exchange overlaps the other CTAs' streaming and no second launch is needed.

A rank that stops stepping makes the others' combines time out (device error
flag); tqkv.health.StepMonitor detects it on the host between steps.

Both are plain kernel launches on the caller's stream, so a step can be
captured in a CUDA graph.  No NCCL call and no multicast object is involved.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
import torch.distributed as dist

from ._lib import check, load
from .ops import (Workspace, _bhsd, _check_int8_kv, _need, _stream_handle, _workspace,
                  workspace_bytes)


class PeerExchange:
    def __init__(self, world: int, rank: int, BH: int, D: int, group=None):
        lib = load()
        self.world, self.rank, self.BH, self.D = world, rank, BH, D
        self.group = group
        nbytes = int(lib.tqkv_exchange_bytes(world, BH, D))
        if nbytes == 0:
            raise ValueError(f"unsupported exchange shape world={world} BH={BH} D={D}")
        own = ctypes.c_void_p()
        check("tqkv_exchange_alloc", lib.tqkv_exchange_alloc(nbytes, ctypes.byref(own)))
        self.own = own.value
        handle = (ctypes.c_ubyte * 64)()
        check("tqkv_ipc_get_handle", lib.tqkv_ipc_get_handle(self.own, handle))
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        ptrs, self._opened = [], []
        for r in range(world):
            if r == rank:
                ptrs.append(self.own)
                continue
            h = (ctypes.c_ubyte * 64).from_buffer_copy(handles[r])
            p = ctypes.c_void_p()
            check("tqkv_ipc_open_handle", lib.tqkv_ipc_open_handle(h, ctypes.byref(p)))
            ptrs.append(p.value)
            self._opened.append(p.value)
        self.bufs = (ctypes.c_void_p * world)(*ptrs)
        torch.cuda.synchronize()
        dist.barrier(group=group)  # every buffer is zeroed and mapped before the first step

    def publish(self, q, kq, ks, vq, vs, block_size: int, workspace: Optional[Workspace] = None,
                stream=None) -> None:
        B, H, S, D = _check_int8_kv(kq, ks, vq, vs, block_size)
        if B * H != self.BH or D != self.D:
            raise ValueError(f"exchange is for BH={self.BH} D={self.D}, got {B * H} x {D}")
        _need(q, "q", B * H * D, 2, kq)
        ws = _workspace(workspace, q.device)
        wptr, wbytes = ws.get(workspace_bytes(B, H, S, D), stream)
        check("tqkv_decode_int8_publish", load().tqkv_decode_int8_publish(
            q.data_ptr(), kq.data_ptr(), ks.data_ptr(), vq.data_ptr(), vs.data_ptr(),
            B, H, S, D, block_size, wptr, wbytes, self.bufs, self.world, self.rank,
            _stream_handle(stream)))

    def publish_append(self, q, k_new, v_new, kq, ks, vq, vs, S: int, block_size: int,
                       workspace: Optional[Workspace] = None, stream=None) -> None:
        """publish() over the first S rows of caches [B, H, S_cap, D] after
        appending the T newest tokens (k_new / v_new fp16 [B, H, T, D]) at rows
        [S - T, S), in the same launch."""
        B, H, S_cap, D = _check_int8_kv(kq, ks, vq, vs, block_size)
        if B * H != self.BH or D != self.D:
            raise ValueError(f"exchange is for BH={self.BH} D={self.D}, got {B * H} x {D}")
        Bn, Hn, T, Dn = _bhsd(k_new, "k_new")
        if (Bn, Hn, Dn) != (B, H, D) or v_new.shape != k_new.shape:
            raise ValueError("k_new and v_new must be [B, H, T, D] matching the caches")
        for t, n in ((k_new, "k_new"), (v_new, "v_new")):
            _need(t, n, B * H * T * D, 2, kq)
        _need(q, "q", B * H * D, 2, kq)
        ws = _workspace(workspace, q.device)
        wptr, wbytes = ws.get(workspace_bytes(B, H, S, D), stream)
        check("tqkv_decode_int8_append_publish", load().tqkv_decode_int8_append_publish(
            q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), kq.data_ptr(), ks.data_ptr(),
            vq.data_ptr(), vs.data_ptr(), B, H, T, S, S_cap, D, block_size, wptr, wbytes,
            self.bufs, self.world, self.rank, _stream_handle(stream)))

    def step(self, q, kq, ks, vq, vs, block_size: int, out: torch.Tensor,
             workspace: Optional[Workspace] = None, stream=None) -> torch.Tensor:
        """publish() and combine(out) in one launch (tqkv_decode_int8_exchange);
        the same O, bit for bit."""
        B, H, S, D = _check_int8_kv(kq, ks, vq, vs, block_size)
        if B * H != self.BH or D != self.D:
            raise ValueError(f"exchange is for BH={self.BH} D={self.D}, got {B * H} x {D}")
        _need(q, "q", B * H * D, 2, kq)
        _need(out, "out", B * H * D, 2, kq)
        ws = _workspace(workspace, q.device)
        wptr, wbytes = ws.get(workspace_bytes(B, H, max(S, 1), D), stream)
        check("tqkv_decode_int8_exchange", load().tqkv_decode_int8_exchange(
            q.data_ptr(), kq.data_ptr(), ks.data_ptr(), vq.data_ptr(), vs.data_ptr(),
            out.data_ptr(), B, H, S, D, block_size, wptr, wbytes, self.bufs, self.world,
            self.rank, _stream_handle(stream)))
        return out

    def step_append(self, q, k_new, v_new, kq, ks, vq, vs, S: int, block_size: int,
                    out: torch.Tensor, workspace: Optional[Workspace] = None,
                    stream=None) -> torch.Tensor:
        """publish_append() and combine(out) in one launch
        (tqkv_decode_int8_append_exchange)."""
        B, H, S_cap, D = _check_int8_kv(kq, ks, vq, vs, block_size)
        if B * H != self.BH or D != self.D:
            raise ValueError(f"exchange is for BH={self.BH} D={self.D}, got {B * H} x {D}")
        Bn, Hn, T, Dn = _bhsd(k_new, "k_new")
        if (Bn, Hn, Dn) != (B, H, D) or v_new.shape != k_new.shape:
            raise ValueError("k_new and v_new must be [B, H, T, D] matching the caches")
        for t, n in ((k_new, "k_new"), (v_new, "v_new")):
            _need(t, n, B * H * T * D, 2, kq)
        _need(q, "q", B * H * D, 2, kq)
        _need(out, "out", B * H * D, 2, kq)
        ws = _workspace(workspace, q.device)
        wptr, wbytes = ws.get(workspace_bytes(B, H, S, D), stream)
        check("tqkv_decode_int8_append_exchange", load().tqkv_decode_int8_append_exchange(
            q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), kq.data_ptr(), ks.data_ptr(),
            vq.data_ptr(), vs.data_ptr(), out.data_ptr(), B, H, T, S, S_cap, D, block_size,
            wptr, wbytes, self.bufs, self.world, self.rank, _stream_handle(stream)))
        return out

    def combine(self, out: torch.Tensor, stream=None) -> torch.Tensor:
        _need(out, "out", self.BH * self.D, 2, out)
        check("tqkv_exchange_combine", load().tqkv_exchange_combine(
            self.bufs, out.data_ptr(), self.world, self.rank, self.BH, self.D,
            _stream_handle(stream)))
        return out

    def close(self) -> None:
        """Unmap and free, once no rank can still write into any buffer."""
        if self.own is None:
            return
        lib = load()
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self._opened:
            check("tqkv_ipc_close_handle", lib.tqkv_ipc_close_handle(p))
        self._opened = []
        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # nobody still holds a mapping of our buffer
        check("tqkv_exchange_free", lib.tqkv_exchange_free(self.own))
        self.own = None


class LocalExchange:
    """The same two-launch step with a single rank (world = 1), on one GPU:
    the combine waits only for this rank's own flag, which the publish launch
    before it on the same stream has raised."""

    def __init__(self, BH: int, D: int):
        lib = load()
        self.world, self.rank, self.BH, self.D = 1, 0, BH, D
        nbytes = int(lib.tqkv_exchange_bytes(1, BH, D))
        own = ctypes.c_void_p()
        check("tqkv_exchange_alloc", lib.tqkv_exchange_alloc(nbytes, ctypes.byref(own)))
        self.own = own.value
        self.bufs = (ctypes.c_void_p * 1)(self.own)

    publish = PeerExchange.publish
    publish_append = PeerExchange.publish_append
    combine = PeerExchange.combine
    step = PeerExchange.step
    step_append = PeerExchange.step_append

    def close(self) -> None:
        if self.own is not None:
            torch.cuda.synchronize()
            check("tqkv_exchange_free", load().tqkv_exchange_free(self.own))
            self.own = None
