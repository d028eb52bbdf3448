"""The reference's on-disk KV exchange format, sharded for multi-GPU decode.

A directory holds meta.json (integer keys B, H, D, S, plus seed / dtype /
mode / block_size) and raw little-endian fp16 tensors Q.bin [B,H,D],
K.bin and V.bin [B,H,S,D] — what the reference's drivers read with
--load-kv-from and write after a run (reference src/main.cpp:72-78, 214-246;
python/capture_kv.py writes the same layout from captured model KV).

load_kv() reads only one rank's share, through a memory map:
  shard="s"  tokens [s0, s1) of every head (split-S decode);
  shard="bh" heads [h0, h1) of the flattened B*H, every token (no collective).
The slices are exactly those of workloads.token_slice / head_slice.
"""
from __future__ import annotations

import json
import os
from typing import Optional, Tuple

import numpy as np
import torch

from .workloads import head_slice, token_slice

META_KEYS = ("B", "H", "D", "S")


def read_meta(path: str) -> dict:
    with open(os.path.join(path, "meta.json")) as f:
        meta = json.load(f)
    for k in META_KEYS:
        if not isinstance(meta.get(k), int) or meta[k] < 0:
            raise ValueError(f"meta.json: missing or invalid integer key {k!r}")
    return meta


def save_kv(path: str, q: np.ndarray, k: np.ndarray, v: np.ndarray, **extra) -> None:
    """Write q [B,H,D], k, v [B,H,S,D] (float16) in the reference's layout."""
    q, k, v = (np.ascontiguousarray(a, dtype=np.float16) for a in (q, k, v))
    B, H, S, D = k.shape
    if v.shape != k.shape or q.shape != (B, H, D):
        raise ValueError("shapes must be q [B,H,D], k = v [B,H,S,D]")
    os.makedirs(path, exist_ok=True)
    q.tofile(os.path.join(path, "Q.bin"))
    k.tofile(os.path.join(path, "K.bin"))
    v.tofile(os.path.join(path, "V.bin"))
    meta = {"B": B, "H": H, "D": D, "S": S, "dtype": "float16"}
    meta.update(extra)
    with open(os.path.join(path, "meta.json"), "w") as f:
        json.dump(meta, f, indent=2)


def _map(path: str, name: str, shape) -> np.ndarray:
    fn = os.path.join(path, name)
    need = int(np.prod(shape)) * 2
    have = os.path.getsize(fn)
    if have < need:
        raise ValueError(f"{fn}: {have} bytes, expected {need} for shape {shape}")
    return np.memmap(fn, dtype=np.float16, mode="r", shape=tuple(shape))


def load_kv(path: str, rank: int = 0, world: int = 1, shard: str = "s",
            device: Optional[torch.device] = None
            ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, dict]:
    """This rank's (q, k, v) as fp16 tensors (on `device` if given) and the
    meta dict extended with the slice bounds: shard "s" -> q [B,H,D],
    k/v [B,H,s1-s0,D]; shard "bh" -> q [1,h1-h0,D], k/v [1,h1-h0,S,D]."""
    meta = read_meta(path)
    B, H, D, S = (meta[k] for k in ("B", "H", "D", "S"))
    q = _map(path, "Q.bin", (B, H, D))
    k = _map(path, "K.bin", (B, H, S, D))
    v = _map(path, "V.bin", (B, H, S, D))
    if shard == "s":
        s0, s1 = token_slice(S, rank, world)
        parts = (np.array(q), np.array(k[:, :, s0:s1]), np.array(v[:, :, s0:s1]))
        meta = dict(meta, s0=s0, s1=s1)
    elif shard == "bh":
        h0, h1 = head_slice(B * H, rank, world)
        parts = (np.array(q.reshape(1, B * H, D)[:, h0:h1]),
                 np.array(k.reshape(1, B * H, S, D)[:, h0:h1]),
                 np.array(v.reshape(1, B * H, S, D)[:, h0:h1]))
        meta = dict(meta, h0=h0, h1=h1)
    else:
        raise ValueError("shard must be 's' or 'bh'")
    out = tuple(torch.from_numpy(np.ascontiguousarray(a)) for a in parts)
    if device is not None:
        out = tuple(t.to(device) for t in out)
    return out[0], out[1], out[2], meta
