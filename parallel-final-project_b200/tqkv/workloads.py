"""Seeded synthetic decode workloads (the five benchmark configurations).

The reference measures on random K/V (its drivers draw N(0,1) * 0.1 from
std::mt19937, reference src/main.cpp:129-137) and on GPT-2 KV captured from
HuggingFace weights, which are not available offline.  These generators
stand in for both with the shapes and value distributions of the five
configurations below; the GPT-2-shaped configuration with outlier channels
replaces the captured KV.

Generation is on the device (torch's counter-based CUDA generator), in
chunks of `CHUNK` tokens that are seeded independently, so any token slice
[s0, s1) of any configuration can be produced on its own and is bit-identical
to the same slice of the full tensor.  That lets every rank of a split-S run
build only its own slice while the result stays comparable to one GPU.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch

CHUNK = 2048  # tokens per independently seeded generation chunk


@dataclass(frozen=True)
class Workload:
    name: str
    B: int
    H: int
    S: int
    D: int
    block_size: int  # 0 for the fp16 path
    seed: int
    dist: str        # "normal" | "lognormal_channels" | "outlier_channels"
    description: str

    @property
    def BH(self) -> int:
        return self.B * self.H

    def kv_bytes_int8(self, S: Optional[int] = None) -> int:
        """Algorithmic bytes one decode step reads: K and V codes plus their
        fp16 scales (the reference's bytes_kv, src/benchmark.cpp:251)."""
        S = self.S if S is None else S
        bs = self.block_size
        return 2 * self.BH * S * self.D + 2 * self.BH * S * (self.D // bs) * 2

    def kv_bytes_fp16(self, S: Optional[int] = None) -> int:
        S = self.S if S is None else S
        return 2 * self.BH * S * self.D * 2


WORKLOADS = {
    "fp16_small": Workload(
        "fp16_small", 1, 4, 128, 64, 0, 0, "normal",
        "FP16 decode B1 H4 D64 S128, q/K/V ~ N(0,1), seed 0"),
    "int8_b2h8": Workload(
        "int8_b2h8", 2, 8, 2048, 128, 64, 1, "normal",
        "INT8 compress + decode B2 H8 D128 S2048 bs64, q/K/V ~ N(0,1), seed 1"),
    "int8_bh_shard": Workload(
        "int8_bh_shard", 16, 32, 8192, 128, 32, 2, "lognormal_channels",
        "INT8 decode B16 H32 D128 S8192 bs32, K/V ~ N(0,1) x per-(h,d) exp(N(0,0.5)), seed 2; "
        "sharded over B*H"),
    "int8_gpt2_outlier": Workload(
        "int8_gpt2_outlier", 8, 12, 1024, 64, 64, 3, "outlier_channels",
        "INT8 decode B8 H12 D64 S1024 bs64, K/V ~ N(0,1) with ceil(1% of D) channel per head "
        "x10, V + per-(h,d) N(0,0.1) bias, seed 3"),
    "int8_longctx_s16k": Workload(
        "int8_longctx_s16k", 4, 32, 16384, 128, 128, 4, "normal",
        "INT8 decode B4 H32 D128 S16384 bs128, K/V ~ N(0,1), seed 4: one GPU's token slice of "
        "the long-context configuration at 8 GPUs (its first 16384 tokens)"),
    "int8_longctx": Workload(
        "int8_longctx", 4, 32, 131072, 128, 128, 4, "normal",
        "INT8 long-context decode B4 H32 D128 S131072 bs128, K/V ~ N(0,1), seed 4; "
        "S split across GPUs"),
}

_TENSOR_IDS = {"q": 1, "k": 2, "v": 3, "kmul": 4, "vmul": 5, "kout": 6, "vout": 7, "vbias": 8}


def _gen(seed: int, tensor: str, chunk: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(((seed * 1_000_003 + _TENSOR_IDS[tensor]) * 65_537 + chunk) & 0x7FFF_FFFF_FFFF)
    return g


def _channel_factors(w: Workload, which: str, device) -> Optional[torch.Tensor]:
    """Per-(h, d) multiplier (fp32 [H, D]) for K or V, or None."""
    if w.dist == "lognormal_channels":
        z = torch.randn((w.H, w.D), generator=_gen(w.seed, which + "mul", 0, device),
                        device=device, dtype=torch.float32)
        return torch.exp(0.5 * z)
    if w.dist == "outlier_channels":
        n_out = -(-w.D // 100)  # ceil(1% of D)
        f = torch.ones((w.H, w.D), device=device, dtype=torch.float32)
        g = _gen(w.seed, which + "out", 0, device)
        for h in range(w.H):
            idx = torch.randperm(w.D, generator=g, device=device)[:n_out]
            f[h, idx] = 10.0
        return f
    return None


def _v_bias(w: Workload, device) -> Optional[torch.Tensor]:
    if w.dist != "outlier_channels":
        return None
    return 0.1 * torch.randn((w.H, w.D), generator=_gen(w.seed, "vbias", 0, device),
                             device=device, dtype=torch.float32)


def make_q(w: Workload, device="cuda") -> torch.Tensor:
    """q fp16 [B, H, D] ~ N(0, 1)."""
    q = torch.randn((w.B, w.H, w.D), generator=_gen(w.seed, "q", 0, device), device=device,
                    dtype=torch.float32)
    return q.to(torch.float16)


def make_kv_slice(w: Workload, which: str, s0: int = 0, s1: Optional[int] = None,
                  device="cuda") -> torch.Tensor:
    """K or V fp16 [B, H, s1 - s0, D] for tokens [s0, s1) of the configuration."""
    assert which in ("k", "v")
    s1 = w.S if s1 is None else s1
    out = torch.empty((w.B, w.H, s1 - s0, w.D), dtype=torch.float16, device=device)
    fac = _channel_factors(w, which, device)
    bias = _v_bias(w, device) if which == "v" else None
    c0, c1 = s0 // CHUNK, (s1 + CHUNK - 1) // CHUNK
    for c in range(c0, c1):
        t0, t1 = c * CHUNK, min((c + 1) * CHUNK, w.S)
        x = torch.randn((w.B, w.H, t1 - t0, w.D), generator=_gen(w.seed, which, c, device),
                        device=device, dtype=torch.float32)
        if fac is not None:
            x.mul_(fac[None, :, None, :])
        if bias is not None:
            x.add_(bias[None, :, None, :])
        a, b = max(t0, s0), min(t1, s1)
        out[:, :, a - s0:b - s0, :] = x[:, :, a - t0:b - t0, :].to(torch.float16)
        del x
    return out


def make_inputs(w: Workload, s0: int = 0, s1: Optional[int] = None,
                device="cuda") -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(q, K, V) for tokens [s0, s1) of the configuration, all fp16 on `device`."""
    return make_q(w, device), make_kv_slice(w, "k", s0, s1, device), \
        make_kv_slice(w, "v", s0, s1, device)


def token_slice(S: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous split of S tokens over `world` ranks, chunk-aligned where possible."""
    per = -(-S // world)
    if per % CHUNK and S >= world * CHUNK:
        per = -(-per // CHUNK) * CHUNK
    s0 = min(rank * per, S)
    return s0, min(s0 + per, S)


def head_slice(BH: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous split of the B*H heads over `world` ranks."""
    per = -(-BH // world)
    h0 = min(rank * per, BH)
    return h0, min(h0 + per, BH)
