"""TEST INFRASTRUCTURE ONLY — the reference's own CPU implementation of the
path, restated: its Python check computes the decode output on the host with
torch in fp32 (reference python/check_correctness.py:38-56):

    dequantize:  fp16(float32(code) * float32(scale))           (:47-56)
    attention:   einsum('bhd,bhsd->bhs') * scale -> softmax -> einsum('bhs,bhsd->bhd'),
                 fp32, cast to fp16                              (:38-44)

bench.py times this on the host cores as the CPU baseline (kind "port"); the
tests use it to pin the C oracle against the reference's own formulation.
"""
from __future__ import annotations

import math

import torch


def dequantize(xq: torch.Tensor, scales: torch.Tensor, block_size: int) -> torch.Tensor:
    """int8 [B,H,S,D] + fp16 [B,H,S,D/bs] -> fp16 [B,H,S,D] (CPU tensors)."""
    s_full = scales.to(torch.float32).repeat_interleave(block_size, dim=-1)
    return (xq.to(torch.float32) * s_full).to(torch.float16)


def attention_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """q [B,H,D], k/v [B,H,S,D] -> fp16 [B,H,D], computed in fp32."""
    D = q.shape[-1]
    qt, kt, vt = q.to(torch.float32), k.to(torch.float32), v.to(torch.float32)
    scores = torch.einsum("bhd,bhsd->bhs", qt, kt) * (1.0 / math.sqrt(D))
    probs = torch.softmax(scores, dim=-1)
    return torch.einsum("bhs,bhsd->bhd", probs, vt).to(torch.float16)


def int8_decode_step(q, kq, ks, vq, vs, block_size: int) -> torch.Tensor:
    """The full INT8 decode step of the reference's CPU path: dequantise K and V,
    then fp32 attention."""
    return attention_fp32(q, dequantize(kq, ks, block_size), dequantize(vq, vs, block_size))
