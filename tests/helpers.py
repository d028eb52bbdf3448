"""Helpers shared by the GPU parity tests (device tensors <-> oracle)."""
import numpy as np
import torch

from oracle import oracle as O


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def oracle_int8_reference(q, kq, ks, vq, vs, bs, exact=True):
    """Oracle output (float32 [B,H,D]) on the dequantised K/V.
    exact=True: K/V = code * scale in fp32 (exact), what the reference kernels
    and these kernels compute in registers — the reference for tight bounds.
    exact=False: K/V rounded to fp16 first, as the reference's Python check
    does (python/check_correctness.py:47-56, 121-129) — the reference for its
    1e-2 acceptance bound."""
    kd = O.dequantize(to_np(kq), to_np(ks), bs, exact=exact)
    vd = O.dequantize(to_np(vq), to_np(vs), bs, exact=exact)
    return O.attention(to_np(q).astype(np.float32), kd, vd)


def max_abs(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b))) if a.size else 0.0


def assert_tight(got, ref):
    """|got - ref| <= 1e-3 + |ref| * 2^-10 elementwise: far inside the
    reference's 1e-2 check; the second term is one fp16 ulp of the output."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    bad = np.abs(got - ref) > 1e-3 + np.abs(ref) * 2.0 ** -10
    assert not bad.any(), (np.abs(got - ref)[bad].max(), int(bad.sum()))
