"""Seeded CPU inputs for the golden fixtures (numpy PCG64 -> fp16).

Shared by the fixture-generating scripts and the tests that check against the
fixtures, so both see bit-identical inputs.  Shapes and distributions follow
the benchmark configurations at sizes the CPU oracle handles in seconds.
"""
import numpy as np

CASES = {
    # name: (B, H, S, D, block_size, seed, dist)
    "fp16_small": (1, 4, 128, 64, 0, 0, "normal"),
    "int8_b2h8": (2, 8, 2048, 128, 64, 1, "normal"),
    "int8_gpt2_outlier": (8, 12, 1024, 64, 64, 3, "outlier_channels"),
    "int8_bs32_lognormal": (2, 4, 1000, 128, 32, 2, "lognormal_channels"),
    "int8_bs128_ragged": (1, 3, 777, 128, 128, 4, "normal"),
}


def inputs(name):
    """(q [B,H,D], k [B,H,S,D], v [B,H,S,D]) as float16 arrays."""
    B, H, S, D, bs, seed, dist = CASES[name]
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, H, D), dtype=np.float32)
    k = rng.standard_normal((B, H, S, D), dtype=np.float32)
    v = rng.standard_normal((B, H, S, D), dtype=np.float32)
    if dist == "lognormal_channels":
        k *= np.exp(0.5 * rng.standard_normal((1, H, 1, D), dtype=np.float32))
        v *= np.exp(0.5 * rng.standard_normal((1, H, 1, D), dtype=np.float32))
    elif dist == "outlier_channels":
        n_out = -(-D // 100)
        for t in (k, v):
            for h in range(H):
                t[:, h, :, rng.choice(D, n_out, replace=False)] *= 10.0
        v += 0.1 * rng.standard_normal((1, H, 1, D), dtype=np.float32)
    return q.astype(np.float16), k.astype(np.float16), v.astype(np.float16)


def tie_rich_rows(D, rows=1024, seed=99):
    """fp16 rows where many elements sit exactly at +-m/2 of their block max
    (the tie class of the quantisation rule), plus zeros and subnormals."""
    rng = np.random.default_rng(seed)
    m = (rng.random((rows, 1)) * 8 + 0.01).astype(np.float16).astype(np.float32)
    pick = rng.integers(0, 5, (rows, D))
    noise = rng.standard_normal((rows, D)).astype(np.float32) * m / 3
    x = np.where(pick == 0, m / 2, np.where(pick == 1, -m / 2, noise))
    x = np.where(pick == 4, m * 2.0 ** -20, x)
    x[:, 0] = m[:, 0]
    x[::17] = 0.0
    return x.astype(np.float16)
