"""Incremental decode: tqkv_kv_append writes new tokens into a preallocated
INT8 cache (bit-identical to compressing those rows in place), and
tqkv_decode_int8_cache attends over the first S rows of such a cache."""
import numpy as np
import pytest
import torch

import tqkv
from oracle import oracle as O

from helpers import max_abs, oracle_int8_reference, to_np

pytestmark = pytest.mark.gpu

VALID = [(64, 32), (64, 64), (128, 32), (128, 64), (128, 128)]


def _rand(shape, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(shape, generator=g, device="cuda").half()


@pytest.mark.parametrize("D,bs", VALID)
@pytest.mark.parametrize("T,t0,S_cap", [(1, 0, 1), (1, 99, 100), (7, 13, 64), (64, 0, 64),
                                        (5, 1000, 2048)])
def test_append_matches_in_place_compress(D, bs, T, t0, S_cap):
    B, H = 2, 3
    x_full = _rand((B, H, S_cap, D), D + bs + T)
    q_full, s_full = tqkv.kv_compress(x_full, bs)
    cache_q = torch.full((B, H, S_cap, D), 55, dtype=torch.int8, device="cuda")
    cache_s = torch.full((B, H, S_cap, D // bs), 7.0, dtype=torch.float16, device="cuda")
    x_new = x_full[:, :, t0:t0 + T].contiguous()
    tqkv.kv_append(x_new, cache_q, cache_s, t0, bs)
    torch.cuda.synchronize()
    assert torch.equal(cache_q[:, :, t0:t0 + T], q_full[:, :, t0:t0 + T])
    assert torch.equal(cache_s[:, :, t0:t0 + T].view(torch.int16),
                       s_full[:, :, t0:t0 + T].view(torch.int16))
    # rows outside [t0, t0 + T) untouched
    mask = torch.ones(S_cap, dtype=torch.bool, device="cuda")
    mask[t0:t0 + T] = False
    assert bool((cache_q[:, :, mask] == 55).all()) and bool((cache_s[:, :, mask] == 7.0).all())


@pytest.mark.parametrize("D,bs", [(128, 128), (128, 32), (64, 64)])
@pytest.mark.parametrize("S,S_cap", [(1, 8), (777, 1000), (4097, 4100), (20000, 32768)])
def test_cache_decode_equals_contiguous_decode(D, bs, S, S_cap):
    B, H = 2, 3
    q = _rand((B, H, D), S)
    k, v = _rand((B, H, S_cap, D), S + 1), _rand((B, H, S_cap, D), S + 2)
    kq, ks = tqkv.kv_compress(k, bs)
    vq, vs = tqkv.kv_compress(v, bs)
    o = tqkv.decode_int8_cache(q, kq, ks, vq, vs, S, bs)
    ref = tqkv.decode_int8(q, kq[:, :, :S].contiguous(), ks[:, :, :S].contiguous(),
                           vq[:, :, :S].contiguous(), vs[:, :, :S].contiguous(), bs)
    torch.cuda.synchronize()
    assert torch.equal(o, ref)


def test_decode_loop_append_then_attend():
    """Prefill S0 tokens, then per step append one token's K and V and attend
    over everything so far; every step matches the oracle."""
    B, H, D, bs, S0, steps = 2, 4, 128, 64, 3000, 6
    S_cap = S0 + steps
    k_all, v_all = _rand((B, H, S_cap, D), 1), _rand((B, H, S_cap, D), 2)
    kq = torch.empty((B, H, S_cap, D), dtype=torch.int8, device="cuda")
    vq = torch.empty_like(kq)
    ks = torch.empty((B, H, S_cap, D // bs), dtype=torch.float16, device="cuda")
    vs = torch.empty_like(ks)
    tqkv.kv_append(k_all[:, :, :S0].contiguous(), kq, ks, 0, bs)
    tqkv.kv_append(v_all[:, :, :S0].contiguous(), vq, vs, 0, bs)
    for i in range(steps):
        t = S0 + i
        tqkv.kv_append(k_all[:, :, t:t + 1].contiguous(), kq, ks, t, bs)
        tqkv.kv_append(v_all[:, :, t:t + 1].contiguous(), vq, vs, t, bs)
        q = _rand((B, H, D), 100 + i)
        o = tqkv.decode_int8_cache(q, kq, ks, vq, vs, t + 1, bs)
        torch.cuda.synchronize()
        ref = oracle_int8_reference(q, kq[:, :, :t + 1], ks[:, :, :t + 1], vq[:, :, :t + 1],
                                    vs[:, :, :t + 1], bs)
        got = to_np(o).astype(np.float64)
        assert np.all(np.abs(got - ref) <= 1e-3 + np.abs(ref) * 2.0 ** -10), i
    # the whole cache equals a one-shot compress
    kq_ref, _ = tqkv.kv_compress(k_all, bs)
    torch.cuda.synchronize()
    assert torch.equal(kq, kq_ref)


def test_append_rejects_out_of_range_rows():
    x = _rand((1, 1, 4, 64), 3)
    cache_q = torch.zeros((1, 1, 8, 64), dtype=torch.int8, device="cuda")
    cache_s = torch.zeros((1, 1, 8, 2), dtype=torch.float16, device="cuda")
    with pytest.raises(tqkv.TqkvError):
        tqkv.kv_append(x, cache_q, cache_s, 5, 32)       # 5 + 4 > 8
    with pytest.raises(tqkv.TqkvError):
        tqkv.kv_append(x, cache_q, cache_s, -1, 32)
