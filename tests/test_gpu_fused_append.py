"""Append fused into decode: tqkv_decode_int8_append quantises the T newest
tokens into rows [S - T, S) of the INT8 cache and attends over rows [0, S) in
one launch.  It must leave exactly the cache bytes tqkv_kv_append writes and
return exactly the O that tqkv_decode_int8_cache gives over that cache (the
same kernel schedule reads the same codes, so the results are bit-identical);
tqkv_decode_int8_cache itself is checked against the oracle in
test_gpu_append.py."""
import ctypes

import pytest
import torch

import tqkv
from tqkv import _lib

from helpers import assert_tight, oracle_int8_reference, to_np

pytestmark = pytest.mark.gpu

VALID = [(64, 32), (64, 64), (128, 32), (128, 64), (128, 128)]


def _rand(shape, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(shape, generator=g, device="cuda").half()


def _case(B, H, D, bs, T, S, S_cap, seed):
    q = _rand((B, H, D), seed)
    kq, ks = tqkv.kv_compress(_rand((B, H, S_cap, D), seed + 1), bs)
    vq, vs = tqkv.kv_compress(_rand((B, H, S_cap, D), seed + 2), bs)
    k_new, v_new = _rand((B, H, T, D), seed + 3), _rand((B, H, T, D), seed + 4)
    return q, kq, ks, vq, vs, k_new, v_new


def _separate(q, kq, ks, vq, vs, k_new, v_new, S, bs):
    kq, ks, vq, vs = kq.clone(), ks.clone(), vq.clone(), vs.clone()
    T = k_new.shape[2]
    tqkv.kv_append(k_new, kq, ks, S - T, bs)
    tqkv.kv_append(v_new, vq, vs, S - T, bs)
    return tqkv.decode_int8_cache(q, kq, ks, vq, vs, S, bs), (kq, ks, vq, vs)


def _poison(kq, ks, vq, vs, S, T):
    """Stale bytes in the rows being appended: the fused kernel must not read them."""
    kq, ks, vq, vs = kq.clone(), ks.clone(), vq.clone(), vs.clone()
    for c in (kq, vq):
        c[:, :, S - T:S] = 55
    for s in (ks, vs):
        s[:, :, S - T:S] = 7.0
    return kq, ks, vq, vs


def _same_cache(a, b):
    for x, y in zip(a, b):
        if x.dtype == torch.float16:
            x, y = x.view(torch.int16), y.view(torch.int16)
        if not torch.equal(x, y):
            return False
    return True


@pytest.mark.parametrize("D,bs", VALID)
@pytest.mark.parametrize("T,S,S_cap", [(1, 1, 1), (1, 100, 100), (1, 4097, 4100), (3, 65, 80),
                                       (7, 129, 200), (64, 64, 64), (130, 2000, 2048),
                                       (1, 20000, 20001)])
def test_fused_append_equals_append_then_decode(D, bs, T, S, S_cap):
    B, H = 2, 3
    q, kq, ks, vq, vs, k_new, v_new = _case(B, H, D, bs, T, S, S_cap, D + bs + T + S)
    ref, ref_cache = _separate(q, kq, ks, vq, vs, k_new, v_new, S, bs)
    cache = _poison(kq, ks, vq, vs, S, T)
    o = tqkv.decode_int8_append(q, k_new, v_new, *cache, S, bs)
    torch.cuda.synchronize()
    assert _same_cache(cache, ref_cache)
    assert torch.equal(o, ref)
    assert tqkv.read_device_error() == 0


def test_fused_append_matches_oracle_and_leaves_other_rows():
    B, H, D, bs, T, S, S_cap = 2, 4, 128, 64, 2, 3000, 3010
    q, kq, ks, vq, vs, k_new, v_new = _case(B, H, D, bs, T, S, S_cap, 5)
    cache = _poison(kq, ks, vq, vs, S, T)
    before = [c.clone() for c in cache]
    o = tqkv.decode_int8_append(q, k_new, v_new, *cache, S, bs)
    torch.cuda.synchronize()
    for c, b in zip(cache, before):   # rows outside [S - T, S) untouched
        assert torch.equal(c[:, :, :S - T], b[:, :, :S - T])
        assert torch.equal(c[:, :, S:], b[:, :, S:])
    kq1, ks1, vq1, vs1 = cache
    ref = oracle_int8_reference(q, kq1[:, :, :S], ks1[:, :, :S], vq1[:, :, :S], vs1[:, :, :S], bs)
    assert_tight(to_np(o), ref)


def test_fused_append_decode_loop():
    """Prefill, then per step one fused call per new token; every step equals
    the separate append + decode sequence on its own cache."""
    B, H, D, bs, S0, steps = 2, 4, 128, 128, 2000, 5
    S_cap = S0 + steps
    q, kq, ks, vq, vs, _, _ = _case(B, H, D, bs, 1, S0, S_cap, 9)
    fused = [c.clone() for c in (kq, ks, vq, vs)]
    sep = [c.clone() for c in (kq, ks, vq, vs)]
    ws = tqkv.Workspace()
    for i in range(steps):
        S = S0 + 1 + i
        k_new, v_new = _rand((B, H, 1, D), 40 + i), _rand((B, H, 1, D), 60 + i)
        q = _rand((B, H, D), 80 + i)
        o = tqkv.decode_int8_append(q, k_new, v_new, *fused, S, bs, workspace=ws)
        tqkv.kv_append(k_new, sep[0], sep[1], S - 1, bs)
        tqkv.kv_append(v_new, sep[2], sep[3], S - 1, bs)
        ref = tqkv.decode_int8_cache(q, *sep, S, bs, workspace=ws)
        torch.cuda.synchronize()
        assert torch.equal(o, ref), i
    assert _same_cache(fused, sep)


def test_fused_append_publish_single_rank():
    """The kOutPeers epilogue with the fused append, world = 1."""
    B, H, D, bs, T, S, S_cap = 2, 3, 128, 32, 1, 5000, 5000
    q, kq, ks, vq, vs, k_new, v_new = _case(B, H, D, bs, T, S, S_cap, 11)
    _, ref_cache = _separate(q, kq, ks, vq, vs, k_new, v_new, S, bs)
    cache = _poison(kq, ks, vq, vs, S, T)
    ex = tqkv.LocalExchange(B * H, D)
    try:
        out = torch.empty((B, H, D), dtype=torch.float16, device="cuda")
        for _ in range(3):   # steps alternate record slots
            ex.publish_append(q, k_new, v_new, *cache, S, bs)
            ex.combine(out)
        torch.cuda.synchronize()
    finally:
        ex.close()
    assert _same_cache(cache, ref_cache)
    kq1, ks1, vq1, vs1 = cache
    assert_tight(to_np(out), oracle_int8_reference(q, kq1, ks1, vq1, vs1, bs))


def test_fused_append_rejects_bad_arguments():
    lib = _lib.load()
    B, H, D, bs = 1, 2, 128, 64
    t = torch.zeros(4096, dtype=torch.float16, device="cuda")
    p = t.data_ptr()
    s = torch.cuda.current_stream().cuda_stream

    def call(T, S, S_cap, k_new=p, D_=D, bs_=bs):
        return lib.tqkv_decode_int8_append(p, k_new, p, p, p, p, p, p, B, H, T, S, S_cap, D_,
                                           bs_, None, 0, s)
    assert call(0, 4, 4) == 2          # T >= 1
    assert call(5, 4, 4) == 2          # T <= S
    assert call(1, 5, 4) == 2          # S <= S_cap
    assert call(1, 4, 4, k_new=p + 2) == 3
    assert call(1, 4, 4, D_=96) == 1
    assert call(1, 4, 4, bs_=256) == 1
    assert lib.tqkv_decode_int8_append(p, None, p, p, p, p, p, p, B, H, 1, 4, 4, D, bs, None, 0,
                                       s) == 6
