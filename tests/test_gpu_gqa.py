"""Grouped-query / multi-query decode (tqkv_decode_int8_gqa): query head h
attends over K/V head h // (H_q // H_kv).  The result must equal
tqkv_decode_int8 on K/V whose heads are repeated H_q // H_kv times (same
schedule, same codes: bit-identical) and stay within the tight bound of the
oracle."""
import pytest
import torch

import tqkv
from tqkv import _lib

from helpers import assert_tight, oracle_int8_reference, to_np

pytestmark = pytest.mark.gpu


def _rand(shape, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(shape, generator=g, device="cuda").half()


@pytest.mark.parametrize("D,bs", [(128, 128), (128, 32), (64, 64)])
@pytest.mark.parametrize("B,H_q,H_kv,S", [(2, 8, 2, 1000), (1, 32, 8, 20000), (3, 6, 1, 257),
                                          (2, 4, 4, 4097), (1, 16, 1, 70000)])
def test_gqa_equals_repeated_heads(D, bs, B, H_q, H_kv, S):
    q = _rand((B, H_q, D), S + H_q)
    kq, ks = tqkv.kv_compress(_rand((B, H_kv, S, D), S + 1), bs)
    vq, vs = tqkv.kv_compress(_rand((B, H_kv, S, D), S + 2), bs)
    o = tqkv.decode_int8_gqa(q, kq, ks, vq, vs, bs)
    g = H_q // H_kv
    rep = [t.repeat_interleave(g, dim=1).contiguous() for t in (kq, ks, vq, vs)]
    ref = tqkv.decode_int8(q, *rep, bs)
    torch.cuda.synchronize()
    assert torch.equal(o, ref)
    assert tqkv.read_device_error() == 0
    if S <= 4097:
        assert_tight(to_np(o), oracle_int8_reference(q, *[t.cpu() for t in rep], bs))


def test_gqa_rejects_bad_groups():
    lib = _lib.load()
    t = torch.zeros(4096, dtype=torch.float16, device="cuda")
    p, s = t.data_ptr(), torch.cuda.current_stream().cuda_stream
    assert lib.tqkv_decode_int8_gqa(p, p, p, p, p, p, 1, 6, 4, 8, 128, 64, None, 0, s) == 2
    assert lib.tqkv_decode_int8_gqa(p, p, p, p, p, p, 1, 6, 0, 8, 128, 64, None, 0, s) == 2
    assert lib.tqkv_decode_int8_gqa(p, p, p, p, p, p, 1, 6, 3, 8, 96, 64, None, 0, s) == 1
