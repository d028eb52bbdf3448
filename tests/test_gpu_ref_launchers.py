"""The reference-signature C++ launchers (include/attention.h,
include/quantization.h) called through their exported mangled symbols: same
results as the C ABI, and the reference's edge behaviour (empty grids leave
cudaErrorInvalidConfiguration pending; S == 0 gives NaN for the online
kernel and 0 for the two-pass and baseline kernels)."""
import ctypes
import os

import numpy as np
import pytest
import torch

import tqkv
from tqkv import _lib
from oracle import oracle as O

from helpers import max_abs, oracle_int8_reference, to_np

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(REPO, "oracle", "_ref", "libtqkv_ref.so")
CUDA_ERROR_INVALID_CONFIGURATION = 9


def _s():
    return torch.cuda.current_stream().cuda_stream


def _rand(shape, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(shape, generator=g, device="cuda").half()


def _pending_cuda_error() -> int:
    """cudaGetLastError() of the process's (shared) CUDA runtime — the same
    instance libtqkv_b200.so is linked against."""
    rt = ctypes.CDLL("libcudart.so.12")
    rt.cudaGetLastError.restype = ctypes.c_int
    return rt.cudaGetLastError()


@pytest.mark.parametrize("D,bs", [(64, 32), (128, 64), (128, 128)])
def test_launchers_match_c_abi(D, bs):
    B, H, S = 2, 3, 1500
    x = _rand((B, H, S, D), 1)
    q = _rand((B, H, D), 2)
    v = _rand((B, H, S, D), 3)
    kq, ks = tqkv.kv_compress(x, bs)
    vq, vs = tqkv.kv_compress(v, bs)

    kq2, ks2 = torch.empty_like(kq), torch.empty_like(ks)
    _lib.ref_launcher("launch_kv_compress")(x.data_ptr(), kq2.data_ptr(), ks2.data_ptr(),
                                            B, H, S, D, bs, _s())
    y = torch.empty_like(x)
    _lib.ref_launcher("launch_kv_reconstruct")(kq.data_ptr(), ks.data_ptr(), y.data_ptr(),
                                               B, H, S, D, bs, _s())
    o_on = torch.empty_like(q)
    _lib.ref_launcher("launch_decode_attn_int8_fused_online")(
        q.data_ptr(), kq.data_ptr(), ks.data_ptr(), vq.data_ptr(), vs.data_ptr(), o_on.data_ptr(),
        B, H, S, D, bs, 2, 32, _s())
    o_fu = torch.empty_like(q)
    _lib.ref_launcher("launch_decode_attn_int8_fused")(
        q.data_ptr(), kq.data_ptr(), ks.data_ptr(), vq.data_ptr(), vs.data_ptr(), o_fu.data_ptr(),
        B, H, S, D, bs, _s())
    o_16 = torch.empty_like(q)
    _lib.ref_launcher("launch_decode_attn_baseline")(
        q.data_ptr(), x.data_ptr(), v.data_ptr(), o_16.data_ptr(), B, H, S, D, _s())
    torch.cuda.synchronize()

    assert torch.equal(kq2, kq) and torch.equal(ks2.view(torch.int16), ks.view(torch.int16))
    assert torch.equal(y, tqkv.kv_reconstruct(kq, ks, bs))
    o_abi = tqkv.decode_int8(q, kq, ks, vq, vs, bs)
    torch.cuda.synchronize()
    assert torch.equal(o_on, o_abi) and torch.equal(o_fu, o_abi)
    assert max_abs(to_np(o_on), oracle_int8_reference(q, kq, ks, vq, vs, bs)) < 2e-3
    assert max_abs(to_np(o_16), O.attention(to_np(q), to_np(x), to_np(v))) < 2e-3


def test_launchers_s_zero_semantics():
    B, H, D, bs = 1, 2, 128, 64
    q = _rand((B, H, D), 9)
    e8 = torch.zeros(16, dtype=torch.int8, device="cuda")
    e16 = torch.zeros(16, dtype=torch.float16, device="cuda")
    o = torch.empty_like(q)
    _lib.ref_launcher("launch_decode_attn_int8_fused_online")(
        q.data_ptr(), e8.data_ptr(), e16.data_ptr(), e8.data_ptr(), e16.data_ptr(), o.data_ptr(),
        B, H, 0, D, bs, 4, 32, _s())
    torch.cuda.synchronize()
    assert torch.isnan(o.float()).all()
    o.fill_(1.0)
    _lib.ref_launcher("launch_decode_attn_int8_fused")(
        q.data_ptr(), e8.data_ptr(), e16.data_ptr(), e8.data_ptr(), e16.data_ptr(), o.data_ptr(),
        B, H, 0, D, bs, _s())
    torch.cuda.synchronize()
    assert (o.float() == 0).all()
    o.fill_(1.0)
    _lib.ref_launcher("launch_decode_attn_baseline")(
        q.data_ptr(), e16.data_ptr(), e16.data_ptr(), o.data_ptr(), B, H, 0, D, _s())
    torch.cuda.synchronize()
    assert (o.float() == 0).all()


@pytest.mark.skipif(not os.path.exists(REF_LIB), reason="reference build not present")
@pytest.mark.parametrize("D,bs,L,T", [(128, 64, 4, 32), (128, 128, 2, 64), (64, 32, 2, 32)])
def test_online_output_vs_reference_build(D, bs, L, T):
    """The reference's own Kernel D on the same device buffers: both outputs
    are the same function, so they agree to well inside the 1e-2 contract."""
    lib = ctypes.CDLL(REF_LIB)
    P = ctypes.c_void_p
    lib.ref_decode_int8_online.argtypes = [P] * 6 + [ctypes.c_int] * 7 + [P]
    B, H, S = 2, 8, 2048
    q = _rand((B, H, D), 41)
    k, v = _rand((B, H, S, D), 42), _rand((B, H, S, D), 43)
    kq, ks = tqkv.kv_compress(k, bs)
    vq, vs = tqkv.kv_compress(v, bs)
    o = tqkv.decode_int8(q, kq, ks, vq, vs, bs)
    o_ref = torch.empty_like(o)
    lib.ref_decode_int8_online(q.data_ptr(), kq.data_ptr(), ks.data_ptr(), vq.data_ptr(),
                               vs.data_ptr(), o_ref.data_ptr(), B, H, S, D, bs, L, T, _s())
    torch.cuda.synchronize()
    assert max_abs(to_np(o), to_np(o_ref)) < 2e-3


@pytest.mark.parametrize("B,H,S", [(0, 2, 10), (2, 0, 10), (2, 2, 0)])
def test_empty_grid_leaves_invalid_configuration_pending(B, H, S):
    """The reference launches <<<B*H*S, D>>> (compress) and <<<(B, H), ...>>>
    (attention); an empty grid leaves cudaErrorInvalidConfiguration for the
    caller's cudaGetLastError().  The launchers here do the same."""
    buf = torch.zeros(1 << 16, dtype=torch.float16, device="cuda")
    b8 = torch.zeros(1 << 16, dtype=torch.int8, device="cuda")
    torch.cuda.synchronize()
    _pending_cuda_error()  # clear
    _lib.ref_launcher("launch_kv_compress")(buf.data_ptr(), b8.data_ptr(), buf.data_ptr(),
                                            B, H, S, 128, 64, _s())
    assert _pending_cuda_error() == CUDA_ERROR_INVALID_CONFIGURATION
    if S != 0:
        _lib.ref_launcher("launch_decode_attn_int8_fused_online")(
            buf.data_ptr(), b8.data_ptr(), buf.data_ptr(), b8.data_ptr(), buf.data_ptr(),
            buf.data_ptr(), B, H, S, 128, 64, 4, 32, _s())
        assert _pending_cuda_error() == CUDA_ERROR_INVALID_CONFIGURATION
    assert _pending_cuda_error() == 0
