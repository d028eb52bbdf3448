"""tqkv_decode_int8_noalloc — INT8 decode for callers that cannot allocate.

Some callers may not allocate device memory where they run decode: a runtime
whose memory planner owns every buffer, a plugin host that passes a plugin
only its inputs and outputs, an FFI binding with no device allocator.  For
them the library carries a fixed scratch array in its own device memory
(TQKV_NOALLOC_SCRATCH_BYTES per GPU) and this entry point takes no workspace.

These tests call it through the C ABI (ctypes) twice in a row and compare
each result with the workspace-taking entry point tqkv_decode_int8 on the
same inputs.  Both run the same kernel with the same work split and merge
order, so the outputs must be bit-identical (a stricter check than the decode
tests' tolerance, which is asserted as well); they also check that a shape too
large for the array is refused.  This file is collected last, and
it passes both on its own in a fresh process and after the other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

import tqkv
from tqkv import _lib

pytestmark = pytest.mark.gpu

TQKV_OK = 0
TQKV_ERR_WORKSPACE = 4
NOALLOC_SCRATCH_BYTES = 4 * 1024 * 1024   # TQKV_NOALLOC_SCRATCH_BYTES in include/tqkv.h


def _rand(shape, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(shape, generator=g, device="cuda").half()


def _within_decode_tolerance(got, ref):
    # the per-element bound of tests/test_gpu_decode.py: 1e-3 + one fp16 ulp
    got = got.float().cpu().numpy().astype(np.float64)
    ref = ref.float().cpu().numpy().astype(np.float64)
    return bool(np.all(np.abs(got - ref) <= 1e-3 + np.abs(ref) * 2.0 ** -10))


def _noalloc(q, kq, ks, vq, vs, o, bs):
    B, H, S, D = kq.shape
    return _lib.load().tqkv_decode_int8_noalloc(
        q.data_ptr(), kq.data_ptr(), ks.data_ptr(), vq.data_ptr(), vs.data_ptr(), o.data_ptr(),
        B, H, S, D, bs, torch.cuda.current_stream().cuda_stream)


# (B, H, S, D, block size): heads split across many CTAs (the scratch is used),
# then a shape with many short heads
CALLS = [(1, 2, 50000, 128, 64), (2, 8, 2048, 128, 128)]


def test_noalloc_matches_workspace_entry_point_two_calls_in_a_row():
    lib = _lib.load()
    for i, (B, H, S, D, bs) in enumerate(CALLS):
        assert lib.tqkv_decode_workspace_bytes(B, H, S, D) <= NOALLOC_SCRATCH_BYTES
        q = _rand((B, H, D), 10 + i)
        kq, ks = tqkv.kv_compress(_rand((B, H, S, D), 20 + i), bs)
        vq, vs = tqkv.kv_compress(_rand((B, H, S, D), 30 + i), bs)
        o = torch.empty((B, H, D), dtype=torch.float16, device="cuda")
        assert _noalloc(q, kq, ks, vq, vs, o, bs) == TQKV_OK
        ref = tqkv.decode_int8(q, kq, ks, vq, vs, bs)   # the existing entry point
        torch.cuda.synchronize()
        assert torch.equal(o, ref), i
        assert _within_decode_tolerance(o, ref), i
    assert tqkv.read_device_error() == 0


def test_noalloc_repeated_call_same_inputs():
    """Back-to-back calls reuse the array; results stay identical."""
    B, H, S, D, bs = 1, 3, 70000, 128, 32
    q = _rand((B, H, D), 1)
    kq, ks = tqkv.kv_compress(_rand((B, H, S, D), 2), bs)
    vq, vs = tqkv.kv_compress(_rand((B, H, S, D), 3), bs)
    o1 = torch.empty((B, H, D), dtype=torch.float16, device="cuda")
    o2 = torch.empty_like(o1)
    assert _noalloc(q, kq, ks, vq, vs, o1, bs) == TQKV_OK
    assert _noalloc(q, kq, ks, vq, vs, o2, bs) == TQKV_OK
    ref = tqkv.decode_int8(q, kq, ks, vq, vs, bs)
    torch.cuda.synchronize()
    assert torch.equal(o1, ref) and torch.equal(o2, ref)
    assert _within_decode_tolerance(o1, ref)


def test_noalloc_refuses_shapes_beyond_the_array():
    lib = _lib.load()
    B, H, S, D, bs = 64, 64, 1 << 20, 128, 128   # needs far more than 4 MiB of scratch
    assert lib.tqkv_decode_workspace_bytes(B, H, S, D) > NOALLOC_SCRATCH_BYTES
    small8 = torch.zeros(64, dtype=torch.int8, device="cuda")
    small16 = torch.zeros(64, dtype=torch.float16, device="cuda")
    st = lib.tqkv_decode_int8_noalloc(small16.data_ptr(), small8.data_ptr(), small16.data_ptr(),
                                      small8.data_ptr(), small16.data_ptr(), small16.data_ptr(),
                                      B, H, S, D, bs, torch.cuda.current_stream().cuda_stream)
    assert st == TQKV_ERR_WORKSPACE
