"""The split-S exchange step on one GPU: the one-launch form
(tqkv_decode_int8_exchange: decode, record exchange and merge in one
launch) against the two-launch form (publish + combine) and the
plain decode; ranks whose token slice is empty; and the bounded waits for
peer records running out.

With one rank the exchange has nobody to wait for, and the merge of one
record per head is the plain decode's own arithmetic, so all three forms must
agree bit for bit.  The multi-GPU form of the same step is tested in
tests/test_gpu_multi.py.

Timeouts are made the permitted way: records that nothing writes.  A combine
launched without any publish, and a one-launch step told that a second rank
exists whose buffer is a local allocation nobody writes, each wait about a
second, then return with the device error flag set to 4 and NaN in O; the
context stays usable and a fresh exchange works afterwards."""
import ctypes
import time

import numpy as np
import pytest
import torch

import tqkv
from tqkv import _lib

from helpers import assert_tight, oracle_int8_reference, to_np

pytestmark = pytest.mark.gpu

PEER_WAIT_TIMEOUT = 4   # kErrPeerWaitTimeout (csrc/device_common.cuh)


def _rand(shape, seed, scale=1.0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return (torch.randn(shape, generator=g, device="cuda") * scale).half()


def _kv(B, H, S, D, bs, seed):
    kq, ks = tqkv.kv_compress(_rand((B, H, S, D), seed), bs)
    vq, vs = tqkv.kv_compress(_rand((B, H, S, D), seed + 1), bs)
    return kq, ks, vq, vs


# (B, H, S, D, block size): one run per CTA; dynamic chunks (at least 16384
# rows per CTA); a single chunk (tiny, no cut heads); D = 64
SHAPES = [(2, 5, 9000, 128, 128), (1, 8, 1300000, 128, 128), (1, 1, 40, 128, 32),
          (3, 4, 5000, 64, 32)]


@pytest.mark.parametrize("B,H,S,D,bs", SHAPES)
def test_one_launch_step_equals_two_launches_and_decode(B, H, S, D, bs):
    kq, ks, vq, vs = _kv(B, H, S, D, bs, 11)
    one, two = tqkv.LocalExchange(B * H, D), tqkv.LocalExchange(B * H, D)
    ws = tqkv.Workspace()
    try:
        for step in range(4):      # both record slots, twice
            q = _rand((B, H, D), 100 + step)
            o1 = one.step(q, kq, ks, vq, vs, bs, torch.empty((B, H, D), dtype=torch.float16,
                                                             device="cuda"), workspace=ws)
            two.publish(q, kq, ks, vq, vs, bs, workspace=ws)
            o2 = two.combine(torch.empty((B, H, D), dtype=torch.float16, device="cuda"))
            ref = tqkv.decode_int8(q, kq, ks, vq, vs, bs, workspace=ws)
            torch.cuda.synchronize()
            assert torch.equal(o1, o2), step
            assert torch.equal(o1, ref), step
        if B * H * S <= 200000:    # the float64 oracle, where it finishes in seconds
            assert_tight(to_np(o1), oracle_int8_reference(q, kq, ks, vq, vs, bs))
        assert tqkv.read_device_error() == 0
        # the one-launch kernel left the shared workspace as it found it
        kq2, ks2, vq2, vs2 = _kv(2, 3, 7000, D, bs, 40)
        q2 = _rand((2, 3, D), 41)
        o = tqkv.decode_int8(q2, kq2, ks2, vq2, vs2, bs, workspace=ws)
        torch.cuda.synchronize()
        assert_tight(to_np(o), oracle_int8_reference(q2, kq2, ks2, vq2, vs2, bs))
    finally:
        one.close()
        two.close()


def test_one_launch_and_two_launch_steps_interleave():
    """A sequence of steps may use either form, step by step."""
    B, H, S, D, bs = 2, 4, 6000, 128, 128
    kq, ks, vq, vs = _kv(B, H, S, D, bs, 21)
    ex = tqkv.LocalExchange(B * H, D)
    try:
        for step in range(6):
            q = _rand((B, H, D), 200 + step)
            out = torch.empty((B, H, D), dtype=torch.float16, device="cuda")
            if step % 3 == 1:
                ex.publish(q, kq, ks, vq, vs, bs)
                ex.combine(out)
            else:
                ex.step(q, kq, ks, vq, vs, bs, out)
            ref = tqkv.decode_int8(q, kq, ks, vq, vs, bs)
            torch.cuda.synchronize()
            assert torch.equal(out, ref), step
        assert tqkv.read_device_error() == 0
    finally:
        ex.close()


def test_one_launch_step_with_fused_append():
    """step_append: the newest tokens quantised into the cache inside the same
    launch; equals publish_append + combine and decode_int8_append."""
    B, H, S, D, bs, T = 2, 3, 5000, 128, 64, 2
    S_cap = S + 16
    kq, ks, vq, vs = _kv(B, H, S_cap, D, bs, 31)
    caches = [[t.clone() for t in (kq, ks, vq, vs)] for _ in range(3)]
    one, two = tqkv.LocalExchange(B * H, D), tqkv.LocalExchange(B * H, D)
    try:
        for step in range(3):
            kn, vn = _rand((B, H, T, D), 300 + step), _rand((B, H, T, D), 310 + step)
            q = _rand((B, H, D), 320 + step)
            n = S + T * (step + 1)
            o1 = one.step_append(q, kn, vn, *caches[0], n, bs,
                                 torch.empty((B, H, D), dtype=torch.float16, device="cuda"))
            two.publish_append(q, kn, vn, *caches[1], n, bs)
            o2 = two.combine(torch.empty((B, H, D), dtype=torch.float16, device="cuda"))
            ref = tqkv.decode_int8_append(q, kn, vn, *caches[2], n, bs)
            torch.cuda.synchronize()
            assert torch.equal(o1, o2) and torch.equal(o1, ref), step
            for a, b in zip(caches[0], caches[2]):
                assert torch.equal(a, b), step
        assert tqkv.read_device_error() == 0
    finally:
        one.close()
        two.close()


def test_empty_slice_publishes_empty_records():
    """A rank with S == 0 publishes m = -inf, l = 0, acc = 0: with one rank O
    is NaN (0 * (1/0)), as the plain decode gives for S == 0; the step
    counter still advances, so the next step is right."""
    B, H, D, bs = 2, 3, 128, 128
    empty = [torch.empty((B, H, 0, D), dtype=torch.int8, device="cuda"),
             torch.empty((B, H, 0, 1), dtype=torch.float16, device="cuda")] * 2
    kq, ks, vq, vs = _kv(B, H, 3000, D, bs, 51)
    ex = tqkv.LocalExchange(B * H, D)
    try:
        q = _rand((B, H, D), 52)
        o = ex.step(q, *empty, bs, torch.empty((B, H, D), dtype=torch.float16, device="cuda"))
        ex.publish(q, *empty, bs)
        o2 = ex.combine(torch.empty((B, H, D), dtype=torch.float16, device="cuda"))
        torch.cuda.synchronize()
        assert torch.isnan(o.float()).all() and torch.isnan(o2.float()).all()
        for form in ("one", "two"):
            out = torch.empty((B, H, D), dtype=torch.float16, device="cuda")
            if form == "one":
                ex.step(q, kq, ks, vq, vs, bs, out)
            else:
                ex.publish(q, kq, ks, vq, vs, bs)
                ex.combine(out)
            ref = tqkv.decode_int8(q, kq, ks, vq, vs, bs)
            torch.cuda.synchronize()
            assert torch.equal(out, ref), form
        assert tqkv.read_device_error() == 0
    finally:
        ex.close()


def test_combine_without_publish_times_out():
    """The two-launch combine waits for records nobody publishes: about a
    second later it returns, with the device error flag at 4 and O NaN."""
    assert tqkv.read_device_error() == 0
    ex = tqkv.LocalExchange(2, 128)
    try:
        out = torch.zeros((1, 2, 128), dtype=torch.float16, device="cuda")
        t0 = time.monotonic()
        ex.combine(out)
        torch.cuda.synchronize()
        waited = time.monotonic() - t0
        assert tqkv.read_device_error() == PEER_WAIT_TIMEOUT
        assert torch.isnan(out.float()).all()
        assert 0.2 < waited < 30, waited
    finally:
        ex.close()
    # a fresh exchange works, and the flag stays clear
    B, H, D, bs = 1, 2, 128, 128
    kq, ks, vq, vs = _kv(B, H, 4000, D, bs, 61)
    q = _rand((B, H, D), 62)
    ex = tqkv.LocalExchange(B * H, D)
    try:
        ex.publish(q, kq, ks, vq, vs, bs)
        o = ex.combine(torch.empty((B, H, D), dtype=torch.float16, device="cuda"))
        ref = tqkv.decode_int8(q, kq, ks, vq, vs, bs)
        torch.cuda.synchronize()
        assert torch.equal(o, ref)
        assert tqkv.read_device_error() == 0
    finally:
        ex.close()


def test_one_launch_step_times_out_on_a_silent_peer():
    """The one-launch step with world = 2 on one GPU, where rank 1's buffer is
    a local allocation that no process writes: rank 0 publishes into both
    buffers, then waits for rank 1's records, gives up after about a second,
    and returns with the device error flag at 4 and O NaN."""
    lib = _lib.load()
    B, H, S, D, bs = 1, 2, 4000, 128, 128
    BH = B * H
    kq, ks, vq, vs = _kv(B, H, S, D, bs, 71)
    q = _rand((B, H, D), 72)
    nbytes = int(lib.tqkv_exchange_bytes(2, BH, D))
    bufs = []
    for _ in range(2):
        p = ctypes.c_void_p()
        assert lib.tqkv_exchange_alloc(nbytes, ctypes.byref(p)) == 0
        bufs.append(p.value)
    arr = (ctypes.c_void_p * 2)(*bufs)
    ws = tqkv.Workspace()
    wptr, wbytes = ws.get(tqkv.workspace_bytes(B, H, S, D))
    out = torch.zeros((B, H, D), dtype=torch.float16, device="cuda")
    try:
        t0 = time.monotonic()
        st = lib.tqkv_decode_int8_exchange(
            q.data_ptr(), kq.data_ptr(), ks.data_ptr(), vq.data_ptr(), vs.data_ptr(),
            out.data_ptr(), B, H, S, D, bs, wptr, wbytes, arr, 2, 0,
            torch.cuda.current_stream().cuda_stream)
        assert st == 0
        torch.cuda.synchronize()
        waited = time.monotonic() - t0
        assert tqkv.read_device_error() == PEER_WAIT_TIMEOUT
        assert torch.isnan(out.float()).all()
        assert 0.2 < waited < 30, waited
        # what rank 0 published into "rank 1"'s buffer: every entry of its
        # records in slot 1 carries step 1
        host = (ctypes.c_uint8 * nbytes)()
        cudart = ctypes.CDLL("libcudart.so.12")
        assert cudart.cudaMemcpy(host, ctypes.c_void_p(bufs[1]), ctypes.c_size_t(nbytes), 2) == 0
        hdr = 512   # kExchangeHeaderBytes
        n = 2 * 2 * BH * (D + 2)
        rec = np.frombuffer(bytes(host)[hdr:hdr + 8 * n], dtype=np.uint64).reshape(2, 2, BH, D + 2)
        assert ((rec[1, 0] >> np.uint64(32)) == 1).all()
    finally:
        torch.cuda.synchronize()
        for p in bufs:
            lib.tqkv_exchange_free(p)
    # the context is usable and a normal step works afterwards
    ex = tqkv.LocalExchange(BH, D)
    try:
        o = ex.step(q, kq, ks, vq, vs, bs, torch.empty((B, H, D), dtype=torch.float16,
                                                      device="cuda"))
        ref = tqkv.decode_int8(q, kq, ks, vq, vs, bs)
        torch.cuda.synchronize()
        assert torch.equal(o, ref)
        assert tqkv.read_device_error() == 0
    finally:
        ex.close()
