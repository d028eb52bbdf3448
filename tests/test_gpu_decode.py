"""GPU parity of the decode attention kernels against the CPU oracle.

The reference's acceptance threshold is max_abs < 1e-2 on the INT8 output
against fp32 attention over the dequantised K/V, and on the FP16 output
against fp32 attention (reference python/check_correctness.py:25-26,
78, 128).  The B200 kernels are held to that bound and to a much tighter per-element
one (tight(): 1e-3 plus one fp16 ulp of the output) that catches numerical
regressions long before the contract would.
"""
import numpy as np
import pytest
import torch

import tqkv
from tqkv import workloads as W
from oracle import oracle as O

from helpers import max_abs, oracle_int8_reference, to_np

pytestmark = pytest.mark.gpu

REF_TOL = 1e-2   # reference contract (check_correctness.py:26)


def tight(ref) -> np.ndarray:
    """Per-element bound far inside the contract: 1e-3 absolute plus one fp16
    ulp of the output (the kernel's output is fp16, the oracle's is not; an
    output of magnitude 8..16 alone carries up to 2^-8 of rounding)."""
    return 1e-3 + np.abs(np.asarray(ref, dtype=np.float64)) * 2.0 ** -10


def assert_tight(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    bad = np.abs(got - ref) > tight(ref)
    assert not bad.any(), (np.abs(got - ref)[bad].max(), int(bad.sum()))


def _compress_kv(k, v, bs):
    kq, ks = tqkv.kv_compress(k, bs)
    vq, vs = tqkv.kv_compress(v, bs)
    return kq, ks, vq, vs


def _rand(shape, seed, scale=1.0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return (torch.randn(shape, generator=g, device="cuda") * scale).half()


@pytest.mark.parametrize("name", ["int8_b2h8", "int8_gpt2_outlier"])
def test_int8_decode_full_config(name):
    w = W.WORKLOADS[name]
    q, k, v = W.make_inputs(w)
    kq, ks, vq, vs = _compress_kv(k, v, w.block_size)
    o = tqkv.decode_int8(q, kq, ks, vq, vs, w.block_size)
    torch.cuda.synchronize()
    ref = oracle_int8_reference(q, kq, ks, vq, vs, w.block_size, exact=False)
    err = max_abs(to_np(o), ref)
    assert err < REF_TOL, err
    assert_tight(to_np(o), oracle_int8_reference(q, kq, ks, vq, vs, w.block_size))
    assert tqkv.read_device_error() == 0


@pytest.mark.parametrize("name,heads", [("int8_bh_shard", [0, 1, 257, 511]),
                                        ("int8_longctx", [0, 63, 127])])
def test_int8_decode_large_config_sampled_heads(name, heads):
    """Full-size configurations: the whole step runs on the GPU; a sample of
    heads is checked against the oracle."""
    w = W.WORKLOADS[name]
    q, k, v = W.make_inputs(w)
    kq, ks, vq, vs = _compress_kv(k, v, w.block_size)
    del k, v
    o = tqkv.decode_int8(q, kq, ks, vq, vs, w.block_size)
    torch.cuda.synchronize()
    qf, of = q.reshape(w.BH, w.D), o.reshape(w.BH, w.D)
    kqf, vqf = kq.reshape(w.BH, w.S, w.D), vq.reshape(w.BH, w.S, w.D)
    ksf, vsf = ks.reshape(w.BH, w.S, -1), vs.reshape(w.BH, w.S, -1)
    for h in heads:
        ref = oracle_int8_reference(qf[h][None, None], kqf[h][None, None], ksf[h][None, None],
                                    vqf[h][None, None], vsf[h][None, None], w.block_size)
        assert_tight(to_np(of[h]), ref.reshape(-1))
    assert torch.isfinite(o.float()).all()
    assert tqkv.read_device_error() == 0


SHAPES = [(1, 1, 1), (1, 2, 2), (2, 1, 7), (1, 3, 63), (1, 1, 64), (2, 2, 65), (1, 2, 127),
          (3, 1, 129), (1, 2, 1000), (1, 2, 4097), (2, 3, 300), (1, 1, 20000)]


@pytest.mark.parametrize("D,bs", [(64, 32), (64, 64), (128, 32), (128, 64), (128, 128)])
@pytest.mark.parametrize("B,H,S", SHAPES)
def test_int8_decode_ragged_shapes(B, H, S, D, bs):
    """S = 1, S not a multiple of the tile, heads split across CTAs."""
    seed = B * 1000003 + H * 1009 + S * 7 + D + bs
    q = _rand((B, H, D), seed)
    k = _rand((B, H, S, D), seed + 1)
    v = _rand((B, H, S, D), seed + 2)
    kq, ks, vq, vs = _compress_kv(k, v, bs)
    o = tqkv.decode_int8(q, kq, ks, vq, vs, bs)
    torch.cuda.synchronize()
    assert_tight(to_np(o), oracle_int8_reference(q, kq, ks, vq, vs, bs))


def test_int8_decode_unaligned_scales_and_q():
    """Scale arrays and q that start 2 bytes past a 16-byte boundary: the
    producer's ragged-edge loads, and the consumers' scalar q path."""
    B, H, S, D, bs = 2, 3, 1001, 128, 128
    q0 = _rand((B * H * D + 8,), 11)
    k = _rand((B, H, S, D), 12)
    v = _rand((B, H, S, D), 13)
    kq, ks, vq, vs = _compress_kv(k, v, bs)
    ks_buf = torch.empty(ks.numel() + 8, dtype=torch.float16, device="cuda")
    vs_buf = torch.empty(vs.numel() + 8, dtype=torch.float16, device="cuda")
    ks_u = ks_buf[1:1 + ks.numel()].view(ks.shape)
    vs_u = vs_buf[3:3 + vs.numel()].view(vs.shape)
    ks_u.copy_(ks)
    vs_u.copy_(vs)
    q = q0[1:1 + B * H * D].view(B, H, D)
    o = tqkv.decode_int8(q, kq, ks_u, vq, vs_u, bs)
    o_ref = tqkv.decode_int8(q.contiguous().clone(), kq, ks, vq, vs, bs)
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref)
    assert_tight(to_np(o), oracle_int8_reference(q, kq, ks, vq, vs, bs))


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("B,H,S", [(1, 4, 128), (2, 2, 1), (2, 3, 777), (1, 2, 5000)])
def test_fp16_decode(B, H, S, D):
    seed = 77 + S + D
    q = _rand((B, H, D), seed)
    k = _rand((B, H, S, D), seed + 1)
    v = _rand((B, H, S, D), seed + 2)
    o = tqkv.decode_fp16(q, k, v)
    torch.cuda.synchronize()
    assert_tight(to_np(o), O.attention(to_np(q), to_np(k), to_np(v)))


def test_fp16_small_config():
    w = W.WORKLOADS["fp16_small"]
    q, k, v = W.make_inputs(w)
    o = tqkv.decode_fp16(q, k, v)
    torch.cuda.synchronize()
    ref = O.attention(to_np(q), to_np(k), to_np(v))
    assert max_abs(to_np(o), ref) < REF_TOL
    assert_tight(to_np(o), ref)


@pytest.mark.parametrize("R", [1, 2, 3, 8])
def test_partials_and_lse_combine(R):
    """Splitting S into R slices, partial records per slice, and the LSE
    combine reproduce the single-launch output (the multi-GPU data path,
    emulated on one GPU)."""
    B, H, S, D, bs = 2, 4, 3000, 128, 64
    q = _rand((B, H, D), 5)
    k = _rand((B, H, S, D), 6)
    v = _rand((B, H, S, D), 7)
    kq, ks, vq, vs = _compress_kv(k, v, bs)
    full = tqkv.decode_int8(q, kq, ks, vq, vs, bs)
    bounds = [S * i // R for i in range(R + 1)]
    recs = torch.empty((R, B * H, D + 2), dtype=torch.float32, device="cuda")
    for i in range(R):
        s0, s1 = bounds[i], bounds[i + 1]
        tqkv.decode_int8_partial(q, kq[:, :, s0:s1].contiguous(), ks[:, :, s0:s1].contiguous(),
                                 vq[:, :, s0:s1].contiguous(), vs[:, :, s0:s1].contiguous(),
                                 bs, out=recs[i])
    o = tqkv.lse_combine(recs, D).view(B, H, D)
    torch.cuda.synchronize()
    assert max_abs(to_np(o), to_np(full)) < 1e-3
    # records against the oracle's partial records, on K/V dequantised the
    # way the kernel does it (code * scale in fp32, exact, no fp16 rounding)
    kd = O.dequantize(to_np(kq), to_np(ks), bs, exact=True)
    vd = O.dequantize(to_np(vq), to_np(vs), bs, exact=True)
    for i in range(R):
        s0, s1 = bounds[i], bounds[i + 1]
        ref = O.attention_partial(to_np(q), kd[:, :, s0:s1], vd[:, :, s0:s1])
        got = to_np(recs[i]).astype(np.float64)
        assert max_abs(got[:, D], ref[:, D]) < 1e-4                      # m
        np.testing.assert_allclose(got[:, D + 1], ref[:, D + 1], rtol=1e-4)  # l
        np.testing.assert_allclose(got[:, :D] / got[:, D + 1:], ref[:, :D] / ref[:, D + 1:],
                                   atol=1e-4)


def test_partial_empty_slice_and_combine():
    """A rank with no tokens contributes (m = -inf, l = 0, acc = 0)."""
    B, H, S, D, bs = 1, 2, 100, 64, 32
    q = _rand((B, H, D), 21)
    k, v = _rand((B, H, S, D), 22), _rand((B, H, S, D), 23)
    kq, ks, vq, vs = _compress_kv(k, v, bs)
    recs = torch.empty((2, B * H, D + 2), dtype=torch.float32, device="cuda")
    tqkv.decode_int8_partial(q, kq, ks, vq, vs, bs, out=recs[0])
    e = torch.empty((B, H, 0, D), dtype=torch.int8, device="cuda")
    es = torch.empty((B, H, 0, D // bs), dtype=torch.float16, device="cuda")
    tqkv.decode_int8_partial(q, e, es, e, es, bs, out=recs[1])
    torch.cuda.synchronize()
    assert torch.isneginf(recs[1][:, D]).all() and (recs[1][:, D + 1] == 0).all()
    o = tqkv.lse_combine(recs, D).view(B, H, D)
    full = tqkv.decode_int8(q, kq, ks, vq, vs, bs)
    torch.cuda.synchronize()
    assert max_abs(to_np(o), to_np(full)) < 1e-3


def test_s_zero_outputs_nan():
    B, H, D, bs = 1, 2, 128, 128
    q = _rand((B, H, D), 1)
    e = torch.empty((B, H, 0, D), dtype=torch.int8, device="cuda")
    es = torch.empty((B, H, 0, 1), dtype=torch.float16, device="cuda")
    o = tqkv.decode_int8(q, e, es, e, es, bs)
    torch.cuda.synchronize()
    assert torch.isnan(o.float()).all()


def test_workspace_left_zeroed():
    B, H, S, D, bs = 1, 2, 50000, 128, 128
    q = _rand((B, H, D), 31)
    k, v = _rand((B, H, S, D), 32), _rand((B, H, S, D), 33)
    kq, ks, vq, vs = _compress_kv(k, v, bs)
    ws = tqkv.Workspace()
    for _ in range(3):
        tqkv.decode_int8(q, kq, ks, vq, vs, bs, workspace=ws)
    torch.cuda.synchronize()
    nb = tqkv.workspace_bytes(B, H, S, D)
    assert nb > 0
    # counters and every piece record: the whole workspace is zero again
    assert int(ws.buf.count_nonzero()) == 0


def test_workspace_reused_across_shapes():
    """One workspace serves calls of different shapes in any order: a call
    never takes a record left by an earlier call for one of its own pieces
    (every call leaves the records zero)."""
    ws = tqkv.Workspace()
    shapes = [(1, 2, 40000, 128, 128), (8, 12, 3000, 64, 64), (1, 1, 90000, 128, 32),
              (4, 32, 2500, 128, 64), (1, 3, 70000, 64, 32)]
    for i, (B, H, S, D, bs) in enumerate(shapes):
        q = _rand((B, H, D), 100 + i)
        k, v = _rand((B, H, S, D), 200 + i), _rand((B, H, S, D), 300 + i)
        kq, ks, vq, vs = _compress_kv(k, v, bs)
        o = tqkv.decode_int8(q, kq, ks, vq, vs, bs, workspace=ws)
        torch.cuda.synchronize()
        assert_tight(to_np(o), oracle_int8_reference(q, kq, ks, vq, vs, bs))
        assert int(ws.buf.count_nonzero()) == 0


def test_repeat_calls_identical():
    """Deterministic: same inputs, same bits, call after call."""
    w = W.WORKLOADS["int8_b2h8"]
    q, k, v = W.make_inputs(w)
    kq, ks, vq, vs = _compress_kv(k, v, w.block_size)
    o1 = tqkv.decode_int8(q, kq, ks, vq, vs, w.block_size).clone()
    for _ in range(5):
        o2 = tqkv.decode_int8(q, kq, ks, vq, vs, w.block_size)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)


def _golden():
    import json
    import os
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                        "ref_build_golden.json")
    with open(path) as f:
        return json.load(f)["cases"]


@pytest.mark.parametrize("name", ["fp16_small", "int8_b2h8", "int8_gpt2_outlier",
                                  "int8_bs32_lognormal", "int8_bs128_ragged"])
def test_decode_vs_reference_kernels_golden(name):
    """Outputs of the reference's own kernels (online Kernel D, two-pass
    Kernel C, fp16 baseline), recorded on the same inputs: ours agree to well
    inside the 1e-2 contract."""
    import golden.gen as gen
    case = _golden()[name]
    q, k, v = (torch.from_numpy(a).cuda() for a in gen.inputs(name))
    bs = case["block_size"]
    if bs == 0:
        o = tqkv.decode_fp16(q, k, v)
        refs = [case["O_baseline_bits"]]
    else:
        kq, ks, vq, vs = _compress_kv(k, v, bs)
        o = tqkv.decode_int8(q, kq, ks, vq, vs, bs)
        refs = [case["O_online_bits"], case["O_fused_bits"]]
    torch.cuda.synchronize()
    got = to_np(o).reshape(-1).astype(np.float64)
    for bits in refs:
        ref = np.asarray(bits, np.uint16).view(np.float16).astype(np.float64)
        assert max_abs(got, ref) < REF_TOL
        assert_tight(got, ref)


@pytest.mark.parametrize("D,bs", [(128, 128), (64, 32)])
def test_exchange_publish_combine_single_rank(D, bs):
    """The NVLink exchange path with one rank on one GPU: publish (records +
    step flag) then combine, for several consecutive steps (both record slots,
    changing q), equals the plain decode."""
    B, H, S = 2, 5, 9000
    k, v = _rand((B, H, S, D), 51), _rand((B, H, S, D), 52)
    kq, ks, vq, vs = _compress_kv(k, v, bs)
    ex = tqkv.LocalExchange(B * H, D)
    try:
        for step in range(5):
            q = _rand((B, H, D), 60 + step)
            ex.publish(q, kq, ks, vq, vs, bs)
            o = ex.combine(torch.empty((B, H, D), dtype=torch.float16, device="cuda"))
            ref = tqkv.decode_int8(q, kq, ks, vq, vs, bs)
            torch.cuda.synchronize()
            assert max_abs(to_np(o), to_np(ref)) < 1e-3, step
        assert tqkv.read_device_error() == 0
    finally:
        ex.close()
