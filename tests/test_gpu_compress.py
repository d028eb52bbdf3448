"""GPU parity of Kernel A (compress) and Kernel B (reconstruct).

Bit-exactness is the bar: INT8 codes and fp16 scales must equal
  * the reference's own Kernel A, built for sm_100a with its own flags
    (oracle/_ref/libtqkv_ref.so), on every element, when that build is
    present; and
  * the CPU oracle on every element outside the "tie class" (elements whose
    exact quotient 127*x/m is a half-integer, where the result depends on the
    last bit of the division; see oracle/tqkv_oracle.c), with scales equal
    everywhere.  In the tie class the code may differ from the IEEE oracle
    by exactly one.
Kernel B must equal the oracle bit for bit.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

import tqkv
from tqkv import workloads as W
from oracle import oracle as O

from helpers import to_np

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(REPO, "oracle", "_ref", "libtqkv_ref.so")
VALID = [(64, 32), (64, 64), (128, 32), (128, 64), (128, 128)]


def _ref_lib():
    if not os.path.exists(REF_LIB):
        pytest.skip("reference build oracle/_ref/libtqkv_ref.so not present")
    lib = ctypes.CDLL(REF_LIB)
    P = ctypes.c_void_p
    lib.ref_kv_compress.argtypes = [P, P, P] + [ctypes.c_int] * 5 + [P]
    lib.ref_kv_reconstruct.argtypes = [P, P, P] + [ctypes.c_int] * 5 + [P]
    return lib


def _stream():
    return torch.cuda.current_stream().cuda_stream


def check_against_oracle(x: torch.Tensor, bs: int, q: torch.Tensor, s: torch.Tensor):
    xn = to_np(x).reshape(-1, x.shape[-1])
    qo, so = O.kv_compress(xn, bs)
    mask, _ = O.tie_mask(xn, bs)
    qg = to_np(q).reshape(qo.shape)
    sg = to_np(s).reshape(so.shape)
    assert np.array_equal(sg.view(np.uint16), so.view(np.uint16)), "fp16 scales differ"
    diff = qg != qo
    assert not np.any(diff & (mask == 0)), "codes differ outside the tie class"
    assert np.all(np.abs(qg.astype(np.int32) - qo.astype(np.int32)) <= 1)


def _rand(shape, seed, scale=1.0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return (torch.randn(shape, generator=g, device="cuda") * scale).half()


@pytest.mark.parametrize("name", ["int8_b2h8", "int8_gpt2_outlier"])
@pytest.mark.parametrize("which", ["k", "v"])
def test_compress_config_vs_oracle(name, which):
    w = W.WORKLOADS[name]
    x = W.make_kv_slice(w, which)
    q, s = tqkv.kv_compress(x, w.block_size)
    torch.cuda.synchronize()
    check_against_oracle(x, w.block_size, q, s)


@pytest.mark.parametrize("D,bs", VALID)
def test_compress_vs_reference_build(D, bs):
    """Bit-identical codes and scales to the reference's own Kernel A."""
    lib = _ref_lib()
    x = _rand((3, 5, 4001, D), D * 10 + bs)
    q, s = tqkv.kv_compress(x, bs)
    qr = torch.empty_like(q)
    sr = torch.empty_like(s)
    lib.ref_kv_compress(x.data_ptr(), qr.data_ptr(), sr.data_ptr(), 3, 5, 4001, D, bs, _stream())
    torch.cuda.synchronize()
    assert torch.equal(q, qr)
    assert torch.equal(s.view(torch.int16), sr.view(torch.int16))


@pytest.mark.parametrize("name", ["int8_bh_shard", "int8_longctx"])
def test_compress_large_config_vs_reference_build(name):
    """Full-size configurations against the reference build, every element."""
    lib = _ref_lib()
    w = W.WORKLOADS[name]
    x = W.make_kv_slice(w, "k")
    q, s = tqkv.kv_compress(x, w.block_size)
    qr = torch.empty_like(q)
    sr = torch.empty_like(s)
    lib.ref_kv_compress(x.data_ptr(), qr.data_ptr(), sr.data_ptr(), w.B, w.H, w.S, w.D,
                        w.block_size, _stream())
    torch.cuda.synchronize()
    assert torch.equal(q, qr)
    assert torch.equal(s.view(torch.int16), sr.view(torch.int16))
    # and a row sample against the CPU oracle
    rows = x.reshape(-1, w.D)[:: 997][:4096]
    check_against_oracle(rows, w.block_size, q.reshape(-1, w.D)[:: 997][:4096],
                         s.reshape(-1, w.D // w.block_size)[:: 997][:4096])


def _edge_rows(D: int) -> torch.Tensor:
    """Known-answer rows: all-zero block, +-max -> +-127, exact .5 ties,
    fp16 subnormals, mixed signs of zero."""
    rows = []
    rows.append(np.zeros(D, np.float16))                                 # s = 1, codes 0
    r = np.zeros(D, np.float16); r[0] = 127; r[1:6] = [0.5, 1.5, 2.5, -0.5, -1.5]
    rows.append(r)                                                       # s = 1: ties to even
    r = np.linspace(-3, 3, D).astype(np.float16); rows.append(r)         # +-max -> +-127
    r = (np.arange(D) % 7 + 1).astype(np.float16) * np.float16(2 ** -24); rows.append(r)  # subnormals
    r = np.full(D, -0.0, np.float16); r[3] = 0.0; rows.append(r)        # signed zeros
    r = np.full(D, 65504, np.float16); r[::2] = -65504; rows.append(r)   # fp16 extremes
    r = np.zeros(D, np.float16); r[:] = np.float16(1.0); r[0] = 2.0; rows.append(r)  # x = m / 2
    return torch.from_numpy(np.stack(rows)).cuda().reshape(1, 1, len(rows), D)


@pytest.mark.parametrize("D,bs", VALID)
def test_compress_known_answers(D, bs):
    x = _edge_rows(D)
    q, s = tqkv.kv_compress(x, bs)
    torch.cuda.synchronize()
    qn, sn = to_np(q)[0, 0], to_np(s)[0, 0]
    assert (qn[0] == 0).all() and (sn[0] == 1.0).all()
    if bs >= 8:
        assert list(qn[1, :6]) == [127, 0, 2, 2, 0, -2]
    assert qn[2].max() == 127 and qn[2].min() == -127
    assert (qn[5] == np.where(np.arange(D) % 2 == 0, -127, 127)).all()
    check_against_oracle(x, bs, q, s)
    if os.path.exists(REF_LIB):
        lib = _ref_lib()
        qr, sr = torch.empty_like(q), torch.empty_like(s)
        lib.ref_kv_compress(x.data_ptr(), qr.data_ptr(), sr.data_ptr(), 1, 1, x.shape[2], D, bs,
                            _stream())
        torch.cuda.synchronize()
        assert torch.equal(q, qr) and torch.equal(s.view(torch.int16), sr.view(torch.int16))


def test_compress_nonfinite_matches_reference_build():
    """NaN and Inf inputs follow the reference build exactly (fmaxf ignores
    NaN; x / inf = 0; NaN codes are 0)."""
    lib = _ref_lib()
    D, bs = 128, 32
    x = _rand((1, 1, 64, D), 5)
    x[0, 0, 0, 3] = float("nan")
    x[0, 0, 1, :32] = float("nan")
    x[0, 0, 2, 40] = float("inf")
    x[0, 0, 3, 70] = float("-inf")
    q, s = tqkv.kv_compress(x, bs)
    qr, sr = torch.empty_like(q), torch.empty_like(s)
    lib.ref_kv_compress(x.data_ptr(), qr.data_ptr(), sr.data_ptr(), 1, 1, 64, D, bs, _stream())
    torch.cuda.synchronize()
    assert torch.equal(q, qr)
    assert torch.equal(s.view(torch.int16), sr.view(torch.int16))


@pytest.mark.parametrize("D,bs", VALID)
@pytest.mark.parametrize("S", [1, 3, 64, 1001])
def test_reconstruct_bit_exact(D, bs, S):
    x = _rand((2, 3, S, D), S + D + bs, scale=2.0)
    q, s = tqkv.kv_compress(x, bs)
    y = tqkv.kv_reconstruct(q, s, bs)
    torch.cuda.synchronize()
    yo = O.kv_reconstruct(to_np(q), to_np(s), bs)
    assert np.array_equal(to_np(y).view(np.uint16), yo.view(np.uint16))


def test_reconstruct_exhaustive_codes_and_scales():
    """Every code (all 256 bytes) times every fp16 scale bit pattern (65,536,
    subnormals, infinities and NaNs included): bit-identical to the reference
    build's Kernel B, and to the oracle wherever the oracle's result is not a
    NaN (there the kernel must give a NaN too; the NaN payload is the GPU's)."""
    rows = 65536 * 2
    codes = (torch.arange(256, dtype=torch.int32, device="cuda").to(torch.uint8)
             .view(torch.int8).repeat(65536).reshape(1, 1, rows, 128))
    scales = (torch.arange(65536, dtype=torch.int32, device="cuda").to(torch.int16)
              .repeat_interleave(2).view(torch.half).reshape(1, 1, rows, 1))
    y = tqkv.kv_reconstruct(codes, scales, 128)
    torch.cuda.synchronize()
    yb = to_np(y).view(np.uint16)
    yo = O.kv_reconstruct(to_np(codes), to_np(scales), 128).view(np.uint16)
    nan_o = (yo & 0x7c00) == 0x7c00
    nan_o &= (yo & 0x03ff) != 0
    nan_g = ((yb & 0x7c00) == 0x7c00) & ((yb & 0x03ff) != 0)
    assert np.array_equal(nan_g, nan_o)
    assert np.array_equal(yb[~nan_o], yo[~nan_o])
    if os.path.exists(REF_LIB):
        lib = _ref_lib()
        yr = torch.empty_like(y)
        lib.ref_kv_reconstruct(codes.data_ptr(), scales.data_ptr(), yr.data_ptr(), 1, 1, rows,
                               128, 128, _stream())
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int16), yr.view(torch.int16))


def test_roundtrip_bound_full_longctx():
    """Size-independent property on the largest configuration: every
    element's round-trip error |x - code*scale| is at most half a scale step
    (plus the fp16 scale rounding), the bound the reference checks
    (python/check_correctness.py:102-119), and every nonzero block holds a
    +-127 code."""
    w = W.WORKLOADS["int8_longctx"]
    x = W.make_kv_slice(w, "v")
    q, s = tqkv.kv_compress(x, w.block_size)
    y = tqkv.kv_reconstruct(q, s, w.block_size)
    torch.cuda.synchronize()
    xf = x.float().reshape(-1, w.D)
    sf = s.float().reshape(-1, 1)
    err = (xf - y.float().reshape(-1, w.D)).abs()
    # codes are rounded against the fp32 scale s32 (|x/s32 - code| <= 1/2);
    # reconstruction uses fp16(s32), off by <= 2^-11 relative, times |code| <= 127;
    # the fp16 output adds <= 2^-11 relative rounding.
    bound = sf * (0.5 * (1 + 2 ** -10) + 127 * 2 ** -10) + xf.abs() * 2 ** -10 + 2 ** -24
    assert bool((err <= bound).all())
    # the reference's own acceptance test (check_correctness.py:109-119)
    assert float(err.max()) <= 1.5 * (0.5 * float(sf.max()) + 1e-3)
    assert bool((q.reshape(-1, w.D).abs().amax(dim=1) == 127).all())


def _golden_cases():
    path = os.path.join(REPO, "tests", "golden", "ref_build_golden.json")
    if not os.path.exists(path):
        return []
    import json
    with open(path) as f:
        return sorted(json.load(f)["cases"].items())


@pytest.mark.parametrize("name,case", _golden_cases(), ids=[n for n, _ in _golden_cases()])
def test_compress_matches_reference_build_golden(name, case):
    """Codes and scales hash-identical (sha256 of the full arrays) to what the
    reference's own Kernel A produced on the same inputs — no reference build
    needed at test time."""
    import hashlib
    import golden.gen as gen
    bs = case["block_size"]
    if bs == 0:
        pytest.skip("fp16 case")
    if name.startswith("tie_rich"):
        D = case["shape"][3]
        tensors = {"X": gen.tie_rich_rows(D).reshape(1, 1, -1, D)}
    else:
        _, k, v = gen.inputs(name)
        tensors = {"K": k, "V": v}
    for t, x in tensors.items():
        q, s = tqkv.kv_compress(torch.from_numpy(x).cuda(), bs)
        torch.cuda.synchronize()
        assert hashlib.sha256(to_np(q).tobytes()).hexdigest() == case[t]["codes_sha256"], t
        assert hashlib.sha256(to_np(s).view(np.uint16).tobytes()).hexdigest() == \
            case[t]["scales_sha256"], t
