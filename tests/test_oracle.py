"""The CPU oracle, pinned: fp16 conversions against numpy, the quantisation
rule's known answers, the dequantise/attention formulas against the golden
outputs of the reference's own Python check (python_golden.npz), and the
codes against the reference build's golden hashes (ref_build_golden.json)."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from oracle import torch_port

import golden.gen as gen

HERE = os.path.dirname(os.path.abspath(__file__))
PY_GOLDEN = os.path.join(HERE, "golden", "python_golden.npz")
REF_GOLDEN = os.path.join(HERE, "golden", "ref_build_golden.json")


def test_half_to_float_exhaustive():
    h = np.arange(65536, dtype=np.uint16)
    f = O.half_bits_to_float(h)
    ref = h.view(np.float16).astype(np.float32)
    assert np.array_equal(np.isnan(f), np.isnan(ref))
    assert np.array_equal(f[~np.isnan(f)], ref[~np.isnan(ref)])


def test_float_to_half_rne():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(1 << 18).astype(np.float32) * s
                        for s in (1e-7, 1e-5, 1e-3, 1, 1e3, 6e4)])
    fin = np.unique(np.arange(65536, dtype=np.uint16).view(np.float16).astype(np.float32))
    fin = fin[np.isfinite(fin)]
    mid = ((fin[:-1].astype(np.float64) + fin[1:]) / 2).astype(np.float32)  # exact ties
    for arr in (x, fin, mid):
        with np.errstate(over="ignore"):
            want = arr.astype(np.float16).view(np.uint16)
        assert np.array_equal(O.float_to_half_bits(arr), want)


def test_compress_known_answers():
    D, bs = 64, 32
    rows = np.zeros((4, D), np.float16)
    rows[1, :6] = [127, 0.5, 1.5, 2.5, -0.5, -1.5]        # s = 1: ties to even
    rows[2, :32] = np.linspace(-3, 3, 32)                  # +-max -> +-127
    rows[3, :] = np.float16(2.0 ** -24) * (np.arange(D) % 5 + 1)  # subnormals
    q, s = O.kv_compress(rows, bs)
    assert (q[0] == 0).all() and (s[0] == 1).all()         # all-zero block: scale 1
    assert list(q[1, :6]) == [127, 0, 2, 2, 0, -2]
    assert q[2, :32].max() == 127 and q[2, :32].min() == -127
    assert s[1, 0] == np.float16(1.0)
    assert (np.abs(q[3]) <= 127).all() and (q[3].reshape(2, 32).max(axis=1) == 127).all()


def test_tie_mask():
    x = np.zeros((1, 32), np.float16)
    x[0, 0] = 2.0
    x[0, 1] = 1.0       # 127 * 1 / 2 = 63.5: tie
    x[0, 2] = -1.0      # tie
    x[0, 3] = 0.75      # 47.625: not a tie
    m, n = O.tie_mask(x, 32)
    assert n == 2 and m[0, 1] == 1 and m[0, 2] == 1 and m[0, 3] == 0


def test_oracle_attention_matches_reference_formulation():
    """Binary64 oracle vs the reference's fp32 torch formulation."""
    q, k, v = gen.inputs("int8_bs128_ragged")
    a = O.attention(q, k, v)
    b = torch_port.attention_fp32(torch.from_numpy(q), torch.from_numpy(k),
                                  torch.from_numpy(v)).float().numpy()
    assert np.max(np.abs(a - b)) < 2e-3


@pytest.mark.parametrize("name", list(gen.CASES))
def test_oracle_vs_python_golden(name):
    g = np.load(PY_GOLDEN)
    B, H, S, D, bs, seed, dist = gen.CASES[name]
    q, k, v = gen.inputs(name)
    if bs == 0:
        ref = g[f"{name}/O"].astype(np.float32)
        got = O.attention(q, k, v)
    else:
        kq, ks = O.kv_compress(k, bs)
        vq, vs = O.kv_compress(v, bs)
        kd = O.dequantize(kq, ks, bs)
        vd = O.dequantize(vq, vs, bs)
        # dequantise: bit-identical to the reference's formula
        assert hashlib.sha256(kd.astype(np.float16).tobytes()).hexdigest() == \
            str(g[f"{name}/K_recon_sha256"])
        assert hashlib.sha256(vd.astype(np.float16).tobytes()).hexdigest() == \
            str(g[f"{name}/V_recon_sha256"])
        ref = g[f"{name}/O_int8"].astype(np.float32)
        got = O.attention(q, kd, vd)
        # the reference's torch port reproduces its own golden bit for bit
        tp = torch_port.int8_decode_step(torch.from_numpy(q), torch.from_numpy(kq),
                                         torch.from_numpy(ks), torch.from_numpy(vq),
                                         torch.from_numpy(vs), bs)
        assert np.array_equal(tp.numpy().view(np.uint16), g[f"{name}/O_int8"].view(np.uint16))
    # fp32 torch (rounded to fp16) vs binary64: within one fp16 ulp + fp32 noise
    tol = 1e-5 + np.abs(ref) * 2.0 ** -10
    assert (np.abs(got - ref) <= tol).all(), float(np.max(np.abs(got - ref)))


def _ref_golden():
    if not os.path.exists(REF_GOLDEN):
        pytest.skip("ref_build_golden.json not generated yet")
    with open(REF_GOLDEN) as f:
        return json.load(f)


def _apply_overrides(codes, rec):
    flat = codes.reshape(-1).copy()
    flat[np.asarray(rec["override_index"], dtype=np.int64)] = np.asarray(rec["override_code"],
                                                                          dtype=np.int8)
    return flat.reshape(codes.shape)


def _cases():
    if not os.path.exists(REF_GOLDEN):
        return []
    with open(REF_GOLDEN) as f:
        return sorted(json.load(f)["cases"])


@pytest.mark.parametrize("name", _cases())
def test_oracle_vs_reference_build_golden(name):
    """IEEE oracle + the recorded tie-class overrides reproduce the reference
    build's codes and scales bit for bit (sha256 of the full arrays)."""
    case = _ref_golden()["cases"][name]
    if case["block_size"] == 0:
        q, k, v = gen.inputs(name)
        ref = np.asarray(case["O_baseline_bits"], np.uint16).view(np.float16).astype(np.float32)
        got = O.attention(q, k, v).reshape(-1)
        assert np.max(np.abs(got - ref)) < 1e-2
        return
    bs = case["block_size"]
    if name.startswith("tie_rich"):
        D = case["shape"][3]
        tensors = {"X": gen.tie_rich_rows(D).reshape(1, 1, -1, D)}
    else:
        q, k, v = gen.inputs(name)
        tensors = {"K": k, "V": v}
    codes = {}
    for t, x in tensors.items():
        rec = case[t]
        qo, so = O.kv_compress(x, bs)
        assert rec["overrides_outside_tie_class"] == 0
        assert rec["ieee_oracle_scale_mismatches"] == 0
        mask, n_ties = O.tie_mask(x, bs)
        assert n_ties == rec["tie_class_size"]
        assert mask.reshape(-1)[np.asarray(rec["override_index"], dtype=np.int64)].all()
        fixed = _apply_overrides(qo, rec)
        assert hashlib.sha256(fixed.tobytes()).hexdigest() == rec["codes_sha256"]
        assert hashlib.sha256(so.view(np.uint16).tobytes()).hexdigest() == rec["scales_sha256"]
        codes[t] = (fixed, so)
    if "O_online_bits" in case:
        (kq, ks), (vq, vs) = codes["K"], codes["V"]
        ref_o = O.attention(q, O.dequantize(kq, ks, bs), O.dequantize(vq, vs, bs)).reshape(-1)
        for key in ("O_online_bits", "O_fused_bits"):
            o = np.asarray(case[key], np.uint16).view(np.float16).astype(np.float32)
            assert np.max(np.abs(o - ref_o)) < 1e-2   # the reference's own acceptance bound
