"""The reference's own decode flow, end to end, on this library.

The reference's unmodified driver (src/main.cpp of the reference project) is
built twice by oracle/Makefile: against the reference's kernels
(oracle/_ref/tqkv_decode) and against this repository's include/ and
libtqkv_b200.so (oracle/_ref/tqkv_decode_b200).  For the cases of the
reference's README (correctness section) and of its smoke grid
(scripts/run_a100.sh: int8_fused_online, D 64/128, lanes 2/4), plus a case
read with --load-kv-from and a long sequence, both drivers run with the same
arguments, so they draw the same Q/K/V (std::mt19937 from --seed) or read the
same files, and write the reference's output directory (Q/K/V, O_cuda and,
for the INT8 modes, Kq/Vq/K_scales/V_scales .bin, meta.json).

Checked here:
  * the INT8 codes and fp16 scales this library wrote are byte-equal to the
    reference build's;
  * the directory passes the reference's correctness check
    (python/check_correctness.py:63-140), restated with its own torch
    formulation (oracle/torch_port.py): max_abs < 1e-2 against fp32 attention
    (on the dequantised K/V for INT8 modes) and the round-trip bound
    1.5 * (0.5 * max scale + 1e-3);
  * O is within the same 1e-2 of the reference kernels' O.

With TQKV_DRIVER_OUT set, every output directory is also copied there, so the
unmodified check_correctness.py can be run on it where the reference sources
are present.
"""
import json
import math
import os
import shutil
import subprocess
import tempfile

import numpy as np
import pytest
import torch

from oracle import torch_port

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(REPO, "oracle", "_ref")
OURS = os.path.join(REF, "tqkv_decode_b200")
THEIRS = os.path.join(REF, "tqkv_decode")

CASES = {
    "readme_fp16_d64": ["--B", "1", "--H", "4", "--D", "64", "--S", "128", "--seed", "0"],
    "readme_fp16_d128": ["--B", "1", "--H", "4", "--D", "128", "--S", "2048", "--seed", "0"],
    "readme_int8_nonfused": ["--B", "2", "--H", "8", "--D", "128", "--S", "2048",
                             "--mode", "int8_nonfused", "--block-size", "64", "--seed", "1"],
    "readme_int8_fused": ["--B", "2", "--H", "8", "--D", "128", "--S", "2048",
                          "--mode", "int8_fused", "--block-size", "64", "--seed", "1"],
    "smoke_online_d64_l2": ["--B", "2", "--H", "8", "--D", "64", "--S", "2048",
                            "--mode", "int8_fused_online", "--tile-n", "32", "--lanes", "2",
                            "--block-size", "64", "--seed", "1"],
    "smoke_online_d128_l2": ["--B", "2", "--H", "8", "--D", "128", "--S", "2048",
                             "--mode", "int8_fused_online", "--tile-n", "32", "--lanes", "2",
                             "--block-size", "64", "--seed", "1"],
    "smoke_online_d128_l4": ["--B", "2", "--H", "8", "--D", "128", "--S", "2048",
                             "--mode", "int8_fused_online", "--tile-n", "32", "--lanes", "4",
                             "--block-size", "64", "--seed", "1"],
    "online_bs32_t64": ["--B", "4", "--H", "4", "--D", "128", "--S", "3000",
                        "--mode", "int8_fused_online", "--tile-n", "64", "--lanes", "4",
                        "--block-size", "32", "--seed", "7"],
    # a sequence long enough that heads are split across many CTAs
    "online_long": ["--B", "1", "--H", "2", "--D", "128", "--S", "60000",
                    "--mode", "int8_fused_online", "--block-size", "128", "--seed", "5"],
}
LOADED = "loaded_outlier_online"   # --load-kv-from: GPT-2-shaped outlier channels


def _need_drivers():
    for p in (OURS, THEIRS):
        if not os.path.exists(p):
            pytest.skip(f"{os.path.basename(p)} not built here (oracle/Makefile ref)")


def _load(d, name, shape, dtype):
    a = np.fromfile(os.path.join(d, name), dtype=dtype)
    assert a.size == int(np.prod(shape)), name
    return a.reshape(shape)


def _check_like_reference(d):
    """The reference's check (python/check_correctness.py:63-140) on an output
    directory; returns the max abs error of O."""
    meta = json.load(open(os.path.join(d, "meta.json")))
    B, H, D, S, mode = meta["B"], meta["H"], meta["D"], meta["S"], meta["mode"]
    Q = torch.from_numpy(_load(d, "Q.bin", (B, H, D), np.float16))
    K = torch.from_numpy(_load(d, "K.bin", (B, H, S, D), np.float16))
    V = torch.from_numpy(_load(d, "V.bin", (B, H, S, D), np.float16))
    O = _load(d, "O_cuda.bin", (B, H, D), np.float16).astype(np.float32)
    if mode == "fp16":
        ref = torch_port.attention_fp32(Q, K, V).float().numpy()
        err = float(np.max(np.abs(O - ref)))
        assert err < 1e-2, (d, err)
        return err
    bs = meta["block_size"]
    nsub = D // bs
    Kq = torch.from_numpy(_load(d, "Kq.bin", (B, H, S, D), np.int8))
    Vq = torch.from_numpy(_load(d, "Vq.bin", (B, H, S, D), np.int8))
    Ks = torch.from_numpy(_load(d, "K_scales.bin", (B, H, S, nsub), np.float16))
    Vs = torch.from_numpy(_load(d, "V_scales.bin", (B, H, S, nsub), np.float16))
    Kr = torch_port.dequantize(Kq, Ks, bs)
    Vr = torch_port.dequantize(Vq, Vs, bs)
    res = max(float((K.float() - Kr.float()).abs().max()), float((V.float() - Vr.float()).abs().max()))
    bound = max(float(Ks.float().abs().max()), float(Vs.float().abs().max())) * 0.5 + 1e-3
    assert res <= 1.5 * bound, (d, res, bound)
    ref = torch_port.attention_fp32(Q, Kr, Vr).float().numpy()
    err = float(np.max(np.abs(O - ref)))
    assert err < 1e-2, (d, err)
    return err


def _run(exe, args, out):
    r = subprocess.run([exe] + args + ["--out", out], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, (exe, args, r.stdout, r.stderr)
    return r.stdout


def _compare(name, args, tmp):
    ours, theirs = os.path.join(tmp, "ours"), os.path.join(tmp, "theirs")
    _run(OURS, args, ours)
    _run(THEIRS, args, theirs)
    meta = json.load(open(os.path.join(ours, "meta.json")))
    assert meta == json.load(open(os.path.join(theirs, "meta.json")))
    for f in ("Q.bin", "K.bin", "V.bin"):       # the same inputs went in
        assert open(os.path.join(ours, f), "rb").read() == open(os.path.join(theirs, f), "rb").read()
    if meta["mode"] != "fp16":                  # Kernel A: bit-exact codes and scales
        for f in ("Kq.bin", "Vq.bin", "K_scales.bin", "V_scales.bin"):
            a = open(os.path.join(ours, f), "rb").read()
            b = open(os.path.join(theirs, f), "rb").read()
            assert a == b, (name, f)
    err = _check_like_reference(ours)
    B, H, D = meta["B"], meta["H"], meta["D"]
    o1 = _load(ours, "O_cuda.bin", (B, H, D), np.float16).astype(np.float32)
    o2 = _load(theirs, "O_cuda.bin", (B, H, D), np.float16).astype(np.float32)
    assert float(np.max(np.abs(o1 - o2))) < 1e-2
    keep = os.environ.get("TQKV_DRIVER_OUT")
    if keep:
        shutil.copytree(ours, os.path.join(keep, name), dirs_exist_ok=True)
    return err


@pytest.mark.parametrize("name", sorted(CASES))
def test_reference_driver_flow(name):
    _need_drivers()
    with tempfile.TemporaryDirectory() as tmp:
        _compare(name, CASES[name], tmp)


def test_reference_driver_flow_with_loaded_kv():
    """--load-kv-from a directory in the reference's format, written by this
    repository's kvfile module: the GPT-2-shaped configuration (B8 H12 D64
    S1024, one channel per head x10, V biased per channel)."""
    _need_drivers()
    from tqkv import kvfile
    from tqkv import workloads as W
    w = W.WORKLOADS["int8_gpt2_outlier"]
    with tempfile.TemporaryDirectory() as tmp:
        src = os.path.join(tmp, "kv")
        q, k, v = (t.cpu().numpy() for t in W.make_inputs(w, device="cuda"))
        kvfile.save_kv(src, q, k, v, seed=w.seed)
        args = ["--load-kv-from", src, "--mode", "int8_fused_online", "--tile-n", "32",
                "--lanes", "2", "--block-size", str(w.block_size)]
        _compare(LOADED, args, tmp)
