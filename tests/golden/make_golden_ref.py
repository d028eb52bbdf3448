"""Generates ref_build_golden.json from the reference's own kernels, built for
sm_100a with the reference's flags by oracle/Makefile (oracle/_ref/libtqkv_ref.so).
Needs a B200:

    python tests/golden/make_golden_ref.py OUT.json

For every INT8 case of gen.py and each of K and V it records
  * sha256 of the reference build's full int8 code array and fp16 scale array;
  * the reference's code at every tie-class position (where the exact
    quotient 127*x/m is a half-integer; see oracle/tqkv_oracle.c) — the only
    positions where a correctly rounded division may round differently;
and the reference kernels' decode outputs (fp16 bits): the online kernel
(Kernel D), the two-pass kernel (Kernel C) and, for the fp16 case, the
baseline.  With these, the CPU oracle's codes plus the tie overrides must
reproduce the reference hashes exactly, and the GPU kernels must match them.
"""
import ctypes
import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)
import gen  # noqa: E402
from oracle import oracle as O  # noqa: E402

P = ctypes.c_void_p
I = ctypes.c_int


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    out_path = sys.argv[1]
    lib = ctypes.CDLL(os.path.join(REPO, "oracle", "_ref", "libtqkv_ref.so"))
    lib.ref_kv_compress.argtypes = [P, P, P] + [I] * 5 + [P]
    lib.ref_decode_fp16.argtypes = [P] * 4 + [I] * 4 + [P]
    lib.ref_decode_int8_fused.argtypes = [P] * 6 + [I] * 5 + [P]
    lib.ref_decode_int8_online.argtypes = [P] * 6 + [I] * 7 + [P]
    lib.ref_last_error.restype = I
    st = 0  # legacy default stream, as the reference drivers use
    dev = torch.device("cuda", 0)
    golden = {"generator": "tests/golden/make_golden_ref.py",
              "reference_build": "oracle/Makefile ref (nvcc -O3 --use_fast_math, sm_100a)",
              "cases": {}}

    def compress(x: np.ndarray, bs: int):
        B, H, S, D = x.shape
        xt = torch.from_numpy(x).to(dev)
        qt = torch.empty(x.shape, dtype=torch.int8, device=dev)
        sc = torch.empty((B, H, S, D // bs), dtype=torch.float16, device=dev)
        lib.ref_kv_compress(xt.data_ptr(), qt.data_ptr(), sc.data_ptr(), B, H, S, D, bs, st)
        torch.cuda.synchronize()
        assert lib.ref_last_error() == 0
        return qt, sc

    def record(x, bs, qt, sc):
        codes = qt.cpu().numpy()
        scales = sc.cpu().numpy()
        mask, n_ties = O.tie_mask(x, bs)
        qo, so = O.kv_compress(x, bs)
        idx = np.flatnonzero((qo != codes).reshape(-1))
        return {
            "codes_sha256": sha(codes), "scales_sha256": sha(scales.view(np.uint16)),
            "tie_class_size": n_ties,
            # positions where the reference build's code differs from the IEEE
            # oracle's, with the reference's code (all expected in the tie class)
            "override_index": idx.tolist(),
            "override_code": codes.reshape(-1)[idx].astype(int).tolist(),
            "overrides_outside_tie_class": int((mask.reshape(-1)[idx] == 0).sum()),
            "ieee_oracle_scale_mismatches": int((so.view(np.uint16) != scales.view(np.uint16)).sum()),
        }

    for name, (B, H, S, D, bs, seed, dist) in gen.CASES.items():
        q, k, v = gen.inputs(name)
        case = {"shape": [B, H, S, D], "block_size": bs, "seed": seed, "dist": dist}
        qd = torch.from_numpy(q).to(dev)
        o = torch.empty((B, H, D), dtype=torch.float16, device=dev)
        if bs == 0:
            kd, vd = torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev)
            lib.ref_decode_fp16(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), o.data_ptr(),
                                B, H, S, D, st)
            torch.cuda.synchronize()
            case["O_baseline_bits"] = o.cpu().numpy().view(np.uint16).reshape(-1).tolist()
            golden["cases"][name] = case
            continue
        kq, ks = compress(k, bs)
        vq, vs = compress(v, bs)
        case["K"] = record(k, bs, kq, ks)
        case["V"] = record(v, bs, vq, vs)
        lanes = 4 if D == 128 else 2
        lib.ref_decode_int8_online(qd.data_ptr(), kq.data_ptr(), ks.data_ptr(), vq.data_ptr(),
                                   vs.data_ptr(), o.data_ptr(), B, H, S, D, bs, lanes, 32, st)
        torch.cuda.synchronize()
        case["O_online_bits"] = o.cpu().numpy().view(np.uint16).reshape(-1).tolist()
        case["online_lanes_tile"] = [lanes, 32]
        lib.ref_decode_int8_fused(qd.data_ptr(), kq.data_ptr(), ks.data_ptr(), vq.data_ptr(),
                                  vs.data_ptr(), o.data_ptr(), B, H, S, D, bs, st)
        torch.cuda.synchronize()
        case["O_fused_bits"] = o.cpu().numpy().view(np.uint16).reshape(-1).tolist()
        assert lib.ref_last_error() == 0
        golden["cases"][name] = case

    for D, bss in ((64, (32, 64)), (128, (32, 64, 128))):
        x = gen.tie_rich_rows(D).reshape(1, 1, -1, D)
        for bs in bss:
            qt, sc = compress(x, bs)
            golden["cases"][f"tie_rich_D{D}_bs{bs}"] = {
                "shape": list(x.shape), "block_size": bs, "rows": "gen.tie_rich_rows",
                "X": record(x, bs, qt, sc)}
    with open(out_path, "w") as f:
        json.dump(golden, f, separators=(",", ":"))
    print("wrote", out_path, os.path.getsize(out_path), "bytes")


if __name__ == "__main__":
    main()
