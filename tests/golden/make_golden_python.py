"""Generates python_golden.npz from the reference's own Python check
(python/check_correctness.py of the reference project: `dequantize` and
`torch_attention_fp32`), run on the seeded inputs of gen.py.

Run where the reference is mounted (not on the GPU box):
    python tests/golden/make_golden_python.py [REFERENCE_ROOT]
REFERENCE_ROOT defaults to $TQKV_REF_ROOT, else a checkout named `reference`
beside this repository.
The codes fed to `dequantize` come from the CPU oracle's compress (any valid
codes pin the dequantise/attention formulas; the codes themselves are pinned
separately by ref_build_golden.json).
"""
import hashlib
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)
import gen  # noqa: E402
from oracle import oracle as O  # noqa: E402


def main():
    ref_root = (sys.argv[1] if len(sys.argv) > 1 else
                os.environ.get("TQKV_REF_ROOT", os.path.join(os.path.dirname(REPO), "reference")))
    spec = importlib.util.spec_from_file_location(
        "check_correctness", os.path.join(ref_root, "python", "check_correctness.py"))
    cc = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(cc)
    out = {}
    for name, (B, H, S, D, bs, seed, dist) in gen.CASES.items():
        q, k, v = gen.inputs(name)
        scale = 1.0 / np.sqrt(D)
        if bs == 0:
            out[f"{name}/O"] = cc.torch_attention_fp32(q, k, v, scale)
            continue
        kq, ks = O.kv_compress(k, bs)
        vq, vs = O.kv_compress(v, bs)
        kd = cc.dequantize(kq, ks, bs)
        vd = cc.dequantize(vq, vs, bs)
        out[f"{name}/K_recon_sha256"] = np.array(hashlib.sha256(kd.tobytes()).hexdigest())
        out[f"{name}/V_recon_sha256"] = np.array(hashlib.sha256(vd.tobytes()).hexdigest())
        out[f"{name}/O_int8"] = cc.torch_attention_fp32(q, kd, vd, scale)
        out[f"{name}/O_fp16truth"] = cc.torch_attention_fp32(q, k, v, scale)
    np.savez_compressed(os.path.join(HERE, "python_golden.npz"), **out)
    print("wrote", {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
