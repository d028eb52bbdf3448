"""The reference's on-disk KV format: written by tqkv.kvfile.save_kv, read
back whole and as rank shards (by tokens and by heads), and parsed by the C++
helpers in include/io_util.h the reference's drivers use."""
import os
import subprocess
import tempfile

import numpy as np
import pytest

from tqkv import kvfile

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _tensors(B=2, H=3, S=101, D=64, seed=0):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, H, D)).astype(np.float16)
    k = rng.standard_normal((B, H, S, D)).astype(np.float16)
    v = rng.standard_normal((B, H, S, D)).astype(np.float16)
    return q, k, v


def test_roundtrip_whole():
    q, k, v = _tensors()
    with tempfile.TemporaryDirectory() as d:
        kvfile.save_kv(d, q, k, v, seed=7, mode="int8_fused_online", block_size=64)
        q2, k2, v2, meta = kvfile.load_kv(d)
        assert meta["B"] == 2 and meta["S"] == 101 and meta["seed"] == 7
        assert np.array_equal(q2.numpy(), q) and np.array_equal(k2.numpy(), k)
        assert np.array_equal(v2.numpy(), v)
        # same bytes the reference's drivers read (Q.bin, K.bin, V.bin)
        assert os.path.getsize(os.path.join(d, "K.bin")) == k.size * 2


@pytest.mark.parametrize("world", [2, 3, 8])
def test_token_shards_reassemble(world):
    q, k, v = _tensors()
    with tempfile.TemporaryDirectory() as d:
        kvfile.save_kv(d, q, k, v)
        ks, vs = [], []
        for r in range(world):
            qr, kr, vr, meta = kvfile.load_kv(d, r, world, "s")
            assert np.array_equal(qr.numpy(), q)
            ks.append(kr.numpy())
            vs.append(vr.numpy())
        assert np.array_equal(np.concatenate(ks, axis=2), k)
        assert np.array_equal(np.concatenate(vs, axis=2), v)


@pytest.mark.parametrize("world", [2, 4])
def test_head_shards_reassemble(world):
    q, k, v = _tensors()
    with tempfile.TemporaryDirectory() as d:
        kvfile.save_kv(d, q, k, v)
        parts = [kvfile.load_kv(d, r, world, "bh") for r in range(world)]
        kk = np.concatenate([p[1].numpy() for p in parts], axis=1).reshape(k.shape)
        qq = np.concatenate([p[0].numpy() for p in parts], axis=1).reshape(q.shape)
        assert np.array_equal(kk, k) and np.array_equal(qq, q)


def test_truncated_file_is_rejected():
    q, k, v = _tensors()
    with tempfile.TemporaryDirectory() as d:
        kvfile.save_kv(d, q, k, v)
        with open(os.path.join(d, "V.bin"), "r+b") as f:
            f.truncate(100)
        with pytest.raises(ValueError):
            kvfile.load_kv(d)


PROG = r'''
#include "io_util.h"
#include <cstdio>
int main(int, char** argv) {
    std::string m = tqkv_slurp(std::string(argv[1]) + "/meta.json");
    std::printf("%d %d %d %d\n", tqkv_read_meta_int(m, "B"), tqkv_read_meta_int(m, "H"),
                tqkv_read_meta_int(m, "D"), tqkv_read_meta_int(m, "S"));
    return 0;
}
'''


def test_meta_readable_by_the_drivers_parser():
    q, k, v = _tensors(B=1, H=2, S=33, D=128)
    with tempfile.TemporaryDirectory() as d:
        kvfile.save_kv(d, q, k, v, seed=3)
        src, exe = os.path.join(d, "m.cpp"), os.path.join(d, "m")
        open(src, "w").write(PROG)
        subprocess.run(["g++", "-std=c++17", "-I", os.path.join(REPO, "include"), src, "-o", exe],
                       check=True)
        out = subprocess.run([exe, d], capture_output=True, text=True, check=True).stdout
        assert out.split() == ["1", "2", "128", "33"]
