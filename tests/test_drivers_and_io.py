"""Drop-in link test and the on-disk KV format.

* The reference's unmodified drivers (src/main.cpp, src/benchmark.cpp of the
  reference project) compiled against this repository's include/ only and
  linked to libtqkv_b200.so (built by `make -C oracle ref`, where the
  reference sources are present): they resolve every launcher from the
  library and run (--help needs no GPU).
* include/io_util.h parses meta.json and reads .bin tensors with the
  reference's failure behaviour (exit code 2)."""
import os
import subprocess
import tempfile

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(REPO, "oracle", "_ref")
LAUNCHERS = ["launch_kv_compress", "launch_kv_reconstruct", "launch_decode_attn_baseline",
             "launch_decode_attn_int8_fused", "launch_decode_attn_int8_fused_online"]


@pytest.mark.parametrize("exe", ["tqkv_decode_b200", "tqkv_bench_b200"])
def test_reference_drivers_link_against_library(exe):
    path = os.path.join(REF, exe)
    if not os.path.exists(path):
        pytest.skip("link-test drivers not built here (needs the reference sources)")
    ldd = subprocess.run(["ldd", path], capture_output=True, text=True, check=True).stdout
    assert "libtqkv_b200.so" in ldd and "not found" not in ldd
    und = subprocess.run(["nm", "-uC", path], capture_output=True, text=True, check=True).stdout
    used = [n for n in LAUNCHERS if n + "(" in und]
    assert used, und
    r = subprocess.run([path, "--help"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "usage:" in r.stdout


PROG = r'''
#include "io_util.h"
#include <cstdio>
#include <vector>
int main(int argc, char** argv) {
    std::string meta = tqkv_slurp(std::string(argv[1]) + "/meta.json");
    int B = tqkv_read_meta_int(meta, "B"), S = tqkv_read_meta_int(meta, "S");
    int neg = tqkv_read_meta_int(meta, "neg");
    std::vector<unsigned short> q(4);
    tqkv_read_bin(std::string(argv[1]) + "/Q.bin", q.data(), 8);
    std::printf("%d %d %d %u %u\n", B, S, neg, q[0], q[3]);
    if (argc > 2) tqkv_read_meta_int(meta, argv[2]);
    return 0;
}
'''


def test_io_util_meta_and_bin():
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "t.cpp")
        exe = os.path.join(d, "t")
        open(src, "w").write(PROG)
        subprocess.run(["g++", "-std=c++17", "-I", os.path.join(REPO, "include"), src, "-o", exe],
                       check=True)
        kv = os.path.join(d, "kv")
        os.mkdir(kv)
        open(os.path.join(kv, "meta.json"), "w").write(
            '{\n  "B": 2,\n  "H": 8,\n  "S":   2048,\n  "neg": -7,\n  "dtype": "float16"\n}\n')
        open(os.path.join(kv, "Q.bin"), "wb").write(bytes([1, 0, 2, 0, 3, 0, 4, 1]))
        r = subprocess.run([exe, kv], capture_output=True, text=True)
        assert r.returncode == 0 and r.stdout.split() == ["2", "2048", "-7", "1", "260"]
        r = subprocess.run([exe, kv, "missing"], capture_output=True, text=True)
        assert r.returncode == 2 and 'missing key "missing"' in r.stderr
        r = subprocess.run([exe, kv, "dtype"], capture_output=True, text=True)
        assert r.returncode == 2 and "non-integer" in r.stderr
        open(os.path.join(kv, "Q.bin"), "wb").write(bytes([1, 0]))
        r = subprocess.run([exe, kv], capture_output=True, text=True)
        assert r.returncode == 2 and "could not read 8 bytes" in r.stderr
