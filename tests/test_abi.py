"""The C ABI library loads without a GPU and exports exactly what include/
declares: every tqkv_* function of tqkv.h and the five C++ launchers of
attention.h / quantization.h under their Itanium-mangled names."""
import os
import re
import subprocess

import pytest

import tqkv
from tqkv import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(REPO, "include")


def _exported():
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], check=True,
                         capture_output=True, text=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_library_loads_without_gpu():
    lib = tqkv.load()
    assert lib.tqkv_version().decode().startswith("tqkv-b200")
    assert lib.tqkv_status_string(0) == b"ok"
    assert lib.tqkv_status_string(4).startswith(b"workspace")


def test_every_c_abi_function_is_exported():
    decl = open(os.path.join(INC, "tqkv.h")).read()
    names = set(re.findall(r"\b(tqkv_[a-z0-9_]+)\s*\(", decl))
    assert len(names) >= 12
    exported = _exported()
    missing = names - exported
    assert not missing, missing
    assert names == set(_lib.C_ABI), names ^ set(_lib.C_ABI)


def test_reference_launchers_exported_with_reference_mangling():
    decls = open(os.path.join(INC, "attention.h")).read() + \
        open(os.path.join(INC, "quantization.h")).read()
    names = set(re.findall(r"\bvoid\s+(launch_[a-z0-9_]+)\s*\(", decls))
    assert names == set(_lib.REF_LAUNCHERS)
    exported = _exported()
    for name, mangled in _lib.REF_LAUNCHERS.items():
        assert mangled in exported, name
    dem = subprocess.run(["c++filt"] + list(_lib.REF_LAUNCHERS.values()), capture_output=True,
                         text=True, check=True).stdout.splitlines()
    assert dem[0] == ("launch_kv_compress(__half const*, signed char*, __half*, int, int, int, "
                      "int, int, CUstream_st*)")


def test_nothing_else_exported():
    exported = _exported()
    ours = {s for s in exported if s.startswith("tqkv_")} | set(_lib.REF_LAUNCHERS.values())
    assert exported == ours, sorted(exported - ours)[:10]


def test_fused_append_argument_checks_need_no_gpu():
    """tqkv_decode_int8_append validates sizes, pointers and alignment before
    touching the device (the pointers below are never dereferenced)."""
    lib = tqkv.load()
    p = 1 << 20

    def call(T, S, S_cap, k_new=p, D=128, bs=64):
        return lib.tqkv_decode_int8_append(p, k_new, p, p, p, p, p, p, 1, 2, T, S, S_cap, D, bs,
                                           None, 0, None)
    assert call(0, 4, 4) == 2
    assert call(5, 4, 4) == 2
    assert call(1, 5, 4) == 2
    assert call(1, 4, 4, k_new=p + 8) == 3
    assert call(1, 4, 4, D=96) == 1
    assert call(1, 4, 4, k_new=None) == 6
