"""The reference-signature launchers reject exactly the shapes the reference
rejects, with its message and std::abort() (reference src/kv_compress.cu:130-135,
src/kv_reconstruct.cu:45-50, src/attention_baseline.cu:151-154,
src/attention_int8_fused.cu:185-190, src/attention_int8_fused_online.cu:209-238).
Validation happens before any CUDA call, so these run without a GPU, each in a
child process (an abort ends the process)."""
import os
import signal
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CALL = {
    "launch_kv_compress": "f(None, None, None, 1, 1, 1, {D}, {bs}, None)",
    "launch_kv_reconstruct": "f(None, None, None, 1, 1, 1, {D}, {bs}, None)",
    "launch_decode_attn_baseline": "f(None, None, None, None, 1, 1, 1, {D}, None)",
    "launch_decode_attn_int8_fused": "f(None, None, None, None, None, None, 1, 1, 1, {D}, {bs}, None)",
    "launch_decode_attn_int8_fused_online":
        "f(None, None, None, None, None, None, 1, 1, 1, {D}, {bs}, {L}, {T}, None)",
}


def run_launcher(name, **kw):
    code = (f"import sys; sys.path.insert(0, {os.path.join(REPO, 'parallel-final-project_b200')!r});"
            f"from tqkv import _lib; f = _lib.ref_launcher({name!r}); " + CALL[name].format(**kw))
    return subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)


INVALID_INT8 = [(96, 32), (64, 128), (128, 16), (128, 256), (32, 32), (0, 0)]


@pytest.mark.parametrize("D,bs", INVALID_INT8)
@pytest.mark.parametrize("name", ["launch_kv_compress", "launch_kv_reconstruct",
                                  "launch_decode_attn_int8_fused"])
def test_unsupported_int8_shapes_abort(name, D, bs):
    r = run_launcher(name, D=D, bs=bs)
    assert r.returncode == -signal.SIGABRT, (r.returncode, r.stderr)
    assert f"{name}: unsupported (D={D}, block_size={bs})" in r.stderr


@pytest.mark.parametrize("D", [0, 32, 96, 256])
def test_baseline_unsupported_d_aborts(D):
    r = run_launcher("launch_decode_attn_baseline", D=D)
    assert r.returncode == -signal.SIGABRT
    assert f"D must be 64 or 128 (got {D})" in r.stderr


ONLINE_INVALID = [
    (64, 32, 4, 32),    # D=64 with 4 lanes
    (64, 128, 2, 32),   # bs > D
    (128, 64, 3, 32),   # lanes
    (128, 64, 4, 48),   # tile
    (128, 64, 4, 128),
    (96, 32, 2, 32),
]


@pytest.mark.parametrize("D,bs,L,T", ONLINE_INVALID)
def test_online_unsupported_aborts(D, bs, L, T):
    r = run_launcher("launch_decode_attn_int8_fused_online", D=D, bs=bs, L=L, T=T)
    assert r.returncode == -signal.SIGABRT
    assert (f"launch_decode_attn_int8_fused_online: unsupported "
            f"(D={D}, block_size={bs}, L={L}, T={T})") in r.stderr


def test_online_accepted_set_matches_reference():
    """The accepted (D, bs, L, T) set, enumerated: exactly the reference
    dispatcher's 16 combinations (src/attention_int8_fused_online.cu:209-231)."""
    sys.path.insert(0, os.path.join(REPO, "parallel-final-project_b200"))
    accepted = set()
    for D in (32, 64, 96, 128, 256):
        for bs in (16, 32, 64, 128, 256):
            for L in (1, 2, 3, 4, 8):
                for T in (16, 32, 48, 64, 128):
                    ok = ((D == 128 and L in (2, 4) and T in (32, 64) and bs in (32, 64, 128)) or
                          (D == 64 and L == 2 and T in (32, 64) and bs in (32, 64)))
                    if ok:
                        accepted.add((D, bs, L, T))
    assert len(accepted) == 16
    # spot-check both sides of the boundary in child processes (a valid call
    # would reach the GPU, so only invalid neighbours are executed here)
    for D, bs, L, T in [(64, 64, 4, 64), (128, 128, 2, 16)]:
        assert (D, bs, L, T) not in accepted
        assert run_launcher("launch_decode_attn_int8_fused_online", D=D, bs=bs, L=L,
                            T=T).returncode == -signal.SIGABRT
