"""Host-side logic of the multi-GPU decode, on CPU ranks over gloo
(world size 2 and 3): the token split (workloads.token_slice), the partial
record format (acc[D], m, l), the all-gather and the log-sum-exp merge
reproduce single-device attention.  The device kernels of the same path are
covered by the GPU tests; this checks the orchestration and the math."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tqkv import workloads as W

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, case, result_q):
    import sys
    sys.path.insert(0, REPO)
    sys.path.insert(0, os.path.join(REPO, "tests"))
    from oracle import oracle as O
    import golden.gen as gen
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, H, S, D, bs, seed, dist_name = gen.CASES[case]
        q, k, v = gen.inputs(case)
        s0, s1 = W.token_slice(S, rank, world)
        kq, ks = O.kv_compress(np.ascontiguousarray(k[:, :, s0:s1]), bs)
        vq, vs = O.kv_compress(np.ascontiguousarray(v[:, :, s0:s1]), bs)
        if s1 > s0:
            rec = O.attention_partial(q, O.dequantize(kq, ks, bs), O.dequantize(vq, vs, bs))
        else:
            rec = np.zeros((B * H, D + 2))
            rec[:, D] = -np.inf
        local = torch.from_numpy(rec.astype(np.float64))
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local)
        o = O.lse_combine(torch.stack(parts).numpy())
        if rank == 0:
            kq, ks = O.kv_compress(k, bs)
            vq, vs = O.kv_compress(v, bs)
            full = O.attention(q, O.dequantize(kq, ks, bs), O.dequantize(vq, vs, bs))
            result_q.put(float(np.max(np.abs(o.reshape(full.shape) - full))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("case", ["int8_bs128_ragged", "int8_bs32_lognormal"])
def test_split_s_gather_combine(world, case):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    err = q.get(timeout=10)
    assert err < 1e-5, err


@pytest.mark.parametrize("S", [1, 7, 2048, 131072, 100_003])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_token_slices_partition(S, world):
    covered = []
    for r in range(world):
        s0, s1 = W.token_slice(S, r, world)
        assert 0 <= s0 <= s1 <= S
        covered.extend(range(s0, s1)) if S < 5000 else covered.append((s0, s1))
    if S < 5000:
        assert covered == list(range(S))
    else:
        assert covered[0][0] == 0 and covered[-1][1] == S
        assert all(a[1] == b[0] for a, b in zip(covered, covered[1:]))


@pytest.mark.parametrize("BH", [1, 5, 128, 512])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_head_slices_partition(BH, world):
    seen = []
    for r in range(world):
        h0, h1 = W.head_slice(BH, r, world)
        seen.extend(range(h0, h1))
    assert seen == list(range(BH))


def test_longctx_slices_are_chunk_aligned():
    w = W.WORKLOADS["int8_longctx"]
    for world in (2, 4, 8):
        for r in range(world):
            s0, s1 = W.token_slice(w.S, r, world)
            assert s0 % W.CHUNK == 0 and (s1 - s0) == w.S // world
