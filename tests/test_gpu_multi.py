"""Split-S decode across GPUs: each rank holds a token slice of every head,
runs the partial kernel, the records are all-gathered over NCCL and merged by
the LSE combine kernel on every rank; and the same split over NVLink peer
mappings (publish + combine, no NCCL) for several consecutive steps, also
with the newest token appended inside the last rank's publish launch.  All
must equal the one-GPU decode of the whole sequence, and the NVLink steps,
two-launch (publish + combine) and one-launch (tqkv_decode_int8_exchange)
alternating, must give every rank the same O bit for bit.  Runs as one child
process per GPU (2 to 4 GPUs, NCCL with NVLS off); skipped when fewer than 2
GPUs are visible."""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q_out):
    import sys
    sys.path.insert(0, os.path.join(REPO, "parallel-final-project_b200"))
    import torch.distributed as dist
    import tqkv
    from tqkv import workloads as W
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        w = W.Workload("t", 2, 4, 20000, 128, 64, 7, "lognormal_channels", "test")
        s0, s1 = W.token_slice(w.S, rank, world)
        q = W.make_q(w, dev)
        k = W.make_kv_slice(w, "k", s0, s1, dev)
        v = W.make_kv_slice(w, "v", s0, s1, dev)
        kq, ks = tqkv.kv_compress(k, w.block_size)
        vq, vs = tqkv.kv_compress(v, w.block_size)
        rec = tqkv.decode_int8_partial(q, kq, ks, vq, vs, w.block_size)
        gathered = torch.empty((world,) + tuple(rec.shape), dtype=rec.dtype, device=dev)
        dist.all_gather_into_tensor(gathered, rec)
        o = tqkv.lse_combine(gathered, w.D).view(w.B, w.H, w.D)
        # one-GPU reference on the full sequence (every rank can build it)
        kf, vf = W.make_kv_slice(w, "k", 0, w.S, dev), W.make_kv_slice(w, "v", 0, w.S, dev)
        kqf, ksf = tqkv.kv_compress(kf, w.block_size)
        vqf, vsf = tqkv.kv_compress(vf, w.block_size)
        full = tqkv.decode_int8(q, kqf, ksf, vqf, vsf, w.block_size)
        torch.cuda.synchronize()
        err = (o.float() - full.float()).abs().max().item()
        # the same split over NVLink peer mappings (no NCCL), several steps
        ex = tqkv.PeerExchange(world, rank, w.BH, w.D)
        try:
            for step in range(8):
                qs = (q.float() * (1.0 + 0.25 * step)).half()
                if step % 2 == 0:      # two launches: publish, then combine
                    ex.publish(qs, kq, ks, vq, vs, w.block_size)
                    o2 = ex.combine(torch.empty_like(o))
                else:                  # one launch
                    o2 = ex.step(qs, kq, ks, vq, vs, w.block_size, torch.empty_like(o))
                ref2 = tqkv.decode_int8(qs, kqf, ksf, vqf, vsf, w.block_size)
                torch.cuda.synchronize()
                err = max(err, (o2.float() - ref2.float()).abs().max().item())
                # every rank merges the same records in the same order
                allo = [torch.empty_like(o2) for _ in range(world)]
                dist.all_gather(allo, o2)
                assert all(torch.equal(a, o2) for a in allo), step
            # decode loop: the rank holding the sequence end appends each new
            # token inside its publish launch; reference: the one-GPU fused
            # append + decode over the whole, growing cache
            steps, S_loc = 4, s1 - s0
            last = rank == world - 1

            def grow(t, rows):
                c = torch.zeros(t.shape[:2] + (rows,) + t.shape[3:], dtype=t.dtype, device=dev)
                c[:, :, :t.shape[2]] = t
                return c
            mine = [grow(t, S_loc + steps) for t in (kq, ks, vq, vs)]
            whole = [grow(t, w.S + steps) for t in (kqf, ksf, vqf, vsf)]
            gen = torch.Generator(device=dev)
            for i in range(steps):
                gen.manual_seed(1000 + i)
                kn = torch.randn((w.B, w.H, 1, w.D), generator=gen, device=dev).half()
                vn = torch.randn((w.B, w.H, 1, w.D), generator=gen, device=dev).half()
                qs = torch.randn((w.B, w.H, w.D), generator=gen, device=dev).half()
                one_launch = i % 2 == 1
                if last and one_launch:
                    o3 = ex.step_append(qs, kn, vn, *mine, S_loc + i + 1, w.block_size,
                                        torch.empty_like(o))
                elif one_launch:
                    o3 = ex.step(qs, kq, ks, vq, vs, w.block_size, torch.empty_like(o))
                else:
                    if last:
                        ex.publish_append(qs, kn, vn, *mine, S_loc + i + 1, w.block_size)
                    else:
                        ex.publish(qs, kq, ks, vq, vs, w.block_size)
                    o3 = ex.combine(torch.empty_like(o))
                ref3 = tqkv.decode_int8_append(qs, kn, vn, *whole, w.S + i + 1, w.block_size)
                torch.cuda.synchronize()
                err = max(err, (o3.float() - ref3.float()).abs().max().item())
        finally:
            ex.close()
        q_out.put((rank, err, tqkv.read_device_error()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 or more GPUs")
def test_split_s_over_nccl_matches_single_gpu():
    world = min(4, torch.cuda.device_count())
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    for rank, err, dev_err in res:
        assert err < 1e-3, (rank, err)
        assert dev_err == 0
