#!/usr/bin/env python3
"""Decode benchmark: INT8 fused online-softmax decode attention on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload int8_longctx]

One step = one decode step of the whole workload: every head's attention of
one query over its int8 KV cache (K and V codes plus fp16 block scales,
resident in HBM).  Default workload: B4 H32 D128 S131072, block size 128
(4.36 GB of KV per step, far above the 126 MB L2, so no L2 flush is needed;
a rank whose KV is under twice the L2 rotates its steps through copies of
the KV, more than three L2s in all, and the L2-hot figure is reported
beside it).

Multi-GPU (torchrun, one process per GPU): the S tokens of every head are
split across ranks; in one launch per step each rank decodes its slice,
pushes each head's (acc, m, l) record to every rank through NVLink peer
mappings and merges every rank's records into O (default; --exchange p2p2
makes that two launches, --exchange nccl all-gathers the records over NCCL
and merges them with the log-sum-exp combine kernel).  Total work is fixed,
so scaling is strong.  --shard bh splits heads instead, with no collective.
Time is device time (CUDA events), max over ranks; every N > 1 line carries
its O checked against the one-GPU decode of sampled heads.

The end-to-end figure (e2e) runs each step through the public API from pinned
host memory: H2D of q and the new token's k, v; decode with the append of
k, v fused into the same launch; D2H of O.

Rank 0 prints one JSON line.  --impl reference times the reference's CPU
formulation of the same step (its Python check's dequantise + fp32
attention, restated in oracle/torch_port.py) on the host cores.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "parallel-final-project_b200"))
sys.path.insert(0, REPO)

import torch  # noqa: E402

METRIC = ("decode µs/step & effective HBM GB/s (% of ~8 TB/s), INT8 fused-online, "
          "1/2/4/8 GPU")
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
DECODE_KERNEL = "decode_attn_kernel"
TRAFFIC_PROFILE = os.path.join(REPO, "profiles", "decode_int8_longctx_traffic.txt")


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", default="int8_longctx")
    p.add_argument("--shard", choices=["auto", "s", "bh"], default="auto",
                   help="multi-GPU split: tokens (s, with NCCL all-gather) or heads (bh, no "
                        "collective); auto = bh for int8_bh_shard, s otherwise")
    p.add_argument("--no-graph", action="store_true", help="launch eagerly instead of CUDA graphs")
    p.add_argument("--no-kernel-table", action="store_true",
                   help="skip the per-kernel measurements of compress / reconstruct / fp16 decode")
    p.add_argument("--exchange", choices=["p2p", "p2p2", "nccl"], default="p2p",
                   help="split-S record exchange: NVLink peer writes and the bounded-wait "
                        "merge in the decode launch itself (p2p, one cooperative launch per "
                        "step), the same as two launches, decode then combine (p2p2), or NCCL "
                        "all-gather + combine kernel (nccl, never graph-captured)")
    p.add_argument("--no-cpu-baseline", action="store_true",
                   help="skip the CPU baseline leg (rank 0, N=1)")
    p.add_argument("--cpu-budget-s", type=float, default=20.0,
                   help="host seconds for the CPU baseline sample")
    p.add_argument("--csv", default=None,
                   help="also append a row in the reference bench's CSV schema "
                        "(src/benchmark.cpp:109) plus gpus, eff_GBps, pct_peak (rank 0)")
    return p.parse_args()


CSV_HEADER = ("mode,B,H,D,S,block_size,iters,attn_us,reconstruct_us,compress_us,total_us,"
              "std_us,min_us,bytes_kv,tile_n,lanes_per_thread,gpus,eff_GBps,pct_peak")


def append_csv(path: str, row: dict) -> None:
    """One row of the reference bench's CSV (same columns, same meaning; the
    tile and lane knobs do not apply and are 0) with three added columns."""
    new = not os.path.exists(path) or os.path.getsize(path) == 0
    with open(path, "a") as f:
        if new:
            f.write(CSV_HEADER + "\n")
        f.write(",".join(str(row[c]) for c in CSV_HEADER.split(",")) + "\n")


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def decode_plan(tqkv, BH: int, S: int, device) -> dict:
    """The decode kernel's work split for this rank's slice (host-only query
    of the library), assuming 4 resident CTAs per SM."""
    import ctypes
    try:
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        out = [ctypes.c_longlong() for _ in range(4)]
        if tqkv.load().tqkv_decode_plan(BH, S, sms * 4, *[ctypes.byref(o) for o in out]) != 0:
            return None
        grid, chunk, nchunks, max_parts = (o.value for o in out)
        return {"grid": grid, "chunk_rows": chunk, "chunks": nchunks,
                "schedule": "dynamic chunks" if nchunks > grid else "one run per CTA",
                "max_pieces_per_head": max_parts}
    except Exception:  # informational only
        return None


def traffic_per_launch(workload_name: str, n_gpus: int):
    """DRAM bytes per decode launch from the committed ncu summary
    (`traffic_bytes_per_launch <workload> <n_gpus> <bytes>` lines), or None."""
    try:
        with open(TRAFFIC_PROFILE) as f:
            for line in f:
                parts = line.split()
                if (len(parts) == 4 and parts[0] == "traffic_bytes_per_launch"
                        and parts[1] == workload_name and int(parts[2]) == n_gpus):
                    return int(parts[3])
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------
# NVML sampling loop, run in a child process so that it keeps sampling while
# the benchmark's main thread sits in CUDA calls (which can hold the GIL when
# the launch queue is full).  Prints "ready", then one line per sample:
# "monotonic_s sm_mhz mem_mhz power_mw reasons_mask", until its stdin closes.
_SAMPLER_SRC = r"""
import sys, threading, time
import pynvml
pynvml.nvmlInit()
h = pynvml.nvmlDeviceGetHandleByIndex(int(sys.argv[1]))
interval = float(sys.argv[2])
stop = threading.Event()
threading.Thread(target=lambda: (sys.stdin.read(), stop.set()), daemon=True).start()
print("ready", pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM), flush=True)
while not stop.is_set():
    try:
        print(time.monotonic(), pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
              pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_MEM),
              pynvml.nvmlDeviceGetPowerUsage(h),
              pynvml.nvmlDeviceGetCurrentClocksEventReasons(h), flush=True)
    except pynvml.NVMLError:
        pass
    time.sleep(interval)
"""


class ClockSampler:
    """Samples SM clock, memory clock, power and clock-event (throttle)
    reasons with NVML from a child process while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, interval_s: float = 0.002):
        self.samples, self.reasons = [], set()
        self.mem_mhz, self.power_w = [], []
        self.max_mhz = None
        self.device_index, self.interval = device_index, interval_s
        self.proc = None
        self.window = [None, None]   # host monotonic times bracketing the timed region

    def mark_start(self):
        self.window[0] = time.monotonic()

    def mark_end(self):
        self.window[1] = time.monotonic()

    def __enter__(self):
        import subprocess
        try:
            self.proc = subprocess.Popen(
                [sys.executable, "-c", _SAMPLER_SRC, str(self.device_index), str(self.interval)],
                stdin=subprocess.PIPE, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
            first = self.proc.stdout.readline().split()
            if first[:1] == ["ready"]:
                self.max_mhz = int(first[1])
            else:
                self.proc.kill()
                self.proc = None
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is None:
            return
        out, _ = self.proc.communicate(input="", timeout=30)
        rows = []
        for line in out.splitlines():
            f = line.split()
            if len(f) != 5:
                continue
            rows.append((float(f[0]),) + tuple(int(x) for x in f[1:]))
        # keep the samples taken while the timed region ran (the sampler also
        # runs through the barrier before it, when the GPU may sit idle)
        t0, t1 = self.window
        if t0 is not None and t1 is not None:
            inside = [r for r in rows if t0 <= r[0] <= t1]
            rows = inside if inside else rows
        for _, sm, mem, mw, mask in rows:
            self.samples.append(sm)
            self.mem_mhz.append(mem)
            self.power_w.append(mw / 1000.0)
            for bit, name in self.REASONS.items():
                if mask & bit and name != "gpu_idle":
                    self.reasons.add(name)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "sm_mhz_min": min(self.samples), "mem_mhz": statistics.median(self.mem_mhz),
                "power_w_median": statistics.median(self.power_w),
                "power_w_max": max(self.power_w),
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
def cpu_baseline_sample(w, budget_s: float, steps: int = 0):
    """Times the reference's CPU formulation (dequantise + fp32 attention) on a
    bounded sample of the workload: `nh` whole heads (or, if one head is too
    slow for the budget, a token prefix of one head).  Returns a dict with
    GB/s on the algorithmic KV bytes of the sample."""
    import numpy as np
    from oracle import oracle as O
    from oracle import torch_port

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(w.seed)

    def make(nh, S):
        q = torch.randn((1, nh, w.D), generator=g).half()
        k = torch.randn((1, nh, S, w.D), generator=g).half()
        v = torch.randn((1, nh, S, w.D), generator=g).half()
        kq, ks = O.kv_compress(k.numpy(), w.block_size)
        vq, vs = O.kv_compress(v.numpy(), w.block_size)
        return (q, torch.from_numpy(kq), torch.from_numpy(ks), torch.from_numpy(vq),
                torch.from_numpy(vs))

    def run(args):
        t0 = time.perf_counter()
        torch_port.int8_decode_step(*args, w.block_size)
        return time.perf_counter() - t0

    # calibrate on a 1/8-head prefix
    S_cal = max(w.S // 8, 64)
    cal = make(1, S_cal)
    run(cal)
    t_cal = run(cal)
    per_head_s = t_cal * (w.S / S_cal)
    per_step_budget = budget_s / max(1, steps if steps else 5)
    if per_head_s <= per_step_budget:
        nh = int(max(1, min(w.BH, per_step_budget // per_head_s)))
        S_s = w.S
    else:
        nh = 1
        S_s = int(max(64, min(w.S, w.S * per_step_budget / per_head_s)))
    args = make(nh, S_s)
    sample_bytes = w.kv_bytes_int8(S_s) * nh // w.BH
    desc = (f"{nh} head(s) x {S_s} tokens of {w.name} (of {w.BH} heads x {w.S}); "
            f"torch fp32 dequantise + einsum/softmax/einsum, {threads} threads")
    return args, run, sample_bytes, desc, threads


def run_reference(args, w):
    """--impl reference: the reference's CPU path on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    steps, warmup = args.steps, args.warmup
    budget = min(150.0, 2.0 * (steps + warmup))
    sample, run, sample_bytes, desc, threads = cpu_baseline_sample(w, budget, steps + warmup)
    for _ in range(warmup):
        run(sample)
    times = [run(sample) for _ in range(steps)]
    t = statistics.mean(times)
    gbs = sample_bytes / t / 1e9
    full_step_ms = t * 1e3 * (w.kv_bytes_int8() / sample_bytes)
    line = {
        "metric": METRIC, "value": gbs, "unit": "GB/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": steps, "warmup": warmup,
        "ms_per_step": full_step_ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": w.name, "B": w.B, "H": w.H, "S": w.S, "D": w.D,
                   "block_size": w.block_size, "parallelism": "host cores"},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": desc + "; ms_per_step extrapolated to the full step"},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
def kernel_table(w, tqkv, kq, ks, vq, vs, q, comp_us, ws, reps: int = 5):
    """Each kernel of the path on the workload's own tensors: algorithmic
    bytes per launch, mean CUDA-event time, GB/s and the fraction of the
    measured HBM peak.  Kernel C (two-pass INT8) is the same kernel as Kernel D
    here, so it shares the headline numbers."""
    peak, _ = measured_peaks()
    BH, S, D, bs = w.BH, w.S, w.D, w.block_size
    rows = BH * S
    scale_b = rows * (D // bs) * 2
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        ev0.record()
        for _ in range(reps):
            fn()
        ev1.record()
        torch.cuda.synchronize()
        return ev0.elapsed_time(ev1) * 1e3 / reps

    def entry(nbytes, us, what):
        gbs = nbytes / (us * 1e-6) / 1e9
        return {"us": us, "algorithmic_bytes": nbytes, "GBps": gbs, "frac_of_peak": gbs / peak,
                "bytes": what}

    out = {}
    comp = statistics.mean(comp_us)
    out["kv_compress (Kernel A), per tensor"] = entry(
        rows * D * 2 + rows * D + scale_b, comp, "fp16 in + int8 codes + fp16 scales out")
    k16 = torch.empty(kq.shape, dtype=torch.float16, device=kq.device)
    v16 = torch.empty_like(k16)
    us = timed(lambda: tqkv.kv_reconstruct(kq, ks, bs, y=k16))
    out["kv_reconstruct (Kernel B), per tensor"] = entry(
        rows * D + scale_b + rows * D * 2, us, "int8 codes + fp16 scales in, fp16 out")
    tqkv.kv_reconstruct(vq, vs, bs, y=v16)
    o16 = torch.empty((q.shape[0], q.shape[1], D), dtype=torch.float16, device=q.device)
    us = timed(lambda: tqkv.decode_fp16(q, k16, v16, out=o16, workspace=ws))
    out["decode_fp16 (baseline attention)"] = entry(
        2 * rows * D * 2, us, "fp16 K + V (the reference's fp16 bytes_kv, src/benchmark.cpp:152)")
    out["decode_int8 two-pass (Kernel C)"] = "same kernel and numbers as Kernel D (headline)"
    del k16, v16
    torch.cuda.empty_cache()
    return out



def timing_check(step_ms: float, e2e_ms: float, comparable: bool) -> str:
    """The device-timed step must not be slower than the end-to-end step,
    which does the same work plus copies and a host sync every step."""
    if not comparable:
        return "n/a (device-timed steps rotate through KV copies to read from HBM; e2e steps reuse one)"
    if step_ms <= e2e_ms * 1.02:
        return "ok: device step <= e2e step"
    msg = (f"device step {step_ms * 1e3:.1f} us > e2e step {e2e_ms * 1e3:.1f} us: "
           "the device timing includes waits that are not the step")
    print("bench: " + msg, file=sys.stderr, flush=True)
    return "FAILED: " + msg


PARITY_TOL = 1e-3


def multi_gpu_parity(w, tqkv, out, shard: str, rank: int, world: int, h0: int, dev):
    """O of the multi-GPU step (every rank's, gathered to rank 0) against the
    one-GPU decode of a sample of heads over the whole sequence.  The
    reference's codes are compressed here from the workload's generator, so
    this also checks that every rank's slice holds the right tokens.  Split-S
    ranks all merge the same records in the same order, so their O must be
    bit-identical.  Returns a dict on rank 0 (None elsewhere)."""
    import torch.distributed as dist
    from tqkv import workloads as W
    mine = out.view(-1, w.D).cpu()
    gathered = [None] * world
    dist.all_gather_object(gathered, (rank, h0, mine))
    if rank != 0:
        return None
    BH, D = w.BH, w.D
    if shard == "s":
        full = gathered[0][2]
        identical = all(torch.equal(g[2], full) for g in gathered)
        heads = sorted({0, BH // 3, (2 * BH) // 3, BH - 1})
    else:
        full = torch.empty((BH, D), dtype=torch.float16)
        heads = []
        for _, hh0, o in gathered:
            full[hh0:hh0 + o.shape[0]] = o
            if o.shape[0]:
                heads += [hh0, hh0 + o.shape[0] - 1]
        heads = sorted(set(heads))
        identical = None
    nh = len(heads)
    idx = torch.tensor(heads, device=dev)
    codes = []
    for which in ("k", "v"):
        xq = torch.empty((1, nh, w.S, D), dtype=torch.int8, device=dev)
        xs = torch.empty((1, nh, w.S, D // w.block_size), dtype=torch.float16, device=dev)
        for t0 in range(0, w.S, W.CHUNK):
            t1 = min(t0 + W.CHUNK, w.S)
            x = W.make_kv_slice(w, which, t0, t1, dev).reshape(BH, t1 - t0, D)
            x = x.index_select(0, idx).reshape(1, nh, t1 - t0, D).contiguous()
            cq, cs = tqkv.kv_compress(x, w.block_size)
            xq[:, :, t0:t1] = cq
            xs[:, :, t0:t1] = cs
            del x, cq, cs
        codes += [xq, xs]
    q = W.make_q(w, dev).reshape(BH, D).index_select(0, idx).reshape(1, nh, D).contiguous()
    ref = tqkv.decode_int8(q, *codes, w.block_size).reshape(nh, D).cpu()
    got = full.index_select(0, torch.tensor(heads))
    err = float((got.float() - ref.float()).abs().max())
    finite = bool(torch.isfinite(got.float()).all())
    ok = finite and err <= PARITY_TOL and identical is not False
    return {"max_abs": err, "tol": PARITY_TOL, "heads": heads, "ok": ok,
            "ranks_bit_identical": identical,
            "reference": "one-GPU tqkv_decode_int8 over the whole sequence of the sampled "
                         "heads, codes compressed here from the workload generator"}


def main():
    args = parse_args()
    from tqkv import workloads as W
    w = W.WORKLOADS[args.workload]
    if w.block_size == 0:
        raise SystemExit("bench.py measures the INT8 path; pick an int8_* workload")
    if args.impl == "reference":
        return run_reference(args, w)

    import tqkv
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    # ---- inputs: this rank's share of the workload ----
    shard = args.shard if args.shard != "auto" else ("bh" if w.name == "int8_bh_shard" else "s")
    if world == 1:
        shard = "s"
    BH, D = w.BH, w.D
    if shard == "s":      # every head, tokens [s0, s1)
        s0, s1 = W.token_slice(w.S, rank, world)
        h0, h1 = 0, BH
    else:                 # heads [h0, h1), every token; no collective
        s0, s1 = 0, w.S
        h0, h1 = W.head_slice(BH, rank, world)
    S_loc, BH_loc = s1 - s0, h1 - h0
    q = W.make_q(w, dev).reshape(1, BH, D)[:, h0:h1].contiguous()
    comp_us = []
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kvq = []
    for which in ("k", "v"):
        x = W.make_kv_slice(w, which, s0, s1, dev).reshape(1, BH, S_loc, D)
        if shard == "bh":
            x = x[:, h0:h1].contiguous()
        xq = torch.empty(x.shape, dtype=torch.int8, device=dev)
        xs = torch.empty(x.shape[:3] + (D // w.block_size,), dtype=torch.float16, device=dev)
        for rep in range(3):  # the first rep is warm-up; outputs are overwritten each rep
            ev0.record()
            tqkv.kv_compress(x, w.block_size, xq=xq, scales=xs)
            ev1.record()
            torch.cuda.synchronize()
            if rep:
                comp_us.append(ev0.elapsed_time(ev1) * 1e3)
        kvq.append((xq, xs))
        del x
        torch.cuda.empty_cache()
    (kq, ks), (vq, vs) = kvq
    # A rank whose KV is smaller than twice the L2 rotates through copies of it,
    # more than three L2s in all, so that every timed step reads its KV from
    # HBM with no other work in the timed region; back-to-back steps on one
    # copy (L2-hot) are reported beside it.
    local_bytes = w.kv_bytes_int8(S_loc) * BH_loc // BH
    l2_bytes = torch.cuda.get_device_properties(dev).L2_cache_size
    n_sets = 1 if local_bytes >= 2 * l2_bytes else min(64, -(-3 * l2_bytes // local_bytes))
    kv_sets = [(kq, ks, vq, vs)] + [tuple(t.clone() for t in (kq, ks, vq, vs))
                                    for _ in range(n_sets - 1)]
    set_idx = [0]                     # the copy kernel() streams
    out = torch.empty((1, BH_loc, D), dtype=torch.float16, device=dev)
    ws = tqkv.Workspace(dev)
    collective = world > 1 and shard == "s"
    use_p2p = collective and args.exchange in ("p2p", "p2p2")
    one_launch = use_p2p and args.exchange == "p2p"
    local_rec = torch.empty((BH, D + 2), dtype=torch.float32, device=dev)
    gathered = torch.empty((world, BH, D + 2), dtype=torch.float32, device=dev)
    exchange = tqkv.PeerExchange(world, rank, BH, D) if use_p2p else None

    def kernel():
        kq, ks, vq, vs = kv_sets[set_idx[0]]
        if one_launch:
            exchange.step(q, kq, ks, vq, vs, w.block_size, out, workspace=ws)
        elif use_p2p:
            exchange.publish(q, kq, ks, vq, vs, w.block_size, workspace=ws)
        elif collective:
            tqkv.decode_int8_partial(q, kq, ks, vq, vs, w.block_size, out=local_rec, workspace=ws)
        else:
            tqkv.decode_int8(q, kq, ks, vq, vs, w.block_size, out=out, workspace=ws)

    def comm():
        if one_launch:
            return                   # merged inside the step's launch
        if use_p2p:
            exchange.combine(out)
        elif collective:
            dist.all_gather_into_tensor(gathered, local_rec)
            tqkv.lse_combine(gathered, D, out=out.view(BH, D))

    # End-to-end decode step through the public API: the new token's q, k and
    # v come from pinned host memory, k and v are appended to the int8 cache
    # (tqkv_kv_append at the last row of the rank that holds the sequence's
    # end), the step runs, and O goes back to the host.
    q_host = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    q_host.copy_(q.cpu())
    o_host = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    owns_last = S_loc > 0 and s1 == w.S
    kv_new = torch.empty((2, 1, BH_loc, 1, D), dtype=torch.float16, device=dev)
    kv_new_host = torch.empty(kv_new.shape, dtype=torch.float16, pin_memory=True)
    if owns_last:
        # the token being re-appended is the one already cached at the last row
        # (its fp16 original), so the cache contents stay those of the workload
        last = W.make_kv_slice(w, "k", w.S - 1, w.S, dev).reshape(1, BH, 1, D)[:, h0:h1]
        kv_new_host[0].copy_(last.cpu())
        last = W.make_kv_slice(w, "v", w.S - 1, w.S, dev).reshape(1, BH, 1, D)[:, h0:h1]
        kv_new_host[1].copy_(last.cpu())
        del last

    def e2e_step():
        q.copy_(q_host, non_blocking=True)
        if owns_last:
            kv_new.copy_(kv_new_host, non_blocking=True)
        if owns_last and not collective:      # append fused into the decode launch
            tqkv.decode_int8_append(q, kv_new[0], kv_new[1], kq, ks, vq, vs, S_loc,
                                    w.block_size, out=out, workspace=ws)
        elif owns_last and one_launch:
            exchange.step_append(q, kv_new[0], kv_new[1], kq, ks, vq, vs, S_loc,
                                 w.block_size, out, workspace=ws)
        elif owns_last and use_p2p:
            exchange.publish_append(q, kv_new[0], kv_new[1], kq, ks, vq, vs, S_loc,
                                    w.block_size, workspace=ws)
        elif one_launch:
            exchange.step(q, kq, ks, vq, vs, w.block_size, out, workspace=ws)
        else:
            if owns_last:                     # NCCL path: separate append launches
                tqkv.kv_append(kv_new[0], kq, ks, S_loc - 1, w.block_size)
                tqkv.kv_append(kv_new[1], vq, vs, S_loc - 1, w.block_size)
            kernel()
        comm()
        o_host.copy_(out, non_blocking=True)

    for _ in range(max(args.warmup, 2)):   # also sets kernel attributes and the workspace
        kernel()
        comm()
    torch.cuda.synchronize()

    # CUDA graphs: one for the decode kernel, one for gather + combine, one for
    # the whole end-to-end step; replays keep the GPU fed without launch gaps.
    graphs = []
    steps_graph = None
    # NCCL collectives are never captured (capturing them hung here); the p2p
    # exchange is two plain kernels and captures like the single-GPU step.
    if not args.no_graph and not (collective and not use_p2p):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for fn in (kernel, comm, e2e_step):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        captured = []
        two_part = collective and not one_launch
        for fn in ((kernel, comm, e2e_step) if two_part else (kernel, e2e_step)):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            graphs.append(g)
            captured.append(g.replay)
        # one kernel graph per further KV copy
        set_graphs = [graphs[0]]
        for i in range(1, n_sets):
            set_idx[0] = i
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                kernel()
            set_graphs.append(g)
        set_idx[0] = 0
        graphs += set_graphs[1:]
        turn = [0]

        def replay_next():
            set_graphs[turn[0] % n_sets].replay()
            turn[0] += 1
        if two_part:
            run_kernel, run_comm, run_e2e = captured
        else:                   # one launch per step: nothing else to run
            (run_kernel, run_e2e), run_comm = captured, comm
        if n_sets > 1:
            run_kernel = replay_next
        run_kernel_hot = set_graphs[0].replay
        # With one launch per step, the timed steps are one graph of K launches,
        # as a decoder that captures its decode loop runs them: consecutive
        # launches then start ~2 us apart, where replaying one graph per step
        # leaves 3-8 us between them.  Step i streams copy (1 + i) % n_sets; the
        # aligning step before it streams copy 0.
        if not two_part:
            steps_graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(steps_graph):
                for i in range(args.steps):
                    set_idx[0] = (1 + i) % n_sets
                    kernel()
            set_idx[0] = 0
            graphs.append(steps_graph)
    else:
        turn = [0]

        def eager_next():
            set_idx[0] = turn[0] % n_sets
            turn[0] += 1
            kernel()
            set_idx[0] = 0
        run_kernel, run_comm, run_e2e = (eager_next if n_sets > 1 else kernel), comm, e2e_step
        run_kernel_hot = kernel
    graphs_used = len(graphs) > 0
    if steps_graph is not None:
        steps_graph.replay()          # warm-up of the graph itself
    for _ in range(args.warmup):
        run_kernel()
        run_comm()
    torch.cuda.synchronize()


    # ---- timed region: exactly K steps ----
    # The clock sampler starts before the barrier: it spawns a process, and
    # host-side work between the barrier and the first timed launch would
    # land inside the other ranks' timed regions (their combines wait for this
    # rank).  After the barrier one untimed step goes first, with no host sync
    # between it and the timed steps: every rank's combine ends only once all
    # ranks have published that step, so whatever host skew the ranks leave
    # the barrier with is absorbed there and the timed regions start together.
    # With one launch per step and no L2 overwrite, nothing but the steps runs
    # in the timed region: its time / K is both the step and the launch time,
    # and per-step events (a few us of their own per step) stay out of it;
    # per-step samples come from a second pass below.
    single_launch = not (collective and not one_launch)
    per_step_events = not single_launch
    kev = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(3))
           for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        barrier()
        torch.cuda.synchronize()
        clk.mark_start()
        (run_kernel_hot if steps_graph is not None else run_kernel)()
        run_comm()
        torch.cuda.nvtx.range_push("tqkv_timed")  # lets ncu --nvtx-include select this region
        ev0.record()
        if steps_graph is not None:
            steps_graph.replay()
        else:
            for i in range(args.steps):
                if per_step_events:
                    kev[i][0].record()
                run_kernel()
                if per_step_events:
                    kev[i][1].record()
                run_comm()
                if per_step_events:
                    kev[i][2].record()
        ev1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        clk.mark_end()
    barrier()
    step_ms_local = ev0.elapsed_time(ev1) / args.steps
    if per_step_events:
        kern_ms_local = statistics.mean(a.elapsed_time(b) for a, b, _ in kev)
    else:
        kern_ms_local = step_ms_local
        # per-step samples: the same K steps again, each bracketed by events
        torch.cuda.synchronize()
        barrier()
        run_kernel()
        run_comm()
        for i in range(args.steps):
            kev[i][0].record()
            run_kernel()
            kev[i][1].record()
            run_comm()
            kev[i][2].record()
        torch.cuda.synchronize()
        barrier()
    step_samples_ms = [a.elapsed_time(c) for a, _, c in kev]   # per step, this rank
    # step-to-step period (start of one step to the start of the next)
    period_ms_local = (statistics.median(kev[i][0].elapsed_time(kev[i + 1][0])
                                         for i in range(args.steps - 1))
                       if args.steps > 1 else step_ms_local)
    hot_ms_local = step_ms_local
    if n_sets > 1:                # the same steps back to back on one copy, KV left in L2
        torch.cuda.synchronize()
        barrier()
        run_kernel_hot()
        run_comm()
        ev0.record()
        for i in range(args.steps):
            run_kernel_hot()
            run_comm()
        ev1.record()
        torch.cuda.synchronize()
        barrier()
        hot_ms_local = ev0.elapsed_time(ev1) / args.steps
    err = tqkv.read_device_error()

    # ---- end to end through the public API: H2D q, decode, D2H O, per step ----
    e2e_steps = max(1, min(args.steps, 50))
    for _ in range(3):
        run_e2e()
        torch.cuda.current_stream().synchronize()
    barrier()
    torch.cuda.synchronize()
    run_e2e()          # aligns the ranks, as before the timed region above
    torch.cuda.current_stream().synchronize()
    ev0.record()
    for _ in range(e2e_steps):
        run_e2e()
        torch.cuda.current_stream().synchronize()  # the next token needs O on the host
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms_local = ev0.elapsed_time(ev1) / e2e_steps

    # the timed steps again as one graph replay per step (no per-step events),
    # after the end-to-end steps so that they run in the same state as before
    graph_per_step_ms_local = step_ms_local
    if steps_graph is not None:
        torch.cuda.synchronize()
        barrier()
        run_kernel()
        run_comm()
        ev0.record()
        for i in range(args.steps):
            run_kernel()
            run_comm()
        ev1.record()
        torch.cuda.synchronize()
        barrier()
        graph_per_step_ms_local = ev0.elapsed_time(ev1) / args.steps
    k_graph = steps_graph is not None
    del graphs, steps_graph, run_kernel, run_comm, run_e2e

    # ---- the path's other kernels, on this workload (one GPU only) ----
    kernels = None
    if world == 1 and not args.no_kernel_table:
        kernels = kernel_table(w, tqkv, kq, ks, vq, vs, q, comp_us, ws)

    # ---- max over ranks ----
    t = torch.tensor([step_ms_local, kern_ms_local, e2e_ms_local, hot_ms_local, float(err),
                      period_ms_local, graph_per_step_ms_local], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms, kern_ms, e2e_ms, hot_ms, err_max, period_ms, graph_per_step_ms = t.tolist()

    # ---- multi-GPU parity: O against the one-GPU decode of sampled heads ----
    parity = None
    if world > 1:
        parity = multi_gpu_parity(w, tqkv, out, shard, rank, world, h0, dev)

    total_bytes = w.kv_bytes_int8()
    peak, peak_kind = measured_peaks()
    value = total_bytes / (step_ms * 1e-3) / 1e9
    achieved = local_bytes / (kern_ms * 1e-3) / 1e9
    traffic = traffic_per_launch(w.name, world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sample, run, sample_bytes, desc, threads = cpu_baseline_sample(w, args.cpu_budget_s)
        run(sample)
        times = [run(sample) for _ in range(5)]
        cpu_t = statistics.median(times)
        cpu = {"value": sample_bytes / cpu_t / 1e9, "unit": "GB/s", "cores": threads,
               "kind": "port", "sample": desc + f"; median of 5 runs, {cpu_t * 1e3:.1f} ms each"}

    if exchange is not None:
        exchange.close()
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": step_ms,
        "us_per_step": step_ms * 1e3,
        "pct_of_8TBps": 100.0 * value / world / NOMINAL_HBM_GBS,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8",
        "data": f"synthetic, generated on device: {w.description}",
        "config": {
            "workload": w.name, "B": w.B, "H": w.H, "S": w.S, "D": w.D,
            "block_size": w.block_size, "global_batch": w.B, "seq_len": w.S,
            "parallelism": (f"split-S x{world} + NVLink peer exchange, one launch per step"
                            if one_launch else
                            f"split-S x{world} + NVLink peer exchange, decode + combine launches"
                            if use_p2p else
                            f"split-S x{world} + NCCL all-gather" if collective else
                            f"B*H shards x{world}, no collective" if world > 1 else "1 GPU"),
            "arithmetic": "int8 codes; K-dot in s32 (dp4a); softmax and V accumulation in fp32",
            "cuda_graphs": bool(graphs_used),
            "decode_plan": decode_plan(tqkv, BH_loc, S_loc, dev) if S_loc > 0 else None,
            "l2": (f"KV {local_bytes / 1e6:.1f} MB per GPU per step >= 2x the "
                   f"{l2_bytes / 1e6:.0f} MB L2; no flush needed" if n_sets == 1 else
                   f"KV {local_bytes / 1e6:.1f} MB per GPU per step < 2x the {l2_bytes / 1e6:.0f} "
                   f"MB L2: steps rotate through {n_sets} copies of it "
                   f"({n_sets * local_bytes / 1e6:.0f} MB), so each reads its KV from HBM"),
        },
        "roofline": {
            "bound": "hbm",
            "kernel": DECODE_KERNEL + (" (split-S, records exchanged and merged in the launch)"
                                       if one_launch else
                                       " (split-S partial)" if collective else ""),
            "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "peak_source": peak_kind, "traffic": traffic,
            "algorithmic_bytes_per_launch": local_bytes, "launch_ms": kern_ms,
            "launch_timing": ("timed region / K: one launch per step, the K launches in one "
                              "CUDA graph" if k_graph else
                              "timed region / K: one launch per step, back to back"
                              if not per_step_events else
                              "mean of per-launch CUDA events inside the timed region"),
        },
        "timed_launches": ("one CUDA graph holding the K steps, replayed once" if k_graph
                           else "one CUDA graph replay per step" if graphs_used
                           else "eager launches"),
        "us_per_step_one_graph_per_step": graph_per_step_ms * 1e3 if k_graph else None,
        "cpu_baseline": cpu,
        "e2e": {"value": total_bytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                "us_per_step": e2e_ms * 1e3,
                "h2d_bytes_per_step": q.numel() * q.element_size() +
                (kv_new.numel() * kv_new.element_size() if owns_last else 0),
                "d2h_bytes_per_step": out.numel() * out.element_size(),
                "step": "H2D q, k_new, v_new (pinned) -> " +
                        ("append k, v to the int8 cache (separate launches) -> decode"
                         if collective and not use_p2p else
                         "decode with the append of k, v, the record exchange and the merge "
                         "fused in one launch (tqkv_decode_int8_append_exchange on the rank "
                         "holding the newest tokens, tqkv_decode_int8_exchange elsewhere)"
                         if one_launch else
                         "decode with the append of k, v fused in (tqkv_decode_int8_append" +
                         ("_publish on the rank holding the newest tokens)" if collective else ")")) +
                        (" -> exchange + combine" if collective and not one_launch else "") +
                        " -> D2H O -> host sync"},
        "gpu_launches": args.steps * (2 if collective and not one_launch else 1),
        "clocks": clk.summary(),
        "compress": {"us_per_tensor": statistics.mean(comp_us),
                     "GBps": (w.BH * S_loc * w.D * 3 + w.BH * S_loc * (w.D // w.block_size) * 2)
                     / (statistics.mean(comp_us) * 1e-6) / 1e9},
        "l2_hot": None if n_sets == 1 else {
            "us_per_step": hot_ms * 1e3, "GBps": total_bytes / (hot_ms * 1e-3) / 1e9,
            "note": "same steps back to back, KV resident in L2"},
        "device_error": int(err_max),
        "step_period_us_median": period_ms * 1e3,
        "timing_check": timing_check(step_ms, e2e_ms, n_sets == 1),
        "parity_max_abs": None if parity is None else parity["max_abs"],
        "parity": parity,
        "kernels": kernels,
    }
    print(json.dumps(line), flush=True)
    if args.csv:
        append_csv(args.csv, {
            "mode": "int8_fused_online", "B": w.B, "H": w.H, "D": w.D, "S": w.S,
            "block_size": w.block_size, "iters": args.steps, "attn_us": step_ms * 1e3,
            "reconstruct_us": 0, "compress_us": statistics.mean(comp_us),
            "total_us": step_ms * 1e3,
            "std_us": statistics.pstdev(step_samples_ms) * 1e3,
            "min_us": min(step_samples_ms) * 1e3, "bytes_kv": total_bytes, "tile_n": 0,
            "lanes_per_thread": 0, "gpus": world, "eff_GBps": value,
            "pct_peak": 100.0 * value / world / NOMINAL_HBM_GBS})
    if parity is not None and not parity["ok"]:
        print(f"bench: multi-GPU output differs from the one-GPU decode: {parity}",
              file=sys.stderr, flush=True)
        return 1
    if int(err_max) != 0:
        print(f"bench: device error code {int(err_max)}", file=sys.stderr, flush=True)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
