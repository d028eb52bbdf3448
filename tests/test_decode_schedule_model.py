"""CPU model of the decode kernel's schedule and memory accesses.

Compute-sanitizer is not available for this kernel's GPU runs, so its bounds
are established here instead: the host plan (make_plan in tqkv_capi.cu), the
producer's chunk and tile loops and bulk-copy spans, the consumers' shared-
memory reads and the workspace part indices (decode_attn.cuh) are re-enacted
for many shapes, asserting that
  * every token row of every head is covered exactly once, whichever CTA
    claims which chunk (chunks are handed out dynamically, so the model walks
    chunks rather than CTAs);
  * every bulk copy is 16-byte aligned, a multiple of 16 bytes, inside its
    global buffer and inside its shared-memory slot;
  * every plain edge load is inside its buffer and its slot;
  * every consumer read of scales and q stays inside the stage;
  * part indices stay below max_parts of the workspace layout.
The tile size, stage count and planning constants are read from the sources,
so the model follows the code."""
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(REPO, "parallel-final-project_b200", "csrc")


def _const(path, name):
    src = open(os.path.join(CSRC, path)).read()
    m = re.search(rf"constexpr\s+(?:long long|int)\s+{name}\s*=\s*([0-9]+)", src)
    assert m, name
    return int(m.group(1))


TILE_BYTES = _const("decode_attn.cuh", "kDecodeTileBytes")
STAGES = _const("decode_attn.cuh", "kDecodeStages")
WARPS = _const("decode_attn.cuh", "kDecodeConsumerWarps")
MIN_ROWS = _const("tqkv_capi.cu", "kMinRowsPerCta")
CHUNKS_PER_CTA = _const("tqkv_capi.cu", "kChunksPerCta")
CHUNK_ALIGN = _const("tqkv_capi.cu", "kChunkAlign")
MIN_DYNAMIC = _const("tqkv_capi.cu", "kMinDynamicRowsPerCta")
BOUND_OCC = _const("tqkv_capi.cu", "kMaxCtasPerSmBound")
SMS = 148


def make_plan(BH, S, max_ctas):
    """(grid, chunk rows C, number of chunks, max_parts)"""
    total = BH * S
    g = max(min(-(-total // MIN_ROWS), max_ctas), 1)
    c = -(-total // g)
    if c >= MIN_DYNAMIC:
        c = -(-total // (g * CHUNKS_PER_CTA))
        c = -(-c // CHUNK_ALIGN) * CHUNK_ALIGN
    elif g > 1:
        c = -(-c // 16) * 16
    n = -(-total // c)
    return min(n, g), c, n, (S - 1) // c + 2


def plan_span(src, n, lo, hi):
    a16 = src & ~15
    b16 = (src + n + 15) & ~15
    blo, bhi = max(a16, (lo + 15) & ~15), min(b16, hi & ~15)
    return (blo, blo - a16, bhi - blo) if blo < bhi else (0, 0, 0)


def check(BH, S, D, bs, half, occ, offs=(0, 0), S_stride=None, T_new=0, group=1):
    """T_new > 0: the fused-append variant, whose tiles get rows >= S - T_new
    from the consumer warps' quantisation instead of the bulk copies.
    group > 1: BH query heads over BH / group K/V heads (GQA)."""
    S_stride = S if S_stride is None else S_stride
    elem = 2 if half else 1
    RB = D * elem
    LPR = RB // 16
    G = WARPS * 32 // LPR
    TILE = TILE_BYTES // RB
    assert TILE == 4 * G
    nsub = 1 if half else D // bs
    slot = 0 if half else TILE * nsub * 2 + 32
    qslot = D * 2 + 32
    total = BH * S
    grid, R, nchunks, _ = make_plan(BH, S, SMS * occ)
    # workspace layout bound: the most parts per head over every grid cap
    maxp = max(make_plan(BH, S, SMS * o)[3] for o in range(1, BOUND_OCC + 1))
    assert 1 <= grid <= nchunks and nchunks < 2 ** 32
    if nchunks == 1:      # no workspace: the one chunk holds every head whole
        assert R >= total
    kbase, sbase, qbase = 1 << 40, (1 << 41) + offs[0], (1 << 42) + offs[1]
    assert BH % group == 0
    k_end = kbase + BH // group * S_stride * RB
    s_end, q_end = sbase + BH // group * S_stride * nsub * 2, qbase + BH * D * 2
    covered = 0
    for c in range(nchunks):
        r0, r1 = c * R, min((c + 1) * R, total)
        assert r0 < r1
        r = r0
        while r < r1:
            bh = r // S
            head0 = bh * S
            ta, tb = r - head0, min(r1 - head0, S)
            tiles = list(range(ta, tb, TILE))
            # every tile of small cases; first/last few of big ones
            if len(tiles) > 8:
                tiles = tiles[:4] + tiles[-4:]
            if T_new:   # every tile holding new rows, too
                tiles = sorted(set(tiles) | {t for t in range(ta, tb, TILE)
                                             if t + TILE > S - T_new})
            for t0 in tiles:
                cnt = min(TILE, tb - t0)
                nb = min(max(S - T_new - t0, 0), cnt) if T_new else cnt   # rows from the cache
                row0 = bh // group * S_stride + t0   # memory row, as the kernel computes it
                assert 0 < cnt <= TILE and t0 + cnt <= S
                assert (kbase + row0 * RB) % 16 == 0 and nb * RB % 16 == 0
                assert kbase <= kbase + row0 * RB and kbase + (row0 + nb) * RB <= k_end
                assert cnt * RB <= TILE_BYTES
                if not half:
                    n = nb * nsub * 2
                    src = sbase + row0 * nsub * 2
                    hi = src + n if nb < cnt else s_end
                    b_src, b_off, b_n = plan_span(src, n, sbase, hi)
                    if nb < cnt:
                        # the bulk copy stops short of the new rows' scales,
                        # which the consumer warps write into the same slot
                        assert not b_n or b_off + b_n <= (src & 15) + n
                        for t in range(nb, cnt):
                            for j in range(nsub):
                                o = (src & 15) + (t * nsub + j) * 2
                                assert o + 2 <= slot
                                assert sbase <= src + (t * nsub + j) * 2 < s_end
                    if b_n:
                        assert sbase <= b_src and b_src + b_n <= s_end
                        assert b_src % 16 == 0 and b_n % 16 == 0 and b_off % 16 == 0
                        assert b_off + b_n <= slot
                    assert (src & 15) + 2 * TILE * nsub <= slot      # consumer reads
                    a16 = src & ~15
                    for p in range(src, src + n, 2):                 # edge plain loads
                        if not (b_n and b_src <= p < b_src + b_n):
                            assert sbase <= p < s_end and p - a16 + 2 <= slot
                if t0 == ta:
                    qsrc = qbase + bh * D * 2
                    b_src, b_off, b_n = plan_span(qsrc, D * 2, qbase, q_end)
                    if b_n:
                        assert b_off + b_n <= qslot and qbase <= b_src and b_src + b_n <= q_end
                    assert (qsrc & 15) + D * 2 <= qslot
            c_first, c_last = head0 // R, (head0 + S - 1) // R
            assert 0 <= c - c_first < c_last - c_first + 1 <= maxp
            covered += tb - ta
            r = head0 + tb
    assert covered == total
    # the merge claims: every cut head is a candidate exactly once
    cut = {h for h in range(BH) if (h * S) // R != (h * S + S - 1) // R}
    if R <= S:
        cands = [h for h in range(BH) if (h * S) // R != (h * S + S - 1) // R]
    else:
        cands = [(i + 1) * R // S for i in range(nchunks - 1) if ((i + 1) * R) % S]
        cands = [h for h in cands if (h * S) // R != (h * S + S - 1) // R]
    assert sorted(cands) == sorted(cut) and len(cands) == len(set(cands))


KINDS = [(64, 32, False), (64, 64, False), (128, 32, False), (128, 64, False), (128, 128, False),
         (64, 64, True), (128, 128, True)]
SHAPES = [(1, 1), (2, 7), (3, 63), (4, 65), (3, 129), (2, 1000), (2, 4097), (6, 300),
          (1, 20000), (16, 2048), (96, 1024), (512, 8192), (128, 131072), (1, 1 << 20), (7, 999)]


@pytest.mark.parametrize("D,bs,half", KINDS)
@pytest.mark.parametrize("occ", [1, 4])
def test_schedule_in_bounds(D, bs, half, occ):
    for BH, S in SHAPES:
        for offs in ((0, 0), (2, 14), (6, 2)):
            check(BH, S, D, bs, half, occ, offs)


@pytest.mark.parametrize("D,bs", [(128, 128), (128, 32), (64, 64)])
def test_schedule_in_bounds_with_cache_stride(D, bs):
    """Decode over the first S rows of caches holding S_stride rows per head."""
    for BH, S, S_stride in [(2, 1, 8), (6, 777, 1000), (6, 4097, 4100), (3, 20000, 32768),
                            (128, 16384, 16385)]:
        for offs in ((0, 0), (2, 14)):
            check(BH, S, D, bs, False, 4, offs, S_stride)


def test_stage_layout_fits_four_ctas_per_sm():
    """3-stage ring + merge scratch + barriers + tile descriptors + control
    block of the largest instantiation (INT8, D = 128, bs = 32) leave room
    for four CTAs in 228 KB."""
    RB, nsub, D = 128, 4, 128
    TILE = TILE_BYTES // RB
    stage = 2 * TILE_BYTES + 2 * (TILE * nsub * 2 + 32) + (D * 2 + 32)
    slices = WARPS * 32 // (D // 4)
    merge = -(-max(WARPS * (D + 2), slices * (D + 4)) * 4 // 16) * 16
    smem = STAGES * stage + merge + 2 * STAGES * 8 + STAGES * 32 + 32
    assert 4 * (smem + 1024) <= 228 * 1024, smem


@pytest.mark.parametrize("D,bs", [(128, 128), (128, 32), (64, 64), (64, 32)])
def test_schedule_in_bounds_with_fused_append(D, bs):
    """The fused-append variant: new rows [S - T, S) of each head."""
    for BH, S, S_stride, T in [(2, 1, 1, 1), (3, 65, 80, 3), (6, 129, 200, 7), (2, 64, 64, 64),
                               (6, 2000, 2048, 130), (3, 20000, 20001, 1), (128, 4096, 4096, 2)]:
        for offs in ((0, 0), (2, 14), (6, 2)):
            check(BH, S, D, bs, False, 4, offs, S_stride, T)


@pytest.mark.parametrize("D,bs", [(128, 128), (128, 32), (64, 64)])
def test_schedule_in_bounds_with_kv_groups(D, bs):
    """GQA/MQA: query head bh reads K/V head bh // group."""
    for BH, S, group in [(8, 1000, 4), (32, 20000, 4), (6, 257, 6), (16, 70000, 16), (4, 4097, 1)]:
        for offs in ((0, 0), (2, 14)):
            check(BH, S, D, bs, False, 4, offs, None, 0, group)


def _library_plan(BH, S, max_ctas):
    import ctypes
    from tqkv import _lib
    lib = _lib.load()
    out = [ctypes.c_longlong() for _ in range(4)]
    st = lib.tqkv_decode_plan(BH, S, max_ctas, *[ctypes.byref(o) for o in out])
    assert st == 0
    return tuple(o.value for o in out)


def test_model_plan_is_the_library_plan():
    """The plan modelled here is the one the library computes (host-only
    entry point tqkv_decode_plan, no GPU)."""
    shapes = [(BH, S) for BH, S in SHAPES] + [(512, 8192), (128, 131072), (128, 65536),
                                               (128, 16384), (16, 2048), (96, 1024), (1, 3)]
    for BH, S in shapes:
        for max_ctas in (1, 148, 296, 592, 1000):
            assert _library_plan(BH, S, max_ctas) == make_plan(BH, S, max_ctas), (BH, S, max_ctas)


def test_plan_entry_point_rejects_bad_arguments():
    import ctypes
    from tqkv import _lib
    lib = _lib.load()
    x = ctypes.c_longlong()
    r = [ctypes.byref(x)] * 4
    assert lib.tqkv_decode_plan(0, 8, 4, *r) == 2
    assert lib.tqkv_decode_plan(4, 0, 4, *r) == 2
    assert lib.tqkv_decode_plan(4, 8, 0, *r) == 2
    assert lib.tqkv_decode_plan(4, 8, 4, None, *r[1:]) == 6


def test_exchange_buffer_holds_every_entry():
    """Every offset the publish epilogue writes and the combine kernel reads
    (header words, and entry ((slot * world + rank) * BH + bh) * (D + 2) + j
    of 8 bytes) lies inside tqkv_exchange_bytes(world, BH, D)."""
    from tqkv import _lib
    lib = _lib.load()
    hdr = _const("decode_attn.cuh", "kExchangeHeaderBytes")
    epoch, done = _const("decode_attn.cuh", "kHdrEpoch"), _const("decode_attn.cuh", "kHdrDone")
    peers = _const("decode_attn.cuh", "kMaxPeers")
    assert 4 * max(epoch, done) + 4 <= hdr and hdr % 16 == 0
    for world in range(1, peers + 1):
        for BH in (1, 7, 128, 512, 4096):
            for D in (64, 128):
                nbytes = lib.tqkv_exchange_bytes(world, BH, D)
                last = hdr + (((1 * world + world - 1) * BH + BH - 1) * (D + 2) + D + 1) * 8
                assert last + 8 <= nbytes, (world, BH, D)
    assert lib.tqkv_exchange_bytes(peers + 1, 4, 128) == 0
    assert lib.tqkv_exchange_bytes(2, 4, 96) == 0


def test_workspace_counters_fit_before_the_records():
    """The four workspace counters (next chunk, cut heads claimed, exchange
    heads claimed, CTAs finished: ctr[0..3]) lie before the records of the
    pieces of cut heads, which start on 16 bytes."""
    src = open(os.path.join(CSRC, "decode_attn.cuh")).read()
    used = {int(i) for i in re.findall(r"a\.ctr\[(\d+)\]", src)}
    assert used == {0, 1, 2, 3}, used
    capi = open(os.path.join(CSRC, "tqkv_capi.cu")).read()
    recs = re.search(r"w\.parts_off = (\d+);", capi)
    assert recs and 4 * (max(used) + 1) <= int(recs.group(1)) and int(recs.group(1)) % 16 == 0
