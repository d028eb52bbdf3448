// decode_attn.cuh — split-S single-token decode attention for sm_100a.
//
// One kernel serves Kernel D (INT8 KV, fused online softmax; reference
// src/attention_int8_fused_online.cu:16-176), Kernel C (same function,
// reference src/attention_int8_fused.cu:18-143) and the FP16 baseline
// (reference src/attention_baseline.cu:11-129):
//
//   O[bh, :] = sum_t softmax_t(q . k_t / sqrt(D)) * v_t
//
// with k_t = code_t * scale_t(block) for INT8 KV (dequantised in registers,
// never written back).
//
// Work split ("flat split-S").  The B*H*S token rows, heads laid end to end,
// are cut into fixed chunks of C rows: about one chunk per CTA (C =
// ceil(B*H*S / grid)), so every CTA streams the same number of bytes whatever
// B, H and S are; or, when a CTA would stream very many rows, ~8 chunks per
// CTA.  Either way the CTAs claim chunks from a counter in the workspace.  A chunk covers the tail of one
// head, whole heads, and the head of another; each piece ("segment") yields an
// online-softmax state (m, l, acc[D]).  A head that lies inside one chunk is
// finished there.  A head cut across chunks has every piece store its state
// to the workspace as a record whose values carry a presence tag (no fence,
// no atomic).  A CTA whose producer has found no chunk left claims cut heads
// from a second counter and merges each head's records by log-sum-exp, in
// piece order, then writes O.  It waits only for pieces of chunks that other
// CTAs have already claimed (the pool is empty) and that those CTAs stream
// without waiting for anyone, so every wait ends, whatever CTAs are resident.
// The merge zeroes the records it read and the last CTA of the launch resets
// the counters, so the workspace stays zeroed between calls.
//
// CTA = 4 consumer warps + 1 producer warp.  One producer lane streams tiles
// of TILE tokens (K rows, V rows, their fp16 scales, and q at the start of a
// segment) from HBM into a ring of STAGES shared-memory buffers with 1-D bulk
// async copies (cp.async.bulk, mbarrier completion, L2 evict-first; no
// multicast), and describes each tile (head, offset, segment flags) in a
// per-stage descriptor.  Consumers never touch global memory on the hot loop.
//
// Variants: OUT selects the epilogue (O, partial records, records pushed to
// every GPU's exchange buffer, or pushed and then merged into O by the same
// launch); APPEND (fused append) has the consumers
// quantise the newest rows of each head into the cache and the tile; group > 1
// maps query head bh to K/V head bh / group (GQA/MQA).
//
// Consumer mapping.  A token row is split over LPR lanes, 16 bytes each
// (LPR = 8 for D = 128 INT8).  The LPR lanes of a "lane group" own 4 rows of
// every tile (rows g, g + G, g + 2G, g + 3G for G groups, so a warp's 16-byte
// shared loads cover consecutive rows without bank conflicts) and keep their
// own online-softmax state; the 16 (32) group states are merged once per
// segment, with shuffles inside a warp and shared memory across warps.
//
// INT8 dot products.  q is turned once per segment into a 16-bit fixed-point
// vector with a power-of-two scale (exact for every element within 2^4 of
// max|q|; absolute error <= max|q| * 2^-15 otherwise) split into a signed
// high byte and an unsigned low byte, so q . code is an exact integer built
// from 8 dp4a per lane per token — no int8 -> float conversion on the K side.
// The score is that integer times (scale_t * 2^-shift / sqrt(D) * log2 e).
// V codes are converted with the exponent trick
// (float bits 0x4B000000 | (byte ^ 0x80)) - (2^23 + 128), exact, one byte
// permute and one add per element, then accumulated with FMA in fp32.
// Softmax runs in base 2 with ex2.approx (the reference uses __expf).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

#include "device_common.cuh"
#include "kv_compress.cuh"

namespace tqkv {

constexpr int kDecodeConsumerWarps = 4;
constexpr int kDecodeConsumers = kDecodeConsumerWarps * 32;
constexpr int kDecodeThreads = kDecodeConsumers + 32;
constexpr int kDecodeTileBytes = 8192;  // bytes of K (and of V) per stage
constexpr int kDecodeStages = 3;        // 3 stages x ~17.7 KB: four CTAs fit on an SM

enum DecodeOut : int {
    kOutHalf = 0,     // write O (fp16)
    kOutPartial = 1,  // write per-head (acc[D], m, l) records, natural-log units
    kOutPeers = 2,    // write the records, tagged with the step number, into every
                      // rank's exchange buffer (split-S over NVLink)
    kOutExchange = 3, // kOutPeers, then merge every rank's records into O in the
                      // same launch (exchange_epilogue)
};

// Exchange buffer of one rank (split-S across the GPUs of a node), written by
// every rank through CUDA IPC peer mappings (no multicast).  Each value
// travels with its step number in one naturally aligned 64-bit store
// ({float bits, step}), so a reader knows a value has arrived when its step
// matches: no fences or flags sit between the producer and the consumer.
//   header (512 B): step   at +128   steps this rank has completed (combined)
//                   done   at +256   combine CTAs finished in the current step
//   records:        uint64 [2][world][BH][D + 2]   slot = step parity; entry
//                   (slot, r, bh) holds rank r's (acc[0..D-1], m, l) of head bh
constexpr int kMaxPeers = 8;
constexpr int kHdrEpoch = 32;     // in uint32 units
constexpr int kHdrDone = 64;
constexpr int kExchangeHeaderBytes = 512;

struct PeerArgs {
    unsigned long long* recs[kMaxPeers];  // records area of each rank's buffer
    unsigned int* own;                    // this rank's header
    unsigned long long* own_recs;         // this rank's records area
    int world;
    int rank;
};

__device__ __forceinline__ void st_volatile_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long pack_step(float v, unsigned int step) {
    return (static_cast<unsigned long long>(step) << 32) | __float_as_uint(v);
}
// Workspace records of cut heads' pieces: {float bits, 1}; zero = not stored.
__device__ __forceinline__ unsigned long long tag_present(float v) {
    return (1ull << 32) | __float_as_uint(v);
}
__device__ __forceinline__ bool is_present(unsigned long long w) {
    return static_cast<unsigned int>(w >> 32) == 1u;
}
__device__ __forceinline__ float tagged_value(unsigned long long w) {
    return __uint_as_float(static_cast<unsigned int>(w));
}
struct DecodeArgs {
    const void* q;             // fp16 [BH][D]
    const void* k;             // int8 or fp16 [BH][S][D]
    const void* v;
    const uint16_t* ks;        // fp16 [BH][S][D/BS] (INT8 only)
    const uint16_t* vs;
    void* out;                 // fp16 O [BH][D] or float [BH][D+2]
    unsigned long long* recs;  // workspace [BH][max_parts][D+2]: tagged records of the pieces
                               // of cut heads (acc[D], m in log2 units, l); zero between calls
    long long total_rows;      // BH * S
    long long chunk_rows;      // C: chunk u is rows [u * C, (u + 1) * C) of the BH * S rows
    unsigned int nchunks;      // ceil(total_rows / C)
    unsigned int* ctr;         // workspace counters: [0] next chunk to hand out, [1] cut heads
                               // claimed for merging, [2] heads claimed for the exchange merge,
                               // [3] CTAs finished; null when one CTA streams everything
    int S;                     // rows attended per head
    int S_stride;              // rows between consecutive heads in K/V/scales (>= S)
    int group;                 // query heads per K/V head (GQA/MQA; 1 = one K/V head each)
    int BH;
    int max_parts;
    float score_scale_log2;    // log2(e) / sqrt(D)
    PeerArgs peer;             // kOutPeers, kOutExchange
    const void* k_new;         // fused append only: fp16 [BH][T_new][D], rows [S - T_new, S)
    const void* v_new;
    int T_new;
    // the next launch in the stream may be dispatched from each CTA's start
    // (1) or from the end of its producer's last tile (0)
    int early_dependents;
};

template <int D, int BS, bool kHalfKV>
struct DecodeCfg {
    static constexpr int kElem = kHalfKV ? 2 : 1;
    static constexpr int kRowBytes = D * kElem;
    static constexpr int kLPR = kRowBytes / 16;                 // lanes per token row
    static constexpr int kGroups = kDecodeConsumers / kLPR;     // lane groups per CTA
    static constexpr int kTile = kDecodeTileBytes / kRowBytes;  // tokens per stage
    static constexpr int kTPG = kTile / kGroups;                // tokens per group per stage
    static constexpr int kEPL = 16 / kElem;                     // elements per lane
    static constexpr int kNSub = kHalfKV ? 1 : D / BS;          // scales per row
    static constexpr int kScaleBytes = kHalfKV ? 0 : kTile * kNSub * 2;
    static constexpr int kScaleSlot = kHalfKV ? 0 : kScaleBytes + 32;  // + alignment slack
    static constexpr int kQSlot = D * 2 + 32;
    // stage layout (all offsets multiples of 16)
    static constexpr int kOffK = 0;
    static constexpr int kOffV = kDecodeTileBytes;
    static constexpr int kOffKS = 2 * kDecodeTileBytes;
    static constexpr int kOffVS = kOffKS + kScaleSlot;
    static constexpr int kOffQ = kOffVS + kScaleSlot;
    static constexpr int kStageBytes = kOffQ + kQSlot;
    // merge scratch after the ring
    static constexpr int kOffMerge = kDecodeStages * kStageBytes;
    // Workspace record of a cut head's piece: D + 2 tagged 64-bit values
    // (acc[D], m, l); 16-byte aligned, so the merge reads value pairs.
    static constexpr int kRecWords = D + 2;
    // The merge of a cut head gives each thread 4 dims (kRecLanes threads per
    // record) and splits the records into kRecSlices slices.
    static constexpr int kRecLanes = D / 4;
    static constexpr int kRecSlices = kDecodeConsumers / kRecLanes;
    // merge area: the warps' states ([warp][D + 2] floats), or the slices'
    // states of a cut head's merge ([slice][D + 4]: rows start on 16 bytes)
    static constexpr int kSliceStride = D + 4;
    static constexpr int kMergeFloats =
        kDecodeConsumerWarps * (D + 2) > kRecSlices * kSliceStride
            ? kDecodeConsumerWarps * (D + 2)
            : kRecSlices * kSliceStride;
    static constexpr int kMergeBytes = (kMergeFloats * 4 + 15) / 16 * 16;
    static constexpr int kOffBars = kOffMerge + kMergeBytes;
    static constexpr int kOffMeta = kOffBars + 2 * kDecodeStages * 8;  // int[stages][8]
    static constexpr int kOffCtl = kOffMeta + kDecodeStages * 32;      // CtaCtl
    static constexpr int kSmemBytes = kOffCtl + 32;

    static_assert(kTPG == 4, "each lane group owns 4 rows per stage");
    static_assert(kStageBytes % 16 == 0, "stage must stay 16-byte aligned");
    static_assert(kOffMerge % 16 == 0 && kOffBars % 8 == 0, "alignment");
};

// Per-stage tile descriptor, written by the producer before the stage's
// mbarrier arrive and read by the consumers after their wait.
enum TileFlags : int { kTileFirst = 1, kTileLast = 2, kTileDone = 4 };
struct TileMeta {
    int bh, t0, cnt, flags, part, nparts;
    int n_old;  // rows [0, n_old) came from the cache; [n_old, cnt) are appended (fused append)
    int pad;
};

// CTA control block in shared memory: the slot through which thread 0 hands
// a claimed head to the other consumer threads, and an abort flag that a warp
// whose bounded wait ran out raises so that the others leave as well.
struct CtaCtl {
    int flag;
    unsigned int abort;
    unsigned int pad[6];
};
static_assert(sizeof(CtaCtl) == 32, "CtaCtl layout");

constexpr int kConsumerBarrier = 1;  // named barrier of the consumer warps (id 0: __syncthreads)

__device__ __forceinline__ unsigned int ld_volatile_shared(const unsigned int* p) {
    return *reinterpret_cast<const volatile unsigned int*>(p);
}

// Barrier of the consumer warps (bar.sync on kConsumerBarrier).  Returns
// false when the CTA is aborting; the caller then leaves through
// consumer_leave.
//
// Why it cannot hang: a consumer warp only ever leaves the kernel early
// through consumer_leave, which raises the abort flag and then arrives once
// at the consumer barrier.  The consumer warps pass the same sequence of
// barrier instances, so a leaving warp's arrival stands in for it at the
// instance the others are waiting at (or will reach next); that instance
// completes, and every warp sees the abort flag right after it and leaves.
__device__ __forceinline__ bool consumer_barrier(CtaCtl* c) {
    named_barrier_sync(kConsumerBarrier, kDecodeConsumers);
    return ld_volatile_shared(&c->abort) == 0u;
}

__device__ __forceinline__ void consumer_leave(CtaCtl* c) {
    if ((threadIdx.x & 31) == 0) atomicExch(&c->abort, 1u);
    __threadfence_block();
    __syncwarp();
    named_barrier_arrive(kConsumerBarrier, kDecodeConsumers);
}

// Bytes [src, src + n) (src even, n even) of the buffer [lo, hi) land in
// shared memory at dst + (src & 15).  The 16-byte-aligned part that lies
// inside the buffer goes by bulk copy (returned: its byte count, to be added
// to the stage's expected transaction count); the at most two ragged ends at
// the buffer's own edges are copied with plain 2-byte loads.  Never reads
// outside [lo, hi).
struct Span {
    uint64_t bulk_src;
    uint32_t bulk_dst_off;
    uint32_t bulk_bytes;
};

__device__ __forceinline__ Span plan_span(uint64_t src, uint32_t n, uint64_t lo, uint64_t hi) {
    const uint64_t a16 = src & ~uint64_t(15);
    const uint64_t b16 = (src + n + 15) & ~uint64_t(15);
    const uint64_t lo16 = (lo + 15) & ~uint64_t(15);
    const uint64_t hi16 = hi & ~uint64_t(15);
    const uint64_t blo = a16 > lo16 ? a16 : lo16;
    const uint64_t bhi = b16 < hi16 ? b16 : hi16;
    Span s;
    if (blo < bhi) {
        s.bulk_src = blo;
        s.bulk_dst_off = static_cast<uint32_t>(blo - a16);
        s.bulk_bytes = static_cast<uint32_t>(bhi - blo);
    } else {
        s.bulk_src = 0;
        s.bulk_dst_off = 0;
        s.bulk_bytes = 0;
    }
    return s;
}

// Plain-load the parts of [src, src + n) not covered by the bulk span.
__device__ __forceinline__ void copy_span_edges(uint8_t* dst, uint64_t src, uint32_t n,
                                                const Span& s) {
    const uint64_t a16 = src & ~uint64_t(15);
    const uint64_t end = src + n;
    const uint64_t cov_lo = s.bulk_bytes ? s.bulk_src : end;
    const uint64_t cov_hi = s.bulk_bytes ? s.bulk_src + s.bulk_bytes : end;
#pragma unroll 1
    for (uint64_t p = src; p < end; p += 2) {
        if (p >= cov_lo && p < cov_hi) {
            p = cov_hi - 2;  // skip the bulk-covered range
            continue;
        }
        const uint16_t v = __ldg(reinterpret_cast<const unsigned short*>(p));
        *reinterpret_cast<uint16_t*>(dst + (p - a16)) = v;
    }
}

__device__ __forceinline__ uint4 lds128(const uint8_t* p) {
    return *reinterpret_cast<const uint4*>(p);
}

// ---------------------------------------------------------------------------
// Fused append: the newest T rows of every head (rows [S - T, S)) are not yet
// in the cache.  The bulk copies of a tile cover only its older rows; the
// consumer warps quantise the new ones from fp16 (k_new / v_new [BH][T][D]),
// write codes and scales to the cache and into the tile's shared-memory
// slots, and meet at a barrier before consuming the tile.
constexpr int kNoAppend = -1;

// Tile rows n0, n0 + step, ... < n1 (relative to the tile start t0, memory
// row row0) are new tokens; one warp quantises each.  Lanes [0, D/8) take the
// K row, lanes [D/8, D/4) the V row, with the compress kernel's rounding
// (division form MODE).
template <int D, int BS, int MODE>
__device__ __forceinline__ void append_rows(const DecodeArgs& a, uint8_t* st, int bh, int t0,
                                            int n0, int n1, int step, long long row0, int ks_off,
                                            int vs_off) {
    using C = DecodeCfg<D, BS, false>;
    constexpr int kLPR = D / 8;  // lanes per row, 8 values each
    constexpr int kLPB = BS / 8;
    constexpr int kNSub = D / BS;
    const int lane = threadIdx.x & 31;
    const int tensor = lane / kLPR;  // 0: K, 1: V, 2..3: idle (D = 64)
    const int c = lane % kLPR;
    const bool active = tensor < 2;
    const uint4* src = static_cast<const uint4*>(tensor == 0 ? a.k_new : a.v_new);
    uint2* cache_q = static_cast<uint2*>(const_cast<void*>(tensor == 0 ? a.k : a.v));
    __half* cache_s = reinterpret_cast<__half*>(const_cast<uint16_t*>(tensor == 0 ? a.ks : a.vs));
    const int off_q = tensor == 0 ? C::kOffK : C::kOffV;
    const int off_s = tensor == 0 ? C::kOffKS + ks_off : C::kOffVS + vs_off;
    const int first_new = a.S - a.T_new;
    for (int t = n0; t < n1; t += step) {
        const long long j = static_cast<long long>(bh) * a.T_new + (t0 + t - first_new);
        const uint4 raw = active ? __ldg(src + j * kLPR + c) : make_uint4(0u, 0u, 0u, 0u);
        __half sc;
        const uint2 codes = quantize_lane<BS, MODE>(raw, sc);
        if (active) {
            const long long mrow = row0 + t;
            *reinterpret_cast<uint2*>(st + off_q + t * C::kRowBytes + c * 8) = codes;
            cache_q[mrow * kLPR + c] = codes;
            if (c % kLPB == 0) {
                *reinterpret_cast<__half*>(st + off_s + (t * kNSub + c / kLPB) * 2) = sc;
                cache_s[mrow * kNSub + c / kLPB] = sc;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Producer: one lane streams every tile of the chunks this CTA claims into
// the ring.
template <int D, int BS, bool kHalfKV, int APPEND>
__device__ __forceinline__ void decode_producer(const DecodeArgs& a, uint8_t* smem,
                                                uint64_t* full, uint64_t* empty,
                                                TileMeta* meta, CtaCtl* ctl) {
    using C = DecodeCfg<D, BS, kHalfKV>;
    constexpr bool kAppend = APPEND != kNoAppend;
    static_assert(!(kAppend && kHalfKV), "fused append is INT8 only");
    const uint64_t policy = make_evict_first_policy();
    const uint64_t q_lo = reinterpret_cast<uint64_t>(a.q);
    const uint64_t q_hi = q_lo + static_cast<uint64_t>(a.BH) * D * 2;
    const uint64_t ks_lo = reinterpret_cast<uint64_t>(a.ks);
    const uint64_t vs_lo = reinterpret_cast<uint64_t>(a.vs);
    const uint64_t sc_bytes =
        static_cast<uint64_t>(a.BH / a.group) * a.S_stride * C::kNSub * 2;
    const uint8_t* kbase = static_cast<const uint8_t*>(a.k);
    const uint8_t* vbase = static_cast<const uint8_t*>(a.v);
    const int first_new = kAppend ? a.S - a.T_new : a.S;  // rows >= first_new are appended

    int stage = 0;
    uint32_t phase = 0;
    long long issued = 0;
    bool ok = true;
    // Chunks are claimed from a counter, so SMs that stream faster take more
    // of them, and every chunk has been claimed by a running CTA before any
    // CTA starts waiting for merges (see merge_epilogue).  Chunk boundaries
    // are fixed, which keeps the pieces of a split head (and their indices)
    // deterministic.  A chunk may cover the end of one head and the start of
    // the next: one segment per head.  Without counters (one CTA, one chunk)
    // the CTA takes chunk 0.
    bool took_only_chunk = false;
    while (ok) {
        unsigned int chunk;
        if (a.ctr != nullptr) {
            chunk = atomicAdd(&a.ctr[0], 1u);
        } else {
            chunk = took_only_chunk ? a.nchunks : 0u;
            took_only_chunk = true;
        }
        if (chunk >= a.nchunks) break;
        const long long c0 = static_cast<long long>(chunk) * a.chunk_rows;
        const long long c1 = (c0 + a.chunk_rows) < a.total_rows ? c0 + a.chunk_rows : a.total_rows;
        for (long long r = c0; r < c1 && ok;) {
            const int bh = static_cast<int>(r / a.S);
            const long long head0 = static_cast<long long>(bh) * a.S;
            const int t_a = static_cast<int>(r - head0);
            const int t_b = static_cast<int>((c1 - head0) < a.S ? (c1 - head0) : a.S);
            // the chunks holding pieces of this head: u_first .. u_last
            const long long u_first = head0 / a.chunk_rows;
            const long long u_last = (head0 + a.S - 1) / a.chunk_rows;
            for (int t0 = t_a; t0 < t_b; t0 += C::kTile) {
                const int cnt = (t_b - t0) < C::kTile ? (t_b - t0) : C::kTile;
                if (ld_volatile_shared(&ctl->abort)) {
                    ok = false;
                    break;
                }
                if (!mbar_wait_bounded(&empty[stage], phase ^ 1u)) {
                    record_device_error(kErrEmptyWaitTimeout);
                    atomicExch(&ctl->abort, 1u);
                    ok = false;
                    break;
                }
                uint8_t* st = smem + stage * C::kStageBytes;
                // memory row: K/V head bh / group holds this query head's keys
                const long long row0 = static_cast<long long>(bh / a.group) * a.S_stride + t0;
                // rows [0, nb) of the tile come from the cache, [nb, cnt) are new
                int nb = first_new - t0;
                nb = nb < 0 ? 0 : (nb > cnt ? cnt : nb);
                const uint64_t ks_src = ks_lo + static_cast<uint64_t>(row0) * C::kNSub * 2;
                const uint64_t vs_src = vs_lo + static_cast<uint64_t>(row0) * C::kNSub * 2;
                {
                    const uint32_t kv_bytes = static_cast<uint32_t>(nb) * C::kRowBytes;
                    uint32_t tx = 2 * kv_bytes;

                    TileMeta& m = meta[stage];
                    m.bh = bh;
                    m.t0 = t0;
                    m.cnt = cnt;
                    m.flags = (t0 == t_a ? kTileFirst : 0) | (t0 + C::kTile >= t_b ? kTileLast : 0);
                    m.part = static_cast<int>(chunk - u_first);
                    m.nparts = static_cast<int>(u_last - u_first + 1);
                    m.n_old = nb;

                    Span sk{}, sv{}, sq{};
                    uint64_t q_src = 0;
                    if constexpr (!kHalfKV) {
                        const uint32_t sc_n = static_cast<uint32_t>(nb) * C::kNSub * 2;
                        // with appended rows the bulk span must stop short of their
                        // scales, which the consumers write into the same slot
                        const uint64_t k_hi = nb < cnt ? ks_src + sc_n : ks_lo + sc_bytes;
                        const uint64_t v_hi = nb < cnt ? vs_src + sc_n : vs_lo + sc_bytes;
                        sk = plan_span(ks_src, sc_n, ks_lo, k_hi);
                        sv = plan_span(vs_src, sc_n, vs_lo, v_hi);
                        tx += sk.bulk_bytes + sv.bulk_bytes;
                        copy_span_edges(st + C::kOffKS, ks_src, sc_n, sk);
                        copy_span_edges(st + C::kOffVS, vs_src, sc_n, sv);
                    }
                    const bool first = (t0 == t_a);
                    if (first) {
                        q_src = q_lo + static_cast<uint64_t>(bh) * D * 2;
                        sq = plan_span(q_src, D * 2, q_lo, q_hi);
                        tx += sq.bulk_bytes;
                        copy_span_edges(st + C::kOffQ, q_src, D * 2, sq);
                    }
                    mbar_arrive_expect_tx(&full[stage], tx);
                    if (kv_bytes) {
                        bulk_copy_g2s(st + C::kOffK, kbase + row0 * C::kRowBytes, kv_bytes,
                                      &full[stage], policy);
                        bulk_copy_g2s(st + C::kOffV, vbase + row0 * C::kRowBytes, kv_bytes,
                                      &full[stage], policy);
                    }
                    if constexpr (!kHalfKV) {
                        if (sk.bulk_bytes)
                            bulk_copy_g2s(st + C::kOffKS + sk.bulk_dst_off,
                                          reinterpret_cast<const void*>(sk.bulk_src), sk.bulk_bytes,
                                          &full[stage], policy);
                        if (sv.bulk_bytes)
                            bulk_copy_g2s(st + C::kOffVS + sv.bulk_dst_off,
                                          reinterpret_cast<const void*>(sv.bulk_src), sv.bulk_bytes,
                                          &full[stage], policy);
                    }
                    if (first && sq.bulk_bytes) {
                        bulk_copy_g2s(st + C::kOffQ + sq.bulk_dst_off,
                                      reinterpret_cast<const void*>(sq.bulk_src), sq.bulk_bytes,
                                      &full[stage], policy);
                    }
                    ++issued;
                }
                if (++stage == kDecodeStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            r = head0 + t_b;
        }
    }
    if (!a.early_dependents) griddep_launch_dependents();
    // end-of-work marker for the consumers
    if (ok) {
        if (mbar_wait_bounded(&empty[stage], phase ^ 1u)) {
            meta[stage].flags = kTileDone;
            mbar_arrive(&full[stage]);
            ++issued;
            if (++stage == kDecodeStages) {
                stage = 0;
                phase ^= 1u;
            }
        } else {
            record_device_error(kErrEmptyWaitTimeout);
            atomicExch(&ctl->abort, 1u);
        }
    }
    // Drain: do not leave the CTA while copies into its shared memory are in
    // flight.  In a normal run every stage was consumed long ago.
    const int outstanding = issued < kDecodeStages ? static_cast<int>(issued) : kDecodeStages;
    for (int i = 0; i < outstanding; ++i) {
        if (--stage < 0) {
            stage = kDecodeStages - 1;
            phase ^= 1u;
        }
        if (!mbar_wait_bounded(&full[stage], phase)) {
            record_device_error(kErrDrainTimeout);
            break;
        }
    }
}

// ---------------------------------------------------------------------------
// Consumer-side per-segment state and tile processing.

template <int D, int BS, bool kHalfKV>
struct SegState {
    using C = DecodeCfg<D, BS, kHalfKV>;
    float m2;             // reference max of base-2 scores (raised lazily, see kLazyRescale)
    float mx;             // true running max of base-2 scores
    float l;              // running sum of 2^(s - m2)
    float2 acc[C::kEPL / 2];  // running sum of 2^(s - m2) * v over this lane's dims (pairs)
    // INT8: q as fixed point, high and low bytes, 4 dims per word
    int qh[4];
    uint32_t ql[4];
    float cq;             // 2^-shift * log2(e) / sqrt(D)
    // FP16: q in fp32
    float qf[kHalfKV ? C::kEPL : 1];
};

template <int D, int BS, bool kHalfKV>
__device__ __forceinline__ void load_q(SegState<D, BS, kHalfKV>& st, const uint8_t* qsm,
                                       int r, float score_scale_log2) {
    using C = DecodeCfg<D, BS, kHalfKV>;
    const bool aligned = (reinterpret_cast<uintptr_t>(qsm) & 15) == 0;
    const uint16_t* qh16 = reinterpret_cast<const uint16_t*>(qsm) + r * C::kEPL;
    float qv[C::kEPL];
    if (aligned) {
        uint32_t w[C::kEPL / 2];
#pragma unroll
        for (int i = 0; i < C::kEPL / 8; ++i) {
            const uint4 v = *reinterpret_cast<const uint4*>(qh16 + 8 * i);
            w[4 * i + 0] = v.x;
            w[4 * i + 1] = v.y;
            w[4 * i + 2] = v.z;
            w[4 * i + 3] = v.w;
        }
#pragma unroll
        for (int i = 0; i < C::kEPL / 2; ++i) {
            const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
            qv[2 * i] = __low2float(h);
            qv[2 * i + 1] = __high2float(h);
        }
    } else {
#pragma unroll
        for (int i = 0; i < C::kEPL; ++i) qv[i] = half_bits_to_float(qh16[i]);
    }

    if constexpr (kHalfKV) {
#pragma unroll
        for (int i = 0; i < C::kEPL; ++i) st.qf[i] = qv[i];
        st.cq = score_scale_log2;
    } else {
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < C::kEPL; ++i) amax = fmaxf(amax, fabsf(qv[i]));
#pragma unroll
        for (int off = 1; off < C::kLPR; off <<= 1)
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        // shift so that max|q| * 2^shift lies in [2^14, 2^15): |Qi| <= 32752
        const int e = amax > 0.0f ? ((__float_as_int(amax) >> 23) & 0xff) - 127 : 0;
        const int shift = 14 - e;
        const float mul = __int_as_float((shift + 127) << 23);
        const float inv = __int_as_float((127 - shift) << 23);
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            uint32_t hi = 0, lo = 0;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int qi = __float2int_rn(qv[4 * w + b] * mul);
                hi |= (static_cast<uint32_t>(qi >> 8) & 0xffu) << (8 * b);
                lo |= (static_cast<uint32_t>(qi) & 0xffu) << (8 * b);
            }
            st.qh[w] = static_cast<int>(hi);
            st.ql[w] = lo;
        }
        st.cq = inv * score_scale_log2;
    }
    st.m2 = -INFINITY;
    st.mx = -INFINITY;
    st.l = 0.0f;
#pragma unroll
    for (int i = 0; i < C::kEPL / 2; ++i) st.acc[i] = make_float2(0.0f, 0.0f);
}


// Exact int8 -> fp32 of bytes b and b+1 of a word already XOR-ed with
// 0x80808080: the float with bits 0x4B0000uu is 2^23 + uu, uu = code + 128,
// so one packed subtraction of (2^23 + 128) leaves the two codes exactly.
template <int b>
__device__ __forceinline__ float2 biased_bytes_to_float2(uint32_t u) {
    const float2 f = make_float2(
        __int_as_float(static_cast<int>(__byte_perm(u, 0x4B000000u, 0x7440u + b))),
        __int_as_float(static_cast<int>(__byte_perm(u, 0x4B000000u, 0x7440u + b + 1))));
    return __fadd2_rn(f, make_float2(-8388736.0f, -8388736.0f));
}

// Shared-memory byte offset, inside a stage's scale slot, of the first scale
// of a tile whose first row is `row0`: the producer places global byte
// address A at slot + (A & 15).
__device__ __forceinline__ int scale_slot_offset(const uint16_t* base, long long row0, int nsub) {
    return static_cast<int>((reinterpret_cast<uint64_t>(base) + static_cast<uint64_t>(row0) * nsub * 2) & 15);
}

// Reduce-scatter of four per-lane partials (one per token of the lane group)
// over the LPR lanes of a group: afterwards lane r holds the full sum of
// token  ((r & LPR/2) ? 2 : 0) + ((r & LPR/4) ? 1 : 0).  Two halving stages
// move 2 + 1 values per lane, the remaining stages 1 value: 4 + log2(LPR/4)
// shuffles instead of 4 * log2(LPR) for four all-reduces.
template <int LPR, typename T>
__device__ __forceinline__ T reduce_scatter4(T v0, T v1, T v2, T v3, int r) {
    constexpr int h = LPR / 2, q = LPR / 4;
    const bool up = (r & h) != 0;
    T k0 = up ? v2 : v0, k1 = up ? v3 : v1;
    const T s0 = up ? v0 : v2, s1 = up ? v1 : v3;
    k0 += __shfl_xor_sync(0xffffffffu, s0, h);
    k1 += __shfl_xor_sync(0xffffffffu, s1, h);
    const bool odd = (r & q) != 0;
    T k = odd ? k1 : k0;
    k += __shfl_xor_sync(0xffffffffu, odd ? k0 : k1, q);
#pragma unroll
    for (int off = q / 2; off >= 1; off >>= 1) k += __shfl_xor_sync(0xffffffffu, k, off);
    return k;
}

// Token of the group (0..3) whose full sum lane r holds after reduce_scatter4,
// and the first lane holding token j.
template <int LPR>
__device__ __forceinline__ int scattered_token(int r) {
    return ((r & (LPR / 2)) ? 2 : 0) + ((r & (LPR / 4)) ? 1 : 0);
}
template <int LPR>
__device__ __forceinline__ int holder_lane(int j) {
    return (j >> 1) * (LPR / 2) + (j & 1) * (LPR / 4);
}

// The running max is only raised when a tile's max exceeds it by more than
// 2^kLazyRescale: until then 2^(s - m2) <= 2^kLazyRescale stays well inside
// fp32 and acc / l keep their scale, so the rescale of acc (EPL multiplies
// per lane) is skipped on almost every tile.
constexpr float kLazyRescale = 8.0f;

template <int D, int BS, bool kHalfKV>
__device__ __forceinline__ void consume_tile(SegState<D, BS, kHalfKV>& st, const uint8_t* stage,
                                             int cnt, int ks_off, int vs_off, int g, int r) {
    using C = DecodeCfg<D, BS, kHalfKV>;
    constexpr int kLPR = C::kLPR;
    const int lane = threadIdx.x & 31;
    const int gbase = lane - r;  // first lane of this group in the warp
    int rows[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) rows[j] = g + C::kGroups * j;
    const int tj = scattered_token<kLPR>(r);
    const int row_own = g + C::kGroups * tj;
    const bool valid_own = row_own < cnt;

    // ---- scores, base 2: lane r ends with the score of its own token tj ----
    float s;
    if constexpr (!kHalfKV) {
        const uint8_t* ksm = stage + C::kOffKS + ks_off;
        int dot[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint4 kw = lds128(stage + C::kOffK + rows[j] * C::kRowBytes + 16 * r);
            int h = dp4a_ss(static_cast<int>(kw.x), st.qh[0], 0);
            h = dp4a_ss(static_cast<int>(kw.y), st.qh[1], h);
            h = dp4a_ss(static_cast<int>(kw.z), st.qh[2], h);
            h = dp4a_ss(static_cast<int>(kw.w), st.qh[3], h);
            int t = dp4a_us(st.ql[0], static_cast<int>(kw.x), h << 8);
            t = dp4a_us(st.ql[1], static_cast<int>(kw.y), t);
            t = dp4a_us(st.ql[2], static_cast<int>(kw.z), t);
            t = dp4a_us(st.ql[3], static_cast<int>(kw.w), t);
            dot[j] = t;
        }
        if constexpr (C::kNSub == 1) {
            // one scale per row: reduce exact integers, scale once
            const int tot = reduce_scatter4<kLPR>(dot[0], dot[1], dot[2], dot[3], r);
            const float ks = half_bits_to_float(*reinterpret_cast<const uint16_t*>(ksm + 2 * row_own));
            s = static_cast<float>(tot) * (ks * st.cq);
        } else {
            // several blocks per row: scale each lane's block partial first
            const int blk = (16 * r) / BS;
            float f[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float ks = half_bits_to_float(*reinterpret_cast<const uint16_t*>(
                    ksm + 2 * (rows[j] * C::kNSub + blk)));
                f[j] = static_cast<float>(dot[j]) * ks;
            }
            s = reduce_scatter4<kLPR>(f[0], f[1], f[2], f[3], r) * st.cq;
        }
    } else {
        float d[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint4 kw = lds128(stage + C::kOffK + rows[j] * C::kRowBytes + 16 * r);
            const uint32_t w[4] = {kw.x, kw.y, kw.z, kw.w};
            float2 a = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int i = 0; i < 4; ++i)
                a = __ffma2_rn(make_float2(st.qf[2 * i], st.qf[2 * i + 1]),
                               __half22float2(*reinterpret_cast<const __half2*>(&w[i])), a);
            d[j] = a.x + a.y;
        }
        s = reduce_scatter4<kLPR>(d[0], d[1], d[2], d[3], r) * st.cq;
    }
    s = valid_own ? s : -INFINITY;

    // ---- online softmax over the group's 4 tokens (base 2, lazy rescale) ----
    float mt = fmaxf(s, __shfl_xor_sync(0xffffffffu, s, kLPR / 4));
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, kLPR / 2));
    st.mx = fmaxf(st.mx, mt);
    const bool raise = mt > st.m2 + kLazyRescale;  // false while mt == -inf
    if (__any_sync(0xffffffffu, raise)) {            // warp-uniform, rare
        const float m_new = raise ? mt : st.m2;
        const float alpha = raise ? fast_exp2(st.m2 - m_new) : 1.0f;  // 2^-inf = 0
        st.l *= alpha;
#pragma unroll
        for (int i = 0; i < C::kEPL / 2; ++i) st.acc[i] = __fmul2_rn(st.acc[i], make_float2(alpha, alpha));
        st.m2 = m_new;
    }
    const float base = st.m2 == -INFINITY ? 0.0f : st.m2;
    const float e = fast_exp2(s - base);  // 0 for masked rows
    float es = e + __shfl_xor_sync(0xffffffffu, e, kLPR / 4);
    es += __shfl_xor_sync(0xffffffffu, es, kLPR / 2);
    st.l += es;

    // ---- weighted V ----
    float w[4];
    if constexpr (!kHalfKV) {
        const uint8_t* vsm = stage + C::kOffVS + vs_off;
        if constexpr (C::kNSub == 1) {
            const float vsc = half_bits_to_float(*reinterpret_cast<const uint16_t*>(vsm + 2 * row_own));
            const float w_own = valid_own ? e * vsc : 0.0f;  // stale rows: weight exactly 0
#pragma unroll
            for (int j = 0; j < 4; ++j)
                w[j] = __shfl_sync(0xffffffffu, w_own, gbase + holder_lane<kLPR>(j));
        } else {
            const int blk = (16 * r) / BS;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float ej = __shfl_sync(0xffffffffu, e, gbase + holder_lane<kLPR>(j));
                const float vsc = half_bits_to_float(*reinterpret_cast<const uint16_t*>(
                    vsm + 2 * (rows[j] * C::kNSub + blk)));
                w[j] = rows[j] < cnt ? ej * vsc : 0.0f;
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint4 vw = lds128(stage + C::kOffV + rows[j] * C::kRowBytes + 16 * r);
            const uint32_t u[4] = {vw.x ^ 0x80808080u, vw.y ^ 0x80808080u, vw.z ^ 0x80808080u,
                                   vw.w ^ 0x80808080u};
            const float2 ww = make_float2(w[j], w[j]);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                st.acc[2 * i] = __ffma2_rn(ww, biased_bytes_to_float2<0>(u[i]), st.acc[2 * i]);
                st.acc[2 * i + 1] = __ffma2_rn(ww, biased_bytes_to_float2<2>(u[i]), st.acc[2 * i + 1]);
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = __shfl_sync(0xffffffffu, e, gbase + holder_lane<kLPR>(j));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (rows[j] < cnt) {  // stale fp16 rows may hold Inf/NaN: skip, do not weight by 0
                const uint4 vw = lds128(stage + C::kOffV + rows[j] * C::kRowBytes + 16 * r);
                const uint32_t w4[4] = {vw.x, vw.y, vw.z, vw.w};
                const float2 ww = make_float2(w[j], w[j]);
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    st.acc[i] = __ffma2_rn(ww, __half22float2(*reinterpret_cast<const __half2*>(&w4[i])),
                                           st.acc[i]);
            }
        }
    }
}

// Merge two base-2 online-softmax states: (m, l, acc) <- (m, l, acc) (+) (mo, lo, acco).
__device__ __forceinline__ void lse_factors(float m, float mo, float& M, float& fa, float& fb) {
    M = fmaxf(m, mo);
    const float base = M == -INFINITY ? 0.0f : M;
    fa = fast_exp2(m - base);
    fb = fast_exp2(mo - base);
}

// Pause between polls of records that have not arrived: from kPollNapMinNs,
// doubling up to kPollNapMaxNs.  Waiting CTAs then load little from L2 while
// the CTAs still streaming KV need it, and notice an arrival within ~0.5 us.
constexpr unsigned int kPollNapMinNs = 32;
constexpr unsigned int kPollNapMaxNs = 512;
__device__ __forceinline__ void poll_nap(unsigned int& ns) {
    __nanosleep(ns);
    ns = ns < kPollNapMaxNs ? 2 * ns : kPollNapMaxNs;
}

// Called by the 32 lanes of one warp: waits (bounded, napping between rounds)
// until the 64-bit values first[i * stride], i < n, all carry `tag` in their
// high word.  One value per record is watched, one lane per record, before
// the CTA loads whole records: far fewer L2 requests than every thread
// polling every value it needs.  Gives up silently after ~2^31 SM cycles (the
// per-value polls that follow time out and report).
__device__ __forceinline__ void lanes_wait_tagged(const unsigned long long* first, long long stride,
                                                  int n, unsigned int tag) {
    const int lane = threadIdx.x & 31;
    const long long start = clock64();
    unsigned int nap = kPollNapMinNs;
    for (int i0 = 0; i0 < n; i0 += 32) {
        const int i = i0 + lane;
        bool ok = i >= n || static_cast<unsigned int>(ld_volatile_u64(first + i * stride) >> 32) == tag;
        while (!__all_sync(0xffffffffu, ok)) {
            if (clock64() - start > (1ll << 31)) return;
            poll_nap(nap);
            if (!ok) ok = static_cast<unsigned int>(ld_volatile_u64(first + i * stride) >> 32) == tag;
        }
    }
}

// Merge the `world` records of head bh for `step` from this rank's exchange
// buffer into O[bh][t] (one thread per dim t < D), natural-log units.  Every
// load of the thread's 3 * world entries is issued at once (one round trip
// when the peers are done, the usual case); only entries still carrying an
// older step are polled again (poll_nap between rounds), for at most ~2^31 SM
// cycles (about a second).
// On timeout the device error flag gets kErrPeerWaitTimeout and O[bh][t] is
// NaN, so a lost peer shows in the output as well.
template <int D>
__device__ __forceinline__ void combine_head(const PeerArgs& p, int BH, int bh, int t,
                                             unsigned int step, __half* __restrict__ o) {
    const long long stride = static_cast<long long>(BH) * (D + 2);
    const unsigned long long* rec =
        p.own_recs + (static_cast<long long>(step & 1u) * p.world * BH + bh) * (D + 2);
    unsigned long long v[3 * kMaxPeers];
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r) {
        if (r < p.world) {
            v[3 * r] = ld_volatile_u64(rec + r * stride + D);
            v[3 * r + 1] = ld_volatile_u64(rec + r * stride + D + 1);
            v[3 * r + 2] = ld_volatile_u64(rec + r * stride + t);
        }
    }
    bool ready = true;
#pragma unroll
    for (int i = 0; i < 3 * kMaxPeers; ++i)
        if (i < 3 * p.world) ready = ready && static_cast<unsigned int>(v[i] >> 32) == step;
    if (!ready) {
        const long long start = clock64();
#pragma unroll 1
        unsigned int nap = kPollNapMinNs;
        for (uint32_t it = 0; it < (1u << 30) && !ready; ++it) {
            poll_nap(nap);
            ready = true;
#pragma unroll
            for (int r = 0; r < kMaxPeers; ++r) {
                if (r < p.world) {
                    const unsigned long long* base = rec + r * stride;
                    if (static_cast<unsigned int>(v[3 * r] >> 32) != step) v[3 * r] = ld_volatile_u64(base + D);
                    if (static_cast<unsigned int>(v[3 * r + 1] >> 32) != step) v[3 * r + 1] = ld_volatile_u64(base + D + 1);
                    if (static_cast<unsigned int>(v[3 * r + 2] >> 32) != step) v[3 * r + 2] = ld_volatile_u64(base + t);
                    ready = ready && static_cast<unsigned int>(v[3 * r] >> 32) == step &&
                            static_cast<unsigned int>(v[3 * r + 1] >> 32) == step &&
                            static_cast<unsigned int>(v[3 * r + 2] >> 32) == step;
                }
            }
            if (clock64() - start > (1ll << 31)) break;
        }
        if (!ready) {
            record_device_error(kErrPeerWaitTimeout);
            o[static_cast<long long>(bh) * D + t] = __ushort_as_half(static_cast<unsigned short>(0x7e00u));
            return;
        }
    }
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r)
        if (r < p.world) M = fmaxf(M, __uint_as_float(static_cast<unsigned int>(v[3 * r])));
    const float base = M == -INFINITY ? 0.0f : M;
    float A = 0.0f, L = 0.0f;
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r) {
        if (r < p.world) {
            const float f = __expf(__uint_as_float(static_cast<unsigned int>(v[3 * r])) - base);
            L = fmaf(__uint_as_float(static_cast<unsigned int>(v[3 * r + 1])), f, L);
            A = fmaf(__uint_as_float(static_cast<unsigned int>(v[3 * r + 2])), f, A);
        }
    }
    o[static_cast<long long>(bh) * D + t] = __float2half_rn(A * (1.0f / L));
}

// Write a finished head: O (fp16), a partial record, or the record in every
// rank's exchange buffer followed, for the step's last head, by the step flag.
// All consumer threads call it; A is this thread's dim (tid < D); M2 is in
// base-2 units.
template <int D, int OUT>
__device__ __forceinline__ void emit_head(const DecodeArgs& a, int bh, int tid, float A, float M2,
                                          float L) {
    constexpr float kLn2 = 0.69314718055994530942f;
    if constexpr (OUT == kOutHalf) {
        if (tid < D)
            static_cast<__half*>(a.out)[static_cast<long long>(bh) * D + tid] =
                __float2half_rn(A * (1.0f / L));
    } else if constexpr (OUT == kOutPartial) {
        if (tid < D) {
            float* rec = static_cast<float*>(a.out) + static_cast<long long>(bh) * (D + 2);
            rec[tid] = A;
            if (tid == 0) {
                rec[D] = M2 * kLn2;
                rec[D + 1] = L;
            }
        }
    } else {
        // every rank's buffer gets this head's record, each value stored
        // together with the step number (see the exchange buffer layout)
        const unsigned int step = __ldcg(a.peer.own + kHdrEpoch) + 1u;
        const long long off =
            ((static_cast<long long>(step & 1u) * a.peer.world + a.peer.rank) * a.BH + bh) *
            (D + 2);
        if (tid < D) {
            const unsigned long long va = pack_step(A, step);
            const unsigned long long vm = pack_step(M2 * kLn2, step);
            const unsigned long long vl = pack_step(L, step);
#pragma unroll
            for (int p = 0; p < kMaxPeers; ++p) {
                if (p < a.peer.world) {
                    unsigned long long* rec = a.peer.recs[p] + off;
                    st_volatile_u64(rec + tid, va);
                    if (tid == 0) {
                        st_volatile_u64(rec + D, vm);
                        st_volatile_u64(rec + D + 1, vl);
                    }
                }
            }
        }
    }
}

// Finish one segment: merge the lane-group states of the CTA, then either
// write O / the partial record (head held by one chunk), or store the piece's
// tagged record for the head's merge (merge_cut_head).
// Returns false when a consumer barrier gave up (the CTA then leaves).
template <int D, int BS, bool kHalfKV, int OUT>
__device__ __forceinline__ bool finish_segment(SegState<D, BS, kHalfKV>& st, const DecodeArgs& a,
                                               float* merge, CtaCtl* ctl, int bh, int part,
                                               int nparts, int tid) {
    using C = DecodeCfg<D, BS, kHalfKV>;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    // 0) move each group's reference max to its true max, so that records
    //    carry m = max_t s_t (the lazy rescale let m2 lag behind by < 2^8)
    {
        const float alpha = st.mx == -INFINITY ? 1.0f : fast_exp2(st.m2 - st.mx);
        st.l *= alpha;
#pragma unroll
        for (int i = 0; i < C::kEPL / 2; ++i) st.acc[i] = __fmul2_rn(st.acc[i], make_float2(alpha, alpha));
        st.m2 = st.mx;
    }
    // 1) lane groups inside a warp: lanes l, l + LPR, ... hold the same dims
#pragma unroll
    for (int off = C::kLPR; off < 32; off <<= 1) {
        const float mo = __shfl_xor_sync(0xffffffffu, st.m2, off);
        const float lo = __shfl_xor_sync(0xffffffffu, st.l, off);
        float M, fa, fb;
        lse_factors(st.m2, mo, M, fa, fb);
        st.l = st.l * fa + lo * fb;
#pragma unroll
        for (int i = 0; i < C::kEPL / 2; ++i) {
            float2 ao;
            ao.x = __shfl_xor_sync(0xffffffffu, st.acc[i].x, off);
            ao.y = __shfl_xor_sync(0xffffffffu, st.acc[i].y, off);
            st.acc[i] = __ffma2_rn(st.acc[i], make_float2(fa, fa),
                                   __fmul2_rn(ao, make_float2(fb, fb)));
        }
        st.m2 = M;
    }
    // 2) warps, through shared memory: merge[w][0..D-1] = acc, [D] = m2, [D+1] = l
    float* mw = merge + warp * (D + 2);
    if (lane < C::kLPR) {
#pragma unroll
        for (int i = 0; i < C::kEPL / 2; ++i) {
            mw[lane * C::kEPL + 2 * i] = st.acc[i].x;
            mw[lane * C::kEPL + 2 * i + 1] = st.acc[i].y;
        }
        if (lane == 0) {
            mw[D] = st.m2;
            mw[D + 1] = st.l;
        }
    }
    if (!consumer_barrier(ctl)) return false;

    float A = 0.0f, M = -INFINITY, L = 0.0f;
    if (tid < D) {
#pragma unroll
        for (int w = 0; w < kDecodeConsumerWarps; ++w) M = fmaxf(M, merge[w * (D + 2) + D]);
        const float base = M == -INFINITY ? 0.0f : M;
#pragma unroll
        for (int w = 0; w < kDecodeConsumerWarps; ++w) {
            const float f = fast_exp2(merge[w * (D + 2) + D] - base);
            L = fmaf(merge[w * (D + 2) + D + 1], f, L);
            A = fmaf(merge[w * (D + 2) + tid], f, A);
        }
    }

    if (nparts == 1) {
        emit_head<D, OUT>(a, bh, tid, A, M, L);
        return consumer_barrier(ctl);  // merge[] is reused by the next segment
    }

    // A piece of a head cut across chunks: store its record, every value
    // tagged as present, and go on streaming; the head is merged by a CTA
    // that has finished streaming (merge_epilogue).
    unsigned long long* rec =
        a.recs + (static_cast<long long>(bh) * a.max_parts + part) * C::kRecWords;
    if (tid < D) st_relaxed_u64(rec + tid, tag_present(A));
    if (tid == 0) {
        st_relaxed_u64(rec + D, tag_present(M));
        st_relaxed_u64(rec + D + 1, tag_present(L));
    }
    // merge[] is reused by the next segment
    return consumer_barrier(ctl);
}

// Merge the `nparts` records of cut head bh (log-sum-exp, in part order, so
// the result does not depend on which CTA streamed which piece) and emit the
// head.  Warp 0 first waits until every record's m value is stored; then
// threads take 4 dims each (kRecLanes per record) and one slice of the
// records (parts sl, sl + kRecSlices, ...), loading 4 parts at a time and
// polling, bounded (~2^31 SM cycles), only values whose tag is not yet set;
// the slices' states are then merged through shared memory.  The records are
// zeroed afterwards.  On timeout: kErrPieceWaitTimeout, the head is emitted
// from the pieces that did arrive.  Returns false when a consumer barrier
// gave up.
template <int D, int BS, bool kHalfKV, int OUT>
__device__ __forceinline__ bool merge_cut_head(const DecodeArgs& a, float* merge, CtaCtl* ctl, int bh,
                                            int nparts, int tid) {
    using C = DecodeCfg<D, BS, kHalfKV>;
    constexpr int kBatch = 4;
    const int dq = tid % C::kRecLanes;   // dims 4*dq .. 4*dq + 3
    const int sl = tid / C::kRecLanes;   // records sl, sl + kRecSlices, ...
    const unsigned long long* recs =
        a.recs + static_cast<long long>(bh) * a.max_parts * C::kRecWords;
    // warp 0 watches each record's m value until every piece has stored it
    if (tid < 32) lanes_wait_tagged(recs + D, C::kRecWords, nparts, 1u);
    if (!consumer_barrier(ctl)) return false;
    float M = -INFINITY, L = 0.0f;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const long long start = clock64();
    bool late = false;
#pragma unroll 1
    for (int p0 = sl; p0 < nparts; p0 += kBatch * C::kRecSlices) {
        ulonglong2 ml[kBatch], a01[kBatch], a23[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const int p = p0 + j * C::kRecSlices;
            if (p < nparts) {
                const unsigned long long* r = recs + p * C::kRecWords;
                ml[j] = ld_relaxed_u64x2(r + D);
                a01[j] = ld_relaxed_u64x2(r + 4 * dq);
                a23[j] = ld_relaxed_u64x2(r + 4 * dq + 2);
            }
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const int p = p0 + j * C::kRecSlices;
            if (p >= nparts) continue;
            const unsigned long long* r = recs + p * C::kRecWords;
            // poll only what has not arrived yet
#pragma unroll 1
            unsigned int nap = kPollNapMinNs;
            while (!(is_present(ml[j].x) && is_present(ml[j].y) && is_present(a01[j].x) &&
                     is_present(a01[j].y) && is_present(a23[j].x) && is_present(a23[j].y))) {
                if (late || clock64() - start > (1ll << 31)) {
                    late = true;
                    break;
                }
                poll_nap(nap);
                if (!(is_present(ml[j].x) && is_present(ml[j].y))) ml[j] = ld_relaxed_u64x2(r + D);
                if (!(is_present(a01[j].x) && is_present(a01[j].y))) a01[j] = ld_relaxed_u64x2(r + 4 * dq);
                if (!(is_present(a23[j].x) && is_present(a23[j].y)))
                    a23[j] = ld_relaxed_u64x2(r + 4 * dq + 2);
            }
            if (late && !(is_present(ml[j].x) && is_present(ml[j].y))) continue;
            const float m = tagged_value(ml[j].x), l = tagged_value(ml[j].y);
            if (m > M) {
                const float s = fast_exp2(M - m);  // 2^-inf = 0 for the first piece
                L *= s;
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[i] *= s;
                M = m;
            }
            const float f = fast_exp2(m - M);
            L = fmaf(l, f, L);
            acc[0] = fmaf(tagged_value(a01[j].x), f, acc[0]);
            acc[1] = fmaf(tagged_value(a01[j].y), f, acc[1]);
            acc[2] = fmaf(tagged_value(a23[j].x), f, acc[2]);
            acc[3] = fmaf(tagged_value(a23[j].y), f, acc[3]);
        }
    }
    if (late) record_device_error(kErrPieceWaitTimeout);
    // the slices' states: merge[sl][0..D-1] = acc, [D] = M, [D+1] = L
    float* ms = merge + sl * C::kSliceStride;
    *reinterpret_cast<float4*>(ms + 4 * dq) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    if (dq == 0) {
        ms[D] = M;
        ms[D + 1] = L;
    }
    if (!consumer_barrier(ctl)) return false;
    float At = 0.0f, Mt = -INFINITY, Lt = 0.0f;
    if (tid < D) {
#pragma unroll
        for (int k = 0; k < C::kRecSlices; ++k) Mt = fmaxf(Mt, merge[k * C::kSliceStride + D]);
        const float base = Mt == -INFINITY ? 0.0f : Mt;
#pragma unroll
        for (int k = 0; k < C::kRecSlices; ++k) {
            const float f = fast_exp2(merge[k * C::kSliceStride + D] - base);
            Lt = fmaf(merge[k * C::kSliceStride + D + 1], f, Lt);
            At = fmaf(merge[k * C::kSliceStride + tid], f, At);
        }
    }
    emit_head<D, OUT>(a, bh, tid, At, Mt, Lt);
    // leave the workspace all-zero for the next call, whatever its shape
    unsigned long long* z =
        a.recs + static_cast<long long>(bh) * a.max_parts * C::kRecWords;
    for (int i = tid; i < nparts * C::kRecWords; i += kDecodeConsumers) z[i] = 0ull;
    return consumer_barrier(ctl);  // merge[] is reused by the next merge
}

// After its last chunk a CTA claims cut heads from ctr[1] and merges them
// (merge_cut_head).  Its producer has found the chunk pool empty, so every
// chunk is held by a CTA that streams it and stores its records without
// waiting for anyone: the waits end whichever CTAs are resident, and no
// cooperative launch is needed.  Candidates are the heads when a chunk is no
// longer than a head (uncut heads are skipped), else the interior chunk
// boundaries, each of which cuts at most one head.  Returns false when a
// consumer barrier gave up.
template <int D, int BS, bool kHalfKV, int OUT>
__device__ __forceinline__ bool merge_epilogue(const DecodeArgs& a, float* merge, CtaCtl* ctl,
                                               int tid) {
    const long long C = a.chunk_rows;
    const bool by_head = C <= a.S;
    const long long ncand = by_head ? static_cast<long long>(a.BH)
                                    : static_cast<long long>(a.nchunks) - 1;
    for (;;) {
        if (tid == 0) ctl->flag = static_cast<int>(atomicAdd(&a.ctr[1], 1u));
        if (!consumer_barrier(ctl)) return false;
        const long long i = static_cast<unsigned int>(*reinterpret_cast<volatile int*>(&ctl->flag));
        // every thread has read the claim before thread 0 writes the next one
        if (!consumer_barrier(ctl)) return false;
        if (i >= ncand) break;
        long long head0;
        if (by_head) {
            head0 = i * a.S;
        } else {
            const long long row = (i + 1) * C;
            if (row % a.S == 0) continue;  // the boundary falls between heads
            head0 = row / a.S * a.S;
        }
        const long long u_first = head0 / C;
        const long long u_last = (head0 + a.S - 1) / C;
        if (u_first == u_last) continue;   // a whole head, finished where it was streamed
        if (!merge_cut_head<D, BS, kHalfKV, OUT>(a, merge, ctl, static_cast<int>(head0 / a.S),
                                                 static_cast<int>(u_last - u_first + 1), tid))
            return false;
    }
    return true;
}

// kOutExchange, after the merges: the CTA claims heads from ctr[2] and merges
// every rank's records of each into O (combine_head), warp 0 first watching
// each rank's m entry.  A head's entries come from every rank, this one
// included, i.e. from CTAs of this launch that are past their own streaming
// (merges of cut heads wait only as described at merge_epilogue), so all
// waits end.  Across ranks nothing is circular: each rank emits all of its
// records of the step before any of its CTAs waits for a peer.  `step` is the
// step being completed.  Returns false when a consumer barrier gave up.
template <int D>
__device__ __forceinline__ bool exchange_epilogue(const DecodeArgs& a, CtaCtl* ctl, int tid,
                                                  unsigned int& step) {
    step = __ldcg(a.peer.own + kHdrEpoch) + 1u;
    __half* o = static_cast<__half*>(a.out);
    const long long stride = static_cast<long long>(a.BH) * (D + 2);
    for (;;) {
        if (tid == 0) ctl->flag = static_cast<int>(atomicAdd(&a.ctr[2], 1u));
        if (!consumer_barrier(ctl)) return false;
        const int h = *reinterpret_cast<volatile int*>(&ctl->flag);
        if (!consumer_barrier(ctl)) return false;
        if (h < 0 || h >= a.BH) break;
        if (tid < 32) {
            const unsigned long long* m0 = a.peer.own_recs +
                (static_cast<long long>(step & 1u) * a.peer.world * a.BH + h) * (D + 2) + D;
            lanes_wait_tagged(m0, stride, a.peer.world, step);
        }
        if (!consumer_barrier(ctl)) return false;
        if (tid < D) combine_head<D>(a.peer, a.BH, h, tid, step, o);
    }
    return true;
}

// Before its dependency wait, a CTA asks L2 for the K and V rows of the
// first kDecodeStages tiles of chunk blockIdx.x: the first claims hand out
// chunks 0 .. grid - 1 in about that order, so whichever CTA streams the
// chunk finds them there.  Only a hint: it reads inputs and writes nothing,
// and L2 serves later writes of those rows by the previous launch (a fused
// append) like any other.
template <int D, int BS, bool kHalfKV>
__device__ __forceinline__ void prefetch_first_tiles(const DecodeArgs& a) {
    using C = DecodeCfg<D, BS, kHalfKV>;
    if (a.S <= 0 || blockIdx.x >= a.nchunks) return;
    const long long c0 = static_cast<long long>(blockIdx.x) * a.chunk_rows;
    if (c0 >= a.total_rows) return;
    const long long bh = c0 / a.S;
    const long long t0 = c0 - bh * a.S;
    long long rows = static_cast<long long>(kDecodeStages) * C::kTile;
    if (rows > a.S - t0) rows = a.S - t0;
    if (c0 + rows > a.total_rows) rows = a.total_rows - c0;
    const long long row0 = (bh / a.group) * a.S_stride + t0;
    const uint32_t bytes = static_cast<uint32_t>(rows) * C::kRowBytes;
    bulk_prefetch_l2(static_cast<const uint8_t*>(a.k) + row0 * C::kRowBytes, bytes);
    bulk_prefetch_l2(static_cast<const uint8_t*>(a.v) + row0 * C::kRowBytes, bytes);
}

// ---------------------------------------------------------------------------
constexpr int kDecodeCtasPerSm = 4;  // target residency (smem: 3 stages; regs: <= 102 per thread)

template <int D, int BS, bool kHalfKV, int OUT, int APPEND = kNoAppend>
__global__ void __launch_bounds__(kDecodeThreads, kDecodeCtasPerSm)
    decode_attn_kernel(const DecodeArgs a) {
    using C = DecodeCfg<D, BS, kHalfKV>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kOffBars);
    uint64_t* empty = full + kDecodeStages;
    TileMeta* meta = reinterpret_cast<TileMeta*>(smem + C::kOffMeta);
    CtaCtl* ctl = reinterpret_cast<CtaCtl*>(smem + C::kOffCtl);
    float* merge = reinterpret_cast<float*>(smem + C::kOffMerge);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kDecodeStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kDecodeConsumerWarps);
        }
        ctl->flag = 0;
        ctl->abort = 0u;
        fence_barrier_init();
    }
    // Launched as a programmatic dependent (decode launches are), this CTA
    // may start while the previous launch in the stream is finishing: it
    // lets the next launch be dispatched (here, or after its producer's last
    // tile: early_dependents), asks L2 for the first rows it is likely to
    // stream, and touches no other global memory until the previous launch
    // has completed.
    if (a.early_dependents) griddep_launch_dependents();
    if (threadIdx.x == kDecodeConsumers) prefetch_first_tiles<D, BS, kHalfKV>(a);
    griddep_wait();
    __syncthreads();

    const int warp = threadIdx.x >> 5;
    if (warp == kDecodeConsumerWarps) {
        if ((threadIdx.x & 31) == 0)
            decode_producer<D, BS, kHalfKV, APPEND>(a, smem, full, empty, meta, ctl);
        return;
    }

    const int tid = threadIdx.x;
    const int g = tid / C::kLPR;
    const int r = tid % C::kLPR;
    const int lane = tid & 31;
    int stage = 0;
    uint32_t phase = 0;
    SegState<D, BS, kHalfKV> st;

    for (;;) {
        const bool ok = mbar_wait_bounded(&full[stage], phase);
        // warp-uniform decision: every lane leaves, or none does
        if (__any_sync(0xffffffffu, !ok || ld_volatile_shared(&ctl->abort) != 0u)) {
            if (lane == 0 && !ok) record_device_error(kErrFullWaitTimeout);
            consumer_leave(ctl);
            return;
        }
        const TileMeta m = meta[stage];
        if (m.flags & kTileDone) {
            if (a.ctr == nullptr) return;  // one CTA streamed everything: nothing was cut
            if (a.nchunks > 1 && !merge_epilogue<D, BS, kHalfKV, OUT>(a, merge, ctl, tid)) {
                consumer_leave(ctl);
                return;
            }
            unsigned int step = 0;
            if constexpr (OUT == kOutExchange) {
                if (!exchange_epilogue<D>(a, ctl, tid, step)) {
                    consumer_leave(ctl);
                    return;
                }
            }
            // the last CTA to get here hands the counters back zeroed (every
            // CTA has made its last claim) and, exchanging, completes the step
            if (tid == 0) {
                __threadfence();
                if (atomicAdd(&a.ctr[3], 1u) == gridDim.x - 1) {
                    atomicExch(&a.ctr[0], 0u);
                    atomicExch(&a.ctr[1], 0u);
                    atomicExch(&a.ctr[2], 0u);
                    atomicExch(&a.ctr[3], 0u);
                    if constexpr (OUT == kOutExchange) a.peer.own[kHdrEpoch] = step;
                }
            }
            return;
        }
        const uint8_t* sp = smem + stage * C::kStageBytes;
        if (m.flags & kTileFirst) {
            const int q_off = static_cast<int>(
                (reinterpret_cast<uint64_t>(a.q) + static_cast<uint64_t>(m.bh) * D * 2) & 15);
            load_q<D, BS, kHalfKV>(st, sp + C::kOffQ + q_off, r, a.score_scale_log2);
        }
        int ks_off = 0, vs_off = 0;
        if constexpr (!kHalfKV) {
            const long long mrow0 = static_cast<long long>(m.bh / a.group) * a.S_stride + m.t0;
            ks_off = scale_slot_offset(a.ks, mrow0, C::kNSub);
            vs_off = scale_slot_offset(a.vs, mrow0, C::kNSub);
            if constexpr (APPEND != kNoAppend) {
                if (m.n_old < m.cnt) {  // CTA-uniform: new rows in this tile
                    append_rows<D, BS, APPEND>(a, const_cast<uint8_t*>(sp), m.bh, m.t0,
                                               m.n_old + warp, m.cnt, kDecodeConsumerWarps,
                                               mrow0, ks_off, vs_off);
                    if (!consumer_barrier(ctl)) {
                        consumer_leave(ctl);
                        return;
                    }
                }
            }
        }
        consume_tile<D, BS, kHalfKV>(st, sp, m.cnt, ks_off, vs_off, g, r);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (++stage == kDecodeStages) {
            stage = 0;
            phase ^= 1u;
        }
        if (m.flags & kTileLast) {
            if (!finish_segment<D, BS, kHalfKV, OUT>(st, a, merge, ctl, m.bh, m.part, m.nparts,
                                                     tid)) {
                consumer_leave(ctl);
                return;
            }
        }
    }
}

// Log-sum-exp merge of R partial records per head (natural-log units):
// partials [R][BH][D + 2] -> O fp16 [BH][D].  One warp-group per head.
template <int D>
__global__ void __launch_bounds__(D)
    lse_combine_kernel(const float* __restrict__ partials, __half* __restrict__ o, int R, int BH) {
    const int bh = blockIdx.x;
    const int t = threadIdx.x;
    const long long stride = static_cast<long long>(BH) * (D + 2);
    const float* rec = partials + static_cast<long long>(bh) * (D + 2);
    float M = -INFINITY;
    for (int r = 0; r < R; ++r) M = fmaxf(M, rec[r * stride + D]);
    const float base = M == -INFINITY ? 0.0f : M;
    float A = 0.0f, L = 0.0f;
    for (int r = 0; r < R; ++r) {
        const float f = __expf(rec[r * stride + D] - base);
        L = fmaf(rec[r * stride + D + 1], f, L);
        A = fmaf(rec[r * stride + t], f, A);
    }
    o[static_cast<long long>(bh) * D + t] = __float2half_rn(A * (1.0f / L));
}

// Split-S step over NVLink, second half (two-launch form): wait (bounded)
// until every rank has published the current step into this rank's exchange
// buffer, then merge the world records of each head into O.  One CTA per
// head; the last CTA advances this rank's step counter.
template <int D>
__global__ void __launch_bounds__(D)
    exchange_combine_kernel(const PeerArgs p, __half* __restrict__ o, int BH) {
    const int bh = blockIdx.x;
    const int t = threadIdx.x;
    const unsigned int step = __ldcg(p.own + kHdrEpoch) + 1u;
    if (t < 32) {
        const unsigned long long* m0 =
            p.own_recs + (static_cast<long long>(step & 1u) * p.world * BH + bh) * (D + 2) + D;
        lanes_wait_tagged(m0, static_cast<long long>(BH) * (D + 2), p.world, step);
    }
    __syncthreads();
    combine_head<D>(p, BH, bh, t, step, o);
    // the last CTA of the step advances this rank's step counter; every CTA
    // has read it above, before adding itself to the count
    __syncthreads();
    if (t == 0) {
        __threadfence();
        const unsigned int prev = atomicAdd(p.own + kHdrDone, 1u);
        if (prev == static_cast<unsigned int>(BH - 1)) {
            p.own[kHdrDone] = 0u;
            p.own[kHdrEpoch] = step;
        }
    }
}

// Empty records (acc = 0, m = -inf, l = 0) of the current step into every
// rank's exchange buffer, for a rank whose token slice is empty (S == 0).
// One CTA per head, one thread per dim.
template <int D>
__global__ void __launch_bounds__(D) publish_empty_kernel(const PeerArgs p, int BH) {
    const int bh = blockIdx.x;
    const int t = threadIdx.x;
    const unsigned int step = __ldcg(p.own + kHdrEpoch) + 1u;
    const long long off =
        ((static_cast<long long>(step & 1u) * p.world + p.rank) * BH + bh) * (D + 2);
    for (int r = 0; r < kMaxPeers; ++r) {
        if (r < p.world) {
            unsigned long long* rec = p.recs[r] + off;
            st_volatile_u64(rec + t, pack_step(0.0f, step));
            if (t == 0) {
                st_volatile_u64(rec + D, pack_step(-INFINITY, step));
                st_volatile_u64(rec + D + 1, pack_step(0.0f, step));
            }
        }
    }
}

// Fill `n` fp16 values with `bits` (used for S == 0 outputs).
__global__ void fill_half_kernel(uint16_t* __restrict__ p, long long n, uint16_t bits) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        p[i] = bits;
}

// Empty partial records (m = -inf, l = 0, acc = 0) for a device with S == 0.
__global__ void fill_empty_partials_kernel(float* __restrict__ p, long long heads, int D) {
    const long long n = heads * (D + 2);
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % (D + 2));
        p[i] = c == D ? -INFINITY : 0.0f;
    }
}

}  // namespace tqkv
