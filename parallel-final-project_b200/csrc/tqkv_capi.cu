// tqkv_capi.cu — kernel instantiations, launch planning, the per-stream
// workspace cache and the extern "C" ABI declared in include/tqkv.h.
//
// Everything device-side lives in this one translation unit (no relocatable
// device code), so the device error flag of device_common.cuh is this TU's.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>

#include "decode_attn.cuh"
#include "device_common.cuh"
#include "kv_compress.cuh"
#include "tqkv.h"
#include "tqkv_internal.h"
#include "ws_cache.h"

#ifndef TQKV_COMPRESS_DIV_MODE
// Division form used by Kernel A.  The reference is built with
// --use_fast_math (CMakeLists.txt:21), under which its '/' is an approximate
// division; div.approx.ftz.f32 reproduces its codes and scales bit for bit
// (measured on the B200 against the reference build: 0 differences over
// 2.9e9 elements of the five configurations and 3.7e7 tie-rich elements,
// while IEEE division differs on ~15% of the tie-class elements).
#define TQKV_COMPRESS_DIV_MODE tqkv::kDivApproxFtz
#endif

namespace tqkv {

namespace {

thread_local int t_last_cuda_error = 0;

constexpr long long kMinRowsPerCta = 256;  // below this a CTA is mostly pipeline fill
constexpr long long kChunksPerCta = 8;     // scheduling chunks per CTA (load balance)
constexpr long long kChunkAlign = 128;     // chunk rows: a multiple of every tile height
// Below this many rows per CTA the rows are cut into one chunk per CTA:
// every chunk boundary inside a head costs a head piece (a record, consumer
// barriers, a share of the head's merge), which short chunks cannot
// amortise.  Measured on one B200 with 592 CTAs: ~8 chunks per CTA win 1.4 %
// at 28k rows per CTA (long-context decode), and lose 14 % at 7k rows per
// CTA (B16 H32 S8192).
constexpr long long kMinDynamicRowsPerCta = 16384;
constexpr int kMaxCtasPerSmBound = 4;      // >= any decode kernel's occupancy (smem-bound)

struct KernelKey {
    const void* fn;
    int device;
    bool operator<(const KernelKey& o) const {
        return fn < o.fn || (fn == o.fn && device < o.device);
    }
};

std::mutex g_kernel_mu;
std::map<KernelKey, int> g_occupancy;  // resident CTAs per SM, after smem opt-in
std::map<int, int> g_sm_count;

int sm_count(int device) {
    std::lock_guard<std::mutex> lock(g_kernel_mu);
    auto it = g_sm_count.find(device);
    if (it != g_sm_count.end()) return it->second;
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) n = 0;
    g_sm_count[device] = n;
    return n;
}

// Opts the kernel into its dynamic shared memory once per device and returns
// how many of its CTAs fit on one SM (0 on failure).
template <typename Fn>
int prepare_kernel(Fn fn, int threads, int smem_bytes, int device) {
    const KernelKey key{reinterpret_cast<const void*>(fn), device};
    std::lock_guard<std::mutex> lock(g_kernel_mu);
    auto it = g_occupancy.find(key);
    if (it != g_occupancy.end()) return it->second;
    if (smem_bytes > 48 * 1024) {
        if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) !=
            cudaSuccess)
            return 0;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem_bytes) !=
        cudaSuccess)
        per_sm = 0;
    g_occupancy[key] = per_sm;
    return per_sm;
}

struct DecodePlan {
    int grid;
    long long chunk_rows;
    long long nchunks;
    int max_parts;
};

// The B*H*S rows, heads laid end to end, are cut into fixed chunks of C rows,
// which the CTAs claim from a counter.  Normally there is one chunk per CTA
// (C = rows / grid, rounded to 16): equal work for every CTA and the fewest
// head pieces.  When a CTA would stream at least kMinDynamicRowsPerCta rows,
// C is cut to about 1/kChunksPerCta of that (a multiple of 128), so SMs that
// stream faster take more chunks; each chunk is then long enough (>= 32
// tiles) to amortise the extra head pieces it creates.  `max_ctas` caps the
// grid (resident CTAs).
DecodePlan make_plan(long long BH, int S, long long max_ctas) {
    DecodePlan p{};
    const long long total_rows = BH * S;
    long long g = (total_rows + kMinRowsPerCta - 1) / kMinRowsPerCta;
    if (g > max_ctas) g = max_ctas;
    if (g < 1) g = 1;
    long long c = (total_rows + g - 1) / g;
    if (c >= kMinDynamicRowsPerCta) {
        c = (total_rows + g * kChunksPerCta - 1) / (g * kChunksPerCta);
        c = (c + kChunkAlign - 1) / kChunkAlign * kChunkAlign;
    } else if (g > 1) {
        c = (c + 15) / 16 * 16;
    }
    p.chunk_rows = c;
    p.nchunks = (total_rows + c - 1) / c;
    p.grid = static_cast<int>(p.nchunks < g ? p.nchunks : g);
    p.max_parts = static_cast<int>((static_cast<long long>(S) - 1) / c + 2);
    return p;
}

// The workspace layout is fixed by an upper bound on the parts per head over
// every grid cap a decode kernel can have (SMs x 1..kMaxCtasPerSmBound
// resident CTAs), so that its size does not depend on which kernel runs.
DecodePlan bound_plan(long long BH, int S, int device) {
    const long long sms = sm_count(device) > 0 ? sm_count(device) : 1;
    DecodePlan b = make_plan(BH, S, sms);
    for (long long occ = 2; occ <= kMaxCtasPerSmBound; ++occ) {
        const DecodePlan p = make_plan(BH, S, sms * occ);
        if (p.max_parts > b.max_parts) b = p;
    }
    return b;
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// [0, 16): counters (next chunk, cut heads claimed for merging, heads
// claimed for the exchange merge, CTAs finished); from 256: max_parts tagged
// records of D + 2 64-bit values per head.  All zero between calls.
struct WsLayout {
    size_t sched_off, parts_off, total;
};

WsLayout ws_layout(long long BH, int max_parts, int D) {
    WsLayout w{};
    w.sched_off = 0;
    w.parts_off = 256;
    w.total = w.parts_off +
              align_up(static_cast<size_t>(BH) * max_parts * (D + 2) * sizeof(unsigned long long),
                       256);
    return w;
}

__global__ void empty_grid_kernel() {}

// Launch through cudaLaunchKernel so the launch status comes back as a return
// value without clearing (or reading) the host thread's pending CUDA error:
// a failed launch stays visible to the caller's next error query, as with
// the reference's <<<...>>> launches.
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*fn)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, Args... args) {
    static_assert(sizeof...(KArgs) == sizeof...(Args), "argument count");
    std::tuple<KArgs...> vals(static_cast<KArgs>(args)...);
    void* ptrs[sizeof...(KArgs) > 0 ? sizeof...(KArgs) : 1];
    std::apply([&](auto&... v) {
        int i = 0;
        ((ptrs[i++] = static_cast<void*>(&v)), ...);
    }, vals);
    return cudaLaunchKernel(reinterpret_cast<const void*>(fn), grid, block, ptrs, smem, stream);
}

// Launch as a programmatic dependent of the previous launch in the stream:
// the kernel's CTAs may be dispatched while that launch finishes, and wait
// for it (griddepcontrol.wait) before touching global memory.  Used for the
// decode kernels, whose consecutive launches (one per decode step) otherwise
// leave ~2 us between the end of one and the start of the next.
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel_dependent(void (*fn)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                    cudaStream_t stream, Args... args) {
    static_assert(sizeof...(KArgs) == sizeof...(Args), "argument count");
    std::tuple<KArgs...> vals(static_cast<KArgs>(args)...);
    void* ptrs[sizeof...(KArgs) > 0 ? sizeof...(KArgs) : 1];
    std::apply([&](auto&... v) {
        int i = 0;
        ((ptrs[i++] = static_cast<void*>(&v)), ...);
    }, vals);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(fn), ptrs);
}

template <int D, int BS>
tqkv_status compress_impl(const void* x, int8_t* xq, void* scales, long long rows, int T,
                          int S_cap, int t0, cudaStream_t stream) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return from_cuda(e);
    auto fn = T == S_cap ? kv_compress_kernel<D, BS, TQKV_COMPRESS_DIV_MODE, false>
                         : kv_compress_kernel<D, BS, TQKV_COMPRESS_DIV_MODE, true>;
    const int per_sm = prepare_kernel(fn, kCompressThreads, 0, dev);
    const long long rows_per_block =
        static_cast<long long>(kCompressUnroll) * (kCompressThreads / 32) * (32 / (D / 8));
    long long grid = (rows + rows_per_block - 1) / rows_per_block;
    const long long cap = static_cast<long long>(sm_count(dev)) * (per_sm > 0 ? per_sm : 1);
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    return from_cuda(launch_kernel(fn, dim3(static_cast<unsigned>(grid)), dim3(kCompressThreads), 0,
                                   stream, static_cast<const uint4*>(x),
                                   reinterpret_cast<uint2*>(xq), static_cast<__half*>(scales),
                                   rows, T, S_cap, t0));
}

template <int D, int BS>
tqkv_status reconstruct_impl(const int8_t* xq, const void* scales, void* y, long long rows,
                             cudaStream_t stream) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return from_cuda(e);
    auto fn = kv_reconstruct_kernel<D, BS>;
    const int per_sm = prepare_kernel(fn, kCompressThreads, 0, dev);
    // one warp step covers 32 * kReconstructInFlight groups of 8 codes
    const long long groups_per_block = (kCompressThreads / 32) * 32 * kReconstructInFlight;
    long long grid = (rows * (D / 8) + groups_per_block - 1) / groups_per_block;
    const long long cap = static_cast<long long>(sm_count(dev)) * (per_sm > 0 ? per_sm : 1);
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    return from_cuda(launch_kernel(fn, dim3(static_cast<unsigned>(grid)), dim3(kCompressThreads), 0,
                                   stream, reinterpret_cast<const uint2*>(xq),
                                   static_cast<const __half*>(scales), static_cast<uint4*>(y),
                                   rows));
}

template <int D, int BS, bool kHalfKV, int OUT, int APPEND = kNoAppend>
tqkv_status decode_impl(DecodeArgs a, long long total_rows, int S, int BH, void* workspace,
                        size_t workspace_bytes, cudaStream_t stream) {
    // a.peer is set by the caller (kOutPeers) or zero; a.S_stride and a.group
    // by the caller
    using C = DecodeCfg<D, BS, kHalfKV>;
    if (a.group < 1 || BH % a.group != 0) return TQKV_ERR_INVALID_SIZE;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return from_cuda(e);
    auto fn = decode_attn_kernel<D, BS, kHalfKV, OUT, APPEND>;
    const int per_sm = prepare_kernel(fn, kDecodeThreads, C::kSmemBytes, dev);
    if (per_sm <= 0) return from_cuda(cudaErrorInvalidConfiguration);

    const DecodePlan bound = bound_plan(BH, S, dev);
    const WsLayout lay = ws_layout(BH, bound.max_parts, D);
    // the workspace bound covers up to kMaxCtasPerSmBound CTAs per SM
    const int occ = per_sm < kMaxCtasPerSmBound ? per_sm : kMaxCtasPerSmBound;
    const long long resident = static_cast<long long>(sm_count(dev)) * occ;
    const DecodePlan plan = make_plan(BH, S, resident);
    if (plan.max_parts > bound.max_parts) return TQKV_ERR_WORKSPACE;  // cannot happen: occ <= bound
    // records and tickets for cut heads; the claim counter for dynamic chunks;
    // the merge counters of the one-launch exchange
    constexpr bool kFold = OUT == kOutExchange;
    const bool needs_ws = plan.nchunks > 1 || kFold;
    if (needs_ws && (workspace == nullptr || workspace_bytes < lay.total)) return TQKV_ERR_WORKSPACE;

    uint8_t* ws = static_cast<uint8_t*>(workspace);
    // chunk claims, merge and exchange claims, CTAs finished; without a
    // workspace one CTA streams the single chunk
    a.ctr = needs_ws ? reinterpret_cast<unsigned int*>(ws + lay.sched_off) : nullptr;
    a.recs = needs_ws ? reinterpret_cast<unsigned long long*>(ws + lay.parts_off) : nullptr;
    a.total_rows = static_cast<long long>(BH) * S;
    a.chunk_rows = plan.chunk_rows;
    a.nchunks = static_cast<unsigned int>(plan.nchunks);
    a.S = S;
    a.BH = BH;
    a.max_parts = bound.max_parts;
    a.score_scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(D)));
    // Every decode launch is a programmatic dependent of the previous one.
    // When the grid covers every SM it lets the next launch be dispatched
    // from each CTA's start; a smaller grid does so only after each CTA's
    // last tile is issued, because the next launch's CTAs would otherwise
    // sit in the idle SMs through the whole launch.  Measured on one B200,
    // steps replayed in one graph, against plain launches: B4 H32 S16384
    // (591 CTAs) 87.6-88.1 -> 84.2-84.3 us with the early signal (85.0-85.1
    // with the late one); B4 H32 S131072 617-620 -> 615 us; B8 H12 S1024 D64
    // (384 CTAs) 10.5 -> 10.0 us; B2 H8 S2048 (128 CTAs) 10.3-10.7 -> 9.7-9.8
    // us with the late signal (11.6 with the early one).
    a.early_dependents = plan.grid >= sm_count(dev) ? 1 : 0;
    return from_cuda(launch_kernel_dependent(fn, dim3(plan.grid), dim3(kDecodeThreads),
                                             C::kSmemBytes, stream, a));
}

template <int D, int BS, bool kHalfKV>
tqkv_status decode_out(OutKind out, const DecodeArgs& a, long long total, int S, int BH,
                       void* ws, size_t wsb, cudaStream_t stream) {
    if constexpr (!kHalfKV) {
        // fused append: quantise the newest rows with the compress kernel's rounding
        constexpr int kAppend = TQKV_COMPRESS_DIV_MODE;
        if (a.T_new > 0 && out == OutKind::kHalfO)
            return decode_impl<D, BS, false, kOutHalf, kAppend>(a, total, S, BH, ws, wsb, stream);
        if (a.T_new > 0 && out == OutKind::kPeers)
            return decode_impl<D, BS, false, kOutPeers, kAppend>(a, total, S, BH, ws, wsb, stream);
        if (a.T_new > 0 && out == OutKind::kExchange)
            return decode_impl<D, BS, false, kOutExchange, kAppend>(a, total, S, BH, ws, wsb, stream);
    }
    if (a.T_new > 0) return TQKV_ERR_UNSUPPORTED;
    if (out == OutKind::kHalfO)
        return decode_impl<D, BS, kHalfKV, kOutHalf>(a, total, S, BH, ws, wsb, stream);
    if (out == OutKind::kPartial)
        return decode_impl<D, BS, kHalfKV, kOutPartial>(a, total, S, BH, ws, wsb, stream);
    if constexpr (!kHalfKV) {
        if (out == OutKind::kExchange)
            return decode_impl<D, BS, kHalfKV, kOutExchange>(a, total, S, BH, ws, wsb, stream);
        return decode_impl<D, BS, kHalfKV, kOutPeers>(a, total, S, BH, ws, wsb, stream);
    }
    return TQKV_ERR_UNSUPPORTED;
}

// INT8 decode with the kOutPeers epilogue (split-S over NVLink), or with
// kOutExchange (the same, then the merge into O in the same launch).
tqkv_status launch_decode_peers(OutKind o_kind, const PeerArgs& peer, const void* q, const void* k,
                                const void* ks, const void* v, const void* vs, void* o, int BH,
                                int S, int D, int bs, void* workspace, size_t workspace_bytes,
                                cudaStream_t stream, int S_stride = 0,
                                const AppendRows* append = nullptr) {
    DecodeArgs a{};
    a.q = q;
    a.k = k;
    a.v = v;
    a.ks = static_cast<const uint16_t*>(ks);
    a.vs = static_cast<const uint16_t*>(vs);
    a.out = o_kind == OutKind::kExchange ? o : nullptr;
    a.peer = peer;
    a.S_stride = S_stride > 0 ? S_stride : S;
    a.group = 1;
    if (append != nullptr) {
        a.k_new = append->k_new;
        a.v_new = append->v_new;
        a.T_new = append->T;
    }
    const long long total = static_cast<long long>(BH) * S;
    const OutKind kind = o_kind;
    if (D == 64 && bs == 32) return decode_out<64, 32, false>(kind, a, total, S, BH, workspace, workspace_bytes, stream);
    if (D == 64 && bs == 64) return decode_out<64, 64, false>(kind, a, total, S, BH, workspace, workspace_bytes, stream);
    if (D == 128 && bs == 32) return decode_out<128, 32, false>(kind, a, total, S, BH, workspace, workspace_bytes, stream);
    if (D == 128 && bs == 64) return decode_out<128, 64, false>(kind, a, total, S, BH, workspace, workspace_bytes, stream);
    if (D == 128 && bs == 128) return decode_out<128, 128, false>(kind, a, total, S, BH, workspace, workspace_bytes, stream);
    return TQKV_ERR_UNSUPPORTED;
}

size_t exchange_bytes(int world, long long BH, int D) {
    return kExchangeHeaderBytes +
           align_up(static_cast<size_t>(2) * world * BH * (D + 2) * sizeof(unsigned long long),
                    256);
}

// PeerArgs from the host array of every rank's exchange buffer.
tqkv_status make_peer_args(void* const* bufs, int world, int rank, PeerArgs* out) {
    PeerArgs peer{};
    for (int r = 0; r < world; ++r) {
        if (!bufs[r]) return TQKV_ERR_NULL;
        uint8_t* base = static_cast<uint8_t*>(bufs[r]);
        peer.recs[r] = reinterpret_cast<unsigned long long*>(base + kExchangeHeaderBytes);
    }
    peer.own = static_cast<unsigned int*>(bufs[rank]);
    peer.own_recs = peer.recs[rank];
    peer.world = world;
    peer.rank = rank;
    *out = peer;
    return TQKV_OK;
}

// The two small launches of a step for a rank whose token slice is empty:
// empty records into every rank's buffer; with `o`, then the merge into O.
tqkv_status publish_empty(const PeerArgs& peer, void* o, int BH, int D, cudaStream_t stream) {
    cudaError_t e;
    if (D == 64)
        e = launch_kernel(publish_empty_kernel<64>, dim3(BH), dim3(64), 0, stream, peer, BH);
    else
        e = launch_kernel(publish_empty_kernel<128>, dim3(BH), dim3(128), 0, stream, peer, BH);
    if (e != cudaSuccess || o == nullptr) return from_cuda(e);
    if (D == 64)
        return from_cuda(launch_kernel(exchange_combine_kernel<64>, dim3(BH), dim3(64), 0, stream,
                                       peer, static_cast<__half*>(o), BH));
    return from_cuda(launch_kernel(exchange_combine_kernel<128>, dim3(BH), dim3(128), 0, stream,
                                   peer, static_cast<__half*>(o), BH));
}

template <int D>
tqkv_status combine_impl(const float* partials, void* o, int R, int BH, cudaStream_t stream) {
    return from_cuda(launch_kernel(lse_combine_kernel<D>, dim3(BH), dim3(D), 0, stream, partials,
                                   static_cast<__half*>(o), R, BH));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

tqkv_status from_cuda(cudaError_t err) {
    if (err == cudaSuccess) return TQKV_OK;
    t_last_cuda_error = static_cast<int>(err);
    return TQKV_ERR_CUDA;
}

bool is_supported_int8(int D, int block_size) {
    if (D == 64) return block_size == 32 || block_size == 64;
    if (D == 128) return block_size == 32 || block_size == 64 || block_size == 128;
    return false;
}

tqkv_status launch_compress(const void* x, int8_t* xq, void* scales, long long rows, int D,
                            int bs, cudaStream_t stream, int T, int S_cap, int t0) {
    if (T <= 0) {  // whole tensors: rows land where they come from
        T = 1;
        S_cap = 1;
        t0 = 0;
    }
    if (D == 64 && bs == 32) return compress_impl<64, 32>(x, xq, scales, rows, T, S_cap, t0, stream);
    if (D == 64 && bs == 64) return compress_impl<64, 64>(x, xq, scales, rows, T, S_cap, t0, stream);
    if (D == 128 && bs == 32) return compress_impl<128, 32>(x, xq, scales, rows, T, S_cap, t0, stream);
    if (D == 128 && bs == 64) return compress_impl<128, 64>(x, xq, scales, rows, T, S_cap, t0, stream);
    if (D == 128 && bs == 128) return compress_impl<128, 128>(x, xq, scales, rows, T, S_cap, t0, stream);
    return TQKV_ERR_UNSUPPORTED;
}

tqkv_status launch_reconstruct(const int8_t* xq, const void* scales, void* y, long long rows,
                               int D, int bs, cudaStream_t stream) {
    if (D == 64 && bs == 32) return reconstruct_impl<64, 32>(xq, scales, y, rows, stream);
    if (D == 64 && bs == 64) return reconstruct_impl<64, 64>(xq, scales, y, rows, stream);
    if (D == 128 && bs == 32) return reconstruct_impl<128, 32>(xq, scales, y, rows, stream);
    if (D == 128 && bs == 64) return reconstruct_impl<128, 64>(xq, scales, y, rows, stream);
    if (D == 128 && bs == 128) return reconstruct_impl<128, 128>(xq, scales, y, rows, stream);
    return TQKV_ERR_UNSUPPORTED;
}

tqkv_status launch_decode(KvKind kv, OutKind out, const void* q, const void* k, const void* ks,
                          const void* v, const void* vs, void* o, int BH, int S, int D, int bs,
                          void* workspace, size_t workspace_bytes, cudaStream_t stream,
                          int S_stride, const AppendRows* append, int group) {
    DecodeArgs a{};
    a.S_stride = S_stride > 0 ? S_stride : S;
    a.group = group;
    if (group > 1 && append != nullptr) return TQKV_ERR_UNSUPPORTED;
    if (append != nullptr) {
        if (kv != KvKind::kInt8) return TQKV_ERR_UNSUPPORTED;
        a.k_new = append->k_new;
        a.v_new = append->v_new;
        a.T_new = append->T;
    }
    a.q = q;
    a.k = k;
    a.v = v;
    a.ks = static_cast<const uint16_t*>(ks);
    a.vs = static_cast<const uint16_t*>(vs);
    a.out = o;
    const long long total = static_cast<long long>(BH) * S;
    if (kv == KvKind::kHalf) {
        if (D == 64) return decode_out<64, 64, true>(out, a, total, S, BH, workspace, workspace_bytes, stream);
        if (D == 128) return decode_out<128, 128, true>(out, a, total, S, BH, workspace, workspace_bytes, stream);
        return TQKV_ERR_UNSUPPORTED;
    }
    if (D == 64 && bs == 32) return decode_out<64, 32, false>(out, a, total, S, BH, workspace, workspace_bytes, stream);
    if (D == 64 && bs == 64) return decode_out<64, 64, false>(out, a, total, S, BH, workspace, workspace_bytes, stream);
    if (D == 128 && bs == 32) return decode_out<128, 32, false>(out, a, total, S, BH, workspace, workspace_bytes, stream);
    if (D == 128 && bs == 64) return decode_out<128, 64, false>(out, a, total, S, BH, workspace, workspace_bytes, stream);
    if (D == 128 && bs == 128) return decode_out<128, 128, false>(out, a, total, S, BH, workspace, workspace_bytes, stream);
    return TQKV_ERR_UNSUPPORTED;
}

tqkv_status launch_fill_half(void* o, long long n, uint16_t bits, cudaStream_t stream) {
    if (n <= 0) return TQKV_OK;
    long long grid = (n + 255) / 256;
    if (grid > 1024) grid = 1024;
    return from_cuda(launch_kernel(fill_half_kernel, dim3(static_cast<unsigned>(grid)), dim3(256),
                                   0, stream, static_cast<uint16_t*>(o), n, bits));
}

tqkv_status launch_empty_partials(float* p, long long heads, int D, cudaStream_t stream) {
    const long long n = heads * (D + 2);
    if (n <= 0) return TQKV_OK;
    long long grid = (n + 255) / 256;
    if (grid > 1024) grid = 1024;
    return from_cuda(launch_kernel(fill_empty_partials_kernel, dim3(static_cast<unsigned>(grid)),
                                   dim3(256), 0, stream, p, heads, D));
}

size_t decode_workspace_bytes(long long BH, int S, int D) {
    if (BH <= 0 || S <= 0) return 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    const DecodePlan bound = bound_plan(BH, S, dev);
    return ws_layout(BH, bound.max_parts, D).total;
}

namespace {
// cudaMalloc + zero fill in stream order; the failing call's error is kept
// for the calling thread (tqkv_last_cuda_error).
struct CudaZeroedAlloc {
    void* operator()(int /*device: current*/, cudaStream_t stream, size_t bytes) const {
        void* p = nullptr;
        cudaError_t e = cudaMalloc(&p, bytes);
        if (e == cudaSuccess) e = cudaMemsetAsync(p, 0, bytes, stream);
        if (e != cudaSuccess) {
            if (p) cudaFree(p);
            from_cuda(e);
            return nullptr;
        }
        return p;
    }
};
WorkspaceCache<cudaStream_t, CudaZeroedAlloc>& ws_cache() {
    static WorkspaceCache<cudaStream_t, CudaZeroedAlloc> cache{CudaZeroedAlloc{}};
    return cache;
}
}  // namespace

void* cached_workspace(cudaStream_t stream, size_t bytes, tqkv_status* status) {
    *status = TQKV_OK;
    if (bytes == 0) return nullptr;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        *status = from_cuda(e);
        return nullptr;
    }
    void* p = ws_cache().get(dev, stream, bytes);
    if (p == nullptr) *status = TQKV_ERR_CUDA;
    return p;
}

void raise_empty_grid_error(cudaStream_t stream) {
    (void)launch_kernel(empty_grid_kernel, dim3(0), dim3(1), 0, stream);
}

}  // namespace tqkv

// ===========================================================================
// extern "C" ABI
// ===========================================================================
using tqkv::KvKind;
using tqkv::OutKind;

extern "C" {

const char* tqkv_status_string(tqkv_status s) {
    switch (s) {
        case TQKV_OK: return "ok";
        case TQKV_ERR_UNSUPPORTED: return "unsupported D / block_size / lanes / tile";
        case TQKV_ERR_INVALID_SIZE: return "invalid size";
        case TQKV_ERR_MISALIGNED: return "pointer not 16-byte aligned";
        case TQKV_ERR_WORKSPACE: return "workspace missing or too small";
        case TQKV_ERR_CUDA: return "CUDA runtime error";
        case TQKV_ERR_NULL: return "null pointer";
    }
    return "unknown status";
}

int tqkv_last_cuda_error(void) { return tqkv::t_last_cuda_error; }

const char* tqkv_version(void) { return "tqkv-b200 0.1.0 sm_100a"; }

tqkv_status tqkv_kv_compress(const void* x, int8_t* xq, void* scales, int B, int H, int S, int D,
                             int block_size, cudaStream_t stream) {
    if (!tqkv::is_supported_int8(D, block_size)) return TQKV_ERR_UNSUPPORTED;
    if (B <= 0 || H <= 0 || S <= 0) return TQKV_ERR_INVALID_SIZE;
    if (!x || !xq || !scales) return TQKV_ERR_NULL;
    if (!tqkv::aligned16(x) || !tqkv::aligned16(xq)) return TQKV_ERR_MISALIGNED;
    const long long rows = static_cast<long long>(B) * H * S;
    return tqkv::launch_compress(x, xq, scales, rows, D, block_size, stream);
}

tqkv_status tqkv_kv_reconstruct(const int8_t* xq, const void* scales, void* y, int B, int H,
                                int S, int D, int block_size, cudaStream_t stream) {
    if (!tqkv::is_supported_int8(D, block_size)) return TQKV_ERR_UNSUPPORTED;
    if (B <= 0 || H <= 0 || S <= 0) return TQKV_ERR_INVALID_SIZE;
    if (!xq || !scales || !y) return TQKV_ERR_NULL;
    if (!tqkv::aligned16(xq) || !tqkv::aligned16(y)) return TQKV_ERR_MISALIGNED;
    const long long rows = static_cast<long long>(B) * H * S;
    return tqkv::launch_reconstruct(xq, scales, y, rows, D, block_size, stream);
}

tqkv_status tqkv_kv_append(const void* x, int8_t* cache_q, void* cache_s, int B, int H, int T,
                           int D, int block_size, int S_cap, int t0, cudaStream_t stream) {
    if (!tqkv::is_supported_int8(D, block_size)) return TQKV_ERR_UNSUPPORTED;
    if (B <= 0 || H <= 0 || T <= 0 || S_cap <= 0 || t0 < 0 ||
        static_cast<long long>(t0) + T > S_cap)
        return TQKV_ERR_INVALID_SIZE;
    if (!x || !cache_q || !cache_s) return TQKV_ERR_NULL;
    if (!tqkv::aligned16(x) || !tqkv::aligned16(cache_q)) return TQKV_ERR_MISALIGNED;
    const long long rows = static_cast<long long>(B) * H * T;
    return tqkv::launch_compress(x, cache_q, cache_s, rows, D, block_size, stream, T, S_cap, t0);
}

tqkv_status tqkv_decode_int8_cache(const void* q, const int8_t* kq, const void* ks,
                                   const int8_t* vq, const void* vs, void* o, int B, int H, int S,
                                   int S_cap, int D, int block_size, void* workspace,
                                   size_t workspace_bytes, cudaStream_t stream) {
    if (!tqkv::is_supported_int8(D, block_size)) return TQKV_ERR_UNSUPPORTED;
    if (B <= 0 || H <= 0 || S < 0 || S_cap <= 0 || S > S_cap) return TQKV_ERR_INVALID_SIZE;
    if (!q || !o) return TQKV_ERR_NULL;
    const long long BH = static_cast<long long>(B) * H;
    if (BH > 0x7fffffffLL) return TQKV_ERR_INVALID_SIZE;
    if (S == 0) return tqkv::launch_fill_half(o, BH * D, 0x7e00u, stream);
    if (!kq || !ks || !vq || !vs) return TQKV_ERR_NULL;
    if (!tqkv::aligned16(kq) || !tqkv::aligned16(vq)) return TQKV_ERR_MISALIGNED;
    return tqkv::launch_decode(KvKind::kInt8, OutKind::kHalfO, q, kq, ks, vq, vs, o,
                               static_cast<int>(BH), S, D, block_size, workspace, workspace_bytes,
                               stream, S_cap);
}

tqkv_status tqkv_decode_int8_append(const void* q, const void* k_new, const void* v_new,
                                    int8_t* kq, void* ks, int8_t* vq, void* vs, void* o, int B,
                                    int H, int T, int S, int S_cap, int D, int block_size,
                                    void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (!tqkv::is_supported_int8(D, block_size)) return TQKV_ERR_UNSUPPORTED;
    if (B <= 0 || H <= 0 || T <= 0 || S < T || S_cap < S) return TQKV_ERR_INVALID_SIZE;
    if (!q || !o || !k_new || !v_new || !kq || !ks || !vq || !vs) return TQKV_ERR_NULL;
    if (!tqkv::aligned16(kq) || !tqkv::aligned16(vq) || !tqkv::aligned16(k_new) ||
        !tqkv::aligned16(v_new))
        return TQKV_ERR_MISALIGNED;
    const long long BH = static_cast<long long>(B) * H;
    if (BH > 0x7fffffffLL) return TQKV_ERR_INVALID_SIZE;
    const tqkv::AppendRows rows{k_new, v_new, T};
    return tqkv::launch_decode(KvKind::kInt8, OutKind::kHalfO, q, kq, ks, vq, vs, o,
                               static_cast<int>(BH), S, D, block_size, workspace, workspace_bytes,
                               stream, S_cap, &rows);
}

tqkv_status tqkv_decode_int8_gqa(const void* q, const int8_t* kq, const void* ks,
                                 const int8_t* vq, const void* vs, void* o, int B, int H_q,
                                 int H_kv, int S, int D, int block_size, void* workspace,
                                 size_t workspace_bytes, cudaStream_t stream) {
    if (!tqkv::is_supported_int8(D, block_size)) return TQKV_ERR_UNSUPPORTED;
    if (B <= 0 || H_q <= 0 || H_kv <= 0 || S < 0 || H_q % H_kv != 0) return TQKV_ERR_INVALID_SIZE;
    if (!q || !o) return TQKV_ERR_NULL;
    const long long BH = static_cast<long long>(B) * H_q;
    if (BH > 0x7fffffffLL) return TQKV_ERR_INVALID_SIZE;
    if (S == 0) return tqkv::launch_fill_half(o, BH * D, 0x7e00u, stream);
    if (!kq || !ks || !vq || !vs) return TQKV_ERR_NULL;
    if (!tqkv::aligned16(kq) || !tqkv::aligned16(vq)) return TQKV_ERR_MISALIGNED;
    return tqkv::launch_decode(KvKind::kInt8, OutKind::kHalfO, q, kq, ks, vq, vs, o,
                               static_cast<int>(BH), S, D, block_size, workspace, workspace_bytes,
                               stream, S, nullptr, H_q / H_kv);
}

tqkv_status tqkv_decode_plan(long long BH, int S, int max_ctas, long long* grid,
                             long long* chunk_rows, long long* nchunks, long long* max_parts) {
    if (BH <= 0 || S <= 0 || max_ctas <= 0) return TQKV_ERR_INVALID_SIZE;
    if (!grid || !chunk_rows || !nchunks || !max_parts) return TQKV_ERR_NULL;
    const tqkv::DecodePlan p = tqkv::make_plan(BH, S, max_ctas);
    *grid = p.grid;
    *chunk_rows = p.chunk_rows;
    *nchunks = p.nchunks;
    *max_parts = p.max_parts;
    return TQKV_OK;
}

size_t tqkv_decode_workspace_bytes(int B, int H, int S, int D) {
    if (B <= 0 || H <= 0 || S <= 0 || (D != 64 && D != 128)) return 0;
    return tqkv::decode_workspace_bytes(static_cast<long long>(B) * H, S, D);
}

tqkv_status tqkv_workspace_init(void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (workspace_bytes == 0) return TQKV_OK;
    if (!workspace) return TQKV_ERR_NULL;
    return tqkv::from_cuda(cudaMemsetAsync(workspace, 0, workspace_bytes, stream));
}

tqkv_status tqkv_decode_int8(const void* q, const int8_t* kq, const void* ks, const int8_t* vq,
                             const void* vs, void* o, int B, int H, int S, int D, int block_size,
                             void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (!tqkv::is_supported_int8(D, block_size)) return TQKV_ERR_UNSUPPORTED;
    if (B <= 0 || H <= 0 || S < 0) return TQKV_ERR_INVALID_SIZE;
    if (!q || !o) return TQKV_ERR_NULL;
    const long long BH = static_cast<long long>(B) * H;
    if (BH > 0x7fffffffLL) return TQKV_ERR_INVALID_SIZE;
    if (S == 0) return tqkv::launch_fill_half(o, BH * D, 0x7e00u, stream);  // NaN, as 0 * (1/0)
    if (!kq || !ks || !vq || !vs) return TQKV_ERR_NULL;
    if (!tqkv::aligned16(kq) || !tqkv::aligned16(vq)) return TQKV_ERR_MISALIGNED;
    return tqkv::launch_decode(KvKind::kInt8, OutKind::kHalfO, q, kq, ks, vq, vs, o,
                               static_cast<int>(BH), S, D, block_size, workspace, workspace_bytes,
                               stream);
}

tqkv_status tqkv_decode_fp16(const void* q, const void* k, const void* v, void* o, int B, int H,
                             int S, int D, void* workspace, size_t workspace_bytes,
                             cudaStream_t stream) {
    if (D != 64 && D != 128) return TQKV_ERR_UNSUPPORTED;
    if (B <= 0 || H <= 0 || S < 0) return TQKV_ERR_INVALID_SIZE;
    if (!q || !o) return TQKV_ERR_NULL;
    const long long BH = static_cast<long long>(B) * H;
    if (BH > 0x7fffffffLL) return TQKV_ERR_INVALID_SIZE;
    if (S == 0) return tqkv::launch_fill_half(o, BH * D, 0x0000u, stream);
    if (!k || !v) return TQKV_ERR_NULL;
    if (!tqkv::aligned16(k) || !tqkv::aligned16(v)) return TQKV_ERR_MISALIGNED;
    return tqkv::launch_decode(KvKind::kHalf, OutKind::kHalfO, q, k, nullptr, v, nullptr, o,
                               static_cast<int>(BH), S, D, D, workspace, workspace_bytes, stream);
}

tqkv_status tqkv_decode_int8_partial(const void* q, const int8_t* kq, const void* ks,
                                     const int8_t* vq, const void* vs, float* partial, int B,
                                     int H, int S, int D, int block_size, void* workspace,
                                     size_t workspace_bytes, cudaStream_t stream) {
    if (!tqkv::is_supported_int8(D, block_size)) return TQKV_ERR_UNSUPPORTED;
    if (B <= 0 || H <= 0 || S < 0) return TQKV_ERR_INVALID_SIZE;
    if (!q || !partial) return TQKV_ERR_NULL;
    const long long BH = static_cast<long long>(B) * H;
    if (BH > 0x7fffffffLL) return TQKV_ERR_INVALID_SIZE;
    if (S == 0) return tqkv::launch_empty_partials(partial, BH, D, stream);
    if (!kq || !ks || !vq || !vs) return TQKV_ERR_NULL;
    if (!tqkv::aligned16(kq) || !tqkv::aligned16(vq)) return TQKV_ERR_MISALIGNED;
    return tqkv::launch_decode(KvKind::kInt8, OutKind::kPartial, q, kq, ks, vq, vs, partial,
                               static_cast<int>(BH), S, D, block_size, workspace, workspace_bytes,
                               stream);
}

tqkv_status tqkv_lse_combine(const float* partials, void* o, int R, int BH, int D,
                             cudaStream_t stream) {
    if (D != 64 && D != 128) return TQKV_ERR_UNSUPPORTED;
    if (R <= 0 || BH <= 0) return TQKV_ERR_INVALID_SIZE;
    if (!partials || !o) return TQKV_ERR_NULL;
    if (D == 64) return tqkv::combine_impl<64>(partials, o, R, BH, stream);
    return tqkv::combine_impl<128>(partials, o, R, BH, stream);
}

tqkv_status tqkv_read_device_error(uint32_t* code_out) {
    if (!code_out) return TQKV_ERR_NULL;
    unsigned int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, tqkv::g_device_error, sizeof(v));
    if (e != cudaSuccess) return tqkv::from_cuda(e);
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(tqkv::g_device_error, &zero, sizeof(zero));
    if (e != cudaSuccess) return tqkv::from_cuda(e);
    *code_out = v;
    return TQKV_OK;
}

}  // extern "C"

// ===========================================================================
// Split-S across the GPUs of one node over NVLink peer mappings (no NCCL)
// ===========================================================================
extern "C" {

size_t tqkv_exchange_bytes(int world, int BH, int D) {
    if (world <= 0 || world > tqkv::kMaxPeers || BH <= 0 || (D != 64 && D != 128)) return 0;
    return tqkv::exchange_bytes(world, BH, D);
}

tqkv_status tqkv_exchange_alloc(size_t bytes, void** buf_out) {
    if (!buf_out || bytes == 0) return TQKV_ERR_NULL;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);  // a whole allocation: its IPC handle maps exactly it
    if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        return tqkv::from_cuda(e);
    }
    *buf_out = p;
    return TQKV_OK;
}

tqkv_status tqkv_exchange_free(void* buf) {
    if (!buf) return TQKV_OK;
    return tqkv::from_cuda(cudaFree(buf));
}

tqkv_status tqkv_ipc_get_handle(const void* buf, void* handle_out) {
    if (!buf || !handle_out) return TQKV_ERR_NULL;
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(buf));
    if (e != cudaSuccess) return tqkv::from_cuda(e);
    std::memcpy(handle_out, &h, sizeof(h));
    return TQKV_OK;
}

tqkv_status tqkv_ipc_open_handle(const void* handle, void** buf_out) {
    if (!handle || !buf_out) return TQKV_ERR_NULL;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return tqkv::from_cuda(e);
    *buf_out = p;
    return TQKV_OK;
}

tqkv_status tqkv_ipc_close_handle(void* buf) {
    if (!buf) return TQKV_OK;
    return tqkv::from_cuda(cudaIpcCloseMemHandle(buf));
}

namespace {
// Shared by the publish (two-launch) and exchange (one-launch) entry points.
tqkv_status decode_split_step(OutKind kind, const void* q, const int8_t* kq, const void* ks,
                              const int8_t* vq, const void* vs, void* o, int B, int H, int S,
                              int D, int block_size, void* workspace, size_t workspace_bytes,
                              void* const* exchange_bufs, int world, int rank,
                              cudaStream_t stream) {
    if (!tqkv::is_supported_int8(D, block_size)) return TQKV_ERR_UNSUPPORTED;
    if (B <= 0 || H <= 0 || S < 0 || world <= 0 || world > tqkv::kMaxPeers || rank < 0 ||
        rank >= world)
        return TQKV_ERR_INVALID_SIZE;
    if (!q || !exchange_bufs || (kind == OutKind::kExchange && !o)) return TQKV_ERR_NULL;
    const long long BH = static_cast<long long>(B) * H;
    if (BH > 0x7fffffffLL) return TQKV_ERR_INVALID_SIZE;
    tqkv::PeerArgs peer{};
    const tqkv_status pst = tqkv::make_peer_args(exchange_bufs, world, rank, &peer);
    if (pst != TQKV_OK) return pst;
    if (S == 0)
        return tqkv::publish_empty(peer, kind == OutKind::kExchange ? o : nullptr,
                                   static_cast<int>(BH), D, stream);
    if (!kq || !ks || !vq || !vs) return TQKV_ERR_NULL;
    if (!tqkv::aligned16(kq) || !tqkv::aligned16(vq)) return TQKV_ERR_MISALIGNED;
    return tqkv::launch_decode_peers(kind, peer, q, kq, ks, vq, vs, o, static_cast<int>(BH), S, D,
                                     block_size, workspace, workspace_bytes, stream);
}

tqkv_status decode_split_step_append(OutKind kind, const void* q, const void* k_new,
                                     const void* v_new, int8_t* kq, void* ks, int8_t* vq,
                                     void* vs, void* o, int B, int H, int T, int S, int S_cap,
                                     int D, int block_size, void* workspace,
                                     size_t workspace_bytes, void* const* exchange_bufs,
                                     int world, int rank, cudaStream_t stream) {
    if (!tqkv::is_supported_int8(D, block_size)) return TQKV_ERR_UNSUPPORTED;
    if (B <= 0 || H <= 0 || T <= 0 || S < T || S_cap < S || world <= 0 ||
        world > tqkv::kMaxPeers || rank < 0 || rank >= world)
        return TQKV_ERR_INVALID_SIZE;
    if (!q || !k_new || !v_new || !kq || !ks || !vq || !vs || !exchange_bufs) return TQKV_ERR_NULL;
    if (kind == OutKind::kExchange && !o) return TQKV_ERR_NULL;
    if (!tqkv::aligned16(kq) || !tqkv::aligned16(vq) || !tqkv::aligned16(k_new) ||
        !tqkv::aligned16(v_new))
        return TQKV_ERR_MISALIGNED;
    const long long BH = static_cast<long long>(B) * H;
    if (BH > 0x7fffffffLL) return TQKV_ERR_INVALID_SIZE;
    tqkv::PeerArgs peer{};
    const tqkv_status pst = tqkv::make_peer_args(exchange_bufs, world, rank, &peer);
    if (pst != TQKV_OK) return pst;
    const tqkv::AppendRows rows{k_new, v_new, T};
    return tqkv::launch_decode_peers(kind, peer, q, kq, ks, vq, vs, o, static_cast<int>(BH), S, D,
                                     block_size, workspace, workspace_bytes, stream, S_cap, &rows);
}
}  // namespace

tqkv_status tqkv_decode_int8_publish(const void* q, const int8_t* kq, const void* ks,
                                     const int8_t* vq, const void* vs, int B, int H, int S, int D,
                                     int block_size, void* workspace, size_t workspace_bytes,
                                     void* const* exchange_bufs, int world, int rank,
                                     cudaStream_t stream) {
    return decode_split_step(OutKind::kPeers, q, kq, ks, vq, vs, nullptr, B, H, S, D, block_size,
                             workspace, workspace_bytes, exchange_bufs, world, rank, stream);
}

tqkv_status tqkv_decode_int8_exchange(const void* q, const int8_t* kq, const void* ks,
                                      const int8_t* vq, const void* vs, void* o, int B, int H,
                                      int S, int D, int block_size, void* workspace,
                                      size_t workspace_bytes, void* const* exchange_bufs,
                                      int world, int rank, cudaStream_t stream) {
    return decode_split_step(OutKind::kExchange, q, kq, ks, vq, vs, o, B, H, S, D, block_size,
                             workspace, workspace_bytes, exchange_bufs, world, rank, stream);
}

tqkv_status tqkv_decode_int8_append_publish(const void* q, const void* k_new, const void* v_new,
                                            int8_t* kq, void* ks, int8_t* vq, void* vs, int B,
                                            int H, int T, int S, int S_cap, int D, int block_size,
                                            void* workspace, size_t workspace_bytes,
                                            void* const* exchange_bufs, int world, int rank,
                                            cudaStream_t stream) {
    return decode_split_step_append(OutKind::kPeers, q, k_new, v_new, kq, ks, vq, vs, nullptr, B,
                                    H, T, S, S_cap, D, block_size, workspace, workspace_bytes,
                                    exchange_bufs, world, rank, stream);
}

tqkv_status tqkv_decode_int8_append_exchange(const void* q, const void* k_new, const void* v_new,
                                             int8_t* kq, void* ks, int8_t* vq, void* vs, void* o,
                                             int B, int H, int T, int S, int S_cap, int D,
                                             int block_size, void* workspace,
                                             size_t workspace_bytes, void* const* exchange_bufs,
                                             int world, int rank, cudaStream_t stream) {
    return decode_split_step_append(OutKind::kExchange, q, k_new, v_new, kq, ks, vq, vs, o, B, H,
                                    T, S, S_cap, D, block_size, workspace, workspace_bytes,
                                    exchange_bufs, world, rank, stream);
}

tqkv_status tqkv_exchange_combine(void* const* exchange_bufs, void* o, int world, int rank,
                                  int BH, int D, cudaStream_t stream) {
    if (D != 64 && D != 128) return TQKV_ERR_UNSUPPORTED;
    if (world <= 0 || world > tqkv::kMaxPeers || rank < 0 || rank >= world || BH <= 0)
        return TQKV_ERR_INVALID_SIZE;
    if (!exchange_bufs || !o) return TQKV_ERR_NULL;
    tqkv::PeerArgs peer{};
    const tqkv_status pst = tqkv::make_peer_args(exchange_bufs, world, rank, &peer);
    if (pst != TQKV_OK) return pst;
    if (D == 64)
        return tqkv::from_cuda(tqkv::launch_kernel(tqkv::exchange_combine_kernel<64>, dim3(BH),
                                                   dim3(64), 0, stream, peer,
                                                   static_cast<__half*>(o), BH));
    return tqkv::from_cuda(tqkv::launch_kernel(tqkv::exchange_combine_kernel<128>, dim3(BH),
                                               dim3(128), 0, stream, peer,
                                               static_cast<__half*>(o), BH));
}

}  // extern "C"

// ===========================================================================
// INT8 decode without any allocation: the split-S scratch is a fixed array in
// this file's device memory instead of a caller-provided workspace.
// ===========================================================================
namespace tqkv {
namespace {

constexpr size_t kNoAllocScratchBytes = TQKV_NOALLOC_SCRATCH_BYTES;
constexpr int kNoAllocMaxDevices = 64;

// One copy per GPU that loads this library, alive until the process exits.
// Host code must not pass this name to a kernel: on the host it is only a
// stand-in; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch, per device ordinal, looked up once.
std::atomic<void*> g_noalloc_addr[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

tqkv_status noalloc_scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return from_cuda(e);
    if (dev < 0 || dev >= kNoAllocMaxDevices) return TQKV_ERR_UNSUPPORTED;
    void* p = g_noalloc_addr[dev].load(std::memory_order_acquire);
    if (p == nullptr) {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        p = g_noalloc_addr[dev].load(std::memory_order_relaxed);
        if (p == nullptr) {
            // with `dev` current: the address of this device's copy of the array
            e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess) return from_cuda(e);
            g_noalloc_addr[dev].store(p, std::memory_order_release);
        }
    }
    *out = p;
    return TQKV_OK;
}

}  // namespace
}  // namespace tqkv

extern "C" tqkv_status tqkv_decode_int8_noalloc(const void* q, const int8_t* kq, const void* ks,
                                                const int8_t* vq, const void* vs, void* o, int B,
                                                int H, int S, int D, int block_size,
                                                cudaStream_t stream) {
    if (!tqkv::is_supported_int8(D, block_size)) return TQKV_ERR_UNSUPPORTED;
    if (B <= 0 || H <= 0 || S < 0) return TQKV_ERR_INVALID_SIZE;
    if (!q || !o) return TQKV_ERR_NULL;
    const long long BH = static_cast<long long>(B) * H;
    if (BH > 0x7fffffffLL) return TQKV_ERR_INVALID_SIZE;
    if (S == 0) return tqkv::launch_fill_half(o, BH * D, 0x7e00u, stream);
    if (!kq || !ks || !vq || !vs) return TQKV_ERR_NULL;
    if (!tqkv::aligned16(kq) || !tqkv::aligned16(vq)) return TQKV_ERR_MISALIGNED;
    // shapes whose split-S scratch does not fit the fixed array are refused
    const size_t need = tqkv::decode_workspace_bytes(BH, S, D);
    if (need > tqkv::kNoAllocScratchBytes) return TQKV_ERR_WORKSPACE;
    void* scratch = nullptr;
    tqkv_status st = tqkv::noalloc_scratch_address(&scratch);
    if (st != TQKV_OK) return st;
    // The array keeps whatever the previous call left.  A launch needs the
    // counters at its start and the records of this shape at zero (a record
    // whose values are tagged counts as stored); a completed call leaves them
    // zero, an interrupted one might not, so clear them every time.
    if (need > 0) {
        st = tqkv::from_cuda(cudaMemsetAsync(scratch, 0, need, stream));
        if (st != TQKV_OK) return st;
    }
    return tqkv::launch_decode(tqkv::KvKind::kInt8, tqkv::OutKind::kHalfO, q, kq, ks, vq, vs, o,
                               static_cast<int>(BH), S, D, block_size, scratch,
                               tqkv::kNoAllocScratchBytes, stream);
}
