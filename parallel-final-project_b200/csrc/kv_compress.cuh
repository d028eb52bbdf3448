// kv_compress.cuh — Kernel A (blockwise FP16 -> INT8) and Kernel B
// (INT8 -> FP16 reconstruct) device code for sm_100a.
//
// Quantisation rule (reference src/kv_compress.cu:41-95), per token row and
// per block of BS lanes along D:
//     m     = max |x|                      (fp32 of the fp16 inputs)
//     s     = m / 127 ; s = 1 if s == 0    (fp32)
//     scale = fp16(s), round-to-nearest-even
//     code  = clamp(round_half_even(x / s), -127, 127)   (x / s with fp32 s)
//
// B200 layout: one lane owns 8 consecutive elements (one 16-byte load of
// fp16, one 8-byte store of codes); D/8 lanes cover a token row, so a warp
// handles 32/(D/8) rows per step and the block max is a shuffle reduction
// over BS/8 lanes.  A grid-stride loop over row groups replaces the
// reference's one-CTA-per-row launch (16.7 M CTAs at S = 131072); the loop
// is software-pipelined, so while a warp quantises kCompressUnroll row
// groups the 16-byte loads of the next kCompressUnroll are in flight.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

#include "device_common.cuh"

namespace tqkv {

// How x / y is evaluated inside Kernel A.  The reference is compiled with
// --use_fast_math, under which a plain '/' is not an IEEE division.  The two
// can round differently only where the exact quotient 127*x/m is a
// half-integer (the "tie class"); there the approximate forms below all agree
// with the reference build and IEEE does not.  The library instantiates
// kDivApproxFtz (tqkv_capi.cu); the others are kept for the parity probe.
enum DivMode : int {
    kDivIEEE = 0,        // correctly rounded (div.rn.f32)
    kDivApprox = 1,      // div.approx.f32
    kDivApproxFtz = 2,   // div.approx.ftz.f32
    kDivFull = 3,        // div.full.f32
    kDivFullFtz = 4,     // div.full.ftz.f32
};

template <int MODE>
__device__ __forceinline__ float kv_div(float a, float b) {
    float r;
    if constexpr (MODE == kDivIEEE) {
        r = __fdiv_rn(a, b);
    } else if constexpr (MODE == kDivApprox) {
        asm("div.approx.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    } else if constexpr (MODE == kDivApproxFtz) {
        asm("div.approx.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    } else if constexpr (MODE == kDivFull) {
        asm("div.full.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    } else {
        asm("div.full.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    }
    return r;
}

// x / b for many x and one b.  The approximate forms are defined as
// x * (1 / b) (PTX ISA, div.approx), so the reciprocal is taken once and each
// quotient is one multiply, with the same flush-to-zero behaviour; the
// correctly rounded forms divide each x.
template <int MODE>
struct KvQuotient {
    float b, r;
    __device__ __forceinline__ explicit KvQuotient(float b_) : b(b_), r(0.0f) {
        if constexpr (MODE == kDivApproxFtz) {
            asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(b));
        } else if constexpr (MODE == kDivApprox) {
            asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(b));
        }
    }
    __device__ __forceinline__ float operator()(float x) const {
        float q;
        if constexpr (MODE == kDivApproxFtz) {
            asm("mul.ftz.f32 %0, %1, %2;" : "=f"(q) : "f"(x), "f"(r));
        } else if constexpr (MODE == kDivApprox) {
            asm("mul.f32 %0, %1, %2;" : "=f"(q) : "f"(x), "f"(r));
        } else {
            q = kv_div<MODE>(x, b);
        }
        return q;
    }
};

// round-to-nearest-even of x as a signed byte, saturated to [-128, 127], NaN
// to 0, in the low byte of the result (PTX lets cvt write a narrow integer
// type into a 32-bit register)
__device__ __forceinline__ uint32_t cvt_rni_sat_s8(float x) {
    uint32_t v;
    asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(v) : "f"(x));
    return v;
}

constexpr int kCompressThreads = 256;
constexpr int kCompressUnroll = 4;  // row groups whose loads a warp keeps in flight
// 8-code groups whose loads a Kernel B lane keeps in flight.  Kernel B runs
// one 256-thread CTA per SM (about 150 registers a thread); on B200 that
// streams faster than 8 groups a lane at 2 to 4 CTAs per SM, or 12 or 24
// groups a lane (B4 H32 S131072 D128: 1.03 ms against 1.07 to 1.16 ms per
// 6.5 GB tensor).
constexpr int kReconstructInFlight = 16;

__device__ __forceinline__ uint4 ld_stream_v4(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint2 ld_stream_v2(const uint2* p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
                 : "=r"(v.x), "=r"(v.y)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void st_stream_v2(uint2* p, uint2 v) {
    asm volatile("st.global.cs.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}

__device__ __forceinline__ void st_stream_v4(uint4* p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

// Quantise the 8 fp16 values in `raw` (one lane's share of a row): returns
// their codes (8 bytes) and sets `scale` to the fp16 scale of the lane's
// block.  The block max is a shuffle over aligned groups of BS/8 lanes, so
// every lane of the warp must call it.
template <int BS, int MODE>
__device__ __forceinline__ uint2 quantize_lane(uint4 raw, __half& scale) {
    constexpr int kLPB = BS / 8;  // lanes per block
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
        f[2 * i] = __low2float(h);
        f[2 * i + 1] = __high2float(h);
    }
    // max |x| with fmaxf semantics (a NaN operand is ignored unless both are NaN),
    // which makes the result independent of the reduction order.
    float a = fabsf(f[0]);
#pragma unroll
    for (int i = 1; i < 8; ++i) a = fmaxf(a, fabsf(f[i]));
#pragma unroll
    for (int off = 1; off < kLPB; off <<= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));

    float s = kv_div<MODE>(a, 127.0f);
    if (s == 0.0f) s = 1.0f;
    scale = __float2half_rn(s);
    const KvQuotient<MODE> by_s(s);  // x / s for the lane's 8 values

    // code = clamp(round_half_even(x / s), -127, 127), NaN -> 0, as one
    // saturating conversion per value.  Its range is [-128, 127], and the
    // bound -127 is never reached from below: |x| <= m, so in every division
    // mode |x / s| <= 127 * (1 + 1e-6) < 127.5.  An x that is NaN, or +-inf
    // (then s = inf and x / s is NaN), converts to 0.  The codes are packed
    // by byte permutes from the low bytes of the conversions.
    uint32_t c[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] = cvt_rni_sat_s8(by_s(f[i]));
    const uint32_t lo = __byte_perm(__byte_perm(c[0], c[1], 0x0040), __byte_perm(c[2], c[3], 0x0040),
                                    0x5410);
    const uint32_t hi = __byte_perm(__byte_perm(c[4], c[5], 0x0040), __byte_perm(c[6], c[7], 0x0040),
                                    0x5410);
    return make_uint2(lo, hi);
}

// Quantise lane c's 8 values of a row and store its codes and, on the first
// lane of each block, the block's fp16 scale.
template <int D, int BS, int MODE>
__device__ __forceinline__ void compress_lane(uint4 raw, long long row, bool valid, int c,
                                              uint2* __restrict__ xq,
                                              __half* __restrict__ scales) {
    // `row` is the destination row of codes and scales
    constexpr int kLPR = D / 8;   // lanes per row
    constexpr int kLPB = BS / 8;  // lanes per block
    constexpr int kNSub = D / BS;
    __half scale;
    const uint2 codes = quantize_lane<BS, MODE>(raw, scale);
    if (valid && (c % kLPB) == 0) scales[row * kNSub + c / kLPB] = scale;
    if (valid) st_stream_v2(xq + row * kLPR + c, codes);
}

// Destination row of source row `r` when T rows per head are written at rows
// [t0, t0 + T) of a cache holding S_cap rows per head (identity for whole
// tensors, APPEND false).
template <bool APPEND>
__device__ __forceinline__ long long append_row(long long r, int T, int S_cap, int t0) {
    if constexpr (!APPEND) {
        return r;
    } else {
        const long long bh = r / T;
        return bh * S_cap + t0 + (r - bh * T);
    }
}

// x: fp16 rows as uint4 (8 halves each), xq: codes as uint2 (8 bytes each).
// Source rows are [B*H*T]; see append_row for where they land.
template <int D, int BS, int MODE, bool APPEND>
__global__ void __launch_bounds__(kCompressThreads)
    kv_compress_kernel(const uint4* __restrict__ x, uint2* __restrict__ xq,
                       __half* __restrict__ scales, long long rows, int T, int S_cap, int t0) {
    constexpr int kLPR = D / 8;
    constexpr int kRPW = 32 / kLPR;  // rows per warp step
    const int lane = threadIdx.x & 31;
    const int c = lane % kLPR;
    const int rsub = lane / kLPR;
    const long long warp = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;

    // Software-pipelined: the loads of the next row groups are issued before
    // the current ones are quantised and stored, so 2 * kU 16-byte loads per
    // lane are in flight while the warp computes.  A step whose next row
    // groups all lie below `rows` (every step but a warp's last one or two)
    // runs without per-row bounds checks; the test is warp-uniform.
    constexpr int kU = kCompressUnroll;
    constexpr int kRowsPerStep = kU * kRPW;
    const long long step = nwarps * kRowsPerStep;
    long long r0 = warp * kRowsPerStep;
    uint4 raw[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
        const long long row = r0 + u * kRPW + rsub;
        raw[u] = row < rows ? ld_stream_v4(x + row * kLPR + c) : make_uint4(0, 0, 0, 0);
    }
    for (; r0 < rows; r0 += step) {
        uint4 nxt[kU];
        if (r0 + step + kRowsPerStep <= rows) {
            const uint4* src = x + (r0 + step + rsub) * kLPR + c;
#pragma unroll
            for (int u = 0; u < kU; ++u) nxt[u] = ld_stream_v4(src + u * kRPW * kLPR);
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const long long row = r0 + u * kRPW + rsub;
                compress_lane<D, BS, MODE>(raw[u], append_row<APPEND>(row, T, S_cap, t0), true, c,
                                           xq, scales);
            }
        } else {
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const long long row = r0 + step + u * kRPW + rsub;
                nxt[u] = row < rows ? ld_stream_v4(x + row * kLPR + c) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const long long row = r0 + u * kRPW + rsub;
                compress_lane<D, BS, MODE>(raw[u], append_row<APPEND>(row, T, S_cap, t0),
                                           row < rows, c, xq, scales);
            }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) raw[u] = nxt[u];
    }
}

// Kernel B: y = fp16(float(code) * float(scale)).  The product of a code
// (at most 8 bits) and an fp16 scale (11 significant bits) is exact in fp32,
// so the reference's only rounding is the final fp16 conversion
// (src/kv_reconstruct.cu:33).  The same value comes out of fp16x2 arithmetic
// with no conversions at all:
//   * the code c becomes the fp16 value 1024 + (c + 128) by placing the byte
//     c ^ 0x80 under the exponent byte 0x64 (a byte permute), and subtracting
//     1152 leaves c exactly;
//   * one fp16x2 multiply, round-to-nearest-even with subnormals kept, rounds
//     the exact product c * scale once, as the conversion of the exact fp32
//     product does (overflow to inf, NaN, signed zeros included).
// The codes are taken as a flat run of 8-code groups (8 divides BS and D, so
// a group never straddles a scale block): lane l of a warp instruction reads
// group g0 + l (8 bytes) and writes its 8 halves (16 bytes), so every load
// covers 256 contiguous bytes and every store 512.  Each warp step issues
// kReconstructInFlight such loads per lane before converting any of them.
__device__ __forceinline__ uint4 reconstruct_group(uint2 codes, __half scale) {
    const __half2 s2 = __half2half2(scale);
    const __half2 bias = __half2half2(__ushort_as_half(0x6480));  // 1152
    const uint32_t w[2] = {codes.x ^ 0x80808080u, codes.y ^ 0x80808080u};
    uint32_t out[4];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
#pragma unroll
        for (int p = 0; p < 2; ++p) {
            // bytes (low to high): code 2p, 0x64, code 2p+1, 0x64
            const uint32_t biased = __byte_perm(w[i], 0x64646464u, p == 0 ? 0x4140 : 0x4342);
            const __half2 c = __hsub2_rn(*reinterpret_cast<const __half2*>(&biased), bias);
            const __half2 y = __hmul2_rn(c, s2);
            out[2 * i + p] = *reinterpret_cast<const uint32_t*>(&y);
        }
    }
    return make_uint4(out[0], out[1], out[2], out[3]);
}

template <int D, int BS>
__global__ void __launch_bounds__(kCompressThreads)
    kv_reconstruct_kernel(const uint2* __restrict__ xq, const __half* __restrict__ scales,
                          uint4* __restrict__ y, long long rows) {
    constexpr int kN = kReconstructInFlight;  // group loads in flight per lane
    constexpr int kGroupsPerStep = 32 * kN;
    static_assert(BS % 8 == 0 && D % BS == 0, "8-code groups inside scale blocks");
    const long long n8 = rows * (D / 8);
    const int lane = threadIdx.x & 31;
    const long long warp = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;

    // Software-pipelined as Kernel A: the next step's groups are loaded before
    // the current ones are converted and stored; a step whose next groups all
    // lie below n8 runs without per-group bounds checks (warp-uniform test).
    const long long step = nwarps * kGroupsPerStep;
    long long g0 = warp * kGroupsPerStep;
    uint2 raw[kN];
    __half sh[kN];
#pragma unroll
    for (int u = 0; u < kN; ++u) {
        const long long g = g0 + u * 32 + lane;
        raw[u] = g < n8 ? ld_stream_v2(xq + g) : make_uint2(0u, 0u);
        sh[u] = g < n8 ? scales[(g * 8) / BS] : __ushort_as_half(0);
    }
    for (; g0 < n8; g0 += step) {
        uint2 nraw[kN];
        __half nsh[kN];
        if (g0 + step + kGroupsPerStep <= n8) {
            const long long gn = g0 + step + lane;
#pragma unroll
            for (int u = 0; u < kN; ++u) {
                nraw[u] = ld_stream_v2(xq + gn + u * 32);
                nsh[u] = scales[((gn + u * 32) * 8) / BS];
            }
#pragma unroll
            for (int u = 0; u < kN; ++u)
                st_stream_v4(y + g0 + u * 32 + lane, reconstruct_group(raw[u], sh[u]));
        } else {
#pragma unroll
            for (int u = 0; u < kN; ++u) {
                const long long g = g0 + step + u * 32 + lane;
                nraw[u] = g < n8 ? ld_stream_v2(xq + g) : make_uint2(0u, 0u);
                nsh[u] = g < n8 ? scales[(g * 8) / BS] : __ushort_as_half(0);
            }
#pragma unroll
            for (int u = 0; u < kN; ++u) {
                const long long g = g0 + u * 32 + lane;
                if (g < n8) st_stream_v4(y + g, reconstruct_group(raw[u], sh[u]));
            }
        }
#pragma unroll
        for (int u = 0; u < kN; ++u) {
            raw[u] = nraw[u];
            sh[u] = nsh[u];
        }
    }
}

}  // namespace tqkv
