// ref_launchers.cpp — the reference's five launchers with their exact C++
// signatures (reference include/attention.h:6-35, include/quantization.h:15-27),
// implemented on the B200 kernels.  Behaviour kept from the reference:
//   * void return, asynchronous on `stream`, nothing allocated per call
//     (the split-S scratch comes from a per-(device, stream) cache that grows
//     on first use and is then reused);
//   * an unsupported (D, block_size, lanes, tile) prints a message to stderr
//     and calls std::abort() (reference src/kv_compress.cu:130-135,
//     src/kv_reconstruct.cu:45-50, src/attention_baseline.cu:151-154,
//     src/attention_int8_fused.cu:185-190,
//     src/attention_int8_fused_online.cu:234-238);
//   * an empty grid (B*H*S == 0 for the row kernels, B or H == 0 for
//     attention) leaves cudaErrorInvalidConfiguration pending, and launch
//     failures stay pending for the caller's cudaGetLastError();
//   * S == 0 gives O = NaN for the online kernel (0 * (1/0)) and O = 0 for
//     the two-pass and baseline kernels, as the reference kernels compute.
// One deliberate difference: K/V tensors must be 16-byte aligned (the
// reference needs 4); a misaligned pointer aborts with a message.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>

#include "attention.h"
#include "quantization.h"
#include "tqkv.h"
#include "tqkv_internal.h"

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

[[noreturn]] void die_misaligned(const char* fn) {
    std::fprintf(stderr, "%s: K/V tensors must be 16-byte aligned\n", fn);
    std::abort();
}

// Status of a launch that passed the shim's own checks.  Launch failures are
// already pending for cudaGetLastError(); anything else is a broken invariant.
void finish(const char* fn, tqkv_status s) {
    if (s == TQKV_OK || s == TQKV_ERR_CUDA) return;
    std::fprintf(stderr, "%s: %s\n", fn, tqkv_status_string(s));
    std::abort();
}

// Attention common path: empty-grid and S <= 0 handling, workspace, launch.
void attention(const char* fn, tqkv::KvKind kv, const void* q, const void* k, const void* ks,
               const void* v, const void* vs, void* o, int B, int H, int S, int D, int bs,
               bool online, cudaStream_t stream) {
    if (B <= 0 || H <= 0) {
        tqkv::raise_empty_grid_error(stream);
        return;
    }
    const long long BH = static_cast<long long>(B) * H;
    if (S <= 0) {
        if (online) {
            finish(fn, tqkv::launch_fill_half(o, BH * D, 0x7e00u, stream));
        } else if (S == 0) {
            finish(fn, tqkv::launch_fill_half(o, BH * D, 0x0000u, stream));
        } else {
            // the reference asks for S * 4 bytes of dynamic shared memory
            tqkv::raise_empty_grid_error(stream);
        }
        return;
    }
    if (!aligned16(k) || !aligned16(v)) die_misaligned(fn);
    tqkv_status st = TQKV_OK;
    const size_t need = tqkv::decode_workspace_bytes(BH, S, D);
    void* ws = tqkv::cached_workspace(stream, need, &st);
    if (st != TQKV_OK) return;  // allocation failure is pending as a CUDA error
    finish(fn, tqkv::launch_decode(kv, tqkv::OutKind::kHalfO, q, k, ks, v, vs, o,
                                   static_cast<int>(BH), S, D, bs, ws, need, stream));
}

}  // namespace

void launch_kv_compress(const __half* dX, int8_t* dXq, __half* dScales, int B, int H, int S,
                        int D, int block_size, cudaStream_t stream) {
    if (!tqkv::is_supported_int8(D, block_size)) {
        std::fprintf(stderr,
                     "launch_kv_compress: unsupported (D=%d, block_size=%d). "
                     "Supported: D in {64,128}, block_size in {32,64,128}, block_size <= D.\n",
                     D, block_size);
        std::abort();
    }
    const long long rows = static_cast<long long>(B) * H * S;
    if (rows <= 0) {
        tqkv::raise_empty_grid_error(stream);
        return;
    }
    if (!aligned16(dX) || !aligned16(dXq)) die_misaligned("launch_kv_compress");
    finish("launch_kv_compress",
           tqkv::launch_compress(dX, dXq, dScales, rows, D, block_size, stream));
}

void launch_kv_reconstruct(const int8_t* dXq, const __half* dScales, __half* dY, int B, int H,
                           int S, int D, int block_size, cudaStream_t stream) {
    if (!tqkv::is_supported_int8(D, block_size)) {
        std::fprintf(stderr, "launch_kv_reconstruct: unsupported (D=%d, block_size=%d).\n", D,
                     block_size);
        std::abort();
    }
    const long long rows = static_cast<long long>(B) * H * S;
    if (rows <= 0) {
        tqkv::raise_empty_grid_error(stream);
        return;
    }
    if (!aligned16(dXq) || !aligned16(dY)) die_misaligned("launch_kv_reconstruct");
    finish("launch_kv_reconstruct",
           tqkv::launch_reconstruct(dXq, dScales, dY, rows, D, block_size, stream));
}

void launch_decode_attn_baseline(const __half* dQ, const __half* dK, const __half* dV, __half* dO,
                                 int B, int H, int S, int D, cudaStream_t stream) {
    if (D != 64 && D != 128) {
        std::fprintf(stderr, "launch_decode_attn_baseline: D must be 64 or 128 (got %d)\n", D);
        std::abort();
    }
    attention("launch_decode_attn_baseline", tqkv::KvKind::kHalf, dQ, dK, nullptr, dV, nullptr,
              dO, B, H, S, D, D, /*online=*/false, stream);
}

void launch_decode_attn_int8_fused(const __half* dQ, const int8_t* dKq, const __half* dKs,
                                   const int8_t* dVq, const __half* dVs, __half* dO, int B, int H,
                                   int S, int D, int block_size, cudaStream_t stream) {
    if (!tqkv::is_supported_int8(D, block_size)) {
        std::fprintf(stderr,
                     "launch_decode_attn_int8_fused: unsupported (D=%d, block_size=%d). "
                     "Supported: D in {64,128}, block_size in {32,64,128}, block_size <= D.\n",
                     D, block_size);
        std::abort();
    }
    attention("launch_decode_attn_int8_fused", tqkv::KvKind::kInt8, dQ, dKq, dKs, dVq, dVs, dO, B,
              H, S, D, block_size, /*online=*/false, stream);
}

void launch_decode_attn_int8_fused_online(const __half* dQ, const int8_t* dKq, const __half* dKs,
                                          const int8_t* dVq, const __half* dVs, __half* dO, int B,
                                          int H, int S, int D, int block_size,
                                          int lanes_per_thread, int tile_n, cudaStream_t stream) {
    // accepted set of the reference dispatcher
    bool ok = false;
    if (D == 128 && (lanes_per_thread == 2 || lanes_per_thread == 4) &&
        (tile_n == 32 || tile_n == 64))
        ok = block_size == 32 || block_size == 64 || block_size == 128;
    else if (D == 64 && lanes_per_thread == 2 && (tile_n == 32 || tile_n == 64))
        ok = block_size == 32 || block_size == 64;
    if (!ok) {
        std::fprintf(stderr,
                     "launch_decode_attn_int8_fused_online: unsupported "
                     "(D=%d, block_size=%d, L=%d, T=%d)\n",
                     D, block_size, lanes_per_thread, tile_n);
        std::abort();
    }
    attention("launch_decode_attn_int8_fused_online", tqkv::KvKind::kInt8, dQ, dKq, dKs, dVq,
              dVs, dO, B, H, S, D, block_size, /*online=*/true, stream);
}
