// attention.h — decode-attention launchers with the reference's exact C++
// signatures (reference include/attention.h:6-35), so its tqkv_decode and
// tqkv_bench drivers link against this library unchanged.
//
// Each launcher validates the same (D, block_size, lanes, tile) set as the
// reference, prints the reference's message and calls std::abort() on an
// unsupported combination, and is asynchronous on `stream`.  All three run on
// the split-S kernels of the C ABI (tqkv.h); the split-S scratch they need
// comes from a per-(device, stream) cache that is allocated on first use.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

// FP16 decode attention; replaces reference src/attention_baseline.cu:133-155.
void launch_decode_attn_baseline(
    const __half* dQ, const __half* dK, const __half* dV, __half* dO,
    int B, int H, int S, int D,
    cudaStream_t stream);

// INT8 decode attention with in-register dequantisation; replaces reference
// src/attention_int8_fused.cu:161-191 (its two-pass softmax and S <= ~12k
// limit are gone; the output is the same function).
void launch_decode_attn_int8_fused(
    const __half* dQ,
    const int8_t* dKq, const __half* dKs,
    const int8_t* dVq, const __half* dVs,
    __half* dO,
    int B, int H, int S, int D, int block_size,
    cudaStream_t stream);

// INT8 decode attention, single-pass online softmax; replaces reference
// src/attention_int8_fused_online.cu:195-239.  lanes_per_thread and tile_n are
// checked against the reference's accepted set and otherwise ignored: the
// B200 kernel picks its own tiling.
void launch_decode_attn_int8_fused_online(
    const __half* dQ,
    const int8_t* dKq, const __half* dKs,
    const int8_t* dVq, const __half* dVs,
    __half* dO,
    int B, int H, int S, int D, int block_size,
    int lanes_per_thread, int tile_n,
    cudaStream_t stream);
