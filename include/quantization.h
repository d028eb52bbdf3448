// quantization.h — KV compression launchers with the reference's exact C++
// signatures (reference include/quantization.h:15-27).
//
// Layout shared by K and V:
//   X      : __half  [B, H, S, D]
//   Xq     : int8_t  [B, H, S, D]
//   scales : __half  [B, H, S, D / block_size]
// Accepted: D in {64, 128}; block_size in {32, 64, 128}; D % block_size == 0.
// Anything else prints a message and calls std::abort(), as the reference.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

// Kernel A; replaces reference src/kv_compress.cu:111-136.
void launch_kv_compress(
    const __half* dX, int8_t* dXq, __half* dScales,
    int B, int H, int S, int D, int block_size,
    cudaStream_t stream);

// Kernel B; replaces reference src/kv_reconstruct.cu:38-62.
void launch_kv_reconstruct(
    const int8_t* dXq, const __half* dScales, __half* dY,
    int B, int H, int S, int D, int block_size,
    cudaStream_t stream);
