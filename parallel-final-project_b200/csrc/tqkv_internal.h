// tqkv_internal.h — C++ entry points shared by the C ABI (tqkv_capi.cu) and
// the reference-signature shims (ref_launchers.cpp).  Not installed.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime_api.h>

#include "tqkv.h"

namespace tqkv {

enum class KvKind : int { kInt8 = 0, kHalf = 1 };
enum class OutKind : int { kHalfO = 0, kPartial = 1, kPeers = 2, kExchange = 3 };

// Records `err` as this host thread's last CUDA error and returns
// TQKV_ERR_CUDA, or returns TQKV_OK for cudaSuccess.
tqkv_status from_cuda(cudaError_t err);

bool is_supported_int8(int D, int block_size);

// Kernel launches with all checks done by the caller except alignment.
// T > 0: the rows are T new tokens per head, written to rows [t0, t0 + T) of a
// cache holding S_cap rows per head; T <= 0: whole tensors, in place.
tqkv_status launch_compress(const void* x, int8_t* xq, void* scales, long long rows, int D,
                            int block_size, cudaStream_t stream, int T = 0, int S_cap = 0,
                            int t0 = 0);
tqkv_status launch_reconstruct(const int8_t* xq, const void* scales, void* y, long long rows,
                               int D, int block_size, cudaStream_t stream);
// The newest T rows of every head, given in fp16 ([BH][T][D] each), that a
// fused decode quantises into rows [S - T, S) of the INT8 cache before
// attending over them.
struct AppendRows {
    const void* k_new;
    const void* v_new;
    int T;
};

// S rows attended per head; S_stride rows between heads in memory (0: S).
// With `append`, K/V/scales are the cache the new rows are written into.
// `group` query heads share one K/V head (BH counts query heads; K/V hold
// BH / group heads); fused append needs group == 1.
tqkv_status launch_decode(KvKind kv, OutKind out, const void* q, const void* k, const void* ks,
                          const void* v, const void* vs, void* o, int BH, int S, int D,
                          int block_size, void* workspace, size_t workspace_bytes,
                          cudaStream_t stream, int S_stride = 0,
                          const AppendRows* append = nullptr, int group = 1);
tqkv_status launch_fill_half(void* o, long long n, uint16_t bits, cudaStream_t stream);
tqkv_status launch_empty_partials(float* p, long long heads, int D, cudaStream_t stream);

// Workspace bytes the decode kernels need for (BH, S, D) on the current device.
size_t decode_workspace_bytes(long long BH, int S, int D);

// Per-(device, stream) grow-only workspace used by the reference-signature
// launchers, which have no workspace argument (ws_cache.h).  Zero-filled on
// allocation (the kernels keep it zeroed); a buffer once handed out is never
// freed, so a launch enqueued after another thread grew the cache still runs
// on valid memory.  Mutex-guarded; returns nullptr on failure.
void* cached_workspace(cudaStream_t stream, size_t bytes, tqkv_status* status);

// Sets cudaErrorInvalidConfiguration as the pending launch error, exactly as
// a <<<0, ...>>> launch in the reference does for an empty grid.
void raise_empty_grid_error(cudaStream_t stream);

}  // namespace tqkv
