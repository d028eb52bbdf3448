// ref_shim.cpp — TEST INFRASTRUCTURE ONLY.
//
// extern "C" wrappers around the reference's own launchers, linked with the
// reference's unmodified kernel sources into oracle/_ref/libtqkv_ref.so by
// oracle/Makefile.  The GPU parity tests call these to compare the B200
// kernels with the reference kernels (built for sm_100a with the reference's
// flags, -O3 --use_fast_math) on identical device buffers.  The declarations
// come from the reference's own headers (include/attention.h,
// include/quantization.h of the reference project).
#include "attention.h"
#include "quantization.h"

extern "C" {

void ref_kv_compress(const void* x, void* xq, void* scales, int B, int H, int S, int D, int bs,
                     void* stream) {
    launch_kv_compress(static_cast<const __half*>(x), static_cast<int8_t*>(xq),
                       static_cast<__half*>(scales), B, H, S, D, bs,
                       static_cast<cudaStream_t>(stream));
}

void ref_kv_reconstruct(const void* xq, const void* scales, void* y, int B, int H, int S, int D,
                        int bs, void* stream) {
    launch_kv_reconstruct(static_cast<const int8_t*>(xq), static_cast<const __half*>(scales),
                          static_cast<__half*>(y), B, H, S, D, bs,
                          static_cast<cudaStream_t>(stream));
}

void ref_decode_fp16(const void* q, const void* k, const void* v, void* o, int B, int H, int S,
                     int D, void* stream) {
    launch_decode_attn_baseline(static_cast<const __half*>(q), static_cast<const __half*>(k),
                                static_cast<const __half*>(v), static_cast<__half*>(o), B, H, S, D,
                                static_cast<cudaStream_t>(stream));
}

void ref_decode_int8_fused(const void* q, const void* kq, const void* ks, const void* vq,
                           const void* vs, void* o, int B, int H, int S, int D, int bs,
                           void* stream) {
    launch_decode_attn_int8_fused(static_cast<const __half*>(q), static_cast<const int8_t*>(kq),
                                  static_cast<const __half*>(ks), static_cast<const int8_t*>(vq),
                                  static_cast<const __half*>(vs), static_cast<__half*>(o), B, H, S,
                                  D, bs, static_cast<cudaStream_t>(stream));
}

void ref_decode_int8_online(const void* q, const void* kq, const void* ks, const void* vq,
                            const void* vs, void* o, int B, int H, int S, int D, int bs, int lanes,
                            int tile, void* stream) {
    launch_decode_attn_int8_fused_online(
        static_cast<const __half*>(q), static_cast<const int8_t*>(kq),
        static_cast<const __half*>(ks), static_cast<const int8_t*>(vq),
        static_cast<const __half*>(vs), static_cast<__half*>(o), B, H, S, D, bs, lanes, tile,
        static_cast<cudaStream_t>(stream));
}

int ref_last_error(void) { return static_cast<int>(cudaGetLastError()); }

}  // extern "C"
