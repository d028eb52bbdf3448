/*
 * tqkv.h — C ABI of the B200 INT8 KV-cache decode path.
 *
 * Plain C: every argument is a pointer, a size or a stream; every entry point
 * returns a tqkv_status and never aborts.  The C++ launchers that keep the
 * reference's exact signatures (attention.h, quantization.h) are thin shims
 * over these functions.
 *
 * Layouts (identical to the reference, quantization.h:5-12 of the reference):
 *   Q, O       : fp16 [B, H, D]
 *   K, V       : fp16 [B, H, S, D]
 *   Kq, Vq     : int8 [B, H, S, D]
 *   Ks, Vs     : fp16 [B, H, S, D / block_size]
 * fp16 tensors are passed as `void*` / `const void*` holding IEEE binary16.
 *
 * All device pointers are owned by the caller.  All launches are
 * asynchronous on `stream`.
 *
 * Alignment contract: Kq, Vq, K and V (and the fp16 rows of new tokens given
 * to the append entry points) must be 16-byte aligned (cudaMalloc and torch
 * allocations are 256-byte aligned).  Q, O, scale arrays and partials need
 * only their natural alignment.
 */
#ifndef TQKV_H_
#define TQKV_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum tqkv_status {
    TQKV_OK = 0,
    /* D / block_size / lanes / tile outside the set the reference accepts */
    TQKV_ERR_UNSUPPORTED = 1,
    /* B, H or S negative or zero where the operation has no defined result,
       or an element count that overflows */
    TQKV_ERR_INVALID_SIZE = 2,
    /* a pointer that must be 16-byte aligned is not */
    TQKV_ERR_MISALIGNED = 3,
    /* workspace pointer null or smaller than tqkv_decode_workspace_bytes() */
    TQKV_ERR_WORKSPACE = 4,
    /* a CUDA runtime call failed; tqkv_last_cuda_error() names it */
    TQKV_ERR_CUDA = 5,
    /* a required pointer is null */
    TQKV_ERR_NULL = 6
} tqkv_status;

/* Human-readable name of a status. */
const char* tqkv_status_string(tqkv_status s);

/* The cudaError_t (as int) behind the most recent TQKV_ERR_CUDA on this host
   thread, 0 if none. */
int tqkv_last_cuda_error(void);

/* Library version string, e.g. "tqkv-b200 0.1.0 sm_100a". */
const char* tqkv_version(void);

/* ------------------------------------------------------------------------ */
/* Kernel A — blockwise symmetric FP16 -> INT8 compression.
 *
 * Replaces launch_kv_compress (reference include/quantization.h:15-20,
 * src/kv_compress.cu:111-136).  Per token row and per block of `block_size`
 * lanes along D: m = max|x|, s = m / 127 (s = 1 when m == 0), the fp16 scale
 * is fp16(s) rounded to nearest-even, and each code is
 * round-half-even(x / s) clamped to [-127, 127] — with the fp32 s, not the
 * fp16 one (reference src/kv_compress.cu:81-95).  The divisions use the same
 * fast-math division the reference is built with (CMakeLists.txt:21), so codes
 * and scales are bit-identical to the reference build.
 *
 * Accepted: D in {64, 128}; block_size in {32, 64, 128}; block_size <= D.
 */
tqkv_status tqkv_kv_compress(const void* x, int8_t* xq, void* scales,
                             int B, int H, int S, int D, int block_size,
                             cudaStream_t stream);

/* Kernel B — y = fp16(float(code) * float(scale)).
 * Replaces launch_kv_reconstruct (reference include/quantization.h:22-27,
 * src/kv_reconstruct.cu:10-34).  Same accepted set as tqkv_kv_compress. */
tqkv_status tqkv_kv_reconstruct(const int8_t* xq, const void* scales, void* y,
                                int B, int H, int S, int D, int block_size,
                                cudaStream_t stream);

/* Incremental append (the step before attention in a decoder; no counterpart
 * in the reference, whose compress takes whole tensors).  Quantises T new
 * tokens per head, x = fp16 [B, H, T, D], into rows [t0, t0 + T) of an INT8
 * cache with room for S_cap rows per head: cache_q int8 [B, H, S_cap, D],
 * cache_s fp16 [B, H, S_cap, D / block_size].  Codes and scales are those
 * tqkv_kv_compress gives for the same rows (same rule, same division).
 * Requires 0 <= t0 and t0 + T <= S_cap; x and cache_q 16-byte aligned. */
tqkv_status tqkv_kv_append(const void* x, int8_t* cache_q, void* cache_s,
                           int B, int H, int T, int D, int block_size,
                           int S_cap, int t0, cudaStream_t stream);

/* ------------------------------------------------------------------------ */
/* Decode attention: O[b,h,:] = softmax(q . K^T / sqrt(D)) . V per (b, h).
 *
 * The B*H*S token rows are cut into fixed chunks: one per CTA, or, for very
 * long runs per CTA, about eight per CTA claimed from a counter in
 * `workspace`.  A head that spans several chunks leaves one record per piece
 * in `workspace`; CTAs that have no chunk left merge them (log-sum-exp, in
 * piece order: results do not depend on which CTA streamed which chunk).
 * Size the workspace with
 * tqkv_decode_workspace_bytes() and zero it once with tqkv_workspace_init()
 * before its first use; every decode call leaves it zeroed again (after a
 * device error, zero it again).  Calls that share one workspace must be
 * ordered (same stream, or events).
 *
 * Every decode launch is a programmatic dependent
 * (cudaLaunchAttributeProgrammaticStreamSerialization): its CTAs may be
 * dispatched while the previous kernel in the stream is finishing, and each
 * waits for it (griddepcontrol.wait) before touching global memory, so
 * stream order holds as for a plain launch.  Before that wait a CTA only
 * asks L2 to prefetch the first K and V rows it is likely to stream.
 */
size_t tqkv_decode_workspace_bytes(int B, int H, int S, int D);

/* The decode kernels' work split for BH heads of S rows with at most
 * `max_ctas` CTAs (the device's SMs x resident CTAs per SM): the grid, the
 * chunk size in rows, the number of chunks, and the most pieces a head can be
 * cut into.  Host-only (no device is touched); for capacity planning and
 * tests. */
tqkv_status tqkv_decode_plan(long long BH, int S, int max_ctas, long long* grid,
                             long long* chunk_rows, long long* nchunks, long long* max_parts);

tqkv_status tqkv_workspace_init(void* workspace, size_t workspace_bytes,
                                cudaStream_t stream);

/* Kernel D — fused INT8 decode with single-pass online softmax.
 * Replaces launch_decode_attn_int8_fused_online (reference
 * include/attention.h:28-35, src/attention_int8_fused_online.cu:16-239) and
 * launch_decode_attn_int8_fused (attention.h:17-23,
 * src/attention_int8_fused.cu:18-191): both compute the same function.
 * Accepted: D in {64, 128}; block_size in {32, 64, 128}; block_size <= D.
 * S == 0 writes NaN to O (what the reference online kernel yields). */
tqkv_status tqkv_decode_int8(const void* q,
                             const int8_t* kq, const void* ks,
                             const int8_t* vq, const void* vs,
                             void* o,
                             int B, int H, int S, int D, int block_size,
                             void* workspace, size_t workspace_bytes,
                             cudaStream_t stream);

/* tqkv_decode_int8 over the first S rows of each head of caches that hold
 * S_cap >= S rows per head (the layout tqkv_kv_append fills):
 * kq/vq int8 [B, H, S_cap, D], ks/vs fp16 [B, H, S_cap, D / block_size].
 * Workspace as for tqkv_decode_int8 with the same B, H, S, D. */
tqkv_status tqkv_decode_int8_cache(const void* q,
                                   const int8_t* kq, const void* ks,
                                   const int8_t* vq, const void* vs,
                                   void* o,
                                   int B, int H, int S, int S_cap, int D, int block_size,
                                   void* workspace, size_t workspace_bytes,
                                   cudaStream_t stream);

/* Append fused into decode (no counterpart in the reference, whose drivers
 * compress whole tensors and then attend).  Equivalent to
 *   tqkv_kv_append(k_new, kq, ks, B, H, T, D, block_size, S_cap, S - T);
 *   tqkv_kv_append(v_new, vq, vs, ...same...);
 *   tqkv_decode_int8_cache(q, kq, ks, vq, vs, o, B, H, S, S_cap, D, ...);
 * in one launch: the T newest tokens of each head, k_new / v_new fp16
 * [B, H, T, D], are quantised (same codes and scales as tqkv_kv_compress) by
 * the CTA whose tile holds them, written to rows [S - T, S) of the caches and
 * attended from shared memory without being read back.  Rows [0, S - T) must
 * already hold codes.  Requires 1 <= T <= S <= S_cap; k_new, v_new, kq and vq
 * 16-byte aligned.  Workspace as for tqkv_decode_int8 with the same B, H, S, D. */
tqkv_status tqkv_decode_int8_append(const void* q, const void* k_new, const void* v_new,
                                    int8_t* kq, void* ks, int8_t* vq, void* vs,
                                    void* o,
                                    int B, int H, int T, int S, int S_cap, int D,
                                    int block_size,
                                    void* workspace, size_t workspace_bytes,
                                    cudaStream_t stream);

/* Grouped-query / multi-query attention (no counterpart in the reference,
 * whose K/V have one head per query head).  q and o are [B, H_q, D]; kq/vq
 * int8 [B, H_kv, S, D] and ks/vs fp16 [B, H_kv, S, D / block_size], with
 * H_q a multiple of H_kv: query head h attends over K/V head h / (H_q / H_kv)
 * (MQA: H_kv = 1).  The result equals tqkv_decode_int8 on K/V whose heads
 * are repeated H_q / H_kv times.  Query heads that share a K/V head run on
 * neighbouring CTAs, so their K/V reads meet in L2.  Workspace:
 * tqkv_decode_workspace_bytes(B, H_q, S, D). */
tqkv_status tqkv_decode_int8_gqa(const void* q,
                                 const int8_t* kq, const void* ks,
                                 const int8_t* vq, const void* vs,
                                 void* o,
                                 int B, int H_q, int H_kv, int S, int D, int block_size,
                                 void* workspace, size_t workspace_bytes,
                                 cudaStream_t stream);

/* FP16 decode attention on the same split-S skeleton.
 * Replaces launch_decode_attn_baseline (reference include/attention.h:6-12,
 * src/attention_baseline.cu:11-155) without its S <= ~12k shared-memory cap.
 * Accepted: D in {64, 128}.  S == 0 writes 0 to O (as the reference). */
tqkv_status tqkv_decode_fp16(const void* q, const void* k, const void* v,
                             void* o, int B, int H, int S, int D,
                             void* workspace, size_t workspace_bytes,
                             cudaStream_t stream);

/* ------------------------------------------------------------------------ */
/* Split-S decode across devices (no counterpart in the reference, which has
 * no multi-GPU path).  Each device holds a slice [s0, s0 + S) of the tokens
 * of every head and calls tqkv_decode_int8_partial on it; the partial record
 * of head i is `partial + i * (D + 2)` floats laid out as
 *     acc[0..D-1]  = sum_t exp(s_t - m) * v_t      (un-normalised)
 *     acc[D]       = m = max_t s_t                  (natural-log units)
 *     acc[D + 1]   = l = sum_t exp(s_t - m)
 * with s_t = q . k_t / sqrt(D).  The records of R devices, gathered into
 * [R][B*H][D + 2], are merged by tqkv_lse_combine into O.  S may be 0 for a
 * device that holds no tokens (its record is m = -inf, l = 0, acc = 0). */
tqkv_status tqkv_decode_int8_partial(const void* q,
                                     const int8_t* kq, const void* ks,
                                     const int8_t* vq, const void* vs,
                                     float* partial,
                                     int B, int H, int S, int D, int block_size,
                                     void* workspace, size_t workspace_bytes,
                                     cudaStream_t stream);

tqkv_status tqkv_lse_combine(const float* partials, void* o,
                             int R, int BH, int D, cudaStream_t stream);

/* ------------------------------------------------------------------------ */
/* Split-S decode across the GPUs of one node over NVLink, without NCCL (no
 * counterpart in the reference, which has no multi-GPU path).
 *
 * Every rank allocates one exchange buffer (tqkv_exchange_alloc, size
 * tqkv_exchange_bytes(world, B*H, D)), exports it with tqkv_ipc_get_handle,
 * and maps every other rank's buffer with tqkv_ipc_open_handle (plain CUDA
 * IPC peer mappings; no multicast objects).  `exchange_bufs[r]` is rank r's
 * buffer as mapped in the calling process.  Per decode step, on each rank's
 * stream:
 *   tqkv_decode_int8_publish  computes this rank's per-head records
 *       (acc[D], m, l) over its token slice and stores them into every rank's
 *       buffer through the peer mappings; each value travels with the step
 *       number in one 64-bit store, so no fence or flag is needed (S == 0:
 *       empty records, m = -inf, l = 0, acc = 0);
 *   tqkv_exchange_combine     waits (bounded, ~1 s) until every rank's
 *       entries of this step have arrived in this rank's buffer, merges them
 *       into O and advances this rank's step counter.
 * Steps alternate between two record slots, so a rank can run one step ahead
 * of another without overwriting records still being read.  Buffers must be
 * zero when first used (tqkv_exchange_alloc zeroes them) and stay in use for
 * the whole sequence of steps.  An entry that never arrives sets the device
 * error flag (tqkv_read_device_error) instead of hanging.  world <= 8. */
size_t tqkv_exchange_bytes(int world, int BH, int D);
tqkv_status tqkv_exchange_alloc(size_t bytes, void** buf_out);
tqkv_status tqkv_exchange_free(void* buf);
/* 64-byte CUDA IPC handle of an exchange buffer, and its mapping in another process. */
tqkv_status tqkv_ipc_get_handle(const void* buf, void* handle_out);
tqkv_status tqkv_ipc_open_handle(const void* handle, void** buf_out);
tqkv_status tqkv_ipc_close_handle(void* buf);

tqkv_status tqkv_decode_int8_publish(const void* q,
                                     const int8_t* kq, const void* ks,
                                     const int8_t* vq, const void* vs,
                                     int B, int H, int S, int D, int block_size,
                                     void* workspace, size_t workspace_bytes,
                                     void* const* exchange_bufs, int world, int rank,
                                     cudaStream_t stream);
/* tqkv_decode_int8_publish with the fused append of tqkv_decode_int8_append:
 * the rank that holds the end of the sequence appends the T newest tokens
 * at rows [S - T, S) of its slice (a cache of S_cap rows per head). */
tqkv_status tqkv_decode_int8_append_publish(const void* q,
                                            const void* k_new, const void* v_new,
                                            int8_t* kq, void* ks, int8_t* vq, void* vs,
                                            int B, int H, int T, int S, int S_cap, int D,
                                            int block_size,
                                            void* workspace, size_t workspace_bytes,
                                            void* const* exchange_bufs, int world, int rank,
                                            cudaStream_t stream);
tqkv_status tqkv_exchange_combine(void* const* exchange_bufs, void* o,
                                  int world, int rank, int BH, int D, cudaStream_t stream);

/* One split-S decode step in ONE launch: the work of tqkv_decode_int8_publish
 * followed by that of tqkv_exchange_combine, O (fp16 [B,H,D]) out.  After its
 * share of the token slice, each CTA takes heads from a counter in the
 * workspace, waits (bounded, ~1 s) for every rank's records of the head,
 * merges them and writes O; the last CTA to finish advances this rank's step
 * counter.  Same O as the two-launch pair, bit for bit, with the same buffers
 * and record slots: a sequence of steps may use either form, step by step.  S == 0 (a rank whose
 * slice is empty) publishes empty records and merges with two small launches.
 * A wait that runs out leaves NaN in that head's O and sets the device error
 * flag; after a device error, re-zero the workspace (tqkv_workspace_init) and
 * the exchange buffers before further steps. */
tqkv_status tqkv_decode_int8_exchange(const void* q,
                                      const int8_t* kq, const void* ks,
                                      const int8_t* vq, const void* vs,
                                      void* o,
                                      int B, int H, int S, int D, int block_size,
                                      void* workspace, size_t workspace_bytes,
                                      void* const* exchange_bufs, int world, int rank,
                                      cudaStream_t stream);
/* tqkv_decode_int8_exchange with the fused append of tqkv_decode_int8_append
 * (rows [S - T, S) of a cache of S_cap rows per head; T >= 1). */
tqkv_status tqkv_decode_int8_append_exchange(const void* q,
                                             const void* k_new, const void* v_new,
                                             int8_t* kq, void* ks, int8_t* vq, void* vs,
                                             void* o,
                                             int B, int H, int T, int S, int S_cap, int D,
                                             int block_size,
                                             void* workspace, size_t workspace_bytes,
                                             void* const* exchange_bufs, int world, int rank,
                                             cudaStream_t stream);

/* ------------------------------------------------------------------------ */
/* INT8 decode for callers that cannot allocate device memory.
 * No counterpart in the reference.
 *
 * Who needs it: code that may not call cudaMalloc (or any allocator) on the
 * path where it runs decode — an inference runtime whose memory planner owns
 * every device buffer and forbids allocations inside an operator, a plugin
 * host that hands a plugin its inputs and outputs but no allocator, or a thin
 * FFI binding with no device allocator of its own.  tqkv_decode_int8 needs a
 * caller-provided workspace for heads that are split across CTAs; this
 * variant instead uses a fixed scratch array of TQKV_NOALLOC_SCRATCH_BYTES
 * compiled into the library, present on every GPU that loads the library
 * until the process exits.  The caller still provides q, K/V codes and
 * scales, and O.  Same arguments, accepted set and results as
 * tqkv_decode_int8, without the workspace pair.
 *
 * Limits and rules:
 *   - shapes whose scratch (tqkv_decode_workspace_bytes) exceeds
 *     TQKV_NOALLOC_SCRATCH_BYTES are refused with TQKV_ERR_WORKSPACE;
 *   - the first call on a device looks up the array's device address (and
 *     may load the library's device code); make that first call before any
 *     stream capture;
 *   - all calls on a device share the one array: calls that can overlap on
 *     the GPU (different streams, or unordered host threads) race and must be
 *     ordered by the caller;
 *   - the array's address is looked up once per device and kept for the life
 *     of the process: after cudaDeviceReset (which unloads the library's
 *     device code) this entry point must not be called again.
 * Nothing is allocated: no cudaMalloc/cudaFree and no allocating library
 * routine; each call clears the part of the array its shape uses (counters
 * and the records of split heads) with a memset on `stream` before
 * launching. */
#define TQKV_NOALLOC_SCRATCH_BYTES (4u * 1024u * 1024u)

tqkv_status tqkv_decode_int8_noalloc(const void* q,
                                     const int8_t* kq, const void* ks,
                                     const int8_t* vq, const void* vs,
                                     void* o,
                                     int B, int H, int S, int D, int block_size,
                                     cudaStream_t stream);

/* ------------------------------------------------------------------------ */
/* Device-side failure flag.  Every wait inside the kernels is bounded; a wait
 * that runs out records a nonzero code here (and the kernel returns early)
 * instead of hanging the GPU.  Reads and clears the flag of the current
 * device (synchronous). */
tqkv_status tqkv_read_device_error(uint32_t* code_out);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* TQKV_H_ */
