/* Allocation-free split-KV decode attention, callable from C.
 *
 * This entry point has no counterpart in the reference: the reference (and
 * the regular minisgl.ops.decode_attention path) takes its split-KV scratch
 * from the caller, who allocates it with the framework's allocator. Some
 * callers cannot allocate device memory at all: code that runs inside an
 * allocator or memory-pool callback, a host thread that must not take the
 * allocator's lock, or an embedding runtime that owns every device byte and
 * forbids cudaMalloc. They can call this function instead. It calls no
 * cudaMalloc, cudaFree or other allocating routine (no torch either): its
 * scratch is a fixed array in device global memory that is part of the
 * loaded library.
 *
 * Scratch limit: the partial outputs and log-sum-exp values of one call,
 *   B * hq * max_splits * (d + 1) * 4 bytes (+ 256 bytes of alignment),
 * must fit in MINISGL_NOALLOC_SCRATCH_BYTES (8 MiB). For Qwen3-style heads
 * (hq = 16, d = 128) with 16 splits that is up to 63 requests per call; with
 * max_splits = 1 no scratch is used and any batch size is accepted.
 *
 * Shared state: every call, on every stream and every host thread, uses the
 * same scratch array of the current device, which keeps the contents of the
 * last call. Calls whose kernels overlap on the GPU (different streams, or
 * concurrent graph branches) race on it and produce wrong results; serialise
 * them (one stream, or events). Nothing in the scratch has to start at zero:
 * every partial row the merge step reads is written earlier in the same call.
 *
 * Set-up: the first call on each device (with that device current) looks up
 * the scratch array's device address with cudaGetSymbolAddress and sets the
 * kernel's shared-memory limit; make that first call before any stream
 * capture begins.
 *
 * Return value: 0 on success, otherwise one of the codes below; when `msg`
 * is not NULL a one-line reason is written to it (at most msg_len bytes,
 * NUL-terminated).
 */
#ifndef MINISGL_NOALLOC_H_
#define MINISGL_NOALLOC_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MINISGL_NOALLOC_SCRATCH_BYTES (8u << 20)

#define MINISGL_NOALLOC_OK 0
#define MINISGL_NOALLOC_EINVAL 1      /* unsupported shape, layout or pointer */
#define MINISGL_NOALLOC_ETOOLARGE 2   /* scratch needed exceeds MINISGL_NOALLOC_SCRATCH_BYTES */
#define MINISGL_NOALLOC_ECUDA 3       /* a CUDA runtime call failed (set-up or launch) */

/* One decode step of paged attention (one query token per request), the
 * same computation as minisgl.ops.decode_attention.
 *
 *   out        bf16 [B, hq * d], contiguous
 *   q          bf16 [B, >= hq * d], row stride ld_q elements (the q heads
 *              may sit at the start of a fused qkv row)
 *   kv_pool    bf16 [2, num_layers, num_pages, hk, page_size, d], contiguous
 *   layer      layer index into the pool
 *   page_table int32 [rows, ld_pt] (ld_pt >= 1): token slot (page * page_size + offset)
 *              of every position of a request's row
 *   req_rows   int32 [B]: page-table row of each request
 *   seq_lens   int32 [B]: key count of each request (>= 1)
 *   max_splits 1..16 key-range splits per (request, kv head)
 *   err        device int32[2] error word (first error code, location); may
 *              be NULL. Bounded waits inside the kernel report here.
 *   stream     cudaStream_t to launch on (NULL = legacy default stream)
 * Requirements: d == 128, hq % hk == 0, hq / hk <= 16, page_size a power of
 * two >= 16, q / out / kv_pool 16-byte aligned, ld_q a multiple of 8.
 */
int minisgl_decode_attention_noalloc(void* out, const void* q, int ld_q, const void* kv_pool,
                                     int num_layers, int num_pages, int layer,
                                     const int32_t* page_table, int ld_pt, const int32_t* req_rows,
                                     const int32_t* seq_lens, int B, int hq, int hk, int d,
                                     int page_size, float scale, int max_splits, int* err,
                                     void* stream, char* msg, size_t msg_len);

#ifdef __cplusplus
}
#endif

#endif /* MINISGL_NOALLOC_H_ */
