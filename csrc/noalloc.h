// Allocation-free C entry point for split-KV decode attention.
//
// This entry point has no counterpart in the reference implementation; it is
// an addition of this library.
//
// Who it is for: callers that cannot allocate device memory themselves --
// for example a host runtime that owns every device allocation through its
// own arena, a plugin called from a language or framework with no CUDA
// allocator binding, or code that must not introduce allocations into a
// region its caller is about to record. They pass device pointers for the
// inputs and the output; the temporary partial results of the split-KV
// reduction live in a fixed-size array in this library's device memory.
//
// Limits and behaviour:
//  * scratch capacity: AFD_NOALLOC_SCRATCH_BYTES (8 MiB) per GPU, held by
//    every GPU that loads the library until process exit. A call with
//    n_split > 1 needs batch * n_q_heads * n_split * (head_dim + 2) * 4 bytes
//    of it; calls that need more are rejected with AFD_NOALLOC_ERR_TOO_LARGE
//    before anything runs. n_split == 1 uses no scratch.
//  * the first call on a device (with that device current) looks up the
//    device address of the scratch array; make that first call before any
//    stream capture.
//  * every call shares the one scratch array. Calls whose kernels can
//    overlap on the GPU (different streams without ordering) race on it;
//    order them on one stream or with events. No part of the scratch must
//    start zeroed: each call overwrites every slot it reads.
//  * no cudaMalloc, cudaFree or allocating library routine is called.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AFD_NOALLOC_SCRATCH_BYTES (8u << 20)

enum {
  AFD_NOALLOC_OK = 0,
  AFD_NOALLOC_ERR_TOO_LARGE = 1,      // scratch need exceeds AFD_NOALLOC_SCRATCH_BYTES
  AFD_NOALLOC_ERR_BAD_ARG = 2,        // null pointer, bad shape or unsupported head layout
  AFD_NOALLOC_ERR_SYMBOL = 3,         // cudaGetSymbolAddress failed on this device
  AFD_NOALLOC_ERR_LAUNCH = 4,         // the kernel launch itself failed
  AFD_NOALLOC_ERR_PENDING = 5,        // an earlier CUDA error was pending; nothing launched
};

// Device-side code written to `status[0]` when *start_pos lies outside
// [0, max_seq): the kernel then reads no key and writes zeros to `out`.
#define AFD_NOALLOC_STATUS_BAD_POSITION 3

// Decode attention (one query token per sequence) over a KV cache laid out
// [max_batch, n_kv_heads, max_seq, head_dim] (bf16), for the sequences in
// cache rows batch_offset .. batch_offset + batch - 1, attending to positions
// 0 .. *start_pos (device int32). q and out are [batch, n_q_heads, head_dim]
// bf16. n_split >= 1 key-range splits per (sequence, kv head). Launches on
// `stream`. Returns an AFD_NOALLOC_* code.
//
// Preconditions:
//  * batch_offset + batch <= max_batch (checked on the host: BAD_ARG);
//  * supported head layouts: (n_q_heads / n_kv_heads, head_dim) in
//    {(8, 128), (4, 128), (8, 64), (2, 64)} (checked on the host: BAD_ARG);
//  * 0 <= *start_pos < max_seq. The value lives on the device, so it is
//    checked by the kernel: outside that range nothing is read from the
//    cache, `out` gets zeros, and AFD_NOALLOC_STATUS_BAD_POSITION is written
//    to status[0] (with a call-site number in status[1]) when `status` is
//    given. `status` is optional (may be null), a device int32[2] that the
//    caller zeroes; the first error recorded in it is kept.
__attribute__((visibility("default"))) int afd_decode_attention_noalloc(
    const void* q, const void* k_cache, const void* v_cache, void* out, const int* start_pos,
    int* status, int batch, int n_q_heads, int n_kv_heads, int head_dim, int max_batch,
    int max_seq, int batch_offset, int n_split, cudaStream_t stream);

// Human-readable text of a return code.
__attribute__((visibility("default"))) const char* afd_noalloc_error_string(int code);

#ifdef __cplusplus
}
#endif
