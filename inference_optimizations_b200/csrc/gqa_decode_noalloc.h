// Allocation-free C entry point for the GQA split-K decode / verify attention kernel.
//
// This entry point has no counterpart in the reference.  It exists for callers that cannot allocate device memory on
// their own: an engine running inside a pre-sized memory arena (every byte budgeted at start-up), a plugin that is
// handed raw pointers by a host runtime with its own allocator, or code on a path where a cudaMalloc would
// synchronize the device or could fail under memory pressure.  The regular entry point (`iob::gqa_decode`) needs
// the caller to pass split-K scratch buffers; this one keeps that scratch in a fixed array compiled into the library
// instead, so the caller passes only inputs and outputs.
//
// Scratch: one file-scope device array per GPU, holding at most IOB_NOALLOC_MAX_PARTIAL_FLOATS fp32 partial outputs
// (4 MiB) and IOB_NOALLOC_MAX_PARTIAL_ROWS fp32 partial log-sum-exps (256 KiB), plus a status word.  Every GPU that
// loads the library keeps this memory until the process exits.
//
// Contract:
//   * Every call looks up the array's device address (cudaGetSymbolAddress) with the calling thread's current device
//     current; the first call on a device may initialize the module there, so make it outside any CUDA-graph stream
//     capture.  The address is not cached, so the entry point stays valid after a device reset.
//   * All calls on a device share the one array: calls that overlap on the GPU (different streams, or concurrent
//     graph replays) race on it.  Serialize them.
//   * A call whose split-K workspace would not fit returns IOB_NOALLOC_ETOOBIG and launches nothing.
//   * No call allocates or frees memory (no cudaMalloc / cudaFree / library allocator); the status word is cleared
//     with cudaMemsetAsync on the given stream.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define IOB_NOALLOC_MAX_PARTIAL_FLOATS (1 << 20)
#define IOB_NOALLOC_MAX_PARTIAL_ROWS (1 << 16)

#define IOB_NOALLOC_OK 0
#define IOB_NOALLOC_ETOOBIG (-1)   /* B * Hk * num_splits * rows * D exceeds the built-in scratch */
#define IOB_NOALLOC_EINVAL (-2)    /* bad argument (null pointer, unsupported shape) */
#define IOB_NOALLOC_ESETUP (-3)    /* device lookup or cudaGetSymbolAddress failed */

#ifdef __cplusplus
extern "C" {
#endif

// Same semantics as the allocating entry point: q bf16 [B * n_q, Hq, D] (normed + roped), pool = one layer's paged
// pool, page_table int32 [rows, pt_stride], req_idx int32 [B] (or null: row b), kv_len int32 [B], out bf16
// [B * n_q, Hq, D].  fmt: 0 bf16, 1 fp8, 2 nvfp4.  Returns IOB_NOALLOC_OK, one of the negative codes above, or a
// positive cudaError_t from the launch.
int iob_gqa_decode_noalloc(const void* q, const void* pool, const int* page_table, int pt_stride, const int* req_idx,
                           const int* kv_len, void* out, int B, int n_q, int Hq, int Hk, int D, int window, int fmt,
                           int tiles_per_split, int num_splits, float sm_scale, float k_scale, float v_scale,
                           int exact, cudaStream_t stream);

// The kernel's status word of the last call on the current device, read into *host_out after `stream` drained:
// 0 = ok; non-zero = a bounded wait inside the kernel gave up (its output is then not valid).  The decode call itself
// only reports launch errors, so a caller that needs to know whether the result is valid reads this after it.
// Returns IOB_NOALLOC_OK or an error code like the decode call.
int iob_gqa_decode_noalloc_status(int* host_out, cudaStream_t stream);

// Human-readable text for a return code of iob_gqa_decode_noalloc.
const char* iob_gqa_decode_noalloc_strerror(int code);

#ifdef __cplusplus
}
#endif
