// Allocation-free entry point of the packed-varlen attention backward.
//
// This entry point has no counterpart in the reference project; it exists for callers of this
// library that must not allocate device memory while they run: code inside a CUDA-graph
// memory pool or an inference server with a fixed memory budget (where a cudaMalloc can fail
// or reshape the pool), plain C/C++ programs that link this library without PyTorch's caching
// allocator, and tools that replay kernels under strict memory accounting. It computes the
// same dQ/dK/dV as the PyTorch-facing `attn_bwd`, but its scratch (the per-row softmax
// correction `delta` and the per-token document end) lives in a fixed device array that is
// part of the library itself, so a call performs no cudaMalloc, cudaFree or allocating
// library call. The caller provides every input and output buffer.
//
// Limits and rules:
//  * The scratch array holds ME_ATTN_BWD_NOALLOC_SCRATCH_BYTES (8 MiB) on every GPU that loads
//    the library, for the life of the process. A call needs align256(Hq*T*4) + align256(T*4)
//    bytes of it; larger problems are rejected with ME_NOALLOC_ERR_TOO_LARGE (see
//    me_noalloc_last_error() for the message) and nothing is launched.
//  * The first call on a device looks up the array's device address (cudaGetSymbolAddress)
//    with that device current. Make that first call before any stream capture.
//  * Every call shares the one array: calls whose kernels overlap on the GPU (two streams, or
//    two host threads on one device) race on it. Serialize them.
//  * The array keeps the previous call's contents; every element a call reads is written by
//    that call first, so nothing needs clearing between calls.
//  * dout, q, k, v, o, dq, dk and dv must start on 16-byte boundaries (the kernels move them 16
//    bytes at a time) and lse and doc_start on 4-byte boundaries; other pointers are refused with
//    ME_NOALLOC_ERR_ARGS. doc_start must be non-decreasing (packed documents), as from doc_starts.
//  * A CUDA error already pending when the call starts (from earlier, unrelated work) is left
//    pending and reported as ME_NOALLOC_ERR_LAUNCH; nothing is launched then.
#pragma once

#include <cuda_runtime.h>

#define ME_ATTN_BWD_NOALLOC_SCRATCH_BYTES (8u << 20)

enum {
  ME_NOALLOC_OK = 0,
  ME_NOALLOC_ERR_ARGS = -1,       // a null or misaligned pointer, a bad size or an unsupported head_dim
  ME_NOALLOC_ERR_TOO_LARGE = -2,  // the problem needs more scratch than the fixed array holds
  ME_NOALLOC_ERR_SETUP = -3,      // cudaGetSymbolAddress failed on this device
  ME_NOALLOC_ERR_LAUNCH = -4,     // an earlier error was pending, a shared-memory opt-in or a launch failed
};

#ifdef __cplusplus
extern "C" {
#endif

// dq [T,Hq,D], dk/dv [T,Hk,D] (bf16, caller-allocated) from dout/o/q [T,Hq,D], k/v [T,Hk,D]
// (bf16), lse [Hq,T] (fp32, from the forward) and doc_start [T] (int32). window <= 0 means no
// sliding window. Work is enqueued on `stream`; returns ME_NOALLOC_OK or an error code.
int me_attn_bwd_noalloc(const void* dout, const void* q, const void* k, const void* v, const void* o,
                        const float* lse, const int* doc_start, int T, int Hq, int Hk, int D, int window,
                        float scale, void* dq, void* dk, void* dv, cudaStream_t stream);

// A static description of the last error of me_attn_bwd_noalloc on this thread.
const char* me_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
