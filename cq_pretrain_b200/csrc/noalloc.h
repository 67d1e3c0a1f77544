// Public C interface of the allocation-free causal-conv backward in cqb_kernels.so.
//
// This interface has no counterpart in the reference framework. It is for callers that cannot
// allocate device memory while they run the backward pass of the short convolution: hooks that
// run inside a caching allocator or memory pool (they cannot re-enter the allocator they belong
// to), C or C++ hosts that drive the kernels without PyTorch (they have no tensor allocator), and
// steps whose device memory was reserved once up front (a late cudaMalloc could fail or fragment
// the reserved pool). The caller passes every input and output buffer; the kernels' only scratch
// is a static device array of cqb_conv_bwd_noalloc_scratch_floats() floats (8 MiB) that every GPU
// which loads the library holds until the process exits.
//
// Contract (details at the definitions in conv.cu):
//   * ceil(n / 256) * C * 4 floats must fit in the scratch array (for C = 6144: n <= 21,760;
//     for C = 8192: n <= 16,384); larger inputs return CQB_NOALLOC_TOO_LARGE;
//   * the first call on a device, or cqb_conv_bwd_noalloc_init() with that device current, looks
//     up the array's device address; make that first call before any stream capture begins;
//   * every call on a device shares the array and it keeps the last call's contents: calls that
//     overlap on the GPU race on it, so serialise them on one stream or order them with events;
//   * no cudaMalloc, cudaFree or allocating library routine is called;
//   * on failure the return code is non-zero and cqb_noalloc_last_error() (per host thread)
//     describes it.
#pragma once

#include <stddef.h>

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

enum CqbNoAllocStatus {
  CQB_NOALLOC_OK = 0,
  CQB_NOALLOC_BAD_ARGUMENT = 1,   // null or misaligned pointer, C not a positive multiple of 8, ...
  CQB_NOALLOC_TOO_LARGE = 2,      // the partials would not fit in the static scratch array
  CQB_NOALLOC_CUDA_ERROR = 3,     // a CUDA call or launch failed, or an earlier CUDA error is pending
};

// Message of the last failed call on this host thread.
const char* cqb_noalloc_last_error(void);

// Capacity of the static scratch array, in floats.
size_t cqb_conv_bwd_noalloc_scratch_floats(void);

// Looks up the scratch array's device address for the current device (idempotent).
int cqb_conv_bwd_noalloc_init(void);

// Backward of y = silu(causal_conv(x, w)) per document, enqueued on `stream`.
//   dy, x, dx: bf16 [n, C] row-major, 16-byte aligned;  wT: fp32 [4, C] (the transpose of the
//   [C, 4] weight), 16-byte aligned;  pos: int32 [n], index of each row inside its document;
//   dw: fp32 [C, 4] output (overwritten).  C must be a positive multiple of 8.
int cqb_conv_bwd_noalloc(const void* dy, const void* x, const float* wT, const int* pos, void* dx, float* dw, long n,
                         long C, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
