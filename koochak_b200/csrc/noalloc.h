// C declaration of the allocation-free LayerNorm backward entry point that
// norm.cu defines and the extension library exports.
//
// This entry point has no counterpart in the reference framework.
//
// It exists for callers that cannot allocate device memory where they need
// the op: engines that own a fixed device-memory arena and must not call the
// allocator once it is carved up, and C callers that link the library
// without PyTorch (so without its caching allocator).
// Its scratch is one file-scope device array of 4 MiB (2 * grid * C fp32
// partials; the grid shrinks to fit). Rows wider than 4096 are rejected.
// All calls share that array: overlapping calls race and must be serialised
// by the caller. The first call on each device resolves the array's address
// with cudaGetSymbolAddress; that address is then remembered per device for
// the life of the process, which assumes the device is not reset
// (cudaDeviceReset) in between.
//
// dy: bf16 [M, C]; x, w, mean, rstd, dx, dw, db: fp32, contiguous.
// Returns 0 on success, -1 for bad arguments, -2 when C > 4096, otherwise
// the cudaError_t value of the failing runtime call.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

int kb_layernorm_backward_noalloc(const void* dy, const float* x, const float* w, const float* mean,
                                  const float* rstd, float* dx, float* dw, float* db, int M, int C,
                                  cudaStream_t stream);

#ifdef __cplusplus
}
#endif
