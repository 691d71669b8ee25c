// Entry point of brain_b200 that allocates no device memory.
//
// This declaration has no counterpart in the reference framework (uxle/brain): it exists for
// callers of this library that cannot allocate device memory while they run - for example a C or
// C++ host that links libbrain_kernels.so without PyTorch or any allocator, or a serving process
// that reserved all GPU memory up front under a fixed budget.
//
// brain_norm_bwd_noalloc is the RMSNorm (kind 0) / LayerNorm (kind 1) backward of
// brain_norm_bwd (norms.cu) with its f32 partial-sum workspace replaced by a fixed 4 MiB
// __device__ array inside the library: D <= 8192 (larger D returns BRAIN_NOALLOC_TOO_LARGE = -1000),
// at most 64 partial rows. The caller still passes every input and output. The first call on
// each device looks up the array's device address (cudaGetSymbolAddress) with that device
// current; make it before any stream capture. All calls share the array, which keeps the last
// call's contents (each call overwrites what it reads, so no clearing is needed): calls that
// overlap on the GPU race and must be serialised by the caller.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

// A code no other entry point of the library returns.
#define BRAIN_NOALLOC_TOO_LARGE (-1000)

#ifdef __cplusplus
extern "C" {
#endif
int brain_norm_bwd_noalloc(int kind, const void* dy, int64_t lddy, const void* x, int64_t ldx, const void* w,
                           const float* mean_in, const float* rstd_in, void* dx, int64_t lddx, const void* dres,
                           int64_t lddres, void* dw, void* db, int dw_f32, int accumulate, int M, int D,
                           cudaStream_t st);
#ifdef __cplusplus
}
#endif
