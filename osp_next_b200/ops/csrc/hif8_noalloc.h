// No-allocation entry point for per-tensor HiF8 fake quantisation.
//
// This entry point has no counterpart in the reference; it is an addition of this
// library for callers that cannot allocate GPU memory themselves (and must not
// have the library allocate on their behalf): code running inside a fixed memory
// budget or a pre-reserved pool, or host code that is not allowed to call
// cudaMalloc / cudaFree (or a caching allocator such as torch's) at the point of
// the call.  The regular entry point (`hif8_qdq` in misc.cu) takes a 4-byte
// scratch word from the torch allocator; this one uses a fixed scratch array in
// device memory that is part of the library image instead.
//
// Limits and behaviour:
//  * At most OSP_HIF8_NOALLOC_MAX_ELEMS elements per call (64 Mi = 16384 partial
//    maxima of 4096 elements; the scratch array is 64 KiB + one word and stays
//    resident on every GPU that loads the library until the process exits).
//    Larger inputs are rejected with cudaErrorInvalidValue and nothing is launched.
//  * The first call on a device looks up the scratch address for that device
//    (cudaGetSymbolAddress); make that first call before any stream capture.
//  * All calls share the one scratch array, and it keeps the previous call's
//    contents (every call overwrites what it reads).  Calls that can overlap on
//    the GPU — on different streams without ordering — race on it; issue them in
//    order on one stream.
//  * No cudaMalloc / cudaFree or allocating library routine is called.
//  * The looked-up scratch address is kept for the life of the process, per device
//    ordinal.  Do not use the entry point across a device reset (cudaDeviceReset, or
//    destroying and re-creating the primary context): the cached address would no
//    longer be valid there.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define OSP_HIF8_NOALLOC_MAX_PARTIALS 16384
#define OSP_HIF8_NOALLOC_ELEMS_PER_BLOCK 4096
#define OSP_HIF8_NOALLOC_MAX_ELEMS ((int64_t)OSP_HIF8_NOALLOC_MAX_PARTIALS * OSP_HIF8_NOALLOC_ELEMS_PER_BLOCK)

#ifdef __cplusplus
extern "C" {
#endif

// out = dequant(quant_hif8(x · s)) / s with s = scale_max / max(|x|, 1e-8), one
// scale for the whole tensor (the same result as the allocating `hif8_qdq`).
// dtype: 0 = float32, 1 = bfloat16 (x and out share it).  x and out are device
// pointers to n contiguous elements on the current device (make that device
// current before calling); out may equal x.  Returns cudaSuccess or
// the CUDA error (cudaErrorInvalidValue for n < 0, n > OSP_HIF8_NOALLOC_MAX_ELEMS,
// an unknown dtype or null pointers).  Work is queued on `stream`.
int osp_hif8_qdq_noalloc(const void* x, void* out, int64_t n, int dtype, float scale_max, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
