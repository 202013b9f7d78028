// Host-side helpers: TMA tensor-map encoding (driver entry point fetched at run
// time, so the extension does not link libcuda) and the per-device error word
// that bounded device-side waits write to.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <c10/util/Exception.h>
#include <c10/cuda/CUDAException.h>
#include <mutex>

namespace osp {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    C10_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && p != nullptr, "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Rank-N bf16 tensor map with 128-byte swizzle.  dims/strides innermost first;
// strides in elements for dims 1..N-1.  The innermost box must be 64 elements
// (128 bytes) for the SW128 UMMA layouts used by the kernels.
inline CUtensorMap make_tmap_bf16(void* ptr, int rank, const uint64_t* dims, const uint64_t* strides_elems,
                                  const uint32_t* box) {
  CUtensorMap m;
  cuuint64_t gdim[5], gstride[4];
  cuuint32_t bdim[5], estr[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estr[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) {
    gstride[i] = strides_elems[i] * 2;
    TORCH_CHECK(gstride[i] % 16 == 0, "TMA stride must be a multiple of 16 bytes");
  }
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK(box[0] * 2 == 128, "innermost TMA box must be 128 bytes (SW128)");
  CUresult r = encode_tiled_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, ptr, gdim, gstride, bdim, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

inline CUtensorMap make_tmap_2d_bf16(void* ptr, int64_t inner, int64_t outer, int64_t row_stride_elems,
                                     uint32_t box_inner, uint32_t box_outer) {
  uint64_t dims[2] = {(uint64_t)inner, (uint64_t)outer};
  uint64_t strides[1] = {(uint64_t)row_stride_elems};
  uint32_t box[2] = {box_inner, box_outer};
  return make_tmap_bf16(ptr, 2, dims, strides, box);
}

constexpr int kMaxDevices = 64;

// One int per device; device code records the first error code (atomicCAS 0→code).
int* error_word(int device);

// Streaming multiprocessors of `device` (cached per device).
int num_sms(int device);

// Opt `kernel` into `bytes` of dynamic shared memory on the current device.  The
// attribute is per device, so the setting is remembered per (kernel, device) pair.
void smem_opt_in(const void* kernel, int bytes);

}  // namespace osp
