// No-allocation variant of the per-tensor HiF8 quantise→dequantise (see hif8_noalloc.h).
//
// Three launches on the caller's stream, all reading / writing a file-scope device
// array instead of allocated scratch:
//   1. per-block max(|x|) over 4096-element slices → scratch[block]
//   2. one block reduces the partial maxima       → scratch[kMaxPartials]
//   3. elementwise rounding with s = (1 / max(amax, 1e-8)) · scale_max
// Every word that stage 2 and 3 read is written by the previous stage of the same
// call, so nothing needs clearing between calls.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <mutex>

#include "hif8_noalloc.h"

namespace {

constexpr int kPartials = OSP_HIF8_NOALLOC_MAX_PARTIALS;
constexpr int kPerBlock = OSP_HIF8_NOALLOC_ELEMS_PER_BLOCK;
constexpr int kThreads = 256;

// partial maxima + the final amax word; resident on every GPU that loads the library
static __device__ __align__(256) float g_hif8_scratch[kPartials + 1];

__device__ __forceinline__ float load_elem(const void* x, int dtype, int64_t i) {
  return dtype == 0 ? static_cast<const float*>(x)[i]
                    : __bfloat162float(static_cast<const __nv_bfloat16*>(x)[i]);
}

// same rounding as misc.cu's hif8_round_dev (Ascend kernel semantics)
__device__ __forceinline__ float hif8_round_na(float v) {
  const float a = fabsf(v);
  const int e = (int)((__float_as_uint(a) >> 23) & 0xFF) - 127;
  const int ae = abs(e);
  const int m = ae <= 3 ? 3 : (ae <= 7 ? 2 : (ae <= 15 ? 1 : 0));
  const int se = max(e, -22) - m;
  float q = floorf(ldexpf(a, -se) + 0.5f);
  q = ldexpf(q, se);
  if (a < 1.1920928955078125e-07f) q = 0.f;
  if (a >= 40960.f) q = __int_as_float(0x7f800000);
  return copysignf(q, v);
}

__global__ void partial_absmax(const void* x, int dtype, int64_t n, float* scratch) {
  __shared__ float red[kThreads / 32];
  const int64_t base = (int64_t)blockIdx.x * kPerBlock;
  float m = 0.f;
  for (int i = threadIdx.x; i < kPerBlock; i += kThreads) {
    const int64_t k = base + i;
    if (k < n) m = fmaxf(m, fabsf(load_elem(x, dtype, k)));
  }
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float r = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) r = fmaxf(r, red[w]);
    scratch[blockIdx.x] = r;
  }
}

__global__ void reduce_partials(int nblocks, float* scratch) {
  __shared__ float red[kThreads / 32];
  float m = 0.f;
  for (int i = threadIdx.x; i < nblocks; i += kThreads) m = fmaxf(m, scratch[i]);
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float r = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) r = fmaxf(r, red[w]);
    scratch[kPartials] = r;
  }
}

__global__ void quantize(const void* x, void* out, int dtype, int64_t n, float scale_max, const float* scratch) {
  const float s = (1.0f / fmaxf(scratch[kPartials], 1e-8f)) * scale_max;   // as hif8_qdq computes it
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
    const float y = hif8_round_na(load_elem(x, dtype, i) * s) / s;
    if (dtype == 0) static_cast<float*>(out)[i] = y;
    else static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16(y);
  }
}

// device address of the scratch array, looked up once per device
std::mutex g_mu;
float* g_addr[64] = {nullptr};

cudaError_t scratch_for_current_device(float** p) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void* a = nullptr;
    e = cudaGetSymbolAddress(&a, g_hif8_scratch);
    if (e != cudaSuccess) return e;
    g_addr[dev] = static_cast<float*>(a);
  }
  *p = g_addr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int osp_hif8_qdq_noalloc(const void* x, void* out, int64_t n,
                                                                         int dtype, float scale_max,
                                                                         cudaStream_t stream) {
  if (n < 0 || n > OSP_HIF8_NOALLOC_MAX_ELEMS || (dtype != 0 && dtype != 1) || (n > 0 && (!x || !out)))
    return (int)cudaErrorInvalidValue;
  if (n == 0) return (int)cudaSuccess;
  float* scratch = nullptr;
  cudaError_t e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess) return (int)e;
  const int nblocks = (int)((n + kPerBlock - 1) / kPerBlock);
  partial_absmax<<<nblocks, kThreads, 0, stream>>>(x, dtype, n, scratch);
  reduce_partials<<<1, kThreads, 0, stream>>>(nblocks, scratch);
  const int64_t qb = (n + kThreads - 1) / kThreads;
  quantize<<<(int)(qb < 148 * 16 ? qb : 148 * 16), kThreads, 0, stream>>>(x, out, dtype, n, scale_max, scratch);
  return (int)cudaGetLastError();
}
