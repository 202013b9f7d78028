// Peer-to-peer buffers over NVLink and a bounded device-side barrier.
//
// The SSP exchange of the reference is an NCCL all_to_all_single of the residual
// stream between two sparse blocks (ospnext/modules/skiparse_func.py:58-93).  Here
// the producing GEMM stores every output row straight into the buffer of the rank
// that owns the row in the next layout (gemm.cu, peer-pointer epilogue), so the
// transfer overlaps the GEMM tile by tile.  This file provides what that needs:
//
//  * p2p_alloc / p2p_open / p2p_close / p2p_free: one cudaMalloc'd buffer per rank,
//    exported with a CUDA IPC handle and mapped by the peers (plain loads/stores
//    over NVLink; no multicast object is created);
//  * p2p_barrier: rank r writes `epoch` into slot r of every peer's flag array
//    (system-scope release after a system fence), then waits — bounded by
//    %globaltimer — until every peer's slot in its own array reaches `epoch`.
//    On timeout it records kErrP2P in the error word and returns, so a missing
//    peer never hangs the GPU; the host checks the error word.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <string>
#include <vector>

#include "common.cuh"
#include "tma_host.h"

namespace osp {

std::tuple<int64_t, std::string> p2p_alloc(int64_t bytes) {
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, (size_t)bytes));
  C10_CUDA_CHECK(cudaMemset(p, 0, (size_t)bytes));
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  return {reinterpret_cast<int64_t>(p), std::string(reinterpret_cast<const char*>(&h), sizeof(h))};
}

int64_t p2p_open(const std::string& handle) {
  TORCH_CHECK(handle.size() == sizeof(cudaIpcMemHandle_t), "p2p_open: bad handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void p2p_close(int64_t ptr) { C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }

void p2p_free(int64_t ptr) { C10_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr))); }

at::Tensor p2p_view(int64_t ptr, std::vector<int64_t> shape, at::ScalarType dtype, int64_t device) {
  auto opts = at::TensorOptions().dtype(dtype).device(at::kCUDA, device);
  return at::from_blob(reinterpret_cast<void*>(ptr), shape, [](void*) {}, opts);
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// flag_ptrs[r] = base of rank r's flag array (int[world]); slot s of rank r's array is
// written by rank s.  One thread per peer.
__global__ void p2p_barrier_kernel(const int64_t* flag_ptrs, int rank, int world, int epoch,
                                   unsigned long long limit_ns, int* err) {
  const int r = threadIdx.x;
  if (r < world) {
    __threadfence_system();          // this rank's earlier peer stores are visible first
    int* peer_flags = reinterpret_cast<int*>(flag_ptrs[r]);
    st_release_sys(peer_flags + rank, epoch);
  }
  __syncthreads();
  if (r < world) {
    const int* mine = reinterpret_cast<const int*>(flag_ptrs[rank]);
    const uint64_t t0 = globaltimer();
    while (ld_acquire_sys(mine + r) < epoch) {
      if (globaltimer() - t0 > limit_ns) {
        record_error(err, kErrP2P);
        break;
      }
      __nanosleep(100);
    }
  }
}

void p2p_barrier(const at::Tensor& flag_ptrs, int64_t rank, int64_t world, int64_t epoch, double limit_s) {
  TORCH_CHECK(flag_ptrs.is_cuda() && flag_ptrs.scalar_type() == at::kLong && flag_ptrs.numel() == world,
              "p2p_barrier: int64 device tensor of peer flag pointers");
  TORCH_CHECK(world <= 1024, "p2p_barrier: world too large");
  c10::cuda::CUDAGuard guard(flag_ptrs.device());
  p2p_barrier_kernel<<<1, 32 * ((world + 31) / 32), 0, at::cuda::getCurrentCUDAStream()>>>(
      flag_ptrs.data_ptr<int64_t>(), (int)rank, (int)world, (int)epoch, (unsigned long long)(limit_s * 1e9),
      error_word(flag_ptrs.get_device()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace osp
