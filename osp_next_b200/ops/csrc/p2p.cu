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
//  * FSDP collectives over peer memory (parallel/fsdp_comm.py): every rank keeps a ring
//    of slots in one IPC arena, allocated in the same order on every rank, so a slot has
//    the same offset everywhere.  A tagged barrier (epoch + the slot's offset, checked
//    against every peer's) precedes a pull kernel: all-gather copies each peer's shard
//    out of that peer's slot, reduce-scatter sums this rank's chunk of every peer's slot.
//    A mismatched offset or a timeout sets an abort word that the pull kernel honours.
//  * p2p_pull: the training SSP exchange and the Ulysses all-to-all.  Every rank stages its
//    rows in a slot of peer memory, one p2p_barrier orders the stages, then every rank pulls
//    exactly the chunks it owns from the ranks that hold them (a host-built table of
//    (source rank, byte offset) per output chunk), summing several sources in fp32 where a
//    row has replicas (the backward of a dense layout's replicated rows).
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

// ---------------------------------------------------------------------------- FSDP collectives
// Flag array layout per rank: [0, world) epochs written by each peer, [world, 3·world) the
// tag (slot offset) each peer used, one array per epoch parity (a peer can already be one
// barrier ahead when this rank reads, never two), [3·world] this rank's abort word.
__global__ void p2p_barrier_tagged_kernel(const int64_t* flag_ptrs, int rank, int world, int epoch, int tag,
                                          unsigned long long limit_ns, int* err) {
  const int r = threadIdx.x;
  int* mine = reinterpret_cast<int*>(flag_ptrs[rank]);
  const int tag_base = world + (epoch & 1) * world;
  if (r == 0) mine[3 * world] = 0;
  if (r < world) {
    __threadfence_system();
    int* peer = reinterpret_cast<int*>(flag_ptrs[r]);
    peer[tag_base + rank] = tag;                   // ordered before the epoch by the release below
    st_release_sys(peer + rank, epoch);
  }
  __syncthreads();
  if (r < world) {
    const uint64_t t0 = globaltimer();
    bool ok = true;
    while (ld_acquire_sys(mine + r) < epoch) {
      if (globaltimer() - t0 > limit_ns) {
        record_error(err, kErrP2P);
        ok = false;
        break;
      }
      __nanosleep(100);
    }
    if (ok && *reinterpret_cast<volatile int*>(mine + tag_base + r) != tag) {
      record_error(err, kErrP2PTag);
      ok = false;
    }
    if (!ok) atomicExch(mine + 3 * world, 1);
  }
}

void p2p_barrier_tagged(const at::Tensor& flag_ptrs, int64_t rank, int64_t world, int64_t epoch, int64_t tag,
                        double limit_s) {
  TORCH_CHECK(flag_ptrs.is_cuda() && flag_ptrs.scalar_type() == at::kLong && flag_ptrs.numel() == world &&
              world <= 1024, "p2p_barrier_tagged: int64 device tensor of peer flag pointers");
  c10::cuda::CUDAGuard guard(flag_ptrs.device());
  p2p_barrier_tagged_kernel<<<1, 32 * ((world + 31) / 32), 0, at::cuda::getCurrentCUDAStream()>>>(
      flag_ptrs.data_ptr<int64_t>(), (int)rank, (int)world, (int)epoch, (int)tag,
      (unsigned long long)(limit_s * 1e9), error_word(flag_ptrs.get_device()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// All-gather: bases[p] = rank p's arena (peers mapped); copy each peer's shard
// [off + p·shard, +shard) of its own slot into the same range of this rank's slot.
template <typename V>
__global__ void p2p_gather_kernel(const int64_t* bases, long off, long shard_bytes, int rank, int world,
                                  const int* abort_word) {
  if (*reinterpret_cast<const volatile int*>(abort_word)) return;
  const long nv = shard_bytes / (long)sizeof(V);
  const long total = nv * (world - 1);
  char* dst = reinterpret_cast<char*>(bases[rank]) + off;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    // peers in ring order starting after this rank, so that at any moment every rank is
    // pulling from a different peer instead of all of them hammering rank 0's links
    const int pi = (int)(i / nv);
    const int p = (rank + 1 + pi) % world;
    const long j = i - (long)pi * nv;
    const V* src = reinterpret_cast<const V*>(reinterpret_cast<const char*>(bases[p]) + off + p * shard_bytes) + j;
    reinterpret_cast<V*>(dst + p * shard_bytes)[j] = *src;
  }
}

// Reduce-scatter (fp32): out[i] = scale · Σ_p slot_p[rank·S + i], peers' slots read in place.
__global__ void p2p_reduce_scatter_f32_kernel(float* __restrict__ out, const int64_t* bases, long off, long S,
                                              int rank, int world, float scale, const int* abort_word) {
  if (*reinterpret_cast<const volatile int*>(abort_word)) return;
  const bool vec = (S % 4) == 0 && (off % 16) == 0;
  const long n = vec ? S / 4 : S;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    if (vec) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int k = 0; k < world; ++k) {
        const int p = (rank + 1 + k) % world;        // start at a different peer on every rank
        const float4 v = reinterpret_cast<const float4*>(
            reinterpret_cast<const char*>(bases[p]) + off + (long)rank * S * 4)[i];
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      reinterpret_cast<float4*>(out)[i] = make_float4(acc.x * scale, acc.y * scale, acc.z * scale, acc.w * scale);
    } else {
      float acc = 0.f;
      for (int k = 0; k < world; ++k) {
        const int p = (rank + 1 + k) % world;
        acc += reinterpret_cast<const float*>(reinterpret_cast<const char*>(bases[p]) + off + (long)rank * S * 4)[i];
      }
      out[i] = acc * scale;
    }
  }
}

// Reduce-scatter of bf16 gradients with fp32 accumulation: out[i] (fp32) = scale · Σ_p
// float(peer p's bf16 slot at off)[rank·S + i].  Casting each bf16 value to fp32 is exact,
// so this is the fp32 reduce-scatter of the bf16 gradients (FSDP's reduce_dtype = fp32) with
// the cast fused into the pull and half the bytes on NVLink.
__global__ void p2p_reduce_scatter_bf16_kernel(float* __restrict__ out, const int64_t* bases, long off, long S,
                                               int rank, int world, float scale, const int* abort_word) {
  if (*reinterpret_cast<const volatile int*>(abort_word)) return;
  const bool vec = (S % 8) == 0 && (off % 16) == 0;
  const long n = vec ? S / 8 : S;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    if (vec) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int k = 0; k < world; ++k) {
        const int p = (rank + 1 + k) % world;        // start at a different peer on every rank
        const uint4 v = reinterpret_cast<const uint4*>(
            reinterpret_cast<const char*>(bases[p]) + off + (long)rank * S * 2)[i];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          acc[2 * e] += f.x;
          acc[2 * e + 1] += f.y;
        }
      }
      float4* o = reinterpret_cast<float4*>(out) + 2 * i;
      o[0] = make_float4(acc[0] * scale, acc[1] * scale, acc[2] * scale, acc[3] * scale);
      o[1] = make_float4(acc[4] * scale, acc[5] * scale, acc[6] * scale, acc[7] * scale);
    } else {
      float acc = 0.f;
      for (int k = 0; k < world; ++k) {
        const int p = (rank + 1 + k) % world;
        acc += __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(
            reinterpret_cast<const char*>(bases[p]) + off + (long)rank * S * 2)[i]);
      }
      out[i] = acc * scale;
    }
  }
}

static int pull_grid(long work) {
  return (int)std::max<long>(1, std::min<long>((work + 255) / 256, 148L * 8));
}

void p2p_gather(const at::Tensor& bases, int64_t off, int64_t shard_bytes, int64_t rank, int64_t world,
                int64_t abort_ptr) {
  TORCH_CHECK(bases.is_cuda() && bases.scalar_type() == at::kLong && bases.numel() == world, "p2p_gather: bases");
  c10::cuda::CUDAGuard guard(bases.device());
  if (world < 2 || shard_bytes == 0) return;
  auto st = at::cuda::getCurrentCUDAStream();
  const int64_t* b = bases.data_ptr<int64_t>();
  const int* ab = reinterpret_cast<const int*>(abort_ptr);
  if (shard_bytes % 16 == 0 && off % 16 == 0)
    p2p_gather_kernel<int4><<<pull_grid(shard_bytes / 16 * (world - 1)), 256, 0, st>>>(b, off, shard_bytes, rank, world, ab);
  else if (shard_bytes % 4 == 0 && off % 4 == 0)
    p2p_gather_kernel<int><<<pull_grid(shard_bytes / 4 * (world - 1)), 256, 0, st>>>(b, off, shard_bytes, rank, world, ab);
  else
    p2p_gather_kernel<char><<<pull_grid(shard_bytes * (world - 1)), 256, 0, st>>>(b, off, shard_bytes, rank, world, ab);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void p2p_reduce_scatter_f32(at::Tensor& out, const at::Tensor& bases, int64_t off, int64_t shard_elems, int64_t rank,
                            int64_t world, double scale, int64_t abort_ptr) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() == shard_elems,
              "p2p_reduce_scatter_f32: fp32 contiguous out [S]");
  TORCH_CHECK(bases.scalar_type() == at::kLong && bases.numel() == world, "p2p_reduce_scatter_f32: bases");
  c10::cuda::CUDAGuard guard(out.device());
  if (shard_elems == 0) return;
  p2p_reduce_scatter_f32_kernel<<<pull_grid(shard_elems / 4 + 1), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      out.data_ptr<float>(), bases.data_ptr<int64_t>(), off, shard_elems, (int)rank, (int)world, (float)scale,
      reinterpret_cast<const int*>(abort_ptr));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void p2p_reduce_scatter_bf16(at::Tensor& out, const at::Tensor& bases, int64_t off, int64_t shard_elems,
                             int64_t rank, int64_t world, double scale, int64_t abort_ptr) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() == shard_elems,
              "p2p_reduce_scatter_bf16: fp32 contiguous out [S]");
  TORCH_CHECK(bases.scalar_type() == at::kLong && bases.numel() == world, "p2p_reduce_scatter_bf16: bases");
  c10::cuda::CUDAGuard guard(out.device());
  if (shard_elems == 0) return;
  p2p_reduce_scatter_bf16_kernel<<<pull_grid(shard_elems / 8 + 1), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      out.data_ptr<float>(), bases.data_ptr<int64_t>(), off, shard_elems, (int)rank, (int)world, (float)scale,
      reinterpret_cast<const int*>(abort_ptr));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------- table-driven pull
// out chunk u (chunk_vecs 16-byte vectors, contiguous in `out`) = the chunk at
// ptrs[rank[u·R + k]] + off[u·R + k]: copied (R == 1; rank < 0 → zeros) or the fp32 sum over
// k (kSum; sources with rank < 0 are skipped, none → zeros).  One thread per 16-byte vector;
// the chunk's table entries are warp-uniform whenever a chunk spans a warp.
template <bool kSum>
__global__ void __launch_bounds__(256) p2p_pull_kernel(int4* __restrict__ out, const int64_t* __restrict__ ptrs,
                                                       const int* __restrict__ rank, const int64_t* __restrict__ off,
                                                       int R, long n_chunks, int chunk_vecs) {
  const long total = n_chunks * chunk_vecs;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long u = i / chunk_vecs;
    const int v = (int)(i - u * chunk_vecs);
    if (!kSum) {
      const int r = __ldg(rank + u);
      int4 val = make_int4(0, 0, 0, 0);
      if (r >= 0) val = reinterpret_cast<const int4*>(reinterpret_cast<const char*>(ptrs[r]) + __ldg(off + u))[v];
      out[i] = val;
    } else {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int k = 0; k < R; ++k) {
        const int r = __ldg(rank + u * R + k);
        if (r < 0) continue;
        const int4 raw =
            reinterpret_cast<const int4*>(reinterpret_cast<const char*>(ptrs[r]) + __ldg(off + u * R + k))[v];
        acc.x += __int_as_float(raw.x); acc.y += __int_as_float(raw.y);
        acc.z += __int_as_float(raw.z); acc.w += __int_as_float(raw.w);
      }
      out[i] = make_int4(__float_as_int(acc.x), __float_as_int(acc.y), __float_as_int(acc.z), __float_as_int(acc.w));
    }
  }
}

void p2p_pull(at::Tensor& out, const at::Tensor& ptrs, const at::Tensor& rank, const at::Tensor& off, int64_t R,
              int64_t chunk_bytes, bool sum) {
  TORCH_CHECK(out.is_cuda() && out.is_contiguous(), "p2p_pull: contiguous CUDA output");
  TORCH_CHECK(chunk_bytes > 0 && chunk_bytes % 16 == 0, "p2p_pull: chunk size must be a multiple of 16 bytes");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0, "p2p_pull: output not 16-byte aligned");
  const int64_t nbytes = out.numel() * out.element_size();
  TORCH_CHECK(nbytes % chunk_bytes == 0, "p2p_pull: output is not a whole number of chunks");
  const int64_t n_chunks = nbytes / chunk_bytes;
  TORCH_CHECK(R >= 1 && rank.scalar_type() == at::kInt && off.scalar_type() == at::kLong &&
              rank.numel() == n_chunks * R && off.numel() == n_chunks * R && rank.is_cuda() && off.is_cuda() &&
              rank.is_contiguous() && off.is_contiguous(), "p2p_pull: int32 rank / int64 offset tables [chunks·R]");
  TORCH_CHECK(ptrs.is_cuda() && ptrs.scalar_type() == at::kLong, "p2p_pull: int64 device table of slot pointers");
  TORCH_CHECK(!sum || out.scalar_type() == at::kFloat, "p2p_pull: the summing pull is fp32");
  TORCH_CHECK(sum || R == 1, "p2p_pull: a copying pull has one source per chunk");
  c10::cuda::CUDAGuard guard(out.device());
  if (n_chunks == 0) return;
  const int vecs = (int)(chunk_bytes / 16);
  const long work = n_chunks * vecs;
  const int grid = (int)std::max<long>(1, std::min<long>((work + 255) / 256, 148L * 16));
  auto st = at::cuda::getCurrentCUDAStream();
  if (sum)
    p2p_pull_kernel<true><<<grid, 256, 0, st>>>(reinterpret_cast<int4*>(out.data_ptr()), ptrs.data_ptr<int64_t>(),
                                                rank.data_ptr<int>(), off.data_ptr<int64_t>(), (int)R, n_chunks, vecs);
  else
    p2p_pull_kernel<false><<<grid, 256, 0, st>>>(reinterpret_cast<int4*>(out.data_ptr()), ptrs.data_ptr<int64_t>(),
                                                 rank.data_ptr<int>(), off.data_ptr<int64_t>(), 1, n_chunks, vecs);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace osp
