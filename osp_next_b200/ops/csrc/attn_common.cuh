// Host helpers shared by the attention forward and backward launchers.
#pragma once
#include <torch/extension.h>
#include "common.cuh"
#include "tma_host.h"
#include "attn_math.cuh"

namespace osp {

// TMA map over a [B, N, H, D] bf16 view (last dim contiguous, packed heads, uniform token
// stride across the batch) as a 3-D tensor (D, H, B·N) with 64 × 1 × 128 boxes (128B swizzle).
static inline CUtensorMap attn_tmap(const at::Tensor& x, int D) {
  // x: [B, N, H, D] view, last dim contiguous, packed heads, uniform token stride across batch
  const int64_t B = x.size(0), N = x.size(1), H = x.size(2);
  TORCH_CHECK(x.stride(3) == 1, "attention: last dim must be contiguous");
  TORCH_CHECK(H == 1 || x.stride(2) == D, "attention: heads must be packed (stride D)");
  TORCH_CHECK(B == 1 || x.stride(0) == N * x.stride(1), "attention: batch stride must equal N·token stride");
  uint64_t dims[3] = {(uint64_t)D, (uint64_t)H, (uint64_t)(B * N)};
  uint64_t strides[2] = {(uint64_t)D, (uint64_t)x.stride(1)};
  uint32_t box[3] = {64, 1, 128};
  return make_tmap_bf16(x.data_ptr(), 3, dims, strides, box);
}

}  // namespace osp
