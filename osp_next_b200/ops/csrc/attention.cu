// Host launcher of the segmented flash-attention forward (kernel: attention_fwd.cuh).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "attention_fwd.cuh"
#include "attn_common.cuh"

namespace osp {

// P published in two halves (the PV MMA starts on keys 0..63 while 64..127 are being
// exponentiated); all exponentials on MUFU.  At the 14B shapes (4 × 20 160-key segments,
// 40 heads, batch 2): 1122 TFLOP/s against 1078 for one-piece P with 1/8 of the
// exponentials on the FMA pipe.
constexpr uint32_t kFwdPoly = 0x00u;
constexpr bool kFwdSplitP = true;

template <int D>
static void launch_attn_fwd(dim3 grid, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                            const AttnArgs& a, cudaStream_t stream) {
  using L = AttnFwdCfg<D>;
  auto kern = attn_fwd_kernel<D, kFwdPoly, kFwdSplitP>;
  smem_opt_in(reinterpret_cast<const void*>(kern), L::BYTES);
  kern<<<grid, L::kThreads, L::BYTES, stream>>>(tq, tk, tv, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void attention_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& seg_q,
                   const at::Tensor& seg_k, at::Tensor& out, at::Tensor& lse, double scale, int64_t max_q) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda(), "attention: CUDA tensors");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
              "attention: bf16 q/k/v");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "attention: [B, N, H, D]");
  const int D = (int)q.size(3);
  TORCH_CHECK(D == 64 || D == 128, "attention: head_dim 64 or 128");
  TORCH_CHECK(k.size(3) == D && v.size(3) == D && k.size(2) == q.size(2) && v.size(2) == q.size(2) &&
              k.size(0) == q.size(0) && v.size(0) == q.size(0) && v.size(1) == k.size(1), "attention: shapes");
  TORCH_CHECK(seg_q.scalar_type() == at::kInt && seg_k.scalar_type() == at::kInt && seg_q.numel() == seg_k.numel(),
              "attention: int32 segments of equal count");
  TORCH_CHECK(seg_q.is_cuda() && seg_k.is_cuda(), "attention: segments on the device");
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == at::kBFloat16 && out.sizes() == q.sizes(),
              "attention: bf16 contiguous out [B, Nq, H, D]");
  c10::cuda::CUDAGuard guard(q.device());
  const int B = (int)q.size(0), H = (int)q.size(2);
  const int nseg = (int)seg_q.numel() - 1;
  if (nseg <= 0 || max_q <= 0 || B == 0) return;
  CUtensorMap tq = attn_tmap(q, D), tk = attn_tmap(k, D), tv = attn_tmap(v, D);
  AttnArgs a;
  a.seg_q = seg_q.data_ptr<int>();
  a.seg_k = seg_k.data_ptr<int>();
  a.Nq = (int)q.size(1);
  a.Nk = (int)k.size(1);
  a.H = H;
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.lse = (lse.defined() && lse.numel() > 0) ? lse.data_ptr<float>() : nullptr;
  if (a.lse) TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.numel() == (int64_t)B * H * a.Nq, "attention: lse");
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.err = error_word(q.get_device());
  dim3 grid((unsigned)((max_q + 2 * kQT - 1) / (2 * kQT)), (unsigned)nseg, (unsigned)(B * H));
  auto stream = at::cuda::getCurrentCUDAStream();
  if (D == 128) launch_attn_fwd<128>(grid, tq, tk, tv, a, stream);
  else launch_attn_fwd<64>(grid, tq, tk, tv, a, stream);
}

}  // namespace osp
