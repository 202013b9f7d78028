// Row-wise normalisation kernels (one CTA of 256 threads per row, fp32 math,
// row held in registers between the statistics pass and the output pass).
//
//   ln_modulate   bf16 out = LN(x)·(1+scale[b]) + shift[b]     (osp_next.py:941, 954)
//                 or affine LN(x)·w + b (norm3, osp_next.py:949)
//   rms_norm      bf16 out = x·rsqrt(mean(x²)+eps)·w            (want2v.py:77-93)
//   qk_norm_rope  in place on fused qkv [rows, 3C]: full-row RMSNorm of q and k
//                 (over all heads, as the reference) then interleaved-pair 3-D RoPE
//                 with each token's true (t,h,w) (osp_next.py:550-644, 742-752); the
//                 rotation reads a precomputed (cos, sin) table instead of evaluating sincos
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace osp {

constexpr int kRowThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kRowThreads / 32; ++i) s += red[i];
  return s;
}

template <typename InT>
__device__ __forceinline__ float4 load4(const InT* p);
template <>
__device__ __forceinline__ float4 load4<float>(const float* p) { return *reinterpret_cast<const float4*>(p); }
template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&u.x);
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&u.y);
  float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

// MAXV = max float4 chunks per thread (C ≤ MAXV·4·256)
template <typename InT, int MAXV>
__global__ void __launch_bounds__(kRowThreads)
ln_modulate_kernel(const InT* __restrict__ x, const float* __restrict__ shift, const float* __restrict__ scale,
                   const float* __restrict__ w, const float* __restrict__ b, __nv_bfloat16* __restrict__ out,
                   int C, int rows_per_batch, float eps) {
  __shared__ float red[kRowThreads / 32];
  const long row = blockIdx.x;
  const int bidx = (int)(row / rows_per_batch);
  const InT* xr = x + row * C;
  const int nv = C / 4;
  float4 v[MAXV];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c4 = threadIdx.x + i * kRowThreads;
    if (c4 < nv) {
      v[i] = load4<InT>(xr + 4 * c4);
      s += v[i].x + v[i].y + v[i].z + v[i].w;
    }
  }
  const float mean = block_sum(s, red) / C;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c4 = threadIdx.x + i * kRowThreads;
    if (c4 < nv) {
      float a = v[i].x - mean, bb = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
      q += a * a + bb * bb + c * c + d * d;
    }
  }
  const float rstd = rsqrtf(block_sum(q, red) / C + eps);
  const float* sh = shift ? shift + (long)bidx * C : nullptr;
  const float* sc = scale ? scale + (long)bidx * C : nullptr;
  __nv_bfloat16* orow = out + row * C;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c4 = threadIdx.x + i * kRowThreads;
    if (c4 < nv) {
      float y[4] = {(v[i].x - mean) * rstd, (v[i].y - mean) * rstd, (v[i].z - mean) * rstd, (v[i].w - mean) * rstd};
      if (w) {
        float4 ww = *reinterpret_cast<const float4*>(w + 4 * c4);
        y[0] *= ww.x; y[1] *= ww.y; y[2] *= ww.z; y[3] *= ww.w;
      }
      if (b) {
        float4 bb = *reinterpret_cast<const float4*>(b + 4 * c4);
        y[0] += bb.x; y[1] += bb.y; y[2] += bb.z; y[3] += bb.w;
      }
      if (sc) {
        float4 s4 = *reinterpret_cast<const float4*>(sc + 4 * c4);
        float4 h4 = *reinterpret_cast<const float4*>(sh + 4 * c4);
        y[0] = y[0] * (1.f + s4.x) + h4.x;
        y[1] = y[1] * (1.f + s4.y) + h4.y;
        y[2] = y[2] * (1.f + s4.z) + h4.z;
        y[3] = y[3] * (1.f + s4.w) + h4.w;
      }
      uint2 u;
      u.x = pack_bf16x2(y[0], y[1]);
      u.y = pack_bf16x2(y[2], y[3]);
      *reinterpret_cast<uint2*>(orow + 4 * c4) = u;
    }
  }
}

template <int MAXV>
__global__ void __launch_bounds__(kRowThreads)
rms_norm_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w, __nv_bfloat16* __restrict__ out,
                int C, float eps) {
  __shared__ float red[kRowThreads / 32];
  const long row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * C;
  const int nv = C / 4;
  float4 v[MAXV];
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c4 = threadIdx.x + i * kRowThreads;
    if (c4 < nv) {
      v[i] = load4<__nv_bfloat16>(xr + 4 * c4);
      q += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
  }
  const float r = rsqrtf(block_sum(q, red) / C + eps);
  __nv_bfloat16* orow = out + row * C;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c4 = threadIdx.x + i * kRowThreads;
    if (c4 < nv) {
      float4 ww = w ? *reinterpret_cast<const float4*>(w + 4 * c4) : make_float4(1.f, 1.f, 1.f, 1.f);
      uint2 u;
      u.x = pack_bf16x2(v[i].x * r * ww.x, v[i].y * r * ww.y);
      u.y = pack_bf16x2(v[i].z * r * ww.z, v[i].w * r * ww.w);
      *reinterpret_cast<uint2*>(orow + 4 * c4) = u;
    }
  }
}

// One CTA per row of the fused [rows, 3C] qkv buffer.  Each thread owns float4
// chunks (two RoPE pairs) of q and of k.
template <int MAXV>
__global__ void __launch_bounds__(kRowThreads)
qk_norm_rope_kernel(__nv_bfloat16* __restrict__ qkv, const float* __restrict__ wq, const float* __restrict__ wk,
                    const int* __restrict__ pos, const float2* __restrict__ cstab, int C, int D, int rows_per_batch,
                    float eps) {
  __shared__ float red[kRowThreads / 32];
  const long row = blockIdx.x;
  const int m = (int)(row % rows_per_batch);
  __nv_bfloat16* qr = qkv + row * 3L * C;
  __nv_bfloat16* kr = qr + C;
  const int nv = C / 4;
  float4 qv[MAXV], kv[MAXV];
  float sq = 0.f, sk = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c4 = threadIdx.x + i * kRowThreads;
    if (c4 < nv) {
      qv[i] = load4<__nv_bfloat16>(qr + 4 * c4);
      kv[i] = load4<__nv_bfloat16>(kr + 4 * c4);
      sq += qv[i].x * qv[i].x + qv[i].y * qv[i].y + qv[i].z * qv[i].z + qv[i].w * qv[i].w;
      sk += kv[i].x * kv[i].x + kv[i].y * kv[i].y + kv[i].z * kv[i].z + kv[i].w * kv[i].w;
    }
  }
  const float rq = rsqrtf(block_sum(sq, red) / C + eps);
  const float rk = rsqrtf(block_sum(sk, red) / C + eps);
  const int half = D / 2;
  const int ch = half / 3;            // h and w pairs
  const int ct = half - 2 * ch;       // t pairs
  const int pt = pos[3 * m], ph = pos[3 * m + 1], pw = pos[3 * m + 2];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c4 = threadIdx.x + i * kRowThreads;
    if (c4 < nv) {
      const int e = 4 * c4;
      float4 w1 = *reinterpret_cast<const float4*>(wq + e);
      float4 w2 = *reinterpret_cast<const float4*>(wk + e);
      float qa[4] = {qv[i].x * rq * w1.x, qv[i].y * rq * w1.y, qv[i].z * rq * w1.z, qv[i].w * rq * w1.w};
      float ka[4] = {kv[i].x * rk * w2.x, kv[i].y * rk * w2.y, kv[i].z * rk * w2.z, kv[i].w * rk * w2.w};
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const int j = ((e % D) >> 1) + p;             // pair index inside the head
        const int prow = j < ct ? pt : (j < ct + ch ? ph : pw);
        const float2 t = cstab[(long)prow * half + j];      // (cos, sin) of the angle
        const float cs = t.x, sn = t.y;
        const float q1 = qa[2 * p], q2 = qa[2 * p + 1];
        qa[2 * p] = q1 * cs - q2 * sn;
        qa[2 * p + 1] = q1 * sn + q2 * cs;
        const float k1 = ka[2 * p], k2 = ka[2 * p + 1];
        ka[2 * p] = k1 * cs - k2 * sn;
        ka[2 * p + 1] = k1 * sn + k2 * cs;
      }
      uint2 u;
      u.x = pack_bf16x2(qa[0], qa[1]);
      u.y = pack_bf16x2(qa[2], qa[3]);
      *reinterpret_cast<uint2*>(qr + e) = u;
      u.x = pack_bf16x2(ka[0], ka[1]);
      u.y = pack_bf16x2(ka[2], ka[3]);
      *reinterpret_cast<uint2*>(kr + e) = u;
    }
  }
}

#define OSP_ROW_DISPATCH(C, ...)                                           \
  do {                                                                    \
    const int nvec = ((C) / 4 + kRowThreads - 1) / kRowThreads;           \
    if (nvec <= 1) { constexpr int MV = 1; __VA_ARGS__; }                  \
    else if (nvec <= 2) { constexpr int MV = 2; __VA_ARGS__; }             \
    else if (nvec <= 4) { constexpr int MV = 4; __VA_ARGS__; }             \
    else if (nvec <= 5) { constexpr int MV = 5; __VA_ARGS__; }             \
    else if (nvec <= 8) { constexpr int MV = 8; __VA_ARGS__; }             \
    else TORCH_CHECK(false, "row too long: C=", C);                        \
  } while (0)

void ln_modulate(const at::Tensor& x, const c10::optional<at::Tensor>& shift, const c10::optional<at::Tensor>& scale,
                 const c10::optional<at::Tensor>& w, const c10::optional<at::Tensor>& b, at::Tensor& out, double eps) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && out.is_contiguous(), "ln_modulate: contiguous CUDA tensors");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16, "ln_modulate: bf16 out");
  const int C = (int)x.size(-1);
  TORCH_CHECK(C % 4 == 0, "ln_modulate: C % 4 == 0");
  const long rows = x.numel() / C;
  const int rpb = x.dim() == 3 ? (int)x.size(1) : (int)rows;
  if (scale.has_value()) {
    TORCH_CHECK(shift.has_value() && scale->scalar_type() == at::kFloat && shift->scalar_type() == at::kFloat,
                "ln_modulate: f32 shift/scale");
    TORCH_CHECK(scale->numel() == (rows / rpb) * C && shift->numel() == (rows / rpb) * C, "ln_modulate: [B, C]");
  }
  c10::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  if (rows == 0) return;
  const float* sh = shift.has_value() ? shift->data_ptr<float>() : nullptr;
  const float* sc = scale.has_value() ? scale->data_ptr<float>() : nullptr;
  const float* wp = w.has_value() ? w->data_ptr<float>() : nullptr;
  const float* bp = b.has_value() ? b->data_ptr<float>() : nullptr;
  auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (x.scalar_type() == at::kFloat) {
    OSP_ROW_DISPATCH(C, (ln_modulate_kernel<float, MV><<<rows, kRowThreads, 0, stream>>>(
                            x.data_ptr<float>(), sh, sc, wp, bp, o, C, rpb, (float)eps)));
  } else {
    TORCH_CHECK(x.scalar_type() == at::kBFloat16, "ln_modulate: f32 or bf16 input");
    OSP_ROW_DISPATCH(C, (ln_modulate_kernel<__nv_bfloat16, MV><<<rows, kRowThreads, 0, stream>>>(
                            reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), sh, sc, wp, bp, o, C, rpb,
                            (float)eps)));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rms_norm(const at::Tensor& x, const c10::optional<at::Tensor>& w, at::Tensor& out, double eps) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && x.scalar_type() == at::kBFloat16, "rms_norm: bf16 contiguous");
  const int C = (int)x.size(-1);
  TORCH_CHECK(C % 4 == 0, "rms_norm: C % 4 == 0");
  const long rows = x.numel() / C;
  c10::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  if (rows == 0) return;
  const float* wp = w.has_value() ? w->data_ptr<float>() : nullptr;
  OSP_ROW_DISPATCH(C, (rms_norm_kernel<MV><<<rows, kRowThreads, 0, stream>>>(
                          reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), wp,
                          reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), C, (float)eps)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void qk_norm_rope(at::Tensor& qkv, const at::Tensor& wq, const at::Tensor& wk, const at::Tensor& pos,
                  const at::Tensor& freqs, int64_t num_heads, double eps) {
  TORCH_CHECK(qkv.is_cuda() && qkv.is_contiguous() && qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 3,
              "qk_norm_rope: bf16 [B, n, 3C]");
  const int C = (int)(qkv.size(2) / 3);
  const int D = C / (int)num_heads;
  TORCH_CHECK(C % 4 == 0 && D % 4 == 0, "qk_norm_rope: C, D multiples of 4");
  const int n = (int)qkv.size(1);
  TORCH_CHECK(pos.scalar_type() == at::kInt && pos.numel() == 3L * n, "qk_norm_rope: pos int32 [n,3]");
  TORCH_CHECK(freqs.scalar_type() == at::kFloat && freqs.is_contiguous() && freqs.dim() == 3 && freqs.size(1) == D / 2 &&
              freqs.size(2) == 2, "qk_norm_rope: (cos, sin) table f32 [L, D/2, 2]");
  TORCH_CHECK(wq.scalar_type() == at::kFloat && wk.scalar_type() == at::kFloat, "qk_norm_rope: f32 weights");
  const long rows = qkv.size(0) * (long)n;
  c10::cuda::CUDAGuard guard(qkv.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  if (rows == 0) return;
  OSP_ROW_DISPATCH(C, (qk_norm_rope_kernel<MV><<<rows, kRowThreads, 0, stream>>>(
                          reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr()), wq.data_ptr<float>(),
                          wk.data_ptr<float>(), pos.data_ptr<int>(), reinterpret_cast<const float2*>(freqs.data_ptr<float>()), C, D, n,
                          (float)eps)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace osp
