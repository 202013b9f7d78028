// Elementwise kernels: fused CFG + Euler sampler step, HiF8 fake quantisation,
// GRPO SDE step + log-prob, fused AdamW.
//
// References: flow_matching.py:116-127, 178-184 (CFG, Euler);
// quant_cy_npu/base/cusrc/hif8_quant_op.h:88-151 (HiF8 grid); train_osp_RL.py:67-129
// (SDE step); torch.optim.AdamW as configured in train_osp.py:303-311.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tma_host.h"

namespace osp {

template <typename T>
__device__ __forceinline__ float ldf(const T* p, long i) { return static_cast<float>(p[i]); }
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p, long i) { return __bfloat162float(p[i]); }
template <typename T>
__device__ __forceinline__ void stf(T* p, long i, float v) { p[i] = static_cast<T>(v); }
template <>
__device__ __forceinline__ void stf<__nv_bfloat16>(__nv_bfloat16* p, long i, float v) { p[i] = __float2bfloat16(v); }

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16(v); }

// x ← x + (u + g·(c − u))·dt   (fp32 math, stored in the latent dtype)
template <typename TL, typename TP>
__global__ void cfg_euler_kernel(const TL* __restrict__ lat, const TP* __restrict__ cond, const TP* __restrict__ unc,
                                 TL* __restrict__ out, long n, float g, float dt) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float u = ldf(unc, i), c = ldf(cond, i);
    stf(out, i, ldf(lat, i) + (u + g * (c - u)) * dt);
  }
}

static int grid_for(long n) { return (int)std::min<long>((n + 255) / 256, 148L * 16); }

void cfg_euler(const at::Tensor& lat, const at::Tensor& cond, const at::Tensor& unc, at::Tensor& out, double g,
               double dt) {
  TORCH_CHECK(lat.is_contiguous() && cond.is_contiguous() && unc.is_contiguous() && out.is_contiguous(),
              "cfg_euler: contiguous tensors");
  TORCH_CHECK(cond.numel() == lat.numel() && unc.numel() == lat.numel(), "cfg_euler: shapes");
  TORCH_CHECK(cond.scalar_type() == unc.scalar_type(), "cfg_euler: cond/uncond dtypes");
  c10::cuda::CUDAGuard guard(lat.device());
  auto s = at::cuda::getCurrentCUDAStream();
  const long n = lat.numel();
  if (!n) return;
#define OSP_CFG(TL, TP)                                                                                   \
  cfg_euler_kernel<TL, TP><<<grid_for(n), 256, 0, s>>>(reinterpret_cast<const TL*>(lat.data_ptr()),       \
                                                      reinterpret_cast<const TP*>(cond.data_ptr()),      \
                                                      reinterpret_cast<const TP*>(unc.data_ptr()),       \
                                                      reinterpret_cast<TL*>(out.data_ptr()), n, (float)g, (float)dt)
  const bool lb = lat.scalar_type() == at::kBFloat16, pb = cond.scalar_type() == at::kBFloat16;
  TORCH_CHECK(lb || lat.scalar_type() == at::kFloat, "cfg_euler: latents f32/bf16");
  TORCH_CHECK(pb || cond.scalar_type() == at::kFloat, "cfg_euler: preds f32/bf16");
  if (lb && pb) OSP_CFG(__nv_bfloat16, __nv_bfloat16);
  else if (lb) OSP_CFG(__nv_bfloat16, float);
  else if (pb) OSP_CFG(float, __nv_bfloat16);
  else OSP_CFG(float, float);
#undef OSP_CFG
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------------ HiF8
// Round |v| to the HiF8 grid (Ascend kernel semantics): exponent e from the fp32
// bits; mantissa bits m = 3/2/1/0 for |e| ≤ 3/7/15/else; step 2^(max(e,−22)−m);
// round half away from zero; |v| < 2^-23 → 0; |v| ≥ 40960 → ±inf.
__device__ __forceinline__ float hif8_round_dev(float v) {
  const float a = fabsf(v);
  const int e = (int)((__float_as_uint(a) >> 23) & 0xFF) - 127;
  const int ae = abs(e);
  const int m = ae <= 3 ? 3 : (ae <= 7 ? 2 : (ae <= 15 ? 1 : 0));
  const int se = max(e, -22) - m;                          // step = 2^se
  // exact power-of-two scalings built from exponent bits: every finite |v| below the
  // overflow threshold has se in [-25, 15], so 2^±se is a normal float (larger |v| and
  // non-finite v are overwritten below)
  const int sc = min(max(se, -100), 100);
  float q = floorf(a * __int_as_float((127 - sc) << 23) + 0.5f);
  q = q * __int_as_float((127 + sc) << 23);
  if (a < 1.1920928955078125e-07f) q = 0.f;                // 2^-23
  if (a >= 40960.f) q = __int_as_float(0x7f800000);
  if (a != a) q = a;                                       // NaN stays NaN
  return copysignf(q, v);
}

__global__ void hif8_round_kernel(const float* __restrict__ x, float* __restrict__ out, long n, float s) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    out[i] = hif8_round_dev(x[i] * s);
}

void hif8_round(const at::Tensor& x, at::Tensor& out, double s) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous() && out.is_contiguous(), "hif8_round: f32");
  c10::cuda::CUDAGuard guard(x.device());
  const long n = x.numel();
  if (!n) return;
  hif8_round_kernel<<<grid_for(n), 256, 0, at::cuda::getCurrentCUDAStream()>>>(x.data_ptr<float>(),
                                                                               out.data_ptr<float>(), n, (float)s);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// amax(|x|) as the bit pattern of a non-negative float (monotone as uint).  16-byte loads,
// a block reduction, one atomic per block; the ragged tail (n mod 16/sizeof(T)) is
// scalar.
template <typename T>
__global__ void __launch_bounds__(256) absmax_kernel(const T* __restrict__ x, long n, unsigned* __restrict__ amax_bits) {
  constexpr int V = 16 / sizeof(T);
  const long nv = n / V;
  const long tid = blockIdx.x * (long)blockDim.x + threadIdx.x, stride = (long)gridDim.x * blockDim.x;
  float m = 0.f;
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  for (long i = tid; i < nv; i += stride) {
    const uint4 r = __ldg(xv + i);
    const T* e = reinterpret_cast<const T*>(&r);
#pragma unroll
    for (int k = 0; k < V; ++k) m = fmaxf(m, fabsf(to_f(e[k])));
  }
  for (long i = nv * V + tid; i < n; i += stride) m = fmaxf(m, fabsf(ldf(x, i)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float wm[8];
  if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? wm[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0) atomicMax(amax_bits, __float_as_uint(m));
  }
}

// hif8_round_dev(v·s) / s from the fp32 bits, without floor, conversions or a division per
// element.  For |v·s| = a with exponent byte b, the HiF8 grid step is 2^(max(e,−22) − m), so
// rounding half away from zero is "add half a step to the bits, clear the bits below the
// step" (a carry into the exponent field gives the next power of two, which is on the grid):
//   q_bits = (a_bits + half[b]) & mask[b]
// with half = mask = 0 below 2^-23 (q = 0), and at b = 104 (a in [2^-23, 2^-22)) the fixed
// result 2^-22.  Every q has at most three mantissa bits, so its top 11 bits index a table
// of RN(q / s), one true division per entry per block; |a| ≥ 40960 → ±inf by a compare, and
// exponent byte 255 (NaN) indexes NaN entries.  Bit-identical to hif8_round_dev(v·s) / s
// (tests/test_kernels_gpu.py::test_hif8_qdq_bit_exact_against_reference).
struct Hif8Tables {
  uint32_t half[256], mask[256];
  float val[2048];
};

__device__ __forceinline__ void hif8_tables_init(Hif8Tables* t, float s) {
  for (int b = threadIdx.x; b < 256; b += blockDim.x) {
    uint32_t h = 0u, m = 0u;
    if (b == 104) { h = 1u << 23; m = 0xFF800000u; }
    else if (b == 255) { h = 0u; m = 0xFFFFFFFFu; }
    else if (b > 104) {
      const int ae = abs(b - 127);
      const int mb = ae <= 3 ? 3 : (ae <= 7 ? 2 : (ae <= 15 ? 1 : 0));
      h = 1u << (22 - mb);
      m = ~((1u << (23 - mb)) - 1u);
    }
    t->half[b] = h;
    t->mask[b] = m;
  }
  for (int i = threadIdx.x; i < 2048; i += blockDim.x)
    t->val[i] = i >= 2040 ? __int_as_float(0x7fc00000) : __uint_as_float((uint32_t)i << 20) / s;
}

__device__ __forceinline__ float hif8_qdq_elem(float v, float s, const Hif8Tables* t) {
  const float y = v * s;
  const uint32_t ab = __float_as_uint(y) & 0x7fffffffu;
  const uint32_t b = ab >> 23;
  const uint32_t q = (ab + t->half[b]) & t->mask[b];
  float r = t->val[q >> 20];
  if (__uint_as_float(ab) >= 40960.f) r = __int_as_float(0x7f800000);
  return __uint_as_float(__float_as_uint(r) | (__float_as_uint(y) & 0x80000000u));
}

template <typename T>
__global__ void __launch_bounds__(256) hif8_qdq_kernel(const T* __restrict__ x, T* __restrict__ out, long n,
                                                       const unsigned* amax_bits, float scale_max) {
  constexpr int V = 16 / sizeof(T);
  const float amax = fmaxf(__uint_as_float(*amax_bits), 1e-8f);    // x.abs().amax().clamp(min=1e-8)
  // `scale_max / x_max` with a Python number over a tensor is reciprocal-then-multiply in
  // torch (Tensor.__rtruediv__), two roundings; the same here, so ties round alike
  const float s = (1.0f / amax) * scale_max;
  __shared__ Hif8Tables tb;
  hif8_tables_init(&tb, s);
  __syncthreads();
  const bool fast = s > 0.f && s < 3.0e38f;                        // else (amax = inf) the plain form
  const long nv = n / V;
  const long tid = blockIdx.x * (long)blockDim.x + threadIdx.x, stride = (long)gridDim.x * blockDim.x;
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  uint4* ov = reinterpret_cast<uint4*>(out);
  for (long i = tid; i < nv; i += stride) {
    uint4 r = __ldg(xv + i);
    T* e = reinterpret_cast<T*>(&r);
    if (fast) {
#pragma unroll
      for (int k = 0; k < V; ++k) e[k] = from_f<T>(hif8_qdq_elem(to_f(e[k]), s, &tb));
    } else {
#pragma unroll
      for (int k = 0; k < V; ++k) e[k] = from_f<T>(hif8_round_dev(to_f(e[k]) * s) / s);
    }
    ov[i] = r;
  }
  for (long i = nv * V + tid; i < n; i += stride)
    stf(out, i, fast ? hif8_qdq_elem(ldf(x, i), s, &tb) : hif8_round_dev(ldf(x, i) * s) / s);
}

// every block builds the 10 KB rounding tables, so the grid stays at a few blocks per SM
static int qdq_grid(long n) { return (int)std::min<long>((n / 8 + 255) / 256 + 1, 148L * 6); }

// Per-tensor dynamic-scale HiF8 quantise→dequantise (hif8_linear.py:42-50 semantics).
// The amax is reduced into a 4-byte device scratch word from the torch allocator.
void hif8_qdq(const at::Tensor& x, at::Tensor& out, double scale_max) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && out.is_contiguous() && x.scalar_type() == out.scalar_type(),
              "hif8_qdq: contiguous CUDA tensors of one dtype");
  c10::cuda::CUDAGuard guard(x.device());
  auto s = at::cuda::getCurrentCUDAStream();
  const long n = x.numel();
  if (!n) return;
  TORCH_CHECK((reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0 && (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0,
              "hif8_qdq: 16-byte aligned tensors");
  auto amax = at::zeros({1}, x.options().dtype(at::kInt));
  unsigned* ab = reinterpret_cast<unsigned*>(amax.data_ptr<int>());
  if (x.scalar_type() == at::kBFloat16) {
    auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
    absmax_kernel<<<grid_for(n), 256, 0, s>>>(xp, n, ab);
    hif8_qdq_kernel<<<qdq_grid(n), 256, 0, s>>>(xp, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), n, ab,
                                                (float)scale_max);
  } else {
    TORCH_CHECK(x.scalar_type() == at::kFloat, "hif8_qdq: f32/bf16");
    absmax_kernel<<<grid_for(n), 256, 0, s>>>(x.data_ptr<float>(), n, ab);
    hif8_qdq_kernel<<<qdq_grid(n), 256, 0, s>>>(x.data_ptr<float>(), out.data_ptr<float>(), n, ab, (float)scale_max);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------------ AdamW
// Fused decoupled-weight-decay Adam over one flat fp32 shard (torch.optim.AdamW
// update order):  p ← p·(1 − lr·wd);  m ← β1·m + (1−β1)·g;  v ← β2·v + (1−β2)·g²;
//                 p ← p − (lr/bc1)·m / (sqrt(v)/sqrt(bc2) + eps)
// g (bf16 or f32) is multiplied by `gscale` (the clip factor) on load.
template <typename TG>
__global__ void adamw_kernel(float* __restrict__ p, const TG* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, long n, float lr, float b1, float b2, float eps, float wd,
                             float bc1, float bc2_sqrt, float gscale) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float gi = ldf(g, i) * gscale;
    float pi = p[i] * (1.f - lr * wd);
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    pi -= (lr / bc1) * mi / (sqrtf(vi) / bc2_sqrt + eps);
    p[i] = pi;
  }
}

void adamw(at::Tensor& p, const at::Tensor& g, at::Tensor& m, at::Tensor& v, double lr, double b1, double b2,
           double eps, double wd, int64_t step, double gscale) {
  TORCH_CHECK(p.scalar_type() == at::kFloat && m.scalar_type() == at::kFloat && v.scalar_type() == at::kFloat,
              "adamw: f32 state");
  TORCH_CHECK(p.is_contiguous() && g.is_contiguous() && m.is_contiguous() && v.is_contiguous(), "adamw: contiguous");
  TORCH_CHECK(g.numel() == p.numel() && m.numel() == p.numel() && v.numel() == p.numel(), "adamw: sizes");
  c10::cuda::CUDAGuard guard(p.device());
  const long n = p.numel();
  if (!n) return;
  const float bc1 = 1.f - (float)std::pow(b1, (double)step);
  const float bc2s = (float)std::sqrt(1.0 - std::pow(b2, (double)step));
  auto s = at::cuda::getCurrentCUDAStream();
  if (g.scalar_type() == at::kBFloat16)
    adamw_kernel<<<grid_for(n), 256, 0, s>>>(p.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()),
                                             m.data_ptr<float>(), v.data_ptr<float>(), n, (float)lr, (float)b1,
                                             (float)b2, (float)eps, (float)wd, bc1, bc2s, (float)gscale);
  else
    adamw_kernel<<<grid_for(n), 256, 0, s>>>(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(),
                                             v.data_ptr<float>(), n, (float)lr, (float)b1, (float)b2, (float)eps,
                                             (float)wd, bc1, bc2s, (float)gscale);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------------ GRPO SDE
// Mix-GRPO SDE step with log-prob (train_osp_RL.py:67-129) for one step index:
//   std = σmin + (σmax−σmin)·σ;  mean = x·(1 + std²/(2σ)·dt) + v·(1 + std²(1−σ)/(2σ))·dt
//   prev = mean + std·sqrt(−dt)·ξ  (or the given prev sample)
//   logp[b] = mean over the sample of log N(prev; mean, (std·sqrt(−dt))²)
// logp must be zeroed by the caller (per-block partial sums are atomically added).
__global__ void sde_step_kernel(const float* __restrict__ x, const float* __restrict__ v, const float* __restrict__ xi,
                                const float* __restrict__ prev_in, float* __restrict__ prev_out,
                                float* __restrict__ mean_out, float* __restrict__ logp, long per_sample,
                                int batch, float sigma, float dt, float smin, float smax) {
  const float std_t = smin + (smax - smin) * sigma;
  const float sd = std_t * sqrtf(-dt);
  const float c1 = 1.f + std_t * std_t / (2.f * sigma) * dt;
  const float c2 = (1.f + std_t * std_t * (1.f - sigma) / (2.f * sigma)) * dt;
  const float lnorm = logf(sd) + 0.91893853320467274f;      // log(sqrt(2π))
  __shared__ float red[32];
  const long n = per_sample * batch;
  for (long base = (long)blockIdx.x * blockDim.x; base < n; base += (long)gridDim.x * blockDim.x) {
    const long i = base + threadIdx.x;
    float lp = 0.f;
    int b = -1;
    if (i < n) {
      b = (int)(i / per_sample);
      const float mu = x[i] * c1 + v[i] * c2;
      const float p = prev_in ? prev_in[i] : mu + sd * (xi ? xi[i] : 0.f);
      prev_out[i] = p;
      if (mean_out) mean_out[i] = mu;
      const float d = p - mu;
      lp = -(d * d) / (2.f * sd * sd) - lnorm;
    }
    // a block spans at most two samples (per_sample ≥ blockDim): reduce per sample id
    const int b0 = (int)(base / per_sample);
    float s0 = (b == b0) ? lp : 0.f;
    float s1 = (b == b0 + 1) ? lp : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    }
    const int w = threadIdx.x / 32, l = threadIdx.x % 32;
    __syncthreads();
    if (l == 0) { red[w] = s0; red[16 + w] = s1; }
    __syncthreads();
    if (threadIdx.x == 0) {
      float t0 = 0.f, t1 = 0.f;
      for (int k = 0; k < (int)blockDim.x / 32; ++k) { t0 += red[k]; t1 += red[16 + k]; }
      if (b0 < batch) atomicAdd(&logp[b0], t0 / (float)per_sample);
      if (b0 + 1 < batch && t1 != 0.f) atomicAdd(&logp[b0 + 1], t1 / (float)per_sample);
    }
  }
}

void sde_step(const at::Tensor& x, const at::Tensor& v, const c10::optional<at::Tensor>& xi,
              const c10::optional<at::Tensor>& prev_in, at::Tensor& prev_out, const c10::optional<at::Tensor>& mean_out,
              at::Tensor& logp, double sigma, double dt, double smin, double smax) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && v.scalar_type() == at::kFloat && x.is_contiguous() && v.is_contiguous(),
              "sde_step: f32 contiguous");
  const int batch = (int)x.size(0);
  const long per = x.numel() / batch;
  TORCH_CHECK(per >= 512, "sde_step: per-sample size must be >= 512");
  c10::cuda::CUDAGuard guard(x.device());
  const long n = x.numel();
  sde_step_kernel<<<grid_for(n), 512, 0, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), v.data_ptr<float>(), xi.has_value() ? xi->data_ptr<float>() : nullptr,
      prev_in.has_value() ? prev_in->data_ptr<float>() : nullptr, prev_out.data_ptr<float>(),
      mean_out.has_value() ? mean_out->data_ptr<float>() : nullptr, logp.data_ptr<float>(), per, batch, (float)sigma,
      (float)dt, (float)smin, (float)smax);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace osp

namespace osp {
// ------------------------------------------------------------------------------------ wait probes
// Fault-handling self-test without a GPU fault: one CTA waits on an mbarrier phase
// that nothing completes (mode 0) or on a global flag that nothing sets (mode 1),
// with a short limit; the bounded wait records its error code and the kernel
// returns normally, so the context stays usable.
__global__ void wait_probe_kernel(int mode, const int* flag, unsigned long long limit_ns, int* err) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    if (mode == 0) {
      mbar_init(&bar, 1);
      fence_mbar_init();
      mbar_wait(&bar, 0, err, kErrProbeMbar, limit_ns);
    } else {
      flag_wait(flag, 1, err, kErrProbeFlag, limit_ns);
    }
  }
}

void wait_probe(int64_t mode, const at::Tensor& flag, double limit_s) {
  c10::cuda::CUDAGuard guard(flag.device());
  wait_probe_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      (int)mode, flag.data_ptr<int>(), (unsigned long long)(limit_s * 1e9), error_word(flag.get_device()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
}  // namespace osp
