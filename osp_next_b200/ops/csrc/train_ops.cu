// Backward (and training-only forward) kernels of the DiT block's elementwise / row ops.
//
// The training forward runs the same fused kernels as inference; these are their
// gradients, replacing the chains of broadcast PyTorch ops that autograd would otherwise
// record (reference: the block is eager PyTorch under autocast, osp_next.py:926-957):
//
//   ln_modulate_bwd   y = LN(x)·(1+scale[b]) + shift[b]  →  dx, Σ_rows dy·x̂, Σ_rows dy
//   gated_add_fwd/bwd out = resid + y·gate[b]            →  dy = dout·gate, Σ_rows dout·y
//   qk_norm_rope_bwd  full-row RMSNorm(q)·w then 3-D RoPE →  d(raw q), Σ_rows (per-column dw)
//   gelu_tanh_bwd     h = gelu_tanh(pre)                  →  dpre
//   rms_norm_bwd      y = x·rsqrt(mean(x²)+eps)·w (row)   →  dx, Σ_rows dy·x̂
//
// Column reductions (gradients of per-batch modulation vectors and of norm weights) are
// written as per-CTA partial sums [B, chunks, C] that the caller sums over chunks, so the
// result does not depend on scheduling (no float atomics).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace osp {
namespace trn {

constexpr int kThreads = 256;
constexpr int kRowsPerCta = 32;

__device__ __forceinline__ float2 block_sum2(float a, float b, float2* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  __syncthreads();
  if (l == 0) red[w] = make_float2(a, b);
  __syncthreads();
  float2 s = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) { s.x += red[i].x; s.y += red[i].y; }
  return s;
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ld4(const __nv_bfloat16* p) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  float2 a = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u.x));
  float2 b = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void st4(__nv_bfloat16* p, float4 v) {
  uint2 u;
  u.x = pack_bf16x2(v.x, v.y);
  u.y = pack_bf16x2(v.z, v.w);
  *reinterpret_cast<uint2*>(p) = u;
}
__device__ __forceinline__ float4 f4(float a) { return make_float4(a, a, a, a); }
__device__ __forceinline__ float4 add4(float4 a, float4 b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }
__device__ __forceinline__ float4 mul4(float4 a, float4 b) { return make_float4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w); }
__device__ __forceinline__ float dot4(float4 a, float4 b) { return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w; }

// ---------------------------------------------------------------------------- LN + modulate
// grid (ceil(n / R), B); x fp32 [B, n, C]; dy bf16; scale fp32 [B, C].
template <int MAXV>
__global__ void __launch_bounds__(kThreads)
ln_modulate_bwd_kernel(const float* __restrict__ x, const __nv_bfloat16* __restrict__ dy,
                       const float* __restrict__ scale, float* __restrict__ dx, float* __restrict__ dscale_part,
                       float* __restrict__ dshift_part, int n, int C, float eps) {
  __shared__ float2 red[kThreads / 32];
  const int b = blockIdx.y;
  const int r0 = blockIdx.x * kRowsPerCta;
  const int r1 = min(n, r0 + kRowsPerCta);
  const int nv = C / 4;
  float4 s1[MAXV], acc_sc[MAXV], acc_sh[MAXV];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c4 = threadIdx.x + i * kThreads;
    s1[i] = c4 < nv ? add4(ld4(scale + (long)b * C + 4 * c4), f4(1.f)) : f4(0.f);
    acc_sc[i] = acc_sh[i] = f4(0.f);
  }
  const float inv_c = 1.0f / C;
  for (int r = r0; r < r1; ++r) {
    const long off = ((long)b * n + r) * C;
    float4 xv[MAXV], g[MAXV];
    float s = 0.f, ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c4 = threadIdx.x + i * kThreads;
      if (c4 < nv) {
        xv[i] = ld4(x + off + 4 * c4);
        s += xv[i].x + xv[i].y + xv[i].z + xv[i].w;
      }
    }
    const float mu = block_sum2(s, 0.f, red).x * inv_c;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c4 = threadIdx.x + i * kThreads;
      if (c4 < nv) {
        xv[i] = add4(xv[i], f4(-mu));
        ss += dot4(xv[i], xv[i]);
      }
    }
    const float rstd = rsqrtf(block_sum2(ss, 0.f, red).x * inv_c + eps);
    float sg = 0.f, sgx = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c4 = threadIdx.x + i * kThreads;
      if (c4 < nv) {
        xv[i] = mul4(xv[i], f4(rstd));                         // x̂
        const float4 d = ld4(dy + off + 4 * c4);
        acc_sh[i] = add4(acc_sh[i], d);
        acc_sc[i] = add4(acc_sc[i], mul4(d, xv[i]));
        g[i] = mul4(d, s1[i]);
        sg += g[i].x + g[i].y + g[i].z + g[i].w;
        sgx += dot4(g[i], xv[i]);
      }
    }
    const float2 t = block_sum2(sg, sgx, red);
    const float mg = t.x * inv_c, mgx = t.y * inv_c;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c4 = threadIdx.x + i * kThreads;
      if (c4 < nv) {
        float4 o;
        o.x = rstd * (g[i].x - mg - xv[i].x * mgx);
        o.y = rstd * (g[i].y - mg - xv[i].y * mgx);
        o.z = rstd * (g[i].z - mg - xv[i].z * mgx);
        o.w = rstd * (g[i].w - mg - xv[i].w * mgx);
        st4(dx + off + 4 * c4, o);
      }
    }
  }
  const long poff = ((long)b * gridDim.x + blockIdx.x) * C;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c4 = threadIdx.x + i * kThreads;
    if (c4 < nv) {
      st4(dscale_part + poff + 4 * c4, acc_sc[i]);
      st4(dshift_part + poff + 4 * c4, acc_sh[i]);
    }
  }
}

// ---------------------------------------------------------------------------- gated residual add
// out = resid + y·gate[b] (gate may be null = 1); all [B, n, C], y bf16, resid/out fp32.
__global__ void gated_add_fwd_kernel(const float* __restrict__ resid, const __nv_bfloat16* __restrict__ y,
                                     const float* __restrict__ gate, float* __restrict__ out, long total4, int n,
                                     int C) {
  const int nv = C / 4;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total4; i += (long)gridDim.x * blockDim.x) {
    const long e = 4 * i;
    const float4 r = ld4(resid + e);
    const float4 v = ld4(y + e);
    float4 g = f4(1.f);
    if (gate) {
      const long row = i / nv;
      const int b = (int)(row / n);
      g = ld4(gate + (long)b * C + 4 * (i % nv));
    }
    st4(out + e, add4(r, mul4(v, g)));
  }
}

// dy = dout·gate (bf16), dgate_part[b, chunk] = Σ_rows dout·y; grid (ceil(n / R), B)
template <int MAXV>
__global__ void __launch_bounds__(kThreads)
gated_add_bwd_kernel(const float* __restrict__ dout, const __nv_bfloat16* __restrict__ y,
                     const float* __restrict__ gate, __nv_bfloat16* __restrict__ dy, float* __restrict__ dgate_part,
                     int n, int C) {
  const int b = blockIdx.y;
  const int r0 = blockIdx.x * kRowsPerCta;
  const int r1 = min(n, r0 + kRowsPerCta);
  const int nv = C / 4;
  float4 gv[MAXV], acc[MAXV];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c4 = threadIdx.x + i * kThreads;
    gv[i] = c4 < nv ? ld4(gate + (long)b * C + 4 * c4) : f4(0.f);
    acc[i] = f4(0.f);
  }
  for (int r = r0; r < r1; ++r) {
    const long off = ((long)b * n + r) * C;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c4 = threadIdx.x + i * kThreads;
      if (c4 < nv) {
        const float4 d = ld4(dout + off + 4 * c4);
        acc[i] = add4(acc[i], mul4(d, ld4(y + off + 4 * c4)));
        st4(dy + off + 4 * c4, mul4(d, gv[i]));
      }
    }
  }
  const long poff = ((long)b * gridDim.x + blockIdx.x) * C;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c4 = threadIdx.x + i * kThreads;
    if (c4 < nv) st4(dgate_part + poff + 4 * c4, acc[i]);
  }
}

// ---------------------------------------------------------------------------- q/k RMSNorm + RoPE
// Forward (norm.cu qk_norm_rope): u = x·rstd(x)·w, out = rotate(u, θ(pos)).  Given g = dL/dout:
//   du = rotateᵀ(g);  dw += du·x·rstd;  dx = rstd·(du·w − x̂·mean(du·w·x̂)),  x̂ = x·rstd.
// One pass for q (part 0) or k (part 1); raw [rows, ld_raw] bf16 holds the pre-norm
// activations at column offset part·C; g [rows, C] (row stride ld_g); dx written at
// column offset part·C of dqkv [rows, ld_dx].  grid (ceil(n / R), B).
template <int MAXV, typename GT>
__global__ void __launch_bounds__(kThreads)
qk_norm_rope_bwd_kernel(const __nv_bfloat16* __restrict__ raw, int ld_raw, const GT* __restrict__ g, int ld_g,
                        const float* __restrict__ w, const int* __restrict__ pos, const float2* __restrict__ cstab,
                        __nv_bfloat16* __restrict__ dx, int ld_dx, float* __restrict__ dw_part, int part, int n,
                        int C, int D, float eps) {
  __shared__ float2 red[kThreads / 32];
  const int b = blockIdx.y;
  const int r0 = blockIdx.x * kRowsPerCta;
  const int r1 = min(n, r0 + kRowsPerCta);
  const int nv = C / 4;
  const int half = D / 2;
  const int ch = half / 3;
  const int ct = half - 2 * ch;
  float4 wv[MAXV], acc[MAXV];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c4 = threadIdx.x + i * kThreads;
    wv[i] = c4 < nv ? ld4(w + 4 * c4) : f4(0.f);
    acc[i] = f4(0.f);
  }
  const float inv_c = 1.0f / C;
  for (int r = r0; r < r1; ++r) {
    const long row = (long)b * n + r;
    const __nv_bfloat16* xr = raw + row * ld_raw + (long)part * C;
    float4 xv[MAXV], du[MAXV];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c4 = threadIdx.x + i * kThreads;
      if (c4 < nv) {
        xv[i] = ld4(xr + 4 * c4);
        ss += dot4(xv[i], xv[i]);
      }
    }
    const float rstd = rsqrtf(block_sum2(ss, 0.f, red).x * inv_c + eps);
    const int pt = pos[3 * r], ph = pos[3 * r + 1], pw = pos[3 * r + 2];
    float sdot = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c4 = threadIdx.x + i * kThreads;
      if (c4 < nv) {
        const int e = 4 * c4;
        const float4 gg = ld4(g + row * ld_g + e);
        float gv[4] = {gg.x, gg.y, gg.z, gg.w};
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const int j = ((e % D) >> 1) + p;
          const int prow = j < ct ? pt : (j < ct + ch ? ph : pw);
          const float2 t = cstab[(long)prow * half + j];
          const float cs = t.x, sn = t.y;
          const float g1 = gv[2 * p], g2 = gv[2 * p + 1];
          gv[2 * p] = g1 * cs + g2 * sn;                    // rotateᵀ
          gv[2 * p + 1] = -g1 * sn + g2 * cs;
        }
        du[i] = make_float4(gv[0], gv[1], gv[2], gv[3]);
        xv[i] = mul4(xv[i], f4(rstd));                     // x̂
        acc[i] = add4(acc[i], mul4(du[i], xv[i]));
        du[i] = mul4(du[i], wv[i]);                        // du·w
        sdot += dot4(du[i], xv[i]);
      }
    }
    const float m = block_sum2(sdot, 0.f, red).x * inv_c;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c4 = threadIdx.x + i * kThreads;
      if (c4 < nv) {
        float4 o;
        o.x = rstd * (du[i].x - xv[i].x * m);
        o.y = rstd * (du[i].y - xv[i].y * m);
        o.z = rstd * (du[i].z - xv[i].z * m);
        o.w = rstd * (du[i].w - xv[i].w * m);
        st4(dx + row * ld_dx + (long)part * C + 4 * c4, o);
      }
    }
  }
  const long poff = ((long)b * gridDim.x + blockIdx.x) * C;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c4 = threadIdx.x + i * kThreads;
    if (c4 < nv) st4(dw_part + poff + 4 * c4, acc[i]);
  }
}

// ---------------------------------------------------------------------------- GELU (tanh)
__global__ void gelu_tanh_bwd_kernel(const __nv_bfloat16* __restrict__ dh, const __nv_bfloat16* __restrict__ pre,
                                     __nv_bfloat16* __restrict__ dpre, long total4) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total4; i += (long)gridDim.x * blockDim.x) {
    const float4 d = ld4(dh + 4 * i);
    const float4 x = ld4(pre + 4 * i);
    float xs[4] = {x.x, x.y, x.z, x.w}, ds[4] = {d.x, d.y, d.z, d.w}, o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float u = k0 * (xs[j] + k1 * xs[j] * xs[j] * xs[j]);
      const float t = tanhf(u);
      const float du = k0 * (1.f + 3.f * k1 * xs[j] * xs[j]);
      o[j] = ds[j] * (0.5f * (1.f + t) + 0.5f * xs[j] * (1.f - t * t) * du);
    }
    st4(dpre + 4 * i, make_float4(o[0], o[1], o[2], o[3]));
  }
}

// ---------------------------------------------------------------------------- bias gradient
// db = Σ_rows g for g bf16 [M, N] (N % 8 == 0): CTA (column block of 256, row chunk of
// kBiasRows) → part[chunk, cols] fp32.  Each thread owns 8 adjacent columns (16-byte loads);
// the 8 warps take interleaved rows and are combined through shared memory.
constexpr int kBiasRows = 256;
__global__ void __launch_bounds__(256) bias_grad_kernel(const __nv_bfloat16* __restrict__ g, float* __restrict__ part,
                                                        long M, int N) {
  __shared__ float red[8][257];
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  const int c0 = blockIdx.x * 256 + l * 8;
  const long r0 = (long)blockIdx.y * kBiasRows;
  const long r1 = min(M, r0 + kBiasRows);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (c0 < N) {
#pragma unroll 4
    for (long r = r0 + w; r < r1; r += 8) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(g + r * N + c0));
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) red[w][l * 8 + i] = acc[i];
  __syncthreads();
  const int c = blockIdx.x * 256 + threadIdx.x;
  if (c < N) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += red[k][threadIdx.x];
    part[(long)blockIdx.y * N + c] = s;
  }
}

// ---------------------------------------------------------------------------- RMSNorm
// y = x̂·w, x̂ = x·rstd, rstd = rsqrt(mean(x²) + eps) over rows of C.
// dx = rstd·(g − x̂·mean(g·x̂)) with g = dy·w;  dw_part[chunk] = Σ_rows dy·x̂.
// x, dy bf16 [rows, C]; dx bf16; grid ceil(rows / R).
template <int MAXV>
__global__ void __launch_bounds__(kThreads)
rms_norm_bwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ dy,
                    const float* __restrict__ w, __nv_bfloat16* __restrict__ dx, float* __restrict__ dw_part,
                    int rows, int C, float eps) {
  __shared__ float2 red[kThreads / 32];
  const int r0 = blockIdx.x * kRowsPerCta;
  const int r1 = min(rows, r0 + kRowsPerCta);
  const int nv = C / 4;
  float4 wv[MAXV], acc[MAXV];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c4 = threadIdx.x + i * kThreads;
    wv[i] = c4 < nv ? (w ? ld4(w + 4 * c4) : f4(1.f)) : f4(0.f);
    acc[i] = f4(0.f);
  }
  const float inv_c = 1.0f / C;
  for (int r = r0; r < r1; ++r) {
    const long off = (long)r * C;
    float4 xv[MAXV], g[MAXV];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c4 = threadIdx.x + i * kThreads;
      if (c4 < nv) {
        xv[i] = ld4(x + off + 4 * c4);
        ss += dot4(xv[i], xv[i]);
      }
    }
    const float rstd = rsqrtf(block_sum2(ss, 0.f, red).x * inv_c + eps);
    float sgx = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c4 = threadIdx.x + i * kThreads;
      if (c4 < nv) {
        xv[i] = mul4(xv[i], f4(rstd));                         // x̂
        const float4 d = ld4(dy + off + 4 * c4);
        acc[i] = add4(acc[i], mul4(d, xv[i]));
        g[i] = mul4(d, wv[i]);
        sgx += dot4(g[i], xv[i]);
      }
    }
    const float mgx = block_sum2(sgx, 0.f, red).x * inv_c;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c4 = threadIdx.x + i * kThreads;
      if (c4 < nv) {
        float4 o;
        o.x = rstd * (g[i].x - xv[i].x * mgx);
        o.y = rstd * (g[i].y - xv[i].y * mgx);
        o.z = rstd * (g[i].z - xv[i].z * mgx);
        o.w = rstd * (g[i].w - xv[i].w * mgx);
        st4(dx + off + 4 * c4, o);
      }
    }
  }
  const long poff = (long)blockIdx.x * C;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c4 = threadIdx.x + i * kThreads;
    if (c4 < nv) st4(dw_part + poff + 4 * c4, acc[i]);
  }
}

}  // namespace trn

#define OSP_TRN_DISPATCH(C, ...)                                           \
  do {                                                                    \
    const int nvec = ((C) / 4 + trn::kThreads - 1) / trn::kThreads;       \
    if (nvec <= 1) { constexpr int MV = 1; __VA_ARGS__; }                  \
    else if (nvec <= 2) { constexpr int MV = 2; __VA_ARGS__; }             \
    else if (nvec <= 4) { constexpr int MV = 4; __VA_ARGS__; }             \
    else if (nvec <= 5) { constexpr int MV = 5; __VA_ARGS__; }             \
    else if (nvec <= 8) { constexpr int MV = 8; __VA_ARGS__; }             \
    else TORCH_CHECK(false, "row too long: C=", C);                        \
  } while (0)

static int chunks(int n) { return (n + trn::kRowsPerCta - 1) / trn::kRowsPerCta; }

static int ew_blocks(long total4) {
  return (int)std::min<long>((total4 + 255) / 256, 148L * 16);
}

// x fp32 [B,n,C], dy bf16 [B,n,C], scale fp32 [B,C] → dx fp32, partial sums [B, chunks(n), C]
void ln_modulate_bwd(const at::Tensor& x, const at::Tensor& dy, const at::Tensor& scale, at::Tensor& dx,
                     at::Tensor& dscale_part, at::Tensor& dshift_part, double eps) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.is_contiguous() && x.dim() == 3,
              "ln_modulate_bwd: x fp32 [B,n,C]");
  TORCH_CHECK(dy.scalar_type() == at::kBFloat16 && dy.is_contiguous() && dy.sizes() == x.sizes(), "ln_modulate_bwd: dy");
  const int B = (int)x.size(0), n = (int)x.size(1), C = (int)x.size(2);
  TORCH_CHECK(C % 4 == 0 && scale.is_contiguous() && scale.numel() == (int64_t)B * C, "ln_modulate_bwd: scale [B,C]");
  TORCH_CHECK(dx.is_contiguous() && dx.scalar_type() == at::kFloat && dx.sizes() == x.sizes(), "ln_modulate_bwd: dx");
  TORCH_CHECK(dscale_part.numel() == (int64_t)B * chunks(n) * C && dshift_part.numel() == dscale_part.numel(),
              "ln_modulate_bwd: partials [B, chunks, C]");
  c10::cuda::CUDAGuard guard(x.device());
  if (n == 0 || B == 0) return;
  dim3 grid(chunks(n), B);
  auto st = at::cuda::getCurrentCUDAStream();
  OSP_TRN_DISPATCH(C, (trn::ln_modulate_bwd_kernel<MV><<<grid, trn::kThreads, 0, st>>>(
                          x.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()),
                          scale.data_ptr<float>(), dx.data_ptr<float>(), dscale_part.data_ptr<float>(),
                          dshift_part.data_ptr<float>(), n, C, (float)eps)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gated_add_fwd(const at::Tensor& resid, const at::Tensor& y, const c10::optional<at::Tensor>& gate,
                   at::Tensor& out) {
  TORCH_CHECK(resid.is_cuda() && resid.scalar_type() == at::kFloat && resid.is_contiguous() && resid.dim() == 3,
              "gated_add: resid fp32 [B,n,C]");
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && y.is_contiguous() && y.sizes() == resid.sizes(), "gated_add: y");
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == at::kFloat && out.sizes() == resid.sizes(), "gated_add: out");
  const int B = (int)resid.size(0), n = (int)resid.size(1), C = (int)resid.size(2);
  TORCH_CHECK(C % 4 == 0, "gated_add: C % 4");
  if (gate.has_value()) TORCH_CHECK(gate->is_contiguous() && gate->numel() == (int64_t)B * C, "gated_add: gate [B,C]");
  c10::cuda::CUDAGuard guard(resid.device());
  const long total4 = resid.numel() / 4;
  if (total4 == 0) return;
  trn::gated_add_fwd_kernel<<<ew_blocks(total4), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      resid.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()),
      gate.has_value() ? gate->data_ptr<float>() : nullptr, out.data_ptr<float>(), total4, n, C);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gated_add_bwd(const at::Tensor& dout, const at::Tensor& y, const at::Tensor& gate, at::Tensor& dy,
                   at::Tensor& dgate_part) {
  TORCH_CHECK(dout.is_cuda() && dout.scalar_type() == at::kFloat && dout.is_contiguous() && dout.dim() == 3,
              "gated_add_bwd: dout fp32 [B,n,C]");
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && y.is_contiguous() && y.sizes() == dout.sizes(), "gated_add_bwd: y");
  TORCH_CHECK(dy.scalar_type() == at::kBFloat16 && dy.is_contiguous() && dy.sizes() == dout.sizes(),
              "gated_add_bwd: dy");
  const int B = (int)dout.size(0), n = (int)dout.size(1), C = (int)dout.size(2);
  TORCH_CHECK(C % 4 == 0 && gate.is_contiguous() && gate.numel() == (int64_t)B * C, "gated_add_bwd: gate [B,C]");
  TORCH_CHECK(dgate_part.numel() == (int64_t)B * chunks(n) * C, "gated_add_bwd: partials");
  c10::cuda::CUDAGuard guard(dout.device());
  if (n == 0 || B == 0) return;
  dim3 grid(chunks(n), B);
  auto st = at::cuda::getCurrentCUDAStream();
  OSP_TRN_DISPATCH(C, (trn::gated_add_bwd_kernel<MV><<<grid, trn::kThreads, 0, st>>>(
                          dout.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()),
                          gate.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dy.data_ptr()),
                          dgate_part.data_ptr<float>(), n, C)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// raw [B·n, ld_raw] bf16 pre-norm q|k; g [B,n,C] grad of the rotated output (bf16 or fp32,
// row stride ld_g); writes dqkv[:, part·C : (part+1)·C] and dw_part [B, chunks, C].
void qk_norm_rope_bwd(const at::Tensor& raw, const at::Tensor& g, const at::Tensor& w, const at::Tensor& pos,
                      const at::Tensor& freqs, at::Tensor& dqkv, at::Tensor& dw_part, int64_t part, int64_t B,
                      int64_t n, int64_t C, int64_t D, double eps) {
  TORCH_CHECK(raw.is_cuda() && raw.scalar_type() == at::kBFloat16 && raw.stride(-1) == 1, "qk_norm_rope_bwd: raw");
  TORCH_CHECK(dqkv.scalar_type() == at::kBFloat16 && dqkv.stride(-1) == 1, "qk_norm_rope_bwd: dqkv");
  TORCH_CHECK(g.stride(-1) == 1 && (g.scalar_type() == at::kBFloat16 || g.scalar_type() == at::kFloat),
              "qk_norm_rope_bwd: g bf16/fp32 with contiguous rows");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && w.numel() == C, "qk_norm_rope_bwd: w fp32 [C]");
  TORCH_CHECK(pos.scalar_type() == at::kInt && pos.is_contiguous() && pos.numel() == 3 * n, "qk_norm_rope_bwd: pos");
  TORCH_CHECK(freqs.scalar_type() == at::kFloat && freqs.is_contiguous() && freqs.dim() == 3 && freqs.size(2) == 2,
              "qk_norm_rope_bwd: (cos, sin) table f32 [L, D/2, 2]");
  TORCH_CHECK(C % 4 == 0 && D % 4 == 0 && dw_part.numel() == B * chunks((int)n) * C, "qk_norm_rope_bwd: shapes");
  c10::cuda::CUDAGuard guard(raw.device());
  if (n == 0 || B == 0) return;
  const int ld_raw = (int)raw.stride(-2), ld_dx = (int)dqkv.stride(-2), ld_g = (int)g.stride(-2);
  dim3 grid(chunks((int)n), (unsigned)B);
  auto st = at::cuda::getCurrentCUDAStream();
  const auto* rp = reinterpret_cast<const __nv_bfloat16*>(raw.data_ptr());
  auto* dp = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  if (g.scalar_type() == at::kBFloat16) {
    OSP_TRN_DISPATCH((int)C, (trn::qk_norm_rope_bwd_kernel<MV, __nv_bfloat16><<<grid, trn::kThreads, 0, st>>>(
                                 rp, ld_raw, reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), ld_g,
                                 w.data_ptr<float>(), pos.data_ptr<int>(), reinterpret_cast<const float2*>(freqs.data_ptr<float>()), dp, ld_dx,
                                 dw_part.data_ptr<float>(), (int)part, (int)n, (int)C, (int)D, (float)eps)));
  } else {
    OSP_TRN_DISPATCH((int)C, (trn::qk_norm_rope_bwd_kernel<MV, float><<<grid, trn::kThreads, 0, st>>>(
                                 rp, ld_raw, g.data_ptr<float>(), ld_g, w.data_ptr<float>(), pos.data_ptr<int>(),
                                 reinterpret_cast<const float2*>(freqs.data_ptr<float>()), dp, ld_dx,
                                 dw_part.data_ptr<float>(), (int)part, (int)n,
                                 (int)C, (int)D, (float)eps)));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gelu_tanh_bwd(const at::Tensor& dh, const at::Tensor& pre, at::Tensor& dpre) {
  TORCH_CHECK(dh.is_cuda() && dh.scalar_type() == at::kBFloat16 && pre.scalar_type() == at::kBFloat16 &&
              dpre.scalar_type() == at::kBFloat16 && dh.is_contiguous() && pre.is_contiguous() &&
              dpre.is_contiguous() && dh.numel() == pre.numel() && dpre.numel() == pre.numel() &&
              pre.numel() % 4 == 0, "gelu_tanh_bwd: contiguous bf16 of equal size (multiple of 4)");
  c10::cuda::CUDAGuard guard(dh.device());
  const long total4 = pre.numel() / 4;
  if (total4 == 0) return;
  trn::gelu_tanh_bwd_kernel<<<ew_blocks(total4), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dh.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(pre.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(dpre.data_ptr()), total4);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// g bf16 [M, N] contiguous (N % 8 == 0) → part fp32 [ceil(M / 256), N] column sums per row chunk
void bias_grad(const at::Tensor& g, at::Tensor& part) {
  TORCH_CHECK(g.is_cuda() && g.scalar_type() == at::kBFloat16 && g.is_contiguous() && g.dim() == 2,
              "bias_grad: contiguous bf16 [M, N]");
  const long M = g.size(0);
  const int N = (int)g.size(1);
  const long nchunk = (M + trn::kBiasRows - 1) / trn::kBiasRows;
  TORCH_CHECK(N % 8 == 0 && part.scalar_type() == at::kFloat && part.is_contiguous() && part.numel() == nchunk * N,
              "bias_grad: N % 8 and part fp32 [ceil(M/256), N]");
  c10::cuda::CUDAGuard guard(g.device());
  if (M == 0 || N == 0) return;
  dim3 grid((unsigned)((N + 255) / 256), (unsigned)nchunk);
  trn::bias_grad_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), part.data_ptr<float>(), M, N);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// x, dy bf16 [rows, C] contiguous, w fp32 [C] (or undefined) → dx bf16, dw_part fp32 [chunks(rows), C]
void rms_norm_bwd(const at::Tensor& x, const at::Tensor& dy, const c10::optional<at::Tensor>& w, at::Tensor& dx,
                  at::Tensor& dw_part, double eps) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && dy.scalar_type() == at::kBFloat16 &&
              dx.scalar_type() == at::kBFloat16 && x.is_contiguous() && dy.is_contiguous() && dx.is_contiguous(),
              "rms_norm_bwd: contiguous bf16 x, dy, dx");
  const int C = (int)x.size(-1);
  const long rows = x.numel() / C;
  TORCH_CHECK(C % 4 == 0 && dy.numel() == x.numel() && dx.numel() == x.numel(), "rms_norm_bwd: shapes");
  TORCH_CHECK(dw_part.scalar_type() == at::kFloat && dw_part.is_contiguous() &&
              dw_part.numel() == (long)chunks((int)rows) * C, "rms_norm_bwd: dw_part [chunks, C] fp32");
  const float* wp = nullptr;
  if (w.has_value() && w->defined()) {
    TORCH_CHECK(w->scalar_type() == at::kFloat && w->is_contiguous() && w->numel() == C, "rms_norm_bwd: w fp32 [C]");
    wp = w->data_ptr<float>();
  }
  c10::cuda::CUDAGuard guard(x.device());
  if (rows == 0) return;
  auto st = at::cuda::getCurrentCUDAStream();
  const int grid = chunks((int)rows);
  OSP_TRN_DISPATCH(C, (trn::rms_norm_bwd_kernel<MV><<<grid, trn::kThreads, 0, st>>>(
                          reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                          reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), wp,
                          reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), dw_part.data_ptr<float>(), (int)rows, C,
                          (float)eps)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace osp
