// Device math shared by the attention kernels (torch-free, so the kernels can be
// compiled on their own): MUFU exp2, packed fp32x2 FMA/ADD, 3-input max and a
// conversion-free exp2 on the FMA/ALU pipes.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace osp {


__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32x2 helpers (sm_100a FFMA2 / FADD2): two lanes of math per instruction.
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// 2^x for a pair on the FMA/ALU pipes, no MUFU and no float↔int conversion:
// adding 1.5·2²³ rounds x to the nearest integer n inside the mantissa of j, f = x − n
// lies in [−½, ½], a cubic gives 2^f, and (bits(j) << 23) = n << 23 (the magic
// constant's bits shift out) is added to the exponent field.  The cubic is our own
// relative-error minimax fit of 2^f on [−½, ½] (iteratively reweighted least squares),
// max relative error 7.5e-5 (1.4e-4 through this fp32 path), far below bf16's 3.9e-3.
// x is clamped at −125 so the exponent never underflows (such P entries are 0 in bf16).
__device__ __forceinline__ uint64_t exp2_fma2(float x0, float x1) {
  const uint64_t x = pk2(fmaxf(x0, -125.0f), fmaxf(x1, -125.0f));
  const uint64_t j = fadd2(x, pk2(12582912.0f, 12582912.0f));
  const uint64_t n = fadd2(j, pk2(-12582912.0f, -12582912.0f));
  const uint64_t f = ffma2(n, pk2(-1.0f, -1.0f), x);
  uint64_t p = ffma2(f, pk2(0.055170949548482895f, 0.055170949548482895f),
                     pk2(0.2426096349954605f, 0.2426096349954605f));
  p = ffma2(p, f, pk2(0.6932609677314758f, 0.6932609677314758f));
  p = ffma2(p, f, pk2(0.9999281764030457f, 0.9999281764030457f));
  float p0, p1, j0, j1;
  upk2(p, p0, p1);
  upk2(j, j0, j1);
  return pk2(__int_as_float(__float_as_int(p0) + (__float_as_int(j0) << 23)),
             __int_as_float(__float_as_int(p1) + (__float_as_int(j1) << 23)));
}


__device__ __forceinline__ float exp2_fma(float x) {     // scalar form of exp2_fma2
  x = fmaxf(x, -125.0f);
  const float j = x + 12582912.0f;
  const float f = x - (j - 12582912.0f);
  float p = fmaf(f, 0.055170949548482895f, 0.2426096349954605f);
  p = fmaf(p, f, 0.6932609677314758f);
  p = fmaf(p, f, 0.9999281764030457f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(j) << 23));
}

}  // namespace osp
