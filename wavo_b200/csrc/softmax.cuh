// Softmax arithmetic shared by the attention kernels: paired f32 instructions of sm_100
// (fma/add .f32x2), an FMA-pipe exp2 for part of the exponentials, a 3-input maximum.
#pragma once

#include <stdint.h>

#include "ptx.cuh"

namespace wv {

// ---- paired f32 arithmetic (sm_100: fma/add .f32x2, two lanes of work per instruction) ----------

__device__ __forceinline__ void fma2(float &d0, float &d1, float a0, float a1, float b0, float b1,
                                     float c0, float c1) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

__device__ __forceinline__ void add2(float &d0, float &d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// 2^x for two x in [-125, 8] on the FMA pipe: x = n + f with n = round(x), f in [-1/2, 1/2]; 2^f by
// a degree-4 polynomial (coefficients fitted here to the relative error of 2^f, max 7.7e-6 in
// f32), 2^n added to the exponent bits.
__device__ __forceinline__ void exp2_poly2(float &x0, float &x1) {
  constexpr float kRound = 12582912.0f;  // 1.5·2^23: x + kRound holds round(x) in its low bits
  x0 = fmaxf(x0, -125.0f);
  x1 = fmaxf(x1, -125.0f);
  float t0, t1, n0, n1, f0, f1;
  add2(t0, t1, x0, x1, kRound, kRound);
  add2(n0, n1, t0, t1, -kRound, -kRound);
  add2(f0, f1, x0, x1, -n0, -n1);
  float p0, p1;
  fma2(p0, p1, 0.009251425974071026f, 0.009251425974071026f, f0, f1, 0.055853113532066345f,
       0.055853113532066345f);
  fma2(p0, p1, p0, p1, f0, f1, 0.24031664431095123f, 0.24031664431095123f);
  fma2(p0, p1, p0, p1, f0, f1, 0.6931320428848267f, 0.6931320428848267f);
  fma2(p0, p1, p0, p1, f0, f1, 0.9999976754188538f, 0.9999976754188538f);
  x0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  x1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

// Sixteen exponentials 2^p[x] in place: the first 16 - NPOLY on the MUFU (ex2.approx), the last
// NPOLY (even) on the FMA pipe by exp2_poly2. Where the MUFU is not the bound (heads of 128, whose
// tensor work per score is twice that of heads of 64) the polynomial share relieves it; with heads
// of 64 the extra issue slots cost more than the MUFU time they save (measured).
template <int NPOLY>
__device__ __forceinline__ void exp2_16(float *p) {
  static_assert(NPOLY % 2 == 0 && NPOLY <= 16, "polynomial share");
#pragma unroll
  for (int x = 0; x < 16 - NPOLY; ++x) p[x] = ex2(p[x]);
#pragma unroll
  for (int x = 16 - NPOLY; x < 16; x += 2) exp2_poly2(p[x], p[x + 1]);
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

}  // namespace wv
