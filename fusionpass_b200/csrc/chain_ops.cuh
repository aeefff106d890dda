// f32 element ops of the fused chain (lib/Plan/TritonEmitter.cpp:186-226 emits
// the same ops as Triton expressions; python/fusionpass/kernels.py:130-180).
//
// One definition for both execution tiers: the interpreter kernels in chain.cu
// include this header, and the per-program kernels compiled at run time
// (chain_jit.cu) embed this file's text, so both produce identical bits.
#pragma once

// max(x, 0) that propagates NaN like the reference's numpy maximum (one instruction)
__device__ __forceinline__ float op_relu(float x) {
  float y;
  asm("max.NaN.f32 %0, %1, 0f00000000;" : "=f"(y) : "f"(x));
  return y;
}

// 0.5 x (1 + erf(x / sqrt 2)).  With t = x / sqrt 2 and z = |t|, 1 + erf(t) is
// erfc(z) for t < 0 and 2 - erfc(z) otherwise, and erfc(z) is taken as
// (1 + a1 z + ... + a6 z^6)^-16, Abramowitz & Stegun 7.1.28 (Hastings' rational
// form; |error| <= 3e-7 for every z >= 0): one reciprocal on the MUFU, a degree-6
// polynomial and four squarings on the FMA pipe, and no exponential.  The form
// with an exponential (Numerical Recipes' erfcc: a reciprocal and an exp2 per
// element) left bias + GELU over f16 [16384, 3072] instruction-bound at 45.7 us.
// Against 0.5 x (1 + erf) in double precision: max abs error 8.2e-7; max relative
// error 6.6e-5 for |x| < 3 (for x < -3, where the result is below 6e-3 in
// magnitude, the absolute bound is what holds).
#define FPK_GELU_A1 0.0705230784f
#define FPK_GELU_A2 0.0422820123f
#define FPK_GELU_A3 0.0092705272f
#define FPK_GELU_A4 0.0001520143f
#define FPK_GELU_A5 0.0002765672f
#define FPK_GELU_A6 0.0000430638f

__device__ __forceinline__ float op_gelu(float x) {
  const float t = __fmul_rn(x, 0.70710678118654752f);
  const float z = fabsf(t);
  float p = fmaf(FPK_GELU_A6, z, FPK_GELU_A5);
  p = fmaf(p, z, FPK_GELU_A4);
  p = fmaf(p, z, FPK_GELU_A3);
  p = fmaf(p, z, FPK_GELU_A2);
  p = fmaf(p, z, FPK_GELU_A1);
  p = fmaf(p, z, 1.0f);
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(p));
  r = __fmul_rn(r, r);
  r = __fmul_rn(r, r);
  r = __fmul_rn(r, r);
  const float erfc_z = __fmul_rn(r, r);
  const float one_plus_erf = t < 0.0f ? erfc_z : __fsub_rn(2.0f, erfc_z);
  return __fmul_rn(__fmul_rn(x, 0.5f), one_plus_erf);
}

// packed f32 pair helpers: each lane rounds exactly as the scalar op
__device__ __forceinline__ void fpk_fma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c) {
  asm("{\n\t.reg .b64 a, b, c;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\tmov.b64 c, {%6, %6};\n\t"
      "fma.rn.f32x2 a, a, b, c;\n\tmov.b64 {%0, %1}, a;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c));
}
__device__ __forceinline__ void fpk_mul2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 a, b;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
      "mul.rn.f32x2 a, a, b;\n\tmov.b64 {%0, %1}, a;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// op_gelu of two values on packed f32 pairs (fma.rn.f32x2 / mul.rn.f32x2 round each
// lane exactly as fmaf / __fmul_rn), so both results equal op_gelu's bits
__device__ __forceinline__ void op_gelu2(float x0, float x1, float& y0, float& y1) {
  float t0, t1;
  fpk_mul2(t0, t1, x0, x1, 0.70710678118654752f, 0.70710678118654752f);
  const float z0 = fabsf(t0), z1 = fabsf(t1);
  float p0, p1;
  fpk_fma2(p0, p1, FPK_GELU_A6, FPK_GELU_A6, z0, z1, FPK_GELU_A5);
  fpk_fma2(p0, p1, p0, p1, z0, z1, FPK_GELU_A4);
  fpk_fma2(p0, p1, p0, p1, z0, z1, FPK_GELU_A3);
  fpk_fma2(p0, p1, p0, p1, z0, z1, FPK_GELU_A2);
  fpk_fma2(p0, p1, p0, p1, z0, z1, FPK_GELU_A1);
  fpk_fma2(p0, p1, p0, p1, z0, z1, 1.0f);
  float r0, r1;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(p0));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(p1));
  fpk_mul2(r0, r1, r0, r1, r0, r1);
  fpk_mul2(r0, r1, r0, r1, r0, r1);
  fpk_mul2(r0, r1, r0, r1, r0, r1);
  fpk_mul2(r0, r1, r0, r1, r0, r1);
  const float o0 = t0 < 0.0f ? r0 : __fsub_rn(2.0f, r0);
  const float o1 = t1 < 0.0f ? r1 : __fsub_rn(2.0f, r1);
  float h0, h1;
  fpk_mul2(h0, h1, x0, x1, 0.5f, 0.5f);
  fpk_mul2(y0, y1, h0, h1, o0, o1);
}
