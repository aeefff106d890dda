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
// erfc(z) for t < 0 and 2 - erfc(z) otherwise; erfc(z) = u exp(-z^2 + P(u)) with
// u = 1 / (1 + z / 2) and P the degree-9 Chebyshev fit of Numerical Recipes'
// erfcc (fractional error below 1.2e-7 for every z >= 0).  One reciprocal and one
// exp2 on the MUFU and eleven FMAs: 48 vs 59 us for bias + GELU over f16 [16384, 3072]
// with erff, which made the chain instruction-bound.  Against 0.5 x (1 + erf) in
// double precision: max abs error 3.8e-7 (erff form 4.5e-7), max relative error
// 2.9e-6 for |x| < 5, where the erff form lost up to 5e-2 to the cancellation in
// 1 + erf(t) for negative t.
__device__ __forceinline__ float op_gelu(float x) {
  const float t = __fmul_rn(x, 0.70710678118654752f);
  const float z = fabsf(t);
  float u;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(u) : "f"(fmaf(0.5f, z, 1.0f)));
  float p = 0.17087277f;
  p = fmaf(p, u, -0.82215223f);
  p = fmaf(p, u, 1.48851587f);
  p = fmaf(p, u, -1.13520398f);
  p = fmaf(p, u, 0.27886807f);
  p = fmaf(p, u, -0.18628806f);
  p = fmaf(p, u, 0.09678418f);
  p = fmaf(p, u, 0.37409196f);
  p = fmaf(p, u, 1.00002368f);
  p = fmaf(p, u, -1.26551223f);
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(__fmul_rn(fmaf(-z, z, p), 1.44269504088896341f)));
  const float erfc_z = __fmul_rn(u, e);
  const float one_plus_erf = t < 0.0f ? erfc_z : __fsub_rn(2.0f, erfc_z);
  return __fmul_rn(__fmul_rn(x, 0.5f), one_plus_erf);
}

// op_gelu of two values, the erfc polynomial on packed f32 pairs: fma.rn.f32x2 rounds each
// lane exactly as fmaf, so both results equal op_gelu's bits
__device__ __forceinline__ void op_gelu2(float x0, float x1, float& y0, float& y1) {
  const float t0 = __fmul_rn(x0, 0.70710678118654752f), t1 = __fmul_rn(x1, 0.70710678118654752f);
  const float z0 = fabsf(t0), z1 = fabsf(t1);
  float u0, u1;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(u0) : "f"(fmaf(0.5f, z0, 1.0f)));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(u1) : "f"(fmaf(0.5f, z1, 1.0f)));
  const float c[10] = {0.17087277f, -0.82215223f, 1.48851587f, -1.13520398f, 0.27886807f,
                       -0.18628806f, 0.09678418f, 0.37409196f, 1.00002368f, -1.26551223f};
  float p0 = c[0], p1 = c[0];
#pragma unroll
  for (int k = 1; k < 10; ++k) {
    asm("{\n\t.reg .b64 a, b, d;\n\tmov.b64 a, {%0, %1};\n\tmov.b64 b, {%2, %3};\n\tmov.b64 d, {%4, %4};\n\t"
        "fma.rn.f32x2 a, a, b, d;\n\tmov.b64 {%0, %1}, a;\n\t}"
        : "+f"(p0), "+f"(p1)
        : "f"(u0), "f"(u1), "f"(c[k]));
  }
  float e0, e1;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(__fmul_rn(fmaf(-z0, z0, p0), 1.44269504088896341f)));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(__fmul_rn(fmaf(-z1, z1, p1), 1.44269504088896341f)));
  const float ec0 = __fmul_rn(u0, e0), ec1 = __fmul_rn(u1, e1);
  const float o0 = t0 < 0.0f ? ec0 : __fsub_rn(2.0f, ec0);
  const float o1 = t1 < 0.0f ? ec1 : __fsub_rn(2.0f, ec1);
  y0 = __fmul_rn(__fmul_rn(x0, 0.5f), o0);
  y1 = __fmul_rn(__fmul_rn(x1, 0.5f), o1);
}
