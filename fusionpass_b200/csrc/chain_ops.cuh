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

// 0.5 x (1 + erf(x / sqrt 2)), each step rounded as written
__device__ __forceinline__ float op_gelu(float x) {
  const float t = __fmul_rn(x, 0.70710678118654752f);
  const float e = erff(t);
  return __fmul_rn(__fmul_rn(x, 0.5f), __fadd_rn(1.0f, e));
}
