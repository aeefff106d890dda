// LayerNorm over the last axis for the `layer_norm` / `add_layer_norm` torch steps of
// extension plans (the BERT-style block), the latter with the add chain that feeds it.
//
// y = (x - mean) * rstd * w + b over each row of a contiguous [rows, cols] tensor,
// mean and biased variance in f32, rstd = 1 / sqrt(var + eps) correctly rounded
// (as torch.nn.functional.layer_norm computes them, in f32 for f16 input).  One warp
// per row holds the row in registers (VPL 8-element vectors per lane, cols <= 2048),
// so x is read once: the mean, then the variance as the mean of squared deviations
// (two passes over registers, no E[x^2] - mean^2 cancellation), then the normalised
// values.  Every load and store is a 16-byte vector; a warp covers 512 contiguous
// bytes per vector step.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/fpkern.h"
#include "internal.h"

namespace fpk {
namespace ln {

constexpr int kRowsPerCta = 4;  // one warp per row
constexpr int kMaxVpl = 8;      // 8-element vectors per lane: cols <= 32 * 8 * 8 = 2048

__device__ __forceinline__ void load8(const __half* p, float* a) {
  const uint4 u = __ldcs(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    a[2 * i] = f.x;
    a[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8(const float* p, float* a) {
  const float4 x = __ldcs(reinterpret_cast<const float4*>(p));
  const float4 y = __ldcs(reinterpret_cast<const float4*>(p) + 1);
  a[0] = x.x; a[1] = x.y; a[2] = x.z; a[3] = x.w; a[4] = y.x; a[5] = y.y; a[6] = y.z; a[7] = y.w;
}
// per-column parameters: kept in the caches (every row reads them)
__device__ __forceinline__ void load8c(const __half* p, float* a) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    a[2 * i] = f.x;
    a[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8c(const float* p, float* a) {
  const float4 x = __ldg(reinterpret_cast<const float4*>(p));
  const float4 y = __ldg(reinterpret_cast<const float4*>(p) + 1);
  a[0] = x.x; a[1] = x.y; a[2] = x.z; a[3] = x.w; a[4] = y.x; a[5] = y.y; a[6] = y.z; a[7] = y.w;
}
__device__ __forceinline__ void store8(__half* p, const float* a) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(a[2 * i], a[2 * i + 1]);
  __stcs(reinterpret_cast<uint4*>(p), u);
}
__device__ __forceinline__ void store8(float* p, const float* a) {
  __stcs(reinterpret_cast<float4*>(p), make_float4(a[0], a[1], a[2], a[3]));
  __stcs(reinterpret_cast<float4*>(p) + 1, make_float4(a[4], a[5], a[6], a[7]));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// The row's input is the sum of 1..4 addends, each full-shape ([rows, cols]) or per
// column (length cols), added in f32 in the given order (a residual and bias added
// before the normalisation: the add chain that feeds a LayerNorm, fused into it).
struct Addends {
  const void* p[4];
  uint32_t col_mask;  // bit i: addend i is per column
  int n;
};

template <typename T>
__device__ __forceinline__ void load_addend(const Addends& a, int i, int64_t row_off, int col, float* v) {
  const T* base = static_cast<const T*>(a.p[i]);
  if ((a.col_mask >> i) & 1u) load8c(base + col, v);
  else load8(base + row_off + col, v);
}

template <typename T, int VPL>
__global__ void __launch_bounds__(32 * kRowsPerCta) layer_norm_kernel(const Addends a, const T* __restrict__ w,
                                                                      const T* __restrict__ b, T* __restrict__ y,
                                                                      int64_t rows, int cols, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kRowsPerCta + (threadIdx.x >> 5);
  if (row >= rows) return;  // whole warps leave together: the shuffles below stay converged
  const int nv = cols / 8;
  const int64_t row_off = row * cols;
  float v[VPL * 8];
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int vi = k * 32 + lane;
    if (vi < nv) {
      load_addend<T>(a, 0, row_off, vi * 8, v + k * 8);
#pragma unroll
      for (int i = 1; i < 4; ++i) {  // constant indices keep the addend pointers in registers
        if (i < a.n) {
          float t[8];
          load_addend<T>(a, i, row_off, vi * 8, t);
#pragma unroll
          for (int e = 0; e < 8; ++e) v[k * 8 + e] = __fadd_rn(v[k * 8 + e], t[e]);
        }
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[k * 8 + e] = 0.0f;
    }
  }
  const float inv_n = 1.0f / static_cast<float>(cols);
  float s = 0.0f;
#pragma unroll
  for (int e = 0; e < VPL * 8; ++e) s = __fadd_rn(s, v[e]);
  const float mean = __fmul_rn(warp_sum(s), inv_n);
  float q = 0.0f;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    if (k * 32 + lane < nv) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = __fsub_rn(v[k * 8 + e], mean);
        q = __fmaf_rn(d, d, q);
      }
    }
  }
  const float var = __fmul_rn(warp_sum(q), inv_n);
  const float rstd = __frsqrt_rn(__fadd_rn(var, eps));
  T* yr = y + row_off;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int vi = k * 32 + lane;
    if (vi >= nv) continue;
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = __fmul_rn(__fsub_rn(v[k * 8 + e], mean), rstd);
    if (w != nullptr) {
      float wv[8], bv[8];
      load8c(w + vi * 8, wv);
      load8c(b + vi * 8, bv);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = __fmaf_rn(o[e], wv[e], bv[e]);
    }
    store8(yr + vi * 8, o);
  }
}

template <typename T, int VPL>
static int launch_vpl(const fpk_ln_desc* d, const Addends& a, const void* w, const void* b, void* y,
                      cudaStream_t s) {
  const int64_t grid = (d->rows + kRowsPerCta - 1) / kRowsPerCta;
  if (grid > 0x7fffffffLL) return FPK_ERR_UNSUPPORTED;
  layer_norm_kernel<T, VPL><<<static_cast<unsigned>(grid), 32 * kRowsPerCta, 0, s>>>(
      a, static_cast<const T*>(w), static_cast<const T*>(b), static_cast<T*>(y), d->rows, static_cast<int>(d->cols),
      d->eps);
  return cudaGetLastError() == cudaSuccess ? FPK_OK : FPK_ERR_CUDA;
}

template <typename T>
static int launch_t(const fpk_ln_desc* d, const Addends& a, const void* w, const void* b, void* y, cudaStream_t s) {
  const int vpl = static_cast<int>((d->cols / 8 + 31) / 32);
  switch (vpl) {
    case 1: return launch_vpl<T, 1>(d, a, w, b, y, s);
    case 2: return launch_vpl<T, 2>(d, a, w, b, y, s);
    case 3: return launch_vpl<T, 3>(d, a, w, b, y, s);
    case 4: return launch_vpl<T, 4>(d, a, w, b, y, s);
    case 5: return launch_vpl<T, 5>(d, a, w, b, y, s);
    case 6: return launch_vpl<T, 6>(d, a, w, b, y, s);
    case 7: return launch_vpl<T, 7>(d, a, w, b, y, s);
    case 8: return launch_vpl<T, 8>(d, a, w, b, y, s);
    default: return FPK_ERR_UNSUPPORTED;
  }
}

}  // namespace ln

int launch_layer_norm(const fpk_ln_desc* d, const void* const* addends, const int32_t* bcast, int n_addends,
                      const void* w, const void* b, void* y, cudaStream_t stream) {
  using namespace ln;
  if (d->cols <= 0 || d->cols % 8 || d->cols > 32 * 8 * kMaxVpl) return FPK_ERR_UNSUPPORTED;
  if (n_addends < 1 || n_addends > 4) return FPK_ERR_INVALID;
  Addends a{};
  a.n = n_addends;
  uintptr_t mis = reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(b);
  for (int i = 0; i < n_addends; ++i) {
    if (!addends[i] || (bcast[i] != FPK_BCAST_FULL && bcast[i] != FPK_BCAST_COL)) return FPK_ERR_INVALID;
    a.p[i] = addends[i];
    if (bcast[i] == FPK_BCAST_COL) a.col_mask |= 1u << i;
    mis |= reinterpret_cast<uintptr_t>(addends[i]);
  }
  if (d->rows == 0) return FPK_OK;
  if (mis % 16) return FPK_ERR_ALIGN;
  return d->dtype == FPK_F16 ? launch_t<__half>(d, a, w, b, y, stream) : launch_t<float>(d, a, w, b, y, stream);
}

}  // namespace fpk
