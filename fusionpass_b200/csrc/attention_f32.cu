// f32 fp_attention on FP32 FMA (CUDA cores).
//
// Same algorithm as the reference kernel (lib/Plan/TritonEmitter.cpp:73-104,
// twin python/fusionpass/kernels.py:58-89): one CTA per (64 query rows,
// batch*head), K/V streamed in 64-key tiles through shared memory, online
// softmax with f32 running max m_i, sum l_i and accumulator acc, IEEE f32 dot
// products, out-of-range keys at -inf, one division acc / l_i at the end.
//
// 256 threads as a 16 x 16 grid: thread (ty, tx) owns query rows RPT*ty ..
// RPT*ty+RPT-1, score columns tx + 16*c and output columns tx + 16*c.  The 16
// threads of a row form one half-warp, so the row max / sum are half-warp
// shuffles.  RPT = 4 (64-row query tiles) normally; RPT = 1 (16-row tiles, four
// times the CTAs) when the 64-row grid would leave most SMs idle.  With 16-row
// tiles a CTA may also split its key tiles over G groups of 256 threads (key tile
// j to group j % G, each group with its own K / V / P buffers and its own named
// barrier); the groups' (m, l, acc) are merged through shared memory at the end:
// m = max m_g, l = sum l_g e^(m_g - m), acc = sum acc_g e^(m_g - m).
#include <atomic>
#include <cmath>

#include "common.cuh"
#include "internal.h"

namespace fpk {
namespace attn32 {

constexpr int kBN = 64;
constexpr int kThreads = 256;

struct Params {
  const float* q;
  const float* k;
  const float* v;
  float* o;
  int64_t heads, seq, num_mtiles;
  int64_t qs[3], ks[3], vs[3], os[3];  // b, h, s element strides
  float scale;
  int vec4;  // k and v bases and strides allow 16-byte loads
};

// floats of one group's K / V / P buffers
template <int D, int RPT>
__host__ __device__ constexpr int group_floats() {
  return D * (kBN + 1) + kBN * D + 16 * RPT * (kBN + 1);
}

// threads of group `grp` only (named barrier 1 + grp; barrier 0 is __syncthreads)
template <int G>
__device__ __forceinline__ void group_sync(int grp) {
  if constexpr (G == 1) {
    __syncthreads();
  } else {
    asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(kThreads) : "memory");
  }
}

template <int D, int RPT, int G>
__global__ void __launch_bounds__(kThreads * G) attn_f32_kernel(const __grid_constant__ Params p) {
  static_assert(G == 1 || RPT == 1, "key groups are used with 16-row tiles");
  constexpr int DC = D / 16;  // output columns per thread
  constexpr int kBM = 16 * RPT;  // query rows per CTA
  extern __shared__ __align__(16) float smem_f[];
  const int grp = G == 1 ? 0 : static_cast<int>(threadIdx.x) / kThreads;
  float* gbuf = smem_f + D * kBM + grp * group_floats<D, RPT>();
  float(*Qs)[kBM] = reinterpret_cast<float(*)[kBM]>(smem_f);                      // Qs[d][row]
  float(*Ks)[kBN + 1] = reinterpret_cast<float(*)[kBN + 1]>(gbuf);                // Ks[d][key]
  float(*Vs)[D] = reinterpret_cast<float(*)[D]>(gbuf + D * (kBN + 1));           // Vs[key][d]
  float(*Ps)[kBN + 1] = reinterpret_cast<float(*)[kBN + 1]>(gbuf + D * (kBN + 1) + kBN * D);

  const int tid = static_cast<int>(threadIdx.x) % kThreads;  // thread within its group
  const int tx = tid & 15;
  const int ty = tid >> 4;
  const int64_t bh = blockIdx.x / p.num_mtiles;
  const int64_t m0 = (blockIdx.x % p.num_mtiles) * kBM;
  const int64_t b = bh / p.heads, h = bh % p.heads;
  const float* qb = p.q + b * p.qs[0] + h * p.qs[1];
  const float* kb = p.k + b * p.ks[0] + h * p.ks[1];
  const float* vb = p.v + b * p.vs[0] + h * p.vs[1];
  float* ob = p.o + b * p.os[0] + h * p.os[1];
  const int64_t S = p.seq;

  // Q tile -> Qs (rows past S read as 0, kernels.py:66-67)
  for (int idx = static_cast<int>(threadIdx.x); idx < kBM * D; idx += kThreads * G) {
    const int r = idx % kBM, d = idx / kBM;
    const int64_t gr = m0 + r;
    Qs[d][r] = gr < S ? qb[gr * p.qs[2] + d] : 0.0f;
  }

  float m_i[RPT], l_i[RPT], acc[RPT][DC];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    m_i[i] = -INFINITY;
    l_i[i] = 0.0f;
#pragma unroll
    for (int c = 0; c < DC; ++c) acc[i][c] = 0.0f;
  }

  if constexpr (G > 1) __syncthreads();  // Qs written by every group
  for (int64_t n0 = static_cast<int64_t>(grp) * kBN; n0 < S; n0 += static_cast<int64_t>(G) * kBN) {
    group_sync<G>(grp);  // previous tile fully consumed (and Qs written on the first pass)
    if (p.vec4) {
      // 16-byte loads, all of a thread's loads issued before any is stored: one memory
      // latency per key tile instead of one per element
      constexpr int kPer = kBN * D / 4 / kThreads;  // float4 of K (and of V) per thread
      float4 kv4[kPer], vv4[kPer];
#pragma unroll
      for (int u = 0; u < kPer; ++u) {
        const int idx = tid + u * kThreads;
        const int j = idx / (D / 4), d = (idx % (D / 4)) * 4;
        const int64_t gj = n0 + j;
        const bool ok = gj < S;
        kv4[u] = ok ? *reinterpret_cast<const float4*>(kb + gj * p.ks[2] + d) : make_float4(0.f, 0.f, 0.f, 0.f);
        vv4[u] = ok ? *reinterpret_cast<const float4*>(vb + gj * p.vs[2] + d) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kPer; ++u) {
        const int idx = tid + u * kThreads;
        const int j = idx / (D / 4), d = (idx % (D / 4)) * 4;
        Ks[d][j] = kv4[u].x;
        Ks[d + 1][j] = kv4[u].y;
        Ks[d + 2][j] = kv4[u].z;
        Ks[d + 3][j] = kv4[u].w;
        *reinterpret_cast<float4*>(&Vs[j][d]) = vv4[u];
      }
    } else {
      for (int idx = tid; idx < kBN * D; idx += kThreads) {
        const int j = idx / D, d = idx % D;
        const int64_t gj = n0 + j;
        const bool ok = gj < S;
        Ks[d][j] = ok ? kb[gj * p.ks[2] + d] : 0.0f;
        Vs[j][d] = ok ? vb[gj * p.vs[2] + d] : 0.0f;
      }
    }
    group_sync<G>(grp);

    float s[RPT][4];
#pragma unroll
    for (int i = 0; i < RPT; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[i][c] = 0.0f;
#pragma unroll 8
    for (int d = 0; d < D; ++d) {
      float qa[RPT];
      if constexpr (RPT == 4) {
        const float4 qv = *reinterpret_cast<const float4*>(&Qs[d][4 * ty]);
        qa[0] = qv.x;
        qa[1] = qv.y;
        qa[2] = qv.z;
        qa[3] = qv.w;
      } else {
#pragma unroll
        for (int i = 0; i < RPT; ++i) qa[i] = Qs[d][RPT * ty + i];
      }
      float kv[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) kv[c] = Ks[d][tx + 16 * c];
#pragma unroll
      for (int i = 0; i < RPT; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) s[i][c] = fmaf(qa[i], kv[c], s[i][c]);
    }

    float alpha[RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const bool ok = n0 + tx + 16 * c < S;
        s[i][c] = ok ? s[i][c] * p.scale : -INFINITY;  // kernels.py:76-77
        mx = fmaxf(mx, s[i][c]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m_i[i], mx);
      alpha[i] = expf(m_i[i] - m_new);
      float rs = 0.0f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float pv = expf(s[i][c] - m_new);
        Ps[RPT * ty + i][tx + 16 * c] = pv;
        rs += pv;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      l_i[i] = l_i[i] * alpha[i] + rs;
      m_i[i] = m_new;
    }
    group_sync<G>(grp);

    float pv_acc[RPT][DC];
#pragma unroll
    for (int i = 0; i < RPT; ++i)
#pragma unroll
      for (int c = 0; c < DC; ++c) pv_acc[i][c] = 0.0f;
#pragma unroll 4
    for (int j = 0; j < kBN; ++j) {
      float pr[RPT];
#pragma unroll
      for (int i = 0; i < RPT; ++i) pr[i] = Ps[RPT * ty + i][j];
#pragma unroll
      for (int c = 0; c < DC; ++c) {
        const float vv = Vs[j][tx + 16 * c];
#pragma unroll
        for (int i = 0; i < RPT; ++i) pv_acc[i][c] = fmaf(pr[i], vv, pv_acc[i][c]);
      }
    }
#pragma unroll
    for (int i = 0; i < RPT; ++i)
#pragma unroll
      for (int c = 0; c < DC; ++c) acc[i][c] = acc[i][c] * alpha[i] + pv_acc[i][c];
  }

  if constexpr (G > 1) {
    // merge the groups: each group's (m, l, acc) of its rows into its own K buffer
    __syncthreads();
    {
      float* r = gbuf + ty * (D + 2);  // [kBM][D + 2]: acc, then m and l
#pragma unroll
      for (int c = 0; c < DC; ++c) r[tx + 16 * c] = acc[0][c];
      if (tx == 0) {
        r[D] = m_i[0];
        r[D + 1] = l_i[0];
      }
    }
    __syncthreads();
    if (grp != 0) return;
    float m = -INFINITY;
#pragma unroll
    for (int q = 0; q < G; ++q) m = fmaxf(m, smem_f[D * kBM + q * group_floats<D, RPT>() + ty * (D + 2) + D]);
    float l = 0.0f, a[DC];
#pragma unroll
    for (int c = 0; c < DC; ++c) a[c] = 0.0f;
#pragma unroll
    for (int q = 0; q < G; ++q) {
      const float* r = smem_f + D * kBM + q * group_floats<D, RPT>() + ty * (D + 2);
      const float w = r[D] == -INFINITY ? 0.0f : expf(r[D] - m);  // a group without keys adds nothing
      l += r[D + 1] * w;
#pragma unroll
      for (int c = 0; c < DC; ++c) a[c] += r[tx + 16 * c] * w;
    }
    l_i[0] = l;
#pragma unroll
    for (int c = 0; c < DC; ++c) acc[0][c] = a[c];
  }
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int64_t gr = m0 + RPT * ty + i;
    if (gr >= S) continue;
#pragma unroll
    for (int c = 0; c < DC; ++c) ob[gr * p.os[2] + tx + 16 * c] = acc[i][c] / l_i[i];
  }
}

template <int D, int RPT, int G>
constexpr int smem_bytes() {
  constexpr int kBM = 16 * RPT;
  return static_cast<int>(sizeof(float)) * (D * kBM + G * group_floats<D, RPT>());
}

template <int D, int RPT, int G>
static int launch_d(Params p, const fpk_attn_desc* d, cudaStream_t s) {
  static_assert(smem_bytes<D, RPT, G>() <= 227 * 1024, "shared memory of the f32 attention kernel");
  static std::atomic<int> opted[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FPK_ERR_CUDA;
  if (!opted[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(attn_f32_kernel<D, RPT, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem_bytes<D, RPT, G>()) != cudaSuccess)
      return FPK_ERR_CUDA;
    opted[dev].store(1, std::memory_order_release);
  }
  constexpr int kBM = 16 * RPT;
  p.num_mtiles = (d->seq_len + kBM - 1) / kBM;
  const int64_t blocks = d->batch * d->heads * p.num_mtiles;
  if (blocks > 0x7fffffffLL) return FPK_ERR_UNSUPPORTED;
  attn_f32_kernel<D, RPT, G><<<static_cast<unsigned>(blocks), kThreads * G, smem_bytes<D, RPT, G>(), s>>>(p);
  return cudaGetLastError() == cudaSuccess ? FPK_OK : FPK_ERR_CUDA;
}

// 64-row tiles when they fill the SMs; else 16-row tiles, and when even those
// leave SMs idle, key groups per CTA (two, or four for D <= 64 with enough key tiles)
template <int D>
static int launch_dd(const Params& p, const fpk_attn_desc* d, int num_sms, cudaStream_t s) {
  const int64_t bh = d->batch * d->heads;
  if (bh * ((d->seq_len + 63) / 64) >= num_sms) return launch_d<D, 4, 1>(p, d, s);
  const int64_t blocks16 = bh * ((d->seq_len + 15) / 16);
  const int64_t ktiles = (d->seq_len + kBN - 1) / kBN;
  if constexpr (D <= 64) {
    if (ktiles >= 4 && blocks16 * 4 <= 2 * static_cast<int64_t>(num_sms)) return launch_d<D, 1, 4>(p, d, s);
  }
  if (ktiles >= 2 && blocks16 * 2 <= 2 * static_cast<int64_t>(num_sms)) return launch_d<D, 1, 2>(p, d, s);
  return launch_d<D, 1, 1>(p, d, s);
}

}  // namespace attn32

int launch_attention_f32(const fpk_attn_desc* d, const void* q, const void* k, const void* v, void* o,
                         cudaStream_t stream, const DeviceInfo& dev) {
  using namespace attn32;
  const uintptr_t ptrs[4] = {reinterpret_cast<uintptr_t>(q), reinterpret_cast<uintptr_t>(k),
                             reinterpret_cast<uintptr_t>(v), reinterpret_cast<uintptr_t>(o)};
  for (uintptr_t a : ptrs)
    if (a % 4) return FPK_ERR_ALIGN;
  Params p;
  p.q = static_cast<const float*>(q);
  p.k = static_cast<const float*>(k);
  p.v = static_cast<const float*>(v);
  p.o = static_cast<float*>(o);
  p.heads = d->heads;
  p.seq = d->seq_len;
  p.num_mtiles = 0;  // set by the launch for its tile height
  p.vec4 = (reinterpret_cast<uintptr_t>(k) % 16 == 0 && reinterpret_cast<uintptr_t>(v) % 16 == 0) ? 1 : 0;
  for (int i = 0; i < 3; ++i) {
    p.qs[i] = d->q_strides[i];
    p.ks[i] = d->k_strides[i];
    p.vs[i] = d->v_strides[i];
    p.os[i] = d->o_strides[i];
    if (p.ks[i] % 4 || p.vs[i] % 4) p.vec4 = 0;  // every row start stays 16-byte aligned
  }
  p.scale = d->scale;
  const int num_sms = dev.num_sms > 0 ? dev.num_sms : 148;
  switch (d->head_dim) {
    case 16: return launch_dd<16>(p, d, num_sms, stream);
    case 32: return launch_dd<32>(p, d, num_sms, stream);
    case 64: return launch_dd<64>(p, d, num_sms, stream);
    case 128: return launch_dd<128>(p, d, num_sms, stream);
    default: return FPK_ERR_UNSUPPORTED;
  }
}

}  // namespace fpk
