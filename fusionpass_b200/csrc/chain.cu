// Fused elementwise chains: the sm_100a replacement of the reference's
// generated fp_chain_<N> Triton kernels (lib/Plan/TritonEmitter.cpp:14-65,
// twin python/fusionpass/kernels.py:129-211).
//
// One prebuilt kernel per launch mode interprets the compiled op list, so no
// code is generated per model.  The host compiles the descriptor's op DAG into
// an accumulator micro-program: one running value `acc`, the loaded inputs and
// four spill registers, each holding V consecutive elements of the thread.  A
// micro-op is one warp-uniform branch followed by V f32 operations, so the
// dispatch cost is amortised over V elements and every value stays in
// registers.  Arithmetic is f32 with explicit round-to-nearest adds and
// multiplies (no FMA contraction), and the result is rounded once at the
// store, as the reference kernels do.
//
// flat: a persistent grid (1 CTA per SM).  One producer warp streams whole
//   7680-element tiles of every full-shape operand into a ring of shared
//   memory stages with 1-D TMA bulk copies (cp.async.bulk + mbarrier
//   complete_tx, L2 evict_first); 15 consumer warps evaluate the program from
//   shared memory and write 8- or 16-byte vectors straight to HBM.
//   Broadcast operands (per-column vector, per-row value, scalar) are read
//   through the read-only cache with incrementally tracked row/column indices.
// rows: one warp (cols <= 1024) or one CTA (cols <= 16384) per row; the
//   softmax input of the whole row stays in registers, max and sum are reduced
//   with warp shuffles (+ shared memory across warps), then the post-softmax
//   ops run and the row is stored.
#include <atomic>
#include <cmath>
#include <cstring>

#include "chain_ops.cuh"
#include "common.cuh"
#include "internal.h"

namespace fpk {
namespace chain {

constexpr int kMaxIn = FPK_CHAIN_MAX_INPUTS;
constexpr int kNumTmp = 4;
constexpr int kMaxCode = 112;

// ----------------------------------------------------------- micro-ops ---
enum : int {
  C_MOV_IN = 0,   // 0..7   acc = in[i]
  C_MOV_T = 8,    // 8..11  acc = t[j]
  C_SAVE_T = 12,  // 12..15 t[j] = acc
  C_ADD_IN = 16,  // 16..23 acc = acc + in[i]
  C_ADD_T = 24,   // 24..27 acc = acc + t[j]
  C_ADD_ACC = 28, //        acc = acc + acc
  C_MUL_IN = 32,  // 32..39 acc = acc * in[i]
  C_MUL_T = 40,   // 40..43 acc = acc * t[j]
  C_MUL_ACC = 44, //        acc = acc * acc
  C_SCALE = 48,   //        acc = acc * imm
  C_RELU = 49,
  C_EXP = 50,
  C_GELU = 51,
  C_SOFTMAX = 52, // rows mode split point
};

// how the kernel reads an input
enum : int {
  M_STAGED = 0,      // full shape, TMA-staged through shared memory (flat only)
  M_FULL_VEC = 1,    // full shape, aligned vector loads
  M_FULL_SCALAR = 2, // full shape, element loads
  M_COL_VEC = 3,     // per-column vector, cols % 4 == 0, aligned
  M_COL_SCALAR = 4,  // per-column vector, element loads
  M_ROW = 5,         // one value per row
  M_SCALAR = 6,      // single value
  M_NONE = 7,        // unused input slot of a wider template instance
};

struct Input {
  const void* ptr;
  int32_t dtype;
  int32_t mode;
  uint32_t smem_off;
  int32_t pad;
};

struct Params {
  Input in[kMaxIn];
  void* out;
  int* status;
  int64_t numel, rows, cols;
  int64_t num_tiles;
  int64_t row_step_t;   // flat: whole rows advanced per tile step (grid * tile)
  uint32_t col_step_t;  // flat: column advance per tile step, mod cols
  uint32_t col_step_q;  // flat: column advance per quad step inside a tile, mod cols
  uint32_t row_step_q;  // flat: whole rows advanced per quad step inside a tile
  int32_t out_dtype;
  int32_t out_vec;
  int32_t n_code;
  int32_t n_pre;        // rows: index of the SOFTMAX micro-op
  int32_t post_reload;  // rows: post-softmax ops read inputs or spill registers
  int32_t stage_bytes;
  int32_t nstage;
  int32_t need_idx;     // flat: some operand needs the row/column index
  uint32_t flags;
  uint8_t code[kMaxCode];
  float imm[kMaxCode];
};

// ------------------------------------------------------- f32 element ops ---
// op_relu, op_gelu: chain_ops.cuh

template <int NIN, int V, int NT = kNumTmp>
struct Regs {
  float in[NIN][V];
  float t[NT > 0 ? NT : 1][V];
  float acc[V];
};

// Run micro-ops [pc0, pc1) of the program over the V elements held in R.
template <int NIN, int V, int NT>
__device__ __forceinline__ void run_code(const Params& p, int pc0, int pc1, Regs<NIN, V, NT>& R) {
#pragma unroll 1
  for (int pc = pc0; pc < pc1; ++pc) {
    const int c = p.code[pc];
    switch (c) {
#define FPK_IN_CASES(I)                                                          \
  case C_MOV_IN + I:                                                             \
    if constexpr (I < NIN) {                                                     \
      _Pragma("unroll") for (int e = 0; e < V; ++e) R.acc[e] = R.in[I][e];       \
    }                                                                            \
    break;                                                                       \
  case C_ADD_IN + I:                                                             \
    if constexpr (I < NIN) {                                                     \
      _Pragma("unroll") for (int e = 0; e < V; ++e) R.acc[e] =                   \
          __fadd_rn(R.acc[e], R.in[I][e]);                                       \
    }                                                                            \
    break;                                                                       \
  case C_MUL_IN + I:                                                             \
    if constexpr (I < NIN) {                                                     \
      _Pragma("unroll") for (int e = 0; e < V; ++e) R.acc[e] =                   \
          __fmul_rn(R.acc[e], R.in[I][e]);                                       \
    }                                                                            \
    break;
      FPK_IN_CASES(0)
      FPK_IN_CASES(1)
      FPK_IN_CASES(2)
      FPK_IN_CASES(3)
      FPK_IN_CASES(4)
      FPK_IN_CASES(5)
      FPK_IN_CASES(6)
      FPK_IN_CASES(7)
#undef FPK_IN_CASES
#define FPK_T_CASES(J)                                                                        \
  case C_MOV_T + J:                                                                           \
    if constexpr (J < NT) {                                                                   \
      _Pragma("unroll") for (int e = 0; e < V; ++e) R.acc[e] = R.t[J][e];                     \
    }                                                                                         \
    break;                                                                                    \
  case C_SAVE_T + J:                                                                          \
    if constexpr (J < NT) {                                                                   \
      _Pragma("unroll") for (int e = 0; e < V; ++e) R.t[J][e] = R.acc[e];                     \
    }                                                                                         \
    break;                                                                                    \
  case C_ADD_T + J:                                                                           \
    if constexpr (J < NT) {                                                                   \
      _Pragma("unroll") for (int e = 0; e < V; ++e) R.acc[e] = __fadd_rn(R.acc[e], R.t[J][e]); \
    }                                                                                         \
    break;                                                                                    \
  case C_MUL_T + J:                                                                           \
    if constexpr (J < NT) {                                                                   \
      _Pragma("unroll") for (int e = 0; e < V; ++e) R.acc[e] = __fmul_rn(R.acc[e], R.t[J][e]); \
    }                                                                                         \
    break;
      FPK_T_CASES(0)
      FPK_T_CASES(1)
      FPK_T_CASES(2)
      FPK_T_CASES(3)
#undef FPK_T_CASES
      case C_ADD_ACC:
#pragma unroll
        for (int e = 0; e < V; ++e) R.acc[e] = __fadd_rn(R.acc[e], R.acc[e]);
        break;
      case C_MUL_ACC:
#pragma unroll
        for (int e = 0; e < V; ++e) R.acc[e] = __fmul_rn(R.acc[e], R.acc[e]);
        break;
      case C_SCALE: {
        const float s = p.imm[pc];
#pragma unroll
        for (int e = 0; e < V; ++e) R.acc[e] = __fmul_rn(R.acc[e], s);
        break;
      }
      case C_RELU:
#pragma unroll
        for (int e = 0; e < V; ++e) R.acc[e] = op_relu(R.acc[e]);
        break;
      case C_EXP:
#pragma unroll
        for (int e = 0; e < V; ++e) R.acc[e] = expf(R.acc[e]);
        break;
      case C_GELU:
#pragma unroll
        for (int e = 0; e < V; ++e) R.acc[e] = op_gelu(R.acc[e]);
        break;
      default:
        break;
    }
  }
}

// --------------------------------------------------------------- loads ---
// All loaders return a float4 by value so the caller's register arrays are only
// ever indexed with compile-time constants (no local-memory copies).
__device__ __forceinline__ float ld1(const void* base, int64_t idx, int dtype) {
  if (dtype == FPK_F16) return __half2float(__ldg(reinterpret_cast<const __half*>(base) + idx));
  return __ldg(reinterpret_cast<const float*>(base) + idx);
}

__device__ __forceinline__ float4 splat(float x) { return make_float4(x, x, x, x); }

__device__ __forceinline__ float4 h4_to_f4(uint2 u) {
  const float2 a = unpack_half2(u.x), b = unpack_half2(u.y);
  return make_float4(a.x, a.y, b.x, b.y);
}

// 4 consecutive elements at element index idx (aligned: 8 B for f16, 16 B for f32)
__device__ __forceinline__ float4 ld4_vec(const void* base, int64_t idx, int dtype) {
  if (dtype == FPK_F16)
    return h4_to_f4(__ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(base) + idx)));
  return __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx));
}

// streaming (read-once) variant for full-shape operands that are not staged
__device__ __forceinline__ float4 ld4_stream(const void* base, int64_t idx, int dtype) {
  if (dtype == FPK_F16)
    return h4_to_f4(__ldcs(reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(base) + idx)));
  return __ldcs(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx));
}

__device__ __forceinline__ float4 lds4(const uint8_t* p, int dtype) {
  if (dtype == FPK_F16) return h4_to_f4(*reinterpret_cast<const uint2*>(p));
  return *reinterpret_cast<const float4*>(p);
}

// Element-wise loads of the quad starting at flat index e (e + j >= numel reads 0).
__device__ __forceinline__ float4 load_quad_slow(const Input& in, int64_t e, int64_t numel, int64_t cols) {
  float r[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t x = e + j;
    float v = 0.0f;
    if (x < numel) {
      switch (in.mode) {
        case M_COL_VEC:
        case M_COL_SCALAR: v = ld1(in.ptr, x % cols, in.dtype); break;
        case M_ROW: v = ld1(in.ptr, x / cols, in.dtype); break;
        case M_SCALAR: v = ld1(in.ptr, 0, in.dtype); break;
        default: v = ld1(in.ptr, x, in.dtype); break;  // full shape (staged or not)
      }
    }
    r[j] = v;
  }
  return make_float4(r[0], r[1], r[2], r[3]);
}

// Quad of input `in` for row `row`, columns [c, c + nv) of a rows-mode chain.
__device__ __forceinline__ float4 load_quad_row(const Input& in, int64_t row, int64_t rbase, int64_t c, int nv) {
  switch (in.mode) {
    case M_FULL_VEC: return ld4_vec(in.ptr, rbase + c, in.dtype);
    case M_COL_VEC: return ld4_vec(in.ptr, c, in.dtype);
    case M_ROW: return splat(ld1(in.ptr, row, in.dtype));
    case M_SCALAR: return splat(ld1(in.ptr, 0, in.dtype));
    case M_COL_SCALAR: {
      float r[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j] = j < nv ? ld1(in.ptr, c + j, in.dtype) : 0.0f;
      return make_float4(r[0], r[1], r[2], r[3]);
    }
    default: {  // full shape, element loads
      float r[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j] = j < nv ? ld1(in.ptr, rbase + c + j, in.dtype) : 0.0f;
      return make_float4(r[0], r[1], r[2], r[3]);
    }
  }
}

template <int NIN, int V, int NT>
__device__ __forceinline__ void put4(Regs<NIN, V, NT>& R, int i, int at, float4 v) {
  R.in[i][at + 0] = v.x;
  R.in[i][at + 1] = v.y;
  R.in[i][at + 2] = v.z;
  R.in[i][at + 3] = v.w;
}

// Store 4 consecutive outputs at element index idx; `n` (1..4) valid ones.
__device__ __forceinline__ void st4(const Params& p, int64_t idx, float4 v, int n) {
  if (p.out_dtype == FPK_F16) {
    __half* o = reinterpret_cast<__half*>(p.out) + idx;
    if (n == 4 && p.out_vec) {
      uint2 u;
      u.x = pack_half2(v.x, v.y);
      u.y = pack_half2(v.z, v.w);
      *reinterpret_cast<uint2*>(o) = u;
    } else {
      if (n > 0) o[0] = __float2half_rn(v.x);
      if (n > 1) o[1] = __float2half_rn(v.y);
      if (n > 2) o[2] = __float2half_rn(v.z);
      if (n > 3) o[3] = __float2half_rn(v.w);
    }
  } else {
    float* o = reinterpret_cast<float*>(p.out) + idx;
    if (n == 4 && p.out_vec) {
      *reinterpret_cast<float4*>(o) = v;
    } else {
      if (n > 0) o[0] = v.x;
      if (n > 1) o[1] = v.y;
      if (n > 2) o[2] = v.z;
      if (n > 3) o[3] = v.w;
    }
  }
}

template <int NIN, int V, int NT>
__device__ __forceinline__ float4 acc4(const Regs<NIN, V, NT>& R, int at) {
  return make_float4(R.acc[at], R.acc[at + 1], R.acc[at + 2], R.acc[at + 3]);
}

// ================================================================ flat ===
constexpr int kConsumerWarps = 15;
constexpr int kNCT = kConsumerWarps * 32;  // consumer threads
constexpr int kQPT = 4;                    // quads per consumer thread per tile
constexpr int kTile = kNCT * kQPT * 4;     // 7680 elements
constexpr int kFlatThreads = kNCT + 32;    // + 1 producer warp
constexpr int kMaxStages = 8;
constexpr int kMaxStageBytes = 64 * 1024;
constexpr int kStageBudget = 192 * 1024;

template <int NIN, int NT>
__global__ void __launch_bounds__(kFlatThreads, 1) chain_flat_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full_bar[kMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kMaxStages];
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nstage = p.nstage;
  if (threadIdx.x == 0) {
    for (int s = 0; s < nstage; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kConsumerWarps);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const uint64_t limit = (p.flags & FPK_FLAG_TEST_TIMEOUT) ? kTestWaitLimitNs : kWaitLimitNs;
  const int64_t G = gridDim.x;

  if (warp == kConsumerWarps) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int64_t last_li[kMaxStages];
      for (int s = 0; s < kMaxStages; ++s) last_li[s] = -1;
      int64_t li = 0;
      for (int64_t tile = blockIdx.x; tile < p.num_tiles; tile += G, ++li) {
        const int s = static_cast<int>(li % nstage);
        const uint32_t r = static_cast<uint32_t>(li / nstage);
        if (!mbar_wait(&empty_bar[s], (r & 1u) ^ 1u, &abort_flag, p.status, limit)) break;
        if ((p.flags & FPK_FLAG_TEST_TIMEOUT) && li == 0) continue;  // withheld on purpose
        const int64_t e0 = tile * kTile;
        const bool whole = e0 + kTile <= p.numel;
        last_li[s] = li;  // the newest phase of this stage (copy or plain arrive)
        if (whole && p.stage_bytes > 0) {
          mbar_arrive_expect_tx(&full_bar[s], static_cast<uint32_t>(p.stage_bytes));
          uint8_t* dst = smem + static_cast<size_t>(s) * p.stage_bytes;
#pragma unroll
          for (int i = 0; i < NIN; ++i) {
            if (p.in[i].mode == M_STAGED) {
              const int esz = p.in[i].dtype == FPK_F16 ? 2 : 4;
              bulk_g2s(dst + p.in[i].smem_off,
                       reinterpret_cast<const uint8_t*>(p.in[i].ptr) + e0 * esz,
                       static_cast<uint32_t>(kTile * esz), &full_bar[s], pol);
            }
          }
        } else {
          mbar_arrive(&full_bar[s]);
        }
      }
      // Drain: no bulk copy may still be in flight when the CTA exits.  Phases of
      // one barrier complete in order, so waiting for the newest phase of every
      // stage covers all copies issued to it (a parity taken from an older phase
      // could alias a phase two steps later).
      for (int s = 0; s < nstage; ++s) {
        if (last_li[s] < 0) continue;
        const uint32_t par = static_cast<uint32_t>(last_li[s] / nstage) & 1u;
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&full_bar[s], par)) {
          if (globaltimer_ns() - t0 > kWaitLimitNs) {
            record_status(p.status, FPK_ERR_TIMEOUT);
            break;
          }
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  const int ct = threadIdx.x;
  const int64_t cols = p.cols;
  // column / row of this thread's first quad of its first tile
  int64_t col_b = 0, row_b = 0;
  if (p.need_idx) {
    const int64_t e = static_cast<int64_t>(blockIdx.x) * kTile + 4 * ct;
    col_b = e % cols;
    row_b = e / cols;
  }
  int64_t li = 0;
  for (int64_t tile = blockIdx.x; tile < p.num_tiles; tile += G, ++li) {
    const int s = static_cast<int>(li % nstage);
    const uint32_t r = static_cast<uint32_t>(li / nstage);
    if (!mbar_wait(&full_bar[s], r & 1u, &abort_flag, p.status, limit)) break;
    const int64_t e0 = tile * kTile;
    const bool whole = e0 + kTile <= p.numel;
    const uint8_t* stage = smem + static_cast<size_t>(s) * p.stage_bytes;
    int64_t col = col_b, row = row_b;

#pragma unroll 1
    for (int qp = 0; qp < kQPT; qp += 2) {
      Regs<NIN, 8, NT> R;
      int64_t qcol[2], qrow[2];
      qcol[0] = col; qrow[0] = row;
      col += p.col_step_q; row += p.row_step_q;
      if (col >= cols) { col -= cols; ++row; }
      qcol[1] = col; qrow[1] = row;
      col += p.col_step_q; row += p.row_step_q;
      if (col >= cols) { col -= cols; ++row; }

#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int o = 4 * (ct + kNCT * (qp + h));  // element offset inside the tile
        const int64_t e = e0 + o;
#pragma unroll
        for (int i = 0; i < NIN; ++i) {
          const Input& in = p.in[i];
          if (in.mode == M_NONE) continue;
          float4 v;
          if (!whole) {
            v = load_quad_slow(in, e, p.numel, cols);
          } else {
            switch (in.mode) {
              case M_STAGED: v = lds4(stage + in.smem_off + o * (in.dtype == FPK_F16 ? 2 : 4), in.dtype); break;
              case M_FULL_VEC: v = ld4_stream(in.ptr, e, in.dtype); break;
              case M_COL_VEC: v = ld4_vec(in.ptr, qcol[h], in.dtype); break;
              case M_ROW:
                v = p.need_idx ? splat(ld1(in.ptr, qrow[h], in.dtype)) : load_quad_slow(in, e, p.numel, cols);
                break;
              case M_SCALAR: v = splat(ld1(in.ptr, 0, in.dtype)); break;
              default: v = load_quad_slow(in, e, p.numel, cols); break;
            }
          }
          put4(R, i, 4 * h, v);
        }
      }
      run_code(p, 0, p.n_code, R);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int64_t e = e0 + 4 * (ct + kNCT * (qp + h));
        if (whole) {
          st4(p, e, acc4(R, 4 * h), 4);
        } else if (e < p.numel) {
          const int64_t rem = p.numel - e;
          st4(p, e, acc4(R, 4 * h), rem < 4 ? static_cast<int>(rem) : 4);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[s]);
    if (p.need_idx) {
      col_b += p.col_step_t;
      row_b += p.row_step_t;
      if (col_b >= cols) { col_b -= cols; ++row_b; }
    }
  }
}

// ================================================================ rows ===
template <int NIN, int TPR, int QPT>
__global__ void __launch_bounds__(TPR > 32 ? TPR : 256) chain_rows_kernel(const __grid_constant__ Params p) {
  constexpr int kWarpsPerRow = TPR / 32;
  __shared__ float red[2][kWarpsPerRow > 1 ? kWarpsPerRow : 1];
  const int lane = threadIdx.x & 31;
  const int64_t cols = p.cols;

  int64_t row, row_step;
  int lt;  // thread index inside its row group
  if constexpr (TPR == 32) {
    const int wpb = blockDim.x >> 5;
    row = static_cast<int64_t>(blockIdx.x) * wpb + (threadIdx.x >> 5);
    row_step = static_cast<int64_t>(gridDim.x) * wpb;
    lt = lane;
  } else {
    row = blockIdx.x;
    row_step = gridDim.x;
    lt = threadIdx.x;
  }
  const int pre_end = p.n_pre;
  const int post_begin = p.n_pre + 1;

  for (; row < p.rows; row += row_step) {
    float sv[QPT][4];
    float m = -INFINITY;
    const int64_t rbase = row * cols;
#pragma unroll
    for (int q = 0; q < QPT; ++q) {
      const int64_t c = 4 * (lt + static_cast<int64_t>(TPR) * q);
      Regs<NIN, 4> R;
      if (c < cols) {
        const int nv = cols - c < 4 ? static_cast<int>(cols - c) : 4;
#pragma unroll
        for (int i = 0; i < NIN; ++i) {
          const Input& in = p.in[i];
          if (in.mode == M_NONE) continue;
          put4(R, i, 0, load_quad_row(in, row, rbase, c, nv));
        }
        run_code(p, 0, pre_end, R);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          sv[q][j] = j < nv ? R.acc[j] : -INFINITY;
          m = fmaxf(m, sv[q][j]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) sv[q][j] = -INFINITY;
      }
    }
    // row max
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if constexpr (kWarpsPerRow > 1) {
      if (lane == 0) red[0][threadIdx.x >> 5] = m;
      __syncthreads();
      m = red[0][0];
#pragma unroll
      for (int w = 1; w < kWarpsPerRow; ++w) m = fmaxf(m, red[0][w]);
    }
    // exp and row sum
    float sum = 0.0f;
#pragma unroll
    for (int q = 0; q < QPT; ++q) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float x = sv[q][j];
        const float ev = (x == -INFINITY) ? 0.0f : expf(__fsub_rn(x, m));
        sv[q][j] = ev;
        sum = __fadd_rn(sum, ev);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, off));
    if constexpr (kWarpsPerRow > 1) {
      if (lane == 0) red[1][threadIdx.x >> 5] = sum;
      __syncthreads();
      sum = red[1][0];
#pragma unroll
      for (int w = 1; w < kWarpsPerRow; ++w) sum = __fadd_rn(sum, red[1][w]);
      __syncthreads();  // red[] is reused by the next row
    }
    // post-softmax ops and store
#pragma unroll
    for (int q = 0; q < QPT; ++q) {
      const int64_t c = 4 * (lt + static_cast<int64_t>(TPR) * q);
      if (c >= cols) continue;
      const int nv = cols - c < 4 ? static_cast<int>(cols - c) : 4;
      Regs<NIN, 4> R;
      if (p.post_reload) {
#pragma unroll
        for (int i = 0; i < NIN; ++i) {
          const Input& in = p.in[i];
          if (in.mode == M_NONE) continue;
          put4(R, i, 0, load_quad_row(in, row, rbase, c, nv));
        }
        run_code(p, 0, pre_end, R);  // restores spill registers used after the softmax
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) R.acc[j] = __fdiv_rn(sv[q][j], sum);
      run_code(p, post_begin, p.n_code, R);
      st4(p, rbase + c, acc4(R, 0), nv);
    }
  }
}

// ========================================================= row-tiled flat ===
// The common shape of a flat chain: inputs are full [rows, cols] tensors and
// per-column vectors, cols % 8 == 0, one dtype throughout, no spill registers.
// Inputs are put in canonical order (full ones first, then per-column ones) so
// that every micro-op knows the class of its operand at compile time.
// Each consumer thread owns fixed 8-column vectors and keeps only the running
// value (4 vectors = 32 elements, as 16 packed f32 pairs) in registers; full
// operands are read from the TMA stage with 32-bit shared addresses, per-column
// operands from an f32 copy in shared memory whose addresses are fixed per
// thread.  add / mul / scale run as packed add.rn.f32x2 / mul.rn.f32x2 (per
// lane identical to the scalar round-to-nearest ops).  TMA streams whole row
// blocks: one bulk copy per full input per stage.
constexpr int kTS = 4;                // slots (8-element vectors) per dispatch
constexpr int kTV = 8 * kTS;          // elements per dispatch
constexpr int kTP = kTV / 2;          // packed f32 pairs per dispatch
constexpr int kTConsumers = 512;      // 16 consumer warps + 1 producer warp (<= 96 registers)
constexpr int kTThreads = kTConsumers + 32;
constexpr int kTStageBudget = 128 * 1024;
constexpr int kTSmemTotal = 224 * 1024;  // dynamic shared memory of one row-tiled CTA at most
constexpr int kTColBudget = 64 * 1024;  // f32 copies of the per-column operands
constexpr int kTMaxCode = 16;         // program held in two 64-bit registers

struct TParams {
  const void* in_ptr[kMaxIn];    // canonical order: full inputs, then per-column inputs
  void* out;
  int* status;
  int64_t rows, cols;
  int64_t num_blocks;            // row blocks of stage_rows rows
  int32_t cv;                    // cols / 8
  int32_t teff;                  // consumer threads in use
  int32_t rps;                   // rows per thread step (one vector per row per thread: teff / cv)
  int32_t stage_rows;
  int32_t dispatches;            // dispatches per stage
  int32_t in_bytes;              // bytes of one full input inside a stage
  int32_t col_pad;               // floats per per-column operand in shared memory (>= cols)
  int32_t col_pad_bytes;         // padding after the stages for reads of masked slots
  int32_t stage_bytes;
  int32_t nstage;
  int32_t n_code;
  uint32_t flags;
  uint64_t code_lo, code_hi;     // micro-ops 0..7 and 8..15, 8 bits each
  float imm[kTMaxCode];
};

// ---- packed f32 pairs
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// Ordered variants: volatile asm keeps program order, which bounds how many
// slots' operands are live at once (see t_op_in).
__device__ __forceinline__ uint64_t f2_add_o(uint64_t a, uint64_t b) {
  uint64_t d;
  asm volatile("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul_o(uint64_t a, uint64_t b) {
  uint64_t d;
  asm volatile("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t h2_to_f2(uint32_t h) {
  const float2 f = unpack_half2(h);
  return f2_pack(f.x, f.y);
}

// 8 elements at a 32-bit shared address -> 4 packed pairs
template <int DT>
__device__ __forceinline__ void t_lds8(uint32_t addr, uint64_t* v) {
  uint32_t a, b, c, d;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "r"(addr));
  if constexpr (DT == FPK_F16) {
    v[0] = h2_to_f2(a);
    v[1] = h2_to_f2(b);
    v[2] = h2_to_f2(c);
    v[3] = h2_to_f2(d);
  } else {
    uint32_t e, f, g, h;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(e), "=r"(f), "=r"(g), "=r"(h) : "r"(addr + 16));
    v[0] = (static_cast<uint64_t>(b) << 32) | a;
    v[1] = (static_cast<uint64_t>(d) << 32) | c;
    v[2] = (static_cast<uint64_t>(f) << 32) | e;
    v[3] = (static_cast<uint64_t>(h) << 32) | g;
  }
}

// 8 f32 at a 32-bit shared address -> 4 packed pairs
__device__ __forceinline__ void t_lds8f(uint32_t addr, uint64_t* v) {
  asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(v[0]), "=l"(v[1]) : "r"(addr));
  asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(v[2]), "=l"(v[3]) : "r"(addr + 16));
}

// Addressing of the kTS slots of a dispatch: slot q is vector (q % NV) of row
// (q / NV) of the thread's row step, so every address is affine in q with
// warp-uniform strides and only one base offset per dispatch is kept.
template <int NF, int NC>
struct TCtx {
  uint32_t in_base[NF];              // shared address of full input i in the current stage
  uint32_t col[NC > 0 ? NC : 1];     // shared address of this thread's first column vector in input j
  uint32_t row_stride;               // bytes between the rows of consecutive slots (rps rows)
  uint32_t vec_stride;               // bytes between vectors of consecutive slots (teff vectors)
  uint32_t col_stride;               // bytes between per-column vectors of consecutive slots
  uint32_t col_half;                 // bytes from the first to the second 4 floats of a vector
};

// acc (op) operand I (compile-time, canonical order) for the kTS slots at offset e0.
// Software-pipelined: the shared-memory load of slot q+1 is issued before slot
// q is combined, and the volatile loads / packed ops keep exactly that order,
// so only two slots' operands are live at a time (no spills at 96 registers).
// One slot of operand I: f16 data stays as 4 packed half2 words (raw[0..3]);
// f32 data is loaded straight into 4 packed f32 pairs (pair[0..3]).
template <int DT, int NF, int NC, int NV, int I>
__device__ __forceinline__ void t_load_slot(const TCtx<NF, NC>& cx, uint32_t e0, int q, uint32_t* raw,
                                            uint64_t* pair) {
  if constexpr (I < NF) {
    const uint32_t a = cx.in_base[I < NF ? I : 0] + e0 + (q / NV) * cx.row_stride + (q % NV) * cx.vec_stride;
    if constexpr (DT == FPK_F16) {
      asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(raw[0]), "=r"(raw[1]), "=r"(raw[2]), "=r"(raw[3]) : "r"(a));
    } else {
      asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(pair[0]), "=l"(pair[1]) : "r"(a));
      asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(pair[2]), "=l"(pair[3]) : "r"(a + 16));
    }
  } else {
    const uint32_t a = cx.col[I < NF ? 0 : I - NF] + (q % NV) * cx.col_stride;
    asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(pair[0]), "=l"(pair[1]) : "r"(a));
    asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(pair[2]), "=l"(pair[3]) : "r"(a + cx.col_half));
  }
}

template <int DT, int NF, int OP, int I>
__device__ __forceinline__ void t_combine_slot(const uint32_t* raw, const uint64_t* pair, uint64_t* acc4) {
  uint64_t v[4];
  if constexpr (I < NF && DT == FPK_F16) {
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = h2_to_f2(raw[k]);
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = pair[k];
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if constexpr (OP == 0) acc4[k] = v[k];
    else if constexpr (OP == 1) acc4[k] = f2_add_o(acc4[k], v[k]);
    else acc4[k] = f2_mul_o(acc4[k], v[k]);
  }
}

template <int DT, int NF, int NC, int NV, int I, int OP>
__device__ __forceinline__ void t_op_in(const TCtx<NF, NC>& cx, uint32_t e0, uint64_t* acc) {
  uint32_t raw[2][4];
  uint64_t pair[2][4];
  t_load_slot<DT, NF, NC, NV, I>(cx, e0, 0, raw[0], pair[0]);
#pragma unroll
  for (int q = 0; q < kTS; ++q) {
    if (q + 1 < kTS) t_load_slot<DT, NF, NC, NV, I>(cx, e0, q + 1, raw[(q + 1) & 1], pair[(q + 1) & 1]);
    t_combine_slot<DT, NF, OP, I>(raw[q & 1], pair[q & 1], &acc[q * 4]);
  }
}

// TR: the program has exp / gelu.  Their unrolled expansions over 32 live
// elements set the register peak of the whole dispatch switch, so programs
// without them get an instance that does not contain those cases at all.
template <int DT, int NF, int NC, int NV, bool TR>
__device__ __forceinline__ void run_tiled(const TParams& p, const TCtx<NF, NC>& cx, uint32_t e0, uint64_t* acc) {
  uint64_t lo = p.code_lo, hi = p.code_hi;
  // the first micro-op moves an operand into acc; every later one updates acc in place
  switch (static_cast<int>(lo & 0xffu)) {
#define FPK_TMOV(I) \
  case C_MOV_IN + I: \
    if constexpr (I < NF + NC) t_op_in<DT, NF, NC, NV, (I < NF + NC ? I : 0), 0>(cx, e0, acc); \
    break;
    FPK_TMOV(0) FPK_TMOV(1) FPK_TMOV(2) FPK_TMOV(3) FPK_TMOV(4)
#undef FPK_TMOV
    default: break;
  }
  lo = (lo >> 8) | (hi << 56);
  hi >>= 8;
#pragma unroll 1
  for (int pc = 1; pc < p.n_code; ++pc) {
    const int c = static_cast<int>(lo & 0xffu);
    lo = (lo >> 8) | (hi << 56);
    hi >>= 8;
    switch (c) {
#define FPK_TIN(I)                                                                         \
  case C_ADD_IN + I:                                                                       \
    if constexpr (I < NF + NC) t_op_in<DT, NF, NC, NV, (I < NF + NC ? I : 0), 1>(cx, e0, acc);  \
    break;                                                                                 \
  case C_MUL_IN + I:                                                                       \
    if constexpr (I < NF + NC) t_op_in<DT, NF, NC, NV, (I < NF + NC ? I : 0), 2>(cx, e0, acc);  \
    break;
      FPK_TIN(0) FPK_TIN(1) FPK_TIN(2) FPK_TIN(3) FPK_TIN(4)
#undef FPK_TIN
      case C_ADD_ACC:
#pragma unroll
        for (int k = 0; k < kTP; ++k) acc[k] = f2_add(acc[k], acc[k]);
        break;
      case C_MUL_ACC:
#pragma unroll
        for (int k = 0; k < kTP; ++k) acc[k] = f2_mul(acc[k], acc[k]);
        break;
      case C_SCALE: {
        const float sc = p.imm[pc];
        const uint64_t s2 = f2_pack(sc, sc);
#pragma unroll
        for (int k = 0; k < kTP; ++k) acc[k] = f2_mul(acc[k], s2);
        break;
      }
      case C_RELU:
#pragma unroll
        for (int k = 0; k < kTP; ++k) {
          const float2 f = f2_unpack(acc[k]);
          acc[k] = f2_pack(op_relu(f.x), op_relu(f.y));
        }
        break;
      case C_EXP:
        if constexpr (TR) {
#pragma unroll
          for (int k = 0; k < kTP; ++k) {
            const float2 f = f2_unpack(acc[k]);
            acc[k] = f2_pack(expf(f.x), expf(f.y));
          }
        }
        break;
      case C_GELU:
        if constexpr (TR) {
#pragma unroll
          for (int k = 0; k < kTP; ++k) {
            const float2 f = f2_unpack(acc[k]);
            acc[k] = f2_pack(op_gelu(f.x), op_gelu(f.y));
          }
        }
        break;
      default:
        break;
    }
  }
}

template <int DT>
__device__ __forceinline__ void t_st8(void* base, int64_t idx, const uint64_t* v) {
  if constexpr (DT == FPK_F16) {
    uint4 u;
    const float2 a = f2_unpack(v[0]), b = f2_unpack(v[1]), c = f2_unpack(v[2]), d = f2_unpack(v[3]);
    u.x = pack_half2(a.x, a.y);
    u.y = pack_half2(b.x, b.y);
    u.z = pack_half2(c.x, c.y);
    u.w = pack_half2(d.x, d.y);
    *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(base) + idx) = u;
  } else {
    ulonglong2* q = reinterpret_cast<ulonglong2*>(reinterpret_cast<float*>(base) + idx);
    q[0] = make_ulonglong2(v[0], v[1]);
    q[1] = make_ulonglong2(v[2], v[3]);
  }
}

// NV = 8-column vectors a thread owns per row (1 or 2); slot q of a dispatch
// is vector (q % NV) of row (q / NV) of the thread's current row step.
template <int DT, int NF, int NC, int NV, bool TR>
__global__ void __launch_bounds__(kTThreads, 1) chain_tiled_kernel(const __grid_constant__ TParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full_bar[kMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kMaxStages];
  __shared__ volatile int abort_flag;
  constexpr int esz = DT == FPK_F16 ? 2 : 4;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ncw = (p.teff + 31) >> 5;  // consumer warps; the producer is warp ncw
  const int nstage = p.nstage;
  // layout: input stages | read-overrun padding | column area (16-byte aligned)
  float* cols = reinterpret_cast<float*>(
      smem + ((static_cast<size_t>(nstage) * p.stage_bytes + p.col_pad_bytes + 15) & ~static_cast<size_t>(15)));
  if (threadIdx.x == 0) {
    for (int s = 0; s < nstage; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], ncw);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  // per-column operands -> f32 in shared memory (all threads of the CTA help).
  // Vector v's first 4 floats go to half A at [4v, 4v+4), the other 4 to half B
  // (col_pad / 2 floats later), so a warp reading one half per thread touches
  // consecutive 16-byte chunks.  The padding past cols (read by masked slots
  // only) is zero-filled.
#pragma unroll
  for (int j = 0; j < NC; ++j)
    for (int c = threadIdx.x; c < p.col_pad; c += blockDim.x) {
      const int v = c >> 3, k = c & 7;
      cols[j * p.col_pad + (k < 4 ? 0 : p.col_pad / 2) + v * 4 + (k & 3)] =
          c < p.cols ? ld1(p.in_ptr[NF + j], c, DT) : 0.0f;
    }
  __syncthreads();
  const uint64_t limit = (p.flags & FPK_FLAG_TEST_TIMEOUT) ? kTestWaitLimitNs : kWaitLimitNs;
  const int64_t G = gridDim.x;
  const int64_t C = p.cols;
  const int64_t row_bytes = C * esz;

  if (warp == ncw) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int64_t last_li[kMaxStages];
      for (int s = 0; s < kMaxStages; ++s) last_li[s] = -1;
      int64_t li = 0;
      for (int64_t blk = blockIdx.x; blk < p.num_blocks; blk += G, ++li) {
        const int s = static_cast<int>(li % nstage);
        const uint32_t r = static_cast<uint32_t>(li / nstage);
        if (!mbar_wait(&empty_bar[s], (r & 1u) ^ 1u, &abort_flag, p.status, limit)) break;
        if ((p.flags & FPK_FLAG_TEST_TIMEOUT) && li == 0) continue;  // withheld on purpose
        last_li[s] = li;
        const int64_t r0 = blk * p.stage_rows;
        const int64_t nr = (p.rows - r0) < p.stage_rows ? (p.rows - r0) : p.stage_rows;
        const uint32_t bytes = static_cast<uint32_t>(nr * row_bytes);
        mbar_arrive_expect_tx(&full_bar[s], bytes * NF);
        uint8_t* dst = smem + static_cast<size_t>(s) * p.stage_bytes;
#pragma unroll
        for (int i = 0; i < NF; ++i)
          bulk_g2s(dst + i * p.in_bytes, reinterpret_cast<const uint8_t*>(p.in_ptr[i]) + r0 * row_bytes, bytes,
                   &full_bar[s], pol);
      }
      for (int s = 0; s < nstage; ++s) {  // newest phase of every stage: no copy left in flight
        if (last_li[s] < 0) continue;
        const uint32_t par = static_cast<uint32_t>(last_li[s] / nstage) & 1u;
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&full_bar[s], par)) {
          if (globaltimer_ns() - t0 > kWaitLimitNs) {
            record_status(p.status, FPK_ERR_TIMEOUT);
            break;
          }
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  const int t = threadIdx.x;
  const bool active = t < p.teff;
  const int my_row0 = NV == 1 ? t / p.cv : 0;
  const int my_vec0 = NV == 1 ? t % p.cv : t;
  constexpr int kRD = kTS / NV;  // rows per dispatch of one thread
  const int rows_per_dispatch = kRD * p.rps;
  const uint32_t smem0 = smem_u32(smem);
  TCtx<NF, NC> cx;
  cx.row_stride = static_cast<uint32_t>(p.rps * C * esz);
  cx.vec_stride = static_cast<uint32_t>(p.teff * 8 * esz);
  cx.col_stride = static_cast<uint32_t>(p.teff * 4 * 4);
  cx.col_half = static_cast<uint32_t>(p.col_pad / 2 * 4);
#pragma unroll
  for (int j = 0; j < NC; ++j) cx.col[j] = smem_u32(cols) + static_cast<uint32_t>((j * p.col_pad + my_vec0 * 4) * 4);
  uint32_t vec_ok = 0;  // bit q: the vector of slot q lies inside the row
#pragma unroll
  for (int q = 0; q < kTS; ++q) vec_ok |= (my_vec0 + (q % NV) * p.teff < p.cv ? 1u : 0u) << q;
  const uint32_t e_thread = static_cast<uint32_t>((my_row0 * C + my_vec0 * 8) * esz);
  const uint32_t e_dispatch = static_cast<uint32_t>(rows_per_dispatch * C * esz);
  uint64_t acc[kTP];

  int64_t li = 0;
  for (int64_t blk = blockIdx.x; blk < p.num_blocks; blk += G, ++li) {
    const int s = static_cast<int>(li % nstage);
    const uint32_t r = static_cast<uint32_t>(li / nstage);
    if (!mbar_wait(&full_bar[s], r & 1u, &abort_flag, p.status, limit)) break;
    const int64_t r0 = blk * p.stage_rows;
    const int nr = static_cast<int>((p.rows - r0) < p.stage_rows ? (p.rows - r0) : p.stage_rows);
    const uint32_t stage0 = smem0 + static_cast<uint32_t>(s * p.stage_bytes);
#pragma unroll
    for (int i = 0; i < NF; ++i) cx.in_base[i] = stage0 + static_cast<uint32_t>(i * p.in_bytes);
    char* out_blk = reinterpret_cast<char*>(p.out) + r0 * row_bytes;
    if (active) {
#pragma unroll 1
      for (int u = 0; u < p.dispatches; ++u) {
        const uint32_t e0 = e_thread + static_cast<uint32_t>(u) * e_dispatch;
        run_tiled<DT, NF, NC, NV, TR>(p, cx, e0, acc);
        const int row0 = u * rows_per_dispatch + my_row0;
#pragma unroll
        for (int q = 0; q < kTS; ++q) {
          if (((vec_ok >> q) & 1u) && row0 + (q / NV) * p.rps < nr)
            t_st8<DT>(out_blk + e0 + (q / NV) * cx.row_stride + (q % NV) * cx.vec_stride, 0, &acc[q * 4]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[s]);
  }
}

// ========================================================= host compile ===
static int elt_size(int dtype) { return dtype == FPK_F16 ? 2 : 4; }

struct Compiled {
  uint8_t code[kMaxCode];
  float imm[kMaxCode];
  int n = 0;
  int softmax_pc = -1;
  bool uses_tmp = false;
};

// Compile the op DAG of `d` into accumulator micro-code.
static int compile_program(const fpk_chain_desc* d, Compiled* out) {
  const int nin = d->n_inputs;
  const int nops = d->n_ops;
  const int nslots = nin + nops;
  int uses[FPK_CHAIN_MAX_INPUTS + FPK_CHAIN_MAX_OPS] = {0};
  for (int k = 0; k < nops; ++k) {
    const fpk_chain_op& op = d->ops[k];
    uses[op.src_a]++;
    if (op.opcode == FPK_OP_ADD || op.opcode == FPK_OP_MUL) uses[op.src_b]++;
  }
  uses[d->result]++;
  int slot_tmp[FPK_CHAIN_MAX_INPUTS + FPK_CHAIN_MAX_OPS];
  for (int s = 0; s < nslots; ++s) slot_tmp[s] = -1;
  int tmp_slot[kNumTmp] = {-1, -1, -1, -1};
  int acc = -1;
  Compiled& c = *out;
  c.n = 0;
  auto emit = [&](int code, float imm) -> bool {
    if (c.n >= kMaxCode) return false;
    c.code[c.n] = static_cast<uint8_t>(code);
    c.imm[c.n] = imm;
    ++c.n;
    return true;
  };
  auto src_code = [&](int slot, int base_in, int base_t) -> int {
    if (slot < nin) return base_in + slot;
    if (slot_tmp[slot] >= 0) return base_t + slot_tmp[slot];
    return -1;
  };
  // Save the computed value in acc if it is needed after the current op.
  auto spill_if_live = [&](int still_needed) -> bool {
    if (acc < nin || still_needed <= 0 || slot_tmp[acc] >= 0) return true;
    for (int j = 0; j < kNumTmp; ++j) {
      if (tmp_slot[j] < 0) {
        tmp_slot[j] = acc;
        slot_tmp[acc] = j;
        c.uses_tmp = true;
        return emit(C_SAVE_T + j, 0.0f);
      }
    }
    return false;  // more than kNumTmp values live at once
  };
  auto release = [&](int slot) {
    if (slot >= nin && uses[slot] == 0 && slot_tmp[slot] >= 0) {
      tmp_slot[slot_tmp[slot]] = -1;
      slot_tmp[slot] = -1;
    }
  };

  for (int k = 0; k < nops; ++k) {
    const fpk_chain_op& op = d->ops[k];
    const bool binary = op.opcode == FPK_OP_ADD || op.opcode == FPK_OP_MUL;
    const int a = op.src_a;
    const int b = binary ? op.src_b : -1;
    int other = -1;
    if (acc == a) {
      other = b;
    } else if (binary && acc == b) {
      other = a;
    } else {
      if (acc >= 0 && !spill_if_live(uses[acc])) return FPK_ERR_UNSUPPORTED;
      const int mc = src_code(a, C_MOV_IN, C_MOV_T);
      if (mc < 0) return FPK_ERR_INVALID;
      if (!emit(mc, 0.0f)) return FPK_ERR_UNSUPPORTED;
      acc = a;
      other = b;
    }
    // uses of the acc value after this op
    const int used_here = (a == acc) + (binary && b == acc);
    if (!spill_if_live(uses[acc] - used_here)) return FPK_ERR_UNSUPPORTED;
    int code = -1;
    float imm = 0.0f;
    switch (op.opcode) {
      case FPK_OP_ADD:
      case FPK_OP_MUL: {
        const bool add = op.opcode == FPK_OP_ADD;
        if (other == acc) {
          code = add ? C_ADD_ACC : C_MUL_ACC;
        } else {
          code = src_code(other, add ? C_ADD_IN : C_MUL_IN, add ? C_ADD_T : C_MUL_T);
          if (code < 0) return FPK_ERR_INVALID;
        }
        break;
      }
      case FPK_OP_SCALE: code = C_SCALE; imm = op.imm; break;
      case FPK_OP_RELU: code = C_RELU; break;
      case FPK_OP_EXP: code = C_EXP; break;
      case FPK_OP_GELU: code = C_GELU; break;
      case FPK_OP_SOFTMAX:
        code = C_SOFTMAX;
        c.softmax_pc = c.n;
        break;
      default: return FPK_ERR_INVALID;
    }
    if (!emit(code, imm)) return FPK_ERR_UNSUPPORTED;
    uses[a]--;
    if (binary) uses[b]--;
    release(a);
    if (binary) release(b);
    acc = nin + k;
  }
  if (acc != d->result) {
    const int mc = src_code(d->result, C_MOV_IN, C_MOV_T);
    if (mc < 0) return FPK_ERR_INVALID;
    if (!emit(mc, 0.0f)) return FPK_ERR_UNSUPPORTED;
  }
  return FPK_OK;
}

static int validate(const fpk_chain_desc* d, int n_inputs) {
  if (!d || d->size != sizeof(fpk_chain_desc) || d->version != FPK_ABI_VERSION) return FPK_ERR_INVALID;
  if (d->mode != FPK_CHAIN_FLAT && d->mode != FPK_CHAIN_ROWS) return FPK_ERR_INVALID;
  if (d->out_dtype != FPK_F16 && d->out_dtype != FPK_F32) return FPK_ERR_INVALID;
  if (d->rows < 0 || d->cols < 0) return FPK_ERR_INVALID;
  if (d->n_inputs < 1 || d->n_inputs > FPK_CHAIN_MAX_INPUTS || d->n_inputs != n_inputs) return FPK_ERR_INVALID;
  if (d->n_ops < 1 || d->n_ops > FPK_CHAIN_MAX_OPS) return FPK_ERR_INVALID;
  const int nin = d->n_inputs;
  int softmaxes = 0;
  for (int i = 0; i < nin; ++i) {
    if (d->in_dtype[i] != FPK_F16 && d->in_dtype[i] != FPK_F32) return FPK_ERR_INVALID;
    if (d->in_bcast[i] < FPK_BCAST_FULL || d->in_bcast[i] > FPK_BCAST_SCALAR) return FPK_ERR_INVALID;
  }
  for (int k = 0; k < d->n_ops; ++k) {
    const fpk_chain_op& op = d->ops[k];
    if (op.opcode < FPK_OP_ADD || op.opcode > FPK_OP_GELU) return FPK_ERR_INVALID;
    if (op.src_a < 0 || op.src_a >= nin + k) return FPK_ERR_INVALID;
    if (op.opcode == FPK_OP_ADD || op.opcode == FPK_OP_MUL) {
      if (op.src_b < 0 || op.src_b >= nin + k) return FPK_ERR_INVALID;
    }
    if (op.opcode == FPK_OP_SOFTMAX) ++softmaxes;
  }
  if (d->result < 0 || d->result >= nin + d->n_ops) return FPK_ERR_INVALID;
  if (d->mode == FPK_CHAIN_FLAT && softmaxes != 0) return FPK_ERR_INVALID;
  if (d->mode == FPK_CHAIN_ROWS) {
    if (softmaxes != 1) return FPK_ERR_INVALID;
    if (d->cols > FPK_CHAIN_MAX_ROW_COLS) return FPK_ERR_UNSUPPORTED;
  }
  return FPK_OK;
}

// Opt in once per device to the dynamic shared memory the flat kernel may use.
template <int NIN, int NT>
static int launch_flat_n(const Params& p, int grid, int smem, cudaStream_t s) {
  static std::atomic<int> opted[64];
  auto k = chain_flat_kernel<NIN, NT>;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FPK_ERR_CUDA;
  if (!opted[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kStageBudget) != cudaSuccess)
      return FPK_ERR_CUDA;
    opted[dev].store(1, std::memory_order_release);
  }
  k<<<grid, kFlatThreads, smem, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? FPK_OK : FPK_ERR_CUDA;
}

template <int NIN, int TPR, int QPT>
static int launch_rows_cfg(const Params& p, int num_sms, cudaStream_t s) {
  int block, grid;
  if (TPR == 32) {
    block = 256;
    const int64_t rows_per_block = block / 32;
    const int64_t need = (p.rows + rows_per_block - 1) / rows_per_block;
    grid = static_cast<int>(need < num_sms * 8 ? need : num_sms * 8);
  } else {
    block = TPR;
    grid = static_cast<int>(p.rows < num_sms * 8 ? p.rows : num_sms * 8);
  }
  chain_rows_kernel<NIN, TPR, QPT><<<grid, block, 0, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? FPK_OK : FPK_ERR_CUDA;
}

template <int NIN>
static int launch_rows_n(const Params& p, int num_sms, cudaStream_t s) {
  const int64_t c = p.cols;
  if (c <= 128) return launch_rows_cfg<NIN, 32, 1>(p, num_sms, s);
  if (c <= 256) return launch_rows_cfg<NIN, 32, 2>(p, num_sms, s);
  if (c <= 512) return launch_rows_cfg<NIN, 32, 4>(p, num_sms, s);
  if (c <= 1024) return launch_rows_cfg<NIN, 32, 8>(p, num_sms, s);
  if (c <= 2048) return launch_rows_cfg<NIN, 256, 2>(p, num_sms, s);
  if (c <= 4096) return launch_rows_cfg<NIN, 256, 4>(p, num_sms, s);
  if (c <= 8192) return launch_rows_cfg<NIN, 256, 8>(p, num_sms, s);
  return launch_rows_cfg<NIN, 512, 8>(p, num_sms, s);
}

template <int DT, int NF, int NC, int NV, bool TR>
static int launch_tiled_v(const TParams& p, int grid, int block, int smem, cudaStream_t s) {
  static std::atomic<int> opted[64];
  auto k = chain_tiled_kernel<DT, NF, NC, NV, TR>;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FPK_ERR_CUDA;
  if (!opted[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kTSmemTotal) != cudaSuccess)
      return FPK_ERR_CUDA;
    opted[dev].store(1, std::memory_order_release);
  }
  k<<<grid, block, smem, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? FPK_OK : FPK_ERR_CUDA;
}

template <int DT, int NF, int NC>
static int launch_tiled_nv(const TParams& p, int nv, bool tr, int grid, int block, int smem, cudaStream_t s) {
  if (nv == 1)
    return tr ? launch_tiled_v<DT, NF, NC, 1, true>(p, grid, block, smem, s)
              : launch_tiled_v<DT, NF, NC, 1, false>(p, grid, block, smem, s);
  return tr ? launch_tiled_v<DT, NF, NC, 2, true>(p, grid, block, smem, s)
            : launch_tiled_v<DT, NF, NC, 2, false>(p, grid, block, smem, s);
}

template <int DT>
static int launch_tiled_dt(const TParams& p, int nf, int nc, int nv, bool tr, int grid, int block, int smem,
                           cudaStream_t s) {
  switch (nf * 10 + nc) {
    case 10: return launch_tiled_nv<DT, 1, 0>(p, nv, tr, grid, block, smem, s);
    case 11: return launch_tiled_nv<DT, 1, 1>(p, nv, tr, grid, block, smem, s);
    case 12: return launch_tiled_nv<DT, 1, 2>(p, nv, tr, grid, block, smem, s);
    case 20: return launch_tiled_nv<DT, 2, 0>(p, nv, tr, grid, block, smem, s);
    case 21: return launch_tiled_nv<DT, 2, 1>(p, nv, tr, grid, block, smem, s);
    case 30: return launch_tiled_nv<DT, 3, 0>(p, nv, tr, grid, block, smem, s);
    default: return FPK_ERR_UNSUPPORTED;
  }
}

// Row-tiled flat chain for the common operand shapes; FPK_ERR_UNSUPPORTED means
// "use the general flat kernel", any other code is final.
static int try_launch_tiled(const fpk_chain_desc* d, const void* const* inputs, void* out, cudaStream_t stream,
                            const DeviceInfo& dev) {
  const int64_t C = d->cols, Rr = d->rows;
  if (d->mode != FPK_CHAIN_FLAT || (d->flags & FPK_FLAG_NO_STAGING) || C % 8 != 0 ||
      C > 8LL * 2 * kTConsumers)  // at most 2 vectors per row per thread
    return FPK_ERR_UNSUPPORTED;
  const int dt = d->out_dtype;
  const int esz = elt_size(dt);
  if (reinterpret_cast<uintptr_t>(out) % 16) return FPK_ERR_UNSUPPORTED;
  const int nin = d->n_inputs;
  int order[FPK_CHAIN_MAX_INPUTS];
  int nf = 0, nc = 0;
  for (int i = 0; i < nin; ++i) {
    const int bc = d->in_bcast[i];
    if (d->in_dtype[i] != dt || (bc != FPK_BCAST_FULL && bc != FPK_BCAST_COL)) return FPK_ERR_UNSUPPORTED;
    if (bc == FPK_BCAST_FULL) {
      if (reinterpret_cast<uintptr_t>(inputs[i]) % 16) return FPK_ERR_UNSUPPORTED;
      order[nf++] = i;
    }
  }
  for (int i = 0; i < nin; ++i)
    if (d->in_bcast[i] == FPK_BCAST_COL) order[nf + nc++] = i;
  if (nf < 1 || nf > 3 || nc > 2 || nf + nc > 3) return FPK_ERR_UNSUPPORTED;
  if (nc * C * 4 > kTColBudget) return FPK_ERR_UNSUPPORTED;  // exact size check below
  // renumber the input slots into the canonical order
  fpk_chain_desc d2 = *d;
  int newidx[FPK_CHAIN_MAX_INPUTS];
  for (int k = 0; k < nin; ++k) {
    newidx[order[k]] = k;
    d2.in_dtype[k] = d->in_dtype[order[k]];
    d2.in_bcast[k] = d->in_bcast[order[k]];
  }
  for (int k = 0; k < d->n_ops; ++k) {
    if (d2.ops[k].src_a < nin) d2.ops[k].src_a = newidx[d2.ops[k].src_a];
    if ((d2.ops[k].opcode == FPK_OP_ADD || d2.ops[k].opcode == FPK_OP_MUL) && d2.ops[k].src_b < nin)
      d2.ops[k].src_b = newidx[d2.ops[k].src_b];
  }
  if (d2.result < nin) d2.result = newidx[d2.result];
  Compiled prog;
  int rc = compile_program(&d2, &prog);
  if (rc != FPK_OK) return rc;
  if (prog.uses_tmp || prog.n < 1 || prog.n > kTMaxCode || prog.code[0] >= C_MOV_T) return FPK_ERR_UNSUPPORTED;
  for (int pc = 1; pc < prog.n; ++pc)
    if (prog.code[pc] < C_ADD_IN) return FPK_ERR_UNSUPPORTED;  // a later move needs the general kernel

  TParams p;
  std::memset(&p, 0, sizeof(p));
  const int cv = static_cast<int>(C / 8);
  int nv, teff, rps;
  if (cv <= kTConsumers) {
    nv = 1;
    rps = kTConsumers / cv;
    teff = rps * cv;
  } else {
    nv = 2;  // cv <= 2 * kTConsumers was checked above
    teff = (cv + nv - 1) / nv;
    rps = 1;
  }
  const int64_t rows_per_dispatch = (kTS / nv) * rps;
  const int64_t row_bytes_all = C * esz * nf;
  int64_t u = 24576 / (rows_per_dispatch * row_bytes_all);
  if (u < 1) u = 1;
  const int64_t stage_rows = rows_per_dispatch * u;
  const int64_t stage_bytes = stage_rows * row_bytes_all;
  if (stage_bytes > kTStageBudget / 2) return FPK_ERR_UNSUPPORTED;
  for (int k = 0; k < nin; ++k) p.in_ptr[k] = inputs[order[k]];
  p.out = out;
  p.status = dev.status;
  p.rows = Rr;
  p.cols = C;
  p.cv = cv;
  p.teff = teff;
  p.rps = rps;
  p.stage_rows = static_cast<int32_t>(stage_rows);
  p.dispatches = static_cast<int32_t>(u);
  p.num_blocks = (Rr + stage_rows - 1) / stage_rows;
  p.in_bytes = static_cast<int32_t>(stage_rows * C * esz);
  p.stage_bytes = static_cast<int32_t>(stage_bytes);
  p.n_code = prog.n;
  p.flags = d->flags;
  for (int pc = 0; pc < prog.n; ++pc) {
    const uint64_t c = prog.code[pc];
    if (pc < 8) p.code_lo |= c << (8 * pc);
    else p.code_hi |= c << (8 * (pc - 8));
    p.imm[pc] = prog.imm[pc];
  }
  const int grid = static_cast<int>(p.num_blocks < dev.num_sms ? p.num_blocks : dev.num_sms);
  const int block = ((teff + 31) / 32) * 32 + 32;
  // masked slots may read up to (teff * nv * 8 - cols) elements past a row: pad the input area
  const int64_t over = static_cast<int64_t>(teff) * nv * 8 - C;
  p.col_pad = static_cast<int32_t>(C + (over > 0 ? over : 0));
  const int64_t pad_bytes = (over > 0 ? over : 0) * esz + 16;
  p.col_pad_bytes = static_cast<int32_t>(pad_bytes);
  const int64_t fixed = nc * p.col_pad * 4LL + pad_bytes + 32;
  int64_t nst = (kTSmemTotal - fixed) / stage_bytes;
  if (nst > kTStageBudget / stage_bytes) nst = kTStageBudget / stage_bytes;
  if (nst < 2) return FPK_ERR_UNSUPPORTED;
  p.nstage = static_cast<int32_t>(nst > kMaxStages ? kMaxStages : nst);
  const int smem = static_cast<int>(((p.nstage * stage_bytes + pad_bytes + 15) & ~15LL) + nc * p.col_pad * 4LL);
  bool tr = false;
  for (int pc = 0; pc < prog.n; ++pc) tr |= prog.code[pc] == C_EXP || prog.code[pc] == C_GELU;
  return dt == FPK_F16 ? launch_tiled_dt<FPK_F16>(p, nf, nc, nv, tr, grid, block, smem, stream)
                       : launch_tiled_dt<FPK_F32>(p, nf, nc, nv, tr, grid, block, smem, stream);
}

}  // namespace chain

int chain_precompile(const fpk_chain_desc* d) {
  using namespace chain;
  if (!d) return FPK_ERR_INVALID;
  const int rc = validate(d, d->n_inputs);
  if (rc != FPK_OK) return rc;
  return chain_jit_precompile(d);
}

int launch_chain(const fpk_chain_desc* d, const void* const* inputs, void* out, cudaStream_t stream,
                 const DeviceInfo& dev) {
  using namespace chain;
  if (!d || !inputs) return FPK_ERR_INVALID;
  int rc = validate(d, d->n_inputs);
  if (rc != FPK_OK) return rc;
  const int64_t numel = d->rows * d->cols;
  if (numel == 0) return FPK_OK;  // an empty tensor: nothing to launch (its pointers may be null)
  if (!out) return FPK_ERR_INVALID;
  Compiled prog;
  rc = compile_program(d, &prog);
  if (rc != FPK_OK) return rc;


  Params p;
  std::memset(&p, 0, sizeof(p));
  p.out = out;
  p.status = dev.status;
  p.numel = numel;
  p.rows = d->rows;
  p.cols = d->cols;
  p.out_dtype = d->out_dtype;
  p.flags = d->flags;
  p.n_code = prog.n;
  std::memcpy(p.code, prog.code, sizeof(prog.code));
  std::memcpy(p.imm, prog.imm, sizeof(prog.imm));
  const uintptr_t obase = reinterpret_cast<uintptr_t>(out);
  const int osz = elt_size(d->out_dtype);
  // vector store of 4 elements: 8 B (f16) or 16 B (f32) aligned, and rows aligned in rows mode
  p.out_vec = (obase % (4 * osz) == 0) && (d->mode == FPK_CHAIN_FLAT || d->cols % 4 == 0);

  const bool flat = d->mode == FPK_CHAIN_FLAT;
  for (int i = 0; i < kMaxIn; ++i) p.in[i].mode = M_NONE;
  int staged_bytes = 0;
  bool any_col = false, any_row = false;
  for (int i = 0; i < d->n_inputs; ++i) {
    Input& in = p.in[i];
    in.ptr = inputs[i];
    if (!in.ptr) return FPK_ERR_INVALID;
    in.dtype = d->in_dtype[i];
    const int esz = elt_size(in.dtype);
    const uintptr_t a = reinterpret_cast<uintptr_t>(in.ptr);
    if (a % esz) return FPK_ERR_ALIGN;
    const bool vec_ok = a % (4 * esz) == 0;
    switch (d->in_bcast[i]) {
      case FPK_BCAST_FULL:
        if (flat && !(d->flags & FPK_FLAG_NO_STAGING) && a % 16 == 0 &&
            staged_bytes + kTile * esz <= kMaxStageBytes) {
          in.mode = M_STAGED;
          in.smem_off = static_cast<uint32_t>(staged_bytes);
          staged_bytes += kTile * esz;
        } else {
          in.mode = (vec_ok && (flat || d->cols % 4 == 0)) ? M_FULL_VEC : M_FULL_SCALAR;
        }
        break;
      case FPK_BCAST_COL:
        in.mode = (vec_ok && d->cols % 4 == 0) ? M_COL_VEC : M_COL_SCALAR;
        any_col |= in.mode == M_COL_VEC;
        break;
      case FPK_BCAST_ROW:
        in.mode = M_ROW;
        any_row = true;
        break;
      default:
        in.mode = M_SCALAR;
        break;
    }
  }

  if (flat) {
    rc = try_launch_chain_jit(d, inputs, out, stream, dev);
    if (rc != FPK_ERR_UNSUPPORTED) return rc;
    rc = try_launch_tiled(d, inputs, out, stream, dev);
    if (rc != FPK_ERR_UNSUPPORTED) return rc;
    p.num_tiles = (numel + kTile - 1) / kTile;
    p.stage_bytes = staged_bytes;
    int nstage = staged_bytes ? kStageBudget / staged_bytes : 2;
    nstage = nstage < 2 ? 2 : (nstage > kMaxStages ? kMaxStages : nstage);
    p.nstage = nstage;
    const int64_t max_grid = static_cast<int64_t>(dev.num_sms);
    const int grid = static_cast<int>(p.num_tiles < max_grid ? p.num_tiles : max_grid);
    // incremental (row, col) tracking is exact only when quads never straddle rows
    p.need_idx = (any_col || any_row) && d->cols % 4 == 0;
    if (p.need_idx) {
      const int64_t c = d->cols;
      p.col_step_q = static_cast<uint32_t>((4 * kNCT) % c);
      p.row_step_q = static_cast<uint32_t>((4 * kNCT) / c);
      const int64_t tstep = static_cast<int64_t>(grid) * kTile;
      p.col_step_t = static_cast<uint32_t>(tstep % c);
      p.row_step_t = tstep / c;
    }
    const int smem = nstage * staged_bytes;
    const bool spills = prog.uses_tmp;
    switch (d->n_inputs) {
      case 1: return spills ? launch_flat_n<1, 4>(p, grid, smem, stream) : launch_flat_n<1, 0>(p, grid, smem, stream);
      case 2: return spills ? launch_flat_n<2, 4>(p, grid, smem, stream) : launch_flat_n<2, 0>(p, grid, smem, stream);
      case 3: return spills ? launch_flat_n<3, 4>(p, grid, smem, stream) : launch_flat_n<3, 0>(p, grid, smem, stream);
      case 4: return spills ? launch_flat_n<4, 4>(p, grid, smem, stream) : launch_flat_n<4, 0>(p, grid, smem, stream);
      default: return spills ? launch_flat_n<8, 4>(p, grid, smem, stream) : launch_flat_n<8, 0>(p, grid, smem, stream);
    }
  }

  if (prog.softmax_pc < 0) return FPK_ERR_INVALID;
  rc = try_launch_chain_jit(d, inputs, out, stream, dev);
  if (rc != FPK_ERR_UNSUPPORTED) return rc;
  p.n_pre = prog.softmax_pc;
  for (int pc = prog.softmax_pc + 1; pc < prog.n; ++pc) {
    const int c = prog.code[pc];
    if (c < C_SAVE_T || (c >= C_ADD_IN && c < C_ADD_ACC) || (c >= C_MUL_IN && c < C_MUL_ACC)) p.post_reload = 1;
  }
  switch (d->n_inputs) {
    case 1: return launch_rows_n<1>(p, dev.num_sms, stream);
    case 2: return launch_rows_n<2>(p, dev.num_sms, stream);
    case 3: case 4: return launch_rows_n<4>(p, dev.num_sms, stream);
    default: return launch_rows_n<8>(p, dev.num_sms, stream);
  }
}

}  // namespace fpk
