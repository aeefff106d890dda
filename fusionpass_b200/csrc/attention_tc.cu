// f16 fp_attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Computes the reference kernel's result (lib/Plan/TritonEmitter.cpp:73-104,
// twin python/fusionpass/kernels.py:58-89): O = softmax(scale * Q K^T) V per
// (batch, head) with an online softmax, never writing the S x S scores.  Q K^T
// and P V run as f16 x f16 -> f32 UMMAs; the softmax is f32; P is rounded to
// f16 for the P V product; O is rounded once at the store.
//
// CTA = 2 query tiles of 128 rows of one (batch, head), 384 threads:
//   warps 0-3  softmax warpgroup of tile 0 (one thread per query row)
//   warps 4-7  softmax warpgroup of tile 1
//   warp  8    TMA producer: Q, then K_j / V_j 128-key tiles into a ring
//   warp  9    TMEM allocator + UMMA issuer (converged warp, one elected lane issues)
//   warps 10-11 idle (they complete the third warpgroup for setmaxnreg)
// Two kernels share this structure:
//
// attn_tcp_kernel, D <= 64 (split TMEM layout, persistent): S_t at columns
// 128 t, O_t at 256 + 64 t, P_t (f16, two per column) at 384 + 64 t.  Because
// P has its own columns, Q K^T of key tile j+1 is issued as soon as the softmax
// has read S_t(j) into registers and runs while the softmax computes P_t(j).
// One CTA per SM walks its work items; TMEM, the K/V ring and the barrier
// phases carry across items, Q is double-buffered so the next item's first
// Q K^T runs during the current item's last key tile, and O is staged in its
// own buffer, so an item's epilogue overlaps the next item's first tiles.  A
// last round of items that would keep at most half of the SMs busy runs as
// single-tile items (each 256-row block split in two).  The kernel
// is launched as a programmatic dependent launch: its set-up (barriers, TMEM)
// overlaps the end of the stream's previous kernel, and griddepcontrol.wait
// holds every global access until that kernel has completed.
//
// attn_tc_kernel, D = 128 (aliased TMEM layout, one CTA per work item): S_t at
// 128 t, O_t at 256 + 128 t; P_t overwrites the first 64 columns of S_t.  UMMAs
// issued by one thread execute in order, so Q K^T of the next key tile is
// issued into S_t right after the P V UMMA that reads P_t from it.  P_t is
// stored in two halves (keys 0-63, 64-127) with a barrier each: the P V
// k-steps of the first half run while the softmax still computes the second.
//
// In both, the two softmax warpgroups take turns at the exponentials (a pair
// of turn barriers, handed over before the end of each phase); 2 of every 8
// score pairs are exponentiated on the FMA pipe (ex2_poly2) and the rest on
// the MUFU.
//
// Softmax per row (log2 domain, scale folded into one FFMA per score):
// m = running max actually used for the exponentials; O and l are rescaled
// only when the tile max exceeds m by more than 2^8 (P values stay <= 256 and
// exact in f16 range), which leaves the final O = acc / l unchanged
// mathematically.  Out-of-range keys of the last tile get p = 0, out-of-range
// query rows are clipped by the TMA store.
//
// Every mbarrier wait is bounded (see common.cuh); on a timeout all roles stop,
// in-flight TMA loads and UMMAs are drained, TMEM is freed and the kernel
// returns with FPK_ERR_TIMEOUT in the status word.
#include <cuda.h>

#include <atomic>
#include <cmath>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "internal.h"
#include "tmem_ops.cuh"

namespace fpk {
namespace attn_tc {

constexpr int kBM = 128;  // query rows per tile (UMMA M)
constexpr int kBN = 128;  // keys per iteration
constexpr int kTiles = 2; // query tiles per CTA
constexpr int kWG = 128;  // softmax threads per tile
constexpr int kTmaWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 384;  // 3 warpgroups: softmax tile 0, softmax tile 1, TMA + UMMA + 2 idle warps
// setmaxnreg split of the 384 x 168 registers the CTA is launched with:
// 2 x 128 x 216 (softmax) + 128 x 72 (control warpgroup) = 64512.
constexpr int kRegsSoftmax = 216;
constexpr int kRegsCtl = 72;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsCtl <= kThreads * 168, "setmaxnreg split exceeds the launch");
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.0f;
constexpr uint32_t kPolyPairs = 0x11u;  // pairs (c/2) mod 8 in {0, 4} use the FMA-pipe exp2
constexpr int kTurnAt = 104;            // score column after which the exponential turn passes
constexpr int kHalfSignalAt = 78;       // score column at which the first half of P_t is signalled (D = 128)
static_assert(kHalfSignalAt % 2 == 0 && kHalfSignalAt >= kBN / 2 - 2 && kHalfSignalAt < kBN,
              "the half signal follows the store of P for keys 0-63 inside the exponential loop");
constexpr int kMinSmem = 116 * 1024;  // keeps one CTA per SM (it owns all 512 TMEM columns)

template <int D>
struct Cfg {
  static constexpr int kBoxCols = D >= 64 ? 64 : D;     // elements per swizzled row
  static constexpr int kRowBytes = kBoxCols * 2;
  static constexpr int kBoxes = D / kBoxCols;
  static constexpr int kBoxBytes = 128 * kRowBytes;     // 128 rows of one box
  static constexpr int kTileBytes = kBoxes * kBoxBytes; // 128 x D f16
  static constexpr int kStages = D == 128 ? 2 : 3;
  static constexpr uint32_t kLayout = D >= 64 ? 2u : (D == 32 ? 4u : 6u);  // SW128 / SW64 / SW32
  static constexpr uint32_t kSwzMask = D >= 64 ? 7u : (D == 32 ? 3u : 1u);
  static constexpr int kKStepsPerBox = kRowBytes / 32;  // 16 f16 = 32 B per UMMA k-step
  static constexpr int kSmemBytes = (kTiles + 2 * kStages) * kTileBytes + 1024;
  static constexpr int kLaunchSmem = kSmemBytes > kMinSmem ? kSmemBytes : kMinSmem;
};

struct Params {
  int* status;
  int32_t heads;
  int32_t seq;
  int32_t num_mblocks;
  int32_t num_items;   // work items of the persistent kernel
  int32_t split_from;  // persistent kernel: items from here on are single 128-row tiles
  float scale_log2;  // scale * log2(e)
  uint32_t flags;
};

struct Bars {
  uint64_t q_full;
  uint64_t k_full[3], k_empty[3], v_full[3], v_empty[3];
  // p_full / turn: one arrival per softmax warp (lane 0 after __syncwarp)
  uint64_t s_full[kTiles], p_full[kTiles], o_done[kTiles];
  uint64_t p_half[kTiles];  // P_t of keys 0-63 is in TMEM
  uint64_t turn[kTiles];    // ping-pong of the exponential phases of the two tiles
  uint64_t epi[kTiles];     // the 4 warps of a tile before the O store (a bounded wait)
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

// ------------------------------------------------------------- PTX glue ---
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}

// kind::f16 instruction descriptor: f16 A and B, f32 accumulator, A K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n, bool b_mn_major) {
  return (1u << 4) | (b_mn_major ? (1u << 16) : 0u) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                       uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Issue forms for the converged UMMA warp: every lane executes them and the
// lane holding `leader` (from elect_one) issues.  A converged warp issues UMMAs
// markedly faster than a lone lane inside a divergent branch.
__device__ __forceinline__ uint32_t elect_one() {
  uint32_t e;
  asm volatile("{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\tselp.u32 %0, 1, 0, e;\n\t}" : "=r"(e));
  return e;
}
__device__ __forceinline__ void mma_ss_l(uint32_t leader, uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 e, %5, 0;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(leader));
}
__device__ __forceinline__ void mma_ts_l(uint32_t leader, uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                         uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 e, %5, 0;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc), "r"(leader));
}
__device__ __forceinline__ void mma_commit_l(uint32_t leader, uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\tsetp.ne.b32 e, %1, 0;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar)),
      "r"(leader)
      : "memory");
}

template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int x, int y, int z,
                                             int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// three-input max / min (one instruction folds two new scores into a running value)
__device__ __forceinline__ float max3(float a, float b, float c) {
  float y;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(y) : "f"(a), "f"(b), "f"(c));
  return y;
}
__device__ __forceinline__ float min3(float a, float b, float c) {
  float y;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(y) : "f"(a), "f"(b), "f"(c));
  return y;
}

// packed pair arithmetic on two f32 lanes (same IEEE result per lane as the scalar op)
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b, float c) {
  asm("{\n\t.reg .b64 x, y, z;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %4};\n\tmov.b64 z, {%5, %5};\n\t"
      "fma.rn.f32x2 x, x, y, z;\n\tmov.b64 {%0, %1}, x;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b), "f"(c));
}
// d = a * b + c per lane, c broadcast
__device__ __forceinline__ void fma2v(float& d0, float& d1, float a0, float a1, float b0, float b1, float c) {
  asm("{\n\t.reg .b64 x, y, z;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\tmov.b64 z, {%6, %6};\n\t"
      "fma.rn.f32x2 x, x, y, z;\n\tmov.b64 {%0, %1}, x;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c));
}
__device__ __forceinline__ void sub2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 x, y;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\t"
      "sub.rn.f32x2 x, x, y;\n\tmov.b64 {%0, %1}, x;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// 2^x for a pair on the FMA pipe, to offload the MUFU (16 ex2 per clock per SM).
// Range reduction in base 2: n = rint(x) by the 1.5 * 2^23 shifter (whose low
// mantissa bits then hold n), f = x - n in [-1/2, 1/2]; 2^f by a degree-3
// polynomial fitted here by linear programming for minimax relative error on
// [-1/2, 1/2] (max 7.5e-5 in f32 Horner evaluation, below the 4.9e-4 f16
// rounding that P gets next); the result exponent is raised by n with one
// integer add.  x is clamped at -126 first (p(f) may lie below 1, so n >= -126
// keeps the exponent field from wrapping into the sign bit); x = -inf (masked
// keys) then gives a value below 1.2e-38, which is 0 once P is rounded to f16.
constexpr float kExp2C0 = 0.9999280571937561f;
constexpr float kExp2C1 = 0.6932609677314758f;
constexpr float kExp2C2 = 0.2426111251115799f;
constexpr float kExp2C3 = 0.0551716685295105f;
__device__ __forceinline__ void ex2_poly2(float& r0, float& r1, float x0, float x1) {
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
  x0 = fmaxf(x0, -126.0f);
  x1 = fmaxf(x1, -126.0f);
  float t0, t1, n0, n1, f0, f1, p0, p1;
  fma2(t0, t1, x0, x1, 1.0f, kShift);
  sub2(n0, n1, t0, t1, kShift, kShift);
  sub2(f0, f1, x0, x1, n0, n1);
  fma2v(p0, p1, f0, f1, kExp2C3, kExp2C3, kExp2C2);
  fma2v(p0, p1, p0, p1, f0, f1, kExp2C1);
  fma2v(p0, p1, p0, p1, f0, f1, kExp2C0);
  r0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  r1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

__device__ __forceinline__ void add2(float& a0, float& a1, float b0, float b1) {
  asm("{\n\t.reg .b64 x, y;\n\tmov.b64 x, {%0, %1};\n\tmov.b64 y, {%2, %3};\n\t"
      "add.rn.f32x2 x, x, y;\n\tmov.b64 {%0, %1}, x;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1));
}

// non-blocking probe of an mbarrier phase (the UMMA issuer polls two tiles)
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Warp-uniform barrier probes for the converged UMMA warp: lane 0's answer is
// broadcast so every lane takes the same branch.
__device__ __forceinline__ bool mbar_test_w(uint64_t* bar, uint32_t parity) {
  return __shfl_sync(0xffffffffu, mbar_test(bar, parity) ? 1 : 0, 0) != 0;
}
__device__ __forceinline__ bool mbar_wait_w(uint64_t* bar, uint32_t parity, volatile int* abort, int* status,
                                            uint64_t limit_ns) {
  if (mbar_test_w(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (__shfl_sync(0xffffffffu, mbar_try_wait(bar, parity) ? 1 : 0, 0)) return true;
    if ((i & 63u) == 0u) {
      int stop = 0;
      if ((threadIdx.x & 31) == 0) {
        if (*abort) {
          stop = 1;
        } else if (globaltimer_ns() - t0 > limit_ns) {
          record_status(status, FPK_ERR_TIMEOUT);
          *abort = 1;
          stop = 1;
        }
      }
      if (__shfl_sync(0xffffffffu, stop, 0)) return false;
    }
  }
}

// Bounded wait that ignores the abort flag: used to drain in-flight async work.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity, int* status) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      record_status(status, FPK_ERR_TIMEOUT);
      return;
    }
  }
}

// drain_wait for the converged UMMA warp (lane 0 decides, all lanes follow)
__device__ __forceinline__ void drain_wait_w(uint64_t* bar, uint32_t parity, int* status) {
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    int state = 0;
    if ((threadIdx.x & 31) == 0) {
      if (mbar_try_wait(bar, parity)) {
        state = 1;
      } else if (globaltimer_ns() - t0 > kWaitLimitNs) {
        record_status(status, FPK_ERR_TIMEOUT);
        state = 2;
      }
    }
    if (__shfl_sync(0xffffffffu, state, 0)) return;
  }
}

template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t* r) {
  static_assert(N == 8 || N == 16 || N == 32 || N == 64 || N == 128, "no tcgen05.ld form for this width");
  if constexpr (N == 8) tmem_ld_x8(taddr, r);
  else if constexpr (N == 16) tmem_ld_x16(taddr, r);
  else if constexpr (N == 32) tmem_ld_x32(taddr, r);
  else if constexpr (N == 64) tmem_ld_x64(taddr, r);
  else tmem_ld_x128(taddr, r);
}
template <int N>
__device__ __forceinline__ void tmem_st(uint32_t taddr, const uint32_t* r) {
  static_assert(N == 8 || N == 16 || N == 32 || N == 64 || N == 128, "no tcgen05.st form for this width");
  if constexpr (N == 8) tmem_st_x8(taddr, r);
  else if constexpr (N == 16) tmem_st_x16(taddr, r);
  else if constexpr (N == 32) tmem_st_x32(taddr, r);
  else if constexpr (N == 64) tmem_st_x64(taddr, r);
  else tmem_st_x128(taddr, r);
}

// ------------------------------------------------------------- the kernel ---
template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap to,
                   const __grid_constant__ Params p) {
  using C = Cfg<D>;
  constexpr int NS = C::kStages;
  static_assert(D == 128, "D <= 64 runs in attn_tcp_kernel");
  // TMEM columns: S_t at 128 t, O_t at 256 + 128 t; P_t overwrites the first 64
  // columns of S_t (aliased layout).
  constexpr uint32_t kOCol0 = 256u, kOStride = 128u;
  constexpr uint32_t kPCol0 = 0u, kPStride = 128u;
  extern __shared__ uint8_t smem_raw[];
  __shared__ Bars bars;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kTiles * C::kTileBytes;
  uint8_t* sV = sK + NS * C::kTileBytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bh = static_cast<int>(blockIdx.x / p.num_mblocks);
  const int mb = static_cast<int>(blockIdx.x % p.num_mblocks);
  const int hh = bh % p.heads;
  const int bb = bh / p.heads;
  const int S = p.seq;
  const int m0 = mb * (kTiles * kBM);
  const int ntiles = (m0 + kBM < S) ? 2 : 1;
  const int nkv = (S + kBN - 1) / kBN;
  const bool test_timeout = (p.flags & FPK_FLAG_TEST_TIMEOUT) != 0;
  const uint64_t limit = test_timeout ? kTestWaitLimitNs : kWaitLimitNs;
  volatile int* abort = &bars.abort;

  if (threadIdx.x == 0) {
    mbar_init(&bars.q_full, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&bars.k_full[s], 1);
      mbar_init(&bars.k_empty[s], 1);
      mbar_init(&bars.v_full[s], 1);
      mbar_init(&bars.v_empty[s], 1);
    }
    for (int t = 0; t < kTiles; ++t) {
      mbar_init(&bars.s_full[t], 1);
      mbar_init(&bars.p_half[t], kWG / 32);
      mbar_init(&bars.p_full[t], kWG / 32);
      mbar_init(&bars.o_done[t], 1);
      mbar_init(&bars.turn[t], kWG / 32);
      mbar_init(&bars.epi[t], kWG / 32);
    }
    mbar_init(&bars.drain, 1);
    bars.abort = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&bars.tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars.tmem_base;

  if (warp >= 2 * kWG / 32) {
    // TMA producer, UMMA issuer and two idle warps give registers to the softmax
    setmaxnreg_dec<kRegsCtl>();
    if (warp == kTmaWarp) {
      // --------------------------------------------------------- TMA producer
      if (lane == 0) {
        bool q_issued = false;
        int last_k[NS], last_v[NS];
        for (int s = 0; s < NS; ++s) last_k[s] = last_v[s] = -1;
        if (!test_timeout) {  // the timeout test withholds Q on purpose
          mbar_arrive_expect_tx(&bars.q_full, static_cast<uint32_t>(ntiles * C::kTileBytes));
          for (int t = 0; t < ntiles; ++t)
            for (int bx = 0; bx < C::kBoxes; ++bx)
              tma_load_4d(sQ + t * C::kTileBytes + bx * C::kBoxBytes, &tq, bx * C::kBoxCols, m0 + t * kBM, hh,
                          bb, &bars.q_full);
          q_issued = true;
        }
        for (int j = 0; j < nkv; ++j) {
          const int s = j % NS;
          const uint32_t r = static_cast<uint32_t>(j / NS);
          if (!mbar_wait(&bars.k_empty[s], (r & 1u) ^ 1u, abort, p.status, limit)) break;
          mbar_arrive_expect_tx(&bars.k_full[s], C::kTileBytes);
          for (int bx = 0; bx < C::kBoxes; ++bx)
            tma_load_4d(sK + s * C::kTileBytes + bx * C::kBoxBytes, &tk, bx * C::kBoxCols, j * kBN, hh, bb,
                        &bars.k_full[s]);
          last_k[s] = j;
          if (!mbar_wait(&bars.v_empty[s], (r & 1u) ^ 1u, abort, p.status, limit)) break;
          mbar_arrive_expect_tx(&bars.v_full[s], C::kTileBytes);
          for (int bx = 0; bx < C::kBoxes; ++bx)
            tma_load_4d(sV + s * C::kTileBytes + bx * C::kBoxBytes, &tv, bx * C::kBoxCols, j * kBN, hh, bb,
                        &bars.v_full[s]);
          last_v[s] = j;
        }
        // no TMA write may land after the CTA has gone
        if (q_issued) drain_wait(&bars.q_full, 0, p.status);
        for (int s = 0; s < NS; ++s) {
          if (last_k[s] >= 0) drain_wait(&bars.k_full[s], static_cast<uint32_t>(last_k[s] / NS) & 1u, p.status);
          if (last_v[s] >= 0) drain_wait(&bars.v_full[s], static_cast<uint32_t>(last_v[s] / NS) & 1u, p.status);
        }
      }
    } else if (warp == kMmaWarp) {
      // ------------------------------------------------ UMMA issuer (whole warp)
      // The warp runs converged; one elected lane issues.  Descriptors are kept
      // as bases plus compile-time k-step offsets, ring positions as counters, so
      // the issue path is a few instructions per UMMA.
      constexpr uint32_t idesc_qk = idesc_f16(kBM, kBN, false);
      constexpr uint32_t idesc_pv = idesc_f16(kBM, D, true);
      constexpr uint64_t kTileStep = static_cast<uint64_t>(C::kTileBytes >> 4);  // descriptor units
      const uint32_t leader = elect_one();
      const uint64_t q_desc = sdesc(smem_u32(sQ), 16, 8 * C::kRowBytes, C::kLayout);
      const uint64_t k_desc = sdesc(smem_u32(sK), 16, 8 * C::kRowBytes, C::kLayout);
      const uint64_t v_desc = sdesc(smem_u32(sV), C::kBoxBytes, 8 * C::kRowBytes, C::kLayout);
      auto issue_qk = [&](int t, int s) {
        const uint32_t d_tmem = tbase + static_cast<uint32_t>(t * 128);
        const uint64_t a0 = q_desc + static_cast<uint64_t>(t) * kTileStep;
        const uint64_t b0 = k_desc + static_cast<uint64_t>(s) * kTileStep;
  #pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          constexpr int kSteps = C::kKStepsPerBox;
          const uint64_t off = static_cast<uint64_t>((kk / kSteps) * (C::kBoxBytes >> 4) + (kk % kSteps) * 2);
          mma_ss_l(leader, d_tmem, a0 + off, b0 + off, idesc_qk, kk > 0 ? 1u : 0u);
        }
      };
      // P V k-steps of one half of the keys (half 0: keys 0-63, half 1: 64-127)
      auto issue_pv = [&](int t, int s, bool accumulate, int half) {
        const uint32_t d_tmem = tbase + kOCol0 + static_cast<uint32_t>(t) * kOStride;
        const uint32_t a_tmem = tbase + kPCol0 + static_cast<uint32_t>(t) * kPStride;
        const uint64_t b0 = v_desc + static_cast<uint64_t>(s) * kTileStep;
  #pragma unroll
        for (int k2 = 0; k2 < kBN / 32; ++k2) {
          const int kk = half * (kBN / 32) + k2;
          mma_ts_l(leader, d_tmem, a_tmem + static_cast<uint32_t>(kk * 8),
                   b0 + static_cast<uint64_t>(kk * C::kRowBytes), idesc_pv, (accumulate || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait_w(&bars.q_full, 0, abort, p.status, limit) &&
                mbar_wait_w(&bars.k_full[0], 0, abort, p.status, limit);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < ntiles; ++t) {
          issue_qk(t, 0);
          mma_commit_l(leader, &bars.s_full[t]);
        }
        mma_commit_l(leader, &bars.k_empty[0]);
      }
      int s = 0, s1 = 1 % NS;
      uint32_t r = 0u, r1 = NS == 1 ? 1u : 0u;
      for (int j = 0; ok && j < nkv; ++j) {
        const bool more = j + 1 < nkv;
        if (!mbar_wait_w(&bars.v_full[s], r, abort, p.status, limit)) break;
        for (int t = 0; t < ntiles; ++t) {
          if (!mbar_wait_w(&bars.p_half[t], static_cast<uint32_t>(j) & 1u, abort, p.status, limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(t, s, j > 0, 0);
          if (!mbar_wait_w(&bars.p_full[t], static_cast<uint32_t>(j) & 1u, abort, p.status, limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(t, s, j > 0, 1);
          mma_commit_l(leader, &bars.o_done[t]);
          if (more) {
            if (t == 0 && !mbar_wait_w(&bars.k_full[s1], r1, abort, p.status, limit)) {
              ok = false;
              break;
            }
            issue_qk(t, s1);
            mma_commit_l(leader, &bars.s_full[t]);
          }
        }
        if (!ok) break;
        mma_commit_l(leader, &bars.v_empty[s]);
        if (more) mma_commit_l(leader, &bars.k_empty[s1]);
        s = s1;
        r = r1;
        if (++s1 == NS) {
          s1 = 0;
          r1 ^= 1u;
        }
      }
      // every UMMA issued so far must finish before TMEM is freed
      mma_commit_l(leader, &bars.drain);
      drain_wait_w(&bars.drain, 0, p.status);
    }
  } else {
    // ------------------------------------------------------ softmax + epilogue
    setmaxnreg_inc<kRegsSoftmax>();
    const int t = warp >> 2;
    const int row = threadIdx.x & (kWG - 1);
    if (t < ntiles) {
      const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
      const uint32_t tS = tbase + lane_off + static_cast<uint32_t>(t * 128);
      const uint32_t tO = tbase + lane_off + kOCol0 + static_cast<uint32_t>(t) * kOStride;
      const uint32_t tP = tbase + lane_off + kPCol0 + static_cast<uint32_t>(t) * kPStride;
      // scale 0 runs as the smallest normal float: every finite score still maps to
      // 2^0 = 1 in f32, and the masked (infinite) scores of a ragged tile to 0
      const float k2 = p.scale_log2 == 0.0f ? 1.17549435e-38f : p.scale_log2;
      const bool pos = k2 >= 0.0f;
      const float init = pos ? -INFINITY : INFINITY;  // masked score: exp2(init * k2) = 0
      float m_run = -INFINITY;
      float l = 0.0f;
      bool ok = true;
      for (int j = 0; j < nkv; ++j) {
        if (!mbar_wait(&bars.s_full[t], static_cast<uint32_t>(j) & 1u, abort, p.status, limit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[128];
        tmem_ld_x128(tS, sr);
        const int valid = S - j * kBN;  // > 0; < 128 only on the last tile
        if (valid < kBN) {
#pragma unroll
          for (int c = 0; c < kBN; ++c)
            if (c >= valid) sr[c] = __float_as_uint(init);
        }
        // row max (min for a negative scale), two scores per instruction, 8 chains
        float m8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) m8[i] = init;
        if (pos) {
#pragma unroll
          for (int c = 0; c < kBN; c += 2)
            m8[(c >> 1) & 7] = max3(m8[(c >> 1) & 7], __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
        } else {
#pragma unroll
          for (int c = 0; c < kBN; c += 2)
            m8[(c >> 1) & 7] = min3(m8[(c >> 1) & 7], __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
        }
        float mx = pos ? max3(max3(m8[0], m8[1], m8[2]), max3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]))
                       : min3(min3(m8[0], m8[1], m8[2]), min3(m8[3], m8[4], m8[5]), fminf(m8[6], m8[7]));
        mx *= k2;  // row max of the log2-scaled scores
        if (j == 0) {
          m_run = mx;
        } else {
          const bool need = mx > m_run + kRescaleLog2;
          if (__any_sync(0xffffffffu, need)) {
            const float alpha = need ? ex2(m_run - mx) : 1.0f;
            if (need) m_run = mx;
            l *= alpha;
            // O_t holds P_{j-1} V_{j-1}: the commit that signalled S_t covers
            // every earlier UMMA of this CTA.
            constexpr int kChunk = D < 32 ? D : 32;
#pragma unroll
            for (int c0 = 0; c0 < D; c0 += kChunk) {
              uint32_t orow[kChunk];
              tmem_ld<kChunk>(tO + static_cast<uint32_t>(c0), orow);
#pragma unroll
              for (int c = 0; c < kChunk; ++c) orow[c] = __float_as_uint(__uint_as_float(orow[c]) * alpha);
              tmem_st<kChunk>(tO + static_cast<uint32_t>(c0), orow);
            }
          }
        }
        // Ping-pong: the two warpgroups take turns at the exponentials (the MUFU
        // bound), so one tile's max, rescale and TMEM traffic -- and, in the
        // aliased layout, its UMMAs -- overlap the other tile's exponentials.
        // Tile 0 waits for tile 1's previous turn.
        if (ntiles == 2 && (t == 1 || j > 0)) {
          const uint32_t par = static_cast<uint32_t>(t == 1 ? j : j - 1) & 1u;
          if (!mbar_wait(&bars.turn[t], par, abort, p.status, limit)) {
            ok = false;
            break;
          }
        }
        const float neg_m = -m_run;
        float la[4] = {0.0f, 0.0f, 0.0f, 0.0f}, lb[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        // p = 2^(s * scale * log2 e - m); P packed to f16 pairs in place (sr[c/2])
        // 2 of every 8 pairs take the FMA-pipe exp2, the rest the MUFU; the turn
        // passes to the other tile a quarter before the end, so its wake-up
        // overlaps this tile's last exponentials.  P of keys 0-63 goes to TMEM
        // once computed and is signalled a few pairs later (its store has
        // landed by then), so its P V k-steps start during the second half.
#pragma unroll
        for (int c = 0; c < kBN; c += 2) {
          float x0, x1, p0, p1;
          fma2(x0, x1, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]), k2, neg_m);
          if ((kPolyPairs >> ((c >> 1) & 7)) & 1) {
            ex2_poly2(p0, p1, x0, x1);
          } else {
            p0 = ex2(x0);  // masked keys: x = -inf, p = 0
            p1 = ex2(x1);
          }
          add2(la[(c >> 1) & 3], lb[(c >> 1) & 3], p0, p1);
          sr[c >> 1] = pack_half2(p0, p1);
          if (c == kBN / 2 - 2) tmem_st_x32(tP, sr);
          if (c == kHalfSignalAt) {
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars.p_half[t]);
          }
          if (c == kTurnAt && ntiles == 2) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars.turn[1 - t]);
          }
        }
        l += ((la[0] + lb[0]) + (la[1] + lb[1])) + ((la[2] + lb[2]) + (la[3] + lb[3]));
        tmem_st_x32(tP + 32u, sr + 32);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.p_full[t]);
      }
      // epilogue: O / l -> f16 -> swizzled staging (the Q_t buffer) -> TMA store
      if (ok && mbar_wait(&bars.o_done[t], static_cast<uint32_t>(nkv - 1) & 1u, abort, p.status, limit)) {
        tc_fence_after();
        uint8_t* stage = sQ + t * C::kTileBytes;
        // O / l as O * (1 / l): one correctly rounded reciprocal per row instead of
        // an IEEE division per element (within 1 ulp of f32, far below the f16 store)
        const float rl = __frcp_rn(l);
        constexpr int kChunk = D < 32 ? D : 32;
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += kChunk) {
          uint32_t orow[kChunk];
          tmem_ld<kChunk>(tO + static_cast<uint32_t>(c0), orow);
          uint32_t h2[kChunk / 2];
#pragma unroll
          for (int c = 0; c < kChunk; c += 2)
            h2[c / 2] = pack_half2(__fmul_rn(__uint_as_float(orow[c]), rl),
                                   __fmul_rn(__uint_as_float(orow[c + 1]), rl));
#pragma unroll
          for (int q = 0; q < kChunk / 8; ++q) {
            const int col = c0 + q * 8;  // first element of this 16-byte chunk
            const int bx = col / C::kBoxCols;
            const uint32_t off = static_cast<uint32_t>(row * C::kRowBytes + (col % C::kBoxCols) * 2);
            const uint32_t phys = off ^ (((off >> 7) & C::kSwzMask) << 4);
            *reinterpret_cast<uint4*>(stage + bx * C::kBoxBytes + phys) =
                make_uint4(h2[q * 4], h2[q * 4 + 1], h2[q * 4 + 2], h2[q * 4 + 3]);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.epi[t]);
        if (mbar_wait(&bars.epi[t], 0, abort, p.status, limit) && row == 0) {
          for (int bx = 0; bx < C::kBoxes; ++bx)
            tma_store_4d(&to, stage + bx * C::kBoxBytes, bx * C::kBoxCols, m0 + t * kBM, hh, bb);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kTmemCols));
  }
}


// ---------------------------------------------- persistent kernel, D <= 64 ---
// One CTA per SM walks the work items (batch*head, 256-row query block)
// blockIdx.x, blockIdx.x + gridDim.x, ...  TMEM is allocated once; the K/V ring
// and every barrier phase run on across items.  Q is double-buffered by item
// parity: the next item's Q loads during the current item, and the next item's
// first Q K^T is issued at the start of the current item's last key iteration,
// so a softmax warpgroup finds its next S ready when it finishes an item.  O is
// staged in its own buffer, so an item's epilogue overlaps the first tiles of the
// next.  Within an item the schedule is the split-layout one of attn_tc_kernel.
struct PBars {
  uint64_t q_full[2], q_empty[2];  // Q double-buffered by item parity
  uint64_t k_full[3], k_empty[3], v_full[3], v_empty[3];
  uint64_t s_full[kTiles], p_full[kTiles], o_done[kTiles], s_free[kTiles], turn[kTiles];
  uint64_t epi[kTiles][2];  // the 4 warps of a tile, twice per epilogue (bounded waits)
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void tma_store_4d_async(const CUtensorMap* map, const void* src, int x, int y, int z,
                                                   int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tcp_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap to,
                    const __grid_constant__ Params p) {
  static_assert(D <= 64, "the persistent kernel uses the split TMEM layout");
  using C = Cfg<D>;
  constexpr int NS = C::kStages;
  constexpr uint32_t kOCol0 = 256u, kOStride = 64u, kPCol0 = 384u, kPStride = 64u;
  extern __shared__ uint8_t smem_raw[];
  __shared__ PBars bars;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                      // two Q buffers of kTiles tiles (by item parity)
  uint8_t* sK = sQ + 2 * kTiles * C::kTileBytes;
  uint8_t* sV = sK + NS * C::kTileBytes;
  uint8_t* sO = sV + NS * C::kTileBytes;  // O staging for the TMA store, one tile per softmax warpgroup

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = p.seq;
  const int nkv = (S + kBN - 1) / kBN;
  const int total = p.num_items;
  const bool test_timeout = (p.flags & FPK_FLAG_TEST_TIMEOUT) != 0;
  const uint64_t limit = test_timeout ? kTestWaitLimitNs : kWaitLimitNs;
  volatile int* abort = &bars.abort;
  // item w: a (batch*head, 256-row block) pair of query tiles, or, from split_from on,
  // one 128-row half of such a block (items 2i and 2i + 1 past split_from are the two
  // halves of block split_from + i)
  auto coords = [&](int w, int& hh, int& bb, int& m0, int& ntiles) {
    const bool single = w >= p.split_from;
    const int i = w - p.split_from;
    const int pw = single ? p.split_from + (i >> 1) : w;
    const int bh = pw / p.num_mblocks;
    m0 = (pw % p.num_mblocks) * (kTiles * kBM) + (single ? (i & 1) * kBM : 0);
    hh = bh % p.heads;
    bb = bh / p.heads;
    ntiles = (!single && m0 + kBM < S) ? 2 : 1;
  };

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars.q_full[b], 1);
      mbar_init(&bars.q_empty[b], 1);
    }
    for (int s = 0; s < NS; ++s) {
      mbar_init(&bars.k_full[s], 1);
      mbar_init(&bars.k_empty[s], 1);
      mbar_init(&bars.v_full[s], 1);
      mbar_init(&bars.v_empty[s], 1);
    }
    for (int t = 0; t < kTiles; ++t) {
      mbar_init(&bars.s_full[t], 1);
      mbar_init(&bars.p_full[t], kWG / 32);
      mbar_init(&bars.o_done[t], 1);
      mbar_init(&bars.s_free[t], kWG / 32);
      mbar_init(&bars.turn[t], kWG / 32);
      mbar_init(&bars.epi[t][0], kWG / 32);
      mbar_init(&bars.epi[t][1], kWG / 32);
    }
    mbar_init(&bars.drain, 1);
    bars.abort = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&bars.tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars.tmem_base;
  // programmatic dependent launch: the stream's next kernel may be scheduled from now on
  // (its CTAs find no room on an SM before this kernel's CTA there has exited), and this
  // kernel touches global memory only once the previous kernel has completed and its
  // writes are visible
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp >= 2 * kWG / 32) {
    setmaxnreg_dec<kRegsCtl>();
    if (warp == kTmaWarp) {
      // --------------------------------------------------------- TMA producer
      if (lane == 0) {
        int kp = 0, vp = 0;  // ring slot of the next K / V load
        uint32_t kph = 0u, vph = 0u;
        int last_k[NS], last_v[NS];  // phase parity of each slot's last load, -1 if none
        for (int s = 0; s < NS; ++s) last_k[s] = last_v[s] = -1;
        uint32_t qn = 0;  // Q loads issued
        bool ok = !test_timeout;  // the timeout test withholds every load on purpose
        for (int w = blockIdx.x; ok && w < total; w += gridDim.x) {
          int hh, bb, m0, ntiles;
          coords(w, hh, bb, m0, ntiles);
          // Q buffer qb is free once the last Q K^T of the item two back has completed
          const uint32_t qb = qn & 1u;
          if (qn >= 2u && !mbar_wait(&bars.q_empty[qb], ((qn >> 1) - 1u) & 1u, abort, p.status, limit)) break;
          mbar_arrive_expect_tx(&bars.q_full[qb], static_cast<uint32_t>(ntiles * C::kTileBytes));
          for (int t = 0; t < ntiles; ++t)
            for (int bx = 0; bx < C::kBoxes; ++bx)
              tma_load_4d(sQ + (qb * kTiles + t) * C::kTileBytes + bx * C::kBoxBytes, &tq, bx * C::kBoxCols,
                          m0 + t * kBM, hh, bb, &bars.q_full[qb]);
          ++qn;
          for (int j = 0; j < nkv; ++j) {
            if (!mbar_wait(&bars.k_empty[kp], kph ^ 1u, abort, p.status, limit)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bars.k_full[kp], C::kTileBytes);
            for (int bx = 0; bx < C::kBoxes; ++bx)
              tma_load_4d(sK + kp * C::kTileBytes + bx * C::kBoxBytes, &tk, bx * C::kBoxCols, j * kBN, hh, bb,
                          &bars.k_full[kp]);
            last_k[kp] = static_cast<int>(kph);
            if (++kp == NS) {
              kp = 0;
              kph ^= 1u;
            }
            if (!mbar_wait(&bars.v_empty[vp], vph ^ 1u, abort, p.status, limit)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bars.v_full[vp], C::kTileBytes);
            for (int bx = 0; bx < C::kBoxes; ++bx)
              tma_load_4d(sV + vp * C::kTileBytes + bx * C::kBoxBytes, &tv, bx * C::kBoxCols, j * kBN, hh, bb,
                          &bars.v_full[vp]);
            last_v[vp] = static_cast<int>(vph);
            if (++vp == NS) {
              vp = 0;
              vph ^= 1u;
            }
          }
        }
        // no TMA write may land after the CTA has gone
        for (uint32_t b = 0; b < 2u; ++b) {
          const uint32_t loads = (qn + 1u - b) >> 1;  // loads into buffer b
          if (loads > 0u) drain_wait(&bars.q_full[b], (loads - 1u) & 1u, p.status);
        }
        for (int s = 0; s < NS; ++s) {
          if (last_k[s] >= 0) drain_wait(&bars.k_full[s], static_cast<uint32_t>(last_k[s]), p.status);
          if (last_v[s] >= 0) drain_wait(&bars.v_full[s], static_cast<uint32_t>(last_v[s]), p.status);
        }
      }
    } else if (warp == kMmaWarp) {
      // ------------------------------------------------ UMMA issuer (whole warp)
      constexpr uint32_t idesc_qk = idesc_f16(kBM, kBN, false);
      constexpr uint32_t idesc_pv = idesc_f16(kBM, D, true);
      constexpr uint64_t kTileStep = static_cast<uint64_t>(C::kTileBytes >> 4);
      const uint32_t leader = elect_one();
      const uint64_t q_desc = sdesc(smem_u32(sQ), 16, 8 * C::kRowBytes, C::kLayout);
      const uint64_t k_desc = sdesc(smem_u32(sK), 16, 8 * C::kRowBytes, C::kLayout);
      const uint64_t v_desc = sdesc(smem_u32(sV), C::kBoxBytes, 8 * C::kRowBytes, C::kLayout);
      auto issue_qk = [&](int t, uint32_t qb, int s) {
        const uint32_t d_tmem = tbase + static_cast<uint32_t>(t * 128);
        const uint64_t a0 = q_desc + static_cast<uint64_t>(qb * kTiles + t) * kTileStep;
        const uint64_t b0 = k_desc + static_cast<uint64_t>(s) * kTileStep;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          constexpr int kSteps = C::kKStepsPerBox;
          const uint64_t off = static_cast<uint64_t>((kk / kSteps) * (C::kBoxBytes >> 4) + (kk % kSteps) * 2);
          mma_ss_l(leader, d_tmem, a0 + off, b0 + off, idesc_qk, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int t, int s, bool accumulate) {
        const uint32_t d_tmem = tbase + kOCol0 + static_cast<uint32_t>(t) * kOStride;
        const uint32_t a_tmem = tbase + kPCol0 + static_cast<uint32_t>(t) * kPStride;
        const uint64_t b0 = v_desc + static_cast<uint64_t>(s) * kTileStep;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          mma_ts_l(leader, d_tmem, a_tmem + static_cast<uint32_t>(kk * 8),
                   b0 + static_cast<uint64_t>(kk * C::kRowBytes), idesc_pv, (accumulate || kk > 0) ? 1u : 0u);
      };
      int kp = 0, vp = 0;  // ring slot of the next K / V to consume
      uint32_t kph = 0u, vph = 0u;
      uint32_t g0 = 0u, g1 = 0u;  // key iterations done by tile 0 / tile 1 (barrier phases)
      uint32_t qn = 0u;           // items whose Q buffer has been taken (buffer qn & 1, phase qn >> 1)
      bool pre = false;           // this item's first Q K^T was issued during the previous item
      bool ok = true;
      // Q K^T of an item's key tile 0 for tile t from Q buffer qb into S_t, once the
      // tile's previous S_t (key iteration g - 1, when g > 0) has been read out
      auto first_qk = [&](int t, uint32_t qb, uint32_t g) -> bool {
        if (g > 0u && !mbar_wait_w(&bars.s_free[t], (g - 1u) & 1u, abort, p.status, limit)) return false;
        tc_fence_after();
        issue_qk(t, qb, kp);
        mma_commit_l(leader, &bars.s_full[t]);
        return true;
      };
      for (int w = blockIdx.x; ok && w < total; w += gridDim.x) {
        int hh, bb, m0, ntiles;
        coords(w, hh, bb, m0, ntiles);
        const uint32_t qb = qn & 1u;
        if (!pre) {
          if (!mbar_wait_w(&bars.q_full[qb], (qn >> 1) & 1u, abort, p.status, limit) ||
              !mbar_wait_w(&bars.k_full[kp], kph, abort, p.status, limit))
            break;
          for (int t = 0; ok && t < ntiles; ++t) ok = first_qk(t, qb, t == 0 ? g0 : g1);
          if (!ok) break;
          mma_commit_l(leader, &bars.k_empty[kp]);
          if (nkv == 1) mma_commit_l(leader, &bars.q_empty[qb]);
          if (++kp == NS) {
            kp = 0;
            kph ^= 1u;
          }
        }
        ++qn;
        // the next item of this CTA: its first Q K^T per tile is issued at the start of
        // this item's last key iteration (its Q is in the other buffer), before the last
        // P V, so its S is in TMEM when the softmax finishes this item
        const int wn = w + static_cast<int>(gridDim.x);
        int ntn = 0;
        if (wn < total) {
          int h2, b2, m2;
          coords(wn, h2, b2, m2, ntn);
        }
        pre = false;
        for (int j = 0; ok && j < nkv; ++j) {
          if (j + 1 < nkv) {
            if (!mbar_wait_w(&bars.k_full[kp], kph, abort, p.status, limit)) {
              ok = false;
              break;
            }
            for (int t = 0; t < ntiles; ++t) {
              const uint32_t g = (t == 0 ? g0 : g1) + static_cast<uint32_t>(j);
              if (!mbar_wait_w(&bars.s_free[t], g & 1u, abort, p.status, limit)) {
                ok = false;
                break;
              }
              tc_fence_after();
              issue_qk(t, qb, kp);
              mma_commit_l(leader, &bars.s_full[t]);
            }
            if (!ok) break;
            mma_commit_l(leader, &bars.k_empty[kp]);
            if (j + 2 == nkv) mma_commit_l(leader, &bars.q_empty[qb]);  // the item's last Q K^T
            if (++kp == NS) {
              kp = 0;
              kph ^= 1u;
            }
          }
          if (!mbar_wait_w(&bars.v_full[vp], vph, abort, p.status, limit)) {
            ok = false;
            break;
          }
          const bool early = j + 1 == nkv && ntn > 0;
          const uint32_t qbn = qb ^ 1u;
          if (early && (!mbar_wait_w(&bars.q_full[qbn], (qn >> 1) & 1u, abort, p.status, limit) ||
                        !mbar_wait_w(&bars.k_full[kp], kph, abort, p.status, limit))) {
            ok = false;
            break;
          }
          if (early) {
            for (int t = 0; ok && t < ntn; ++t)
              ok = first_qk(t, qbn, (t == 0 ? g0 : g1) + (t < ntiles ? static_cast<uint32_t>(nkv) : 0u));
            if (!ok) break;
            mma_commit_l(leader, &bars.k_empty[kp]);
            if (nkv == 1) mma_commit_l(leader, &bars.q_empty[qbn]);
            if (++kp == NS) {
              kp = 0;
              kph ^= 1u;
            }
            pre = true;
          }
          for (int t = 0; t < ntiles; ++t) {
            const uint32_t g = (t == 0 ? g0 : g1) + static_cast<uint32_t>(j);
            if (!mbar_wait_w(&bars.p_full[t], g & 1u, abort, p.status, limit)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(t, vp, j > 0);
            mma_commit_l(leader, &bars.o_done[t]);
          }
          if (!ok) break;
          mma_commit_l(leader, &bars.v_empty[vp]);
          if (++vp == NS) {
            vp = 0;
            vph ^= 1u;
          }
        }
        g0 += static_cast<uint32_t>(nkv);
        if (ntiles == 2) g1 += static_cast<uint32_t>(nkv);
      }
      // every UMMA issued so far must finish before TMEM is freed
      mma_commit_l(leader, &bars.drain);
      drain_wait_w(&bars.drain, 0, p.status);
    }
  } else {
    // ------------------------------------------------------ softmax + epilogue
    setmaxnreg_inc<kRegsSoftmax>();
    const int t = warp >> 2;
    const int row = threadIdx.x & (kWG - 1);
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tbase + lane_off + static_cast<uint32_t>(t * 128);
    const uint32_t tO = tbase + lane_off + kOCol0 + static_cast<uint32_t>(t) * kOStride;
    const uint32_t tP = tbase + lane_off + kPCol0 + static_cast<uint32_t>(t) * kPStride;
    // scale 0 runs as the smallest normal float: every finite score still maps to
    // 2^0 = 1 in f32, and the masked (infinite) scores of a ragged tile to 0
    const float k2 = p.scale_log2 == 0.0f ? 1.17549435e-38f : p.scale_log2;
    const bool pos = k2 >= 0.0f;
    const float init = pos ? -INFINITY : INFINITY;  // masked score: exp2(init * k2) = 0
    uint8_t* stage = sO + t * C::kTileBytes;
    uint32_t g = 0u;   // key iterations this tile has done (barrier phases)
    uint32_t tt = 0u;  // key iterations of two-tile items done (turn phases)
    uint32_t ne = 0u;  // epilogues done (epi barrier phases)
    bool ok = true;
    for (int w = blockIdx.x; ok && w < total; w += gridDim.x) {
      int hh, bb, m0, ntiles;
      coords(w, hh, bb, m0, ntiles);
      if (t >= ntiles) continue;
      float m_run = -INFINITY;
      float l = 0.0f;
      for (int j = 0; j < nkv; ++j) {
        const uint32_t gj = g + static_cast<uint32_t>(j);
        if (!mbar_wait(&bars.s_full[t], gj & 1u, abort, p.status, limit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[128];
        tmem_ld_x128(tS, sr);
        // S_t is in registers: the next Q K^T may overwrite it
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.s_free[t]);
        const int valid = S - j * kBN;  // > 0; < 128 only on the last tile
        if (valid < kBN) {
#pragma unroll
          for (int c = 0; c < kBN; ++c)
            if (c >= valid) sr[c] = __float_as_uint(init);
        }
        float m8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) m8[i] = init;
        if (pos) {
#pragma unroll
          for (int c = 0; c < kBN; c += 2)
            m8[(c >> 1) & 7] = max3(m8[(c >> 1) & 7], __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
        } else {
#pragma unroll
          for (int c = 0; c < kBN; c += 2)
            m8[(c >> 1) & 7] = min3(m8[(c >> 1) & 7], __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
        }
        float mx = pos ? max3(max3(m8[0], m8[1], m8[2]), max3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]))
                       : min3(min3(m8[0], m8[1], m8[2]), min3(m8[3], m8[4], m8[5]), fminf(m8[6], m8[7]));
        mx *= k2;
        // P V of the previous key tile must be done before O is rescaled or P_t reused
        if (j > 0) {
          if (!mbar_wait(&bars.o_done[t], (gj - 1u) & 1u, abort, p.status, limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        if (j == 0) {
          m_run = mx;
        } else {
          const bool need = mx > m_run + kRescaleLog2;
          if (__any_sync(0xffffffffu, need)) {
            const float alpha = need ? ex2(m_run - mx) : 1.0f;
            if (need) m_run = mx;
            l *= alpha;
            constexpr int kChunk = D < 32 ? D : 32;
#pragma unroll
            for (int c0 = 0; c0 < D; c0 += kChunk) {
              uint32_t orow[kChunk];
              tmem_ld<kChunk>(tO + static_cast<uint32_t>(c0), orow);
#pragma unroll
              for (int c = 0; c < kChunk; ++c) orow[c] = __float_as_uint(__uint_as_float(orow[c]) * alpha);
              tmem_st<kChunk>(tO + static_cast<uint32_t>(c0), orow);
            }
          }
        }
        // ping-pong of the exponential phases (see attn_tc_kernel); the turn
        // phases count only iterations in which both tiles are active
        if (ntiles == 2 && (t == 1 || tt > 0u)) {
          const uint32_t par = (t == 1 ? tt : tt - 1u) & 1u;
          if (!mbar_wait(&bars.turn[t], par, abort, p.status, limit)) {
            ok = false;
            break;
          }
        }
        const float neg_m = -m_run;
        float la[4] = {0.0f, 0.0f, 0.0f, 0.0f}, lb[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int c = 0; c < kBN; c += 2) {
          float x0, x1, p0, p1;
          fma2(x0, x1, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]), k2, neg_m);
          if ((kPolyPairs >> ((c >> 1) & 7)) & 1) {
            ex2_poly2(p0, p1, x0, x1);
          } else {
            p0 = ex2(x0);
            p1 = ex2(x1);
          }
          add2(la[(c >> 1) & 3], lb[(c >> 1) & 3], p0, p1);
          sr[c >> 1] = pack_half2(p0, p1);
          if (c == kTurnAt && ntiles == 2) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars.turn[1 - t]);
          }
        }
        l += ((la[0] + lb[0]) + (la[1] + lb[1])) + ((la[2] + lb[2]) + (la[3] + lb[3]));
        tmem_st_x64(tP, sr);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.p_full[t]);
        if (ntiles == 2) ++tt;
      }
      if (!ok) break;
      g += static_cast<uint32_t>(nkv);
      // epilogue: O / l -> f16 -> swizzled staging -> TMA store (not waited for)
      if (!mbar_wait(&bars.o_done[t], (g - 1u) & 1u, abort, p.status, limit)) break;
      tc_fence_after();
      if (row == 0) bulk_wait_read_all();  // the previous store has read the staging buffer
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.epi[t][0]);
      if (!mbar_wait(&bars.epi[t][0], ne & 1u, abort, p.status, limit)) break;
      // O / l as O * (1 / l): the epilogue lies between one item's last key tile and the
      // next item's first, and 64 IEEE divisions per row cost as much as an exponential
      // phase (B32 H12 S512: 443 -> 546 TFLOP/s; B8 H16 S2048: 743 -> 800)
      const float rl = __frcp_rn(l);
      constexpr int kChunk = D < 32 ? D : 32;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += kChunk) {
        uint32_t orow[kChunk];
        tmem_ld<kChunk>(tO + static_cast<uint32_t>(c0), orow);
        uint32_t h2[kChunk / 2];
#pragma unroll
        for (int c = 0; c < kChunk; c += 2)
          h2[c / 2] = pack_half2(__fmul_rn(__uint_as_float(orow[c]), rl), __fmul_rn(__uint_as_float(orow[c + 1]), rl));
#pragma unroll
        for (int q = 0; q < kChunk / 8; ++q) {
          const int col = c0 + q * 8;
          const int bx = col / C::kBoxCols;
          const uint32_t off = static_cast<uint32_t>(row * C::kRowBytes + (col % C::kBoxCols) * 2);
          const uint32_t phys = off ^ (((off >> 7) & C::kSwzMask) << 4);
          *reinterpret_cast<uint4*>(stage + bx * C::kBoxBytes + phys) =
              make_uint4(h2[q * 4], h2[q * 4 + 1], h2[q * 4 + 2], h2[q * 4 + 3]);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.epi[t][1]);
      if (!mbar_wait(&bars.epi[t][1], ne & 1u, abort, p.status, limit)) break;
      ++ne;
      if (row == 0) {
        for (int bx = 0; bx < C::kBoxes; ++bx)
          tma_store_4d_async(&to, stage + bx * C::kBoxBytes, bx * C::kBoxCols, m0 + t * kBM, hh, bb);
      }
    }
    if (row == 0) bulk_wait_all();  // every O store has completed before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kTmemCols));
  }
}

// ------------------------------------------------------------- host side ---
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encoder() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 4-D map over [batch, heads, seq, D] (dims listed innermost first), 128-row boxes.
static int make_map(CUtensorMap* m, const void* base, const int64_t* st, const fpk_attn_desc* d) {
  EncodeTiledFn enc = encoder();
  if (!enc) return FPK_ERR_CUDA;
  const int D = d->head_dim;
  if (reinterpret_cast<uintptr_t>(base) % 16) return FPK_ERR_ALIGN;
  for (int i = 0; i < 3; ++i)
    if (st[i] <= 0 || (st[i] * 2) % 16) return FPK_ERR_ALIGN;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(d->seq_len),
                              static_cast<cuuint64_t>(d->heads), static_cast<cuuint64_t>(d->batch)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(st[2] * 2), static_cast<cuuint64_t>(st[1] * 2),
                                 static_cast<cuuint64_t>(st[0] * 2)};
  const cuuint32_t box[4] = {static_cast<cuuint32_t>(D >= 64 ? 64 : D), 128u, 1u, 1u};
  const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  const CUtensorMapSwizzle swz = D >= 64 ? CU_TENSOR_MAP_SWIZZLE_128B
                                         : (D == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FPK_OK : FPK_ERR_INVALID;
}

template <int D>
static int launch_d(const CUtensorMap* maps, const Params& p, int64_t blocks, cudaStream_t s) {
  static std::atomic<int> opted[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FPK_ERR_CUDA;
  if (!opted[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(attn_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg<D>::kLaunchSmem) != cudaSuccess)
      return FPK_ERR_CUDA;
    opted[dev].store(1, std::memory_order_release);
  }
  attn_tc_kernel<D><<<static_cast<unsigned>(blocks), kThreads, Cfg<D>::kLaunchSmem, s>>>(maps[0], maps[1], maps[2],
                                                                                        maps[3], p);
  return cudaGetLastError() == cudaSuccess ? FPK_OK : FPK_ERR_CUDA;
}

// persistent kernel: two Q buffers, the K / V ring, then the O staging tiles
template <int D>
constexpr int persistent_smem() {
  constexpr int bytes = (3 * kTiles + 2 * Cfg<D>::kStages) * Cfg<D>::kTileBytes + 1024;
  return bytes > kMinSmem ? bytes : kMinSmem;
}

template <int D>
static int launch_p(const CUtensorMap* maps, const Params& p, int64_t items, int num_sms, cudaStream_t s) {
  static std::atomic<int> opted[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FPK_ERR_CUDA;
  if (!opted[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(attn_tcp_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             persistent_smem<D>()) != cudaSuccess)
      return FPK_ERR_CUDA;
    opted[dev].store(1, std::memory_order_release);
  }
  const int64_t grid = items < num_sms ? items : num_sms;  // one CTA per SM, each walks its items
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = persistent_smem<D>();
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, attn_tcp_kernel<D>, maps[0], maps[1], maps[2], maps[3], p) != cudaSuccess)
    return FPK_ERR_CUDA;
  return FPK_OK;
}

}  // namespace attn_tc

int launch_attention_tc(const fpk_attn_desc* d, const void* q, const void* k, const void* v, void* o,
                        cudaStream_t stream, const DeviceInfo& dev) {
  using namespace attn_tc;
  if (d->seq_len > 0x7fffffffLL || d->heads > 0x7fffffffLL || d->batch > 0x7fffffffLL) return FPK_ERR_UNSUPPORTED;
  CUtensorMap maps[4];
  int rc;
  if ((rc = make_map(&maps[0], q, d->q_strides, d)) != FPK_OK) return rc;
  if ((rc = make_map(&maps[1], k, d->k_strides, d)) != FPK_OK) return rc;
  if ((rc = make_map(&maps[2], v, d->v_strides, d)) != FPK_OK) return rc;
  if ((rc = make_map(&maps[3], o, d->o_strides, d)) != FPK_OK) return rc;
  Params p;
  p.status = dev.status;
  p.heads = static_cast<int32_t>(d->heads);
  p.seq = static_cast<int32_t>(d->seq_len);
  p.num_mblocks = static_cast<int32_t>((d->seq_len + kTiles * kBM - 1) / (kTiles * kBM));
  p.scale_log2 = d->scale * 1.4426950408889634f;
  p.flags = d->flags;
  const int64_t blocks = d->batch * d->heads * p.num_mblocks;
  if (blocks > 0x7fffffffLL - 1024) return FPK_ERR_UNSUPPORTED;
  p.num_items = static_cast<int32_t>(blocks);
  p.split_from = p.num_items;
  const int num_sms = dev.num_sms > 0 ? dev.num_sms : 148;
  // Persistent kernel: when the last round of 256-row blocks would leave most SMs idle
  // (at most half of them busy), its blocks run as two single-tile items each, one tile
  // per SM, so that round takes one tile's time instead of a pair's.  Only when every
  // block holds two tiles (no empty half).
  const int64_t rem = blocks % num_sms;
  const int64_t tail = d->seq_len % (kTiles * kBM);
  if (blocks > num_sms && rem > 0 && 2 * rem <= num_sms && (tail == 0 || tail > kBM)) {
    p.split_from = static_cast<int32_t>(blocks - rem);
    p.num_items = static_cast<int32_t>(blocks + rem);
  }
  switch (d->head_dim) {
    case 16: return launch_p<16>(maps, p, p.num_items, num_sms, stream);
    case 32: return launch_p<32>(maps, p, p.num_items, num_sms, stream);
    case 64: return launch_p<64>(maps, p, p.num_items, num_sms, stream);
    case 128: return launch_d<128>(maps, p, blocks, stream);
    default: return FPK_ERR_UNSUPPORTED;
  }
}

}  // namespace fpk
