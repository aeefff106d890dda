// Per-program flat chain kernels compiled at run time.
//
// The reference compiles one Triton kernel per fused chain: the plan emitter
// writes fp_chain_<N> source (lib/Plan/TritonEmitter.cpp:14-65, twin
// python/fusionpass/kernels.py:129-211) and Triton JIT-compiles it at the first
// launch.  This is the sm_100a counterpart for flat chains: the descriptor's op
// list becomes straight-line f32 CUDA (one SSA value per op), NVRTC compiles it
// for sm_100a on first use, and the cubin is loaded with cudaLibraryLoadData and
// cached by source text for the life of the process.  Rows chains (one
// last-axis softmax, up to 16384 columns) get a generated kernel of their own
// (gen_rows_source).  The interpreter kernels in chain.cu stay the path for every
// case this tier does not take (ragged column counts, longer rows, unaligned
// pointers, no run-time compiler, a stream under capture before the first
// compile, the device-wait test flag).
//
// Generated flat kernel: the flattened [rows, cols/8] grid of 8-element vectors
// (16 bytes of f16, 32 of f32) is cut into consecutive runs of 128 vectors, one
// per CTA, which makes a single pass: 128 threads with one vector each, or, for
// chains with an exponential or GELU, 64 threads that take vectors t and t + 64
// and load both before computing either (each load instruction of a warp covers
// 512 contiguous bytes).  Per-column and
// per-row operands are read per vector through the read-only cache (they stay
// in L1/L2).  Full-shape operands are read and the result written with
// streaming (evict-first) cache hints.  Arithmetic uses the same op definitions as the
// interpreter (chain_ops.cuh, embedded below) with explicit round-to-nearest
// adds and multiplies, so both tiers are bit-identical for flat chains.  The
// element loop walks pairs (e, e + 1) so that GELU runs as op_gelu2, whose erfc
// polynomial is evaluated on packed f32 pairs with per-lane results identical to
// op_gelu (bias + GELU over f16 [16384, 3072]: 48.3 -> 45.7 us with the erfcc
// form of GELU; 40.8 us with the present one).
#include <dlfcn.h>
#include <nvrtc.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "internal.h"

namespace fpk {
namespace chain_jit {

static const char kOpsSrc[] =
#include "chain_ops_src.inc"
    ;

constexpr int kVec = 8;        // elements per thread-vector

// Geometry of the generated flat kernel: 2-D tiles of 8-element vectors.  The
// data is viewed as rows of NCV vectors: the chain's own rows (NCV = cols / 8)
// when a per-column or per-row operand needs an element's position, otherwise
// virtual rows of 128 vectors over the flat index (the source then does not
// depend on the shape).  A CTA is TW vectors wide and RPC rows high; thread
// (tr, tc) owns vector column cv = blockIdx.x * TW + tc for the whole launch and
// takes RPT rows spaced RPC apart in each pass: its per-column operands are loaded
// and converted once, all its full-shape loads of a pass are issued before any is
// used, and no index is divided.  NCV is a compile-time constant of the source.
// The one-pass kernel this replaced (one or two vectors per thread over the flat
// index, a position division and the per-column loads and conversions for every
// vector) issued ~170 instructions per 16-byte vector of cfg2 and was close to
// issue-bound (68 % issue active under ncu).  Measured on B200 (CUDA graphs of 20
// launches): relu((x + b) * s) * 0.5 + x over f16 [R, 4096] 12.9-13.0 -> 11.8 /
// 7.6 -> 6.9 / 4.5 -> 4.0 / 3.0 -> 3.0 us for R = 4096 / 2048 / 1024 / 512; bias +
// GELU over [16384, 3072] 41.1 -> 37.0 us; bias + residual over [16384, 768] and
// a two-operand chain over [4096, 4096] within 1 %.  One or two rows per thread
// for a single full-shape operand, or four for two, measured slower.
struct FlatTile {
  long long ncv;  // vectors per row of the view
  int tw, rpc, rpt;
};
static FlatTile flat_tile(const fpk_chain_desc* d) {
  bool pos = false;
  int nfull = 0;
  for (int i = 0; i < d->n_inputs; ++i) {
    pos |= d->in_bcast[i] == FPK_BCAST_COL || d->in_bcast[i] == FPK_BCAST_ROW;
    nfull += d->in_bcast[i] == FPK_BCAST_FULL ? 1 : 0;
  }
  FlatTile t;
  t.ncv = pos ? d->cols / kVec : 128;
  const long long nbx = (t.ncv + 127) / 128;                // CTAs across a row
  t.tw = static_cast<int>((t.ncv + nbx - 1) / nbx);        // <= 128, as even as the row allows
  t.rpc = t.tw >= 64 ? 1 : 128 / t.tw;                     // short rows: several per CTA
  t.rpt = nfull <= 1 ? 4 : (nfull == 2 ? 2 : 1);           // full-shape vectors per thread and pass
  return t;
}

struct JitParams {
  const void* in[FPK_CHAIN_MAX_INPUTS];
  void* out;
  long long rows, cols, ncv, nvec;
};

// ----------------------------------------------------------------- NVRTC ---
struct Nvrtc {
  bool ok = false;
  decltype(&nvrtcCreateProgram) create = nullptr;
  decltype(&nvrtcCompileProgram) compile = nullptr;
  decltype(&nvrtcGetCUBINSize) cubin_size = nullptr;
  decltype(&nvrtcGetCUBIN) cubin = nullptr;
  decltype(&nvrtcGetProgramLogSize) log_size = nullptr;
  decltype(&nvrtcGetProgramLog) log = nullptr;
  decltype(&nvrtcDestroyProgram) destroy = nullptr;
};

static const Nvrtc& nvrtc() {
  static Nvrtc n;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* env = std::getenv("FPK_NVRTC_LIB");
    const char* cands[] = {env, "libnvrtc.so.12", "libnvrtc.so", "/usr/local/cuda/lib64/libnvrtc.so.12"};
    void* h = nullptr;
    for (const char* c : cands)
      if (c && *c && (h = dlopen(c, RTLD_NOW | RTLD_LOCAL)) != nullptr) break;
    if (!h) return;
    n.create = reinterpret_cast<decltype(n.create)>(dlsym(h, "nvrtcCreateProgram"));
    n.compile = reinterpret_cast<decltype(n.compile)>(dlsym(h, "nvrtcCompileProgram"));
    n.cubin_size = reinterpret_cast<decltype(n.cubin_size)>(dlsym(h, "nvrtcGetCUBINSize"));
    n.cubin = reinterpret_cast<decltype(n.cubin)>(dlsym(h, "nvrtcGetCUBIN"));
    n.log_size = reinterpret_cast<decltype(n.log_size)>(dlsym(h, "nvrtcGetProgramLogSize"));
    n.log = reinterpret_cast<decltype(n.log)>(dlsym(h, "nvrtcGetProgramLog"));
    n.destroy = reinterpret_cast<decltype(n.destroy)>(dlsym(h, "nvrtcDestroyProgram"));
    n.ok = n.create && n.compile && n.cubin_size && n.cubin && n.log_size && n.log && n.destroy;
  });
  return n;
}

// ------------------------------------------------------- source generator ---
// Which generated kernel (if any) takes `d`: eligibility that depends on the
// descriptor alone (pointer alignment is checked at launch).
enum JitKind { kNone = 0, kFlat = 1, kRows = 2 };
constexpr int kRowsMaxCols = 16384;

static JitKind jit_kind(const fpk_chain_desc* d) {
  if (d->cols <= 0 || d->rows <= 0 || d->cols % kVec) return kNone;
  if (d->flags & (FPK_FLAG_TEST_TIMEOUT | FPK_FLAG_NO_STAGING | FPK_FLAG_NO_JIT)) return kNone;
  int softmax = 0;
  for (int k = 0; k < d->n_ops; ++k) {
    const int op = d->ops[k].opcode;
    if (op == FPK_OP_SOFTMAX) {
      ++softmax;
      continue;
    }
    if (op != FPK_OP_ADD && op != FPK_OP_MUL && op != FPK_OP_SCALE && op != FPK_OP_RELU && op != FPK_OP_EXP &&
        op != FPK_OP_GELU)
      return kNone;
  }
  if (d->mode == FPK_CHAIN_FLAT) return softmax == 0 ? kFlat : kNone;
  if (d->mode == FPK_CHAIN_ROWS && softmax == 1 && d->cols <= kRowsMaxCols) return kRows;
  return kNone;
}

// Rows kernel geometry, fixed by the column count: TPR threads share a row, each
// holding VPT 8-element vectors (vector v of the row at thread v % TPR, slot v / TPR).
// Four vectors (64 bytes of f16) per thread up to 8192 columns, eight at 16384,
// at most 256 threads per row, 256-thread CTAs: the fastest of the shapes
// measured on B200 for f16 softmax rows of 128 to 16384 columns (12.7-15.8 us
// for 67 MB against 16.1-18.0 us before; one vector per thread for short rows
// left too few bytes in flight; 512-thread rows ran two CTAs per SM in ragged
// waves; eight or sixteen vectors per thread lowered occupancy).
struct RowsGeom {
  int nv, tpr, vpt, block, rows_per_cta;
};
static RowsGeom rows_geom(long long cols) {
  RowsGeom g;
  g.nv = static_cast<int>(cols / kVec);
  auto pow2 = [](int n) { int p = 1; while (p < n) p <<= 1; return p; };
  g.tpr = std::min(256, pow2((g.nv + 3) / 4));
  g.vpt = (g.nv + g.tpr - 1) / g.tpr;
  g.block = 256;
  g.rows_per_cta = g.block / g.tpr;
  return g;
}

static void app(std::string& s, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
// Appends printf-formatted text of any length.
static void app(std::string& s, const char* fmt, ...) {
  char buf[512];
  va_list ap, ap2;
  va_start(ap, fmt);
  va_copy(ap2, ap);
  const int n = vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (n > 0 && n < static_cast<int>(sizeof(buf))) {
    s.append(buf, static_cast<size_t>(n));
  } else if (n > 0) {
    std::string big(static_cast<size_t>(n) + 1, '\0');
    vsnprintf(&big[0], big.size(), fmt, ap2);
    s.append(big.data(), static_cast<size_t>(n));
  }
  va_end(ap2);
}

// First statement of every generated kernel.  The kernels are launched with
// programmatic stream serialization, so a launch can be scheduled while the
// previous kernel of the stream is finishing; no thread reads or writes global
// memory before that kernel has completed and its writes are visible.  The
// trigger for the next launch is the implicit one at exit (an earlier explicit
// trigger let waiting CTAs of the next launch hold residency slots: 12.6 ->
// 17.4 us per cfg2 chain).  Measured: cfg2 f16 [4096, 4096] 12.67 -> 12.61 us
// per launch; the 512-row shard of eight GPUs 3.40 -> 3.17 us.
static const char kWaitPrevGrid[] = "  asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n";

// Types, the shared op definitions and the load / store helpers of every generated kernel.
static void prelude(std::string& s) {
  s.reserve(16384);
  s += "typedef unsigned int u32;\ntypedef unsigned short u16;\ntypedef long long i64;\n";
  s += kOpsSrc;
  s += R"SRC(
struct JitParams { const void* in[8]; void* out; i64 rows, cols, ncv, nvec; };
__device__ __forceinline__ float h2f(u16 h) { float f; asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h)); return f; }
// f32 pair -> f16x2 in one instruction (lo in the low half), round to nearest even
__device__ __forceinline__ u32 f2h2(float lo, float hi) { u32 r; asm("cvt.rn.f16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(lo), "f"(hi)); return r; }
__device__ __forceinline__ void unpack8(uint4 u, float* a) {
  a[0] = h2f((u16)(u.x & 0xffffu)); a[1] = h2f((u16)(u.x >> 16));
  a[2] = h2f((u16)(u.y & 0xffffu)); a[3] = h2f((u16)(u.y >> 16));
  a[4] = h2f((u16)(u.z & 0xffffu)); a[5] = h2f((u16)(u.z >> 16));
  a[6] = h2f((u16)(u.w & 0xffffu)); a[7] = h2f((u16)(u.w >> 16));
}
// 2^x on the MUFU, subnormal results kept (rows softmax)
__device__ __forceinline__ float ex2f_approx(float x) { float y; asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x)); return y; }
// full-shape operands: streaming loads (read once, evict first)
__device__ __forceinline__ void ld8s_f16(const void* b, i64 off, float* a) {
  unpack8(__ldcs(reinterpret_cast<const uint4*>(reinterpret_cast<const u16*>(b) + off)), a);
}
__device__ __forceinline__ void ld8s_f32(const void* b, i64 off, float* a) {
  const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(b) + off);
  const float4 x = __ldcs(p), y = __ldcs(p + 1);
  a[0] = x.x; a[1] = x.y; a[2] = x.z; a[3] = x.w; a[4] = y.x; a[5] = y.y; a[6] = y.z; a[7] = y.w;
}
// broadcast operands: read-only cache (reused by every row)
__device__ __forceinline__ void ld8c_f16(const void* b, i64 off, float* a) {
  unpack8(__ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const u16*>(b) + off)), a);
}
__device__ __forceinline__ void ld8c_f32(const void* b, i64 off, float* a) {
  const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(b) + off);
  const float4 x = __ldg(p), y = __ldg(p + 1);
  a[0] = x.x; a[1] = x.y; a[2] = x.z; a[3] = x.w; a[4] = y.x; a[5] = y.y; a[6] = y.z; a[7] = y.w;
}
// per-column f16 operand: the raw 16 bytes, unpacked only once the full-shape loads are in flight
__device__ __forceinline__ uint4 ldu8c_f16(const void* b, i64 off) {
  return __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const u16*>(b) + off));
}
__device__ __forceinline__ float ld1_f16(const void* b, i64 i) { return h2f(__ldg(reinterpret_cast<const u16*>(b) + i)); }
__device__ __forceinline__ float ld1_f32(const void* b, i64 i) { return __ldg(reinterpret_cast<const float*>(b) + i); }
__device__ __forceinline__ void st8_f16(void* b, i64 off, const float* y) {
  uint4 u;
  u.x = f2h2(y[0], y[1]); u.y = f2h2(y[2], y[3]); u.z = f2h2(y[4], y[5]); u.w = f2h2(y[6], y[7]);
  __stcs(reinterpret_cast<uint4*>(reinterpret_cast<u16*>(b) + off), u);
}
__device__ __forceinline__ void st8_f32(void* b, i64 off, const float* y) {
  float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(b) + off);
  __stcs(p, make_float4(y[0], y[1], y[2], y[3]));
  __stcs(p + 1, make_float4(y[4], y[5], y[6], y[7]));
}
)SRC";
}

// The element program of the thread's k-th vector of a pass (row r0 + k * RPC,
// flat vector w<k>): full-shape values in a<i>_<k>[8], per-column values in
// c<i>[8] (loaded once per thread), per-row values in r<i>_<k>, scalars in s<i>;
// the ops run on element pairs and the result is stored.
static void gen_vector_body(std::string& s, const fpk_chain_desc* d, int k, const char* ind) {
  const int nin = d->n_inputs;
  app(s, "%sfloat y[8];\n%s#pragma unroll\n%sfor (int e = 0; e < 8; e += 2) {\n", ind, ind, ind);
  for (int h = 0; h < 2; ++h) {
    const char* ee = h == 0 ? "e" : "e + 1";
    for (int i = 0; i < nin; ++i) {
      switch (d->in_bcast[i]) {
        case FPK_BCAST_FULL: app(s, "%s  const float v%d_%d = a%d_%d[%s];\n", ind, i, h, i, k, ee); break;
        case FPK_BCAST_COL: app(s, "%s  const float v%d_%d = c%d[%s];\n", ind, i, h, i, ee); break;
        case FPK_BCAST_ROW: app(s, "%s  const float v%d_%d = r%d_%d;\n", ind, i, h, i, k); break;
        default: app(s, "%s  const float v%d_%d = s%d;\n", ind, i, h, i); break;
      }
    }
  }
  for (int q = 0; q < d->n_ops; ++q) {
    const fpk_chain_op& op = d->ops[q];
    const int dst = nin + q;
    if (op.opcode == FPK_OP_GELU) {
      app(s, "%s  float v%d_0, v%d_1;\n%s  op_gelu2(v%d_0, v%d_1, v%d_0, v%d_1);\n", ind, dst, dst, ind, op.src_a, op.src_a, dst, dst);
      continue;
    }
    for (int h = 0; h < 2; ++h) {
      switch (op.opcode) {
        case FPK_OP_ADD: app(s, "%s  const float v%d_%d = __fadd_rn(v%d_%d, v%d_%d);\n", ind, dst, h, op.src_a, h, op.src_b, h); break;
        case FPK_OP_MUL: app(s, "%s  const float v%d_%d = __fmul_rn(v%d_%d, v%d_%d);\n", ind, dst, h, op.src_a, h, op.src_b, h); break;
        case FPK_OP_SCALE: {
          uint32_t bits;
          std::memcpy(&bits, &op.imm, 4);
          app(s, "%s  const float v%d_%d = __fmul_rn(v%d_%d, __uint_as_float(0x%08xu));\n", ind, dst, h, op.src_a, h, bits);
          break;
        }
        case FPK_OP_RELU: app(s, "%s  const float v%d_%d = op_relu(v%d_%d);\n", ind, dst, h, op.src_a, h); break;
        default: app(s, "%s  const float v%d_%d = expf(v%d_%d);\n", ind, dst, h, op.src_a, h); break;
      }
    }
  }
  app(s, "%s  y[e] = v%d_0;\n%s  y[e + 1] = v%d_1;\n%s}\n", ind, d->result, ind, d->result, ind);
  app(s, "%sst8_%s(p.out, w%d * 8, y);\n", ind, d->out_dtype == FPK_F16 ? "f16" : "f32", k);
}

// Flat chains: the 2-D tiles of flat_tile.  Each pass of a CTA covers RPC * RPT
// rows of its TW-vector column block; CTAs step over the passes by gridDim.y.
static std::string gen_flat_source(const fpk_chain_desc* d) {
  const int nin = d->n_inputs;
  const FlatTile ft = flat_tile(d);
  std::string s;
  prelude(s);
  const char* dt[2] = {"f32", "f16"};
  auto idt = [&](int i) { return dt[d->in_dtype[i] == FPK_F16 ? 1 : 0]; };
  app(s, "#define NCV %lldll\n#define TW %d\n#define RPC %d\n#define RPT %d\n", ft.ncv, ft.tw, ft.rpc, ft.rpt);
  app(s, "extern \"C\" __global__ void __launch_bounds__(%d) fpk_jit_chain(const JitParams p) {\n", ft.tw * ft.rpc);
  s += kWaitPrevGrid;
  s += "  const int tc = threadIdx.x % TW, tr = threadIdx.x / TW;\n";
  s += "  const i64 cv = (i64)blockIdx.x * TW + tc;\n";
  s += "  if (NCV % TW != 0 && cv >= NCV) return;\n";
  // per-column operands are read once per thread; f16 ones stay packed until the
  // pass's full-shape loads have been issued, so their latency overlaps
  for (int i = 0; i < nin; ++i) {
    if (d->in_bcast[i] == FPK_BCAST_SCALAR) app(s, "  const float s%d = ld1_%s(p.in[%d], 0);\n", i, idt(i), i);
    if (d->in_bcast[i] != FPK_BCAST_COL) continue;
    if (d->in_dtype[i] == FPK_F16) app(s, "  const uint4 cu%d = ldu8c_f16(p.in[%d], cv * 8);\n", i, i);
    else app(s, "  float c%d[8]; ld8c_f32(p.in[%d], cv * 8, c%d);\n", i, i, i);
  }
  s += "  const i64 passes = (p.rows + RPC * RPT - 1) / (RPC * RPT);\n";
  s += "  for (i64 pass = blockIdx.y; pass < passes; pass += gridDim.y) {\n";
  s += "    const i64 r0 = pass * (RPC * RPT) + tr;\n";
  for (int k = 0; k < ft.rpt; ++k) app(s, "    const i64 w%d = (r0 + %d * RPC) * NCV + cv;\n", k, k);
  for (int i = 0; i < nin; ++i) {
    if (d->in_bcast[i] == FPK_BCAST_FULL) {
      for (int k = 0; k < ft.rpt; ++k)
        app(s, "    float a%d_%d[8];\n    if (w%d < p.nvec) ld8s_%s(p.in[%d], w%d * 8, a%d_%d);\n", i, k, k, idt(i), i, k, i, k);
    } else if (d->in_bcast[i] == FPK_BCAST_ROW) {
      for (int k = 0; k < ft.rpt; ++k)
        app(s, "    const float r%d_%d = w%d < p.nvec ? ld1_%s(p.in[%d], r0 + %d * RPC) : 0.0f;\n", i, k, k, idt(i), i, k);
    }
  }
  for (int i = 0; i < nin; ++i)
    if (d->in_bcast[i] == FPK_BCAST_COL && d->in_dtype[i] == FPK_F16) app(s, "    float c%d[8]; unpack8(cu%d, c%d);\n", i, i, i);
  for (int k = 0; k < ft.rpt; ++k) {
    app(s, "    if (w%d < p.nvec) {\n", k);
    gen_vector_body(s, d, k, "      ");
    s += "    }\n";
  }
  s += "  }\n}\n";
  return s;
}

// Rows mode: one last-axis softmax.  The column count is a compile-time
// constant, so a row's values stay in registers: TPR threads share a row, each
// loads its VPT vectors, evaluates the ops before the softmax, reduces the row
// max and sum (shuffles within a warp, shared memory across the warps of a row),
// then evaluates the ops after it and stores.  Softmax: e = 2^((x - max) * log2 e)
// on the MUFU (ex2.approx, relative error ~5e-7 for every e that is not
// negligible against the row sum; 0 for masked columns), sum by round-to-nearest
// adds, p = e * (1 / sum) with a correctly rounded reciprocal.  An accurate expf
// and an IEEE division per element made this kernel instruction-bound (~40
// instructions per element); these are ~5 and it is bandwidth-bound.  Results
// agree with the interpreter (expf, e / sum) within 2e-5 relative for f32.
static std::string gen_rows_source(const fpk_chain_desc* d) {
  const int nin = d->n_inputs;
  const RowsGeom g = rows_geom(d->cols);
  const int E = g.vpt * kVec;  // elements per thread
  const int wpr = g.tpr > 32 ? g.tpr / 32 : 1;  // warps per row
  std::string s;
  prelude(s);
  const char* dt[2] = {"f32", "f16"};
  auto idt = [&](int i) { return dt[d->in_dtype[i] == FPK_F16 ? 1 : 0]; };
  int ksm = -1;
  for (int k = 0; k < d->n_ops; ++k)
    if (d->ops[k].opcode == FPK_OP_SOFTMAX) ksm = k;

  app(s, "#define TPR %d\n#define VPT %d\n#define NV %d\n#define E %d\n#define WPR %d\n#define RPC %d\n", g.tpr, g.vpt,
      g.nv, E, wpr, g.rows_per_cta);
  s += "#define INFINITY __int_as_float(0x7f800000)\n";
  app(s, "extern \"C\" __global__ void __launch_bounds__(%d) fpk_jit_chain(const JitParams p) {\n", g.block);
  s += kWaitPrevGrid;
  s += "  const int t = threadIdx.x % TPR, rl = threadIdx.x / TPR;\n";
  s += "  const i64 row = (i64)blockIdx.x * RPC + rl;\n";
  s += "  const bool live = row < p.rows;  // every thread takes part in the reductions\n";
  s += "  const i64 base = (live ? row : 0) * p.cols;\n";
  if (wpr > 1) s += "  __shared__ float red[2][RPC][WPR];\n";
  // input values
  for (int i = 0; i < nin; ++i) {
    const int b = d->in_bcast[i];
    if (b == FPK_BCAST_FULL || b == FPK_BCAST_COL) {
      app(s, "  float v%d[E];\n", i);
      app(s, "  #pragma unroll\n  for (int k = 0; k < VPT; ++k) {\n    const int vv = k * TPR + t;\n");
      if (b == FPK_BCAST_FULL)
        app(s, "    if (live && vv < NV) ld8s_%s(p.in[%d], base + vv * 8, v%d + k * 8);\n", idt(i), i, i);
      else
        app(s, "    if (vv < NV) ld8c_%s(p.in[%d], vv * 8, v%d + k * 8);\n", idt(i), i, i);
      app(s, "    else { for (int e = 0; e < 8; ++e) v%d[k * 8 + e] = 0.0f; }\n  }\n", i);
    } else if (b == FPK_BCAST_ROW) {
      app(s, "  const float r%d = live ? ld1_%s(p.in[%d], row) : 0.0f;\n  float v%d[E];\n", i, idt(i), i, i);
      app(s, "  #pragma unroll\n  for (int e = 0; e < E; ++e) v%d[e] = r%d;\n", i, i);
    } else {
      app(s, "  const float s%d = ld1_%s(p.in[%d], 0);\n  float v%d[E];\n", i, idt(i), i, i);
      app(s, "  #pragma unroll\n  for (int e = 0; e < E; ++e) v%d[e] = s%d;\n", i, i);
    }
  }
  auto emit_op = [&](int k) {
    const fpk_chain_op& op = d->ops[k];
    const int dst = nin + k;
    app(s, "  float v%d[E];\n  #pragma unroll\n  for (int e = 0; e < E; ++e) ", dst);
    switch (op.opcode) {
      case FPK_OP_ADD: app(s, "v%d[e] = __fadd_rn(v%d[e], v%d[e]);\n", dst, op.src_a, op.src_b); break;
      case FPK_OP_MUL: app(s, "v%d[e] = __fmul_rn(v%d[e], v%d[e]);\n", dst, op.src_a, op.src_b); break;
      case FPK_OP_SCALE: {
        uint32_t bits;
        std::memcpy(&bits, &op.imm, 4);
        app(s, "v%d[e] = __fmul_rn(v%d[e], __uint_as_float(0x%08xu));\n", dst, op.src_a, bits);
        break;
      }
      case FPK_OP_RELU: app(s, "v%d[e] = op_relu(v%d[e]);\n", dst, op.src_a); break;
      case FPK_OP_EXP: app(s, "v%d[e] = expf(v%d[e]);\n", dst, op.src_a); break;
      default: app(s, "v%d[e] = op_gelu(v%d[e]);\n", dst, op.src_a); break;
    }
  };
  for (int k = 0; k < ksm; ++k) emit_op(k);
  // the softmax
  const int src = d->ops[ksm].src_a, dst = nin + ksm;
  // slots past the row end exist only when VPT * TPR > NV (ragged rows)
  const bool pad = g.vpt * g.tpr > g.nv;
  const char* xval = pad ? "((((e >> 3) * TPR + t) < NV) ? v%d[e] : -INFINITY)" : "v%d[e]";
  char xexpr[128];
  std::snprintf(xexpr, sizeof(xexpr), xval, src);
  // row max in four independent chains
  app(s, "  float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};\n  #pragma unroll\n"
         "  for (int e = 0; e < E; ++e) mq[e & 3] = fmaxf(mq[e & 3], %s);\n"
         "  float m = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));\n", xexpr);
  app(s, "  #pragma unroll\n  for (int off = (TPR < 32 ? TPR : 32) / 2; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));\n");
  if (wpr > 1) {
    s += "  if ((threadIdx.x & 31) == 0) red[0][rl][t >> 5] = m;\n  __syncthreads();\n";
    s += "  m = red[0][rl][0];\n  #pragma unroll\n  for (int w = 1; w < WPR; ++w) m = fmaxf(m, red[0][rl][w]);\n";
  }
  // e = 2^((x - m) log2 e): a -inf score (or a slot past the row end) gives 0 for any finite m
  app(s, "  float ev[E];\n  float sq[4] = {0.0f, 0.0f, 0.0f, 0.0f};\n  #pragma unroll\n  for (int e = 0; e < E; ++e) {\n"
         "    ev[e] = ex2f_approx(__fmul_rn(__fsub_rn(%s, m), 1.44269504088896341f));\n"
         "    sq[e & 3] = __fadd_rn(sq[e & 3], ev[e]);\n  }\n"
         "  float sum = __fadd_rn(__fadd_rn(sq[0], sq[1]), __fadd_rn(sq[2], sq[3]));\n", xexpr);
  app(s, "  #pragma unroll\n  for (int off = (TPR < 32 ? TPR : 32) / 2; off > 0; off >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, off));\n");
  if (wpr > 1) {
    s += "  if ((threadIdx.x & 31) == 0) red[1][rl][t >> 5] = sum;\n  __syncthreads();\n";
    s += "  sum = red[1][rl][0];\n  #pragma unroll\n  for (int w = 1; w < WPR; ++w) sum = __fadd_rn(sum, red[1][rl][w]);\n";
  }
  // 0 * (1 / 0) is NaN like 0 / 0 for a row whose every value is masked
  app(s, "  const float rsum = __frcp_rn(sum);\n  float v%d[E];\n  #pragma unroll\n  for (int e = 0; e < E; ++e) v%d[e] = __fmul_rn(ev[e], rsum);\n", dst, dst);
  for (int k = ksm + 1; k < d->n_ops; ++k) emit_op(k);
  app(s, "  if (live) {\n  #pragma unroll\n  for (int k = 0; k < VPT; ++k) {\n    const int vv = k * TPR + t;\n"
         "    if (vv < NV) st8_%s(p.out, base + vv * 8, v%d + k * 8);\n  }\n  }\n}\n",
      d->out_dtype == FPK_F16 ? "f16" : "f32", d->result);
  return s;
}

static std::string gen_source(const fpk_chain_desc* d, JitKind kind) {
  return kind == kRows ? gen_rows_source(d) : gen_flat_source(d);
}

// ------------------------------------------------------------------ cache ---
struct Entry {
  std::vector<char> cubin;
  cudaLibrary_t lib = nullptr;
  cudaKernel_t kern = nullptr;
  bool failed = false;     // NVRTC could not compile the source: permanent for the process
  int load_failures = 0;   // module loads that failed (retried on later calls, up to a limit)
};
// A module load may fail for a passing reason (another thread capturing in global
// mode, a moment without free device memory); the chain then runs on the
// interpreter and a later call tries again, at most this many times in all.
constexpr int kMaxLoadFailures = 3;

static std::mutex g_mu;
static std::atomic<long long> g_launches{0};
static std::unordered_map<std::string, Entry>& cache() {
  static auto* m = new std::unordered_map<std::string, Entry>();  // lives for the process
  return *m;
}

// NVRTC compile of `src` into e.cubin (caller holds g_mu).
static bool compile_locked(const std::string& src, Entry& e) {
  const Nvrtc& n = nvrtc();
  if (!n.ok) return false;
  nvrtcProgram prog = nullptr;
  if (n.create(&prog, src.c_str(), "fpk_jit_chain.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS) return false;
  // same floating-point contract as the nvcc build of the interpreter
  const char* opts[] = {"--gpu-architecture=sm_100a", "-std=c++17", "--fmad=true", "--ftz=false",
                        "--prec-div=true", "--prec-sqrt=true", "-default-device"};
  const nvrtcResult rc = n.compile(prog, static_cast<int>(sizeof(opts) / sizeof(opts[0])), opts);
  bool ok = rc == NVRTC_SUCCESS;
  if (ok) {
    size_t sz = 0;
    ok = n.cubin_size(prog, &sz) == NVRTC_SUCCESS && sz > 0;
    if (ok) {
      e.cubin.resize(sz);
      ok = n.cubin(prog, e.cubin.data()) == NVRTC_SUCCESS;
    }
  } else if (std::getenv("FPK_JIT_VERBOSE")) {
    size_t ls = 0;
    if (n.log_size(prog, &ls) == NVRTC_SUCCESS && ls > 1) {
      std::string log(ls, '\0');
      n.log(prog, &log[0]);
      std::fprintf(stderr, "[fpkern] chain JIT compile failed:\n%s\n", log.c_str());
    }
  }
  n.destroy(&prog);
  return ok;
}

}  // namespace chain_jit

int chain_jit_precompile(const fpk_chain_desc* d) {
  using namespace chain_jit;
  const JitKind kind = jit_kind(d);
  if (kind == kNone) return FPK_ERR_UNSUPPORTED;
  const std::string src = gen_source(d, kind);
  std::lock_guard<std::mutex> lk(g_mu);
  Entry& e = cache()[src];
  if (e.failed) return FPK_ERR_UNSUPPORTED;
  if (!e.cubin.empty()) return FPK_OK;
  if (!compile_locked(src, e)) {
    e.failed = true;
    return FPK_ERR_UNSUPPORTED;
  }
  return FPK_OK;
}

int try_launch_chain_jit(const fpk_chain_desc* d, const void* const* inputs, void* out, cudaStream_t stream,
                         const DeviceInfo& dev) {
  using namespace chain_jit;
  const JitKind kind = jit_kind(d);
  if (kind == kNone) return FPK_ERR_UNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(out) % 16) return FPK_ERR_UNSUPPORTED;
  for (int i = 0; i < d->n_inputs; ++i) {
    const int b = d->in_bcast[i];
    if ((b == FPK_BCAST_FULL || b == FPK_BCAST_COL) && reinterpret_cast<uintptr_t>(inputs[i]) % 16)
      return FPK_ERR_UNSUPPORTED;
  }
  const std::string src = gen_source(d, kind);
  cudaKernel_t kern = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    Entry& e = cache()[src];
    if (e.failed) return FPK_ERR_UNSUPPORTED;
    if (!e.kern) {
      // compiling or loading modules is not a stream operation, but keep it out of
      // a capture: the interpreter serves this call and the next one compiles
      cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
      if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone)
        return FPK_ERR_UNSUPPORTED;
      if (e.cubin.empty() && !compile_locked(src, e)) {
        e.failed = true;
        return FPK_ERR_UNSUPPORTED;
      }
      if (e.load_failures >= kMaxLoadFailures) return FPK_ERR_UNSUPPORTED;
      // an error the caller left pending is not ours to clear
      const bool clean_before = cudaPeekAtLastError() == cudaSuccess;
      bool loaded = e.lib != nullptr ||
                    cudaLibraryLoadData(&e.lib, e.cubin.data(), nullptr, nullptr, 0, nullptr, nullptr, 0) == cudaSuccess;
      if (!loaded) e.lib = nullptr;
      if (loaded && cudaLibraryGetKernel(&e.kern, e.lib, "fpk_jit_chain") != cudaSuccess) {
        e.kern = nullptr;
        loaded = false;
      }
      if (!loaded) {
        if (clean_before) cudaGetLastError();  // clear only the error this load raised
        ++e.load_failures;
        return FPK_ERR_UNSUPPORTED;
      }
    }
    kern = e.kern;
  }
  JitParams p;
  std::memset(&p, 0, sizeof(p));
  for (int i = 0; i < d->n_inputs; ++i) p.in[i] = inputs[i];
  p.out = out;
  p.rows = d->rows;
  p.cols = d->cols;
  p.ncv = d->cols / kVec;
  p.nvec = d->rows * p.ncv;
  long long grid, grid_x = 1;
  int block;
  if (kind == kRows) {
    const RowsGeom g = rows_geom(d->cols);
    grid = (d->rows + g.rows_per_cta - 1) / g.rows_per_cta;  // one row per TPR-thread group
    block = g.block;
    if (grid > 0x7fffffffLL) return FPK_ERR_UNSUPPORTED;
  } else {
    const FlatTile ft = flat_tile(d);
    p.rows = (p.nvec + ft.ncv - 1) / ft.ncv;  // rows of the tile view (virtual rows cover the flat index)
    const long long per_pass = static_cast<long long>(ft.rpc) * ft.rpt;
    const long long passes = (p.rows + per_pass - 1) / per_pass;
    grid_x = (ft.ncv + ft.tw - 1) / ft.tw;
    grid = passes < 65535 ? passes : 65535;  // CTAs loop over the rest
    if (grid_x > 0x7fffffffLL) return FPK_ERR_UNSUPPORTED;
    block = ft.tw * ft.rpc;
  }
  void* args[] = {&p};
  {
    // programmatic dependent launch: the kernel may be scheduled while the previous
    // kernel of the stream drains; its griddepcontrol.wait holds every thread until
    // that kernel has completed and its writes are visible
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = kind == kRows ? dim3(static_cast<unsigned>(grid))
                                : dim3(static_cast<unsigned>(grid_x), static_cast<unsigned>(grid));
    cfg.blockDim = dim3(block);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(kern), args) != cudaSuccess) return FPK_ERR_CUDA;
  }
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return FPK_OK;
}

long long chain_jit_launches() { return chain_jit::g_launches.load(std::memory_order_relaxed); }

}  // namespace fpk
