/*
 * fpkern.h - C ABI of libfpkern.so, the sm_100a (B200) kernels for the two
 * fused-step families of the fusionpass plan runtime.
 *
 * Every entry point takes plain pointers, sizes and POD descriptors, never
 * allocates or frees device memory for tensors, never synchronises the stream
 * it is given, keeps no per-call state, and returns FPK_OK (0) or a negative
 * FPK_ERR_* status.  It never aborts or traps.  Device buffers are owned by the
 * caller.  One exception to "no device-side setup": the first fpk_chain_fwd of
 * a new chain program (op list, operand types, broadcast modes) compiles its
 * kernel with NVRTC and loads it as a module (cudaLibraryLoadData), which may
 * synchronise the device; the module is cached for the process.  Call
 * fpk_chain_precompile and make one warm-up launch to keep this out of timed
 * regions and stream captures (under capture the prebuilt kernels run instead).
 *
 * Reference interfaces replaced (paths within the reference project):
 *   fpk_attention_fwd  <- kernels.launch_attention + the fp_attention Triton
 *                         kernel (python/fusionpass/kernels.py:303-333,58-89;
 *                         lib/Plan/TritonEmitter.cpp:73-104)
 *   fpk_chain_fwd      <- kernels.launch_flat / launch_rows + the generated
 *                         fp_chain_<N> kernels (python/fusionpass/kernels.py:
 *                         288-300,129-211; lib/Plan/TritonEmitter.cpp:14-65)
 *   the descriptors    <- the per-step launch attributes the plan emitter
 *                         writes (lib/Plan/PlanEmitter.cpp:120-149) plus the
 *                         fused-op body that the reference only writes as
 *                         Triton source
 *   status codes       <- the ValueError/RuntimeError raised by
 *                         kernels.launch_step (python/fusionpass/kernels.py:336-368)
 */
#ifndef FPKERN_H
#define FPKERN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FPK_ABI_VERSION 1

/* ---- status codes -------------------------------------------------------- */
#define FPK_OK               0
#define FPK_ERR_INVALID     -1  /* malformed descriptor or argument            */
#define FPK_ERR_UNSUPPORTED -2  /* well-formed but outside what is implemented */
#define FPK_ERR_ALIGN       -3  /* pointer or stride alignment not met         */
#define FPK_ERR_CUDA        -4  /* CUDA runtime/driver error at launch         */
#define FPK_ERR_DEVICE      -5  /* current device is not an sm_100 GPU         */
#define FPK_ERR_TIMEOUT     -6  /* a bounded device-side wait ran out          */

/* ---- element types ------------------------------------------------------- */
#define FPK_F32 0
#define FPK_F16 1

/* ---- flags (both descriptors) -------------------------------------------- */
/* Test hook: the kernel withholds one producer signal so that a bounded wait
 * runs out after about 5 ms; the launch still returns FPK_OK and
 * fpk_poll_status() then reports FPK_ERR_TIMEOUT.  Nothing faults or hangs. */
#define FPK_FLAG_TEST_TIMEOUT 0x1u
/* Chain only: read every operand with plain loads (no TMA bulk staging). */
#define FPK_FLAG_NO_STAGING   0x2u
/* Chains: skip the per-program kernel compiled at run time and run the prebuilt
 * interpreter kernels (flat chains: identical bits; rows: the same arithmetic
 * with another summation order; tests compare them). */
#define FPK_FLAG_NO_JIT       0x4u

/* ---- attention: O = softmax(scale * Q K^T) V, per (batch, head) ---------- */
/* Tensors are [batch, heads, seq_len, head_dim] with element strides given for
 * the first three dims; the head_dim stride is 1.  f16 runs on the tcgen05
 * tensor cores (f32 accumulate, f32 softmax); f32 stays on FP32 FMA. */
typedef struct fpk_attn_desc {
  uint32_t size;      /* sizeof(fpk_attn_desc)                                 */
  uint32_t version;   /* FPK_ABI_VERSION                                       */
  int32_t  dtype;     /* FPK_F16 or FPK_F32, shared by q, k, v and o           */
  int32_t  head_dim;  /* D: 16, 32, 64 or 128                                  */
  int64_t  batch;     /* B (leading dims before heads, flattened)              */
  int64_t  heads;     /* H                                                      */
  int64_t  seq_len;   /* S >= 1 (self-attention: q, k, v share it)             */
  float    scale;     /* multiplies Q K^T before the softmax                    */
  uint32_t flags;
  int64_t  q_strides[3], k_strides[3], v_strides[3], o_strides[3]; /* b, h, s */
} fpk_attn_desc;

/* ---- fused elementwise chain --------------------------------------------- */
#define FPK_CHAIN_MAX_INPUTS 8
#define FPK_CHAIN_MAX_OPS    32
#define FPK_CHAIN_MAX_ROW_COLS 16384 /* rows mode: the whole row is held on chip */

/* opcodes: f32 math on the operands, one rounding at the final store */
#define FPK_OP_ADD     1  /* a + b                                      */
#define FPK_OP_MUL     2  /* a * b                                      */
#define FPK_OP_SCALE   3  /* a * imm                                    */
#define FPK_OP_RELU    4  /* max(a, 0), NaN propagates                  */
#define FPK_OP_EXP     5  /* exp(a)                                     */
#define FPK_OP_SOFTMAX 6  /* stable softmax of a over the last axis (rows mode) */
#define FPK_OP_GELU    7  /* 0.5 * a * (1 + erf(a / sqrt(2)))           */

/* how an input maps onto the [rows, cols] output */
#define FPK_BCAST_FULL   0  /* same shape as the output, contiguous     */
#define FPK_BCAST_COL    1  /* vector of length cols (per last-dim)     */
#define FPK_BCAST_ROW    2  /* vector of length rows (one per row)      */
#define FPK_BCAST_SCALAR 3  /* single element                           */

#define FPK_CHAIN_FLAT 0   /* no softmax                                  */
#define FPK_CHAIN_ROWS 1   /* exactly one last-axis softmax              */

typedef struct fpk_chain_op {
  int32_t opcode;  /* FPK_OP_*                                              */
  int32_t src_a;   /* slot: 0..n_inputs-1 are inputs, n_inputs+k is op k    */
  int32_t src_b;   /* second slot for ADD / MUL, else -1                    */
  float   imm;     /* SCALE factor                                          */
} fpk_chain_op;

typedef struct fpk_chain_desc {
  uint32_t size;      /* sizeof(fpk_chain_desc)                   */
  uint32_t version;   /* FPK_ABI_VERSION                          */
  int32_t  mode;      /* FPK_CHAIN_FLAT or FPK_CHAIN_ROWS         */
  int32_t  out_dtype; /* FPK_F16 or FPK_F32                       */
  int64_t  rows;      /* output is [rows, cols], contiguous       */
  int64_t  cols;
  int32_t  n_inputs;  /* 1..FPK_CHAIN_MAX_INPUTS                  */
  int32_t  n_ops;     /* 1..FPK_CHAIN_MAX_OPS                     */
  int32_t  result;    /* slot written to out                      */
  uint32_t flags;
  int32_t  in_dtype[FPK_CHAIN_MAX_INPUTS];
  int32_t  in_bcast[FPK_CHAIN_MAX_INPUTS];
  fpk_chain_op ops[FPK_CHAIN_MAX_OPS];
} fpk_chain_desc;

/* ---- layer norm over the last axis ---------------------------------------- */
/* Not part of the reference's fused-step interface (no reference counterpart):
 * the `layer_norm` torch steps that plans of extension graphs carry between their
 * fused steps (the BERT-style block) run here.  x and y are contiguous
 * [rows, cols]; w and b are per-column vectors of length cols, both given or both
 * NULL; one dtype for all four. */
typedef struct fpk_ln_desc {
  uint32_t size;      /* sizeof(fpk_ln_desc)                       */
  uint32_t version;   /* FPK_ABI_VERSION                           */
  int32_t  dtype;     /* FPK_F16 or FPK_F32                        */
  int32_t  reserved;  /* 0                                         */
  int64_t  rows;
  int64_t  cols;      /* a multiple of 8, at most FPK_LN_MAX_COLS   */
  float    eps;
  uint32_t flags;     /* 0                                         */
} fpk_ln_desc;
#define FPK_LN_MAX_COLS 2048

/* ---- entry points --------------------------------------------------------- */
/* ABI version compiled into the library (FPK_ABI_VERSION). */
int fpk_version(void);

/* Static, human-readable text for a status code. */
const char* fpk_status_string(int status);

/* FPK_OK if `device` is an sm_100 GPU the library was built for. */
int fpk_device_check(int device);

/* Fill `d` for contiguous [batch, heads, seq_len, head_dim] tensors. */
int fpk_attn_desc_init(fpk_attn_desc* d, int dtype, int64_t batch, int64_t heads,
                       int64_t seq_len, int head_dim, float scale);

/* Enqueue the attention forward on `stream` (a CUstream/cudaStream_t, NULL =
 * legacy default stream).  q, k, v, o are device pointers. */
int fpk_attention_fwd(const fpk_attn_desc* d, const void* q, const void* k,
                      const void* v, void* o, void* stream);

/* Enqueue one fused chain on `stream`.  inputs[i] is a device pointer laid out
 * as d->in_bcast[i] says; out is a contiguous [rows, cols] device buffer. */
int fpk_chain_fwd(const fpk_chain_desc* d, const void* const* inputs, int n_inputs,
                  void* out, void* stream);

/* Compile (and cache for the process) the per-program kernel of a chain
 * without launching it, as the first fpk_chain_fwd with this op list, operand
 * types and broadcast modes (and, in rows mode, column count) would.  Needs no
 * device.  FPK_OK, or FPK_ERR_UNSUPPORTED when the chain is not one this tier
 * compiles (cols % 8 != 0, rows mode with cols > 16384, FPK_FLAG_NO_JIT /
 * NO_STAGING / TEST_TIMEOUT) or no run-time compiler (libnvrtc.so.12) is
 * available -- fpk_chain_fwd then runs the prebuilt kernels.  Counterpart of the reference's kernel warm-up: Triton
 * compiles each fp_chain_<N> at its first launch (python/fusionpass/kernels.py:
 * 288-300). */
int fpk_chain_precompile(const fpk_chain_desc* d);

/* Diagnostic, no reference counterpart: the number of chains this process has
 * launched through run-time compiled kernels (the rest ran on the prebuilt
 * interpreter kernels). */
int64_t fpk_chain_jit_launches(void);

/* y = (x - mean) / sqrt(var + eps) * w + b over each row (mean and biased variance
 * in f32), enqueued on `stream`.  FPK_ERR_UNSUPPORTED for cols outside
 * (0, FPK_LN_MAX_COLS] or not a multiple of 8 (the caller keeps its own
 * implementation for those); FPK_ERR_ALIGN for pointers not 16-byte aligned. */
int fpk_layer_norm_fwd(const fpk_ln_desc* d, const void* x, const void* w, const void* b, void* y,
                       void* stream);

/* The same LayerNorm of the sum of n_addends (1..4) inputs, added in f32 in the given
 * order: bcast[i] is FPK_BCAST_FULL ([rows, cols], contiguous) or FPK_BCAST_COL
 * (length cols).  The add chain that feeds a LayerNorm (residual + bias), fused into it. */
int fpk_add_layer_norm_fwd(const fpk_ln_desc* d, const void* const* addends, const int32_t* bcast,
                           int n_addends, const void* w, const void* b, void* y, void* stream);

/* Synchronise `stream`, then return and clear the device status word of
 * `device` (FPK_OK or the first FPK_ERR_* a kernel recorded, e.g. a timeout). */
int fpk_poll_status(int device, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FPKERN_H */
