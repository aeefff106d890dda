// C ABI of libfpkern.so (declared in include/fpkern.h).
//
// Replaces the reference's Triton launch boundary kernels.launch_step
// (python/fusionpass/kernels.py:336-368): the caller owns every buffer, the
// library validates the descriptor, picks the kernel for the step's dtype and
// launch mode and enqueues it on the caller's stream.  Errors come back as
// negative status codes instead of Python exceptions.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/fpkern.h"
#include "internal.h"

namespace fpk {

// One status word per device; kernels record the first error they meet
// (e.g. FPK_ERR_TIMEOUT from a bounded wait) and fpk_poll_status reads it.
__device__ int g_status;

namespace {
constexpr int kMaxDevices = 64;
std::once_flag g_once[kMaxDevices];
DeviceInfo g_info[kMaxDevices];

void init_device(int dev) {
  DeviceInfo& di = g_info[dev];
  di.ok = FPK_ERR_DEVICE;
  di.num_sms = 0;
  di.status = nullptr;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return;
  if (prop.major != 10 || prop.minor != 0) return;  // built for sm_100a only
  void* addr = nullptr;
  if (cudaGetSymbolAddress(&addr, g_status) != cudaSuccess) return;
  di.num_sms = prop.multiProcessorCount;
  di.status = static_cast<int*>(addr);
  di.ok = FPK_OK;
}
}  // namespace

int current_device_info(DeviceInfo* out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return FPK_ERR_DEVICE;
  std::call_once(g_once[dev], init_device, dev);
  *out = g_info[dev];
  return out->ok;
}

}  // namespace fpk

extern "C" {

int fpk_version(void) { return FPK_ABI_VERSION; }

const char* fpk_status_string(int status) {
  switch (status) {
    case FPK_OK: return "ok";
    case FPK_ERR_INVALID: return "invalid descriptor or argument";
    case FPK_ERR_UNSUPPORTED: return "unsupported by the sm_100a kernels";
    case FPK_ERR_ALIGN: return "pointer or stride alignment not met";
    case FPK_ERR_CUDA: return "CUDA error while launching";
    case FPK_ERR_DEVICE: return "current device is not an sm_100 (B200) GPU";
    case FPK_ERR_TIMEOUT: return "a bounded device-side wait timed out";
    default: return "unknown fpkern status";
  }
}

int fpk_device_check(int device) {
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) return FPK_ERR_DEVICE;
  if (cudaSetDevice(device) != cudaSuccess) return FPK_ERR_DEVICE;
  fpk::DeviceInfo di;
  const int rc = fpk::current_device_info(&di);
  cudaSetDevice(prev);
  return rc;
}

int fpk_attn_desc_init(fpk_attn_desc* d, int dtype, int64_t batch, int64_t heads, int64_t seq_len,
                       int head_dim, float scale) {
  if (!d) return FPK_ERR_INVALID;
  d->size = sizeof(fpk_attn_desc);
  d->version = FPK_ABI_VERSION;
  d->dtype = dtype;
  d->head_dim = head_dim;
  d->batch = batch;
  d->heads = heads;
  d->seq_len = seq_len;
  d->scale = scale;
  d->flags = 0;
  const int64_t s_stride = head_dim;
  const int64_t h_stride = seq_len * head_dim;
  const int64_t b_stride = heads * h_stride;
  int64_t* all[4] = {d->q_strides, d->k_strides, d->v_strides, d->o_strides};
  for (int64_t* st : all) {
    st[0] = b_stride;
    st[1] = h_stride;
    st[2] = s_stride;
  }
  return FPK_OK;
}

int fpk_attention_fwd(const fpk_attn_desc* d, const void* q, const void* k, const void* v, void* o,
                      void* stream) {
  if (!d || d->size != sizeof(fpk_attn_desc) || d->version != FPK_ABI_VERSION) return FPK_ERR_INVALID;
  if (!q || !k || !v || !o) return FPK_ERR_INVALID;
  if (d->dtype != FPK_F16 && d->dtype != FPK_F32) return FPK_ERR_INVALID;
  if (d->head_dim != 16 && d->head_dim != 32 && d->head_dim != 64 && d->head_dim != 128)
    return FPK_ERR_UNSUPPORTED;  // same contract as FusedAttentionOp::verify
  if (d->batch < 0 || d->heads < 0 || d->seq_len < 0) return FPK_ERR_INVALID;
  if (d->batch == 0 || d->heads == 0 || d->seq_len == 0) return FPK_OK;
  fpk::DeviceInfo dev;
  const int rc = fpk::current_device_info(&dev);
  if (rc != FPK_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (d->dtype == FPK_F16) return fpk::launch_attention_tc(d, q, k, v, o, s, dev);
  return fpk::launch_attention_f32(d, q, k, v, o, s, dev);
}

int fpk_chain_fwd(const fpk_chain_desc* d, const void* const* inputs, int n_inputs, void* out,
                  void* stream) {
  if (!d || d->size != sizeof(fpk_chain_desc) || d->version != FPK_ABI_VERSION) return FPK_ERR_INVALID;
  if (n_inputs != d->n_inputs) return FPK_ERR_INVALID;
  fpk::DeviceInfo dev;
  const int rc = fpk::current_device_info(&dev);
  if (rc != FPK_OK) return rc;
  return fpk::launch_chain(d, inputs, out, static_cast<cudaStream_t>(stream), dev);
}

int fpk_chain_precompile(const fpk_chain_desc* d) {
  if (!d || d->size != sizeof(fpk_chain_desc) || d->version != FPK_ABI_VERSION) return FPK_ERR_INVALID;
  return fpk::chain_precompile(d);
}

int64_t fpk_chain_jit_launches(void) { return static_cast<int64_t>(fpk::chain_jit_launches()); }

namespace {
int ln_checks(const fpk_ln_desc* d, const void* w, const void* b, const void* y) {
  if (!d || d->size != sizeof(fpk_ln_desc) || d->version != FPK_ABI_VERSION) return FPK_ERR_INVALID;
  if ((d->dtype != FPK_F16 && d->dtype != FPK_F32) || d->rows < 0 || d->reserved != 0 || d->flags != 0)
    return FPK_ERR_INVALID;
  if (!y || (w == nullptr) != (b == nullptr) || !(d->eps >= 0.0f)) return FPK_ERR_INVALID;
  return FPK_OK;
}
}  // namespace

int fpk_layer_norm_fwd(const fpk_ln_desc* d, const void* x, const void* w, const void* b, void* y,
                       void* stream) {
  int rc = ln_checks(d, w, b, y);
  if (rc != FPK_OK) return rc;
  if (!x) return FPK_ERR_INVALID;
  fpk::DeviceInfo dev;
  if ((rc = fpk::current_device_info(&dev)) != FPK_OK) return rc;
  const int32_t full = FPK_BCAST_FULL;
  return fpk::launch_layer_norm(d, &x, &full, 1, w, b, y, static_cast<cudaStream_t>(stream));
}

int fpk_add_layer_norm_fwd(const fpk_ln_desc* d, const void* const* addends, const int32_t* bcast, int n_addends,
                           const void* w, const void* b, void* y, void* stream) {
  int rc = ln_checks(d, w, b, y);
  if (rc != FPK_OK) return rc;
  if (!addends || !bcast || n_addends < 1 || n_addends > 4) return FPK_ERR_INVALID;
  fpk::DeviceInfo dev;
  if ((rc = fpk::current_device_info(&dev)) != FPK_OK) return rc;
  return fpk::launch_layer_norm(d, addends, bcast, n_addends, w, b, y, static_cast<cudaStream_t>(stream));
}

int fpk_poll_status(int device, void* stream) {
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) return FPK_ERR_CUDA;
  if (cudaSetDevice(device) != cudaSuccess) return FPK_ERR_DEVICE;
  fpk::DeviceInfo di;
  int rc = fpk::current_device_info(&di);
  if (rc == FPK_OK) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int value = 0;
    const int zero = 0;
    if (cudaStreamSynchronize(s) != cudaSuccess ||
        cudaMemcpyFromSymbolAsync(&value, fpk::g_status, sizeof(int), 0, cudaMemcpyDeviceToHost, s) !=
            cudaSuccess ||
        cudaMemcpyToSymbolAsync(fpk::g_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s) !=
            cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess) {
      rc = FPK_ERR_CUDA;
    } else {
      rc = value;
    }
  }
  cudaSetDevice(prev);
  return rc;
}

}  // extern "C"
