// Host-side interfaces shared by the translation units of libfpkern.so.
#pragma once

#include <cuda_runtime.h>

#include "../../include/fpkern.h"

namespace fpk {

// Per-device facts cached at first use (thread-safe).
struct DeviceInfo {
  int ok;          // FPK_OK or FPK_ERR_DEVICE
  int num_sms;
  int* status;     // device address of this device's status word
};

// Facts for the current device; returns FPK_OK or an error code.
int current_device_info(DeviceInfo* out);

int launch_chain(const fpk_chain_desc* d, const void* const* inputs, void* out,
                 cudaStream_t stream, const DeviceInfo& dev);

// Validate `d` (as fpk_chain_fwd would) and compile its per-program kernel.
int chain_precompile(const fpk_chain_desc* d);

// Per-program flat chain kernels compiled at run time (chain_jit.cu).
// FPK_ERR_UNSUPPORTED when this tier does not take the call; the caller then
// runs the interpreter kernels.
int try_launch_chain_jit(const fpk_chain_desc* d, const void* const* inputs, void* out,
                         cudaStream_t stream, const DeviceInfo& dev);
int chain_jit_precompile(const fpk_chain_desc* d);
long long chain_jit_launches();

int launch_attention_f32(const fpk_attn_desc* d, const void* q, const void* k, const void* v,
                         void* o, cudaStream_t stream, const DeviceInfo& dev);

int launch_attention_tc(const fpk_attn_desc* d, const void* q, const void* k, const void* v,
                        void* o, cudaStream_t stream, const DeviceInfo& dev);

int launch_layer_norm(const fpk_ln_desc* d, const void* const* addends, const int32_t* bcast, int n_addends,
                      const void* w, const void* b, void* y, cudaStream_t stream);

}  // namespace fpk
