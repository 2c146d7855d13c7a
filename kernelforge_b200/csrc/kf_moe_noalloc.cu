// kf_moe_forward_noalloc: the whole layer with its scratch memory in a static
// device array, for callers that cannot allocate device memory (see kf_moe.h).
// It runs the same launch sequence as kf_moe_forward, on this array instead of
// a caller-provided workspace.
#include <cuda_runtime.h>

#include <mutex>

#include "kf_moe.h"

// Scratch of kf_moe_forward_noalloc.  Every GPU that loads this library holds
// its own copy until the process exits.  In host code this name is only a
// handle for cudaGetSymbolAddress, never a device address.
static __device__ __align__(256) unsigned char g_kf_noalloc_scratch[KF_MOE_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the current device's copy of the array, looked up once per
// device (with that device current) and cached.
int noalloc_scratch(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return KF_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_kf_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return KF_ERR_CUDA;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return KF_OK;
}

}  // namespace

extern "C" int kf_moe_forward_noalloc(const float* routing_logits, const void* routing_bias,
                                      const void* hidden_states, const float* hidden_states_scale,
                                      const void* gemm1_weights, const float* gemm1_weights_scale,
                                      const void* gemm2_weights, const float* gemm2_weights_scale,
                                      int32_t num_tokens, int32_t num_local_experts, int32_t local_expert_offset,
                                      float routed_scaling_factor, void* output, void* stream) {
  // the checks kf_moe_forward makes on every call come first, so a call that is
  // invalid there is invalid here too; the static array's own limits come after
  if (num_tokens < 0 || num_tokens > KF_MOE_MAX_TOKENS || num_local_experts < 1 ||
      num_local_experts > KF_MOE_GLOBAL_EXPERTS || local_expert_offset < 0 ||
      local_expert_offset > KF_MOE_GLOBAL_EXPERTS - num_local_experts)
    return KF_ERR_INVALID_ARGUMENT;
  if (num_tokens > KF_MOE_NOALLOC_MAX_TOKENS || num_local_experts > KF_MOE_NOALLOC_MAX_LOCAL_EXPERTS)
    return KF_ERR_EXCEEDS_STATIC_SCRATCH;
  if (num_tokens == 0) return KF_OK;
  const size_t need = kf_moe_workspace_bytes(num_tokens, num_local_experts);
  if (need == 0 || need > static_cast<size_t>(KF_MOE_NOALLOC_SCRATCH_BYTES)) return KF_ERR_EXCEEDS_STATIC_SCRATCH;
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != KF_OK) return rc;
  // kf_moe_forward zeroes the status word on the stream first and writes every
  // other scratch array before it reads it, so the previous call's contents do
  // not leak into this one.
  return kf_moe_forward(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                        gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, num_tokens, num_local_experts,
                        local_expert_offset, routed_scaling_factor, output, scratch,
                        static_cast<size_t>(KF_MOE_NOALLOC_SCRATCH_BYTES), stream);
}

// The status word of kf_moe_forward_noalloc's calls sits at the start of the
// static array (kf_moe_forward keeps it at offset 0 of its scratch): read it and
// clear it on the stream, without allocating.
extern "C" int kf_moe_noalloc_read_status(int32_t* status, void* stream) {
  if (!status) return KF_ERR_INVALID_ARGUMENT;
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != KF_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t v = 0;
  if (cudaMemcpyAsync(&v, scratch, sizeof(int32_t), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess || cudaMemsetAsync(scratch, 0, sizeof(int32_t), s) != cudaSuccess)
    return KF_ERR_CUDA;
  *status = v;
  return v ? KF_ERR_DEVICE_STATUS : KF_OK;
}
