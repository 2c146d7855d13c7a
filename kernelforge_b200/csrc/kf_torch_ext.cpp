// PyTorch C++ extension over the C ABI: the reference operator kernel(...)
// (solution/triton/kernel.py:1817-1950) for torch tensors.
//
// The reference's CUDA stub binds its entry through a framework FFI
// (solution/cuda/binding.py:14-25); this module is the torch-side binding of
// kf_moe_forward: it checks dtypes, shapes and devices, makes the inputs
// contiguous (as the reference does at kernel.py:1881-1886), allocates the bf16
// output and a cached workspace through torch's caching allocator, launches on
// the current torch CUDA stream with the tensors' device current, and turns
// every failure into a Python RuntimeError.
//
// Errors found on the device (a bounded wait that gave up, a bounds check) are
// reported without a host synchronisation per call: after each launch the
// workspace's status word is copied asynchronously into pinned host memory and
// an event is recorded; the next call on that (device, stream) raises for any
// completed copy that holds a set bit, and read_status() synchronises and
// reports at once.  Calls under CUDA-graph capture are not mirrored.
#include <ATen/cuda/CUDAContext.h>
#include <ATen/cuda/CUDAEvent.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <utility>

#include "kf_moe.h"

namespace {

constexpr int64_t kH = KF_MOE_HIDDEN, kI = KF_MOE_INTERMEDIATE, kEG = KF_MOE_GLOBAL_EXPERTS, kB = KF_MOE_BLOCK;

struct Pending {
  at::Tensor mirror;                         // pinned int32 [1]
  std::shared_ptr<at::cuda::CUDAEvent> done;  // recorded after the copy
};

struct Scratch {
  at::Tensor ws;
  std::deque<Pending> pending;
};

std::mutex g_mu;
std::map<std::pair<int64_t, int64_t>, Scratch> g_scratch;  // (device index, stream id)

std::string status_message(int32_t v) {
  static const std::pair<int32_t, const char*> bits[] = {
      {KF_STATUS_TIMEOUT_PRODUCER, "a TMA producer timed out waiting for a free stage"},
      {KF_STATUS_TIMEOUT_MMA, "the MMA issuer timed out waiting for data or tensor memory"},
      {KF_STATUS_TIMEOUT_EPILOGUE, "a promotion/epilogue warp timed out"},
      {KF_STATUS_BAD_EXPERT, "a routed expert id outside [0, 256)"},
      {KF_STATUS_SLOT_OVERFLOW, "a permuted row index beyond the workspace capacity"},
      {KF_STATUS_TIMEOUT_PEER, "a peer rank did not reach a barrier in time"}};
  char head[64];
  snprintf(head, sizeof(head), "device status 0x%x:", static_cast<unsigned>(v));
  std::string s(head);
  int32_t known = 0;
  for (const auto& b : bits) {
    known |= b.first;
    if (v & b.first) s += std::string(" ") + b.second + ";";
  }
  if (v & ~known) s += " unknown bits;";
  return s;
}

// Raise for the first completed status copy with a set bit (copies still in
// flight are left for a later call).
void check_pending(Scratch& sc) {
  while (!sc.pending.empty() && sc.pending.front().done->query()) {
    const int32_t v = *sc.pending.front().mirror.data_ptr<int32_t>();
    sc.pending.pop_front();
    TORCH_CHECK(v == 0, "an earlier call on this stream failed on the device: ", status_message(v));
  }
}

void mirror_status(Scratch& sc, const at::cuda::CUDAStream& stream) {
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream.stream(), &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) return;
  at::Tensor m = at::empty({1}, at::TensorOptions().dtype(at::kInt).pinned_memory(true));
  TORCH_CHECK(cudaMemcpyAsync(m.data_ptr(), sc.ws.data_ptr(), sizeof(int32_t), cudaMemcpyDeviceToHost,
                              stream.stream()) == cudaSuccess,
              "status copy failed");
  auto ev = std::make_shared<at::cuda::CUDAEvent>();
  ev->record(stream);
  sc.pending.push_back(Pending{m, ev});
}

at::Tensor expect(const at::Tensor& t, const char* name, at::ScalarType dtype, at::IntArrayRef shape,
                  const at::Device& dev) {
  TORCH_CHECK(t.scalar_type() == dtype, name, " must be ", dtype, ", got ", t.scalar_type());
  TORCH_CHECK(t.sizes() == shape, name, " must have shape ", shape, ", got ", t.sizes());
  TORCH_CHECK(t.device() == dev, name, " is on ", t.device(), ", expected ", dev);
  return t.contiguous();
}

// kf_moe_forward on torch tensors; value-returning like the reference kernel(...).
at::Tensor kernel(const at::Tensor& routing_logits, const at::Tensor& routing_bias, const at::Tensor& hidden_states,
                  const at::Tensor& hidden_states_scale, const at::Tensor& gemm1_weights,
                  const at::Tensor& gemm1_weights_scale, const at::Tensor& gemm2_weights,
                  const at::Tensor& gemm2_weights_scale, int64_t local_expert_offset, double routed_scaling_factor) {
  const at::Device dev = hidden_states.device();
  TORCH_CHECK(dev.is_cuda(), "kernelforge_b200.kernel needs CUDA tensors on a B200 (sm_100a); no CPU fallback");
  TORCH_CHECK(routing_logits.dim() == 2, "routing_logits must be [T, 256]");
  TORCH_CHECK(gemm1_weights.dim() == 3, "gemm1_weights must be [E, 4096, 7168]");
  const int64_t T = routing_logits.size(0), E = gemm1_weights.size(0);
  const auto f8 = at::kFloat8_e4m3fn;
  at::Tensor logits = expect(routing_logits, "routing_logits", at::kFloat, {T, kEG}, dev);
  at::Tensor bias = expect(routing_bias.reshape({-1}), "routing_bias", at::kBFloat16, {kEG}, dev);
  at::Tensor hid = expect(hidden_states, "hidden_states", f8, {T, kH}, dev);
  at::Tensor hs = expect(hidden_states_scale, "hidden_states_scale", at::kFloat, {kH / kB, T}, dev);
  at::Tensor w13 = expect(gemm1_weights, "gemm1_weights", f8, {E, 2 * kI, kH}, dev);
  at::Tensor w13s = expect(gemm1_weights_scale, "gemm1_weights_scale", at::kFloat, {E, 2 * kI / kB, kH / kB}, dev);
  at::Tensor w2 = expect(gemm2_weights, "gemm2_weights", f8, {E, kH, kI}, dev);
  at::Tensor w2s = expect(gemm2_weights_scale, "gemm2_weights_scale", at::kFloat, {E, kH / kB, kI / kB}, dev);
  TORCH_CHECK(E >= 1 && local_expert_offset >= 0 && local_expert_offset + E <= kEG, "local experts [",
              local_expert_offset, ", ", local_expert_offset + E, ") outside [0, ", kEG, ")");
  TORCH_CHECK(T <= KF_MOE_MAX_TOKENS, "num_tokens ", T, " above ", KF_MOE_MAX_TOKENS);
  c10::cuda::CUDAGuard guard(dev);
  at::Tensor out = at::empty({T, kH}, hid.options().dtype(at::kBFloat16));
  if (T == 0) return out;
  const at::cuda::CUDAStream stream = at::cuda::getCurrentCUDAStream(dev.index());
  std::lock_guard<std::mutex> lock(g_mu);
  Scratch& sc = g_scratch[{dev.index(), stream.id()}];
  check_pending(sc);
  const size_t need = kf_moe_workspace_bytes(static_cast<int32_t>(T), static_cast<int32_t>(E));
  TORCH_CHECK(need > 0, "no workspace size for T=", T, ", E=", E);
  if (!sc.ws.defined() || static_cast<size_t>(sc.ws.numel()) < need)
    sc.ws = at::empty({static_cast<int64_t>(need)}, hid.options().dtype(at::kByte));
  const int rc = kf_moe_forward(logits.data_ptr<float>(), bias.data_ptr(), hid.data_ptr(), hs.data_ptr<float>(),
                                w13.data_ptr(), w13s.data_ptr<float>(), w2.data_ptr(), w2s.data_ptr<float>(),
                                static_cast<int32_t>(T), static_cast<int32_t>(E),
                                static_cast<int32_t>(local_expert_offset), static_cast<float>(routed_scaling_factor),
                                out.data_ptr(), sc.ws.data_ptr(), static_cast<size_t>(sc.ws.numel()), stream.stream());
  TORCH_CHECK(rc == KF_OK, "kf_moe_forward failed: ", kf_moe_error_string(rc), " (code ", rc, ")");
  mirror_status(sc, stream);
  return out;
}

// Synchronise the current stream of `device_index`, then return (and clear) the
// status bits of every call made through this module on it since the last read.
int64_t read_status(int64_t device_index) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device_index));
  const at::cuda::CUDAStream stream = at::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(device_index));
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_scratch.find({device_index, stream.id()});
  if (it == g_scratch.end() || !it->second.ws.defined()) return 0;
  Scratch& sc = it->second;
  int32_t v = 0;
  const int rc = kf_moe_read_status(sc.ws.data_ptr(), &v, stream.stream());
  TORCH_CHECK(rc == KF_OK || rc == KF_ERR_DEVICE_STATUS, "kf_moe_read_status failed: ", kf_moe_error_string(rc));
  for (const Pending& p : sc.pending) v |= *p.mirror.data_ptr<int32_t>();   // the stream is synchronised
  sc.pending.clear();
  return v;
}

// Drop the cached workspaces (they return to torch's caching allocator).
void release_workspaces() {
  std::lock_guard<std::mutex> lock(g_mu);
  g_scratch.clear();
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "kernelforge_b200: torch binding of the C ABI of libkf_moe.so (kf_moe.h)";
  m.def("kernel", &kernel, "the fused MoE layer (kf_moe_forward); returns bf16 [T, 7168]");
  m.def("read_status", &read_status, "synchronise and return, then clear, the device status of this module's calls");
  m.def("release_workspaces", &release_workspaces, "drop the cached workspaces");
}
