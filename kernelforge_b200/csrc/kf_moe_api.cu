// C ABI of the fused MoE layer: argument checks, workspace plan, TMA tensor maps
// and the launch sequence.  No allocation, no host synchronisation (except
// kf_moe_read_status, which exists to synchronise).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "kf_internal.cuh"
#include "kf_moe.h"

namespace kf {

namespace {

constexpr size_t kAlign = 256;
constexpr int kSplitKMaxT = 64;  // calls of at most this many tokens split the GEMMs' K loop
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct DeviceInfo {
  bool ready = false;
  int num_sms = 0;
  int status = KF_OK;
};

std::mutex g_mu;
DeviceInfo g_dev[64];
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

// ------------------------------------------------------------- profiling --
struct Profiler {
  bool on = false;
  std::vector<cudaEvent_t> ev[KF_KERNEL_COUNT];  // start/stop pairs
  size_t used[KF_KERNEL_COUNT] = {};
};
Profiler g_prof;
std::mutex g_prof_mu;

struct ProfScope {
  int k;
  cudaStream_t s;
  cudaEvent_t stop = nullptr;
  ProfScope(int kernel, cudaStream_t stream) : k(kernel), s(stream) {
    if (!g_prof.on) return;
    std::lock_guard<std::mutex> lock(g_prof_mu);
    auto& v = g_prof.ev[k];
    const size_t i = g_prof.used[k];
    while (v.size() < 2 * (i + 1)) {
      cudaEvent_t e;
      if (cudaEventCreate(&e) != cudaSuccess) return;
      v.push_back(e);
    }
    cudaEventRecord(v[2 * i], s);
    stop = v[2 * i + 1];
    g_prof.used[k] = i + 1;
  }
  ~ProfScope() {
    if (stop) cudaEventRecord(stop, s);
  }
};

int ensure_device(int* num_sms) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return KF_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (major != 10 || minor != 0) {
      d.status = KF_ERR_UNSUPPORTED_DEVICE;
    } else if (gemm_set_attributes() != cudaSuccess) {
      d.status = KF_ERR_CUDA;
    } else {
      d.status = KF_OK;
    }
    if (!g_encode && d.status == KF_OK) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
          q != cudaDriverEntryPointSuccess || fn == nullptr) {
        d.status = KF_ERR_DRIVER_ENTRY_POINT;
      } else {
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
      }
    }
    d.ready = true;
  }
  *num_sms = d.num_sms;
  return d.status;
}

// Row-major [outer, inner] elements of 1 (u8), 2 (bf16) or 4 (f32) bytes, box [box_outer, box_inner], 128-byte
// swizzle.
bool encode_2d_uncached(CUtensorMap* map, const void* base, int elem_bytes, uint64_t inner, uint64_t outer,
                        uint32_t box_inner, uint32_t box_outer) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * static_cast<uint64_t>(elem_bytes)};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t elem_strides[2] = {1, 1};
  const CUresult r = g_encode(map,
                              elem_bytes == 4   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                              : elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                : CU_TENSOR_MAP_DATA_TYPE_UINT8,
                              2, const_cast<void*>(base), dims, strides, box, elem_strides,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Tensor maps depend only on (base, shape, box); repeated calls with the same
// weights and workspace reuse the encoded maps.
struct MapCacheEntry {
  const void* base;
  int elem_bytes;
  uint64_t inner, outer;
  uint32_t box_inner, box_outer;
  CUtensorMap map;
};
constexpr int kMapCache = 64;
MapCacheEntry g_maps[kMapCache];
int g_maps_used = 0, g_maps_next = 0;
std::mutex g_maps_mu;

bool encode_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t inner, uint64_t outer,
               uint32_t box_inner, uint32_t box_outer) {
  std::lock_guard<std::mutex> lock(g_maps_mu);
  for (int i = 0; i < g_maps_used; ++i) {
    const MapCacheEntry& c = g_maps[i];
    if (c.base == base && c.elem_bytes == elem_bytes && c.inner == inner && c.outer == outer &&
        c.box_inner == box_inner && c.box_outer == box_outer) {
      *map = c.map;
      return true;
    }
  }
  if (!encode_2d_uncached(map, base, elem_bytes, inner, outer, box_inner, box_outer)) return false;
  MapCacheEntry& c = g_maps[g_maps_next];
  c = MapCacheEntry{base, elem_bytes, inner, outer, box_inner, box_outer, *map};
  g_maps_next = (g_maps_next + 1) % kMapCache;
  if (g_maps_used < kMapCache) ++g_maps_used;
  return true;
}

bool encode_u8_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint32_t box_inner,
                  uint32_t box_outer) {
  return encode_2d(map, base, 1, inner, outer, box_inner, box_outer);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_common(int32_t T, int32_t E, int32_t offset) {
  if (!valid_tokens(T) || E < 1 || E > kMaxLocalExperts) return KF_ERR_INVALID_ARGUMENT;
  if (offset < 0 || offset + E > kEG) return KF_ERR_INVALID_ARGUMENT;
  return KF_OK;
}

// Calls of at most this many tokens run the single-block front end (it gathers
// rows on one SM, which stops paying off beyond a few dozen tokens).
constexpr int kSmallT = 32;

// Permutation (unless the single-block front end already did it), both grouped
// GEMMs and the reduce, from chunk masks already in the workspace.
int run_experts(const Workspace& w, void* ws, const RowLayout& in, const void* w13, const float* w13_scale,
                const void* w2, const float* w2_scale, int T, int E, int offset, void* out, int out_fp32, int num_sms,
                bool front_done, cudaStream_t s, const PeerOut& po = PeerOut{nullptr, nullptr, 0, 1}) {
  int* status = ws_ptr<int>(ws, w.status);
  Meta* meta = ws_ptr<Meta>(ws, w.meta);
  if (!front_done) {
    ProfScope ps(KF_KERNEL_PERMUTE_SCAN, s);
    if (launch_permute_scan(ws_ptr<uint4>(ws, w.chunk_masks), w.nchunk, E, meta, ws_ptr<int32_t>(ws, w.chunk_base),
                            ws_ptr<int32_t>(ws, w.tile_expert), ws_ptr<int32_t>(ws, w.tile_row0),
                            ws_ptr<int32_t>(ws, w.tile_rows), w.nt_cap, status, s) != cudaSuccess)
      return KF_ERR_CUDA;
  }
  if (!front_done) {
    ProfScope ps(KF_KERNEL_PERMUTE_ASSIGN, s);
    if (launch_permute_assign(in, ws_ptr<uint4>(ws, w.chunk_masks), ws_ptr<int32_t>(ws, w.chunk_base),
                              meta, T, E, offset, w.p_cap, ws_ptr<int32_t>(ws, w.token_slot),
                              ws_ptr<int32_t>(ws, w.slot_token), ws_ptr<float>(ws, w.slot_weight),
                              ws_ptr<int32_t>(ws, w.slot_pair), status, s) != cudaSuccess)
      return KF_ERR_CUDA;
  }
  if (!front_done) {
    ProfScope ps(KF_KERNEL_GATHER_ROWS, s);
    if (launch_gather_rows(meta, ws_ptr<int32_t>(ws, w.tile_rows), ws_ptr<int32_t>(ws, w.slot_token), in, w.p_cap,
                           ws_ptr<uint8_t>(ws, w.a_rows), ws_ptr<float>(ws, w.a_scale), 4 * num_sms,
                           s) != cudaSuccess)
      return KF_ERR_CUDA;
  }

  // Row tiles with <= 32 valid rows load only a 32-row A box (the MMA still spans
  // 128 rows; the stale rows only feed accumulator rows that are never stored).
  CUtensorMap tm_a, tm_a32, tm_w13, tm_chi, tm_clo, tm_chi32, tm_clo32, tm_w2;
  if (!encode_u8_2d(&tm_a, ws_ptr<uint8_t>(ws, w.a_rows), kH, w.p_cap, kBlk, kBlk) ||
      !encode_u8_2d(&tm_a32, ws_ptr<uint8_t>(ws, w.a_rows), kH, w.p_cap, kBlk, 32) ||
      !encode_u8_2d(&tm_w13, w13, kH, static_cast<uint64_t>(E) * 2 * kI, kBlk, kBlk) ||
      !encode_u8_2d(&tm_chi, ws_ptr<uint8_t>(ws, w.c_hi), kI, w.p_cap, kBlk, kBlk) ||
      !encode_u8_2d(&tm_clo, ws_ptr<uint8_t>(ws, w.c_lo), kI, w.p_cap, kBlk, kBlk) ||
      !encode_u8_2d(&tm_chi32, ws_ptr<uint8_t>(ws, w.c_hi), kI, w.p_cap, kBlk, 32) ||
      !encode_u8_2d(&tm_clo32, ws_ptr<uint8_t>(ws, w.c_lo), kI, w.p_cap, kBlk, 32) ||
      !encode_u8_2d(&tm_w2, w2, kI, static_cast<uint64_t>(E) * kH, kBlk, 256))
    return KF_ERR_INVALID_ARGUMENT;
  const int32_t* t_exp = ws_ptr<int32_t>(ws, w.tile_expert);
  const int32_t* t_row0 = ws_ptr<int32_t>(ws, w.tile_row0);
  const int32_t* t_rows = ws_ptr<int32_t>(ws, w.tile_rows);
  Gemm1Args g1;
  g1.meta = meta;
  g1.tile_expert = t_exp;
  g1.tile_row0 = t_row0;
  g1.tile_rows = t_rows;
  g1.a_scale = ws_ptr<float>(ws, w.a_scale);
  g1.w13_scale = w13_scale;
  g1.c_hi = ws_ptr<uint8_t>(ws, w.c_hi);
  g1.c_lo = ws_ptr<uint8_t>(ws, w.c_lo);
  g1.c_scale = ws_ptr<float>(ws, w.c_scale);
  g1.p_cap = w.p_cap;
  g1.status = status;
  g1.ksplit = w.ksplit1;
  g1.max_pairs = T * kTopK;
  g1.slot_pair = ws_ptr<int32_t>(ws, w.slot_pair);
  g1.partial = ws_ptr<float>(ws, w.partial);
  g1.decode = T <= 32 ? 1 : 0;
  {
    ProfScope ps(KF_KERNEL_GEMM1, s);
    const int units = w.nt_cap * kIB * g1.ksplit;
    if (launch_gemm1(tm_a, tm_a32, tm_w13, g1, units < num_sms ? units : num_sms, s) != cudaSuccess)
      return KF_ERR_CUDA;
  }
  if (g1.ksplit > 1) {
    ProfScope ps(KF_KERNEL_SWIGLU_QUANT, s);
    if (launch_swiglu_quant(g1, num_sms, s) != cudaSuccess) return KF_ERR_CUDA;
  }

  Gemm2Args g2;
  g2.meta = meta;
  g2.tile_expert = t_exp;
  g2.tile_row0 = t_row0;
  g2.tile_rows = t_rows;
  g2.c_scale = g1.c_scale;
  g2.w2_scale = w2_scale;
  g2.slot_weight = ws_ptr<float>(ws, w.slot_weight);
  g2.y = ws_ptr<__nv_bfloat16>(ws, w.y);
  g2.p_cap = w.p_cap;
  g2.status = status;
  g2.decode = T <= 32 ? 1 : 0;

  {
    ProfScope ps(KF_KERNEL_GEMM2, s);
    const int units = w.nt_cap * (kH / 256);
    CUtensorMap tm_y;
    if (!encode_2d(&tm_y, ws_ptr<__nv_bfloat16>(ws, w.y), 2, kH, w.p_cap, 64, 32)) return KF_ERR_INVALID_ARGUMENT;
    if (launch_gemm2(tm_chi, tm_clo, tm_chi32, tm_clo32, tm_w2, tm_y, g2, units < num_sms ? units : num_sms, s) !=
        cudaSuccess)
      return KF_ERR_CUDA;
  }

  {
    ProfScope ps(KF_KERNEL_REDUCE, s);
    if (launch_reduce(ws_ptr<int32_t>(ws, w.token_slot), ws_ptr<__nv_bfloat16>(ws, w.y), T, out, out_fp32, po, 2 * num_sms,
                      s) !=
        cudaSuccess)
      return KF_ERR_CUDA;
  }
  return KF_OK;
}

int run_front_small(const Workspace& w, void* ws, const float* logits, const void* bias, float rsf,
                    const RowLayout& in, int T, int E, int offset, cudaStream_t s) {
  ProfScope ps(KF_KERNEL_FRONT_SMALL, s);
  return launch_front_small(logits, bias, rsf, in, T, E, offset, w.p_cap, ws_ptr<Meta>(ws, w.meta),
                            ws_ptr<int32_t>(ws, w.tile_expert),
                            ws_ptr<int32_t>(ws, w.tile_row0), ws_ptr<int32_t>(ws, w.tile_rows),
                            ws_ptr<int32_t>(ws, w.token_slot),
                            ws_ptr<int32_t>(ws, w.slot_token), ws_ptr<float>(ws, w.slot_weight),
                            ws_ptr<int32_t>(ws, w.slot_pair), ws_ptr<uint8_t>(ws, w.a_rows),
                            ws_ptr<float>(ws, w.a_scale), ws_ptr<int>(ws, w.status), s) == cudaSuccess
             ? KF_OK
             : KF_ERR_CUDA;
}

}  // namespace

Workspace plan_workspace(int32_t T, int32_t E) {
  Workspace w{};
  const int64_t pairs_max = static_cast<int64_t>(T) * (E < kTopK ? E : kTopK);
  const int64_t rows = align_up(static_cast<size_t>(pairs_max + static_cast<int64_t>(E) * (kBlk - 1)), kBlk);
  w.p_cap = static_cast<int32_t>(rows);
  w.nt_cap = w.p_cap / kBlk;
  w.nchunk = (T + kChunkTokens - 1) / kChunkTokens;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, kAlign);
    return o;
  };
  const size_t tk = static_cast<size_t>(T) * kTopK;
  const size_t pc = static_cast<size_t>(w.p_cap);
  w.status = take(sizeof(int32_t));
  w.meta = take(sizeof(Meta));
  w.topk_idx = take(tk * 4);
  w.topk_w = take(tk * 4);
  w.token_slot = take(tk * 4);
  w.chunk_masks = take(static_cast<size_t>(w.nchunk) * E * 16);
  w.chunk_base = take(static_cast<size_t>(w.nchunk) * E * 4);
  w.tile_expert = take(static_cast<size_t>(w.nt_cap) * 4);
  w.tile_row0 = take(static_cast<size_t>(w.nt_cap) * 4);
  w.tile_rows = take(static_cast<size_t>(w.nt_cap) * 4);
  w.slot_token = take(pc * 4);
  w.slot_weight = take(pc * 4);
  w.slot_pair = take(pc * 4);
  w.a_rows = take(pc * kH);
  w.a_scale = take(pc * kHB * 4);
  w.c_hi = take(pc * kI);
  w.c_lo = take(pc * kI);
  w.c_scale = take(pc * kIB * 4);
  w.y = take(pc * kH * 2);  // bf16 rows
  // split-K of GEMM1 for decode-sized calls: with one row tile per active expert
  // its 16 column blocks per tile give about one wave of units, which a 4-way K
  // split turns into four shorter, evenly filled waves
  w.ksplit1 = T <= kSplitKMaxT ? 4 : 1;
  const size_t max_pairs = static_cast<size_t>(T) * kTopK;
  w.partial = take(w.ksplit1 > 1 ? static_cast<size_t>(w.ksplit1) * 2 * kI * max_pairs * 4 : 0);
  w.total = off;
  return w;
}

}  // namespace kf

using namespace kf;

extern "C" {

size_t kf_moe_workspace_bytes(int32_t num_tokens, int32_t num_local_experts) {
  if (!valid_tokens(num_tokens) || num_local_experts < 1 || num_local_experts > kMaxLocalExperts) return 0;
  return plan_workspace(num_tokens, num_local_experts).total;
}

int32_t kf_moe_launches_per_forward(void) { return 7; }

const char* kf_moe_error_string(int code) {
  switch (code) {
    case KF_OK: return "ok";
    case KF_ERR_INVALID_ARGUMENT: return "invalid argument";
    case KF_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case KF_ERR_CUDA: return "CUDA error";
    case KF_ERR_UNSUPPORTED_DEVICE: return "unsupported device (needs sm_100a / B200)";
    case KF_ERR_DRIVER_ENTRY_POINT: return "cuTensorMapEncodeTiled unavailable";
    case KF_ERR_DEVICE_STATUS: return "device-side error (see status bits)";
    case KF_ERR_EXCEEDS_STATIC_SCRATCH: return "call exceeds the static scratch of kf_moe_forward_noalloc";
    default: return "unknown error";
  }
}

int kf_moe_route(const float* routing_logits, const void* routing_bias, int32_t num_tokens,
                 float routed_scaling_factor, int32_t* topk_idx, float* topk_weight, void* stream) {
  if (!valid_tokens(num_tokens)) return KF_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return KF_OK;
  if (!routing_logits || !routing_bias || !topk_idx || !topk_weight) return KF_ERR_INVALID_ARGUMENT;
  if (!aligned16(routing_logits) || !aligned16(routing_bias)) return KF_ERR_INVALID_ARGUMENT;
  int sms = 0;
  const int st = ensure_device(&sms);
  if (st != KF_OK) return st;
  ProfScope ps(KF_KERNEL_ROUTE, static_cast<cudaStream_t>(stream));
  return launch_route(routing_logits, routing_bias, num_tokens, routed_scaling_factor, topk_idx, topk_weight, 0, 0,
                      nullptr, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? KF_OK
             : KF_ERR_CUDA;
}

int kf_moe_forward(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                   const float* hidden_states_scale, const void* gemm1_weights, const float* gemm1_weights_scale,
                   const void* gemm2_weights, const float* gemm2_weights_scale, int32_t num_tokens,
                   int32_t num_local_experts, int32_t local_expert_offset, float routed_scaling_factor,
                   void* output, void* workspace, size_t workspace_bytes, void* stream) {
  const int T = num_tokens, E = num_local_experts;
  int rc = check_common(T, E, local_expert_offset);
  if (rc != KF_OK) return rc;
  if (T == 0) return KF_OK;
  if (!routing_logits || !routing_bias || !hidden_states || !hidden_states_scale || !gemm1_weights ||
      !gemm1_weights_scale || !gemm2_weights || !gemm2_weights_scale || !output || !workspace)
    return KF_ERR_INVALID_ARGUMENT;
  if (!aligned16(routing_logits) || !aligned16(routing_bias) || !aligned16(hidden_states) ||
      !aligned16(gemm1_weights) || !aligned16(gemm2_weights) || !aligned16(output) || !aligned16(workspace))
    return KF_ERR_INVALID_ARGUMENT;
  const Workspace w = plan_workspace(T, E);
  if (workspace_bytes < w.total) return KF_ERR_WORKSPACE_TOO_SMALL;
  int sms = 0;
  rc = ensure_device(&sms);
  if (rc != KF_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool small = T <= kSmallT;
  // the single-block front end clears the status word itself (one node fewer in
  // the decode chain); the multi-block path clears it first
  if (!small && cudaMemsetAsync(ws_ptr<int>(workspace, w.status), 0, sizeof(int), s) != cudaSuccess)
    return KF_ERR_CUDA;
  int32_t* topk_idx = ws_ptr<int32_t>(workspace, w.topk_idx);
  float* topk_w = ws_ptr<float>(workspace, w.topk_w);
  const RowLayout in = reference_layout(topk_idx, topk_w, hidden_states, hidden_states_scale, T);
  if (small) {
    rc = run_front_small(w, workspace, routing_logits, routing_bias, routed_scaling_factor, in, T, E,
                         local_expert_offset, s);
    if (rc != KF_OK) return rc;
  } else {
    ProfScope ps(KF_KERNEL_ROUTE, s);
    if (launch_route(routing_logits, routing_bias, T, routed_scaling_factor, topk_idx, topk_w, E,
                     local_expert_offset, ws_ptr<uint4>(workspace, w.chunk_masks), s) != cudaSuccess)
      return KF_ERR_CUDA;
  }
  return run_experts(w, workspace, in, gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, T, E,
                     local_expert_offset, output, 0, sms, small, s);
}

}  // extern "C"

namespace kf {
namespace {

// Experts on rows in `in` (reference or packed layout): the shared body of
// kf_moe_experts and kf_moe_experts_packed.
int experts_common(const RowLayout& in, const void* gemm1_weights, const float* gemm1_weights_scale,
                   const void* gemm2_weights, const float* gemm2_weights_scale, int32_t T, int32_t E, int32_t offset,
                   void* output, int32_t output_fp32, void* workspace, size_t workspace_bytes, void* stream,
                   const PeerOut& po = PeerOut{nullptr, nullptr, 0, 1}) {
  int rc = check_common(T, E, offset);
  if (rc != KF_OK) return rc;
  if (T == 0) return KF_OK;
  if (!gemm1_weights || !gemm1_weights_scale || !gemm2_weights || !gemm2_weights_scale || (!output && !po.peer_back) ||
      !workspace)
    return KF_ERR_INVALID_ARGUMENT;
  if (!aligned16(in.hidden) || !aligned16(gemm1_weights) || !aligned16(gemm2_weights) ||
      (output && !aligned16(output)) || !aligned16(workspace))
    return KF_ERR_INVALID_ARGUMENT;
  const Workspace w = plan_workspace(T, E);
  if (workspace_bytes < w.total) return KF_ERR_WORKSPACE_TOO_SMALL;
  int sms = 0;
  rc = ensure_device(&sms);
  if (rc != KF_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* status = ws_ptr<int>(workspace, w.status);
  const bool small = T <= kSmallT;
  if (!small && cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess) return KF_ERR_CUDA;
  if (small) {
    rc = run_front_small(w, workspace, nullptr, nullptr, 0.f, in, T, E, offset, s);
    if (rc != KF_OK) return rc;
  } else {
    ProfScope ps(KF_KERNEL_MASKS, s);
    if (launch_masks_from_topk(in, T, E, offset, ws_ptr<uint4>(workspace, w.chunk_masks), status, s) != cudaSuccess)
      return KF_ERR_CUDA;
  }
  return run_experts(w, workspace, in, gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, T, E,
                     offset, output, output_fp32 ? 1 : 0, sms, small, s, po);
}

}  // namespace
}  // namespace kf

extern "C" {

int kf_moe_experts(const int32_t* topk_idx, const float* topk_weight, const void* hidden_states,
                   const float* hidden_states_scale, const void* gemm1_weights, const float* gemm1_weights_scale,
                   const void* gemm2_weights, const float* gemm2_weights_scale, int32_t num_tokens,
                   int32_t num_local_experts, int32_t local_expert_offset, void* output, int32_t output_fp32,
                   void* workspace, size_t workspace_bytes, void* stream) {
  if (num_tokens > 0 && (!topk_idx || !topk_weight || !hidden_states || !hidden_states_scale))
    return KF_ERR_INVALID_ARGUMENT;
  return experts_common(reference_layout(topk_idx, topk_weight, hidden_states, hidden_states_scale, num_tokens),
                        gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, num_tokens,
                        num_local_experts, local_expert_offset, output, output_fp32, workspace, workspace_bytes,
                        stream);
}

int kf_moe_experts_packed(const void* rows, const void* gemm1_weights, const float* gemm1_weights_scale,
                          const void* gemm2_weights, const float* gemm2_weights_scale, int32_t num_rows,
                          int32_t num_local_experts, int32_t local_expert_offset, void* output, int32_t output_fp32,
                          void* workspace, size_t workspace_bytes, void* stream) {
  if (num_rows > 0 && !rows) return KF_ERR_INVALID_ARGUMENT;
  return experts_common(packed_layout(rows), gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                        num_rows, num_local_experts, local_expert_offset, output, output_fp32, workspace,
                        workspace_bytes, stream);
}

int kf_moe_experts_packed_p2p(const void* rows, const void* gemm1_weights, const float* gemm1_weights_scale,
                              const void* gemm2_weights, const float* gemm2_weights_scale, int32_t num_rows,
                              int32_t num_local_experts, int32_t local_expert_offset, const int32_t* counts,
                              int32_t rank, int32_t world, void* const* peer_back, void* workspace,
                              size_t workspace_bytes, void* stream) {
  if (num_rows > 0 && (!rows || !counts || !peer_back)) return KF_ERR_INVALID_ARGUMENT;
  if (world < 1 || world > 64 || rank < 0 || rank >= world) return KF_ERR_INVALID_ARGUMENT;
  return experts_common(packed_layout(rows), gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                        num_rows, num_local_experts, local_expert_offset, nullptr, 0, workspace, workspace_bytes,
                        stream, PeerOut{peer_back, counts, rank, world});
}

int kf_moe_profile_begin(void) {
  std::lock_guard<std::mutex> lock(g_prof_mu);
  for (int k = 0; k < KF_KERNEL_COUNT; ++k) g_prof.used[k] = 0;
  g_prof.on = true;
  return KF_OK;
}

int kf_moe_profile_end(float* total_ms, int32_t* launches, int32_t n) {
  std::lock_guard<std::mutex> lock(g_prof_mu);
  g_prof.on = false;
  int rc = KF_OK;
  for (int k = 0; k < KF_KERNEL_COUNT; ++k) {
    float sum = 0.f;
    for (size_t i = 0; i < g_prof.used[k]; ++i) {
      float ms = 0.f;
      if (cudaEventSynchronize(g_prof.ev[k][2 * i + 1]) != cudaSuccess ||
          cudaEventElapsedTime(&ms, g_prof.ev[k][2 * i], g_prof.ev[k][2 * i + 1]) != cudaSuccess)
        rc = KF_ERR_CUDA;
      sum += ms;
    }
    if (k < n) {
      if (total_ms) total_ms[k] = sum;
      if (launches) launches[k] = static_cast<int32_t>(g_prof.used[k]);
    }
    g_prof.used[k] = 0;
  }
  return rc;
}

int kf_moe_read_status(void* workspace, int32_t* status, void* stream) {
  if (!workspace || !status) return KF_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const Workspace w = plan_workspace(0, 1);  // the status word is always at offset 0
  int32_t v = 0;
  if (cudaMemcpyAsync(&v, ws_ptr<int>(workspace, w.status), sizeof(int32_t), cudaMemcpyDeviceToHost, s) !=
          cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return KF_ERR_CUDA;
  *status = v;
  if (cudaMemsetAsync(ws_ptr<int>(workspace, w.status), 0, sizeof(int), s) != cudaSuccess) return KF_ERR_CUDA;
  return v ? KF_ERR_DEVICE_STATUS : KF_OK;
}

}  // extern "C"
