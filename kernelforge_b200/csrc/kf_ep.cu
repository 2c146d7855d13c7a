// Expert-parallel dispatch and combine (256 experts sharded over `world` ranks).
//
// Dispatch builds, on the device, the rows each destination rank receives: a
// token goes once to every rank owning at least one of its 8 experts, as one
// 7456-byte row (FP8 hidden row | 56 fp32 scales | 8 expert ids, -1 where the
// destination does not own the expert | 8 weights).  Rows are grouped by
// destination and, inside a destination, in token order.  The per-destination
// row counts (needed by the NCCL all-to-all) and each (token, destination)
// row index are written as well.  The machinery is the permute's: a token
// bitmask per destination and 128-token chunk, a scan over chunks, and the row
// index = destination offset + earlier chunks + popcount below the token.
//
// Combine sums, per token, the partial rows returned by its destinations in
// ascending rank order (fp32), with one bf16 rounding: no atomics, fixed order.
//
// The reference has no multi-GPU path; these kernels serve the expert-parallel
// layer built around its data contract (local_expert_offset, kernel.py:1826).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "kf_internal.cuh"
#include "kf_ptx.cuh"

namespace kf {

namespace {

constexpr int kMaxRanks = 64;
constexpr int kMaxDestPerToken = 8;

struct EpWorkspace {
  size_t dmasks, chunk_base, dest_offset, total;
};

EpWorkspace plan_ep(int T, int world) {
  EpWorkspace w{};
  const size_t nchunk = static_cast<size_t>((T + kChunkTokens - 1) / kChunkTokens);
  size_t off = 0;
  auto take = [&](size_t b) {
    const size_t o = off;
    off = (off + b + 255) / 256 * 256;
    return o;
  };
  w.dmasks = take(nchunk * world * 16);
  w.chunk_base = take(nchunk * world * 4);
  w.dest_offset = take(static_cast<size_t>(world) * 4);
  w.total = off;
  return w;
}

__device__ __forceinline__ int popc4(uint4 m) { return __popc(m.x) + __popc(m.y) + __popc(m.z) + __popc(m.w); }
__device__ __forceinline__ uint32_t word(uint4 m, int w) { return w == 0 ? m.x : w == 1 ? m.y : w == 2 ? m.z : m.w; }

__global__ void __launch_bounds__(256) ep_masks_kernel(const int32_t* __restrict__ topk, int T, int per_rank,
                                                       int world, uint4* __restrict__ dmasks) {
  __shared__ uint32_t m[kMaxRanks * 4];
  const int chunk = blockIdx.x;
  for (int i = threadIdx.x; i < world * 4; i += blockDim.x) m[i] = 0u;
  __syncthreads();
  for (int p = threadIdx.x; p < kChunkTokens * kTopK; p += blockDim.x) {
    const int tl = p >> 3;
    const int t = chunk * kChunkTokens + tl;
    if (t >= T) break;
    const int e = topk[static_cast<size_t>(t) * kTopK + (p & 7)];
    if (e >= 0 && e < kEG) atomicOr(&m[(e / per_rank) * 4 + (tl >> 5)], 1u << (tl & 31));
  }
  __syncthreads();
  for (int d = threadIdx.x; d < world; d += blockDim.x)
    dmasks[static_cast<size_t>(chunk) * world + d] = make_uint4(m[d * 4], m[d * 4 + 1], m[d * 4 + 2], m[d * 4 + 3]);
}

__global__ void __launch_bounds__(kMaxRanks) ep_scan_kernel(const uint4* __restrict__ dmasks, int nchunk, int world,
                                                            int32_t* __restrict__ chunk_base,
                                                            int64_t* __restrict__ send_counts,
                                                            int32_t* __restrict__ dest_offset) {
  __shared__ int32_t tot[kMaxRanks];
  const int d = threadIdx.x;
  if (d < world) {
    int run = 0;
    for (int c = 0; c < nchunk; ++c) {
      chunk_base[static_cast<size_t>(c) * world + d] = run;
      run += popc4(dmasks[static_cast<size_t>(c) * world + d]);
    }
    tot[d] = run;
    send_counts[d] = run;
  }
  __syncthreads();
  if (d == 0) {
    int acc = 0;
    for (int q = 0; q < world; ++q) {
      dest_offset[q] = acc;
      acc += tot[q];
    }
  }
}

__global__ void __launch_bounds__(256) ep_pack_kernel(const int32_t* __restrict__ topk, const float* __restrict__ topk_w,
                                                      const uint8_t* __restrict__ hidden,
                                                      const float* __restrict__ hscale, int T, int per_rank, int world,
                                                      const uint4* __restrict__ dmasks,
                                                      const int32_t* __restrict__ chunk_base,
                                                      const int32_t* __restrict__ dest_offset,
                                                      uint8_t* __restrict__ send_rows, int32_t* __restrict__ pos) {
  __shared__ uint4 m[kMaxRanks];
  __shared__ int32_t base[kMaxRanks];
  __shared__ int2 rows[kChunkTokens * kMaxDestPerToken];
  __shared__ int nrows;
  const int chunk = blockIdx.x;
  for (int d = threadIdx.x; d < world; d += blockDim.x) {
    m[d] = dmasks[static_cast<size_t>(chunk) * world + d];
    base[d] = dest_offset[d] + chunk_base[static_cast<size_t>(chunk) * world + d];
  }
  if (threadIdx.x == 0) nrows = 0;
  __syncthreads();
  for (int q = threadIdx.x; q < kChunkTokens * world; q += blockDim.x) {
    const int tl = q / world, d = q % world;
    const int t = chunk * kChunkTokens + tl;
    if (t >= T) continue;
    const uint4 md = m[d];
    const int w = tl >> 5;
    int slot = -1;
    if ((word(md, w) >> (tl & 31)) & 1u) {
      int r = __popc(word(md, w) & ((1u << (tl & 31)) - 1u));
      for (int k = 0; k < w; ++k) r += __popc(word(md, k));
      slot = base[d] + r;
      rows[atomicAdd(&nrows, 1)] = make_int2(t * kMaxRanks + d, slot);
    }
    pos[static_cast<size_t>(t) * world + d] = slot;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = nrows;
  for (int i = warp; i < n; i += blockDim.x / 32) {
    const int2 r = rows[i];
    const int t = r.x / kMaxRanks, d = r.x % kMaxRanks;
    uint8_t* dst = send_rows + static_cast<size_t>(r.y) * kPackedRowBytes;
    const uint4* src = reinterpret_cast<const uint4*>(hidden + static_cast<size_t>(t) * kH);
    uint4 v[kH / 16 / 32];
#pragma unroll
    for (int j = 0; j < kH / 16 / 32; ++j) v[j] = src[lane + 32 * j];
#pragma unroll
    for (int j = 0; j < kH / 16 / 32; ++j) reinterpret_cast<uint4*>(dst)[lane + 32 * j] = v[j];
    float* dsc = reinterpret_cast<float*>(dst + kH);
    for (int kb = lane; kb < kHB; kb += 32) dsc[kb] = hscale[static_cast<size_t>(kb) * T + t];
    if (lane < kTopK) {
      const int e = topk[static_cast<size_t>(t) * kTopK + lane];
      const bool own = e >= 0 && e < kEG && e / per_rank == d;
      reinterpret_cast<int32_t*>(dst + kH + kHB * 4)[lane] = own ? e : -1;
      reinterpret_cast<float*>(dst + kH + kHB * 4 + kTopK * 4)[lane] =
          own ? topk_w[static_cast<size_t>(t) * kTopK + lane] : 0.f;
    }
  }
}

__global__ void __launch_bounds__(256) ep_combine_kernel(const void* __restrict__ partials, int fp32,
                                                         const int32_t* __restrict__ pos, int world,
                                                         __nv_bfloat16* __restrict__ out) {
  const int t = blockIdx.x;
  int p[kMaxRanks];
  int n = 0;
  for (int d = 0; d < world; ++d) {
    const int v = pos[static_cast<size_t>(t) * world + d];
    if (v >= 0) p[n++] = v;
  }
  for (int c = threadIdx.x; c < kH / 4; c += blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = 0; i < n; ++i) {
      float4 v;
      if (fp32) {
        v = reinterpret_cast<const float4*>(static_cast<const float*>(partials) + static_cast<size_t>(p[i]) * kH)[c];
      } else {
        const uint2 raw = reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(partials) +
                                                         static_cast<size_t>(p[i]) * kH)[c];
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
        v = make_float4(a.x, a.y, b.x, b.y);
      }
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    const __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y);
    const __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z, acc.w);
    uint2 packed;
    packed.x = *reinterpret_cast<const uint32_t*>(&lo);
    packed.y = *reinterpret_cast<const uint32_t*>(&hi);
    reinterpret_cast<uint2*>(out + static_cast<size_t>(t) * kH)[c] = packed;
  }
}

bool valid_world(int world) { return world >= 1 && world <= kMaxRanks && kEG % world == 0; }

}  // namespace
}  // namespace kf

using namespace kf;

extern "C" {

size_t kf_ep_workspace_bytes(int32_t num_tokens, int32_t world) {
  if (num_tokens < 0 || !valid_world(world)) return 0;
  return plan_ep(num_tokens, world).total;
}

int32_t kf_ep_max_send_rows(int32_t num_tokens, int32_t world) {
  if (num_tokens < 0 || !valid_world(world)) return 0;
  return num_tokens * (world < kMaxDestPerToken ? world : kMaxDestPerToken);
}

int kf_ep_dispatch(const int32_t* topk_idx, const float* topk_weight, const void* hidden_states,
                   const float* hidden_states_scale, int32_t num_tokens, int32_t world, void* send_rows,
                   int64_t* send_counts, int32_t* pos, void* workspace, size_t workspace_bytes, void* stream) {
  const int T = num_tokens;
  if (T < 0 || !valid_world(world)) return KF_ERR_INVALID_ARGUMENT;
  if (!send_counts) return KF_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (T == 0) return cudaMemsetAsync(send_counts, 0, sizeof(int64_t) * world, s) == cudaSuccess ? KF_OK : KF_ERR_CUDA;
  if (!topk_idx || !topk_weight || !hidden_states || !hidden_states_scale || !send_rows || !pos || !workspace)
    return KF_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(hidden_states) & 15u) || (reinterpret_cast<uintptr_t>(send_rows) & 15u))
    return KF_ERR_INVALID_ARGUMENT;
  const EpWorkspace w = plan_ep(T, world);
  if (workspace_bytes < w.total) return KF_ERR_WORKSPACE_TOO_SMALL;
  const int nchunk = (T + kChunkTokens - 1) / kChunkTokens;
  uint4* dmasks = ws_ptr<uint4>(workspace, w.dmasks);
  int32_t* chunk_base = ws_ptr<int32_t>(workspace, w.chunk_base);
  int32_t* dest_offset = ws_ptr<int32_t>(workspace, w.dest_offset);
  const int per_rank = kEG / world;
  ep_masks_kernel<<<nchunk, 256, 0, s>>>(topk_idx, T, per_rank, world, dmasks);
  ep_scan_kernel<<<1, kMaxRanks, 0, s>>>(dmasks, nchunk, world, chunk_base, send_counts, dest_offset);
  ep_pack_kernel<<<nchunk, 256, 0, s>>>(topk_idx, topk_weight, static_cast<const uint8_t*>(hidden_states),
                                        hidden_states_scale, T, per_rank, world, dmasks, chunk_base, dest_offset,
                                        static_cast<uint8_t*>(send_rows), pos);
  return cudaGetLastError() == cudaSuccess ? KF_OK : KF_ERR_CUDA;
}

int kf_ep_combine(const void* partials, int32_t partials_fp32, const int32_t* pos, int32_t num_tokens,
                  int32_t world, void* output, void* stream) {
  if (num_tokens < 0 || !valid_world(world)) return KF_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return KF_OK;
  if (!pos || !output) return KF_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(output) & 15u) || (partials && (reinterpret_cast<uintptr_t>(partials) & 15u)))
    return KF_ERR_INVALID_ARGUMENT;
  ep_combine_kernel<<<num_tokens, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      partials, partials_fp32 ? 1 : 0, pos, world, static_cast<__nv_bfloat16*>(output));
  return cudaGetLastError() == cudaSuccess ? KF_OK : KF_ERR_CUDA;
}

}  // extern "C"
