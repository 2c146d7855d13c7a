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
// The rows and partials travel either through NCCL all-to-alls (kf_ep_dispatch
// packs into a local send buffer) or by plain stores into the other ranks'
// symmetric buffers: kf_ep_plan_p2p publishes this rank's per-destination
// counts into every rank's count matrix, kf_ep_pack_p2p stores each packed row
// (optionally quantising bf16 rows on the way) straight into its destination's
// receive area, the expert stage's reduce (or kf_ep_return_p2p) stores each
// partial back into its source's return area, and kf_ep_barrier separates the
// phases with a bounded wait.
//
// The reference has no multi-GPU path; these kernels serve the expert-parallel
// layer built around its data contract (local_expert_offset, kernel.py:1826).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "kf_internal.cuh"
#include "kf_ptx.cuh"
#include "kf_quant.cuh"

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

// peer_counts (peer-to-peer mode only): device array of `world` pointers to each
// rank's [world][world] count matrix; this rank's row `rank` is written into all
// of them (plain stores over NVLink, made visible system-wide before the kernel
// ends).
__global__ void __launch_bounds__(kMaxRanks) ep_scan_kernel(const uint4* __restrict__ dmasks, int nchunk, int world,
                                                            int32_t* __restrict__ chunk_base,
                                                            int64_t* __restrict__ send_counts,
                                                            int32_t* __restrict__ dest_offset,
                                                            int32_t* const* __restrict__ peer_counts, int rank) {
  __shared__ int32_t tot[kMaxRanks];
  const int d = threadIdx.x;
  if (d < world) {
    int run = 0;
    for (int c = 0; c < nchunk; ++c) {
      chunk_base[static_cast<size_t>(c) * world + d] = run;
      run += popc4(dmasks[static_cast<size_t>(c) * world + d]);
    }
    tot[d] = run;
    if (send_counts) send_counts[d] = run;
    if (peer_counts) {
      for (int q = 0; q < world; ++q) peer_counts[q][rank * world + d] = run;
      __threadfence_system();
    }
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

// kBf16In: `hidden` holds bf16 rows [T][7168] (hscale unused) and each packed
// row is quantised on the way out (the upstream FP8 quantisation fused into the
// dispatch); otherwise `hidden` holds the e4m3 rows and hscale their scales.
template <bool kBf16In>
__global__ void __launch_bounds__(256) ep_pack_kernel(const int32_t* __restrict__ topk, const float* __restrict__ topk_w,
                                                      const uint8_t* __restrict__ hidden,
                                                      const float* __restrict__ hscale, int T, int per_rank, int world,
                                                      const uint4* __restrict__ dmasks,
                                                      const int32_t* __restrict__ chunk_base,
                                                      const int32_t* __restrict__ dest_offset,
                                                      uint8_t* __restrict__ send_rows, int32_t* __restrict__ pos,
                                                      uint8_t* const* __restrict__ peer_recv,
                                                      const int32_t* __restrict__ counts, int rank, int recv_cap,
                                                      int* __restrict__ status) {
  __shared__ uint4 m[kMaxRanks];
  __shared__ int32_t base[kMaxRanks];
  __shared__ int32_t pbase[kMaxRanks];
  __shared__ int2 rows[kChunkTokens * kMaxDestPerToken];
  __shared__ int nrows;
  const int chunk = blockIdx.x;
  for (int d = threadIdx.x; d < world; d += blockDim.x) {
    m[d] = dmasks[static_cast<size_t>(chunk) * world + d];
    const int cb = chunk_base[static_cast<size_t>(chunk) * world + d];
    base[d] = dest_offset[d] + cb;
    if (peer_recv) {
      // rank d's receive buffer holds the rows of sources 0, 1, ... in order
      int off = 0;
      for (int s = 0; s < rank; ++s) off += counts[s * world + d];
      pbase[d] = off + cb;
    }
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
      rows[atomicAdd(&nrows, 1)] = make_int2(t * kMaxRanks + d, peer_recv ? pbase[d] + r : slot);
    }
    pos[static_cast<size_t>(t) * world + d] = slot;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = nrows;
  for (int i = warp; i < n; i += blockDim.x / 32) {
    const int2 r = rows[i];
    const int t = r.x / kMaxRanks, d = r.x % kMaxRanks;
    if (peer_recv && r.y >= recv_cap) {  // the ranks disagree on the token count: drop, report
      if (lane == 0) atomicOr(status, KF_STATUS_SLOT_OVERFLOW);
      continue;
    }
    uint8_t* dst = (peer_recv ? peer_recv[d] : send_rows) + static_cast<size_t>(r.y) * kPackedRowBytes;
    float* dsc = reinterpret_cast<float*>(dst + kH);
    if constexpr (kBf16In) {
      // two 128-column blocks per round: lanes 0-15 the even one, 16-31 the odd one
      const uint4* src = reinterpret_cast<const uint4*>(hidden + static_cast<size_t>(t) * kH * 2);
#pragma unroll 4
      for (int i = 0; i < kHB / 2; ++i) {
        const int kb = 2 * i + (lane >> 4);
        float sc;
        const uint2 q = quantize_block16(src[kb * 16 + (lane & 15)], sc);
        reinterpret_cast<uint2*>(dst + kb * kBlk)[lane & 15] = q;
        if ((lane & 15) == 0) dsc[kb] = sc;
      }
    } else {
      const uint4* src = reinterpret_cast<const uint4*>(hidden + static_cast<size_t>(t) * kH);
      uint4 v[kH / 16 / 32];
#pragma unroll
      for (int j = 0; j < kH / 16 / 32; ++j) v[j] = src[lane + 32 * j];
#pragma unroll
      for (int j = 0; j < kH / 16 / 32; ++j) reinterpret_cast<uint4*>(dst)[lane + 32 * j] = v[j];
      for (int kb = lane; kb < kHB; kb += 32) dsc[kb] = hscale[static_cast<size_t>(kb) * T + t];
    }
    if (lane < kTopK) {
      const int e = topk[static_cast<size_t>(t) * kTopK + lane];
      const bool own = e >= 0 && e < kEG && e / per_rank == d;
      reinterpret_cast<int32_t*>(dst + kH + kHB * 4)[lane] = own ? e : -1;
      reinterpret_cast<float*>(dst + kH + kHB * 4 + kTopK * 4)[lane] =
          own ? topk_w[static_cast<size_t>(t) * kTopK + lane] : 0.f;
    }
  }
  if (peer_recv) __threadfence_system();
}

// Peer-to-peer return of the expert partials: received row r came from the
// source s whose block holds it (sources in rank order) and is that source's
// j-th row for this rank; it goes to row (s's rows for ranks below this one) + j
// of s's return buffer, i.e. back to the position the row had in s's send order.
// One warp per row, 16-byte stores over NVLink.
__global__ void __launch_bounds__(256) ep_return_kernel(const __nv_bfloat16* __restrict__ partials, int R, int world,
                                                        int rank, const int32_t* __restrict__ counts,
                                                        __nv_bfloat16* const* __restrict__ peer_back) {
  __shared__ int32_t recv_off[kMaxRanks + 1];
  __shared__ int32_t send_off[kMaxRanks];
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int s = 0; s < world; ++s) {
      recv_off[s] = acc;
      acc += counts[s * world + rank];
      int so = 0;
      for (int d = 0; d < rank; ++d) so += counts[s * world + d];
      send_off[s] = so;
    }
    recv_off[world] = acc;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  // rows past the received total have no place in any source's send order
  const int rows = R < recv_off[world] ? R : recv_off[world];
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    int s = 0;
    while (s + 1 < world && recv_off[s + 1] <= r) ++s;
    const size_t dst_row = static_cast<size_t>(send_off[s]) + (r - recv_off[s]);
    const uint4* src = reinterpret_cast<const uint4*>(partials + static_cast<size_t>(r) * kH);
    uint4* dst = reinterpret_cast<uint4*>(peer_back[s] + dst_row * kH);
#pragma unroll 4
    for (int i = lane; i < kH * 2 / 16; i += 32) dst[i] = src[i];
  }
  __threadfence_system();
}

// Barrier over the ranks' symmetric flag arrays: thread q stores `epoch` into
// slot `rank` of rank q's flags (after a system-scope fence, so every earlier
// peer store of this stream is visible first), then waits until slot q of this
// rank's flags reaches `epoch`.  Bounded: after kWaitCycles it records
// KF_STATUS_TIMEOUT_PEER and returns.  Epochs grow by one per barrier.
__global__ void __launch_bounds__(kMaxRanks) ep_barrier_kernel(int32_t* const* __restrict__ peer_flags,
                                                               const int32_t* __restrict__ my_flags, int rank,
                                                               int world, int epoch, int* __restrict__ status) {
  const int q = threadIdx.x;
  if (q >= world) return;
  __threadfence_system();
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(peer_flags[q] + rank), "r"(epoch) : "memory");
  const long long t0 = clock64();
  while (true) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(my_flags + q) : "memory");
    if (v - epoch >= 0) break;
    if (clock64() - t0 > kWaitCycles) {
      atomicOr(status, KF_STATUS_TIMEOUT_PEER);
      break;
    }
  }
  __threadfence_system();
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
  if (!valid_tokens(num_tokens) || !valid_world(world)) return 0;
  return plan_ep(num_tokens, world).total;
}

int32_t kf_ep_max_send_rows(int32_t num_tokens, int32_t world) {
  if (!valid_tokens(num_tokens) || !valid_world(world)) return 0;
  return num_tokens * (world < kMaxDestPerToken ? world : kMaxDestPerToken);
}

int kf_ep_dispatch(const int32_t* topk_idx, const float* topk_weight, const void* hidden_states,
                   const float* hidden_states_scale, int32_t num_tokens, int32_t world, void* send_rows,
                   int64_t* send_counts, int32_t* pos, void* workspace, size_t workspace_bytes, void* stream) {
  const int T = num_tokens;
  if (!valid_tokens(T) || !valid_world(world)) return KF_ERR_INVALID_ARGUMENT;
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
  ep_scan_kernel<<<1, kMaxRanks, 0, s>>>(dmasks, nchunk, world, chunk_base, send_counts, dest_offset, nullptr, 0);
  ep_pack_kernel<false><<<nchunk, 256, 0, s>>>(topk_idx, topk_weight, static_cast<const uint8_t*>(hidden_states),
                                        hidden_states_scale, T, per_rank, world, dmasks, chunk_base, dest_offset,
                                        static_cast<uint8_t*>(send_rows), pos, nullptr, nullptr, 0, 0, nullptr);
  return cudaGetLastError() == cudaSuccess ? KF_OK : KF_ERR_CUDA;
}

int kf_ep_plan_p2p(const int32_t* topk_idx, int32_t num_tokens, int32_t world, int32_t rank,
                   int32_t* const* peer_counts, void* workspace, size_t workspace_bytes, void* stream) {
  const int T = num_tokens;
  if (!valid_tokens(T) || !valid_world(world) || rank < 0 || rank >= world || !peer_counts || !workspace)
    return KF_ERR_INVALID_ARGUMENT;
  if (T > 0 && !topk_idx) return KF_ERR_INVALID_ARGUMENT;
  const EpWorkspace w = plan_ep(T, world);
  if (workspace_bytes < w.total) return KF_ERR_WORKSPACE_TOO_SMALL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int nchunk = (T + kChunkTokens - 1) / kChunkTokens;
  uint4* dmasks = ws_ptr<uint4>(workspace, w.dmasks);
  if (nchunk > 0) ep_masks_kernel<<<nchunk, 256, 0, s>>>(topk_idx, T, kEG / world, world, dmasks);
  // with no tokens the scan still publishes a row of zeros: the peers wait for it
  ep_scan_kernel<<<1, kMaxRanks, 0, s>>>(dmasks, nchunk, world, ws_ptr<int32_t>(workspace, w.chunk_base), nullptr,
                                         ws_ptr<int32_t>(workspace, w.dest_offset), peer_counts, rank);
  return cudaGetLastError() == cudaSuccess ? KF_OK : KF_ERR_CUDA;
}

int kf_ep_pack_p2p(const int32_t* topk_idx, const float* topk_weight, const void* hidden_states,
                   const float* hidden_states_scale, int32_t num_tokens, int32_t world, int32_t rank,
                   const int32_t* counts, uint8_t* const* peer_recv, int32_t recv_capacity, int32_t* pos,
                   int32_t* status, void* workspace, size_t workspace_bytes, void* stream) {
  const int T = num_tokens;
  if (!valid_tokens(T) || !valid_world(world) || rank < 0 || rank >= world) return KF_ERR_INVALID_ARGUMENT;
  if (T == 0) return KF_OK;
  if (!topk_idx || !topk_weight || !hidden_states || !counts || !peer_recv || !pos || !status || !workspace ||
      recv_capacity < 0)
    return KF_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(hidden_states) & 15u) return KF_ERR_INVALID_ARGUMENT;
  const EpWorkspace w = plan_ep(T, world);
  if (workspace_bytes < w.total) return KF_ERR_WORKSPACE_TOO_SMALL;
  const int nchunk = (T + kChunkTokens - 1) / kChunkTokens;
  const int per_rank = kEG / world;
  if (hidden_states_scale) {
    ep_pack_kernel<false><<<nchunk, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        topk_idx, topk_weight, static_cast<const uint8_t*>(hidden_states), hidden_states_scale, T, per_rank, world,
        ws_ptr<uint4>(workspace, w.dmasks), ws_ptr<int32_t>(workspace, w.chunk_base),
        ws_ptr<int32_t>(workspace, w.dest_offset), nullptr, pos, peer_recv, counts, rank, recv_capacity, status);
  } else {
    ep_pack_kernel<true><<<nchunk, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        topk_idx, topk_weight, static_cast<const uint8_t*>(hidden_states), nullptr, T, per_rank, world,
        ws_ptr<uint4>(workspace, w.dmasks), ws_ptr<int32_t>(workspace, w.chunk_base),
        ws_ptr<int32_t>(workspace, w.dest_offset), nullptr, pos, peer_recv, counts, rank, recv_capacity, status);
  }
  return cudaGetLastError() == cudaSuccess ? KF_OK : KF_ERR_CUDA;
}

int kf_ep_return_p2p(const void* partials, int32_t num_rows, int32_t world, int32_t rank, const int32_t* counts,
                     void* const* peer_back, void* stream) {
  if (!valid_tokens(num_rows) || !valid_world(world) || rank < 0 || rank >= world) return KF_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return KF_OK;
  if (!partials || !counts || !peer_back || (reinterpret_cast<uintptr_t>(partials) & 15u))
    return KF_ERR_INVALID_ARGUMENT;
  const int blocks = (num_rows + 7) / 8 < 4 * 148 ? (num_rows + 7) / 8 : 4 * 148;
  ep_return_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(partials), num_rows, world, rank, counts,
      reinterpret_cast<__nv_bfloat16* const*>(peer_back));
  return cudaGetLastError() == cudaSuccess ? KF_OK : KF_ERR_CUDA;
}

int kf_ep_barrier(int32_t* const* peer_flags, const int32_t* my_flags, int32_t rank, int32_t world, int32_t epoch,
                  int32_t* status, void* stream) {
  if (!valid_world(world) || rank < 0 || rank >= world || !peer_flags || !my_flags || !status)
    return KF_ERR_INVALID_ARGUMENT;
  ep_barrier_kernel<<<1, kMaxRanks, 0, static_cast<cudaStream_t>(stream)>>>(peer_flags, my_flags, rank, world, epoch,
                                                                           status);
  return cudaGetLastError() == cudaSuccess ? KF_OK : KF_ERR_CUDA;
}

int kf_ep_combine(const void* partials, int32_t partials_fp32, const int32_t* pos, int32_t num_tokens,
                  int32_t world, void* output, void* stream) {
  if (!valid_tokens(num_tokens) || !valid_world(world)) return KF_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return KF_OK;
  if (!pos || !output) return KF_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(output) & 15u) || (partials && (reinterpret_cast<uintptr_t>(partials) & 15u)))
    return KF_ERR_INVALID_ARGUMENT;
  ep_combine_kernel<<<num_tokens, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      partials, partials_fp32 ? 1 : 0, pos, world, static_cast<__nv_bfloat16*>(output));
  return cudaGetLastError() == cudaSuccess ? KF_OK : KF_ERR_CUDA;
}

}  // extern "C"
