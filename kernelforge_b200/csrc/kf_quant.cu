// FP8 block quantisation of the layer's input rows (the producer of
// hidden_states / hidden_states_scale): per row and 128 columns,
// scale = absmax / 448 (1 for an all-zero block) and q = e4m3(x / scale),
// rounded to nearest even -- the reference's _quantize_fp8_block_rows
// (solution/triton/kernel.py:126-141) on bf16 input rows.
//
// HBM-bound: each row is read once (2 bytes per element) and written once
// (1 byte + 4 bytes per 128).  A warp quantises two blocks at a time (16 lanes
// per block, 8 bf16 = 16 bytes per lane, absmax by shuffles within the 16
// lanes) and four such pairs per launch slot, their loads issued together.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "kf_internal.cuh"
#include "kf_quant.cuh"

namespace kf {
namespace {

constexpr int kQuantThreads = 256;
constexpr int kPairsPerWarp = 4;  // block pairs per warp: four 16-byte loads in flight per lane

__device__ __forceinline__ void quantize_pair(uint4 raw, int lane, uint8_t* __restrict__ q, float* __restrict__ scale,
                                              size_t base, size_t scale_idx) {
  float s;
  *reinterpret_cast<uint2*>(q + base) = quantize_block16(raw, s);
  if ((lane & 15) == 0) scale[scale_idx] = s;
}

// Work item = a pair of 128-column blocks of one row (28 per row); each warp
// takes kPairsPerWarp consecutive items, loading all of them before any math.
__global__ void __launch_bounds__(kQuantThreads) quantize_rows_kernel(const __nv_bfloat16* __restrict__ x, int T,
                                                                      uint8_t* __restrict__ q,
                                                                      float* __restrict__ scale) {
  const int lane = threadIdx.x & 31;
  const long long warp = (static_cast<long long>(blockIdx.x) * kQuantThreads + threadIdx.x) >> 5;
  const long long items = static_cast<long long>(T) * (kHB / 2);
  const long long first = warp * kPairsPerWarp;
  if (first >= items) return;  // warp-uniform
  uint4 raw[kPairsPerWarp];
  size_t base[kPairsPerWarp], sidx[kPairsPerWarp];
#pragma unroll
  for (int p = 0; p < kPairsPerWarp; ++p) {
    const long long it = first + p < items ? first + p : items - 1;  // tail: repeat the last item (same result)
    const int t = static_cast<int>(it / (kHB / 2));
    const int kb = static_cast<int>(it % (kHB / 2)) * 2 + (lane >> 4);
    base[p] = static_cast<size_t>(t) * kH + static_cast<size_t>(kb) * kBlk + (lane & 15) * 8;
    sidx[p] = static_cast<size_t>(kb) * T + t;
    raw[p] = __ldg(reinterpret_cast<const uint4*>(x + base[p]));
  }
#pragma unroll
  for (int p = 0; p < kPairsPerWarp; ++p) quantize_pair(raw[p], lane, q, scale, base[p], sidx[p]);
}

}  // namespace
}  // namespace kf

extern "C" int kf_quantize_hidden(const void* x, int32_t num_tokens, void* out, float* out_scale, void* stream) {
  if (!kf::valid_tokens(num_tokens) || (num_tokens > 0 && (!x || !out || !out_scale))) return KF_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u) return KF_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return KF_OK;
  const long long warps = (static_cast<long long>(num_tokens) * (kf::kHB / 2) + kf::kPairsPerWarp - 1) / kf::kPairsPerWarp;
  const long long threads = warps * 32;
  const unsigned grid = static_cast<unsigned>((threads + kf::kQuantThreads - 1) / kf::kQuantThreads);
  kf::quantize_rows_kernel<<<grid, kf::kQuantThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), num_tokens, static_cast<uint8_t*>(out), out_scale);
  return cudaGetLastError() == cudaSuccess ? KF_OK : KF_ERR_CUDA;
}
