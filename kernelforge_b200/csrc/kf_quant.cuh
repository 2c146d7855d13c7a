// FP8 block quantisation of one 128-element block by 16 lanes (shared by the
// standalone quantiser and the expert-parallel pack that quantises bf16 rows on
// the way out): the reference's _quantize_fp8_block_rows
// (solution/triton/kernel.py:126-141) for one block.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp8.h>

namespace kf {

// `raw` = this lane's 8 bf16 of the block (lane & 15 = their 16-byte slot); the
// 16 lanes of a half-warp quantise one block together (the absmax is reduced
// by shuffles among them), so both half-warps must call this at the same time.
// Returns the 8 e4m3 codes (round to nearest even, saturating) and sets
// `scale` = absmax / 448 (1 for an all-zero block).
__device__ __forceinline__ uint2 quantize_block16(uint4 raw, float& scale) {
  const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
  float v[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h2[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int off = 8; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  const float s = amax > 0.f ? __fdiv_rn(amax, 448.0f) : 1.0f;
  uint32_t w[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(
        make_float2(__fdiv_rn(v[4 * i], s), __fdiv_rn(v[4 * i + 1], s)), __NV_SATFINITE, __NV_E4M3);
    const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
        make_float2(__fdiv_rn(v[4 * i + 2], s), __fdiv_rn(v[4 * i + 3], s)), __NV_SATFINITE, __NV_E4M3);
    w[i] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
  }
  scale = s;
  return make_uint2(w[0], w[1]);
}

}  // namespace kf
