// FP8 e4m3 helpers of the GEMM1 epilogues: the two-term (hi + lo) encoding of
// the SwiGLU output that GEMM2 consumes.  Shared by GEMM1's own epilogue and the
// split-K finish, so both write bit-identical intermediates.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

namespace kf {

// Four floats -> four e4m3 codes (round to nearest even, saturating), byte i = value i.
__device__ __forceinline__ uint32_t pack_fp8x4(float a, float b, float c, float d) {
  const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

__device__ __forceinline__ float2 fp8x2_to_float2(__nv_fp8x2_storage_t v) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(v, __NV_E4M3);
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// hi = e4m3(x), lo = e4m3(x - hi) for 4 values; returns {hi word, lo word}.
__device__ __forceinline__ uint2 encode_hilo4(float x0, float x1, float x2, float x3) {
  const __nv_fp8x2_storage_t h01 = __nv_cvt_float2_to_fp8x2(make_float2(x0, x1), __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t h23 = __nv_cvt_float2_to_fp8x2(make_float2(x2, x3), __NV_SATFINITE, __NV_E4M3);
  const float2 f01 = fp8x2_to_float2(h01);
  const float2 f23 = fp8x2_to_float2(h23);
  const uint32_t hi = static_cast<uint32_t>(h01) | (static_cast<uint32_t>(h23) << 16);
  const uint32_t lo = pack_fp8x4(x0 - f01.x, x1 - f01.y, x2 - f23.x, x3 - f23.y);
  return make_uint2(hi, lo);
}

}  // namespace kf
