// Grouped FP8 block-scale GEMMs of the MoE layer on the 5th-generation tensor
// cores (tcgen05 + tensor memory), fed by TMA.
//
// Both kernels are persistent (one CTA per SM) and warp-specialised:
//   warp 0        TMA producer: operand tiles + per-chunk scales into a smem ring
//   warp 1        MMA issuer: one thread issues tcgen05.mma into a TMEM partial
//                 buffer (two buffers, so the tensor core runs one K-chunk ahead)
//   warps 2-3     idle (they only hand their registers to the epilogue)
//   warps 4-11    promotion + epilogue: read each chunk's partial from TMEM,
//                 apply the fp32 block scales (a_scale[row] * w_scale), accumulate
//                 in registers, and run the fused epilogue at the end of a tile.
//
// The block scales are arbitrary fp32 (not power-of-two), so they cannot be
// folded into a block-scaled MMA; each 128-wide K chunk (one scale block)
// accumulates in its own TMEM partial and is promoted in fp32 -- the software
// equivalent of the reference's per-K-block "tl.dot(...) * a_scale * w_scale"
// (solution/triton/kernel.py:311-318 and :599-607).
//
// Work unit = (row tile of 128 permuted rows of one expert, column block).
// Units are walked round-robin by the persistent CTAs; consecutive units share
// a row tile so its A tile stays hot in L2, and all tiles of one expert run in
// the same wave so its weight tiles are read from HBM about once.
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "kf_internal.cuh"
#include "kf_ptx.cuh"

namespace kf {

namespace {

constexpr int kThreads = 384;  // 12 warps
constexpr int kEpiWarps = 8;

// ------------------------------------------------------------------ GEMM1 --
// X = A[rows, 7168] . W13[e]^T, N-block = 128 up columns + the matching 128 gate
// columns (one MMA with N = 256).  Epilogue: silu(gate) * up, then a two-term
// FP8 encoding (hi + lo residual) sharing one fp32 scale per 128 columns.
constexpr int G1_S = 4;
constexpr int G1_A = kBlk * kBlk;        // 16 KB
constexpr int G1_B = 2 * kBlk * kBlk;    // 32 KB: up rows then gate rows
constexpr int G1_OFF_B = G1_S * G1_A;
constexpr int G1_OFF_AS = G1_OFF_B + G1_S * G1_B;
constexpr int G1_OFF_WS = G1_OFF_AS + G1_S * kBlk * 4;
constexpr int G1_OFF_BAR = G1_OFF_WS + G1_S * 8;
constexpr int G1_NBAR = 2 * G1_S + 6;
constexpr int G1_OFF_MISC = G1_OFF_BAR + G1_NBAR * 8;
constexpr int G1_OFF_XCH = G1_OFF_MISC + 16;
constexpr int G1_SMEM = G1_OFF_XCH + 2 * 2 * kBlk * 4 + 1024;
constexpr uint32_t G1_TX = 3 * 16384 + kBlk * 4;

// ------------------------------------------------------------------ GEMM2 --
// Y = C[rows, 2048] . W2[e]^T with C = s * (C_hi + C_lo), N-block = 256 output
// columns.  Each K step issues two MMAs (hi and lo) into the same accumulator.
// Epilogue: multiply by the pair's routing weight, store fp32 rows.
constexpr int G2_S = 3;
constexpr int G2_A = kBlk * kBlk;        // 16 KB each for hi and lo
constexpr int G2_B = 2 * kBlk * kBlk;    // 32 KB: 256 rows of W2
constexpr int G2_OFF_ALO = G2_S * G2_A;
constexpr int G2_OFF_B = 2 * G2_S * G2_A;
constexpr int G2_OFF_AS = G2_OFF_B + G2_S * G2_B;
constexpr int G2_OFF_WS = G2_OFF_AS + G2_S * kBlk * 4;
constexpr int G2_OFF_BAR = G2_OFF_WS + G2_S * 8;
constexpr int G2_NBAR = 2 * G2_S + 4;
constexpr int G2_OFF_MISC = G2_OFF_BAR + G2_NBAR * 8;
constexpr int G2_SMEM = G2_OFF_MISC + 16 + 1024;
constexpr uint32_t G2_TX = 2 * 16384 + 32768 + kBlk * 4;
constexpr int kG2NB = kH / 256;  // 28 column blocks of 256

static_assert(G1_SMEM <= 232448, "GEMM1 shared memory");
static_assert(G2_SMEM <= 232448, "GEMM2 shared memory");
// Register split (setmaxnreg): warpgroup 0 drops to 40, warpgroups 1-2 rise to
// 232: 128*40 + 256*232 = 64512 = 384 threads * 168, the launch allocation
// (__launch_bounds__(384, 1); the build checks ptxas reports 168).
constexpr int kRegsLow = 40;
constexpr int kRegsHigh = 232;
static_assert(128 * kRegsLow + 256 * kRegsHigh <= 384 * 168, "register split exceeds the launch allocation");

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023));
}

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

__global__ void __launch_bounds__(kThreads, 1)
    gemm1_swiglu_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w,
                        const Gemm1Args g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + G1_OFF_B;
  float* as_ring = reinterpret_cast<float*>(smem + G1_OFF_AS);
  float2* ws_ring = reinterpret_cast<float2*>(smem + G1_OFF_WS);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G1_OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = bars + G1_S;
  uint64_t* pfull = bars + 2 * G1_S;
  uint64_t* pempty = pfull + 2;
  uint64_t* xbar = pempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + G1_OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + G1_OFF_MISC + 4);
  float* xch = reinterpret_cast<float*>(smem + G1_OFF_XCH);

  const int num_units = g.meta->num_tiles * kIB;
  if (static_cast<int>(blockIdx.x) >= num_units) return;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < G1_S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + kEpiWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], kEpiWarps);
      mbar_init(&xbar[b], kEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_w);
  }
  if (warp == 1) tmem_alloc(tmem_holder, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp < 4) {
    setmaxnreg_dec<kRegsLow>();
    if (warp == 0) {
      // ------------------------------------------------------ TMA producer --
      int stage = 0;
      uint32_t ph = 0, armed = 0, armed_par = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        const int tile = u / kIB, nb = u % kIB;
        const int e = g.tile_expert[tile];
        const int row0 = g.tile_row0[tile];
        const float* wsu = g.w13_scale + (static_cast<size_t>(e) * 32 + nb) * kHB;
        const float* wsg = g.w13_scale + (static_cast<size_t>(e) * 32 + kIB + nb) * kHB;
        const float su0 = wsu[lane], sg0 = wsg[lane];
        const float su1 = (lane + 32 < kHB) ? wsu[lane + 32] : 0.f;
        const float sg1 = (lane + 32 < kHB) ? wsg[lane + 32] : 0.f;
        const int wrow_up = e * (2 * kI) + nb * kBlk;
        for (int kb = 0; kb < kHB; ++kb) {
          const float su = __shfl_sync(0xffffffffu, kb < 32 ? su0 : su1, kb & 31);
          const float sg = __shfl_sync(0xffffffffu, kb < 32 ? sg0 : sg1, kb & 31);
          int good = 1;
          if (lane == 0) {
            good = mbar_wait_abort(&empty[stage], ph ^ 1u, abort_flag, g.status, KF_STATUS_TIMEOUT_PRODUCER);
            if (good) {
              ws_ring[stage] = make_float2(su, sg);
              mbar_arrive_expect_tx(&full[stage], G1_TX);
              tma_load_2d(sA + stage * G1_A, &tm_a, kb * kBlk, row0, &full[stage]);
              tma_load_2d(sB + stage * G1_B, &tm_w, kb * kBlk, wrow_up, &full[stage]);
              tma_load_2d(sB + stage * G1_B + G1_A, &tm_w, kb * kBlk, wrow_up + kI, &full[stage]);
              bulk_load(as_ring + stage * kBlk, g.a_scale + static_cast<size_t>(kb) * g.p_cap + row0, kBlk * 4,
                        &full[stage]);
              armed |= 1u << stage;
              armed_par = ph ? (armed_par | (1u << stage)) : (armed_par & ~(1u << stage));
            }
          }
          good = __shfl_sync(0xffffffffu, good, 0);
          if (!good) {
            ok = false;
            break;
          }
          if (++stage == G1_S) {
            stage = 0;
            ph ^= 1u;
          }
        }
      }
      if (lane == 0) {  // let every TMA write that was issued land before the CTA can exit
        int no_abort = 0;
        for (int s = 0; s < G1_S; ++s)
          if ((armed >> s) & 1u)
            mbar_wait_abort(&full[s], (armed_par >> s) & 1u, &no_abort, g.status, KF_STATUS_TIMEOUT_PRODUCER);
      }
    } else if (warp == 1) {
      // -------------------------------------------------------- MMA issuer --
      if (lane == 0) {
        constexpr uint32_t idesc = idesc_e4m3_f32(128, 256);
        int stage = 0, pb = 0;
        uint32_t ph = 0, pph = 0;
        bool ok = true, committed = false;
        int last_pb = 0;
        uint32_t last_pph = 0;
        for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
          for (int kb = 0; kb < kHB; ++kb) {
            if (!mbar_wait_abort(&pempty[pb], pph ^ 1u, abort_flag, g.status, KF_STATUS_TIMEOUT_MMA) ||
                !mbar_wait_abort(&full[stage], ph, abort_flag, g.status, KF_STATUS_TIMEOUT_MMA)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_u32(sA + stage * G1_A);
            const uint32_t b0 = smem_u32(sB + stage * G1_B);
            const uint32_t d = tmem + static_cast<uint32_t>(pb * 256);
#pragma unroll
            for (int k = 0; k < kBlk / 32; ++k)
              mma_f8(d, sw128_kmajor_desc(a0 + k * 32), sw128_kmajor_desc(b0 + k * 32), idesc, k > 0 ? 1u : 0u);
            mma_commit(&empty[stage]);
            mma_commit(&pfull[pb]);
            committed = true;
            last_pb = pb;
            last_pph = pph;
            if (++stage == G1_S) {
              stage = 0;
              ph ^= 1u;
            }
            if (++pb == 2) {
              pb = 0;
              pph ^= 1u;
            }
          }
        }
        if (committed) {  // the tensor core must be idle before TMEM is released
          int no_abort = 0;
          mbar_wait_abort(&pfull[last_pb], last_pph, &no_abort, g.status, KF_STATUS_TIMEOUT_MMA);
        }
      }
      __syncwarp();
    }
  } else {
    setmaxnreg_inc<kRegsHigh>();
    // ------------------------------------------------ promotion + epilogue --
    const int pw = warp - 4;
    const int h = pw >> 2;        // column half: up/gate columns [64h, 64h+64) of the block
    const int q = warp & 3;       // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    int stage = 0, pb = 0, it = 0;
    uint32_t ph = 0, pph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++it) {
      const int tile = u / kIB, nb = u % kIB;
      const int row0 = g.tile_row0[tile];
      const int nrows = g.tile_rows[tile];
      float acc_u[64], acc_g[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        acc_u[j] = 0.f;
        acc_g[j] = 0.f;
      }
      for (int kb = 0; kb < kHB; ++kb) {
        if (!mbar_wait_abort(&full[stage], ph, abort_flag, g.status, KF_STATUS_TIMEOUT_EPILOGUE)) {
          ok = false;
          break;
        }
        const float a_s = as_ring[stage * kBlk + row];
        const float2 ws = ws_ring[stage];
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (!mbar_wait_abort(&pfull[pb], pph, abort_flag, g.status, KF_STATUS_TIMEOUT_EPILOGUE)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem + lane_base + static_cast<uint32_t>(pb * 256 + h * 64);
        float v[64];
        tmem_ld64_sync(taddr, v);
        const float su = a_s * ws.x;
#pragma unroll
        for (int j = 0; j < 64; ++j) acc_u[j] = fmaf(v[j], su, acc_u[j]);
        tmem_ld64_sync(taddr + 128, v);
        const float sg = a_s * ws.y;
#pragma unroll
        for (int j = 0; j < 64; ++j) acc_g[j] = fmaf(v[j], sg, acc_g[j]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pempty[pb]);
        if (++stage == G1_S) {
          stage = 0;
          ph ^= 1u;
        }
        if (++pb == 2) {
          pb = 0;
          pph ^= 1u;
        }
      }
      if (!ok) break;
      // SwiGLU: silu(X2) * X1 with X1 = up (W13 rows [0, I)), X2 = gate (rows [I, 2I))
      float amax = 0.f;
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        const float gt = acc_g[j];
        const float hv = (gt / (1.0f + expf(-gt))) * acc_u[j];
        acc_u[j] = hv;
        amax = fmaxf(amax, fabsf(hv));
      }
      const int xb = it & 1;
      xch[(xb * 2 + h) * kBlk + row] = amax;
      __syncwarp();
      if (lane == 0) mbar_arrive(&xbar[xb]);
      if (!mbar_wait_abort(&xbar[xb], static_cast<uint32_t>(it >> 1) & 1u, abort_flag, g.status,
                           KF_STATUS_TIMEOUT_EPILOGUE)) {
        ok = false;
        break;
      }
      amax = fmaxf(xch[(xb * 2) * kBlk + row], xch[(xb * 2 + 1) * kBlk + row]);
      const float inv = amax > 0.f ? 448.0f / amax : 1.0f;
      const float scale = amax > 0.f ? amax / 448.0f : 1.0f;
      if (row < nrows) {
        const size_t off = static_cast<size_t>(row0 + row) * kI + nb * kBlk + h * 64;
        uint4* dh = reinterpret_cast<uint4*>(g.c_hi + off);
        uint4* dl = reinterpret_cast<uint4*>(g.c_lo + off);
#pragma unroll
        for (int j = 0; j < 64; j += 16) {
          const uint2 w0 = encode_hilo4(acc_u[j] * inv, acc_u[j + 1] * inv, acc_u[j + 2] * inv, acc_u[j + 3] * inv);
          const uint2 w1 =
              encode_hilo4(acc_u[j + 4] * inv, acc_u[j + 5] * inv, acc_u[j + 6] * inv, acc_u[j + 7] * inv);
          const uint2 w2 =
              encode_hilo4(acc_u[j + 8] * inv, acc_u[j + 9] * inv, acc_u[j + 10] * inv, acc_u[j + 11] * inv);
          const uint2 w3 =
              encode_hilo4(acc_u[j + 12] * inv, acc_u[j + 13] * inv, acc_u[j + 14] * inv, acc_u[j + 15] * inv);
          dh[j / 16] = make_uint4(w0.x, w1.x, w2.x, w3.x);
          dl[j / 16] = make_uint4(w0.y, w1.y, w2.y, w3.y);
        }
        if (h == 0) g.c_scale[static_cast<size_t>(nb) * g.p_cap + row0 + row] = scale;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm2_weighted_kernel(const __grid_constant__ CUtensorMap tm_chi, const __grid_constant__ CUtensorMap tm_clo,
                          const __grid_constant__ CUtensorMap tm_w, const Gemm2Args g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sAhi = smem;
  uint8_t* sAlo = smem + G2_OFF_ALO;
  uint8_t* sB = smem + G2_OFF_B;
  float* as_ring = reinterpret_cast<float*>(smem + G2_OFF_AS);
  float2* ws_ring = reinterpret_cast<float2*>(smem + G2_OFF_WS);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G2_OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = bars + G2_S;
  uint64_t* pfull = bars + 2 * G2_S;
  uint64_t* pempty = pfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + G2_OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + G2_OFF_MISC + 4);

  const int num_units = g.meta->num_tiles * kG2NB;
  if (static_cast<int>(blockIdx.x) >= num_units) return;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < G2_S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + kEpiWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], kEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_chi);
    tma_prefetch_desc(&tm_clo);
    tma_prefetch_desc(&tm_w);
  }
  if (warp == 1) tmem_alloc(tmem_holder, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp < 4) {
    setmaxnreg_dec<kRegsLow>();
    if (warp == 0) {
      int stage = 0;
      uint32_t ph = 0, armed = 0, armed_par = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        const int tile = u / kG2NB, nb2 = u % kG2NB;
        const int e = g.tile_expert[tile];
        const int row0 = g.tile_row0[tile];
        // w2_scale[e][nb][kb], nb = 2*nb2 + {0,1}, kb in [0,16): lane kb holds both
        const float* ws = g.w2_scale + (static_cast<size_t>(e) * kHB + 2 * nb2) * kIB;
        const float s0 = lane < kIB ? ws[lane] : 0.f;
        const float s1 = lane < kIB ? ws[kIB + lane] : 0.f;
        const int wrow = e * kH + nb2 * 256;
        for (int kb = 0; kb < kIB; ++kb) {
          const float w0 = __shfl_sync(0xffffffffu, s0, kb);
          const float w1 = __shfl_sync(0xffffffffu, s1, kb);
          int good = 1;
          if (lane == 0) {
            good = mbar_wait_abort(&empty[stage], ph ^ 1u, abort_flag, g.status, KF_STATUS_TIMEOUT_PRODUCER);
            if (good) {
              ws_ring[stage] = make_float2(w0, w1);
              mbar_arrive_expect_tx(&full[stage], G2_TX);
              tma_load_2d(sAhi + stage * G2_A, &tm_chi, kb * kBlk, row0, &full[stage]);
              tma_load_2d(sAlo + stage * G2_A, &tm_clo, kb * kBlk, row0, &full[stage]);
              tma_load_2d(sB + stage * G2_B, &tm_w, kb * kBlk, wrow, &full[stage]);
              bulk_load(as_ring + stage * kBlk, g.c_scale + static_cast<size_t>(kb) * g.p_cap + row0, kBlk * 4,
                        &full[stage]);
              armed |= 1u << stage;
              armed_par = ph ? (armed_par | (1u << stage)) : (armed_par & ~(1u << stage));
            }
          }
          good = __shfl_sync(0xffffffffu, good, 0);
          if (!good) {
            ok = false;
            break;
          }
          if (++stage == G2_S) {
            stage = 0;
            ph ^= 1u;
          }
        }
      }
      if (lane == 0) {
        int no_abort = 0;
        for (int s = 0; s < G2_S; ++s)
          if ((armed >> s) & 1u)
            mbar_wait_abort(&full[s], (armed_par >> s) & 1u, &no_abort, g.status, KF_STATUS_TIMEOUT_PRODUCER);
      }
    } else if (warp == 1) {
      if (lane == 0) {
        constexpr uint32_t idesc = idesc_e4m3_f32(128, 256);
        int stage = 0, pb = 0;
        uint32_t ph = 0, pph = 0;
        bool ok = true, committed = false;
        int last_pb = 0;
        uint32_t last_pph = 0;
        for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
          for (int kb = 0; kb < kIB; ++kb) {
            if (!mbar_wait_abort(&pempty[pb], pph ^ 1u, abort_flag, g.status, KF_STATUS_TIMEOUT_MMA) ||
                !mbar_wait_abort(&full[stage], ph, abort_flag, g.status, KF_STATUS_TIMEOUT_MMA)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t ahi = smem_u32(sAhi + stage * G2_A);
            const uint32_t alo = smem_u32(sAlo + stage * G2_A);
            const uint32_t b0 = smem_u32(sB + stage * G2_B);
            const uint32_t d = tmem + static_cast<uint32_t>(pb * 256);
#pragma unroll
            for (int k = 0; k < kBlk / 32; ++k) {
              const uint64_t bd = sw128_kmajor_desc(b0 + k * 32);
              mma_f8(d, sw128_kmajor_desc(ahi + k * 32), bd, idesc, k > 0 ? 1u : 0u);
              mma_f8(d, sw128_kmajor_desc(alo + k * 32), bd, idesc, 1u);
            }
            mma_commit(&empty[stage]);
            mma_commit(&pfull[pb]);
            committed = true;
            last_pb = pb;
            last_pph = pph;
            if (++stage == G2_S) {
              stage = 0;
              ph ^= 1u;
            }
            if (++pb == 2) {
              pb = 0;
              pph ^= 1u;
            }
          }
        }
        if (committed) {
          int no_abort = 0;
          mbar_wait_abort(&pfull[last_pb], last_pph, &no_abort, g.status, KF_STATUS_TIMEOUT_MMA);
        }
      }
      __syncwarp();
    }
  } else {
    setmaxnreg_inc<kRegsHigh>();
    const int pw = warp - 4;
    const int h = pw >> 2;        // output columns [128h, 128h+128) of the 256-column block
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    int stage = 0, pb = 0;
    uint32_t ph = 0, pph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      const int tile = u / kG2NB, nb2 = u % kG2NB;
      const int row0 = g.tile_row0[tile];
      const int nrows = g.tile_rows[tile];
      float acc[128];
#pragma unroll
      for (int j = 0; j < 128; ++j) acc[j] = 0.f;
      for (int kb = 0; kb < kIB; ++kb) {
        if (!mbar_wait_abort(&full[stage], ph, abort_flag, g.status, KF_STATUS_TIMEOUT_EPILOGUE)) {
          ok = false;
          break;
        }
        const float a_s = as_ring[stage * kBlk + row];
        const float2 ws = ws_ring[stage];
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (!mbar_wait_abort(&pfull[pb], pph, abort_flag, g.status, KF_STATUS_TIMEOUT_EPILOGUE)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem + lane_base + static_cast<uint32_t>(pb * 256 + h * 128);
        const float sc = a_s * (h ? ws.y : ws.x);
        float v[64];
        tmem_ld64_sync(taddr, v);
#pragma unroll
        for (int j = 0; j < 64; ++j) acc[j] = fmaf(v[j], sc, acc[j]);
        tmem_ld64_sync(taddr + 64, v);
#pragma unroll
        for (int j = 0; j < 64; ++j) acc[64 + j] = fmaf(v[j], sc, acc[64 + j]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pempty[pb]);
        if (++stage == G2_S) {
          stage = 0;
          ph ^= 1u;
        }
        if (++pb == 2) {
          pb = 0;
          pph ^= 1u;
        }
      }
      if (!ok) break;
      if (row < nrows) {
        const float w = g.slot_weight[row0 + row];
        float4* dst = reinterpret_cast<float4*>(g.y + static_cast<size_t>(row0 + row) * kH + nb2 * 256 + h * 128);
#pragma unroll
        for (int j = 0; j < 128; j += 4)
          dst[j / 4] = make_float4(acc[j] * w, acc[j + 1] * w, acc[j + 2] * w, acc[j + 3] * w);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

}  // namespace

cudaError_t gemm_set_attributes() {
  cudaError_t e = cudaFuncSetAttribute(gemm1_swiglu_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, G1_SMEM);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(gemm2_weighted_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, G2_SMEM);
}

cudaError_t launch_gemm1(const CUtensorMap& tm_a, const CUtensorMap& tm_w13, const Gemm1Args& args, int grid,
                         cudaStream_t s) {
  gemm1_swiglu_kernel<<<grid, kThreads, G1_SMEM, s>>>(tm_a, tm_w13, args);
  return cudaGetLastError();
}

cudaError_t launch_gemm2(const CUtensorMap& tm_chi, const CUtensorMap& tm_clo, const CUtensorMap& tm_w2,
                         const Gemm2Args& args, int grid, cudaStream_t s) {
  gemm2_weighted_kernel<<<grid, kThreads, G2_SMEM, s>>>(tm_chi, tm_clo, tm_w2, args);
  return cudaGetLastError();
}

}  // namespace kf
