// Grouped FP8 block-scale GEMMs on CTA pairs: one tcgen05 MMA with M = 256 spans
// the two CTAs of a cluster (cta_group::2).
//
// Why pairs: each work unit streams its A rows and its weight tile through L2
// into shared memory once per K chunk.  With one CTA per 128x256 tile, an SM
// ingests 48 KB (GEMM1) per K chunk, which neither L2 bandwidth nor four stages
// of latency hiding sustain at tensor-core rate.  With a pair, both CTAs load
// their own 128 rows of A and HALF of the 256-row weight tile (GEMM1: CTA 0 the
// 128 up rows, CTA 1 the 128 gate rows), so an SM ingests 32 KB per chunk for
// the same MMA work, and six stages fit in shared memory.
//
// Roles per CTA are those of the single-CTA kernels (warp 0 TMA producer, warp 1
// MMA issuer -- only in the pair leader, CTA rank 0 -- and warps 4-11 promotion
// + epilogue on the CTA's own 128 accumulator rows).  Synchronisation:
//   full[s]   (leader)  counts the operand bytes of BOTH CTAs (their TMA loads
//                       signal the leader's barrier; the leader alone arms it)
//   empty[s]  (each)    arrived by the MMA commit, multicast to both CTAs
//   pfull[b]  (each)    arrived by the MMA commit, multicast to both CTAs
//   pempty[b] (leader)  arrived by the 16 promotion warps of both CTAs
//   sfull/sempty (each) the CTA's own per-row scale ring
// No load uses cluster multicast: every CTA fetches its own tiles.
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "kf_fp8.cuh"
#include "kf_internal.cuh"
#include "kf_ptx.cuh"

namespace kf {

namespace {

constexpr int kThreads = 384;
constexpr int kEpiWarps = 8;
constexpr int kScaleRing = 8;
constexpr int kSmallRows = 32;
constexpr uint16_t kPairMask = 0x3;
constexpr int kRegsLow = 40;
constexpr int kRegsHigh = 232;
static_assert(128 * kRegsLow + 256 * kRegsHigh <= 384 * 168, "register split exceeds the launch allocation");

// GEMM1 pair: per CTA and stage, A 128x128 (16 KB) + half of the up|gate tile (16 KB).
constexpr int P1_S = 6;
constexpr int P1_A = kBlk * kBlk;
constexpr int P1_B = kBlk * kBlk;
constexpr int P1_OFF_B = P1_S * P1_A;
constexpr int P1_OFF_AS = P1_OFF_B + P1_S * P1_B;
constexpr int P1_OFF_WS = P1_OFF_AS + kScaleRing * kBlk * 4;
constexpr int P1_OFF_BAR = P1_OFF_WS + kScaleRing * 8;
constexpr int P1_NBAR = 2 * P1_S + 2 * kScaleRing + 6;
constexpr int P1_OFF_MISC = P1_OFF_BAR + P1_NBAR * 8;
constexpr int P1_OFF_XCH = P1_OFF_MISC + 16;
constexpr int P1_SMEM = P1_OFF_XCH + 2 * 2 * kBlk * 4 + 1024;

// GEMM2 pair: per CTA and stage, A_hi and A_lo 128x128 (16 KB each) + half of the
// 256-row W2 tile (16 KB; the W2 tensor map passed in must have a 128-row box).
constexpr int P2_S = 4;
constexpr int P2_A = kBlk * kBlk;
constexpr int P2_B = kBlk * kBlk;
constexpr int P2_OFF_ALO = P2_S * P2_A;
constexpr int P2_OFF_B = 2 * P2_S * P2_A;
constexpr int P2_OFF_AS = P2_OFF_B + P2_S * P2_B;
constexpr int P2_OFF_WS = P2_OFF_AS + kScaleRing * kBlk * 4;
constexpr int P2_OFF_BAR = P2_OFF_WS + kScaleRing * 8;
constexpr int P2_NBAR = 2 * P2_S + 2 * kScaleRing + 4;
constexpr int P2_OFF_MISC = P2_OFF_BAR + P2_NBAR * 8;
constexpr int P2_SMEM = P2_OFF_MISC + 16 + 1024;
constexpr int kG2NB = kH / 256;

static_assert(P1_SMEM <= 232448 && P2_SMEM <= 232448, "shared memory");

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023));
}

struct RingPos {
  int idx = 0;
  uint32_t ph = 0;
  template <int N>
  __device__ __forceinline__ void advance() {
    if (++idx == N) {
      idx = 0;
      ph ^= 1u;
    }
  }
};

struct ArmedSlots {
  uint32_t armed = 0, par = 0;
  __device__ __forceinline__ void set(int i, uint32_t ph) {
    armed |= 1u << i;
    par = ph ? (par | (1u << i)) : (par & ~(1u << i));
  }
  __device__ __forceinline__ void drain(uint64_t* bars, int n, int* status, int code) const {
    int no_abort = 0;
    for (int i = 0; i < n; ++i)
      if ((armed >> i) & 1u) mbar_wait_abort(&bars[i], (par >> i) & 1u, &no_abort, status, code);
  }
};

__device__ __forceinline__ int clamp_rows(int r) { return r < 0 ? 0 : (r > kBlk ? kBlk : r); }
__device__ __forceinline__ uint32_t a_box_bytes(int rows) {
  return rows == 0 ? 0u : (rows <= kSmallRows ? static_cast<uint32_t>(kSmallRows * kBlk) : static_cast<uint32_t>(kBlk * kBlk));
}

// --------------------------------------------------------------- GEMM1 pair --
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm1_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_a32,
                      const __grid_constant__ CUtensorMap tm_w, const Gemm1Args g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + P1_OFF_B;
  float* as_ring = reinterpret_cast<float*>(smem + P1_OFF_AS);
  float2* ws_ring = reinterpret_cast<float2*>(smem + P1_OFF_WS);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P1_OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = full + P1_S;
  uint64_t* sfull = empty + P1_S;
  uint64_t* sempty = sfull + kScaleRing;
  uint64_t* pfull = sempty + kScaleRing;
  uint64_t* pempty = pfull + 2;
  uint64_t* xbar = pempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + P1_OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + P1_OFF_MISC + 4);
  float* xch = reinterpret_cast<float*>(smem + P1_OFF_XCH);

  const uint32_t rank = cluster_ctarank();
  const int cid = static_cast<int>(blockIdx.x >> 1);
  const int ncl = static_cast<int>(gridDim.x >> 1);
  const int num_units = g.meta->num_ptiles * kIB;
  if (cid >= num_units) return;  // the same for both CTAs of the cluster

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < P1_S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < kScaleRing; ++s) {
      mbar_init(&sfull[s], 1);
      mbar_init(&sempty[s], kEpiWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], 2 * kEpiWarps);
      mbar_init(&xbar[b], kEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_a32);
    tma_prefetch_desc(&tm_w);
  }
  if (warp == 1) tmem_alloc_pair(tmem_holder, 512);
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp < 4) {
    setmaxnreg_dec<kRegsLow>();
    if (warp == 0) {
      // ------------------------------------------------------ TMA producer --
      const uint32_t full_leader = mapa_shared(smem_u32(full), 0);
      RingPos st, ss;
      ArmedSlots armed_st, armed_ss;
      bool ok = true;
      for (int u = cid; u < num_units && ok; u += ncl) {
        const int pt = u / kIB, nb = u % kIB;
        const int e = g.tile_expert[pt];
        const int prows = g.tile_rows[pt];
        const int row0 = g.tile_row0[pt] + static_cast<int>(rank) * kBlk;
        const int myrows = clamp_rows(prows - static_cast<int>(rank) * kBlk);
        const uint32_t my_a = a_box_bytes(myrows);
        const uint32_t tx = a_box_bytes(clamp_rows(prows)) + a_box_bytes(clamp_rows(prows - kBlk)) + 2 * P1_B;
        const float* wsu = g.w13_scale + (static_cast<size_t>(e) * 32 + nb) * kHB;
        const float* wsg = g.w13_scale + (static_cast<size_t>(e) * 32 + kIB + nb) * kHB;
        const float su0 = wsu[lane], sg0 = wsg[lane];
        const float su1 = (lane + 32 < kHB) ? wsu[lane + 32] : 0.f;
        const float sg1 = (lane + 32 < kHB) ? wsg[lane + 32] : 0.f;
        const int wrow = e * (2 * kI) + nb * kBlk + (rank ? kI : 0);  // CTA 0: up rows, CTA 1: gate rows
        for (int kb = 0; kb < kHB; ++kb) {
          const float su = __shfl_sync(0xffffffffu, kb < 32 ? su0 : su1, kb & 31);
          const float sg = __shfl_sync(0xffffffffu, kb < 32 ? sg0 : sg1, kb & 31);
          int good = 1;
          if (lane == 0) {
            good = mbar_wait_abort(&empty[st.idx], st.ph ^ 1u, abort_flag, g.status, KF_STATUS_TIMEOUT_PRODUCER) &&
                   mbar_wait_abort(&sempty[ss.idx], ss.ph ^ 1u, abort_flag, g.status, KF_STATUS_TIMEOUT_PRODUCER);
            if (good) {
              ws_ring[ss.idx] = make_float2(su, sg);
              if (myrows > 0) {
                mbar_arrive_expect_tx(&sfull[ss.idx], kBlk * 4);
                bulk_load(as_ring + ss.idx * kBlk, g.a_scale + static_cast<size_t>(kb) * g.p_cap + row0, kBlk * 4,
                          &sfull[ss.idx]);
              } else {
                mbar_arrive(&sfull[ss.idx]);
              }
              armed_ss.set(ss.idx, ss.ph);
              if (rank == 0) mbar_arrive_expect_tx(&full[st.idx], tx);
              const uint32_t fb = full_leader + static_cast<uint32_t>(st.idx * 8);
              if (my_a)
                tma_load_2d_pair(sA + st.idx * P1_A, my_a == P1_A ? &tm_a : &tm_a32, kb * kBlk, row0, fb);
              tma_load_2d_pair(sB + st.idx * P1_B, &tm_w, kb * kBlk, wrow, fb);
              armed_st.set(st.idx, st.ph);
            }
          }
          good = __shfl_sync(0xffffffffu, good, 0);
          if (!good) {
            ok = false;
            break;
          }
          st.advance<P1_S>();
          ss.advance<kScaleRing>();
        }
      }
      if (lane == 0) {
        // a stage is free again (its copies landed and the MMA read them) once
        // the MMA commit for its last use arrived on this CTA's empty barrier
        armed_st.drain(empty, P1_S, g.status, KF_STATUS_TIMEOUT_PRODUCER);
        armed_ss.drain(sfull, kScaleRing, g.status, KF_STATUS_TIMEOUT_PRODUCER);
      }
    } else if (warp == 1 && rank == 0) {
      // ---------------------------------------------- MMA issuer (leader) --
      if (lane == 0) {
        constexpr uint32_t idesc = idesc_e4m3_f32(256, 256);
        RingPos st, pb, last;
        bool ok = true, committed = false;
        for (int u = cid; u < num_units && ok; u += ncl) {
          for (int kb = 0; kb < kHB; ++kb) {
            if (!mbar_wait_abort_cluster(&pempty[pb.idx], pb.ph ^ 1u, abort_flag, g.status, KF_STATUS_TIMEOUT_MMA) ||
                !mbar_wait_abort_cluster(&full[st.idx], st.ph, abort_flag, g.status, KF_STATUS_TIMEOUT_MMA)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_u32(sA + st.idx * P1_A);
            const uint32_t b0 = smem_u32(sB + st.idx * P1_B);
            const uint32_t d = tmem + static_cast<uint32_t>(pb.idx * 256);
#pragma unroll
            for (int k = 0; k < kBlk / 32; ++k)
              mma_f8_pair(d, sw128_kmajor_desc(a0 + k * 32), sw128_kmajor_desc(b0 + k * 32), idesc,
                          k > 0 ? 1u : 0u);
            mma_commit_pair(&empty[st.idx], kPairMask);
            mma_commit_pair(&pfull[pb.idx], kPairMask);
            committed = true;
            last = pb;
            st.advance<P1_S>();
            pb.advance<2>();
          }
        }
        if (committed) {
          int no_abort = 0;
          mbar_wait_abort(&pfull[last.idx], last.ph, &no_abort, g.status, KF_STATUS_TIMEOUT_MMA);
        }
      }
      __syncwarp();
    }
  } else {
    setmaxnreg_inc<kRegsHigh>();
    // ------------------------------------------------ promotion + epilogue --
    const int pw = warp - 4;
    const int h = pw >> 2;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t pempty_leader = mapa_shared(smem_u32(pempty), 0);
    RingPos ss, pb;
    int it = 0;
    bool ok = true;
    for (int u = cid; u < num_units && ok; u += ncl, ++it) {
      const int pt = u / kIB, nb = u % kIB;
      const int row0 = g.tile_row0[pt] + static_cast<int>(rank) * kBlk;
      const int nrows = clamp_rows(g.tile_rows[pt] - static_cast<int>(rank) * kBlk);
      const bool live = q * 32 < nrows;
      float2 acc_u[32], acc_g[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        acc_u[j] = make_float2(0.f, 0.f);
        acc_g[j] = make_float2(0.f, 0.f);
      }
      for (int kb = 0; kb < kHB; ++kb) {
        if (!mbar_wait_abort(&sfull[ss.idx], ss.ph, abort_flag, g.status, KF_STATUS_TIMEOUT_EPILOGUE)) {
          ok = false;
          break;
        }
        const float a_s = as_ring[ss.idx * kBlk + row];
        const float2 ws = ws_ring[ss.idx];
        __syncwarp();
        if (lane == 0) mbar_arrive(&sempty[ss.idx]);
        if (!mbar_wait_abort(&pfull[pb.idx], pb.ph, abort_flag, g.status, KF_STATUS_TIMEOUT_EPILOGUE)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (live) {
          const uint32_t taddr = tmem + lane_base + static_cast<uint32_t>(pb.idx * 256 + h * 64);
          float v[64];
          tmem_ld64_sync(taddr, v);
          const float2 su = make_float2(a_s * ws.x, a_s * ws.x);
#pragma unroll
          for (int j = 0; j < 32; ++j) acc_u[j] = __ffma2_rn(make_float2(v[2 * j], v[2 * j + 1]), su, acc_u[j]);
          tmem_ld64_sync(taddr + 128, v);
          const float2 sg = make_float2(a_s * ws.y, a_s * ws.y);
#pragma unroll
          for (int j = 0; j < 32; ++j) acc_g[j] = __ffma2_rn(make_float2(v[2 * j], v[2 * j + 1]), sg, acc_g[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(pempty_leader + static_cast<uint32_t>(pb.idx * 8));
        ss.advance<kScaleRing>();
        pb.advance<2>();
      }
      if (!ok) break;
      float amax = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float2 gt = acc_g[j];
        const float hx = silu_f(gt.x) * acc_u[j].x;
        const float hy = silu_f(gt.y) * acc_u[j].y;
        acc_u[j] = make_float2(hx, hy);
        amax = fmaxf(amax, fmaxf(fabsf(hx), fabsf(hy)));
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
        for (int j = 0; j < 32; j += 8) {
          const uint2 w0 = encode_hilo4(acc_u[j].x * inv, acc_u[j].y * inv, acc_u[j + 1].x * inv, acc_u[j + 1].y * inv);
          const uint2 w1 =
              encode_hilo4(acc_u[j + 2].x * inv, acc_u[j + 2].y * inv, acc_u[j + 3].x * inv, acc_u[j + 3].y * inv);
          const uint2 w2 =
              encode_hilo4(acc_u[j + 4].x * inv, acc_u[j + 4].y * inv, acc_u[j + 5].x * inv, acc_u[j + 5].y * inv);
          const uint2 w3 =
              encode_hilo4(acc_u[j + 6].x * inv, acc_u[j + 6].y * inv, acc_u[j + 7].x * inv, acc_u[j + 7].y * inv);
          dh[j / 8] = make_uint4(w0.x, w1.x, w2.x, w3.x);
          dl[j / 8] = make_uint4(w0.y, w1.y, w2.y, w3.y);
        }
        if (h == 0) g.c_scale[static_cast<size_t>(nb) * g.p_cap + row0 + row] = scale;
      }
    }
  }

  tc_fence_before();
  cluster_sync_all();  // neither CTA leaves while its peer may still use its shared memory
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, 512);
}

// --------------------------------------------------------------- GEMM2 pair --
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm2_pair_kernel(const __grid_constant__ CUtensorMap tm_chi, const __grid_constant__ CUtensorMap tm_clo,
                      const __grid_constant__ CUtensorMap tm_chi32, const __grid_constant__ CUtensorMap tm_clo32,
                      const __grid_constant__ CUtensorMap tm_w, const Gemm2Args g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sAhi = smem;
  uint8_t* sAlo = smem + P2_OFF_ALO;
  uint8_t* sB = smem + P2_OFF_B;
  float* as_ring = reinterpret_cast<float*>(smem + P2_OFF_AS);
  float2* ws_ring = reinterpret_cast<float2*>(smem + P2_OFF_WS);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P2_OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = full + P2_S;
  uint64_t* sfull = empty + P2_S;
  uint64_t* sempty = sfull + kScaleRing;
  uint64_t* pfull = sempty + kScaleRing;
  uint64_t* pempty = pfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + P2_OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + P2_OFF_MISC + 4);

  const uint32_t rank = cluster_ctarank();
  const int cid = static_cast<int>(blockIdx.x >> 1);
  const int ncl = static_cast<int>(gridDim.x >> 1);
  const int num_units = g.meta->num_ptiles * kG2NB;
  if (cid >= num_units) return;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < P2_S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < kScaleRing; ++s) {
      mbar_init(&sfull[s], 1);
      mbar_init(&sempty[s], kEpiWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], 2 * kEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_chi);
    tma_prefetch_desc(&tm_clo);
    tma_prefetch_desc(&tm_chi32);
    tma_prefetch_desc(&tm_clo32);
    tma_prefetch_desc(&tm_w);
  }
  if (warp == 1) tmem_alloc_pair(tmem_holder, 512);
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp < 4) {
    setmaxnreg_dec<kRegsLow>();
    if (warp == 0) {
      const uint32_t full_leader = mapa_shared(smem_u32(full), 0);
      RingPos st, ss;
      ArmedSlots armed_st, armed_ss;
      bool ok = true;
      for (int u = cid; u < num_units && ok; u += ncl) {
        const int pt = u / kG2NB, nb2 = u % kG2NB;
        const int e = g.tile_expert[pt];
        const int prows = g.tile_rows[pt];
        const int row0 = g.tile_row0[pt] + static_cast<int>(rank) * kBlk;
        const int myrows = clamp_rows(prows - static_cast<int>(rank) * kBlk);
        const uint32_t my_a = a_box_bytes(myrows);
        const uint32_t tx =
            2 * (a_box_bytes(clamp_rows(prows)) + a_box_bytes(clamp_rows(prows - kBlk))) + 2 * P2_B;
        const float* ws = g.w2_scale + (static_cast<size_t>(e) * kHB + 2 * nb2) * kIB;
        const float s0 = lane < kIB ? ws[lane] : 0.f;
        const float s1 = lane < kIB ? ws[kIB + lane] : 0.f;
        const int wrow = e * kH + nb2 * 256 + static_cast<int>(rank) * kBlk;
        for (int kb = 0; kb < kIB; ++kb) {
          const float w0 = __shfl_sync(0xffffffffu, s0, kb);
          const float w1 = __shfl_sync(0xffffffffu, s1, kb);
          int good = 1;
          if (lane == 0) {
            good = mbar_wait_abort(&empty[st.idx], st.ph ^ 1u, abort_flag, g.status, KF_STATUS_TIMEOUT_PRODUCER) &&
                   mbar_wait_abort(&sempty[ss.idx], ss.ph ^ 1u, abort_flag, g.status, KF_STATUS_TIMEOUT_PRODUCER);
            if (good) {
              ws_ring[ss.idx] = make_float2(w0, w1);
              if (myrows > 0) {
                mbar_arrive_expect_tx(&sfull[ss.idx], kBlk * 4);
                bulk_load(as_ring + ss.idx * kBlk, g.c_scale + static_cast<size_t>(kb) * g.p_cap + row0, kBlk * 4,
                          &sfull[ss.idx]);
              } else {
                mbar_arrive(&sfull[ss.idx]);
              }
              armed_ss.set(ss.idx, ss.ph);
              if (rank == 0) mbar_arrive_expect_tx(&full[st.idx], tx);
              const uint32_t fb = full_leader + static_cast<uint32_t>(st.idx * 8);
              if (my_a) {
                const bool big = my_a == P2_A;
                tma_load_2d_pair(sAhi + st.idx * P2_A, big ? &tm_chi : &tm_chi32, kb * kBlk, row0, fb);
                tma_load_2d_pair(sAlo + st.idx * P2_A, big ? &tm_clo : &tm_clo32, kb * kBlk, row0, fb);
              }
              tma_load_2d_pair(sB + st.idx * P2_B, &tm_w, kb * kBlk, wrow, fb);
              armed_st.set(st.idx, st.ph);
            }
          }
          good = __shfl_sync(0xffffffffu, good, 0);
          if (!good) {
            ok = false;
            break;
          }
          st.advance<P2_S>();
          ss.advance<kScaleRing>();
        }
      }
      if (lane == 0) {
        armed_st.drain(empty, P2_S, g.status, KF_STATUS_TIMEOUT_PRODUCER);
        armed_ss.drain(sfull, kScaleRing, g.status, KF_STATUS_TIMEOUT_PRODUCER);
      }
    } else if (warp == 1 && rank == 0) {
      if (lane == 0) {
        constexpr uint32_t idesc = idesc_e4m3_f32(256, 256);
        RingPos st, pb, last;
        bool ok = true, committed = false;
        for (int u = cid; u < num_units && ok; u += ncl) {
          for (int kb = 0; kb < kIB; ++kb) {
            if (!mbar_wait_abort_cluster(&pempty[pb.idx], pb.ph ^ 1u, abort_flag, g.status, KF_STATUS_TIMEOUT_MMA) ||
                !mbar_wait_abort_cluster(&full[st.idx], st.ph, abort_flag, g.status, KF_STATUS_TIMEOUT_MMA)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t ahi = smem_u32(sAhi + st.idx * P2_A);
            const uint32_t alo = smem_u32(sAlo + st.idx * P2_A);
            const uint32_t b0 = smem_u32(sB + st.idx * P2_B);
            const uint32_t d = tmem + static_cast<uint32_t>(pb.idx * 256);
#pragma unroll
            for (int k = 0; k < kBlk / 32; ++k) {
              const uint64_t bd = sw128_kmajor_desc(b0 + k * 32);
              mma_f8_pair(d, sw128_kmajor_desc(ahi + k * 32), bd, idesc, k > 0 ? 1u : 0u);
              mma_f8_pair(d, sw128_kmajor_desc(alo + k * 32), bd, idesc, 1u);
            }
            mma_commit_pair(&empty[st.idx], kPairMask);
            mma_commit_pair(&pfull[pb.idx], kPairMask);
            committed = true;
            last = pb;
            st.advance<P2_S>();
            pb.advance<2>();
          }
        }
        if (committed) {
          int no_abort = 0;
          mbar_wait_abort(&pfull[last.idx], last.ph, &no_abort, g.status, KF_STATUS_TIMEOUT_MMA);
        }
      }
      __syncwarp();
    }
  } else {
    setmaxnreg_inc<kRegsHigh>();
    const int pw = warp - 4;
    const int h = pw >> 2;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t pempty_leader = mapa_shared(smem_u32(pempty), 0);
    RingPos ss, pb;
    bool ok = true;
    for (int u = cid; u < num_units && ok; u += ncl) {
      const int pt = u / kG2NB, nb2 = u % kG2NB;
      const int row0 = g.tile_row0[pt] + static_cast<int>(rank) * kBlk;
      const int nrows = clamp_rows(g.tile_rows[pt] - static_cast<int>(rank) * kBlk);
      const bool live = q * 32 < nrows;
      float2 acc[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) acc[j] = make_float2(0.f, 0.f);
      for (int kb = 0; kb < kIB; ++kb) {
        if (!mbar_wait_abort(&sfull[ss.idx], ss.ph, abort_flag, g.status, KF_STATUS_TIMEOUT_EPILOGUE)) {
          ok = false;
          break;
        }
        const float a_s = as_ring[ss.idx * kBlk + row];
        const float2 ws = ws_ring[ss.idx];
        __syncwarp();
        if (lane == 0) mbar_arrive(&sempty[ss.idx]);
        if (!mbar_wait_abort(&pfull[pb.idx], pb.ph, abort_flag, g.status, KF_STATUS_TIMEOUT_EPILOGUE)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (live) {
          const uint32_t taddr = tmem + lane_base + static_cast<uint32_t>(pb.idx * 256 + h * 128);
          const float sc = a_s * (h ? ws.y : ws.x);
          const float2 s2 = make_float2(sc, sc);
          float v[64];
          tmem_ld64_sync(taddr, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[j] = __ffma2_rn(make_float2(v[2 * j], v[2 * j + 1]), s2, acc[j]);
          tmem_ld64_sync(taddr + 64, v);
#pragma unroll
          for (int j = 0; j < 32; ++j)
            acc[32 + j] = __ffma2_rn(make_float2(v[2 * j], v[2 * j + 1]), s2, acc[32 + j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(pempty_leader + static_cast<uint32_t>(pb.idx * 8));
        ss.advance<kScaleRing>();
        pb.advance<2>();
      }
      if (!ok) break;
      if (row < nrows) {
        const float w = g.slot_weight[row0 + row];
        float4* dst = reinterpret_cast<float4*>(g.y + static_cast<size_t>(row0 + row) * kH + nb2 * 256 + h * 128);
#pragma unroll
        for (int j = 0; j < 64; j += 2)
          dst[j / 2] = make_float4(acc[j].x * w, acc[j].y * w, acc[j + 1].x * w, acc[j + 1].y * w);
      }
    }
  }

  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, 512);
}

}  // namespace

cudaError_t gemm_pair_set_attributes() {
  cudaError_t e = cudaFuncSetAttribute(gemm1_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P1_SMEM);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(gemm2_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P2_SMEM);
}

int gemm_pair_max_clusters() {
  int n1 = 0, n2 = 0, dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(sms & ~1), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = P1_SMEM;
  if (cudaOccupancyMaxActiveClusters(&n1, gemm1_pair_kernel, &cfg) != cudaSuccess) n1 = 0;
  cfg.dynamicSmemBytes = P2_SMEM;
  if (cudaOccupancyMaxActiveClusters(&n2, gemm2_pair_kernel, &cfg) != cudaSuccess) n2 = 0;
  cudaGetLastError();
  return n1 < n2 ? n1 : n2;
}

cudaError_t launch_gemm1_pair(const CUtensorMap& tm_a, const CUtensorMap& tm_a32, const CUtensorMap& tm_w13,
                              const Gemm1Args& args, int grid, cudaStream_t s) {
  gemm1_pair_kernel<<<grid, kThreads, P1_SMEM, s>>>(tm_a, tm_a32, tm_w13, args);
  return cudaGetLastError();
}

cudaError_t launch_gemm2_pair(const CUtensorMap& tm_chi, const CUtensorMap& tm_clo, const CUtensorMap& tm_chi32,
                              const CUtensorMap& tm_clo32, const CUtensorMap& tm_w2, const Gemm2Args& args, int grid,
                              cudaStream_t s) {
  gemm2_pair_kernel<<<grid, kThreads, P2_SMEM, s>>>(tm_chi, tm_clo, tm_chi32, tm_clo32, tm_w2, args);
  return cudaGetLastError();
}

}  // namespace kf
