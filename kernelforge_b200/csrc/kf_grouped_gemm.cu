// Grouped FP8 block-scale GEMMs of the MoE layer on the 5th-generation tensor
// cores (tcgen05 + tensor memory), fed by TMA.
//
// Both kernels are persistent (one CTA per SM) and warp-specialised:
//   warp 0        TMA producer: operand tiles (GEMM1 also its per-chunk scales,
//                 into a small smem ring; GEMM2's promotion warps read theirs
//                 from L2 directly)
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

#include "kf_fp8.cuh"
#include "kf_internal.cuh"
#include "kf_ptx.cuh"

namespace kf {

namespace {

constexpr int kThreads = 384;  // 12 warps
constexpr int kEpiWarps = 8;
constexpr int kScaleRing = 8;  // per-chunk scale slots; decoupled from the operand stages
constexpr int kSmallRows = 32; // tiles with at most this many valid rows load a 32-row A box

// ------------------------------------------------------------------ GEMM1 --
// X = A[rows, 7168] . W13[e]^T, N-block = 128 up columns + the matching 128 gate
// columns (one MMA with N = 256).  Epilogue: silu(gate) * up, then a two-term
// FP8 encoding (hi + lo residual) sharing one fp32 scale per 128 columns.
//
// Two shared-memory layouts, as for GEMM2 below: 4 stages of 128-row A tiles, or
// for calls with T <= 32 tokens 6 stages of 32-row A slots (4 KB; the MMA's rows
// 32-127 then read the following shared memory and feed accumulator rows that are
// never read), so more of W13 is in flight per SM.
template <bool kDecode>
struct G1Layout {
  static constexpr int S = kDecode ? 6 : 4;
  static constexpr int A = (kDecode ? kSmallRows : kBlk) * kBlk;  // one A slot
  static constexpr int B = 2 * kBlk * kBlk;    // 32 KB: up rows then gate rows
  static constexpr int OFF_B = S * A;
  static constexpr int OFF_AS = OFF_B + S * B;
  static constexpr int OFF_WS = OFF_AS + kScaleRing * kBlk * 4;
  static constexpr int OFF_BAR = OFF_WS + kScaleRing * 8;
  static constexpr int NBAR = 2 * S + 2 * kScaleRing + 6;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int OFF_XCH = OFF_MISC + 16;
  static constexpr int SMEM = OFF_XCH + 2 * 2 * kBlk * 4 + 1024;
  static_assert(OFF_B % 1024 == 0, "128-byte swizzled slots start on 1024-byte boundaries");
  static_assert(SMEM <= 232448, "GEMM1 shared memory");
  static_assert(S <= 32, "ring bitmask");
};

// ------------------------------------------------------------------ GEMM2 --
// Y = C[rows, 2048] . W2[e]^T with C = s * (C_hi + C_lo), N-block = 256 output
// columns.  Each K step issues two MMAs (hi and lo) into the same accumulator.
// Epilogue: multiply by the pair's routing weight, store the rows in bf16 (the
// reduce sums a token's rows in fp32).
//
// Two shared-memory layouts.  The general one holds 3 stages of full 128-row hi
// and lo tiles.  The decode one serves calls with T <= 32 tokens, where no
// expert can have more than 32 rows: it keeps only 32-row A slots (4 KB), which
// makes room for 5 stages, so more of W2 is in flight per SM when W2 streaming
// is the whole cost.  The MMA still spans 128 rows; in the decode layout rows
// 32-127 of an A operand are whatever the following shared memory holds, and
// they only feed accumulator rows that are never read.
// Epilogue staging for TMA stores of y: per promotion warp 32 rows x 32 fp32
// columns (4 KB, 128-byte swizzled as the y tensor map expects), 1024-aligned;
// in the decode layout only the two warps of rows 0-31 store.
constexpr int G2_STG_WARP = 32 * 32 * 4;
template <bool kDecode>
struct G2Layout {
  static constexpr int S = kDecode ? 5 : 3;
  static constexpr int A = (kDecode ? kSmallRows : kBlk) * kBlk;  // one hi or lo slot
  static constexpr int B = 2 * kBlk * kBlk;                       // 32 KB: 256 rows of W2
  static constexpr int OFF_ALO = S * A;
  static constexpr int OFF_B = 2 * S * A;
  static constexpr int OFF_BAR = OFF_B + S * B;
  static constexpr int NBAR = 2 * S + 4;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int OFF_STG = (OFF_MISC + 16 + 1023) / 1024 * 1024;
  static constexpr int STG_SLOTS = kDecode ? 2 : kEpiWarps;
  static constexpr int SMEM = OFF_STG + STG_SLOTS * G2_STG_WARP + 1024;
  static_assert(OFF_ALO % 1024 == 0 && OFF_B % 1024 == 0, "128-byte swizzled slots start on 1024-byte boundaries");
  static_assert(SMEM <= 232448, "GEMM2 shared memory");
  static_assert(S <= 32, "ring bitmask");
};
constexpr int kG2NB = kH / 256;  // 28 column blocks of 256

static_assert(kScaleRing <= 32, "ring bitmask");
// Register split (setmaxnreg): warpgroup 0 drops to 48, warpgroups 1-2 rise to
// 224: 128*48 + 256*224 = 63488 <= 384 threads * 168, the launch allocation
// (__launch_bounds__(384, 1); the build checks ptxas reports 168).  ptxas
// allocates each region up to its setmaxnreg count; of the splits measured this
// one leaves the GEMM1 promotion loop nearly free of spills.
constexpr int kRegsLow = 48;
constexpr int kRegsHigh = 224;
static_assert(128 * kRegsLow + 256 * kRegsHigh <= 384 * 168, "register split exceeds the launch allocation");

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023));
}

// Ring position: index and phase parity, advanced together.
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

// Bitmask record of the last phase armed on each slot of a ring, so the producer
// can wait for its in-flight copies before the CTA exits.
struct ArmedSlots {
  uint32_t armed = 0, par = 0;
  __device__ __forceinline__ void set(int i, uint32_t ph) {
    armed |= 1u << i;
    par = ph ? (par | (1u << i)) : (par & ~(1u << i));
  }
  __device__ __forceinline__ void drain(uint64_t* bars, int n, int* status) const {
    int no_abort = 0;
    for (int i = 0; i < n; ++i)
      if ((armed >> i) & 1u) mbar_wait_abort(&bars[i], (par >> i) & 1u, &no_abort, status, KF_STATUS_TIMEOUT_PRODUCER);
  }
};

template <bool kDecode>
__global__ void __launch_bounds__(kThreads, 1)
    gemm1_swiglu_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_a32,
                        const __grid_constant__ CUtensorMap tm_w, const Gemm1Args g) {
  grid_dep_wait();
  grid_dep_trigger();
  using L = G1Layout<kDecode>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + L::OFF_B;
  float* as_ring = reinterpret_cast<float*>(smem + L::OFF_AS);
  float2* ws_ring = reinterpret_cast<float2*>(smem + L::OFF_WS);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = full + L::S;
  uint64_t* sfull = empty + L::S;
  uint64_t* sempty = sfull + kScaleRing;
  uint64_t* pfull = sempty + kScaleRing;
  uint64_t* pempty = pfull + 2;
  uint64_t* xbar = pempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);
  float* xch = reinterpret_cast<float*>(smem + L::OFF_XCH);

  const int S = g.ksplit;
  const int kb_per = kHB / S;
  const int num_units = g.meta->num_tiles * kIB * S;
  if (static_cast<int>(blockIdx.x) >= num_units) return;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < L::S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < kScaleRing; ++s) {
      mbar_init(&sfull[s], 1);
      mbar_init(&sempty[s], kEpiWarps);
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
    tma_prefetch_desc(&tm_a32);
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
      RingPos st, ss;
      ArmedSlots armed_st, armed_ss;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        const int base = u / S, ks = u % S;
        const int tile = base / kIB, nb = base % kIB;
        const int e = g.tile_expert[tile];
        const int row0 = g.tile_row0[tile];
        const bool small = kDecode || g.tile_rows[tile] <= kSmallRows;
        const uint32_t tx = (small ? kSmallRows * kBlk : L::A) + L::B;
        const float* wsu = g.w13_scale + (static_cast<size_t>(e) * 32 + nb) * kHB;
        const float* wsg = g.w13_scale + (static_cast<size_t>(e) * 32 + kIB + nb) * kHB;
        const float su0 = wsu[lane], sg0 = wsg[lane];
        const float su1 = (lane + 32 < kHB) ? wsu[lane + 32] : 0.f;
        const float sg1 = (lane + 32 < kHB) ? wsg[lane + 32] : 0.f;
        const int wrow_up = e * (2 * kI) + nb * kBlk;
        for (int kb = ks * kb_per; kb < (ks + 1) * kb_per; ++kb) {
          const float su = __shfl_sync(0xffffffffu, kb < 32 ? su0 : su1, kb & 31);
          const float sg = __shfl_sync(0xffffffffu, kb < 32 ? sg0 : sg1, kb & 31);
          int good = 1;
          if (lane == 0) {
            good = mbar_wait_abort(&empty[st.idx], st.ph ^ 1u, abort_flag, g.status, KF_STATUS_TIMEOUT_PRODUCER) &&
                   mbar_wait_abort(&sempty[ss.idx], ss.ph ^ 1u, abort_flag, g.status, KF_STATUS_TIMEOUT_PRODUCER);
            if (good) {
              ws_ring[ss.idx] = make_float2(su, sg);
              mbar_arrive_expect_tx(&sfull[ss.idx], kBlk * 4);
              bulk_load(as_ring + ss.idx * kBlk, g.a_scale + static_cast<size_t>(kb) * g.p_cap + row0, kBlk * 4,
                        &sfull[ss.idx]);
              armed_ss.set(ss.idx, ss.ph);
              mbar_arrive_expect_tx(&full[st.idx], tx);
              tma_load_2d(sA + st.idx * L::A, small ? &tm_a32 : &tm_a, kb * kBlk, row0, &full[st.idx]);
              tma_load_2d(sB + st.idx * L::B, &tm_w, kb * kBlk, wrow_up, &full[st.idx]);
              tma_load_2d(sB + st.idx * L::B + L::B / 2, &tm_w, kb * kBlk, wrow_up + kI, &full[st.idx]);
              armed_st.set(st.idx, st.ph);
            }
          }
          good = __shfl_sync(0xffffffffu, good, 0);
          if (!good) {
            ok = false;
            break;
          }
          st.template advance<L::S>();
          ss.advance<kScaleRing>();
        }
      }
      if (lane == 0) {  // let every copy that was issued land before the CTA can exit
        armed_st.drain(full, L::S, g.status);
        armed_ss.drain(sfull, kScaleRing, g.status);
      }
    } else if (warp == 1) {
      // -------------------------------------------------------- MMA issuer --
      if (lane == 0) {
        constexpr uint32_t idesc = idesc_e4m3_f32(128, 256);
        RingPos st, pb;
        bool ok = true, committed = false;
        RingPos last;
        for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
          for (int kb = 0; kb < kb_per; ++kb) {
            if (!mbar_wait_abort(&pempty[pb.idx], pb.ph ^ 1u, abort_flag, g.status, KF_STATUS_TIMEOUT_MMA) ||
                !mbar_wait_abort(&full[st.idx], st.ph, abort_flag, g.status, KF_STATUS_TIMEOUT_MMA)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_u32(sA + st.idx * L::A);
            const uint32_t b0 = smem_u32(sB + st.idx * L::B);
            const uint32_t d = tmem + static_cast<uint32_t>(pb.idx * 256);
#pragma unroll
            for (int k = 0; k < kBlk / 32; ++k)
              mma_f8(d, sw128_kmajor_desc(a0 + k * 32), sw128_kmajor_desc(b0 + k * 32), idesc, k > 0 ? 1u : 0u);
            mma_commit(&empty[st.idx]);
            mma_commit(&pfull[pb.idx]);
            committed = true;
            last = pb;
            st.template advance<L::S>();
            pb.advance<2>();
          }
        }
        if (committed) {  // the tensor core must be idle before TMEM is released
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
    const int h = pw >> 2;        // column half: up/gate columns [64h, 64h+64) of the block
    const int q = warp & 3;       // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    RingPos ss, pb;
    int it = 0;  // epilogues run so far (phase of the absmax exchange barrier)
    bool ok = true;
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      const int base = u / S, ks = u % S;
      const int tile = base / kIB, nb = base % kIB;
      const int row0 = g.tile_row0[tile];
      const int nrows = g.tile_rows[tile];
      const bool live = q * 32 < nrows;   // this warp's 32 rows hold at least one real pair
      float2 acc_u[32], acc_g[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        acc_u[j] = make_float2(0.f, 0.f);
        acc_g[j] = make_float2(0.f, 0.f);
      }
      for (int kb = 0; kb < kb_per; ++kb) {
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
          const float2 su = make_float2(a_s * ws.x, a_s * ws.x);
          const float2 sg = make_float2(a_s * ws.y, a_s * ws.y);
          {
            float v[32];
            tmem_ld32_sync(taddr, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) acc_u[j] = __ffma2_rn(make_float2(v[2 * j], v[2 * j + 1]), su, acc_u[j]);
          }
          {
            float v[32];
            tmem_ld32_sync(taddr + 32, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) acc_u[16 + j] = __ffma2_rn(make_float2(v[2 * j], v[2 * j + 1]), su, acc_u[16 + j]);
          }
          {
            float v[32];
            tmem_ld32_sync(taddr + 128, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) acc_g[j] = __ffma2_rn(make_float2(v[2 * j], v[2 * j + 1]), sg, acc_g[j]);
          }
          {
            float v[32];
            tmem_ld32_sync(taddr + 160, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) acc_g[16 + j] = __ffma2_rn(make_float2(v[2 * j], v[2 * j + 1]), sg, acc_g[16 + j]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pempty[pb.idx]);
        ss.advance<kScaleRing>();
        pb.advance<2>();
      }
      if (!ok) break;
      if (S > 1) {
        // split-K: store this split's fp32 sums (up | gate) for the pair; the
        // SwiGLU and requantisation run in swiglu_quant_kernel once all splits are in
        if (row < nrows) {
          const size_t prow = static_cast<size_t>(g.slot_pair[row0 + row]);
          float4* pu = reinterpret_cast<float4*>(g.partial + (static_cast<size_t>(ks) * g.max_pairs + prow) * 4096 +
                                                 nb * 256 + h * 64);
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            pu[j / 2] = make_float4(acc_u[j].x, acc_u[j].y, acc_u[j + 1].x, acc_u[j + 1].y);
            pu[32 + j / 2] = make_float4(acc_g[j].x, acc_g[j].y, acc_g[j + 1].x, acc_g[j + 1].y);
          }
        }
        continue;
      }
      // SwiGLU: silu(X2) * X1 with X1 = up (W13 rows [0, I)), X2 = gate (rows [I, 2I))
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
      ++it;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// Two floats rounded to bf16 (nearest even), first in the low half.
__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// A GEMM2 work unit as the promotion warps see it (tile entry read one unit ahead).
struct G2Unit {
  int nb2, e, row0, nrows;
};

__device__ __forceinline__ G2Unit g2_unit(const Gemm2Args& g, int u) {
  G2Unit r;
  const int tile = u / kG2NB;
  r.nb2 = u % kG2NB;
  r.e = g.tile_expert[tile];
  r.row0 = g.tile_row0[tile];
  r.nrows = g.tile_rows[tile];
  return r;
}

// Scales of K chunk kb for one row and one 128-column half h of the unit's 256
// output columns: the C block scale and w2_scale[e][2*nb2 + h][kb].
__device__ __forceinline__ void g2_scales(const Gemm2Args& g, const G2Unit& w, int kb, int row, int h, float& a,
                                          float& ws) {
  a = __ldg(g.c_scale + static_cast<size_t>(kb) * g.p_cap + w.row0 + row);
  ws = __ldg(g.w2_scale + (static_cast<size_t>(w.e) * kHB + 2 * w.nb2 + h) * kIB + kb);
}

template <bool kDecode>
__global__ void __launch_bounds__(kThreads, 1)
    gemm2_weighted_kernel(const __grid_constant__ CUtensorMap tm_chi, const __grid_constant__ CUtensorMap tm_clo,
                          const __grid_constant__ CUtensorMap tm_chi32, const __grid_constant__ CUtensorMap tm_clo32,
                          const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_y,
                          const Gemm2Args g) {
  grid_dep_wait();
  grid_dep_trigger();
  using L = G2Layout<kDecode>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sAhi = smem;
  uint8_t* sAlo = smem + L::OFF_ALO;
  uint8_t* sB = smem + L::OFF_B;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = full + L::S;
  uint64_t* pfull = empty + L::S;
  uint64_t* pempty = pfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  const int num_units = g.meta->num_tiles * kG2NB;
  if (static_cast<int>(blockIdx.x) >= num_units) return;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < L::S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
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
    tma_prefetch_desc(&tm_chi32);
    tma_prefetch_desc(&tm_clo32);
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_y);
  }
  if (warp == 1) tmem_alloc(tmem_holder, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp < 4) {
    setmaxnreg_dec<kRegsLow>();
    if (warp == 0) {
      RingPos st;
      ArmedSlots armed_st;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        const int tile = u / kG2NB, nb2 = u % kG2NB;
        const int e = g.tile_expert[tile];
        const int row0 = g.tile_row0[tile];
        const bool small = kDecode || g.tile_rows[tile] <= kSmallRows;
        const uint32_t tx = 2 * (small ? kSmallRows * kBlk : L::A) + L::B;
        const int wrow = e * kH + nb2 * 256;
        for (int kb = 0; kb < kIB; ++kb) {
          int good = 1;
          if (lane == 0) {
            good = mbar_wait_abort(&empty[st.idx], st.ph ^ 1u, abort_flag, g.status, KF_STATUS_TIMEOUT_PRODUCER);
            if (good) {
              mbar_arrive_expect_tx(&full[st.idx], tx);
              tma_load_2d(sAhi + st.idx * L::A, small ? &tm_chi32 : &tm_chi, kb * kBlk, row0, &full[st.idx]);
              tma_load_2d(sAlo + st.idx * L::A, small ? &tm_clo32 : &tm_clo, kb * kBlk, row0, &full[st.idx]);
              tma_load_2d(sB + st.idx * L::B, &tm_w, kb * kBlk, wrow, &full[st.idx]);
              armed_st.set(st.idx, st.ph);
            }
          }
          good = __shfl_sync(0xffffffffu, good, 0);
          if (!good) {
            ok = false;
            break;
          }
          st.template advance<L::S>();
        }
      }
      if (lane == 0) armed_st.drain(full, L::S, g.status);
    } else if (warp == 1) {
      if (lane == 0) {
        constexpr uint32_t idesc = idesc_e4m3_f32(128, 256);
        RingPos st, pb, last;
        bool ok = true, committed = false;
        for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
          for (int kb = 0; kb < kIB; ++kb) {
            if (!mbar_wait_abort(&pempty[pb.idx], pb.ph ^ 1u, abort_flag, g.status, KF_STATUS_TIMEOUT_MMA) ||
                !mbar_wait_abort(&full[st.idx], st.ph, abort_flag, g.status, KF_STATUS_TIMEOUT_MMA)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t ahi = smem_u32(sAhi + st.idx * L::A);
            const uint32_t alo = smem_u32(sAlo + st.idx * L::A);
            const uint32_t b0 = smem_u32(sB + st.idx * L::B);
            const uint32_t d = tmem + static_cast<uint32_t>(pb.idx * 256);
#pragma unroll
            for (int k = 0; k < kBlk / 32; ++k) {
              const uint64_t bd = sw128_kmajor_desc(b0 + k * 32);
              mma_f8(d, sw128_kmajor_desc(ahi + k * 32), bd, idesc, k > 0 ? 1u : 0u);
              mma_f8(d, sw128_kmajor_desc(alo + k * 32), bd, idesc, 1u);
            }
            mma_commit(&empty[st.idx]);
            mma_commit(&pfull[pb.idx]);
            committed = true;
            last = pb;
            st.template advance<L::S>();
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
    const int h = pw >> 2;        // output columns [128h, 128h+128) of the 256-column block
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    RingPos pb;
    bool ok = true;
    // Block scales stream from L2 two chunks ahead of use, across unit
    // boundaries, with no shared-memory ring or barrier: the row's C block scale
    // and the weight-block scale of this warp's 128 output columns.  (Measured:
    // 6-7% fewer GEMM2 cycles than a producer-filled scale ring; for GEMM1 the
    // ring was as fast or faster, so GEMM1 keeps it.)
    G2Unit cur = g2_unit(g, blockIdx.x);
    float a_n0, w_n0, a_n1, w_n1;
    g2_scales(g, cur, 0, row, h, a_n0, w_n0);
    g2_scales(g, cur, 1, row, h, a_n1, w_n1);
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      const bool has_next = u + static_cast<int>(gridDim.x) < num_units;
      const G2Unit nxt = has_next ? g2_unit(g, u + gridDim.x) : cur;
      const int nb2 = cur.nb2, row0 = cur.row0, nrows = cur.nrows;
      const bool live = kDecode ? q == 0 : q * 32 < nrows;
      // the decode layout holds 32 rows per tile; a call routed here has T <= 32
      if (kDecode && nrows > kSmallRows && pw == 0 && lane == 0) record_error(g.status, KF_STATUS_SLOT_OVERFLOW);
      // the routing weight of this thread's row, for the epilogue: loaded as the unit
      // starts so the L2 round trip is not on the epilogue's critical path
      const float w = row < nrows ? g.slot_weight[row0 + row] : 0.f;
      float2 acc[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) acc[j] = make_float2(0.f, 0.f);
      for (int kb = 0; kb < kIB; ++kb) {
        const float a_s = a_n0, w_s = w_n0;
        a_n0 = a_n1;
        w_n0 = w_n1;
        if (kb + 2 < kIB)
          g2_scales(g, cur, kb + 2, row, h, a_n1, w_n1);
        else if (has_next)
          g2_scales(g, nxt, kb + 2 - kIB, row, h, a_n1, w_n1);
        if (!mbar_wait_abort(&pfull[pb.idx], pb.ph, abort_flag, g.status, KF_STATUS_TIMEOUT_EPILOGUE)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (live) {
          const uint32_t taddr = tmem + lane_base + static_cast<uint32_t>(pb.idx * 256 + h * 128);
          const float sc = a_s * w_s;
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
        if (lane == 0) mbar_arrive(&pempty[pb.idx]);
        pb.advance<2>();
      }
      if (!ok) break;
      if (live) {
        // y rows leave in bf16 through TMA stores: each round the warp writes a
        // 32-row x 64-column tile (this lane = one row, 128 bytes) into its
        // 128-byte-swizzled staging buffer, and one lane stores it to y; the buffer
        // is rewritten only after the previous store has read it.  Rows of the
        // tile beyond nrows are padding rows of this tile, which nothing reads.
        uint8_t* stg = smem + L::OFF_STG + (kDecode ? h : pw) * G2_STG_WARP;
        const int xcol = nb2 * 256 + h * 128;
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          if (lane == 0) bulk_wait_group_read0();
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float2* a = acc + 32 * m + 4 * j;
            uint4 pk;
            pk.x = bf16x2_bits(a[0].x * w, a[0].y * w);
            pk.y = bf16x2_bits(a[1].x * w, a[1].y * w);
            pk.z = bf16x2_bits(a[2].x * w, a[2].y * w);
            pk.w = bf16x2_bits(a[3].x * w, a[3].y * w);
            *reinterpret_cast<uint4*>(stg + lane * 128 + ((j ^ (lane & 7)) << 4)) = pk;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tm_y, xcol + 64 * m, row0 + q * 32, stg);
            bulk_commit_group();
          }
        }
      }
      cur = nxt;
    }
    if (lane == 0) bulk_wait_group0();  // this warp's y stores are complete before the CTA can exit
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// Split-K finish of GEMM1: sum the splits' fp32 partials of one (row, 128-column
// block) in split order, apply SwiGLU and the two-term FP8 encoding -- the
// epilogue of gemm1_swiglu_kernel for calls whose K loop was split.  One warp
// per (permuted row, column block); lane l owns columns 4l..4l+3 of the block.
__global__ void __launch_bounds__(256) swiglu_quant_kernel(const Meta* __restrict__ meta,
                                                           const int32_t* __restrict__ tile_rows,
                                                           const int32_t* __restrict__ slot_pair,
                                                           const float* __restrict__ partial, int ksplit,
                                                           int max_pairs, int p_cap, uint8_t* __restrict__ c_hi,
                                                           uint8_t* __restrict__ c_lo, float* __restrict__ c_scale) {
  grid_dep_wait();
  grid_dep_trigger();
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int nwork = meta->num_tiles * kBlk * kIB;
  for (int wi = blockIdx.x * warps + (threadIdx.x >> 5); wi < nwork; wi += gridDim.x * warps) {
    const int r = wi / kIB, nb = wi % kIB;
    if ((r & (kBlk - 1)) >= tile_rows[r >> 7]) continue;
    const size_t pair = static_cast<size_t>(slot_pair[r]);
    float4 up = make_float4(0.f, 0.f, 0.f, 0.f), gt = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < ksplit; ++s) {
      const float* base = partial + (static_cast<size_t>(s) * max_pairs + pair) * 4096 + nb * 256;
      // per column block the partial row holds [up 128 | gate 128]
      const float4 u = reinterpret_cast<const float4*>(base)[lane];
      const float4 g = reinterpret_cast<const float4*>(base + 128)[lane];
      up.x += u.x; up.y += u.y; up.z += u.z; up.w += u.w;
      gt.x += g.x; gt.y += g.y; gt.z += g.z; gt.w += g.w;
    }
    float hv[4] = {silu_f(gt.x) * up.x, silu_f(gt.y) * up.y, silu_f(gt.z) * up.z, silu_f(gt.w) * up.w};
    float amax = fmaxf(fmaxf(fabsf(hv[0]), fabsf(hv[1])), fmaxf(fabsf(hv[2]), fabsf(hv[3])));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float inv = amax > 0.f ? 448.0f / amax : 1.0f;
    const uint2 w = encode_hilo4(hv[0] * inv, hv[1] * inv, hv[2] * inv, hv[3] * inv);
    const size_t off = static_cast<size_t>(r) * kI + nb * kBlk + lane * 4;
    *reinterpret_cast<uint32_t*>(c_hi + off) = w.x;
    *reinterpret_cast<uint32_t*>(c_lo + off) = w.y;
    if (lane == 0) c_scale[static_cast<size_t>(nb) * p_cap + r] = amax > 0.f ? amax / 448.0f : 1.0f;
  }
}

}  // namespace

cudaError_t gemm_set_attributes() {
  cudaError_t e = cudaFuncSetAttribute(gemm1_swiglu_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       G1Layout<false>::SMEM);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(gemm1_swiglu_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           G1Layout<true>::SMEM);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(gemm2_weighted_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           G2Layout<false>::SMEM);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(gemm2_weighted_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              G2Layout<true>::SMEM);
}

cudaError_t launch_gemm1(const CUtensorMap& tm_a, const CUtensorMap& tm_a32, const CUtensorMap& tm_w13,
                         const Gemm1Args& args, int grid, cudaStream_t s) {
  if (args.decode)
    return launch_chained(gemm1_swiglu_kernel<true>, dim3(grid), dim3(kThreads), G1Layout<true>::SMEM, s, tm_a, tm_a32,
                          tm_w13, args);
  return launch_chained(gemm1_swiglu_kernel<false>, dim3(grid), dim3(kThreads), G1Layout<false>::SMEM, s, tm_a,
                        tm_a32, tm_w13, args);
}

cudaError_t launch_swiglu_quant(const Gemm1Args& g, int grid, cudaStream_t s) {
  return launch_chained(swiglu_quant_kernel, dim3(grid), dim3(256), 0, s, g.meta, g.tile_rows, g.slot_pair, g.partial, g.ksplit, g.max_pairs,
                                           g.p_cap, g.c_hi, g.c_lo, g.c_scale);
}

cudaError_t launch_gemm2(const CUtensorMap& tm_chi, const CUtensorMap& tm_clo, const CUtensorMap& tm_chi32,
                         const CUtensorMap& tm_clo32, const CUtensorMap& tm_w2, const CUtensorMap& tm_y,
                         const Gemm2Args& args, int grid, cudaStream_t s) {
  if (args.decode)
    return launch_chained(gemm2_weighted_kernel<true>, dim3(grid), dim3(kThreads), G2Layout<true>::SMEM, s, tm_chi,
                          tm_clo, tm_chi32, tm_clo32, tm_w2, tm_y, args);
  return launch_chained(gemm2_weighted_kernel<false>, dim3(grid), dim3(kThreads), G2Layout<false>::SMEM, s, tm_chi,
                        tm_clo, tm_chi32, tm_clo32, tm_w2, tm_y, args);
}

}  // namespace kf
