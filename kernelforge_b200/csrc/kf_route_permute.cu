// Routing, permutation and reduction kernels of the fused MoE layer.
//
//   route_kernel          DeepSeek-V3 grouped sigmoid routing, one warp per token
//                         (reference: solution/triton/kernel.py:1842-1867)
//   permute_scan_kernel   per-expert counts, 128-aligned segment starts and the
//                         row-tile work list (reference: _sort_tokens :46-82 and
//                         the tile metadata of _build_launch_tile_metadata :153-201)
//   permute_assign_kernel stable slot of every local (token, expert) pair, and
//                         each token's rows listed in ascending order
//   gather_rows_kernel    gather of FP8 rows and scales into expert-contiguous rows
//   front_small_kernel    all of the above in one block, for decode-sized calls
//   unpermute_reduce_kernel  atomic-free unpermute-reduce into the output
//                         (reference: the index_add_ combine :1920-1925)
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "kf_internal.cuh"
#include "kf_ptx.cuh"

namespace kf {

namespace {

constexpr int kRouteThreads = 256;  // 8 warps, one token each

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// Routes one token with one warp.  Lane l owns experts [8l, 8l+8); group g is
// lanes [4g, 4g+4).  On return lane k < 8 holds the k-th selected expert (in
// descending biased-score order, ties to the lower id) and its weight.
__device__ __forceinline__ void route_one_token(const float* __restrict__ logits_row, const float (&b)[8], float rsf,
                                                int lane, int& e_out, float& w_out) {
  const float4* lp = reinterpret_cast<const float4*>(logits_row + lane * 8);
  const float4 x0 = lp[0], x1 = lp[1];
  const float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
  float s[8], sb[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    s[j] = 1.0f / (1.0f + expf(-x[j]));
    sb[j] = s[j] + b[j];
  }
  // group score: sum of the two largest biased scores of the group's 32 experts
  float m1 = -INFINITY, m2 = -INFINITY;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (sb[j] > m1) {
      m2 = m1;
      m1 = sb[j];
    } else if (sb[j] > m2) {
      m2 = sb[j];
    }
  }
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    const float o1 = __shfl_xor_sync(0xffffffffu, m1, off);
    const float o2 = __shfl_xor_sync(0xffffffffu, m2, off);
    const float n2 = fmaxf(fminf(m1, o1), fmaxf(m2, o2));
    m1 = fmaxf(m1, o1);
    m2 = n2;
  }
  const float gscore = m1 + m2;
  float gs[8];
#pragma unroll
  for (int g = 0; g < 8; ++g) gs[g] = __shfl_sync(0xffffffffu, gscore, 4 * g);
  // keep the 4 best groups (ties: lower group index wins)
  const int my_group = lane >> 2;
  int rank = 0;
#pragma unroll
  for (int g = 0; g < 8; ++g) rank += better(gs[g], g, gs[my_group], my_group) ? 1 : 0;
  uint32_t avail = (rank < 4) ? 0xFFu : 0u;
  // top-8 over the kept experts by biased score (ties: lower expert id wins).
  // Scores are compared as order-preserving unsigned keys (sb is finite and
  // never -0: it is a positive sigmoid plus a finite bias), so one warp max-
  // reduction per round finds the best score; of the lanes holding it the
  // lowest wins, and within a lane the lowest j: ties go to the lower expert id.
  uint32_t key[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t u = __float_as_uint(sb[j]);
    key[j] = ((avail >> j) & 1u) ? ((u & 0x80000000u) ? ~u : (u | 0x80000000u)) : 0u;  // 0: not a candidate
  }
  int sel[8];
  float sel_s[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    uint32_t bk = key[0];
    int bj = 0;
#pragma unroll
    for (int j = 1; j < 8; ++j)
      if (key[j] > bk) {
        bk = key[j];
        bj = j;
      }
    const uint32_t wk = __reduce_max_sync(0xffffffffu, bk);
    const int owner = __ffs(__ballot_sync(0xffffffffu, bk == wk)) - 1;
    float mine = s[0];
#pragma unroll
    for (int j = 1; j < 8; ++j)
      if (j == bj) mine = s[j];
    sel[k] = owner * 8 + __shfl_sync(0xffffffffu, bj, owner);
    sel_s[k] = __shfl_sync(0xffffffffu, mine, owner);
    if (lane == owner) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j == bj) key[j] = 0u;
    }
  }
  // normalise the un-biased scores, summed in ascending expert order, then
  // scale: lane k < 8 takes selection k and its rank among the 8 ids
  int my_e = sel[0];
  float my_s = sel_s[0];
#pragma unroll
  for (int k = 1; k < 8; ++k)
    if (lane == k) {
      my_e = sel[k];
      my_s = sel_s[k];
    }
  int my_rank = 0;
#pragma unroll
  for (int q = 0; q < 8; ++q) my_rank += (sel[q] < my_e) ? 1 : 0;
  float sum = 0.f;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int src = __ffs(__ballot_sync(0xffffffffu, lane < 8 && my_rank == r)) - 1;
    sum += __shfl_sync(0xffffffffu, my_s, src);
  }
  const float denom = sum + 1e-20f;
  e_out = lane < 8 ? my_e : 0;
  w_out = lane < 8 ? (my_s / denom) * rsf : 0.f;
}

__device__ __forceinline__ void load_bias8(const __nv_bfloat16* __restrict__ bias, int lane, float (&b)[8]) {
  const uint4 raw = *reinterpret_cast<const uint4*>(bias + lane * 8);
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(p[j]);
    b[2 * j] = f.x;
    b[2 * j + 1] = f.y;
  }
}

// One warp routes one token.  With chunk_masks (zeroed beforehand), the token's
// bit is set in the mask of each selected local expert for the token's chunk of 128.
__global__ void __launch_bounds__(kRouteThreads) route_kernel(const float* __restrict__ logits,
                                                              const __nv_bfloat16* __restrict__ bias, int T,
                                                              float rsf, int32_t* __restrict__ topk_idx,
                                                              float* __restrict__ topk_w, int E, int offset,
                                                              uint32_t* __restrict__ chunk_masks) {
  grid_dep_wait();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (kRouteThreads / 32) + (threadIdx.x >> 5);
  if (t >= T) return;
  float b[8];
  load_bias8(bias, lane, b);
  int e;
  float w;
  route_one_token(logits + static_cast<size_t>(t) * kEG, b, rsf, lane, e, w);
  if (lane < 8) {
    topk_idx[static_cast<size_t>(t) * kTopK + lane] = e;
    topk_w[static_cast<size_t>(t) * kTopK + lane] = w;
    if (chunk_masks) {
      const int le = e - offset;
      const int tl = t & (kChunkTokens - 1);
      if (le >= 0 && le < E)
        atomicOr(&chunk_masks[(static_cast<size_t>(t / kChunkTokens) * E + le) * 4 + (tl >> 5)], 1u << (tl & 31));
    }
  }
}

// Token bitmasks per local expert from externally supplied routing (expert-parallel receive side).
__global__ void __launch_bounds__(256) masks_from_topk_kernel(const RowLayout in, int T, int E, int offset,
                                                              uint4* __restrict__ chunk_masks, int* status) {
  grid_dep_wait();
  __shared__ uint32_t masks[kMaxLocalExperts * 4];
  const int chunk = blockIdx.x;
  for (int i = threadIdx.x; i < E * 4; i += blockDim.x) masks[i] = 0u;
  __syncthreads();
  for (int p = threadIdx.x; p < kChunkTokens * kTopK; p += blockDim.x) {
    const int tl = p >> 3;
    const int t = chunk * kChunkTokens + tl;
    if (t >= T) break;
    const int e = in.idx(t, p & 7);
    if (e >= kEG) record_error(status, KF_STATUS_BAD_EXPERT);
    const int le = e - offset;
    if (e >= 0 && le >= 0 && le < E) atomicOr(&masks[le * 4 + (tl >> 5)], 1u << (tl & 31));
  }
  __syncthreads();
  uint4* dst = chunk_masks + static_cast<size_t>(chunk) * E;
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    dst[e] = make_uint4(masks[e * 4], masks[e * 4 + 1], masks[e * 4 + 2], masks[e * 4 + 3]);
}

__device__ __forceinline__ int popc4(uint4 m) { return __popc(m.x) + __popc(m.y) + __popc(m.z) + __popc(m.w); }

// One block; thread e owns local expert e.  Running counts over chunks give each
// chunk's base inside the expert's segment (stable: chunk order = token order).
// Each expert's rows are one 128-aligned segment, cut into 128-row tiles.
__global__ void __launch_bounds__(kMaxLocalExperts) permute_scan_kernel(
    const uint4* __restrict__ chunk_masks, int nchunk, int E, Meta* __restrict__ meta,
    int32_t* __restrict__ chunk_base, int32_t* __restrict__ tile_expert, int32_t* __restrict__ tile_row0,
    int32_t* __restrict__ tile_rows, int nt_cap, int* status) {
  grid_dep_wait();
  grid_dep_trigger();
  __shared__ int32_t tiles_scan[kMaxLocalExperts];
  __shared__ int32_t pairs_scan[kMaxLocalExperts];
  const int e = threadIdx.x;
  int run = 0;
  if (e < E) {
    int c = 0;
    for (; c + 4 <= nchunk; c += 4) {
      const uint4 m0 = chunk_masks[static_cast<size_t>(c) * E + e];
      const uint4 m1 = chunk_masks[static_cast<size_t>(c + 1) * E + e];
      const uint4 m2 = chunk_masks[static_cast<size_t>(c + 2) * E + e];
      const uint4 m3 = chunk_masks[static_cast<size_t>(c + 3) * E + e];
      chunk_base[static_cast<size_t>(c) * E + e] = run;
      run += popc4(m0);
      chunk_base[static_cast<size_t>(c + 1) * E + e] = run;
      run += popc4(m1);
      chunk_base[static_cast<size_t>(c + 2) * E + e] = run;
      run += popc4(m2);
      chunk_base[static_cast<size_t>(c + 3) * E + e] = run;
      run += popc4(m3);
    }
    for (; c < nchunk; ++c) {
      chunk_base[static_cast<size_t>(c) * E + e] = run;
      run += popc4(chunk_masks[static_cast<size_t>(c) * E + e]);
    }
  }
  const int ntiles = (run + kBlk - 1) / kBlk;
  tiles_scan[e] = ntiles;
  pairs_scan[e] = run;
  __syncthreads();
  // inclusive Hillis-Steele scans over 256 entries
  for (int off = 1; off < kMaxLocalExperts; off <<= 1) {
    const int a = (e >= off) ? tiles_scan[e - off] : 0;
    const int b = (e >= off) ? pairs_scan[e - off] : 0;
    __syncthreads();
    tiles_scan[e] += a;
    pairs_scan[e] += b;
    __syncthreads();
  }
  const int tstart = tiles_scan[e] - ntiles;
  const int total_tiles = tiles_scan[kMaxLocalExperts - 1];
  if (e < E) {
    meta->expert_count[e] = run;
    meta->expert_pad_start[e] = tstart * kBlk;
    for (int i = 0; i < ntiles; ++i) {
      const int ti = tstart + i;
      if (ti >= nt_cap) {
        record_error(status, KF_STATUS_SLOT_OVERFLOW);
        break;
      }
      tile_expert[ti] = e;
      tile_row0[ti] = ti * kBlk;
      tile_rows[ti] = min(kBlk, run - i * kBlk);
    }
  }
  if (e == 0) {
    meta->num_tiles = min(total_tiles, nt_cap);
    meta->num_pairs = pairs_scan[kMaxLocalExperts - 1];
  }
}

// A token's row of token_slot lists its permuted rows in ascending order (the
// local experts ascending: segments lie in expert order), then -1 for the other
// pairs, so the reduce reads them in the reference's index_add_ order with no
// sort.  A local expert repeated among a token's ids (outside the routing
// contract) counts once, at its first position, so every listed row is distinct.
__device__ __forceinline__ bool pair_is_local_first(const int32_t* ids, int k, int offset, int E) {
  const int e = ids[k], le = e - offset;
  if (e < 0 || le < 0 || le >= E) return false;
#pragma unroll
  for (int j = 0; j < kTopK; ++j)
    if (j < k && ids[j] == e) return false;
  return true;
}

// Position of pair k in its token's token_slot row (ids = the token's 8 ids).
__device__ __forceinline__ int token_slot_position(const int32_t* ids, int k, int offset, int E) {
  uint32_t local = 0;  // bit j: pair j is listed as a row
#pragma unroll
  for (int j = 0; j < kTopK; ++j) local |= pair_is_local_first(ids, j, offset, E) ? (1u << j) : 0u;
  if ((local >> k) & 1u) {
    const int e = ids[k];
    int pos = 0;
#pragma unroll
    for (int j = 0; j < kTopK; ++j) pos += (((local >> j) & 1u) && ids[j] < e) ? 1 : 0;
    return pos;
  }
  return __popc(local) + __popc(~local & ((1u << k) - 1u));
}

// Per chunk: each local pair gets its permuted row (slot) = expert segment start +
// pairs of that expert in earlier chunks + earlier tokens of this chunk with the
// same expert (popcount of the mask below the token).  Stable and deterministic:
// the order inside an expert's segment is token order, as the reference's
// stable argsort gives (solution/triton/kernel.py:67-69).
__global__ void __launch_bounds__(256) permute_assign_kernel(
    const RowLayout in, const uint4* __restrict__ chunk_masks,
    const int32_t* __restrict__ chunk_base, const Meta* __restrict__ meta, int T, int E, int offset, int p_cap,
    int32_t* __restrict__ token_slot, int32_t* __restrict__ slot_token, float* __restrict__ slot_weight,
    int32_t* __restrict__ slot_pair, int* status) {
  grid_dep_wait();
  __shared__ uint4 masks[kMaxLocalExperts];
  __shared__ int32_t base[kMaxLocalExperts];
  __shared__ int32_t ids[kChunkTokens * kTopK];
  const int chunk = blockIdx.x;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    masks[e] = chunk_masks[static_cast<size_t>(chunk) * E + e];
    base[e] = meta->expert_pad_start[e] + chunk_base[static_cast<size_t>(chunk) * E + e];
  }
  for (int p = threadIdx.x; p < kChunkTokens * kTopK; p += blockDim.x) {
    const int t = chunk * kChunkTokens + (p >> 3);
    ids[p] = t < T ? in.idx(t, p & 7) : -1;
  }
  __syncthreads();
  for (int p = threadIdx.x; p < kChunkTokens * kTopK; p += blockDim.x) {
    const int tl = p >> 3;
    const int t = chunk * kChunkTokens + tl;
    if (t >= T) break;
    const size_t ti = static_cast<size_t>(t) * kTopK + (p & 7);
    const int le = ids[p] - offset;
    int slot = -1;
    if (pair_is_local_first(ids + tl * kTopK, p & 7, offset, E)) {
      const uint4 m = masks[le];
      const int w = tl >> 5;
      const uint32_t below = (1u << (tl & 31)) - 1u;
      int r = __popc((w == 0 ? m.x : w == 1 ? m.y : w == 2 ? m.z : m.w) & below);
      if (w > 0) r += __popc(m.x);
      if (w > 1) r += __popc(m.y);
      if (w > 2) r += __popc(m.z);
      slot = base[le] + r;
      if (slot >= p_cap) {
        record_error(status, KF_STATUS_SLOT_OVERFLOW);
        slot = -1;
      } else {
        slot_token[slot] = t;
        slot_weight[slot] = in.w(t, p & 7);
        slot_pair[slot] = static_cast<int32_t>(ti);
      }
    }
    token_slot[static_cast<size_t>(t) * kTopK + token_slot_position(ids + tl * kTopK, p & 7, offset, E)] = slot;
  }
}

// Copies each permuted row's FP8 hidden row (7168 bytes) and its 56 scales into
// the expert-contiguous A buffer.  Rows: one warp per row, grid-strided over all
// row tiles so every SM streams; padding rows of a tile are skipped.  Scales: one
// warp per 32 consecutive rows, so the K-block-major scale array is written in
// whole 128-byte runs.
__global__ void __launch_bounds__(256) gather_rows_kernel(const Meta* __restrict__ meta,
                                                          const int32_t* __restrict__ tile_rows,
                                                          const int32_t* __restrict__ slot_token,
                                                          const RowLayout in, int p_cap,
                                                          uint8_t* __restrict__ a_rows,
                                                          float* __restrict__ a_scale) {
  grid_dep_wait();
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int gw = blockIdx.x * warps + (threadIdx.x >> 5), nw = gridDim.x * warps;
  // the rows: one warp per row, every load of the row issued before the first store
  const int nrows = meta->num_tiles * kBlk;
  for (int r = gw; r < nrows; r += nw) {
    if ((r & (kBlk - 1)) >= tile_rows[r >> 7]) continue;
    const int t = slot_token[r];
    const uint4* src = reinterpret_cast<const uint4*>(in.row(t));
    uint4* dst = reinterpret_cast<uint4*>(a_rows + static_cast<size_t>(r) * kH);
    uint4 v[kH / 16 / 32];
#pragma unroll
    for (int j = 0; j < kH / 16 / 32; ++j) v[j] = src[lane + 32 * j];
#pragma unroll
    for (int j = 0; j < kH / 16 / 32; ++j) dst[lane + 32 * j] = v[j];
  }
  // the scales ([56][p_cap], K-block-major): one warp per 32 consecutive rows, lane
  // = row, so each of a warp's stores fills 128 contiguous bytes (one store per row
  // and K block would write 56 separate sectors per row)
  const int nblk = meta->num_tiles * (kBlk / 32);
  for (int b = gw; b < nblk; b += nw) {
    const int rb = b * 32;
    const int n = tile_rows[rb >> 7] - (rb & (kBlk - 1));  // real rows in this block (<= 0: none)
    if (n <= 0) continue;
    const bool live = lane < n;
    const int t = live ? slot_token[rb + lane] : 0;
    float* dst = a_scale + rb + lane;
#pragma unroll
    for (int kb0 = 0; kb0 < kHB; kb0 += 8) {
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = live ? in.sc(t, kb0 + i) : 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (live) dst[static_cast<size_t>(kb0 + i) * p_cap] = v[i];
    }
  }
}

// Whole front end for a call of at most 128 tokens in ONE block (decode sizes,
// where launch latency dominates): routing (or loading pre-routed ids), the
// per-expert token masks, counts and the tile lists, stable slot assignment and
// the gather of FP8 rows and scales -- the work of route / scan / assign /
// gather_rows, with every intermediate in shared memory.  With at most 128
// tokens an expert has at most 128 rows: one 128-row tile, one pair tile.
constexpr int kFrontThreads = 1024;

__global__ void __launch_bounds__(kFrontThreads) front_small_kernel(
    const float* __restrict__ logits, const __nv_bfloat16* __restrict__ bias, float rsf, const RowLayout in, int T,
    int E, int offset, int p_cap, Meta* __restrict__ meta,
    int32_t* __restrict__ tile_expert, int32_t* __restrict__ tile_row0, int32_t* __restrict__ tile_rows,
    int32_t* __restrict__ token_slot, int32_t* __restrict__ slot_token, float* __restrict__ slot_weight,
    int32_t* __restrict__ slot_pair, uint8_t* __restrict__ a_rows, float* __restrict__ a_scale, int* status) {
  grid_dep_wait();
  grid_dep_trigger();
  __shared__ uint32_t masks[kMaxLocalExperts * 4];
  __shared__ int32_t tk[kChunkTokens * kTopK];
  __shared__ float tw[kChunkTokens * kTopK];
  __shared__ int32_t pad_start[kMaxLocalExperts];
  __shared__ int32_t warp_sums[kMaxLocalExperts / 32];
  __shared__ int2 pairs[kChunkTokens * kTopK];
  __shared__ int npairs, total_pairs;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  __shared__ int bad_expert;
  for (int i = tid; i < kMaxLocalExperts * 4; i += kFrontThreads) masks[i] = 0u;
  if (tid == 0) {
    npairs = 0;
    total_pairs = 0;
    bad_expert = 0;
    // this kernel starts the call: it clears the call's status word (every bit is
    // recorded after the block barrier below, or by a later kernel)
    *status = 0;
  }
  // routing, or the caller's routing
  if (logits) {
    float b[8];
    load_bias8(bias, lane, b);
    for (int t = warp; t < T; t += kFrontThreads / 32) {
      int e;
      float w;
      route_one_token(logits + static_cast<size_t>(t) * kEG, b, rsf, lane, e, w);
      if (lane < 8) {
        tk[t * kTopK + lane] = e;
        tw[t * kTopK + lane] = w;
      }
    }
  } else {
    for (int p = tid; p < T * kTopK; p += kFrontThreads) {
      const int e = in.idx(p >> 3, p & 7);
      if (e >= kEG) bad_expert = 1;
      tk[p] = e;
      tw[p] = in.w(p >> 3, p & 7);
    }
  }
  __syncthreads();
  if (tid == 0 && bad_expert) record_error(status, KF_STATUS_BAD_EXPERT);
  for (int p = tid; p < T * kTopK; p += kFrontThreads) {
    const int e = tk[p], le = e - offset, t = p >> 3;
    if (e >= 0 && le >= 0 && le < E) atomicOr(&masks[le * 4 + (t >> 5)], 1u << (t & 31));
  }
  __syncthreads();
  // counts, 128-aligned segments and the tile lists (an expert has 0 or 1 tile)
  int cnt = 0, nt = 0;
  if (tid < E) {
    cnt = __popc(masks[tid * 4]) + __popc(masks[tid * 4 + 1]) + __popc(masks[tid * 4 + 2]) +
          __popc(masks[tid * 4 + 3]);
    nt = cnt > 0 ? 1 : 0;
    atomicAdd(&total_pairs, cnt);
  }
  int incl = nt;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += n;
  }
  if (lane == 31 && warp < kMaxLocalExperts / 32) warp_sums[warp] = incl;
  __syncthreads();
  if (tid < kMaxLocalExperts) {
    int base = 0, total = 0;
    for (int w = 0; w < kMaxLocalExperts / 32; ++w) {
      if (w < warp) base += warp_sums[w];
      total += warp_sums[w];
    }
    const int tstart = base + incl - nt;
    if (tid < E) {
      pad_start[tid] = tstart * kBlk;
      meta->expert_count[tid] = cnt;
      meta->expert_pad_start[tid] = tstart * kBlk;
      if (nt) {
        tile_expert[tstart] = tid;
        tile_row0[tstart] = tstart * kBlk;
        tile_rows[tstart] = cnt;
      }
    }
    if (tid == 0) meta->num_tiles = total;
  }
  __syncthreads();
  if (tid == 0) meta->num_pairs = total_pairs;
  // stable slots: segment start + earlier tokens of the same expert
  for (int p = tid; p < T * kTopK; p += kFrontThreads) {
    const int le = tk[p] - offset, t = p >> 3;
    int slot = -1;
    if (pair_is_local_first(tk + t * kTopK, p & 7, offset, E)) {
      const int w = t >> 5;
      int r = __popc(masks[le * 4 + w] & ((1u << (t & 31)) - 1u));
      for (int q = 0; q < w; ++q) r += __popc(masks[le * 4 + q]);
      slot = pad_start[le] + r;
      if (slot >= p_cap) {
        record_error(status, KF_STATUS_SLOT_OVERFLOW);
        slot = -1;
      } else {
        slot_token[slot] = t;
        slot_weight[slot] = tw[p];
        slot_pair[slot] = p;
        pairs[atomicAdd(&npairs, 1)] = make_int2(t, slot);
      }
    }
    token_slot[t * kTopK + token_slot_position(tk + t * kTopK, p & 7, offset, E)] = slot;
  }
  __syncthreads();
  // gather: one warp per half row of a local pair (7 x 16 bytes a lane, within
  // the 64 registers a 1024-thread block allows), the first half also copying
  // the row's 56 scales; every load is issued before the first store
  const int n = npairs;
  constexpr int kHalf = kH / 16 / 32 / 2;  // 7 uint4 per lane
  for (int i = warp; i < 2 * n; i += kFrontThreads / 32) {
    const int2 ts = pairs[i >> 1];
    const int h = i & 1;
    const uint4* src = reinterpret_cast<const uint4*>(in.row(ts.x)) + h * kHalf * 32;
    uint4* dst = reinterpret_cast<uint4*>(a_rows + static_cast<size_t>(ts.y) * kH) + h * kHalf * 32;
    uint4 v[kHalf];
#pragma unroll
    for (int j = 0; j < kHalf; ++j) v[j] = src[lane + 32 * j];
    float sc0 = 0.f, sc1 = 0.f;
    if (h == 0) {
      sc0 = in.sc(ts.x, lane);
      if (lane + 32 < kHB) sc1 = in.sc(ts.x, lane + 32);
    }
#pragma unroll
    for (int j = 0; j < kHalf; ++j) dst[lane + 32 * j] = v[j];
    if (h == 0) {
      a_scale[static_cast<size_t>(lane) * p_cap + ts.y] = sc0;
      if (lane + 32 < kHB) a_scale[static_cast<size_t>(lane + 32) * p_cap + ts.y] = sc1;
    }
  }
}

// out[t] = sum of the token's permuted rows of y (already routing-weighted and
// stored in bf16), in ascending row order (= ascending local expert, the
// reference's index_add_ order), accumulated in fp32 from zero and rounded
// once.  With few tokens (T * 4 or T * 2 within the grid) 4 or 2 CTAs share each
// token, one column slice each, so the loads spread over more SMs (T = 16:
// 9.7 -> 7.6 us).  Each group of CTAs walks its tokens t = group + i * groups in
// batches of whole tokens with at most kReduceBatch rows between them: warp 0
// lists a batch's rows and output rows in shared memory, then each thread loads
// its 8 columns (16 bytes of bf16) of every row of the batch at once and sums
// them token by token.  So a call whose tokens have one local row each (a GPU
// holding 32 of the 256 experts) keeps as many loads in flight as one whose
// tokens have eight.
constexpr int kReduceThreads = 448;   // 14 warps: a row's 896 groups of 8 columns in 2 passes
constexpr int kReduceBatch = 8;       // rows of y per batch (a token has at most 8)
constexpr int kMaxWorld = 64;

__device__ __forceinline__ uint32_t bf16x2_word(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Columns 8c .. 8c+7 of an output row: one 16-byte bf16 store, or two fp32 ones.
__device__ __forceinline__ void reduce_store(char* row, bool f32, int c, const float4& a, const float4& b) {
  if (!row) return;
  if (f32) {
    reinterpret_cast<float4*>(row)[2 * c] = a;
    reinterpret_cast<float4*>(row)[2 * c + 1] = b;
  } else {
    reinterpret_cast<uint4*>(row)[c] =
        make_uint4(bf16x2_word(a.x, a.y), bf16x2_word(a.z, a.w), bf16x2_word(b.x, b.y), bf16x2_word(b.z, b.w));
  }
}

__device__ __forceinline__ void add_bf16x8(float4& a, float4& b, const uint4& v) {
  const float2 p0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.x));
  const float2 p1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.y));
  const float2 p2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.z));
  const float2 p3 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.w));
  a.x += p0.x;
  a.y += p0.y;
  a.z += p1.x;
  a.w += p1.y;
  b.x += p2.x;
  b.y += p2.y;
  b.z += p3.x;
  b.w += p3.y;
}

__global__ void __launch_bounds__(kReduceThreads, 2) unpermute_reduce_kernel(const int32_t* __restrict__ token_slot,
                                                     const __nv_bfloat16* __restrict__ y, int T, void* __restrict__ out,
                                                     int out_fp32, const PeerOut po, int csplit) {
  grid_dep_wait();
  // Peer return: received row t came from source s (sources in rank order) as the
  // j-th of s's rows for this rank; it goes back to row (s's rows for lower ranks)
  // + j of s's return buffer.  Each CTA builds the map once: src_end[s] = received
  // rows of sources <= s, src_base[s] = (return row) - (received row) for source s.
  __shared__ int32_t src_end[kMaxWorld];
  __shared__ int32_t src_base[kMaxWorld];
  __shared__ int32_t b_slot[kReduceBatch];  // the batch's rows of y, token after token
  __shared__ int32_t b_end[kReduceBatch];   // token j's rows are b_slot[b_end[j-1] .. b_end[j])
  __shared__ char* b_dst[kReduceBatch];     // token j's output row (null: not stored)
  __shared__ int32_t b_tokens;
  if (po.peer_back) {
    const int s = threadIdx.x;
    int n = 0, so = 0;
    if (s < po.world) {
      n = po.counts[s * po.world + po.rank];
      for (int d = 0; d < po.rank; ++d) so += po.counts[s * po.world + d];
      src_end[s] = n;
      src_base[s] = so;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int off = 0;
      for (int q = 0; q < po.world; ++q) {
        src_base[q] -= off;
        off += src_end[q];
        src_end[q] = off;
      }
    }
    __syncthreads();
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool f32 = out_fp32 && !po.peer_back;
  // csplit CTAs share each token, one slice of kH / csplit columns each
  const int cta = static_cast<int>(blockIdx.x) / csplit, ncta = static_cast<int>(gridDim.x) / csplit;
  const int cw = kH / 8 / csplit, c0 = (static_cast<int>(blockIdx.x) % csplit) * cw;  // groups of 8 columns
  const int ntok = cta < T ? (T - 1 - cta) / ncta + 1 : 0;
  for (int i0 = 0; i0 < ntok;) {
    if (warp == 0) {
      // lane l looks at this CTA's token i0 + l; the batch is the longest run of
      // them (at most kReduceBatch tokens) whose rows number at most kReduceBatch
      // -- never empty, as a token has at most 8 rows
      const int i = i0 + lane;
      const int t = cta + i * ncta;
      int4 a = make_int4(-1, -1, -1, -1), b = a;
      if (i < ntok) {
        const int4* ts = reinterpret_cast<const int4*>(token_slot + static_cast<size_t>(t) * kTopK);
        a = ts[0];
        b = ts[1];
      }
      const int sl[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      int n = 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) n += sl[k] >= 0 ? 1 : 0;
      int incl = n;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const bool take = i < ntok && lane < kReduceBatch && incl <= kReduceBatch;
      const unsigned tm = __ballot_sync(0xffffffffu, take);
      if (take) {
        int pos = incl - n;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (sl[k] >= 0) b_slot[pos++] = sl[k];  // listed rows are ascending; -1 only past them
        b_end[lane] = incl;
        char* d = nullptr;
        if (po.peer_back) {
          // a row past the received total has no place in any source's send order
          int s = 0;
          while (s < po.world && t >= src_end[s]) ++s;
          if (s < po.world)
            d = static_cast<char*>(po.peer_back[s]) + static_cast<size_t>(src_base[s] + t) * kH * 2;
        } else {
          d = static_cast<char*>(out) + static_cast<size_t>(t) * kH * (f32 ? 4 : 2);
        }
        b_dst[lane] = d;
      }
      if (lane == 0) b_tokens = __popc(tm);
    }
    __syncthreads();
    const int nt = b_tokens;
    const int ne = b_end[nt - 1];
    for (int c = c0 + threadIdx.x; c < c0 + cw; c += kReduceThreads) {
      uint4 v[kReduceBatch];  // 8 bf16 columns of each of the batch's rows
#pragma unroll
      for (int e = 0; e < kReduceBatch; ++e)
        if (e < ne) v[e] = __ldg(reinterpret_cast<const uint4*>(y + static_cast<size_t>(b_slot[e]) * kH) + c);
      float4 acc0 = make_float4(0.f, 0.f, 0.f, 0.f), acc1 = acc0;
      int j = 0;
      while (j < nt && b_end[j] == 0) reduce_store(b_dst[j++], f32, c, acc0, acc1);  // tokens without a local row
#pragma unroll
      for (int e = 0; e < kReduceBatch; ++e) {
        if (e < ne) {
          add_bf16x8(acc0, acc1, v[e]);
          while (j < nt && b_end[j] == e + 1) {
            reduce_store(b_dst[j++], f32, c, acc0, acc1);
            acc0 = make_float4(0.f, 0.f, 0.f, 0.f);
            acc1 = acc0;
          }
        }
      }
    }
    i0 += nt;
    __syncthreads();  // the batch lists are rewritten next
  }
  if (po.peer_back) __threadfence_system();
}

}  // namespace

cudaError_t launch_route(const float* logits, const void* bias, int T, float rsf, int32_t* topk_idx,
                         float* topk_w, int E, int offset, uint4* chunk_masks, cudaStream_t s) {
  if (chunk_masks) {
    const int nchunk = (T + kChunkTokens - 1) / kChunkTokens;
    const cudaError_t e = cudaMemsetAsync(chunk_masks, 0, static_cast<size_t>(nchunk) * E * sizeof(uint4), s);
    if (e != cudaSuccess) return e;
  }
  const int warps = kRouteThreads / 32;
  return launch_chained(route_kernel, dim3((T + warps - 1) / warps), dim3(kRouteThreads), 0, s, logits, static_cast<const __nv_bfloat16*>(bias), T,
                                                                 rsf, topk_idx, topk_w, E, offset,
                                                                 reinterpret_cast<uint32_t*>(chunk_masks));
}

cudaError_t launch_masks_from_topk(const RowLayout& in, int T, int E, int offset, uint4* chunk_masks, int* status,
                                   cudaStream_t s) {
  const int nchunk = (T + kChunkTokens - 1) / kChunkTokens;
  return launch_chained(masks_from_topk_kernel, dim3(nchunk), dim3(256), 0, s, in, T, E, offset, chunk_masks, status);
}

cudaError_t launch_permute_scan(const uint4* chunk_masks, int nchunk, int E, Meta* meta, int32_t* chunk_base,
                                int32_t* tile_expert, int32_t* tile_row0, int32_t* tile_rows, int nt_cap, int* status,
                                cudaStream_t s) {
  return launch_chained(permute_scan_kernel, dim3(1), dim3(kMaxLocalExperts), 0, s, chunk_masks, nchunk, E, meta,
                        chunk_base, tile_expert, tile_row0, tile_rows, nt_cap, status);
}

cudaError_t launch_permute_assign(const RowLayout& in, const uint4* chunk_masks, const int32_t* chunk_base,
                                  const Meta* meta, int T, int E, int offset, int p_cap, int32_t* token_slot,
                                  int32_t* slot_token, float* slot_weight, int32_t* slot_pair, int* status,
                                  cudaStream_t s) {
  const int nchunk = (T + kChunkTokens - 1) / kChunkTokens;
  return launch_chained(permute_assign_kernel, dim3(nchunk), dim3(256), 0, s, in, chunk_masks, chunk_base, meta, T, E, offset, p_cap, token_slot,
                                               slot_token, slot_weight, slot_pair, status);
}

cudaError_t launch_front_small(const float* logits, const void* bias, float rsf, const RowLayout& in, int T, int E,
                               int offset, int p_cap, Meta* meta, int32_t* tile_expert, int32_t* tile_row0,
                               int32_t* tile_rows, int32_t* token_slot, int32_t* slot_token, float* slot_weight,
                               int32_t* slot_pair, uint8_t* a_rows, float* a_scale, int* status, cudaStream_t s) {
  return launch_chained(front_small_kernel, dim3(1), dim3(kFrontThreads), 0, s, logits,
                        static_cast<const __nv_bfloat16*>(bias), rsf, in, T, E, offset, p_cap, meta, tile_expert,
                        tile_row0, tile_rows, token_slot, slot_token, slot_weight, slot_pair, a_rows, a_scale, status);
}

cudaError_t launch_gather_rows(const Meta* meta, const int32_t* tile_rows, const int32_t* slot_token,
                               const RowLayout& in, int p_cap, uint8_t* a_rows, float* a_scale, int grid,
                               cudaStream_t s) {
  return launch_chained(gather_rows_kernel, dim3(grid), dim3(256), 0, s, meta, tile_rows, slot_token, in, p_cap, a_rows, a_scale);
}

cudaError_t launch_reduce(const int32_t* token_slot, const __nv_bfloat16* y, int T, void* out, int out_fp32, const PeerOut& po,
                          int grid, cudaStream_t s) {
  if (po.peer_back && (po.world < 1 || po.world > kMaxWorld)) return cudaErrorInvalidValue;
  // few tokens: split each token's columns over 2 or 4 CTAs so more SMs share the loads
  const int cs = T * 4 <= grid ? 4 : (T * 2 <= grid ? 2 : 1);
  const int ctas = T < grid / cs ? T : grid / cs;
  return launch_chained(unpermute_reduce_kernel, dim3(ctas * cs), dim3(kReduceThreads), 0, s, token_slot, y,
                        T, out, out_fp32, po, cs);
}

}  // namespace kf
