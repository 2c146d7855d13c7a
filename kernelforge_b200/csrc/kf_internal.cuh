// Internal layout shared by the kernels and the C-ABI layer.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <utility>

#include "kf_moe.h"

namespace kf {

constexpr int kH = KF_MOE_HIDDEN;             // 7168
constexpr int kI = KF_MOE_INTERMEDIATE;       // 2048
constexpr int kEG = KF_MOE_GLOBAL_EXPERTS;    // 256
constexpr int kTopK = KF_MOE_TOP_K;           // 8
constexpr int kBlk = KF_MOE_BLOCK;            // 128 (quantisation block, MMA tile M and K chunk)
constexpr int kHB = kH / kBlk;                // 56 K-blocks of the hidden dimension
constexpr int kIB = kI / kBlk;                // 16 K-blocks of the intermediate dimension
constexpr int kChunkTokens = 128;             // tokens per routing/permute chunk (4 x 32-bit masks)
constexpr int kMaxLocalExperts = 256;

// Token / row counts every entry point accepts: [0, KF_MOE_MAX_TOKENS].
inline bool valid_tokens(int32_t n) { return n >= 0 && n <= KF_MOE_MAX_TOKENS; }

// silu(x) = x * sigmoid(x) for the SwiGLU epilogues, from the identity
// sigmoid(x) = (1 + tanh(x/2)) / 2: silu(x) = h + h * tanh(h) with h = x/2, one
// hardware tanh approximation (relative error about 2^-11, below the 2^-8 of the
// two-term FP8 intermediate it feeds) instead of an exp2 and a reciprocal.  The
// GEMM1 epilogue runs on the special-function unit while the MMA waits, and the
// single-op form measured 2.7 % less GEMM1 time at the config-3 layer.  Finite for
// every finite x, with no special-value path.
__device__ __forceinline__ float silu_f(float x) {
  const float h = 0.5f * x;
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(h));
  return fmaf(h, t, h);
}

// Per-call metadata written by the permute scan, read by the GEMMs and the reduce.
struct Meta {
  int32_t num_tiles;       // row tiles of 128 permuted rows, over all local experts
  int32_t num_pairs;       // local (token, expert) pairs
  int32_t reserved[62];
  int32_t expert_count[kMaxLocalExperts];      // pairs per local expert
  int32_t expert_pad_start[kMaxLocalExperts];  // first permuted row of each expert (128-aligned)
};

// Offsets (bytes) of every scratch array inside the caller's workspace.
struct Workspace {
  size_t status, meta, topk_idx, topk_w, token_slot, chunk_masks, chunk_base;
  size_t tile_expert, tile_row0, tile_rows, slot_token, slot_weight, slot_pair;
  size_t a_rows, a_scale, c_hi, c_lo, c_scale, y, partial;
  size_t total;
  int32_t p_cap;    // capacity in permuted rows (multiple of 128)
  int32_t nt_cap;   // capacity in row tiles
  int32_t nchunk;   // routing/permute chunks of 128 tokens
  int32_t ksplit1;  // split-K factor of GEMM1 (1 = no split)
};

Workspace plan_workspace(int32_t T, int32_t E);

template <typename T>
inline T* ws_ptr(void* base, size_t off) {
  return reinterpret_cast<T*>(static_cast<char*>(base) + off);
}

// Where the per-token inputs of the expert stage live.  The reference layout is
// topk [T][8], hidden [T][7168] and K-major scales [56][T]; the expert-parallel
// receive buffer holds one 7456-byte row per token (hidden | 56 scales | 8 ids |
// 8 weights).  Element (t, k) of a field is base[t * token_stride + k * inner_stride].
struct RowLayout {
  const int32_t* topk_idx;
  const float* topk_w;
  int64_t topk_stride;          // elements between consecutive tokens' 8 ids / weights
  const uint8_t* hidden;
  int64_t hidden_stride;        // bytes between consecutive tokens' rows
  const float* scale;
  int64_t scale_token_stride;   // elements
  int64_t scale_kb_stride;      // elements
  __device__ __forceinline__ int32_t idx(int t, int k) const { return topk_idx[t * topk_stride + k]; }
  __device__ __forceinline__ float w(int t, int k) const { return topk_w[t * topk_stride + k]; }
  __device__ __forceinline__ const uint8_t* row(int t) const { return hidden + t * hidden_stride; }
  __device__ __forceinline__ float sc(int t, int kb) const { return scale[t * scale_token_stride + kb * scale_kb_stride]; }
};

constexpr int64_t kPackedRowBytes = kH + kHB * 4 + kTopK * 4 + kTopK * 4;  // 7456

inline RowLayout reference_layout(const int32_t* topk_idx, const float* topk_w, const void* hidden,
                                  const float* hidden_scale, int T) {
  return RowLayout{topk_idx, topk_w, kTopK, static_cast<const uint8_t*>(hidden), kH, hidden_scale, 1, T};
}

inline RowLayout packed_layout(const void* rows) {
  const uint8_t* b = static_cast<const uint8_t*>(rows);
  return RowLayout{reinterpret_cast<const int32_t*>(b + kH + kHB * 4),
                   reinterpret_cast<const float*>(b + kH + kHB * 4 + kTopK * 4), kPackedRowBytes / 4, b,
                   kPackedRowBytes, reinterpret_cast<const float*>(b + kH), kPackedRowBytes / 4, 1};
}

// Every kernel of the layer's launch chain is launched with programmatic stream
// serialization: it may start while its predecessor in the stream is finishing,
// and begins with grid_dep_wait().
template <typename... KArgs, typename... Args>
cudaError_t launch_chained(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                           Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Kernel launchers (return cudaGetLastError()).
cudaError_t launch_route(const float* logits, const void* bias, int T, float rsf, int32_t* topk_idx,
                         float* topk_w, int E, int offset, uint4* chunk_masks, cudaStream_t s);
cudaError_t launch_masks_from_topk(const RowLayout& in, int T, int E, int offset, uint4* chunk_masks, int* status,
                                   cudaStream_t s);
cudaError_t launch_permute_scan(const uint4* chunk_masks, int nchunk, int E, Meta* meta, int32_t* chunk_base,
                                int32_t* tile_expert, int32_t* tile_row0, int32_t* tile_rows, int nt_cap, int* status,
                                cudaStream_t s);
cudaError_t launch_permute_assign(const RowLayout& in, const uint4* chunk_masks, const int32_t* chunk_base,
                                  const Meta* meta, int T, int E, int offset, int p_cap, int32_t* token_slot,
                                  int32_t* slot_token, float* slot_weight, int32_t* slot_pair, int* status,
                                  cudaStream_t s);
// Single-block front end for T <= kChunkTokens: routing (logits != nullptr) or the
// caller's routing (topk_in), tile lists, slots and the row gather.
cudaError_t launch_front_small(const float* logits, const void* bias, float rsf, const RowLayout& in, int T, int E,
                               int offset, int p_cap, Meta* meta, int32_t* tile_expert, int32_t* tile_row0,
                               int32_t* tile_rows, int32_t* token_slot, int32_t* slot_token, float* slot_weight, int32_t* slot_pair,
                               uint8_t* a_rows, float* a_scale, int* status, cudaStream_t s);
cudaError_t launch_gather_rows(const Meta* meta, const int32_t* tile_rows, const int32_t* slot_token,
                               const RowLayout& in, int p_cap, uint8_t* a_rows, float* a_scale, int grid,
                               cudaStream_t s);
// Expert-parallel receive side over peer memory: the reduce stores each received
// row's bf16 result straight into its source rank's return buffer (row = the
// row's position in the source's send order) instead of into a local output.
struct PeerOut {
  void* const* peer_back;  // device array: rank q's return buffer (bf16 rows), or null for a local output
  const int32_t* counts;   // this rank's [world][world] count matrix
  int rank, world;
};

cudaError_t launch_reduce(const int32_t* token_slot, const __nv_bfloat16* y, int T, void* out, int out_fp32, const PeerOut& po,
                          int grid, cudaStream_t s);

struct Gemm1Args {
  const Meta* meta;
  const int32_t* tile_expert;
  const int32_t* tile_row0;
  const int32_t* tile_rows;
  const float* a_scale;    // [56][p_cap]
  const float* w13_scale;  // [E][32][56]
  uint8_t* c_hi;           // [p_cap][2048] e4m3
  uint8_t* c_lo;           // [p_cap][2048] e4m3
  float* c_scale;          // [16][p_cap]
  int32_t p_cap;
  int* status;
  // Split-K: ksplit CTAs share a (tile, column block),
  // each over 56/ksplit K chunks, and store their fp32 partial sums in `partial`
  // ([ksplit][max_pairs][4096], indexed by the pair id slot_pair[row]);
  // swiglu_quant_kernel then sums them in split order and runs the epilogue.
  int32_t ksplit;
  int32_t max_pairs;
  const int32_t* slot_pair;
  float* partial;
  // 1 when the call has at most 32 tokens (no row tile holds more than 32 rows):
  // GEMM1 then runs its decode layout (32-row A slots, 6 stages)
  int32_t decode;
};

struct Gemm2Args {
  const Meta* meta;
  const int32_t* tile_expert;
  const int32_t* tile_row0;
  const int32_t* tile_rows;
  const float* c_scale;     // [16][p_cap]
  const float* w2_scale;    // [E][56][16]
  const float* slot_weight; // [p_cap]
  __nv_bfloat16* y;         // [p_cap][7168]: each row's routing-weighted output, one bf16 rounding
  int32_t p_cap;
  int* status;
  // 1 when the call has at most 32 tokens, so no row tile holds more than 32
  // rows: GEMM2 then runs its decode layout (32-row A slots, 5 stages)
  int32_t decode;
};

cudaError_t launch_gemm1(const CUtensorMap& tm_a, const CUtensorMap& tm_a32, const CUtensorMap& tm_w13,
                         const Gemm1Args& args, int grid, cudaStream_t s);
// tm_y: bf16 [p_cap, 7168] output rows, box 64 x 32, 128-byte swizzle (TMA stores).
cudaError_t launch_gemm2(const CUtensorMap& tm_chi, const CUtensorMap& tm_clo, const CUtensorMap& tm_chi32,
                         const CUtensorMap& tm_clo32, const CUtensorMap& tm_w2, const CUtensorMap& tm_y,
                         const Gemm2Args& args, int grid, cudaStream_t s);
// Split-K finish of GEMM1 (sum of the splits, SwiGLU, hi/lo encoding).
cudaError_t launch_swiglu_quant(const Gemm1Args& g, int grid, cudaStream_t s);
cudaError_t gemm_set_attributes();

}  // namespace kf
