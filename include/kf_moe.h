/*
 * kf_moe.h -- C ABI of the B200 (sm_100a) fused DeepSeek-V3 FP8 block-scale MoE layer.
 *
 * Definition: moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048
 * (hidden 7168, intermediate 2048, 256 global experts in 8 groups of 32, top-4
 * groups, top-8 experts, FP8 e4m3 operands with fp32 scales per 128 columns of
 * activations and per 128x128 block of weights).
 *
 * The entry points replace the reference's Python operator
 * ``solution/triton/kernel.py::kernel`` (chinmay29/kernelforge):
 *
 *   kf_moe_forward  <- kernel(...)                       kernel.py:1817-1950
 *   kf_moe_route    <- routing inside kernel(...)         kernel.py:1842-1867
 *                      (= _route_topk_ids_and_weights     kernel.py:967-993)
 *   kf_moe_experts  <- sort + grouped GEMM1/SwiGLU +      kernel.py:1869-1925
 *                      grouped GEMM2 + index_add combine  (_sort_tokens :46-82,
 *                                                          _launch_grouped_gemm1_swiglu :626,
 *                                                          _launch_grouped_gemm2 :688)
 *   kf_quantize_hidden <- _quantize_fp8_block_rows        kernel.py:126-141
 *                      (the FP8 format of hidden_states / hidden_states_scale)
 *
 * All pointers are device pointers (except where noted), all tensors are dense
 * row-major, and every call is asynchronous on `stream` (a cudaStream_t, NULL =
 * legacy default stream).  Calls never synchronise the host and never allocate:
 * scratch memory is the caller's `workspace` of kf_moe_workspace_bytes() bytes.
 * Return value: KF_OK or a KF_ERR_* code (argument / launch errors only; errors
 * found on the device are reported through kf_moe_read_status).
 */
#ifndef KF_MOE_H_
#define KF_MOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KF_MOE_HIDDEN 7168
#define KF_MOE_INTERMEDIATE 2048
#define KF_MOE_GLOBAL_EXPERTS 256
#define KF_MOE_TOP_K 8
#define KF_MOE_N_GROUP 8
#define KF_MOE_TOPK_GROUP 4
#define KF_MOE_BLOCK 128

/* Largest num_tokens / num_rows any entry point accepts (larger values are
 * KF_ERR_INVALID_ARGUMENT, and the size queries return 0).  It keeps every row
 * count, tile count and workspace offset inside 32-bit indexes; the workspace of
 * such a call would already be terabytes, far beyond one GPU's memory. */
#define KF_MOE_MAX_TOKENS (1 << 24)

/* Host-side return codes. */
#define KF_OK 0
#define KF_ERR_INVALID_ARGUMENT 1
#define KF_ERR_WORKSPACE_TOO_SMALL 2
#define KF_ERR_CUDA 3
#define KF_ERR_UNSUPPORTED_DEVICE 4
#define KF_ERR_DRIVER_ENTRY_POINT 5
#define KF_ERR_DEVICE_STATUS 6
#define KF_ERR_EXCEEDS_STATIC_SCRATCH 7

/* Device status bits (OR-ed into the workspace status word by the kernels). */
#define KF_STATUS_TIMEOUT_PRODUCER 0x01 /* a TMA producer waited too long for a free stage */
#define KF_STATUS_TIMEOUT_MMA 0x02      /* the MMA issuer waited too long for data / TMEM */
#define KF_STATUS_TIMEOUT_EPILOGUE 0x04 /* a promotion/epilogue warp waited too long */
#define KF_STATUS_BAD_EXPERT 0x08       /* a routed expert id outside [0, 256) */
#define KF_STATUS_SLOT_OVERFLOW 0x10    /* a permuted row index beyond the workspace capacity */
#define KF_STATUS_TIMEOUT_PEER 0x20     /* a peer rank did not reach kf_ep_barrier in time */

/*
 * Bytes of scratch memory a call with `num_tokens` tokens and `num_local_experts`
 * local experts needs (sized for the worst case: every token routed to
 * min(8, E) local experts).  Replaces the torch allocations the reference makes
 * inside kernel(...).
 */
size_t kf_moe_workspace_bytes(int32_t num_tokens, int32_t num_local_experts);

/*
 * The whole layer, value-returning in the reference; here the caller passes the
 * output buffer.
 *   routing_logits      f32  [T, 256]
 *   routing_bias        bf16 [256]
 *   hidden_states       e4m3 [T, 7168]
 *   hidden_states_scale f32  [56, T]
 *   gemm1_weights       e4m3 [E, 4096, 7168]   rows [0,2048) = up (X1), [2048,4096) = gate (X2)
 *   gemm1_weights_scale f32  [E, 32, 56]
 *   gemm2_weights       e4m3 [E, 7168, 2048]
 *   gemm2_weights_scale f32  [E, 56, 16]
 *   output              bf16 [T, 7168]
 * Local experts are global ids [local_expert_offset, local_expert_offset + E);
 * tokens routed to no local expert produce zero rows.  1 <= E <= 256.
 */
int kf_moe_forward(const float* routing_logits, const void* routing_bias,
                   const void* hidden_states, const float* hidden_states_scale,
                   const void* gemm1_weights, const float* gemm1_weights_scale,
                   const void* gemm2_weights, const float* gemm2_weights_scale,
                   int32_t num_tokens, int32_t num_local_experts, int32_t local_expert_offset,
                   float routed_scaling_factor, void* output,
                   void* workspace, size_t workspace_bytes, void* stream);

/*
 * Routing only.  topk_idx int32 [T, 8] receives the selected global expert ids
 * in descending biased-score order (ties: lowest expert id first); topk_weight
 * f32 [T, 8] the matching normalised, scaled weights.
 */
int kf_moe_route(const float* routing_logits, const void* routing_bias, int32_t num_tokens,
                 float routed_scaling_factor, int32_t* topk_idx, float* topk_weight, void* stream);

/*
 * Experts only, on pre-routed rows (the expert-parallel receive side).
 * topk_idx int32 [T, 8] holds global expert ids or -1 (no expert); entries
 * outside the local range are skipped.  A row's ids must be distinct.
 * output: bf16 [T, 7168] when output_fp32 == 0, else f32 [T, 7168].
 */
int kf_moe_experts(const int32_t* topk_idx, const float* topk_weight,
                   const void* hidden_states, const float* hidden_states_scale,
                   const void* gemm1_weights, const float* gemm1_weights_scale,
                   const void* gemm2_weights, const float* gemm2_weights_scale,
                   int32_t num_tokens, int32_t num_local_experts, int32_t local_expert_offset,
                   void* output, int32_t output_fp32,
                   void* workspace, size_t workspace_bytes, void* stream);

/*
 * Experts on rows in the expert-parallel packed layout: `rows` holds num_rows
 * rows of 7456 bytes (FP8 hidden row [7168] | f32 scales [56] | int32 global
 * expert ids [8], -1 = none | f32 weights [8]), as kf_ep_dispatch writes them
 * and the all-to-all delivers them.  Same computation as kf_moe_experts, read
 * in place (no unpacking copy).  Expert-parallel receive side; the reference
 * has no multi-GPU path (its data contract's local_expert_offset,
 * kernel.py:1826, is what the shards use).
 */
int kf_moe_experts_packed(const void* rows, const void* gemm1_weights, const float* gemm1_weights_scale,
                          const void* gemm2_weights, const float* gemm2_weights_scale, int32_t num_rows,
                          int32_t num_local_experts, int32_t local_expert_offset, void* output, int32_t output_fp32,
                          void* workspace, size_t workspace_bytes, void* stream);

/*
 * Expert-parallel dispatch (no reference counterpart: the reference has no
 * multi-GPU code).  Rank r of `world` owns experts [r*256/world, (r+1)*256/world).
 * For the rank's T routed tokens (topk_idx/topk_weight [T, 8], hidden [T, 7168],
 * scales [56, T]) writes:
 *   send_rows   [kf_ep_max_send_rows(T, world)][7456]: one packed row per (token,
 *               destination owning >= 1 of its experts), grouped by destination,
 *               token order inside a destination; ids the destination does not
 *               own are -1 (weight 0)
 *   send_counts int64 [world] (device): rows per destination
 *   pos         int32 [T, world]: row of (token, destination), -1 if not sent
 * `workspace`: kf_ep_workspace_bytes(T, world) bytes.  world divides 256, <= 64.
 */
size_t kf_ep_workspace_bytes(int32_t num_tokens, int32_t world);
int32_t kf_ep_max_send_rows(int32_t num_tokens, int32_t world);
int kf_ep_dispatch(const int32_t* topk_idx, const float* topk_weight, const void* hidden_states,
                   const float* hidden_states_scale, int32_t num_tokens, int32_t world, void* send_rows,
                   int64_t* send_counts, int32_t* pos, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Expert-parallel combine: output[t] (bf16 [T, 7168]) = sum over destinations d
 * in ascending order of partials[pos[t, d]] (rows of bf16, or f32 when
 * partials_fp32), accumulated in f32 and rounded once.
 */
/*
 * Expert-parallel exchange over peer memory (NVLink / NVSwitch), replacing the
 * two NCCL all-to-alls of the dispatch / combine above with stores into the
 * ranks' symmetric buffers (one allocation per rank at the same layout, mapped
 * into every peer).  Arrays named peer_* are DEVICE arrays of `world` device
 * pointers, entry q pointing into rank q's buffer.  A step, on every rank:
 *
 *   kf_ep_plan_p2p    masks + scan (as kf_ep_dispatch) and publishes this rank's
 *                     per-destination row counts as row `rank` of every rank's
 *                     [world][world] int32 count matrix (peer_counts)
 *   kf_ep_barrier     all count rows have landed
 *   kf_ep_pack_p2p    packs each (token, destination) row (kf_ep_dispatch's
 *                     format) straight into rank d's receive buffer (peer_recv),
 *                     sources in rank order, and writes pos as kf_ep_dispatch;
 *                     with hidden_states_scale == NULL, hidden_states are bf16
 *                     rows [T][7168] and every packed row is quantised on the
 *                     way out exactly as kf_quantize_hidden would (the upstream
 *                     quantisation fused into the dispatch)
 *   kf_ep_barrier     all rows have landed; this rank received
 *                     sum over s of counts[s][rank] rows
 *   (kf_moe_experts_packed on the received rows -> bf16 partials)
 *   kf_ep_return_p2p  sends each partial row back into its source's return
 *                     buffer (peer_back) at the row's position in the source's
 *                     send order
 *   kf_ep_barrier     all partials have landed; kf_ep_combine(return buffer, pos)
 *
 * Every rank's receive area holds recv_capacity rows (the same on all ranks; a
 * row beyond it is dropped and sets KF_STATUS_SLOT_OVERFLOW in *status), which
 * the caller sizes from the complete count matrix available after the first
 * barrier.  counts is this rank's own (complete) count matrix.  The return
 * (kf_ep_return_p2p, kf_moe_experts_packed_p2p) stores only the first
 * sum over s of counts[s][rank] rows: rows past that total have no position in
 * any source's send order, so a num_rows larger than the total never writes
 * into a peer's buffer outside that source's own rows.  The barrier stores `epoch`
 * (one more than the previous barrier's) into slot `rank` of every rank's int32
 * flag array (peer_flags; zeroed before the first barrier) and waits, bounded,
 * until its own flags (my_flags) all reach it; a rank that does not arrive sets
 * KF_STATUS_TIMEOUT_PEER in *status (device int) instead of hanging.  The
 * reference has no multi-GPU path (the layer's data contract carries
 * local_expert_offset, kernel.py:1826).
 */
/*
 * kf_moe_experts_packed for the peer exchange, with the return fused into its
 * last kernel: instead of writing the bf16 partials locally (for
 * kf_ep_return_p2p to send), the reduce stores each received row's partial
 * straight into its source rank's return buffer (peer_back), at the row's
 * position in the source's send order.  Call it between the second and third
 * kf_ep_barrier of a step.
 */
int kf_moe_experts_packed_p2p(const void* rows, const void* gemm1_weights, const float* gemm1_weights_scale,
                              const void* gemm2_weights, const float* gemm2_weights_scale, int32_t num_rows,
                              int32_t num_local_experts, int32_t local_expert_offset, const int32_t* counts,
                              int32_t rank, int32_t world, void* const* peer_back, void* workspace,
                              size_t workspace_bytes, void* stream);

int kf_ep_plan_p2p(const int32_t* topk_idx, int32_t num_tokens, int32_t world, int32_t rank,
                   int32_t* const* peer_counts, void* workspace, size_t workspace_bytes, void* stream);
int kf_ep_pack_p2p(const int32_t* topk_idx, const float* topk_weight, const void* hidden_states,
                   const float* hidden_states_scale, int32_t num_tokens, int32_t world, int32_t rank,
                   const int32_t* counts, uint8_t* const* peer_recv, int32_t recv_capacity, int32_t* pos,
                   int32_t* status, void* workspace, size_t workspace_bytes, void* stream);
int kf_ep_return_p2p(const void* partials, int32_t num_rows, int32_t world, int32_t rank, const int32_t* counts,
                     void* const* peer_back, void* stream);
int kf_ep_barrier(int32_t* const* peer_flags, const int32_t* my_flags, int32_t rank, int32_t world, int32_t epoch,
                  int32_t* status, void* stream);

int kf_ep_combine(const void* partials, int32_t partials_fp32, const int32_t* pos, int32_t num_tokens,
                  int32_t world, void* output, void* stream);

/*
 * FP8 block quantisation of bf16 rows into the layer's input format (the step
 * before kf_moe_forward): x bf16 [T, 7168] -> out e4m3 [T, 7168] and out_scale
 * f32 [56, T] (K-block major, as hidden_states_scale), per row and 128 columns
 * scale = absmax / 448 (1 for an all-zero block), out = e4m3(x / scale) rounded
 * to nearest even.  x and out must be 16-byte aligned.  Inputs holding NaN or
 * infinity are outside the contract (the block maximum skips NaN).
 */
int kf_quantize_hidden(const void* x, int32_t num_tokens, void* out, float* out_scale, void* stream);

/*
 * Synchronises `stream`, then copies the device status word of the last call
 * that used `workspace` into *status (host pointer) and clears it.  Returns
 * KF_ERR_DEVICE_STATUS if any bit was set.
 */
int kf_moe_read_status(void* workspace, int32_t* status, void* stream);

/* Limits of kf_moe_forward_noalloc and the size of its static scratch array. */
#define KF_MOE_NOALLOC_MAX_TOKENS 16
#define KF_MOE_NOALLOC_MAX_LOCAL_EXPERTS 32
#define KF_MOE_NOALLOC_SCRATCH_BYTES (176u << 20) /* 176 MiB */

/*
 * kf_moe_forward for callers that cannot allocate device memory.  This entry
 * point has no counterpart in the reference (its kernel() allocates through
 * torch on every call).
 *
 * Some callers cannot call cudaMalloc, so they cannot hand kf_moe_forward a
 * workspace: a plugin host that owns all device memory and passes a plugin only
 * its input and output buffers, a host language bound to this C ABI without any
 * CUDA allocation binding, or a serving process whose device memory is already
 * fully reserved by its own pools.  This variant takes the same inputs and
 * output but no workspace: its scratch memory is a file-scope static device
 * array of KF_MOE_NOALLOC_SCRATCH_BYTES, which every GPU that loads this library
 * holds until the process exits.  It calls no cudaMalloc, cudaFree or other
 * allocating routine.
 *
 * Limits: num_tokens <= KF_MOE_NOALLOC_MAX_TOKENS and num_local_experts <=
 * KF_MOE_NOALLOC_MAX_LOCAL_EXPERTS (decode-sized calls of the e32 layer);
 * larger calls return KF_ERR_EXCEEDS_STATIC_SCRATCH without doing any work.
 * The first call on a device looks up that device's copy of the array (with
 * that device current); make that first call before any stream capture.
 * All calls on a device share the one array, which keeps the previous call's
 * contents (each call clears the status word it needs zeroed and overwrites
 * everything else before reading it): calls that overlap on the GPU -- on
 * different streams or from different threads -- race on it and must be
 * serialised by the caller.  Their device-side status bits are read with
 * kf_moe_noalloc_read_status below, not with kf_moe_read_status.
 */
int kf_moe_forward_noalloc(const float* routing_logits, const void* routing_bias,
                           const void* hidden_states, const float* hidden_states_scale,
                           const void* gemm1_weights, const float* gemm1_weights_scale,
                           const void* gemm2_weights, const float* gemm2_weights_scale,
                           int32_t num_tokens, int32_t num_local_experts, int32_t local_expert_offset,
                           float routed_scaling_factor, void* output, void* stream);

/*
 * Status word of kf_moe_forward_noalloc's calls on the current device, for the
 * same callers (it has no counterpart in the reference either): synchronises
 * `stream`, copies the word into *status (host pointer) and clears it, all
 * without allocating.  Returns KF_ERR_DEVICE_STATUS if any bit was set (a
 * bounded wait that gave up, or a bounds check that failed, in a call since the
 * last read).
 */
int kf_moe_noalloc_read_status(int32_t* status, void* stream);

/* Kernel ids for the profiling counters. */
#define KF_KERNEL_ROUTE 0
#define KF_KERNEL_MASKS 1
#define KF_KERNEL_PERMUTE_SCAN 2
#define KF_KERNEL_PERMUTE_ASSIGN 3
#define KF_KERNEL_GATHER_ROWS 4
#define KF_KERNEL_GEMM1 5
#define KF_KERNEL_GEMM2 6
#define KF_KERNEL_REDUCE 7
#define KF_KERNEL_FRONT_SMALL 8
#define KF_KERNEL_SWIGLU_QUANT 9
#define KF_KERNEL_COUNT 10

/*
 * Profiling.  Between kf_moe_profile_begin() and kf_moe_profile_end(), every
 * kernel this library launches is bracketed by CUDA events recorded on the
 * launch stream.  kf_moe_profile_end() synchronises those events and writes,
 * for each kernel id < n, the summed device milliseconds and the launch count.
 * Host-side bookkeeping only; intended for benchmarks, not for production calls.
 */
int kf_moe_profile_begin(void);
int kf_moe_profile_end(float* total_ms, int32_t* launches, int32_t n);

/* Diagnostics: number of kernels one kf_moe_forward launches for T > 64 tokens
 * (calls of at most 32 tokens run a single-block front end and a split-K GEMM1
 * finish: 5 kernels; 33..64 tokens: 8). */
int32_t kf_moe_launches_per_forward(void);

/* Human-readable text for a KF_ERR_* code. */
const char* kf_moe_error_string(int code);

#ifdef __cplusplus
}
#endif

#endif /* KF_MOE_H_ */
