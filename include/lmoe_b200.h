/*
 * lmoe_b200.h -- C ABI of the B200 (sm_100a) MoE-layer hot path.
 *
 * Plain pointers, sizes and a CUDA stream; no framework types.  Every entry point:
 *   - launches asynchronously on `stream` (never on the legacy default stream unless the
 *     caller passes it) and performs no host<->device synchronisation (except the
 *     peer-exchange setup and teardown, lmoe_p2p_alloc / _free);
 *   - never allocates device memory: outputs and workspaces are caller-owned (the one
 *     exception is the peer-exchange setup, lmoe_p2p_alloc / _open, run once per layer);
 *   - returns LMOE_OK (0), a negative LMOE_ERR_* for rejected arguments, or a positive
 *     cudaError_t value when a CUDA call failed.
 * Kernels that wait on their own pipelines bound every wait; a wait that gives up writes a
 * nonzero word into the workspace's error slot (read it with lmoe_read_error).
 *
 * Each declaration names the light-moe interface it replaces (file:line in the reference
 * repository Whitehall945/light-moe).
 */
#ifndef LMOE_B200_H_
#define LMOE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LMOE_OK 0
#define LMOE_ERR_INVALID_ARG (-1)    /* shape / dtype / alignment / null pointer          */
#define LMOE_ERR_UNSUPPORTED (-2)    /* valid request outside what the kernels implement  */
#define LMOE_ERR_WORKSPACE (-3)      /* workspace missing or too small                    */
#define LMOE_ERR_DEVICE (-4)         /* current device is not sm_100 / kernel error word  */

/* Element types of floating-point operands (the *_typed entry points). */
#define LMOE_DTYPE_BF16 0
#define LMOE_DTYPE_F16 1
#define LMOE_DTYPE_F32 2

typedef struct CUstream_st* lmoe_stream_t; /* identical to cudaStream_t */

/* Library version as 10000*major + 100*minor + patch. */
int lmoe_version(void);

/* Human-readable text for a status code (static storage). */
const char* lmoe_status_string(int status);

/* Copies the 32-bit device error word of a router / GEMM workspace to *out (synchronises
 * `stream`).  0 means no kernel reported a problem. */
int lmoe_read_error(const void* workspace, uint32_t* out, lmoe_stream_t stream);

/* Caps the number of CTAs (one per SM) of the persistent grouped GEMMs launched afterwards
 * by this process (0 = no cap: one per SM).  Leaving SMs free lets kernels on other streams
 * -- NCCL's all-to-all of the next micro-batch -- run beside a GEMM instead of after it.
 * Process-wide; read at each launch.  New (the reference has no persistent kernels). */
int lmoe_set_gemm_sm_limit(int max_ctas);
int lmoe_get_gemm_sm_limit(void);

/* ------------------------------------------------------------------------------------ */
/* Router: gate logits + fp32 softmax + top-k + renormalise + histogram / offsets /       */
/* stable permutation, in one kernel.                                                     */
/* Replaces fused_gate_topk_cuda (csrc/fused_moe_ops.cu:145-200) and the count / offset / */
/* argsort part of fused_gate_topk_permute_cuda (csrc/fused_moe_ops.cu:205-225).          */
/* ------------------------------------------------------------------------------------ */

/* Workspace bytes needed by lmoe_fused_gate_topk for these sizes. */
size_t lmoe_router_workspace_bytes(int64_t num_tokens, int num_experts);

/*
 * hidden      bf16 [num_tokens, hidden]   row-major, 16-byte aligned, hidden % 64 == 0
 * gate_weight bf16 [num_experts, hidden]  (nn.Linear layout, as the reference binding reads
 *                                          E = gate_weight.size(0), fused_moe_ops.cu:155)
 * gate_bias   fp32 [num_experts] or NULL (MoEGate(bias=True), moe_gate.py:159,171)
 * 1 <= num_experts <= 256, 1 <= top_k <= min(16, num_experts)
 * Outputs (any of the optional ones may be NULL):
 *   ids          int32 [num_tokens, top_k]  descending probability, ties -> lower id
 *   weights      fp32  [num_tokens, top_k]  renormalised to sum 1          (optional)
 *   weights_bf16 bf16  [num_tokens, top_k]  same values rounded to bf16     (optional)
 *   counts       int32 [num_experts]                                      (optional*)
 *   offsets      int32 [num_experts + 1]  exclusive scan of counts        (optional*)
 *   sorted_idx   int32 [num_tokens*top_k]  flat index t*top_k+j ordered by
 *                (expert, token, slot)                                    (optional*)
 *   positions    int32 [num_tokens*top_k]  inverse of sorted_idx: the sorted row of
 *                each flat index (optional; needs the three outputs above)
 *   logits       fp32  [num_tokens, num_experts]  gate logits (+bias), for checking
 * (*) counts, offsets and sorted_idx are produced together: pass all three or none.
 */
int lmoe_fused_gate_topk(const void* hidden, const void* gate_weight, const float* gate_bias,
                         int64_t num_tokens, int hidden_size, int num_experts, int top_k,
                         int32_t* ids, float* weights, void* weights_bf16,
                         int32_t* counts, int32_t* offsets, int32_t* sorted_idx,
                         int32_t* positions, float* logits,
                         void* workspace, size_t workspace_bytes, lmoe_stream_t stream);

/* lmoe_fused_gate_topk for hidden states and gate weight of any of the LMOE_DTYPE_* types
 * (x_dtype, w_dtype), as the reference's binding accepts any floating dtype and computes the
 * logits in fp32 from the converted operands (csrc/fused_moe_ops.cu:158-159):
 *   - both bf16 or both fp16: tensor-core logits (16-bit products are exact in fp32, fp32
 *     accumulation);
 *   - otherwise (fp32 on either side, or bf16 with fp16): fp32 logits on CUDA cores from the
 *     caller's values, each a sequential fp32 sum over the hidden dimension.
 * probs (optional, fp32 [num_tokens, num_experts]) receives the full softmax probabilities,
 * the router_probs of the reference's RoutingOutput (python/light_moe/ops/moe_gate.py:20-36)
 * used by its load-balancing loss (:80-122); bit-identical to the values the top-k selects
 * from.  Workspace: lmoe_router_workspace_bytes_typed().  Everything else as
 * lmoe_fused_gate_topk. */
size_t lmoe_router_workspace_bytes_typed(int64_t num_tokens, int num_experts, int x_dtype, int w_dtype);

int lmoe_fused_gate_topk_typed(const void* hidden, int x_dtype, const void* gate_weight, int w_dtype,
                               const float* gate_bias, int64_t num_tokens, int hidden_size, int num_experts,
                               int top_k, int32_t* ids, float* weights, void* weights_bf16,
                               int32_t* counts, int32_t* offsets, int32_t* sorted_idx,
                               int32_t* positions, float* logits, float* probs,
                               void* workspace, size_t workspace_bytes, lmoe_stream_t stream);

/* lmoe_fused_gate_topk without a workspace argument (no counterpart in the reference): the
 * scratch lives in a fixed 1.25 MB device array inside this library, for callers that may
 * not allocate device memory (an allocator that owns all device memory, a serving loop that
 * forbids allocation after start-up).
 *   - num_tokens <= 16384 (any num_experts <= 256); larger calls return LMOE_ERR_WORKSPACE.
 *   - The first call on a device looks up the array's device address; make that first call
 *     before any stream capture.  Later calls allocate nothing.
 *   - All calls on a device share the one array, which keeps whatever the last call left in
 *     it (each call clears the parts that must start at zero).  Calls that overlap in time,
 *     on different streams or host threads, race on it: serialise them.
 *   - A wait timeout recorded by the kernel stays in the shared array; use
 *     lmoe_fused_gate_topk with a workspace when the device error word must be read.
 * Other arguments, outputs and status codes as lmoe_fused_gate_topk. */
int lmoe_fused_gate_topk_static(const void* hidden, const void* gate_weight, const float* gate_bias,
                                int64_t num_tokens, int hidden_size, int num_experts, int top_k,
                                int32_t* ids, float* weights, void* weights_bf16,
                                int32_t* counts, int32_t* offsets, int32_t* sorted_idx,
                                int32_t* positions, float* logits, lmoe_stream_t stream);

/* ------------------------------------------------------------------------------------ */
/* Row gather / weighted combine                                                          */
/* ------------------------------------------------------------------------------------ */

/* permuted[r, :] = hidden[sorted_idx[r] / top_k, :] for r < rows; elements of elem_bytes
 * (2 or 4) bytes, hidden_size * elem_bytes a multiple of 16, rows copied unchanged.
 * Replaces the expand + index_select of fused_gate_topk_permute_cuda
 * (csrc/fused_moe_ops.cu:227-228) and permute_tokens (python/light_moe/ops/grouped_gemm.py:
 * 202-247). */
int lmoe_permute_rows(const void* hidden, int elem_bytes, const int32_t* sorted_idx, int64_t rows,
                      int hidden_size, int top_k, void* permuted, lmoe_stream_t stream);

/* ------------------------------------------------------------------------------------ */
/* int4 weight format (defined by this library; the reference only has the unused flag    */
/* EngineConfig.use_int4_quantization, python/light_moe/engine/executor.py:44-48).        */
/*   qweight uint8 [rows, K/2]: byte b holds k=2b (low nibble) and k=2b+1 (high nibble),   */
/*           each stored as q+8;  scales fp16 [rows, K/group]: s = fp16(max|w|/7);          */
/*   q = clamp(rint(w / s), -8, 7);  dequantised value = bf16_rn(q * s).                   */
/* ------------------------------------------------------------------------------------ */

/* w: [rows, K] bf16 (w_is_fp32 == 0) or fp32 (w_is_fp32 != 0). */
int lmoe_quantize_w4(const void* w, int w_is_fp32, int64_t rows, int K, int group_size,
                     uint8_t* qweight, uint16_t* scales, lmoe_stream_t stream);

/* out: bf16 [rows, K]. */
int lmoe_dequantize_w4(const uint8_t* qweight, const uint16_t* scales, int64_t rows, int K,
                       int group_size, void* out, lmoe_stream_t stream);

/* Bytes of the device ("prepacked") layout streamed by the W4A16 GEMM for `num_experts`
 * matrices of [rows, K]: super-blocks of 128 rows x 128 K values with their fp16 scales
 * embedded, expert-major.  paired != 0 interleaves two such matrices (gate w1 and up w3) by
 * 64-row blocks, giving 2*rows rows.  K % 128 == 0; group_size a multiple of 64 that
 * divides 128 or is a multiple of it; rows % 128 == 0 (rows % 64 == 0 when paired). */
int lmoe_w4_prepacked_bytes(int num_experts, int rows, int K, int group_size, int paired,
                            size_t* packed_bytes);

/* Canonical int4 weights [num_experts, rows, K/2] + scales -> prepacked layout.  Pass the
 * up-projection as qweight_b / scales_b to build the paired gate/up layout, else NULL. */
int lmoe_prepack_w4(const uint8_t* qweight_a, const uint16_t* scales_a,
                    const uint8_t* qweight_b, const uint16_t* scales_b,
                    int num_experts, int rows, int K, int group_size,
                    uint8_t* packed, lmoe_stream_t stream);

/* ------------------------------------------------------------------------------------ */
/* Grouped GEMMs.  Rows [offsets[e], offsets[e+1]) of `input` (bf16 [total_rows, K]) are  */
/* multiplied by expert e's weight matrix ([N, K]); offsets are int32 or int64 [E+1] and  */
/* are read on the device (no host copy).  Workspace: lmoe_gemm_workspace_bytes().        */
/* ------------------------------------------------------------------------------------ */

size_t lmoe_gemm_workspace_bytes(void);

/* Dense weights [num_experts, N, K] of the input's type.  output [total_rows, N] of the
 * same type; with zero_fill the rows outside every expert range are zeroed first.
 * dtype LMOE_DTYPE_BF16 / LMOE_DTYPE_F16: tcgen05 tensor cores (exact 16-bit products, fp32
 * accumulation, K % 64 == 0); LMOE_DTYPE_F32: fp32 FFMA on CUDA cores (K % 4 == 0), as the
 * reference's fp32 cuBLAS GEMM computes in fp32.
 * Replaces grouped_gemm_cuda (csrc/grouped_gemm.cu:11-43), which zero-fills (:24), copies
 * the offsets to the host (:27) and runs one cuBLAS GEMM per expert in the input dtype
 * (:30-40). */
int lmoe_grouped_gemm(const void* input, int dtype, int64_t total_rows, int K, const void* weights, int N,
                      const void* expert_offsets, int offsets_are_int64, int num_experts,
                      int zero_fill, void* output, void* workspace, size_t workspace_bytes,
                      lmoe_stream_t stream);

/* lmoe_grouped_gemm with dtype LMOE_DTYPE_BF16. */
int lmoe_grouped_gemm_bf16(const void* input, int64_t total_rows, int K, const void* weights, int N,
                           const void* expert_offsets, int offsets_are_int64, int num_experts,
                           int zero_fill, void* output, void* workspace, size_t workspace_bytes,
                           lmoe_stream_t stream);

/* W4A16: prepacked int4 weights (N rows per expert, N % 128 == 0, K % 128 == 0), fp32
 * accumulation.
 * epilogue 0: output[r, n] = acc                               (ldo >= N)
 * epilogue 1: SwiGLU over a paired gate/up matrix of N = 2*F rows:
 *             output[r, f] = silu(gate[r, f]) * up[r, f]         (ldo >= F)
 * epilogue 2: output[dest_rows[r], n] = row_scale[r] * acc       (NULL = identity / 1)
 * segment_expert: weight matrix used by each of the num_experts row segments (NULL: the
 *             identity), so rows grouped by (source, expert) need no re-sort; -1 marks a
 *             hole (padding rows of a fixed-capacity exchange): its rows are skipped and
 *             their output rows are left untouched.
 * num_weight_matrices: matrices held by `packed`; every segment_expert entry (or, without a
 *             map, every segment index) must lie in [0, num_weight_matrices).  A kernel that
 *             finds an entry outside it, or offsets that decrease or pass total_rows, skips
 *             that segment and writes a nonzero error word into the workspace
 *             (lmoe_read_error).
 * max_rows_per_expert: an upper bound of any expert's row count if known (0 = unknown);
 * small bounds select the decode-sized tiles.
 * New op; the reference has no W4A16 GEMM (SparseMoEBlockFast's GroupedLinear calls,
 * python/light_moe/model/moe_block.py:249-256, are its dense counterpart). */
int lmoe_w4a16_grouped_gemm(const void* input, int64_t total_rows, int K, const uint8_t* packed,
                            int N, int group_size,
                            const void* expert_offsets, int offsets_are_int64, int num_experts,
                            const int32_t* segment_expert, int num_weight_matrices,
                            int epilogue, const int32_t* dest_rows, const float* row_scale,
                            int64_t max_rows_per_expert, void* output, int64_t ldo,
                            void* workspace, size_t workspace_bytes, lmoe_stream_t stream);

/* Weighted combine of per-slot expert rows back to tokens:
 *   y[t, :] = sum_j weights[t*top_k+j] * rows[positions[t*top_k+j], :]
 *             + sum_s extra_rows[s*num_tokens + t, :]
 * fp32 accumulation in slot order, bf16 in / out, hidden_size even.
 * Replaces unpermute_tokens (python/light_moe/ops/grouped_gemm.py:250-279) and the
 * expert-parallel unsort + weighted sum (python/light_moe/distributed/expert_parallel.py:
 * 307-317). */
/* Fixed-capacity expert-parallel exchange (decode): every rank sends every rank a block of
 * capacity_rows = capacity_tokens * top_k rows, so the all-to-alls have equal splits and no
 * count reaches the host.  All arrays are device int32.
 * Send plan: counts [ep * experts_per_rank] rows of this rank per (destination rank, local
 * expert) in router order; sorted_idx / positions the router's order and its inverse
 * [num_tokens * top_k]. Writes send_index [ep * capacity_rows] (the sorted row carried by each
 * slot of each destination's block, 0 for padding: gather rows with lmoe_permute_rows) and
 * combine_pos [num_tokens * top_k] (the slot, in the returned blocks, of each (token, choice):
 * the positions argument of lmoe_combine_rows). num_tokens * top_k <= capacity_rows.
 * Receive plan: recv_counts [ep * experts_per_rank] rows received per (source rank, local
 * expert). Writes regroup [ep * capacity_rows] (received row at each expert-major position:
 * expert 0 from every source, expert 1, ..., then all padding), restore (its inverse) and
 * seg_offsets [experts_per_rank + num_shared + 2] (the local experts' segments, one padding
 * hole for segment map entry -1, then num_shared segments of num_tokens rows).
 * New: the reference pads to equal splits by sending every token to every rank
 * (python/light_moe/distributed/expert_parallel.py:186-244). */
int lmoe_capacity_send_plan(const int32_t* counts, const int32_t* sorted_idx, const int32_t* positions,
                            int64_t num_tokens, int top_k, int ep, int experts_per_rank, int64_t capacity_rows,
                            int32_t* send_index, int32_t* combine_pos, lmoe_stream_t stream);
int lmoe_capacity_receive_plan(const int32_t* recv_counts, int ep, int experts_per_rank, int64_t capacity_rows,
                               int num_shared, int64_t num_tokens, int32_t* regroup, int32_t* restore,
                               int32_t* seg_offsets, lmoe_stream_t stream);

/* Expert-parallel exchange over peer memory (NVLink), replacing the NCCL all-to-alls of    */
/* python/light_moe/distributed/expert_parallel.py:186-244 and :275-319.  Every rank         */
/* allocates one buffer of lmoe_p2p_buffer_bytes (same geometry on all ranks; Tc = the      */
/* capacity_tokens every rank passes, num_tokens <= Tc per step) with lmoe_p2p_alloc, sends  */
/* the 64-byte IPC handle to the others, maps theirs with lmoe_p2p_open and keeps a device   */
/* array peers[ep] of the mapped bases (its own allocation at peers[me]).  One step:          */
/*   lmoe_p2p_exchange_counts  counts[E] (the router's) -> seg_offsets[E/ep + 2 + S], the     */
/*                             local segments (experts, a hole, S shared segments of T rows)  */
/*                             of the rows region, and dst_base[E] (scratch for dispatch)     */
/*   lmoe_p2p_dispatch         x rows in router order straight into the owners' rows regions */
/*   lmoe_p2p_wait(which = 1)  the rows of every peer arrived: run the grouped GEMMs on the   */
/*                             rows region (at rows_offset; segment e's weight: experts        */
/*                             0..E/ep-1, -1 for the hole, then the shared experts)           */
/*   lmoe_p2p_send_back        the down GEMM's routed output rows back to their sources' ret  */
/*                             regions (slot t*k + j)                                         */
/*   lmoe_p2p_wait(which = 2)  every routed output of this rank's tokens is in its ret region */
/*                             (at ret_offset): lmoe_combine_rows with positions = slot       */
/* state: int32[4] on the device, zeroed once ([0] step epoch, [1] error word: nonzero when a  */
/* wait ran out of time or counts were inconsistent, [2], [3] internal counters).  Waits are  */
/* bounded (2 s); every rank must run every step, in the same order.  lmoe_p2p_alloc / _free */
/* / _open / _close are the library's only entry points that allocate, map or free device    */
/* memory (and synchronise the device): call them at setup and teardown, never in a step.    */
size_t lmoe_p2p_buffer_bytes(int ep, int num_experts, int64_t capacity_tokens, int top_k, int num_shared,
                             int hidden);
int lmoe_p2p_buffer_offsets(int ep, int num_experts, int64_t capacity_tokens, int top_k, int num_shared,
                            int hidden, size_t* rows_offset, size_t* ret_offset);
int lmoe_p2p_alloc(size_t bytes, void** ptr, void* ipc_handle);
int lmoe_p2p_open(const void* ipc_handle, void** ptr);
int lmoe_p2p_close(void* ptr);
int lmoe_p2p_free(void* ptr);
int lmoe_p2p_exchange_counts(const uint64_t* peers, int me, int ep, int num_experts, int64_t capacity_tokens,
                             int top_k, int num_shared, int hidden, int64_t num_tokens, int32_t* state,
                             const int32_t* counts, int32_t* seg_offsets, int32_t* dst_base,
                             lmoe_stream_t stream);
int lmoe_p2p_dispatch(const uint64_t* peers, int me, int ep, int num_experts, int64_t capacity_tokens, int top_k,
                      int num_shared, int hidden, int64_t num_tokens, int32_t* state, const void* x,
                      const int32_t* sorted_idx, const int32_t* ids, const int32_t* offsets,
                      const int32_t* dst_base, lmoe_stream_t stream);
int lmoe_p2p_wait(const uint64_t* peers, int me, int ep, int num_experts, int64_t capacity_tokens, int top_k,
                  int num_shared, int hidden, int64_t num_tokens, int32_t* state, int which, lmoe_stream_t stream);
int lmoe_p2p_send_back(const uint64_t* peers, int me, int ep, int num_experts, int64_t capacity_tokens, int top_k,
                       int num_shared, int hidden, int64_t num_tokens, int32_t* state, const void* out,
                       const int32_t* seg_offsets, lmoe_stream_t stream);

/* Setup once after mapping the peers (shared experts' destinations in this rank's buffer).  */
int lmoe_p2p_init(const uint64_t* peers, int me, int ep, int num_experts, int64_t capacity_tokens, int top_k,
                  int num_shared, int hidden, int32_t* state, lmoe_stream_t stream);
/* The down projection fused with the return transfer (prefill-sized steps, in place of      */
/* lmoe_p2p_send_back): the W4A16 grouped GEMM on h [rows region rows, ffn_size] (the gate/up */
/* output of the rows region) whose epilogue writes each routed output row straight into its  */
/* source rank's ret slot over NVLink and each shared-expert row into dest_bases[ep]          */
/* ([S * num_tokens, hidden] bf16 of this rank); dest_bases[r < ep] = peers[r] + ret_offset. */
/* Then the sources' return flags are raised.  buffer = this rank's own allocation.           */
int lmoe_p2p_down_gemm(const uint64_t* peers, int me, int ep, int num_experts, int64_t capacity_tokens, int top_k,
                       int num_shared, int hidden, int64_t num_tokens, int32_t* state, void* buffer,
                       const void* h, int ffn_size, const uint8_t* w2_packed, int group_size,
                       const int32_t* seg_offsets, const int32_t* seg_expert, int num_segments,
                       int num_weight_matrices, const uint64_t* dest_bases, lmoe_stream_t stream);

int lmoe_combine_rows(const void* rows, const int32_t* positions, const float* weights,
                      int64_t num_tokens, int top_k, int hidden_size,
                      const void* extra_rows, int num_extra, void* y, lmoe_stream_t stream);

/* ------------------------------------------------------------------------------------ */
/* The W4A16 MoE layer: router -> gather -> gate/up GEMM (SwiGLU) -> down GEMM (routing   */
/* weight, scatter to slot) -> per-token combine, all on `stream` without host syncs.     */
/* Replaces SparseMoEBlock.forward / SparseMoEBlockFast.forward                           */
/* (python/light_moe/model/moe_block.py:119-169, :216-274) with int4 experts.             */
/* ------------------------------------------------------------------------------------ */

size_t lmoe_moe_layer_workspace_bytes(int64_t num_tokens, int hidden_size, int ffn_size,
                                      int num_experts, int top_k, int num_shared);

/*
 * x        bf16 [num_tokens, hidden_size]    (hidden_size % 128 == 0, ffn_size % 128 == 0)
 * gate_*   router weight bf16 [num_experts, hidden_size], optional fp32 bias
 * w13      paired prepacked gate/up weights of num_experts + num_shared experts
 *          (routed experts first), each 2*ffn_size x hidden_size
 * w2       prepacked down weights, each hidden_size x ffn_size
 * num_shared always-on experts (weight 1, every token), 0 for Mixtral
 * y        bf16 [num_tokens, hidden_size], 8-byte aligned
 * ids_out / weights_out: optional copies of the routing (int32 / fp32 [num_tokens, top_k])
 */
int lmoe_moe_layer_w4a16(const void* x, int64_t num_tokens, int hidden_size,
                         const void* gate_weight, const float* gate_bias, int num_experts,
                         int top_k, int num_shared,
                         const uint8_t* w13_packed, const uint8_t* w2_packed,
                         int ffn_size, int group_size, void* y,
                         int32_t* ids_out, float* weights_out,
                         void* workspace, size_t workspace_bytes, lmoe_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* LMOE_B200_H_ */
