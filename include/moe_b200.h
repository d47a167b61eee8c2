/*
 * moe_b200.h -- C ABI of libmoe_b200.so, the sm_100a (B200) MoE expert path.
 *
 * Drop-in boundary for PocketLM's native bridge (src/pcketlm/native/__init__.py
 * of the reference): every entry point keeps the argument order, meaning and
 * return-code convention of the reference C function named beside it, with
 * these differences:
 *
 *   - all tensor pointers are DEVICE pointers (CUDA global memory on the
 *     current device), and every call takes a trailing `void* stream`
 *     (a cudaStream_t; NULL = the legacy default stream).  Calls only enqueue
 *     work and return; results are ready when the stream reaches them.
 *   - expert "pointer tables" (uint64_t per expert, as in the reference:
 *     fp8_linear.cpp:365-370) are DEVICE arrays of device addresses.
 *   - entry points that need scratch memory take `void* workspace,
 *     int64_t workspace_bytes`; pass NULL/0 to let the call allocate it
 *     stream-ordered (cudaMallocAsync / cudaFreeAsync).  The *_workspace_bytes
 *     functions return the size a caller-provided workspace must have.
 *
 * Return codes: 0 = ok; -1 null pointer; -2 bad dimensions; -3 out of memory
 * or workspace too small; -4 index out of range; -5 unsupported shape;
 * <= -100: CUDA error (-100 - cudaError_t).  moe_b200_last_error() returns a
 * message for the last failing call on the calling thread.
 *
 * Element types: e4m3 weights are raw bytes (uint8_t), block scales are fp32
 * [ceil(rows/128), ceil(cols/128)] ("weight_scale_inv"), 16-bit tensors are
 * passed as uint16_t storage with a dtype code (0 = fp16, 1 = bf16, the
 * reference's _u16_storage_dtype_code, native/__init__.py:141-146).
 */
#ifndef MOE_B200_H_
#define MOE_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_B200_ABI_VERSION 1

int moe_b200_abi_version(void);
const char* moe_b200_last_error(void);

/* ---------------------------------------------------------------------------
 * FP8 e4m3 block-scaled linears and expert MLPs.  fp32 activations in and
 * out; e4m3 codes 0x7F/0xFF decode as +0 (fp8_linear.cpp:31-33).
 * ------------------------------------------------------------------------- */

/* replaces fp8_e4m3_block_linear_f32, src/pcketlm/native/fp8_linear.cpp:50 */
int moe_fp8_e4m3_block_linear_f32(const uint8_t* fp8_weight, const float* scale_inv,
                                  const float* hidden, float* out, int64_t batch,
                                  int64_t out_rows, int64_t in_cols, int64_t scale_cols,
                                  void* stream);

/* replaces fp8_e4m3_block_dual_linear_f32, fp8_linear.cpp:119 */
int moe_fp8_e4m3_block_dual_linear_f32(const uint8_t* fp8_weight_a, const float* scale_inv_a,
                                       const uint8_t* fp8_weight_b, const float* scale_inv_b,
                                       const float* hidden, float* out_a, float* out_b,
                                       int64_t batch, int64_t out_rows, int64_t in_cols,
                                       int64_t scale_cols, void* stream);

/* replaces fp8_e4m3_block_mlp_f32, fp8_linear.cpp:212 (and the AVX-512 twin
 * fp8_e4m3_block_mlp_avx512_f32, fp8_linear_avx512.cpp:157) */
int moe_fp8_e4m3_block_mlp_f32(const uint8_t* gate_weight, const float* gate_scale_inv,
                               const uint8_t* up_weight, const float* up_scale_inv,
                               const uint8_t* down_weight, const float* down_scale_inv,
                               const float* hidden, float* out, int64_t batch,
                               int64_t intermediate_rows, int64_t hidden_cols,
                               int64_t gate_scale_cols, int64_t down_scale_cols,
                               void* workspace, int64_t workspace_bytes, void* stream);

/* replaces fp8_e4m3_block_mlp_many_f32, fp8_linear.cpp:364 -- out [E, B, H] */
int moe_fp8_e4m3_block_mlp_many_f32(const uint64_t* gate_weight_ptrs, const uint64_t* gate_scale_ptrs,
                                    const uint64_t* up_weight_ptrs, const uint64_t* up_scale_ptrs,
                                    const uint64_t* down_weight_ptrs, const uint64_t* down_scale_ptrs,
                                    const float* hidden, float* out, int64_t expert_count,
                                    int64_t batch, int64_t intermediate_rows, int64_t hidden_cols,
                                    int64_t gate_scale_cols, int64_t down_scale_cols,
                                    void* workspace, int64_t workspace_bytes, void* stream);

/* replaces fp8_e4m3_block_mlp_many_weighted_f32, fp8_linear.cpp:475 (and
 * fp8_e4m3_block_mlp_many_weighted_avx512_f32, fp8_linear_avx512.cpp:252):
 * out [B, H] = sum_e route_weights[e] * expert_e(hidden) */
int moe_fp8_e4m3_block_mlp_many_weighted_f32(const uint64_t* gate_weight_ptrs, const uint64_t* gate_scale_ptrs,
                                             const uint64_t* up_weight_ptrs, const uint64_t* up_scale_ptrs,
                                             const uint64_t* down_weight_ptrs, const uint64_t* down_scale_ptrs,
                                             const float* hidden, const float* route_weights, float* out,
                                             int64_t expert_count, int64_t batch, int64_t intermediate_rows,
                                             int64_t hidden_cols, int64_t gate_scale_cols,
                                             int64_t down_scale_cols, void* workspace,
                                             int64_t workspace_bytes, void* stream);

/* replaces fp8_e4m3_block_mlp_many_row_weighted_f32, fp8_linear.cpp:591:
 * route_weights [E, B]; zero weights skip that (expert, row) entirely */
int moe_fp8_e4m3_block_mlp_many_row_weighted_f32(const uint64_t* gate_weight_ptrs, const uint64_t* gate_scale_ptrs,
                                                 const uint64_t* up_weight_ptrs, const uint64_t* up_scale_ptrs,
                                                 const uint64_t* down_weight_ptrs, const uint64_t* down_scale_ptrs,
                                                 const float* hidden, const float* route_weights, float* out,
                                                 int64_t expert_count, int64_t batch,
                                                 int64_t intermediate_rows, int64_t hidden_cols,
                                                 int64_t gate_scale_cols, int64_t down_scale_cols,
                                                 void* workspace, int64_t workspace_bytes, void* stream);

/* replaces fp8_e4m3_block_mlp_many_pair_weighted_f32, fp8_linear.cpp:833:
 * (item, row, weight) triples; out [B, H] */
int moe_fp8_e4m3_block_mlp_many_pair_weighted_f32(const uint64_t* gate_weight_ptrs, const uint64_t* gate_scale_ptrs,
                                                  const uint64_t* up_weight_ptrs, const uint64_t* up_scale_ptrs,
                                                  const uint64_t* down_weight_ptrs, const uint64_t* down_scale_ptrs,
                                                  const float* hidden, const int64_t* pair_item_indices,
                                                  const int64_t* pair_row_indices, const float* pair_weights,
                                                  float* out, int64_t expert_count, int64_t pair_count,
                                                  int64_t batch, int64_t intermediate_rows,
                                                  int64_t hidden_cols, int64_t gate_scale_cols,
                                                  int64_t down_scale_cols, void* workspace,
                                                  int64_t workspace_bytes, void* stream);

/* No counterpart in the reference.  The expert MLP of
 * moe_fp8_e4m3_block_mlp_f32 for callers that cannot allocate device memory:
 * a process whose GPU memory is all reserved up front by its own arena, a
 * hot path that must not take the CUDA allocator's locks or its implicit
 * synchronisation, or a binding that only owns the pointers it passes.  It
 * allocates nothing: its scratch (pointer table, chunk list, fp32 SwiGLU
 * activations) is a static device array of MOE_B200_NOALLOC_SCRATCH_BYTES
 * (4 MiB) that every GPU loading the library holds until exit.  Calls needing
 * more (roughly batch * intermediate_rows * 4 bytes plus a few KiB) return -3
 * with a message, checked before any size product is formed; dimensions
 * beyond int32 are unsupported.  All calls share the array, so calls that overlap on the GPU
 * (different streams or devices' threads racing on one device) race; serialise
 * them.  The first call on a device looks the array's address up and should
 * come before any stream capture.  Same arguments and results as
 * moe_fp8_e4m3_block_mlp_f32, minus the workspace. */
#define MOE_B200_NOALLOC_SCRATCH_BYTES (4u << 20)
int moe_fp8_e4m3_block_mlp_f32_noalloc(const uint8_t* gate_weight, const float* gate_scale_inv,
                                       const uint8_t* up_weight, const float* up_scale_inv,
                                       const uint8_t* down_weight, const float* down_scale_inv,
                                       const float* hidden, float* out, int64_t batch,
                                       int64_t intermediate_rows, int64_t hidden_cols,
                                       int64_t gate_scale_cols, int64_t down_scale_cols, void* stream);

/* Workspace bytes for the MLP entry points above, given the number of
 * (expert, row) pairs they evaluate (mlp: batch; many/weighted: E*B;
 * row/pair weighted: the nonzero count or pair_count; pass the upper bound). */
int64_t moe_fp8_mlp_workspace_bytes(int64_t pairs, int64_t segments, int64_t batch,
                                    int64_t intermediate_rows, int64_t hidden_cols);

/* ---------------------------------------------------------------------------
 * FP8 block dequantisation (NaN codes decode to the reference's NaN bits).
 * ------------------------------------------------------------------------- */

/* replaces fp8_e4m3_dequant_to_fp16, src/pcketlm/native/fp8_dequant.cpp:119 */
int moe_fp8_e4m3_dequant_to_fp16(const uint8_t* fp8_weight, const float* scale_inv, uint16_t* out_fp16,
                                 int64_t rows, int64_t cols, int64_t scale_cols, void* stream);

/* replaces fp8_e4m3_dequant_to_bf16, fp8_dequant.cpp:166 */
int moe_fp8_e4m3_dequant_to_bf16(const uint8_t* fp8_weight, const float* scale_inv, uint16_t* out_bf16,
                                 int64_t rows, int64_t cols, int64_t scale_cols, void* stream);

/* ---------------------------------------------------------------------------
 * Routers.
 * ------------------------------------------------------------------------- */

/* replaces ds_router_topk_u16, src/pcketlm/native/ds_forward.cpp:879: one
 * token, softmax with fp64 denominators, top-k (ties to the lower id), fp64
 * renormalisation. */
int moe_ds_router_topk_u16(const uint16_t* hidden_u16, const uint16_t* router_weights_u16,
                           int64_t hidden_dim, int64_t num_experts, int64_t k, int64_t dtype_code,
                           int64_t* output_expert_ids, float* output_weights, void* stream);

/* Batched router; replaces the routing math of run_fp8_router
 * (src/pcketlm/core/runtime/fp8_source.py:1522-1547, group mask :5125-5140),
 * which the reference runs in torch.  scoring: 0 sigmoid, 1 softmax.  With
 * sigmoid scoring the picked scores are renormalised; `renorm` forces it for
 * softmax too (Mixtral norm_topk_prob, core/runtime/layer_bridge.py:2682-2689).
 * hidden_dtype / router_dtype: 0 fp32, 1 bf16, 2 fp16.  bias may be NULL.
 * round_bf16 rounds the final weights through bf16 (the reference casts them
 * to the hidden dtype).  Any of the three outputs may be NULL. */
int moe_route_topk(const void* hidden, int hidden_dtype, const void* router_weight, int router_dtype,
                   const float* bias, int64_t tokens, int64_t hidden_dim, int64_t num_experts,
                   int64_t n_group, int64_t topk_group, int64_t top_k, int scoring, int renorm,
                   float route_scale, int round_bf16, int64_t* out_ids, float* out_weights_f32,
                   uint16_t* out_weights_bf16, void* workspace, int64_t workspace_bytes, void* stream);

int64_t moe_route_topk_workspace_bytes(int64_t tokens, int64_t num_experts);

/* ---------------------------------------------------------------------------
 * Whole DeepSeek-V3 MoE layer: route -> dispatch -> FP8 SwiGLU experts ->
 * weighted combine + shared expert.  Replaces run_fp8_moe
 * (fp8_source.py:1569-1884).  hidden: [tokens, hidden_dim] bf16 (dtype 1) or
 * fp32 (dtype 0).  tables: device uint64 array [6][n_routed + has_shared]
 * (gate w, gate scale, up w, up scale, down w, down scale; the shared expert
 * is the last entry).  nan_free: moe_fp8_nan_free_flags' per-expert flags or
 * NULL.  weight_layout: 0 = row-major weights (the reference's), 1 = the
 * tiled layout below.  out_bf16: [tokens, hidden_dim] bf16.  out_ids (int64)
 * and out_weights_bf16 ([tokens, top_k]) may be NULL.
 * ------------------------------------------------------------------------- */
int moe_ds_moe_layer_fp8(const void* hidden, int hidden_dtype, int64_t tokens, int64_t hidden_dim,
                         int64_t intermediate, const void* router_weight, int router_dtype,
                         const float* router_bias, int64_t n_routed, int64_t n_group, int64_t topk_group,
                         int64_t top_k, int scoring, float route_scale, const uint64_t* tables,
                         int has_shared, const uint8_t* nan_free, int weight_layout, uint16_t* out_bf16,
                         int64_t* out_ids, uint16_t* out_weights_bf16, void* workspace, int64_t workspace_bytes,
                         void* stream);

/* Fragment-native weight layout (no reference counterpart), weight_layout 1
 * of moe_ds_moe_layer_fp8: moe_fp8_tile_weights copies a row-major e4m3
 * [rows, cols] matrix (cols % 128 == 0) into moe_fp8_tiled_bytes(rows, cols)
 * bytes (rows padded to a multiple of 128 with zeros).  For every 128-row
 * group, 128-column k-block and 64-column half, an 8 KiB run holds the
 * group's eight 16-row tiles, each as two 512-byte pieces in the order the
 * decode GEMV's lanes read them (a warp-wide access is 512 contiguous bytes);
 * the prefill GEMM brings a whole run into shared memory with one bulk copy.
 * Same bytes, same results; the block scales keep their layout.  Tables for
 * weight_layout 1 point at tiled copies. */
int64_t moe_fp8_tiled_bytes(int64_t rows, int64_t cols);
int moe_fp8_tile_weights(const uint8_t* weight, uint8_t* tiled, int64_t rows, int64_t cols, void* stream);

/* Per-expert flags for moe_ds_moe_layer_fp8's `nan_free` argument (no
 * reference counterpart): flags[e] = 1 when none of expert e's gate, up and
 * down e4m3 bytes is 0x7F or 0xFF (tables as above, [6][num_experts]; absent
 * experts count as clean), else 0.  The layer decodes those two codes as +0
 * like the reference's linear kernels; an expert known to hold neither skips
 * that per-byte fix-up.  nan_free may be NULL (every expert is fixed up).
 * Compute the flags once per set of resident weights. */
int moe_fp8_nan_free_flags(const uint64_t* tables, int64_t num_experts, int64_t intermediate, int64_t hidden_dim,
                           uint8_t* flags, void* stream);

int64_t moe_ds_moe_layer_workspace_bytes(int64_t tokens, int64_t hidden_dim, int64_t intermediate,
                                         int64_t n_routed, int64_t top_k, int has_shared);

/* ---------------------------------------------------------------------------
 * Q4 (signed int4, two codes per byte with the even flat index in the low
 * nibble, one fp16 scale per output row: q4_quantize.py:21-71) and the
 * 16-bit formats.  Entry points named after a reference C function return
 * that function's own positive codes for null pointers / bad sizes (listed
 * beside each); the others use the negative codes above.
 * ------------------------------------------------------------------------- */

/* replaces q4_dequant_to_fp16, q4_dequant.cpp:171-208 (which returns void):
 * out[c * channel_size + k] = fp16(code * scales[c]).  1: null pointer,
 * 2: non-positive sizes. */
int moe_q4_dequant_to_fp16(const uint8_t* packed, const uint16_t* scales, uint16_t* out, int64_t num_channels,
                           int64_t channel_size, void* stream);

/* replaces q4_dequant_many_to_fp16, q4_dequant.cpp:210-286: HOST arrays of
 * device pointers and sizes, one entry per tensor.  1: a null array,
 * 2: tensor_count <= 0. */
int moe_q4_dequant_many_to_fp16(const uint8_t* const* packed, const uint16_t* const* scales, uint16_t* const* out,
                                const int64_t* num_channels, const int64_t* channel_sizes, int64_t tensor_count,
                                void* stream);

/* replaces q4_moe_selected_forward_u16, q4_dequant.cpp:357-476: one fp16
 * token through `selected_count` experts (device uint64 tables of packed
 * gate/up [intermediate, hidden] and down [hidden, intermediate] codes and
 * their fp16 row scales), out_fp16[h] = fp16(sum_e route[e] * down_e(...)).
 * 1: null pointer or non-positive size (q4_dequant.cpp:370-378). */
int moe_q4_moe_selected_forward_u16(const uint16_t* hidden, const uint64_t* gate_packed, const uint64_t* gate_scales,
                                    const uint64_t* up_packed, const uint64_t* up_scales,
                                    const uint64_t* down_packed, const uint64_t* down_scales,
                                    const float* route_weights, uint16_t* out_fp16, int64_t hidden_size,
                                    int64_t intermediate_size, int64_t selected_count, void* workspace,
                                    int64_t workspace_bytes, void* stream);
int64_t moe_q4_moe_selected_workspace_bytes(int64_t hidden_size, int64_t intermediate_size, int64_t selected);

/* A whole Mixtral-style Q4 MoE layer for a batch of tokens: softmax router
 * over fp32 logits, top-k renormalised (layer_bridge.py:2682-2689), then each
 * token through q4_moe_selected_forward_u16's arithmetic -- the batch form of
 * the reference's per-token loop _run_q4_moe_mlp_token_loop
 * (layer_bridge.py:909-955).  hidden: [tokens, hidden] bf16 (1) or fp16 (2),
 * converted to fp16 as the reference does; tables: device uint64 [6][E];
 * out: [tokens, hidden] in hidden's dtype (the fp16 result, re-rounded to
 * bf16 for a bf16 caller); out_ids int64 / out_weights fp32 [tokens, top_k]
 * may be NULL.  weight_layout 0: tables point at the row-major packed codes
 * (warp-MMA GEMV, any batch); 1: at copies in the Q4 tiled layout
 * (moe_q4_tile_weights) -- the tcgen05 grouped GEMM for prefill-sized
 * batches, hidden % 256 == 0 and intermediate % 128 == 0; scales as given. */
int moe_q4_moe_layer_u16(const void* hidden, int hidden_dtype, int64_t tokens, int64_t hidden_size,
                         int64_t intermediate_size, const void* router_weight, int router_dtype, int64_t num_experts,
                         int64_t top_k, const uint64_t* tables, int weight_layout, void* out, int64_t* out_ids,
                         float* out_weights, void* workspace, int64_t workspace_bytes, void* stream);
int64_t moe_q4_moe_layer_workspace_bytes(int64_t tokens, int64_t hidden_size, int64_t intermediate_size,
                                         int64_t num_experts, int64_t top_k);
/* Q4 tiled layout (no reference counterpart), weight_layout 1 of
 * moe_q4_moe_layer_u16: moe_q4_tile_weights copies packed int4 codes [rows,
 * cols / 2] (cols % 64 == 0) into moe_q4_tiled_bytes(rows, cols) bytes: for
 * every 128-row group and 64-column block a 4 KiB run of the group's rows (32
 * bytes each), rows padded to a multiple of 128 with zeros -- one bulk copy
 * per matrix and pipeline stage of the prefill GEMM.  Same bytes reordered. */
int64_t moe_q4_tiled_bytes(int64_t rows, int64_t cols);
int moe_q4_tile_weights(const uint8_t* packed, uint8_t* tiled, int64_t rows, int64_t cols, void* stream);

/* replaces native_pack_u16_rows8, fp16_packed_gemv.cpp:52-77:
 * packed[(blk * cols + c) * 8 + lane] = weight[blk * 8 + lane, c], zero past
 * the last row.  1: null pointer, 2: negative size. */
int moe_pack_u16_rows8(const uint16_t* weight, uint16_t* packed, int64_t rows, int64_t cols, void* stream);

/* replaces native_packed_gemv_rows8, fp16_packed_gemv.cpp:79-116:
 * out[r] = sum_c hidden[c] * W[r, c] (fp32) from the row8 layout; dtype_code
 * 0 = fp16, 1 = bf16.  1: null pointer, 2: negative size or bad dtype. */
int moe_packed_gemv_rows8(const uint16_t* hidden, const uint16_t* packed, float* out, int64_t rows, int64_t cols,
                          int dtype_code, void* stream);

/* replaces native_moe_selected_forward_u16, fp16_moe.cpp:199-267: every token
 * through every one of `selected_count` experts stacked as gate/up
 * [selected, intermediate, hidden] and down [selected, hidden, intermediate],
 * out[t] = sum_s route_weights[t, s] * expert_s(hidden[t]) in fp32, stored in
 * the 16-bit dtype.  1: null pointer, 2: non-positive size, 3: bad dtype. */
int moe_moe_selected_forward_u16(const uint16_t* hidden, const uint16_t* gate_weight, const uint16_t* up_weight,
                                 const uint16_t* down_weight, const float* route_weights, uint16_t* out,
                                 int64_t seq_len, int64_t hidden_size, int64_t selected_count,
                                 int64_t intermediate_size, int dtype_code, void* workspace, int64_t workspace_bytes,
                                 void* stream);
int64_t moe_moe_selected_forward_workspace_bytes(int64_t seq_len, int64_t hidden_size, int64_t selected_count,
                                                 int64_t intermediate_size, int dtype_code);

/* replaces native_moe_forward_fp16, fp16_moe.cpp:90-197: fp16 router
 * (softmax, top-k, ties to the lower id, optional renorm) then the selected
 * fp16 experts ([E, intermediate, hidden] / [E, hidden, intermediate]).
 * selected_experts (int64) and selected_weights (fp32) [seq_len, top_k] may
 * be NULL.  1: null pointer, 2: non-positive size, 3: top_k > num_experts. */
int moe_moe_forward_fp16(const uint16_t* hidden, const uint16_t* router_weight, const uint16_t* gate_weight,
                         const uint16_t* up_weight, const uint16_t* down_weight, uint16_t* out,
                         int64_t* selected_experts, float* selected_weights, int64_t seq_len, int64_t hidden_size,
                         int64_t num_experts, int64_t top_k, int64_t intermediate_size, int normalize_topk,
                         void* workspace, int64_t workspace_bytes, void* stream);
int64_t moe_moe_forward_fp16_workspace_bytes(int64_t seq_len, int64_t hidden_size, int64_t num_experts,
                                             int64_t top_k, int64_t intermediate_size);

/* ---------------------------------------------------------------------------
 * Expert parallelism (no reference counterpart: the reference runs on one
 * host).  Experts are partitioned contiguously over `world` ranks (rank r
 * owns experts [r * E / world, (r + 1) * E / world)); router and shared
 * expert are replicated.  One layer step per rank:
 *   moe_route_topk -> moe_ep_dispatch_pack -> all-to-all of send_offsets'
 *   counts, rows and expert ids (the caller's collective) ->
 *   moe_ep_experts_fp8 over the received rows (+ the rank's own rows for
 *   the shared expert) -> the outputs rounded to bf16 (round to nearest
 *   even) -> reverse all-to-all of them -> moe_ep_combine.
 * The arithmetic per (token, expert) pair is that of moe_ds_moe_layer_fp8;
 * every expert output is rounded to bf16 before the combine, as the
 * reference rounds it (fp8_source.py:1839-1847) and as the whole layer's
 * prefill does; the combine order is top-k slot order, then the shared
 * expert, in fp32, with one final bf16 rounding.
 * ------------------------------------------------------------------------- */

/* Group the (token, slot) entries of ids / weights ([tokens, top_k]) by
 * destination rank, token order kept inside a rank: send_rows [tokens*top_k,
 * hidden] bf16 copies of the tokens' hidden rows, send_expert the expert id
 * local to its rank, send_offsets [world + 1] the rank boundaries,
 * entry_pos [tokens*top_k] each entry's send position and pos_weight
 * [tokens*top_k] the weight at each send position. */
int moe_ep_dispatch_pack(const int64_t* ids, const float* weights, const uint16_t* hidden_bf16, int64_t tokens,
                         int64_t hidden_dim, int64_t top_k, int64_t num_experts, int64_t world,
                         uint16_t* send_rows, int32_t* send_expert, int32_t* send_offsets, int32_t* entry_pos,
                         float* pos_weight, void* workspace, int64_t workspace_bytes, void* stream);
int64_t moe_ep_dispatch_workspace_bytes(int64_t tokens, int64_t top_k);

/* out[i] = expert_{row_expert[i]}(rows[i]) (fp32 [rows, hidden]) over this
 * rank's experts (device tables [6][num_local]; nan_free and weight_layout as
 * for moe_ds_moe_layer_fp8); a row whose expert id is out of range comes
 * back zero.  hidden and intermediate: multiples of 128. */
int moe_ep_experts_fp8(const uint16_t* rows_bf16, const int32_t* row_expert, int64_t rows, int64_t hidden_dim,
                       int64_t intermediate, const uint64_t* tables, int64_t num_local, const uint8_t* nan_free,
                       int weight_layout, float* out, void* workspace, int64_t workspace_bytes, void* stream);
int64_t moe_ep_experts_workspace_bytes(int64_t rows, int64_t hidden_dim, int64_t intermediate, int64_t num_local);

/* out_bf16[t] = bf16(sum_slot pos_weight[p] * y[p] (+ y[tokens*top_k + t]
 * when has_shared)), p = entry_pos[t * top_k + slot], slots in order, summed
 * in fp32; y holds the output rows as bf16 (y_dtype 1: the exchanges' rounded
 * rows) or fp32 (0). */
int moe_ep_combine(const void* y, int y_dtype, const int32_t* entry_pos, const float* pos_weight, int64_t tokens,
                   int64_t top_k, int64_t hidden_dim, int has_shared, uint16_t* out_bf16, void* stream);

/* No reference counterpart (the reference runs on one host; its ranks do not
 * exist).  A barrier of the expert-parallel ranks over peer memory, in place
 * of a collective: peer_sig [world] holds every rank's signal buffer (world
 * uint32 slots, zero before the first barrier; torch symmetric memory), epoch
 * this rank's device counter (zero at first; one increment per barrier).  Each
 * rank stores its epoch into slot [rank] of every peer's buffer after a
 * system-scope fence -- so everything it stored to peer memory before is
 * visible first -- and waits for every peer's epoch in its own slots, at most
 * limit_us microseconds; with payload (payload_n int32, device memory), that
 * row is first copied into row `rank` of every peer's peer_payload buffer (an
 * all-gather).  A wait that runs out sets code 256 in moe_b200_device_error,
 * after which barriers stop waiting until the code is read.  One launch of
 * one CTA; every rank must call it the same number of times. */
int moe_ep_barrier_p2p(const uint64_t* peer_sig, int64_t world, int64_t rank, uint32_t* epoch,
                       const int32_t* payload, int64_t payload_n, const uint64_t* peer_payload, int64_t limit_us,
                       void* stream);

/* The exchange without collectives on the data path: every rank keeps
 * receive buffers in peer-accessible memory (e.g. torch symmetric memory) --
 * rows [capacity (+ own rows), hidden] bf16, expert int32 [capacity] (-1 =
 * empty, reset before each step), src int32 [capacity], and a return buffer
 * [src_stride + tokens, hidden] bf16 -- whose addresses on every rank the
 * caller passes as device arrays uint64 [world].  A step:
 *   moe_ep_count_ranks -> all-gather of the [world] counts into
 *   count_matrix [world][world] (row = source rank) -> moe_ep_dispatch_p2p
 *   (this rank's rows written into each destination's buffers, token order
 *   kept, ranks in order) -> barrier -> moe_ep_experts_return_p2p over the
 *   local buffer (or moe_ep_experts_fp8 then moe_ep_return_p2p): each output
 *   row is written into row e of its source rank's return buffer, e = the
 *   entry t * top_k + slot -> barrier -> moe_ep_combine with entry_pos =
 *   identity.  The dispatch checks each row's destination rank and receive
 *   slot (counts that disagree with the rows sent would place a row outside
 *   the buffer): such a row is not stored and code 64 is set in
 *   moe_b200_device_error.  src = rank * src_stride + e; src_stride > every return row
 *   (tokens * top_k, or tokens * (top_k + 1) when the rank's own shared-expert
 *   rows go through the same call with e = tokens * top_k + t); capacity >=
 *   the rows any rank receives (world * tokens * top_k suffices).  The
 *   barriers are the caller's: moe_ep_barrier_p2p (its payload carrying the
 *   counts for the all-gather) or any stream-ordered collective.  Same
 *   arithmetic and combine order as the all-to-all exchange above. */
int moe_ep_count_ranks(const int64_t* ids, int64_t tokens, int64_t top_k, int64_t num_experts, int64_t world,
                       int32_t* counts, void* stream);
/* No reference counterpart.  The send side of one decode step of the
 * exchange above in two launches (router logits, then one CTA), instead of
 * routing, count, reset, barrier-with-counts, dispatch, barrier and the
 * copies of this rank's shared-expert rows: the DS-V3 router (sigmoid,
 * correction bias, group-limited top-k, renormalised, scaled, weights
 * rounded through bf16 -- moe_route_topk's results -- into out_ids /
 * out_weights_f32 [tokens, top_k]), this rank's receive slots reset
 * (expert -1 for rows 0 .. capacity - 1) and its own tokens' rows appended
 * at rows capacity + t (expert num_experts / world, the shared expert; src
 * rank * src_stride + tokens * top_k + t), the counts all-gathered through
 * the barrier, every routed row written into its expert's rank (token order
 * kept, ranks in order, slots range-checked: code 64), then the second
 * barrier.  peer_matrix [world] holds every rank's [world][world] counts
 * buffer and peer_sig / epoch are the barrier's (moe_ep_barrier_p2p; the
 * epoch grows by two).  hidden bf16, router_weight bf16 or f16
 * (router_dtype), tokens <= 128 (0: a rank with no tokens still resets,
 * sends its zero counts and takes both barriers), tokens * top_k <= 1024,
 * num_experts <= 256, world <= 32; workspace:
 * moe_ep_route_dispatch_p2p_workspace_bytes. */
int64_t moe_ep_route_dispatch_p2p_workspace_bytes(int64_t tokens, int64_t num_experts);
int moe_ep_route_dispatch_p2p(const uint16_t* hidden_bf16, const void* router_weight, int router_dtype,
                              const float* bias, int64_t tokens, int64_t hidden_dim, int64_t num_experts,
                              int64_t n_group, int64_t topk_group, int64_t top_k, float route_scale, int64_t world,
                              int64_t rank, int64_t capacity, int64_t src_stride, const uint64_t* peer_rows,
                              const uint64_t* peer_expert, const uint64_t* peer_src, const uint64_t* peer_matrix,
                              const uint64_t* peer_sig, uint32_t* epoch, int64_t limit_us, int64_t* out_ids,
                              float* out_weights_f32, void* workspace, int64_t workspace_bytes, void* stream);
int moe_ep_dispatch_p2p(const int64_t* ids, const uint16_t* hidden_bf16, int64_t tokens, int64_t hidden_dim,
                        int64_t top_k, int64_t num_experts, int64_t world, int64_t rank, const int32_t* count_matrix,
                        int64_t capacity, int64_t src_stride, const uint64_t* peer_rows, const uint64_t* peer_expert,
                        const uint64_t* peer_src, void* workspace, int64_t workspace_bytes, void* stream);
int64_t moe_ep_dispatch_p2p_workspace_bytes(int64_t tokens, int64_t top_k, int64_t world);
/* Received row j's fp32 output y[j] (recv_expert[j] >= 0), rounded to bf16,
 * goes to row recv_src[j] % src_stride of rank recv_src[j] / src_stride's
 * return buffer (bf16 rows).  Every src code is checked
 * before the store: a rank outside [0, world) or a row at or past home_rows
 * (the rows of each rank's return buffer, <= src_stride) is skipped and sets
 * code 64 in moe_b200_device_error. */
int moe_ep_return_p2p(const float* y, int64_t rows, const int32_t* recv_expert, const int32_t* recv_src,
                      int64_t hidden_dim, int64_t src_stride, int64_t world, int64_t home_rows,
                      const uint64_t* peer_yback, void* stream);
/* moe_ep_experts_fp8 and moe_ep_return_p2p in one call: received row j's
 * output, rounded to bf16, goes straight to row (row_src[j] % src_stride) of the return buffer
 * of rank row_src[j] / src_stride (peer_yback [world], as above), stored over
 * NVLink by the down GEMM's epilogue or by a copy kernel after the warp-MMA
 * experts.  Rows whose expert id is out of range are neither computed nor
 * sent, so a receive buffer with empty slots costs no expert work.
 * valid_rows: the rows the caller expects to carry a local expert (0 = all);
 * it only picks the kernel -- the GEMM for tiled weights and >= 512 rows, >= 16
 * per local expert -- and the workspace, so any value gives the same result.
 * The caller may route its own tokens' shared-expert rows through the same
 * call (src = rank * src_stride + their return row).  hidden % 4 == 0.
 * The src codes are checked as in moe_ep_return_p2p (world, home_rows): a row
 * whose home is out of range is computed into this rank's own workspace and
 * never sent, and sets code 64 in moe_b200_device_error. */
int moe_ep_experts_return_p2p(const uint16_t* rows_bf16, const int32_t* row_expert, const int32_t* row_src,
                              int64_t rows, int64_t valid_rows, int64_t hidden_dim, int64_t intermediate,
                              const uint64_t* tables, int64_t num_local, const uint8_t* nan_free, int weight_layout,
                              int64_t src_stride, int64_t world, int64_t home_rows, const uint64_t* peer_yback,
                              void* workspace, int64_t workspace_bytes, void* stream);
int64_t moe_ep_experts_return_p2p_workspace_bytes(int64_t rows, int64_t valid_rows, int64_t hidden_dim,
                                                  int64_t intermediate, int64_t num_local, int weight_layout);

/* ---------------------------------------------------------------------------
 * DeepSeek session: opaque handle with the reference's observable counters.
 * ------------------------------------------------------------------------- */

/* replaces ds_session_create / ds_session_destroy, ds_forward.cpp:192-219 */
void* moe_ds_session_create(int64_t num_layers, int64_t hidden_dim, int64_t num_experts, int64_t top_k);
void moe_ds_session_destroy(void* handle);

/* replace ds_monolithic_call_counter, ds_expert_invocation_count and
 * ds_layers_executed_count, ds_forward.cpp:265-335 (-1 for a null handle) */
int64_t moe_ds_monolithic_call_counter(void* handle);
int64_t moe_ds_expert_invocation_count(void* handle);
int64_t moe_ds_layers_executed_count(void* handle);

/* replaces ds_moe_layer_forward_f32, ds_forward.cpp:337:
 * hidden_out[b, h] = sum_e route_weights[e] * expert_outputs[e, b, h] */
int moe_ds_moe_layer_forward_f32(void* handle, const float* expert_outputs, const float* route_weights,
                                 int64_t selected_count, int64_t batch, int64_t hidden_dim,
                                 float* hidden_out, void* stream);

/* replaces ds_moe_layer_forward_fp8_f32, ds_forward.cpp:784 */
int moe_ds_moe_layer_forward_fp8_f32(void* handle, const uint64_t* gate_weight_ptrs,
                                     const uint64_t* gate_scale_ptrs, const uint64_t* up_weight_ptrs,
                                     const uint64_t* up_scale_ptrs, const uint64_t* down_weight_ptrs,
                                     const uint64_t* down_scale_ptrs, const float* hidden,
                                     const float* route_weights, int64_t selected_count, int64_t batch,
                                     int64_t intermediate_rows, int64_t hidden_dim,
                                     int64_t gate_scale_cols, int64_t down_scale_cols, float* hidden_out,
                                     void* workspace, int64_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * MLA attention for one decode token (mla.cu), fp32 like the reference.
 * All pointers are device pointers; workspace may be null (a stream-ordered
 * allocation) or at least the *_workspace_bytes size.
 * ------------------------------------------------------------------------- */

/* replaces ds_attention_invocation_count / ds_fused_attention_invocation_count,
 * ds_forward.cpp:289-304 (-1 for a null handle) */
int64_t moe_ds_attention_invocation_count(void* handle);
int64_t moe_ds_fused_attention_invocation_count(void* handle);

/* Workspace of moe_mla_attention_flash_forward; -1 for dimensions it rejects. */
int64_t moe_mla_attention_workspace_bytes(int64_t num_heads, int64_t cache_len, int64_t qk_nope_dim,
                                          int64_t qk_rope_dim, int64_t kv_lora_rank, int64_t v_head_dim);

/* replaces ds_mla_attention_flash_forward, ds_forward.cpp:517-597 (same
 * arguments, then workspace and stream): q_nope [heads, nope], q_pe
 * [heads, rope] (already rotated), kv_cache [cache_len, kv_lora_rank],
 * pe_cache [cache_len, rope], wkv_b [heads, nope + v, kv_lora_rank] ->
 * output_heads [heads, v].  Returns 0; 1 for a null pointer and 2 for bad
 * dimensions as the reference does; MOE_B200 status codes (negative) for
 * kv_lora_rank > 1024, qk_rope_dim > 256, qk_nope_dim > 8192, a small
 * workspace or a CUDA error. */
int moe_mla_attention_flash_forward(const float* q_nope, const float* q_pe, const float* kv_cache,
                                    const float* pe_cache, const float* wkv_b, float* output_heads, int64_t num_heads,
                                    int64_t cache_len, int64_t qk_nope_dim, int64_t qk_rope_dim, int64_t kv_lora_rank,
                                    int64_t v_head_dim, float softmax_scale, void* workspace, int64_t workspace_bytes,
                                    void* stream);

/* Workspace of moe_ds_attention_block_forward_f32; -1 for dimensions it rejects. */
int64_t moe_ds_attention_block_workspace_bytes(int64_t hidden_dim, int64_t q_lora_rank, int64_t kv_lora_rank,
                                               int64_t num_heads, int64_t qk_nope_dim, int64_t qk_rope_dim,
                                               int64_t v_head_dim, int64_t previous_len);

/* replaces ds_attention_block_forward_f32, ds_forward.cpp:647-782 (same
 * arguments, then workspace and stream): q_low = RMSNorm(q_a . hidden), q =
 * q_b . q_low per head with RoPE on its rope part, the new cache row (kv_a .
 * hidden: RMSNorm on the latent part, RoPE on the pe part) appended after the
 * previous_len rows copied from previous_*_cache, the attention core over
 * previous_len + 1 positions, hidden_out = o_weight . heads.  next_*_cache
 * may equal previous_*_cache (append in place: no copy; the buffers then
 * hold previous_len + 1 rows) and must not otherwise overlap them
 * (MOE_B200 -2).  Returns 0; 1 (null pointer), 2 (bad
 * dimensions), 3 (previous_len > 0 without previous caches) as the reference
 * does; MOE_B200 status codes (negative) otherwise.  Counts one monolithic
 * call and one (fused) attention invocation on the session. */
int moe_ds_attention_block_forward_f32(void* handle, const float* hidden_in, const float* q_a_weight,
                                       const float* q_b_weight, const float* kv_a_weight, const float* kv_b_weight,
                                       const float* o_weight, const float* q_norm_weight, const float* kv_norm_weight,
                                       const float* previous_kv_cache, const float* previous_pe_cache,
                                       const float* rope_cos, const float* rope_sin, float* next_kv_cache,
                                       float* next_pe_cache, float* hidden_out, int64_t hidden_dim,
                                       int64_t q_lora_rank, int64_t kv_lora_rank, int64_t num_heads,
                                       int64_t qk_nope_dim, int64_t qk_rope_dim, int64_t v_head_dim,
                                       int64_t previous_len, float rms_eps, float softmax_scale, void* workspace,
                                       int64_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Profiling (no reference counterpart): when enabled, moe_ds_moe_layer_fp8
 * records CUDA events on its stream at the boundaries of its stages:
 * start | route, dispatch, chunk list (+ f16 staging of x on the MMA path) |
 * gate/up | (f16 staging of the activations on the MMA path |) down |
 * combine.  moe_b200_stage_times waits for the last event and writes the
 * elapsed milliseconds between consecutive marks (returns how many).
 * Single-threaded use only.
 * ------------------------------------------------------------------------- */
int moe_b200_stage_timing(int enable);
int moe_b200_stage_times(float* ms, int max_n);

/* Expert-GEMV implementation (no reference counterpart): 0 = auto (default:
 * the cp.async-fed warp-MMA kernel on the whole-layer path when hidden and
 * intermediate sizes are multiples of 128, the direct-load kernel
 * elsewhere), 1 = the warp-specialised bulk-copy streaming kernel wherever
 * the shape allows, 2 = the direct-load kernel everywhere, 3 = like 0 with
 * the warp-MMA kernel loading its weights straight into registers, 4 = like
 * 0 with the warp-MMA kernel fed through per-warp TMA bulk-copy rings, 5 =
 * same as 0.  For A/B parity tests and measurements. */
int moe_b200_select_gemv(int impl);
/* The current selection (0 for the default, else 1 to 4). */
int moe_b200_selected_gemv(void);
/* No reference counterpart.  Decode-sized layers on the default GEMV run
 * their experts as one persistent launch -- gate/up + SwiGLU, the f16 staging
 * of the activations and the down projection, each phase's weight bytes cut
 * into equal per-warp ranges, down work of an expert waiting (bounded) for that
 * expert's gate/up -- when enabled (1); 0 (the default) runs the three
 * launches.  Same results to fp32 rounding of the partial-sum grouping. */
int moe_b200_fused_decode(int enable);
int moe_b200_fused_decode_enabled(void);
/* No reference counterpart.  A/B knob: k-ranges per task of the decode
 * warp-MMA stages (0, the default: chosen per batch; 1-8: forced).  It sizes
 * the layer workspace too, so set it before querying the workspace. */
int moe_b200_force_ksplit(int ksplit);
/* No reference counterpart.  Decode batches of at most 8 tokens (and 256
 * (token, slot) entries) run selection, dispatch, the chunk list and the f16
 * staging of x in one 256-thread launch (1, the default) or in two launches
 * (0).  Same results bit for bit. */
int moe_b200_decode_prologue(int enable);
/* No reference counterpart.  A/B knob: decode warp-MMA units walk their
 * k-blocks from a unit-dependent offset (1) or in order (0, the default);
 * same results to fp32 rounding of the summation order. */
int moe_b200_kb_rotate(int enable);
/* No reference counterpart.  Decode layers on the default GEMV stage the
 * SwiGLU activations inside the gate/up launch and combine the tokens inside
 * the down launch, by the warp that finishes the last piece each needs (1),
 * or run the staging and the combine as launches of their own (0, the
 * default).  Same results bit for bit. */
int moe_b200_fold_epilogues(int enable);
/* No reference counterpart.  Decode layers (tiled weights, the default GEMV)
 * run the shared expert -- which needs no routing -- on a side stream that
 * forks where the layer starts and joins before the combine, on two CTAs per
 * SM, while the router and the dispatch run (1); 0, the default, runs it
 * with the routed experts.  Same results to fp32 rounding (the side launches split
 * the shared expert's k-blocks for their smaller grid).  The side stream of a
 * device is created by its first such call, which should come before any
 * stream capture; layers captured in a graph must not run concurrently with
 * eager layers on the same device (they share the side stream). */
int moe_b200_shared_side(int enable);
/* No reference counterpart.  Decode layers with the one-CTA prologue and bf16
 * hidden states: the router logits launch stages x as f16 with a row scale in
 * a cluster of its own, beside the logits clusters (1, the default), or the
 * prologue stages it (0).  Same results bit for bit. */
int moe_b200_router_stages_x(int enable);

/* ---------------------------------------------------------------------------
 * Pack-file reads (host only): the FP8 pack loader's byte ranges.
 * ------------------------------------------------------------------------- */

/* replaces native_read_tensor_bytes, native/fp16_loader.cpp:33-67 (POSIX
 * pread instead of ReadFile): nbytes at absolute_offset of the file into
 * out.  0 ok, 1 null argument, 2 the file cannot be opened, 3 the range ends
 * past the file, 4 short read. */
int moe_read_tensor_bytes(const char* path, uint64_t absolute_offset, uint64_t nbytes, uint8_t* out);
/* n ranges of one file, range i into outs[i] (host memory, pinned or not),
 * read in pieces of >= 8 MiB by `threads` threads (0: up to 8).  Codes as
 * above. */
int moe_read_spans(const char* path, int64_t n, const uint64_t* offsets, const uint64_t* lengths,
                   uint8_t* const* outs, int64_t threads);

/* Device error word (no reference counterpart): nonzero when a bounded wait
 * inside a kernel gave up (1: producer, 2: consumer, 4: drain, 8: misaligned
 * weights refused by the streaming kernel, 16: warp-MMA ring, 32: prefill
 * tensor-core GEMM pipeline, 128: fused decode experts -- a down piece gave
 * up waiting for its expert's activations), or when an expert-parallel peer
 * kernel skipped a store whose rank, slot or row read from exchanged data was
 * out of range (64).  Synchronises
 * `stream`, returns the word (-1 if it cannot be read) and clears it. */
int moe_b200_device_error(void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H_ */
