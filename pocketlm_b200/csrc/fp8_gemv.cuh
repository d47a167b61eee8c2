// Grouped FP8 GEMV launchers (fp8_gemv.cu).
#pragma once
#include <cuda_fp16.h>

#include "common.cuh"

namespace moe {

enum GemvEpilogue : int { kEpiStore = 0, kEpiSwiglu = 1, kEpiStoreBoth = 2 };
enum GemvX : int { kXF32 = 0, kXBF16 = 1 };

struct GemvArgs {
  // per-segment device tables of device addresses (uint64): weights and
  // fp32 [ceil(N/128), scale_cols] block scales; w1/s1 only for two streams
  const uint64_t* w0;
  const uint64_t* s0;
  const uint64_t* w1;
  const uint64_t* s1;
  const void* x;             // activations [rows, K] (float or bf16)
  const int32_t* pair_row;   // [P] row of x for each pair, or null: row = pair
  const int32_t* chunk_seg;  // chunk list (dispatch.cuh)
  const int32_t* chunk_start;
  const int32_t* chunk_len;
  const int32_t* n_chunks;   // device scalar
  float* out0;               // [P, N]
  float* out1;               // [P, N] (kEpiStoreBoth)
  int N;                     // output rows per expert
  int K;                     // reduction length
  int scale_cols;            // ceil(K / 128)
};

struct CombineArgs {
  const float* y;            // [P, H] fp32, or null when y16 is given
  const __nv_bfloat16* y16;  // [P, H] bf16 (the prefill GEMM's rounded expert outputs), or null
  const int32_t* row_ptr;    // [T + 1] or null: row t owns [t*stride, (t+1)*stride)
  int stride;
  const int32_t* row_pairs;  // pair index per list entry (-1 = skip), or null: entry = pair
  const float* pair_weight;  // [P] or null: weight 1
  int extra_base;            // >= 0: also add y[extra_base + t] with weight 1 (shared expert)
  int T;
  int H;
  float* out_f32;            // [T, H] or null
  __nv_bfloat16* out_bf16;   // [T, H] or null
  __half* out_f16;           // [T, H] or null
  int bf16_via_f16;          // out_bf16 = bf16(f16(sum)): an fp16 result handed on as bf16
};

// Largest supported chunk size (1, 4 or 8 rows) whose staged rows fit in
// shared memory; 0 when even one row does not fit.
int gemv_chunk_tokens(int K, int x_dtype);
int gemv_grid_ctas();

cudaError_t launch_grouped_gemv(const GemvArgs& a, int x_dtype, int ns, int epi, int nt, bool vec,
                                cudaStream_t stream);
cudaError_t launch_combine(const CombineArgs& a, cudaStream_t stream);

// Warp-specialised variant (fp8_stream.cu): bulk-copy weight ring.  Needs
// K % 16 == 0 and 16-byte aligned weight rows.
bool stream_gemv_supported(int K, int x_dtype, int nt);
cudaError_t launch_stream_gemv(const GemvArgs& a, int x_dtype, int ns, int epi, int nt, cudaStream_t stream);
// Warp-MMA GEMV (fp8_mma.cu), layer path: activations staged as f16 rows with
// per-row power-of-two scales.  Needs K % 128 == 0.
struct MmaArgs {
  const uint64_t* w0;
  const uint64_t* s0;
  const uint64_t* w1;
  const uint64_t* s1;
  const __half* x16;         // [rows, K] activations / scale
  const float* xscale;       // [rows]
  const int32_t* pair_row;   // [P] row of x16 per pair, or null: row = pair
  const int32_t* chunk_seg;  // chunk list (chunks of <= 8 pairs)
  const int32_t* chunk_start;
  const int32_t* chunk_len;
  const int32_t* n_chunks;
  float* out0;               // [P, N]
  int N;
  int K;
  int scale_cols;
  int nanfix;                // decode e4m3 0x7F/0xFF as +0 (the reference's linear semantics)
  const uint8_t* nan_free;   // [segments] or null: 1 = the expert holds no 0x7F/0xFF code (no fix needed)
  int tiled;                 // cp.async kernel: weights in the fragment-native tiled layout (launch_fp8_tile)
  int ksplit;                // register-fed kernel: k-block ranges per task (1: none)
  float* partial;            // [tasks * ksplit, 32, 8] fp32 fragments when ksplit > 1
  int32_t* counters;         // [tasks] arrival counters: zero on entry, left zero on exit
  int kb_rotate;             // cp.async kernels: start each unit's k-block walk at a unit-dependent offset
  // cp.async kernel, gate/up (NS 2) -- fold the activation staging in: the
  // warp completing a chunk's last task stages its pairs' rows out0 -> f16
  // (rows_to_f16_kernel's arithmetic).  Null: no staging.
  __half* stage_x16;         // [P, N]
  float* stage_scale;        // [P]
  int32_t* chunk_done;       // [chunks] completed tasks; zero on entry
  // cp.async kernel, down (NS 1) -- fold the combine in: the warp adding a
  // token's last pair row to a 32-column tile combines that tile (combine_kernel's
  // arithmetic: slots in order, then the shared row, one bf16 rounding).  Null: no combine.
  __nv_bfloat16* comb_out;   // [T, N]
  int32_t* comb_cnt;         // [T, ceil(N / 32)] arrivals; zero on entry
  const int32_t* pair_token; // [P] token of each pair
  const int32_t* entry_pair; // [T * comb_k] pair of each (token, slot), -1 = none
  const float* pair_weight;  // [P]
  int comb_k;                // routed slots per token
  int comb_shared_base;      // >= 0: token t's shared row is pair comb_shared_base + t
  int comb_need;             // pair rows per token (routed slots kept + the shared one)
};
constexpr int kMaxMmaKSplit = 8;
// Rows of one warp task of the MMA kernels: 16 (gate + up) or 32 (one matrix).
constexpr int mma_task_rows(int ns) { return ns == 2 ? 16 : 32; }
bool mma_gemv_supported(int K, int N);
// k-split for an upper bound on the launch's tasks (chunks x row tiles): 1
// when the tasks already occupy every resident warp.
int mma_gemv_ksplit(int64_t tasks_bound, int K);
cudaError_t launch_mma_gemv(const MmaArgs& a, int ns, int epi, int64_t tasks_bound, cudaStream_t stream);
// Same computation, weights staged through a per-warp shared-memory ring by
// cp.async (fp8_mma.cu); tasks_bound as for launch_mma_gemv.
int async_gemv_ksplit(int64_t tasks_bound, int K);
// Resident CTAs per SM of the cp.async kernel, and its k-split for a grid of `ctas` CTAs.
int async_gemv_ctas_per_sm();
int async_gemv_ksplit_for(int64_t tasks_bound, int K, int64_t ctas);
// max_ctas > 0 caps the grid (a launch that shares the GPU with another stream's kernels).
cudaError_t launch_async_mma_gemv(const MmaArgs& a, int ns, int epi, int64_t tasks_bound, cudaStream_t stream,
                                  int64_t max_ctas = 0);
// Fused decode experts (decode_fused_kernel, tiled or row-major weights): the
// gate/up + SwiGLU stage (up), the f16 staging of its activations and the down
// stage (down) in one persistent launch.  up.out0 = act fp32 [P, I]; down.x16 /
// down.xscale = where the activations are staged ([P, I] f16, [P]); down.out0
// = y.  partial: [2][2 * partial_warps][32 * 8] fp32; cnt_up [up tasks],
// cnt_down [down tasks], chunk_up / chunk_ready [chunks]: zero on entry.
struct DecodeFusedArgs {
  MmaArgs up;
  MmaArgs down;
  float* partial;
  int partial_warps;
  int32_t* cnt_up;
  int32_t* cnt_down;
  int32_t* chunk_up;
  int32_t* chunk_ready;
};
// Warps of the fused launch (all resident at once): sizes `partial`.
int decode_fused_warps();
cudaError_t launch_decode_fused(const DecodeFusedArgs& a, cudaStream_t stream);
// Fragment-native ("tiled") weight layout, read by the cp.async decode GEMV
// and the prefill GEMM.  Row tile t = rows 16t .. 16t + 15; group = 8 row
// tiles (128 rows).  For every (group, 128-column k-block kb, 64-column half
// sp) an 8 KiB block holds the group's 8 row tiles in order, 1 KiB each; a
// row tile's 1 KiB is two 512-byte pieces (rr = 0: rows g, rr = 1: rows
// g + 8) of 32 lanes x 16 bytes, lane l = 4g + c holding columns
// 64 sp + 16 c .. + 15 of row 16t + g + 8 rr.  So a warp-wide 16-byte
// access is 512 contiguous bytes (decode), and 128 rows x 64 columns of a
// matrix are one 8 KiB run (one bulk copy of the prefill GEMM).
constexpr int64_t kTileGroupRows = 128;
constexpr int64_t kTileRunBytes = 8192;  // one (group, kb, sp) block
MOE_HD int64_t tiled_offset(int64_t tile, int64_t kb, int sp, int nkb) {
  return (((tile / 8) * nkb + kb) * 2 + sp) * kTileRunBytes + (tile % 8) * 1024;
}
MOE_HD int64_t fp8_tiled_bytes_dev(int64_t rows, int64_t cols) {
  return (rows + kTileGroupRows - 1) / kTileGroupRows * kTileGroupRows * cols;
}
// Bytes of the tiled copy of a row-major e4m3 [rows, cols] matrix (cols %
// 128 == 0; rows padded to a multiple of 128 with zeros), and the repacking launch.
int64_t fp8_tiled_bytes(int64_t rows, int64_t cols);
cudaError_t launch_fp8_tile(const uint8_t* src, uint8_t* dst, int64_t rows, int64_t cols, cudaStream_t stream);
// Per-expert flags for MmaArgs::nan_free: flags[s] = 1 when none of the
// gate / up / down e4m3 weights of expert s (device tables [6][S], absent
// experts count as clean) is 0x7F or 0xFF.
cudaError_t launch_nan_free_flags(const uint64_t* tables, int S, int64_t inter, int64_t hidden, uint8_t* flags,
                                  cudaStream_t stream);
// Same computation, weights fed to each warp by TMA bulk copies (fp8_mma.cu).
cudaError_t launch_tma_mma_gemv(const MmaArgs& a, int ns, int epi, cudaStream_t stream);
int read_and_clear_mma_device_error(cudaStream_t stream);
// the rows_to_f16 staging of fp16 rows (dst = src / power-of-two scale, exact)
cudaError_t launch_f16_rows_to_f16(const void* src, int rows, int K, __half* dst, float* scale, cudaStream_t stream);
// Also zeroes zero[0, zero_n) (the k-split counters of the stages that follow).
cudaError_t launch_rows_to_f16(const void* src, bool src_bf16, int rows, int K, const int32_t* n_rows_dev,
                               __half* dst, float* scale, int32_t* zero, int64_t zero_n, cudaStream_t stream);

// Device error word of the bounded waits; returns it (or -1) and clears it.
int read_and_clear_device_error(cudaStream_t stream);

}  // namespace moe
