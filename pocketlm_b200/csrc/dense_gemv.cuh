// Grouped GEMV launchers for the non-FP8 expert formats (dense_gemv.cu):
// 16-bit dense weights (fp16 / bf16, the reference's fp16_moe.cpp) and
// row-scaled signed int4 (q4_dequant.cpp).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace moe {

enum WeightKind : int { kWF16 = 0, kWBF16 = 1, kWQ4 = 2 };

// Layout of the staged activation rows the MMA kernel reads as its B operand.
//   kStageF16:      f16 [rows, K], x / xscale[row] (a power of two; 1 when unscaled)
//   kStageF16Perm8: the same, each aligned group of 8 stored as k0 k4 k1 k5 k2 k6 k3 k7
//   kStageBF16HiLo: bf16 [2][rows, K]: hi = bf16(x), lo = bf16(x - hi); xscale = 1
enum StageMode : int { kStageF16 = 0, kStageF16Perm8 = 1, kStageBF16HiLo = 2 };

// The stage mode a weight kind's MMA kernel expects.
constexpr int stage_mode_for(int kind) {
  return kind == kWQ4 ? kStageF16Perm8 : kind == kWBF16 ? kStageBF16HiLo : kStageF16;
}

struct DenseArgs {
  // per-segment device tables of device addresses (uint64): weights [N, K]
  // (16-bit elements, or int4 packed two per byte, even k in the low nibble)
  // and, for int4, fp16 row scales [N]; w1/s1 only for two streams
  const uint64_t* w0;
  const uint64_t* s0;
  const uint64_t* w1;
  const uint64_t* s1;
  const uint16_t* xs;        // staged activations (StageMode), MMA kernel
  const float* xscale;       // [rows] staging scales, MMA kernel
  int64_t plane;             // elements between the hi and lo planes (kStageBF16HiLo)
  const float* x;            // fp32 activations [rows, K], generic kernel
  const int32_t* pair_row;   // [P] activation row per pair, or null: row = pair
  const int32_t* chunk_seg;  // chunk list (chunks of <= 8 pairs)
  const int32_t* chunk_start;
  const int32_t* chunk_len;
  const int32_t* n_chunks;
  float* out0;               // [P, N]
  int N;
  int K;
  int ksplit;                // MMA kernel: k ranges per task (1: none)
  float* partial;            // [tasks * ksplit, 32, 8] when ksplit > 1
  int32_t* counters;         // [tasks]: zero on entry, left zero on exit
};

// Whether the MMA kernel takes this shape (K a multiple of its span: 32 for
// 16-bit weights, 128 for int4).
bool dense_mma_supported(int kind, int K);
// Output rows of one warp task (16 with two streams, 32 with one).
constexpr int dense_task_rows(int ns) { return ns == 2 ? 16 : 32; }
int dense_mma_ksplit(int kind, int64_t tasks_bound, int K);
cudaError_t launch_dense_mma_gemv(const DenseArgs& a, int kind, int ns, int epi, int64_t tasks_bound,
                                  cudaStream_t stream);
// Any shape: one warp per (pair, output row), fp32 activations a.x.
cudaError_t launch_dense_generic_gemv(const DenseArgs& a, int kind, int ns, int epi, int64_t pairs,
                                      cudaStream_t stream);

// Activation rows (fp32, bf16 or f16 source: src_dtype Dtype) -> staged
// layout `mode`.  scaled: divide each row by a power of two putting its
// largest magnitude in [2^13, 2^14) (f16 modes); otherwise plain RNE
// conversion.  Rows past *n_rows_dev (when given) are skipped.
cudaError_t launch_stage_rows(const void* src, int src_dtype, int rows, int K, const int32_t* n_rows_dev,
                              int mode, bool scaled, uint16_t* dst, float* scale, int64_t plane,
                              int32_t* zero, int64_t zero_n, cudaStream_t stream);

// Fill table[i] = base + i * stride_bytes for i < n (device).
cudaError_t launch_fill_table(uint64_t* table, const void* base, int64_t stride_bytes, int n, cudaStream_t stream);

// Q4: out[c * size + k] = fp16(code(c * size + k) * scale[c]), code the
// signed int4 at flat index c * size + k (even index in the low nibble).
cudaError_t launch_q4_dequant(const uint8_t* packed, const uint16_t* scales, uint16_t* out, int64_t channels,
                              int64_t size, cudaStream_t stream);
// fp32 copy of n elements of a bf16 / f16 / fp32 array (Dtype).
cudaError_t launch_to_f32(const void* src, int src_dtype, int64_t n, float* dst, cudaStream_t stream);

// row8 layout: packed[(blk * cols + c) * 8 + lane] = w[blk * 8 + lane, c] (0 past rows).
cudaError_t launch_pack_rows8(const uint16_t* w, uint16_t* packed, int64_t rows, int64_t cols, cudaStream_t stream);
// out[r] = sum_c x[c] * W[r, c] in fp32 from the row8 layout; dtype Dtype (bf16 or f16).
cudaError_t launch_rows8_gemv(const uint16_t* x, const uint16_t* packed, float* out, int64_t rows, int64_t cols,
                              int dtype, cudaStream_t stream);

}  // namespace moe
