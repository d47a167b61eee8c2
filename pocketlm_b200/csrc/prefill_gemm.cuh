// Prefill grouped GEMM on tcgen05 (prefill_gemm.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace moe {

struct PrefillArgs {
  // per-segment device tables: weights in the fragment-native tiled layout
  // (launch_fp8_tile) and fp32 block scales [ceil(N/128), scale_cols]
  const uint64_t* w0;      // gate (gate/up GEMM) or down
  const uint64_t* s0;
  const uint64_t* w1;      // up (gate/up GEMM only)
  const uint64_t* s1;
  const __half* a16;       // [rows_a, K] pair-ordered activations / ascale
  const float* ascale;     // [rows_a] power-of-two row scales
  int64_t rows_a;          // pairs (TMA bound; rows past it read as zero)
  const int32_t* seg_offset;  // [n_segments + 1] pair ranges per expert
  const int32_t* mprefix;     // [n_segments + 1] from launch_prefill_tiles
  int n_segments;
  float* out;              // [rows_a, N] fp32 (gate/up: SwiGLU activations)
  // down GEMM only, or null: pair p's output row goes to out_row[p] (N fp32,
  // 16-byte aligned; may be another GPU's memory) instead of out + p * N
  const uint64_t* out_row;
  // down GEMM only, or null: the outputs as bf16 rows [rows_a, N] instead of fp32 (each expert's
  // output rounded once, as the reference rounds it before its weighted add)
  __nv_bfloat16* out16;
  int out_row_bf16;        // with out_row: the table's rows are bf16 (N values), not fp32
  int N;                   // output columns (gate/up: intermediate size)
  int K;
  int scale_cols;          // ceil(K / 128)
  int nanfix;              // decode e4m3 0x7F / 0xFF as +0
  const uint8_t* nan_free; // [n_segments] or null: 1 = the expert holds no such code
  int wformat;             // kPrefillFp8Block or kPrefillQ4Row
};

// Weight formats of the prefill GEMM: e4m3 with 128 x 128 fp32 block scales
// in the fragment-native tiled layout (fp8_gemv.cuh), or signed int4 codes
// (two per byte, even k in the low nibble) with one fp16 scale per output
// row, in the Q4 tiled layout below.
constexpr int kPrefillFp8Block = 0;
constexpr int kPrefillQ4Row = 1;

// Q4 tiled layout: for every 128-row group and 64-code k-block, a 4 KiB run
// holding the group's rows in order, 32 bytes (64 codes) each.  Rows padded to
// a multiple of 128 with zero bytes; K % 64 == 0.
MOE_HD int64_t q4_tiled_offset(int64_t group, int64_t kblk, int64_t nkblk) { return (group * nkblk + kblk) * 4096; }
int64_t q4_tiled_bytes(int64_t rows, int64_t K);
cudaError_t launch_q4_tile(const uint8_t* packed, uint8_t* tiled, int64_t rows, int64_t K, cudaStream_t stream);

size_t prefill_smem_bytes();
// K % 128 == 0; N % 128 (gate/up) or % 256 (down) == 0.
bool prefill_supported(int64_t K, int64_t N, bool gateup);
cudaError_t launch_prefill_tiles(const int32_t* seg_offset, int n_segments, int32_t* mprefix, cudaStream_t stream);
cudaError_t launch_gather_rows(const __half* x16, const float* xscale, const int32_t* pair_row, int64_t P, int64_t K,
                               __half* xa, float* ascale, cudaStream_t stream);
// Stage the tokens' rows as fp16 / power-of-two scale straight into their pairs'
// A rows (entry_pair [T, k], -1 = dropped; with tail_first, the shared pair of
// token t is *tail_first + t): the staging plus gather_rows in one read of x.
// cudaErrorNotSupported when a row exceeds 16 KiB or is not 16-byte aligned.
cudaError_t launch_scatter_rows(const void* x, int x_dtype, int64_t T, int64_t K, const int32_t* entry_pair, int k,
                                const int32_t* tail_first, __half* a16, float* ascale, cudaStream_t stream);
// max_tiles: an upper bound on the tiles (grid size); the kernel reads the real count.
cudaError_t launch_prefill_gemm(const PrefillArgs& a, bool gateup, int64_t max_tiles, cudaStream_t stream);
int read_and_clear_prefill_device_error(cudaStream_t stream);

// Router logits of prefill-sized batches on tcgen05 (prefill_gemm.cu):
// *nparts k-range partials [nparts][tokens][experts] (summed in part order by
// the selection).  cudaErrorNotSupported unless x and w are both bf16 or both
// f16 (dtype codes of router.cuh), 16-byte aligned, hidden % 64 == 0.
constexpr int kMaxRouterTcParts = 16;
int router_tc_parts(int64_t tokens, int64_t hidden, int64_t experts);
cudaError_t launch_router_logits_tc(const void* x, int xdtype, const void* w, int wdtype, float* partial,
                                    int64_t tokens, int64_t hidden, int64_t experts, int* nparts,
                                    cudaStream_t stream);

}  // namespace moe
