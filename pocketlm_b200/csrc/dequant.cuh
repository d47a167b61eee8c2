// FP8 dequant launcher (dequant.cu).
#pragma once
#include <algorithm>
#include "common.cuh"

namespace moe {
cudaError_t launch_fp8_dequant(const uint8_t* w, const float* s, uint16_t* out, int64_t rows, int64_t cols,
                               int64_t scale_cols, bool bf16, cudaStream_t stream);
}  // namespace moe
