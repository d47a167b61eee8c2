// Host-side routing shared by the C entry points (defined in capi.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace moe {

// Router logits + selection on `stream`: ids (int64 and/or int32) and
// weights (fp32 and/or bf16 bits) of the top-k experts per token.  logits:
// scratch of T * E floats.
int route_impl(const void* hidden, int hd, const void* w, int wd, const float* bias, int64_t T, int64_t H,
               int64_t E, int64_t n_group, int64_t topk_group, int64_t k, int scoring, int renorm, int fp64,
               float scale, int round_bf16, int64_t* ids64, int32_t* ids32, float* wf32, uint16_t* wbf16,
               float* logits, cudaStream_t stream);
// Argument checks of the routed entry points (codes of status.cuh).
int check_route(int64_t T, int64_t H, int64_t E, int64_t n_group, int64_t topk_group, int64_t k);

}  // namespace moe
