// Router launchers (router.cu).
#pragma once
#include <cuda_fp16.h>
#include "common.cuh"

namespace moe {

// Element types of activations / router weights.
enum Dtype : int { kDtypeF32 = 0, kDtypeBF16 = 1, kDtypeF16 = 2 };
enum Scoring : int { kScoreSigmoid = 0, kScoreSoftmax = 1 };

struct RouterSelectParams {
  int tokens;
  int experts;       // <= 2048, divisible by n_group
  int top_k;         // <= 32
  int n_group;       // <= 32; 1 disables the group mask
  int topk_group;
  int scoring;       // Scoring
  int renorm;        // divide the picked probabilities by their sum
  int softmax_fp64;  // ds_router_topk_u16 semantics: fp64 denominators
  int round_bf16;    // round the final weights through bf16 (fp8_source.py:1547)
  float route_scale;
};

cudaError_t launch_router_logits(const void* x, int x_dtype, const void* w, int w_dtype, float* logits,
                                 int tokens, int hidden, int experts, cudaStream_t stream);

// Split-K logits for decode batches: partial[q][t][e], q < router_split_parts(hidden)
// (at most kMaxRouterParts), each part router_split_kpart(hidden) columns (a
// multiple of 32); the parts are summed in order by the selection.
constexpr int kMaxRouterParts = 16;
int router_split_parts(int hidden);
int router_split_kpart(int hidden);
cudaError_t launch_router_logits_split(const void* x, int x_dtype, const void* w, int w_dtype, float* partial,
                                       int tokens, int hidden, int experts, cudaStream_t stream);

// Decode-batch logits [T, E] in one launch (clusters of 8 CTAs reduce over k
// in distributed shared memory): bf16 x bf16 or f16 x f16, hidden % 32 == 0,
// 16-byte aligned operands; cudaErrorNotSupported otherwise.  With x16 (and
// xscale; tokens <= 256, 16-byte aligned), one more cluster stages x meanwhile:
// x16 = x / xscale in f16, xscale a power of two per row, exactly the
// rows_to_f16 staging.
cudaError_t launch_router_logits_cluster(const void* x, int x_dtype, const void* w, int w_dtype, float* logits,
                                         int tokens, int hidden, int experts, cudaStream_t stream,
                                         __half* x16 = nullptr, float* xscale = nullptr);

// logits: nparts partial [T, E] matrices part_stride floats apart, summed in part order.
cudaError_t launch_router_select(const float* logits, const float* bias, const RouterSelectParams& p,
                                 int64_t* ids64, int32_t* ids32, float* weights_f32,
                                 __nv_bfloat16* weights_bf16, cudaStream_t stream, int nparts = 1,
                                 int64_t part_stride = 0);
// Whether launch_router_logits_split runs on the tensor cores for these operands
// (bf16 x bf16 or f16 x f16, 16-byte aligned, hidden % 32 == 0).
bool router_split_is_mma(const void* x, int x_dtype, const void* w, int w_dtype, int hidden);

}  // namespace moe
