// Token dispatch: histogram + prefix sum + stable scatter of (row, expert,
// weight) entries into expert-contiguous segments, and the work-chunk list the
// expert kernels walk.
//
// Replaces the per-expert grouping of run_fp8_moe
// (src/pcketlm/core/runtime/fp8_source.py:1598-1605: `torch.where(route_indices
// == e)` for each selected expert in ascending id order) and the pair lists of
// fp8_e4m3_block_mlp_many_pair_weighted_f32 (src/pcketlm/native/fp8_linear.cpp:
// 833-980).  Within a segment, entries keep their input order, which for the
// routed ids [T, k] means ascending token index -- the order torch.where
// returns.  The scatter is deterministic: the rank of an entry inside its
// bucket comes from a per-bucket bitmask of the current 1024-entry window, not
// from atomics.
#include <algorithm>

#include "common.cuh"
#include "dispatch.cuh"
#include "dispatch_device.cuh"
#include "router_device.cuh"

namespace moe {


__global__ void __launch_bounds__(kBucketThreads) bucket_kernel(BucketArgs a) {
  extern __shared__ uint32_t sm[];
  bucket_body(a, sm);
}

__global__ void __launch_bounds__(kBucketThreads) chunk_kernel(ChunkArgs a) {
  chunk_body(a);
}

// Decode batches in one launch: select every token's experts (one warp per
// token, logits given as split-K partials), then bucket the (token, slot)
// entries by expert and build the chunk list -- the work of
// router_select_kernel + bucket_kernel + chunk_kernel without two launch gaps.
__global__ void __launch_bounds__(kBucketThreads) route_dispatch_kernel(RouteDispatchArgs a) {
  extern __shared__ uint32_t sm[];
  const int warp = threadIdx.x / kWarp;
  const int E = a.select.experts, T = a.select.tokens;
  // logits = sum of the split-K partials, in part order, summed by the whole CTA
  float* logits = reinterpret_cast<float*>(sm);
  for (int i = threadIdx.x; i < T * E; i += kBucketThreads) {
    float parts[kMaxRouterParts];
#pragma unroll
    for (int q = 0; q < kMaxRouterParts; ++q) parts[q] = q < a.nparts ? a.partial[q * a.part_stride + i] : 0.0f;
    float v = parts[0];
#pragma unroll
    for (int q = 1; q < kMaxRouterParts; ++q) v += q < a.nparts ? parts[q] : 0.0f;
    logits[i] = v;
  }
  __syncthreads();
  float* scratch = logits + static_cast<size_t>(T) * E + static_cast<size_t>(warp) * 2 * E;
  for (int t = warp; t < T; t += kBucketThreads / kWarp)
    select_token(logits, 1, 0, a.bias, a.select, t, scratch, scratch + E, a.ids64, a.bucket.keys_out,
                 a.bucket.weights_out, a.weights_bf16);
  __syncthreads();
  bucket_body(a.bucket.args, sm);
  __syncthreads();
  chunk_body(a.chunks);
}

size_t route_dispatch_smem_bytes(int tokens, int experts) {
  const size_t select = (static_cast<size_t>(tokens) * experts +
                         static_cast<size_t>(kBucketThreads / kWarp) * 2 * experts) * sizeof(float);
  return std::max(select, bucket_smem_bytes(experts));
}

cudaError_t launch_route_dispatch(const RouteDispatchArgs& a, cudaStream_t stream) {
  const size_t smem = route_dispatch_smem_bytes(a.select.tokens, a.select.experts);
  if (smem > 200 * 1024 || a.nparts > kMaxRouterParts) return cudaErrorInvalidValue;
  cudaError_t err = cudaFuncSetAttribute(route_dispatch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  route_dispatch_kernel<<<1, kBucketThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

size_t bucket_smem_bytes(int n_buckets) {
  return static_cast<size_t>(n_buckets) * kWindowWords * sizeof(uint32_t) +
         static_cast<size_t>(2 * n_buckets + 1) * sizeof(int32_t);
}

cudaError_t launch_bucket(const BucketArgs& a, cudaStream_t stream) {
  const size_t smem = bucket_smem_bytes(a.n_buckets);
  if (a.n_buckets <= 0 || a.n_buckets > kMaxBuckets) return cudaErrorInvalidValue;
  cudaError_t err = cudaFuncSetAttribute(bucket_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  bucket_kernel<<<1, kBucketThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_chunks(const ChunkArgs& a, cudaStream_t stream) {
  chunk_kernel<<<1, kBucketThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace moe
