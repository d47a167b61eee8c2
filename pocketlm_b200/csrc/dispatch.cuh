// Dispatch launchers (dispatch.cu).
#pragma once
#include "common.cuh"
#include "router.cuh"

namespace moe {

constexpr int kMaxBuckets = 1536;  // bitmask window in shared memory: 128 B per bucket

struct BucketArgs {
  const int32_t* keys;     // [n]
  const int32_t* rows;     // [n] or null: row = i / k
  const float* weights;    // [n] or null: weight 1
  int n;
  int k;
  int key_lo;
  int n_buckets;
  int32_t* bucket_offset;  // [n_buckets + 1]
  int32_t* pair_row;       // [total]
  float* pair_weight;      // [total] or null
  int32_t* pair_entry;     // [total] or null: source entry of each pair
  int32_t* entry_pair;     // [n] or null: pair of each entry, -1 when dropped
  int32_t* counts;         // [n_buckets] or null
  int32_t* total;          // [1] or null
  int tail;                // > 0: append one more bucket holding rows 0..tail-1, weight 1
                           // (the shared expert); bucket_offset then has n_buckets + 2 entries
  int32_t* block_counts;   // or null: bucket_scratch_ints(n, n_buckets) ints of workspace for
                           // the multi-CTA path (large n); null keeps the one-CTA kernel
};
// Workspace ints of BucketArgs::block_counts: per-block bucket counts.
int64_t bucket_scratch_ints(int64_t n, int n_buckets);

struct ChunkArgs {
  const int32_t* seg_offset;  // [n_segments + 1]
  int n_segments;
  int chunk;                  // max pairs per chunk
  int32_t* chunk_seg;         // [capacity]
  int32_t* chunk_start;
  int32_t* chunk_len;
  int32_t* n_chunks;          // [1]
};

// Upper bound on the chunk count for `pairs` pairs in `segments` segments.
inline int64_t chunk_capacity(int64_t pairs, int64_t segments, int chunk) {
  return pairs / chunk + segments + 1;
}

// Fused selection + bucket + chunk list (one CTA) for decode batches.
struct RouteDispatchArgs {
  const float* partial;       // split-K router logits partials
  int nparts;
  int64_t part_stride;        // floats between consecutive parts (tokens * experts)
  const float* bias;          // [experts] or null
  RouterSelectParams select;
  int64_t* ids64;             // optional user outputs
  __nv_bfloat16* weights_bf16;
  struct {
    int32_t* keys_out;        // == args.keys (ids32)
    float* weights_out;       // == args.weights (fp32 route weights)
    BucketArgs args;
  } bucket;
  ChunkArgs chunks;
};
size_t route_dispatch_smem_bytes(int tokens, int experts);
cudaError_t launch_route_dispatch(const RouteDispatchArgs& a, cudaStream_t stream);

// route_dispatch_kernel's work plus the x staging (rows_to_f16_kernel) and the
// zeroing of `zero` in one 256-thread CTA, for up to 8 tokens, tokens x top_k <=
// 256 entries and <= 256 routed experts (decode_prologue_supported); rd.nparts must be 1.
constexpr int kPrologueThreads = 256;
struct DecodePrologueArgs {
  RouteDispatchArgs rd;
  const void* x;       // [tokens, hidden] bf16 or fp32, 16-byte aligned rows
  int hidden;
  __half* x16;         // [tokens, hidden] x / xscale
  float* xscale;       // [tokens]
  int stage_x;         // 0: x16 / xscale were staged already (by the router launch)
  int32_t* zero;       // [zero_n] set to 0
  int64_t zero_n;
};
bool decode_prologue_supported(int tokens, int experts, int top_k, int hidden, int x_dtype, const void* x,
                               int n_segments);
cudaError_t launch_decode_prologue(const DecodePrologueArgs& a, int x_dtype, cudaStream_t stream);

size_t bucket_smem_bytes(int n_buckets);
cudaError_t launch_bucket(const BucketArgs& a, cudaStream_t stream);
cudaError_t launch_chunks(const ChunkArgs& a, cudaStream_t stream);

}  // namespace moe
