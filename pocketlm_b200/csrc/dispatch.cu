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
  if (a.n <= kBucketThreads) bucket_body_small(a, sm);
  else bucket_body(a, sm);
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
  if (a.nparts == 1) {
    // one part: eight independent loads in flight per thread
    for (int i0 = threadIdx.x; i0 < T * E; i0 += 8 * kBucketThreads) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * kBucketThreads;
        v[u] = i < T * E ? a.partial[i] : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (i0 + u * kBucketThreads < T * E) logits[i0 + u * kBucketThreads] = v[u];
    }
  } else {
    for (int i = threadIdx.x; i < T * E; i += kBucketThreads) {
      float parts[kMaxRouterParts];
#pragma unroll
      for (int q = 0; q < kMaxRouterParts; ++q) parts[q] = q < a.nparts ? a.partial[q * a.part_stride + i] : 0.0f;
      float v = parts[0];
#pragma unroll
      for (int q = 1; q < kMaxRouterParts; ++q) v += q < a.nparts ? parts[q] : 0.0f;
      logits[i] = v;
    }
  }
  __syncthreads();
  float* scratch = logits + static_cast<size_t>(T) * E + static_cast<size_t>(warp) * 2 * E;
  for (int t = warp; t < T; t += kBucketThreads / kWarp)
    select_token(logits, 1, 0, a.bias, a.select, t, scratch, scratch + E, a.ids64, a.bucket.keys_out,
                 a.bucket.weights_out, a.weights_bf16);
  __syncthreads();
  if (a.bucket.args.n <= kBucketThreads) bucket_body_small(a.bucket.args, sm);
  else bucket_body(a.bucket.args, sm);
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

// ---------------------------------------------------------------- decode prologue
// Small decode batches (tokens x top_k <= 256 entries, <= 256 routed experts)
// in ONE 256-thread CTA: each warp selects its tokens' experts
// (select_token, the routing of route_dispatch_kernel bit for bit) and stages
// their x rows to f16 with a power-of-two row scale (rows_to_f16_kernel's
// arithmetic); then every thread owns one entry: expert buckets in ascending
// expert id, tokens in order inside a bucket (the order of bucket_body_small),
// the shared expert's rows appended, and the chunk list (chunk_body's).  The
// expert kernels' counters are cleared on the way.  Replaces
// route_dispatch_kernel + rows_to_f16_kernel (two launches, one of 1024
// threads mostly waiting at barriers) for batches of up to eight tokens.

// Exclusive scan of one int per thread over 256 threads; *total = the sum.
// Ends with the CTA synchronised.
static __device__ int cta_exclusive_scan256(int v, int* total) {
  __shared__ int part[kPrologueThreads / 32];
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += n;
  }
  __syncthreads();
  if (lane == 31) part[warp] = incl;
  __syncthreads();
  int before = 0, all = 0;
#pragma unroll
  for (int w = 0; w < kPrologueThreads / 32; ++w) {
    before += w < warp ? part[w] : 0;
    all += part[w];
  }
  __syncthreads();
  *total = all;
  return before + incl - v;
}

template <typename XT>
__global__ void __launch_bounds__(kPrologueThreads) decode_prologue_kernel(DecodePrologueArgs a) {
  extern __shared__ float psm[];
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  const RouteDispatchArgs& rd = a.rd;
  const int T = rd.select.tokens, E = rd.select.experts;
  for (int64_t i = tid; i < a.zero_n; i += kPrologueThreads) a.zero[i] = 0;
  // 1. per token, one warp: selection, then the x row staged to f16
  constexpr int V = 16 / sizeof(XT);
  const int n16 = a.hidden / V;
  float* scratch = psm + warp * 2 * E;
  for (int t = warp; t < T; t += kPrologueThreads / kWarp) {
    select_token(rd.partial, 1, 0, rd.bias, rd.select, t, scratch, scratch + E, rd.ids64, rd.bucket.keys_out,
                 rd.bucket.weights_out, rd.weights_bf16);
    if (!a.stage_x) continue;
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const XT*>(a.x) + static_cast<int64_t>(t) * a.hidden);
    float amax = 0.0f;
    for (int i0 = lane; i0 < n16; i0 += 4 * kWarp) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = i0 + u * kWarp < n16 ? __ldg(src + i0 + u * kWarp) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float f[V];
        unpack16<XT>(v[u], f);
#pragma unroll
        for (int j = 0; j < V; ++j) amax = fmaxf(amax, fabsf(f[j]));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    const float sc = (amax > 0.0f && isfinite(amax)) ? ldexpf(1.0f, ilogbf(amax) - 13) : 1.0f;
    const float inv = 1.0f / sc;  // exact: power of two
    __half* dst = a.x16 + static_cast<int64_t>(t) * a.hidden;
    for (int i = lane; i < n16; i += kWarp) {
      float f[V];
      unpack16<XT>(__ldg(src + i), f);
      __align__(16) __half h[V];
#pragma unroll
      for (int j = 0; j < V; ++j) h[j] = __float2half_rn(f[j] * inv);
      if (V == 8) *reinterpret_cast<uint4*>(dst + i * V) = *reinterpret_cast<const uint4*>(h);
      else *reinterpret_cast<uint2*>(dst + i * V) = *reinterpret_cast<const uint2*>(h);
    }
    if (lane == 0) a.xscale[t] = sc;
  }
  __syncthreads();  // the selections (global keys and weights) are visible to the whole CTA

  // 2. buckets: thread i owns entry i
  const BucketArgs& b = rd.bucket.args;
  int* keys_s = reinterpret_cast<int*>(psm);     // [256]
  int* count = keys_s + kPrologueThreads;         // [256]: per-expert counts
  int* start = count + kPrologueThreads;          // [256]: per-expert first pair
  int key = -1;
  if (tid < b.n) {
    key = b.keys[tid] - b.key_lo;
    if (key < 0 || key >= b.n_buckets) key = -1;
  }
  keys_s[tid] = key;
  count[tid] = 0;
  __syncthreads();
  if (key >= 0) atomicAdd(&count[key], 1);
  __syncthreads();
  const int mine = tid < b.n_buckets ? count[tid] : 0;
  int kept = 0;
  const int off = cta_exclusive_scan256(mine, &kept);
  if (tid < b.n_buckets) {
    b.bucket_offset[tid] = off;
    start[tid] = off;
    if (b.counts) b.counts[tid] = mine;
  }
  if (tid == 0) {
    b.bucket_offset[b.n_buckets] = kept;
    if (b.tail > 0) b.bucket_offset[b.n_buckets + 1] = kept + b.tail;
    if (b.total) *b.total = kept + (b.tail > 0 ? b.tail : 0);
  }
  __syncthreads();
  if (key >= 0) {
    int rank = 0;
    for (int j = 0; j < tid; ++j) rank += keys_s[j] == key;
    const int pp = start[key] + rank;
    b.pair_row[pp] = b.rows ? b.rows[tid] : tid / b.k;
    if (b.pair_weight) b.pair_weight[pp] = b.weights ? b.weights[tid] : 1.0f;
    if (b.pair_entry) b.pair_entry[pp] = tid;
    if (b.entry_pair) b.entry_pair[tid] = pp;
  } else if (tid < b.n && b.entry_pair) {
    b.entry_pair[tid] = -1;
  }
  for (int r = tid; r < b.tail; r += kPrologueThreads) {
    b.pair_row[kept + r] = r;
    if (b.pair_weight) b.pair_weight[kept + r] = 1.0f;
    if (b.pair_entry) b.pair_entry[kept + r] = -1;
  }

  // 3. chunks of <= chunk pairs: segment tid (a routed expert), then the appended shared segment
  const ChunkArgs& c = rd.chunks;
  const int cn = c.chunk;
  const int nch = tid < b.n_buckets ? (mine + cn - 1) / cn : 0;
  int routed_chunks = 0;
  int ch = cta_exclusive_scan256(nch, &routed_chunks);
  if (tid < b.n_buckets) {
    for (int q = 0; q < mine; q += cn, ++ch) {
      c.chunk_seg[ch] = tid;
      c.chunk_start[ch] = off + q;
      c.chunk_len[ch] = min(cn, mine - q);
    }
  }
  if (tid == 0) {
    int n = routed_chunks;
    if (c.n_segments > b.n_buckets) {  // the shared expert's segment
      for (int q = 0; q < b.tail; q += cn, ++n) {
        c.chunk_seg[n] = b.n_buckets;
        c.chunk_start[n] = kept + q;
        c.chunk_len[n] = min(cn, b.tail - q);
      }
    }
    *c.n_chunks = n;
  }
}

bool decode_prologue_supported(int tokens, int experts, int top_k, int hidden, int x_dtype, const void* x,
                               int n_segments) {
  const int width = x_dtype == kDtypeF32 ? 4 : 2;
  // one round of the CTA's eight warps: beyond eight tokens the 1024-thread kernel's 32 selecting warps win
  // (measured at 16 tokens: 48 against 34 us for selection, dispatch and x staging)
  return tokens >= 1 && tokens <= kPrologueThreads / kWarp && static_cast<int64_t>(tokens) * top_k <= kPrologueThreads &&
         experts <= kPrologueThreads &&
         (x_dtype == kDtypeBF16 || x_dtype == kDtypeF32) && (static_cast<int64_t>(hidden) * width) % 16 == 0 &&
         (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && n_segments <= experts + 1;
}

cudaError_t launch_decode_prologue(const DecodePrologueArgs& a, int x_dtype, cudaStream_t stream) {
  const RouteDispatchArgs& rd = a.rd;
  if (rd.nparts != 1 || !decode_prologue_supported(rd.select.tokens, rd.select.experts, rd.select.top_k, a.hidden,
                                                   x_dtype, a.x, rd.chunks.n_segments) ||
      rd.bucket.args.n != rd.select.tokens * rd.select.top_k || rd.bucket.args.n_buckets != rd.select.experts)
    return cudaErrorInvalidValue;
  const size_t smem = std::max<size_t>(static_cast<size_t>(kPrologueThreads / kWarp) * 2 * rd.select.experts,
                                       3 * kPrologueThreads) * sizeof(float);
  if (x_dtype == kDtypeBF16)
    decode_prologue_kernel<__nv_bfloat16><<<1, kPrologueThreads, smem, stream>>>(a);
  else
    decode_prologue_kernel<float><<<1, kPrologueThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- multi-CTA
// The same stable bucketing for large n in three launches: every block of
// kBucketThreads consecutive entries counts its keys; one CTA turns the
// counts into bucket offsets and per-block starting slots (bucket-major, so
// entries keep their order inside a bucket); every block then places its
// entries with the shared-memory bitmask rank of the one-CTA kernel.

__global__ void __launch_bounds__(kBucketThreads) bucket_count_kernel(BucketArgs a) {
  extern __shared__ int32_t cnt[];
  for (int b = threadIdx.x; b < a.n_buckets; b += kBucketThreads) cnt[b] = 0;
  __syncthreads();
  const int i = blockIdx.x * kBucketThreads + threadIdx.x;
  if (i < a.n) {
    const int key = a.keys[i] - a.key_lo;
    if (key >= 0 && key < a.n_buckets) atomicAdd(&cnt[key], 1);
  }
  __syncthreads();
  for (int b = threadIdx.x; b < a.n_buckets; b += kBucketThreads)
    a.block_counts[static_cast<int64_t>(blockIdx.x) * a.n_buckets + b] = cnt[b];
}

// One CTA: bucket totals -> offsets; block_counts[blk][b] -> the slot where
// block blk's first entry of bucket b goes.
__global__ void __launch_bounds__(kBucketThreads) bucket_offsets_kernel(BucketArgs a, int blocks) {
  extern __shared__ int32_t tot[];
  const int tid = threadIdx.x;
  for (int b = tid; b < a.n_buckets; b += kBucketThreads) {
    int s = 0;
    for (int blk = 0; blk < blocks; ++blk) s += a.block_counts[static_cast<int64_t>(blk) * a.n_buckets + b];
    tot[b] = s;
  }
  __syncthreads();
  const int per = static_cast<int>(ceil_div(a.n_buckets, kBucketThreads));
  const int b_lo = min(a.n_buckets, tid * per), b_hi = min(a.n_buckets, b_lo + per);
  int mine = 0;
  for (int b = b_lo; b < b_hi; ++b) mine += tot[b];
  int running = 0;
  int off = block_exclusive_scan(mine, &running);
  for (int b = b_lo; b < b_hi; ++b) {
    a.bucket_offset[b] = off;
    if (a.counts) a.counts[b] = tot[b];
    int slot = off;
    for (int blk = 0; blk < blocks; ++blk) {
      int32_t* c = a.block_counts + static_cast<int64_t>(blk) * a.n_buckets + b;
      const int n = *c;
      *c = slot;
      slot += n;
    }
    off += tot[b];
  }
  if (tid == 0) {
    a.bucket_offset[a.n_buckets] = running;
    if (a.tail > 0) a.bucket_offset[a.n_buckets + 1] = running + a.tail;
    if (a.total) *a.total = running + (a.tail > 0 ? a.tail : 0);
  }
}

__global__ void __launch_bounds__(kBucketThreads) bucket_scatter_kernel(BucketArgs a) {
  extern __shared__ uint32_t mask[];  // [n_buckets][kWindowWords]
  const int tid = threadIdx.x;
  for (int j = tid; j < a.n_buckets * kWindowWords; j += kBucketThreads) mask[j] = 0;
  __syncthreads();
  const int i = blockIdx.x * kBucketThreads + tid;
  int key = -1;
  if (i < a.n) {
    key = a.keys[i] - a.key_lo;
    if (key >= 0 && key < a.n_buckets) atomicOr(&mask[key * kWindowWords + tid / 32], 1u << (tid % 32));
    else key = -1;
  }
  __syncthreads();
  if (key >= 0) {
    const uint32_t* mk = mask + key * kWindowWords;
    int rank = __popc(mk[tid / 32] & ((1u << (tid % 32)) - 1u));
    for (int wd = 0; wd < tid / 32; ++wd) rank += __popc(mk[wd]);
    const int p = a.block_counts[static_cast<int64_t>(blockIdx.x) * a.n_buckets + key] + rank;
    a.pair_row[p] = a.rows ? a.rows[i] : i / a.k;
    if (a.pair_weight) a.pair_weight[p] = a.weights ? a.weights[i] : 1.0f;
    if (a.pair_entry) a.pair_entry[p] = i;
    if (a.entry_pair) a.entry_pair[i] = p;
  } else if (i < a.n && a.entry_pair) {
    a.entry_pair[i] = -1;
  }
}

// the appended bucket (rows 0 .. tail - 1) after the kept entries
__global__ void bucket_tail_kernel(BucketArgs a) {
  const int first = a.bucket_offset[a.n_buckets];
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < a.tail; r += gridDim.x * blockDim.x) {
    a.pair_row[first + r] = r;
    if (a.pair_weight) a.pair_weight[first + r] = 1.0f;
    if (a.pair_entry) a.pair_entry[first + r] = -1;
  }
}

int64_t bucket_scratch_ints(int64_t n, int n_buckets) { return ceil_div(n, kBucketThreads) * n_buckets; }

static cudaError_t launch_bucket_multi(const BucketArgs& a, cudaStream_t stream) {
  const int blocks = static_cast<int>(ceil_div(a.n, kBucketThreads));
  const size_t cnt_smem = static_cast<size_t>(a.n_buckets) * sizeof(int32_t);
  const size_t mask_smem = static_cast<size_t>(a.n_buckets) * kWindowWords * sizeof(uint32_t);
  cudaError_t err = cudaFuncSetAttribute(bucket_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(mask_smem));
  if (err != cudaSuccess) return err;
  bucket_count_kernel<<<blocks, kBucketThreads, cnt_smem, stream>>>(a);
  bucket_offsets_kernel<<<1, kBucketThreads, cnt_smem, stream>>>(a, blocks);
  bucket_scatter_kernel<<<blocks, kBucketThreads, mask_smem, stream>>>(a);
  if (a.tail > 0) bucket_tail_kernel<<<static_cast<unsigned>(ceil_div(a.tail, 256)), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

size_t bucket_smem_bytes(int n_buckets) {
  // the bitmask window (bucket_body) or the staged keys (bucket_body_small)
  return std::max(static_cast<size_t>(n_buckets) * kWindowWords * sizeof(uint32_t) +
                      static_cast<size_t>(2 * n_buckets + 1) * sizeof(int32_t),
                  static_cast<size_t>(kBucketThreads + n_buckets) * sizeof(int32_t));
}

cudaError_t launch_bucket(const BucketArgs& a, cudaStream_t stream) {
  const size_t smem = bucket_smem_bytes(a.n_buckets);
  if (a.n_buckets <= 0 || a.n_buckets > kMaxBuckets) return cudaErrorInvalidValue;
  if (a.block_counts && a.n > 2 * kBucketThreads) return launch_bucket_multi(a, stream);
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
