// Device-side bodies of the dispatch kernels (bucket scatter, chunk list),
// shared by dispatch.cu's kernels and its fused route + dispatch kernel.
// Both expect blockDim.x == kBucketThreads and end with the CTA synchronised.
#pragma once
#include "common.cuh"
#include "dispatch.cuh"

namespace moe {

constexpr int kBucketThreads = 1024;
constexpr int kWindowWords = kBucketThreads / 32;

// Exclusive prefix sum of one value per thread over the CTA (blockDim.x ==
// kBucketThreads, called by every thread); *total gets the CTA sum.  Ends
// with the CTA synchronised.
static __device__ int block_exclusive_scan(int v, int* total) {
  __shared__ int warp_part[kBucketThreads / 32];
  __shared__ int sum_all;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += n;
  }
  __syncthreads();  // warp_part may still be read by a previous call
  if (lane == 31) warp_part[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int mine = warp_part[lane];
    int wi = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xFFFFFFFFu, wi, o);
      if (lane >= o) wi += n;
    }
    warp_part[lane] = wi - mine;
    if (lane == 31) sum_all = wi;
  }
  __syncthreads();
  if (total) *total = sum_all;
  return warp_part[warp] + incl - v;
}

// One CTA.  Entry i has key keys[i] (entries whose key falls outside
// [key_lo, key_lo + n_buckets) are dropped), row rows ? rows[i] : i / k and
// weight weights ? weights[i] : 1.
static __device__ void bucket_body(const BucketArgs& a, uint32_t* sm) {
  uint32_t* mask = sm;                                  // [n_buckets][32]
  int32_t* count = reinterpret_cast<int32_t*>(mask + a.n_buckets * kWindowWords);  // [n_buckets]
  int32_t* base = count + a.n_buckets;                 // [n_buckets + 1]
  const int tid = threadIdx.x;

  for (int b = tid; b < a.n_buckets; b += kBucketThreads) count[b] = 0;
  __syncthreads();
  for (int i = tid; i < a.n; i += kBucketThreads) {
    const int key = a.keys[i] - a.key_lo;
    if (key >= 0 && key < a.n_buckets) atomicAdd(&count[key], 1);
  }
  __syncthreads();
  {
    // bucket offsets: thread tid owns buckets [tid * per, tid * per + per)
    const int per = static_cast<int>(ceil_div(a.n_buckets, kBucketThreads));
    const int b_lo = min(a.n_buckets, tid * per), b_hi = min(a.n_buckets, b_lo + per);
    int mine = 0;
    for (int b = b_lo; b < b_hi; ++b) mine += count[b];
    int running = 0;
    int off = block_exclusive_scan(mine, &running);
    for (int b = b_lo; b < b_hi; ++b) {
      base[b] = off;
      a.bucket_offset[b] = off;
      off += count[b];
    }
    if (tid == 0) {
      base[a.n_buckets] = running;
      a.bucket_offset[a.n_buckets] = running;
      if (a.tail > 0) a.bucket_offset[a.n_buckets + 1] = running + a.tail;
      if (a.total) *a.total = running + (a.tail > 0 ? a.tail : 0);
    }
  }
  if (a.counts)
    for (int b = tid; b < a.n_buckets; b += kBucketThreads) a.counts[b] = count[b];
  __syncthreads();
  // base[b] now advances window by window: offset of the next free slot.
  for (int w0 = 0; w0 < a.n; w0 += kBucketThreads) {
    for (int j = tid; j < a.n_buckets * kWindowWords; j += kBucketThreads) mask[j] = 0;
    __syncthreads();
    const int i = w0 + tid;
    int key = -1;
    if (i < a.n) {
      key = a.keys[i] - a.key_lo;
      if (key >= 0 && key < a.n_buckets) {
        atomicOr(&mask[key * kWindowWords + tid / 32], 1u << (tid % 32));
      } else {
        key = -1;
      }
    }
    __syncthreads();
    if (key >= 0) {
      const uint32_t* m = mask + key * kWindowWords;
      int rank = __popc(m[tid / 32] & ((1u << (tid % 32)) - 1u));
      for (int wd = 0; wd < tid / 32; ++wd) rank += __popc(m[wd]);
      const int p = base[key] + rank;
      a.pair_row[p] = a.rows ? a.rows[i] : i / a.k;
      if (a.pair_weight) a.pair_weight[p] = a.weights ? a.weights[i] : 1.0f;
      if (a.pair_entry) a.pair_entry[p] = i;
      if (a.entry_pair) a.entry_pair[i] = p;
    } else if (i < a.n && a.entry_pair) {
      a.entry_pair[i] = -1;
    }
    __syncthreads();
    for (int b = tid; b < a.n_buckets; b += kBucketThreads) {
      int c = 0;
      for (int wd = 0; wd < kWindowWords; ++wd) c += __popc(mask[b * kWindowWords + wd]);
      base[b] += c;
    }
    __syncthreads();
  }
  if (a.tail > 0) {
    const int first = base[a.n_buckets];  // == number of kept entries
    for (int r = tid; r < a.tail; r += kBucketThreads) {
      a.pair_row[first + r] = r;
      if (a.pair_weight) a.pair_weight[first + r] = 1.0f;
      if (a.pair_entry) a.pair_entry[first + r] = -1;
    }
  }
}

// bucket_body for at most kBucketThreads entries (decode batches): thread i
// owns entry i; its rank inside its bucket is the number of earlier entries
// with the same key (keys staged in shared memory, four per load) -- no
// per-bucket bitmask window to clear and count.  Same outputs as bucket_body.
static __device__ void bucket_body_small(const BucketArgs& a, uint32_t* sm) {
  int32_t* keys_s = reinterpret_cast<int32_t*>(sm);  // [kBucketThreads]
  int32_t* start = keys_s + kBucketThreads;         // [n_buckets]: counts, then first slots
  const int tid = threadIdx.x;
  for (int b = tid; b < a.n_buckets; b += kBucketThreads) start[b] = 0;
  int key = -1;
  if (tid < a.n) {
    key = a.keys[tid] - a.key_lo;
    if (key < 0 || key >= a.n_buckets) key = -1;
  }
  keys_s[tid] = key;
  __syncthreads();
  if (key >= 0) atomicAdd(&start[key], 1);
  __syncthreads();
  {
    const int per = static_cast<int>(ceil_div(a.n_buckets, kBucketThreads));
    const int b_lo = min(a.n_buckets, tid * per), b_hi = min(a.n_buckets, b_lo + per);
    int mine = 0;
    for (int b = b_lo; b < b_hi; ++b) mine += start[b];
    int running = 0;
    int off = block_exclusive_scan(mine, &running);
    for (int b = b_lo; b < b_hi; ++b) {
      const int c = start[b];
      if (a.counts) a.counts[b] = c;
      a.bucket_offset[b] = off;
      start[b] = off;
      off += c;
    }
    if (tid == 0) {
      a.bucket_offset[a.n_buckets] = running;
      if (a.tail > 0) a.bucket_offset[a.n_buckets + 1] = running + a.tail;
      if (a.total) *a.total = running + (a.tail > 0 ? a.tail : 0);
    }
  }
  __syncthreads();
  if (key >= 0) {
    int rank = 0;
    const int4* k4 = reinterpret_cast<const int4*>(keys_s);
    for (int j = 0; j < tid / 4; ++j) {
      const int4 q = k4[j];
      rank += (q.x == key) + (q.y == key) + (q.z == key) + (q.w == key);
    }
    for (int j = tid & ~3; j < tid; ++j) rank += keys_s[j] == key;
    const int p = start[key] + rank;
    a.pair_row[p] = a.rows ? a.rows[tid] : tid / a.k;
    if (a.pair_weight) a.pair_weight[p] = a.weights ? a.weights[tid] : 1.0f;
    if (a.pair_entry) a.pair_entry[p] = tid;
    if (a.entry_pair) a.entry_pair[tid] = p;
  } else if (tid < a.n && a.entry_pair) {
    a.entry_pair[tid] = -1;
  }
  if (a.tail > 0) {
    const int first = a.bucket_offset[a.n_buckets];
    for (int r = tid; r < a.tail; r += kBucketThreads) {
      a.pair_row[first + r] = r;
      if (a.pair_weight) a.pair_weight[first + r] = 1.0f;
      if (a.pair_entry) a.pair_entry[first + r] = -1;
    }
  }
  __syncthreads();
}

// One CTA: segments -> chunks of at most `chunk` consecutive pairs.
static __device__ void chunk_body(const ChunkArgs& a) {
  const int tid = threadIdx.x;
  const int per = static_cast<int>(ceil_div(a.n_segments, kBucketThreads));
  const int s_lo = tid * per, s_hi = min(a.n_segments, s_lo + per);
  int mine = 0;
  for (int s = s_lo; s < s_hi; ++s) {
    const int n = a.seg_offset[s + 1] - a.seg_offset[s];
    mine += (n + a.chunk - 1) / a.chunk;
  }
  int total = 0;
  int c = block_exclusive_scan(mine, &total);
  if (tid == 0) *a.n_chunks = total;
  for (int s = s_lo; s < s_hi; ++s) {
    const int lo = a.seg_offset[s], hi = a.seg_offset[s + 1];
    for (int p = lo; p < hi; p += a.chunk, ++c) {
      a.chunk_seg[c] = s;
      a.chunk_start[c] = p;
      a.chunk_len[c] = min(a.chunk, hi - p);
    }
  }
}

}  // namespace moe
