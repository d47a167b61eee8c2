// extern "C" entry points of libmoe_b200.so (declared in include/moe_b200.h).
//
// Each function validates its arguments the way the reference C function it
// replaces does (same return codes for null pointers and bad dimensions),
// plans its scratch memory, and enqueues the kernels on the caller's stream.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/moe_b200.h"
#include "async_copy.cuh"
#include "common.cuh"
#include "dequant.cuh"
#include "dispatch.cuh"
#include "fp8_gemv.cuh"
#include "mla.cuh"
#include "plan.cuh"
#include "prefill_gemm.cuh"
#include "route_host.cuh"
#include "router.cuh"
#include "router_device.cuh"
#include "status.cuh"

using namespace moe;

namespace {

// Error word of the expert-parallel peer kernels (moe_b200_device_error code
// 64): a destination rank, receive slot or return row read from exchanged
// data that lies outside the buffers it indexes.  The access is skipped.
constexpr int kEpRangeError = 64;
// ... and code 256: a wait of the peer-memory barrier (moe_ep_barrier_p2p) ran out.
constexpr int kEpWaitError = 256;
__device__ int g_ep_error = 0;

int read_and_clear_ep_error(cudaStream_t stream) {
  int host = 0;
  if (cudaMemcpyFromSymbolAsync(&host, g_ep_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return -1;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return -1;
  if (host) {
    const int zero = 0;
    if (cudaMemcpyToSymbolAsync(g_ep_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream) != cudaSuccess ||
        cudaStreamSynchronize(stream) != cudaSuccess)
      return -1;
  }
  return host;
}

// Optional stage timing of the fused layer (moe_b200_stage_timing): CUDA events
// recorded on the launching stream between the layer's kernels.
constexpr int kMaxStageEvents = 8;
bool g_timing = false;
cudaEvent_t g_events[kMaxStageEvents] = {};
int g_marks = 0;

// Expert GEMV selection: 0 = auto (warp-MMA kernel on the layer path where the
// shapes allow, direct-load elsewhere), 1 = bulk-copy streaming kernel where
// supported, 2 = direct-load kernel everywhere.
int g_gemv_impl = 0;
// Operand feed of the warp-MMA kernel: 0 = register loads, 1 = TMA bulk-copy
// ring per warp, 2 = cp.async shared-memory ring per warp (default).
int g_mma_feed = 2;
// Decode experts on the cp.async feed as one fused launch (decode_fused_kernel:
// gate/up, activation staging and down) rather than three launches (off by
// default: measured slower than the three launches at 1-64 tokens).
bool g_fused_decode = false;
// K-split of the cp.async warp-MMA stages: 0 = chosen per batch (async_gemv_ksplit), else this many
// k-ranges per task (capped at kMaxMmaKSplit); sizes the workspace too, so it must not change between
// a workspace query and the call it sizes.
int g_force_ksplit = 0;
// Decode batches of <= 256 (token, slot) entries: selection, dispatch, chunk list and x staging in one
// CTA (decode_prologue_kernel) instead of route_dispatch_kernel + rows_to_f16_kernel.
bool g_decode_prologue = true;
// With the decode prologue and bf16 hidden states: the router logits launch stages x (f16 + row scale) in an
// extra cluster that runs beside the logits clusters, instead of the prologue's one warp per token.
bool g_router_stages_x = true;
// Staggered k-block walks in the cp.async warp-MMA stages (MmaArgs::kb_rotate).
int g_kb_rotate = 0;
// cp.async decode stages: the activation staging folded into the gate/up GEMV and the combine into the
// down GEMV (their last-arriving warps), instead of two launches.  Off by default: measured slower from
// 4 tokens on (a fence and an arrival after every task; 64 tokens: 1.86 against 1.59 ms).
bool g_fold_epilogues = false;
// Decode layers (warp-MMA experts, tiled weights): the shared expert -- which needs no routing -- runs on
// a side stream while the router and the dispatch run, on part of the GPU, instead of with the routed
// experts.  Off by default: at one token the routed stages got 6 us faster but the router and dispatch,
// sharing the SMs with the side launches, 11 us slower; the shared expert's own k-split also makes the
// output differ from the one-stream layer in the last bf16 bit.
bool g_shared_side = false;
// CTAs per SM the side stream's expert launches may take (the router's clusters and the dispatch CTA
// keep the rest).
constexpr int kSharedSideCtasPerSm = 2;

cudaError_t gemv(const GemvArgs& a, int x_dtype, int ns, int epi, int nt, bool vec, cudaStream_t stream) {
  if (g_gemv_impl == 1 && vec && stream_gemv_supported(a.K, x_dtype, nt))
    return launch_stream_gemv(a, x_dtype, ns, epi, nt, stream);
  return launch_grouped_gemv(a, x_dtype, ns, epi, nt, vec, stream);
}

void stage_mark(cudaStream_t stream) {
  if (!g_timing || g_marks >= kMaxStageEvents) return;
  cudaEventRecord(g_events[g_marks++], stream);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Scratch of the grouped FP8 MLP: pairs, chunk list, activations and outputs.
struct MlpScratch {
  int32_t* seg_offset;
  int32_t* pair_row;
  float* pair_weight;
  int32_t* pair_entry;
  int32_t* entry_pair;
  int32_t* chunk_seg;
  int32_t* chunk_start;
  int32_t* chunk_len;
  int32_t* n_chunks;
  int32_t* keys;
  int32_t* entry_row;
  float* entry_weight;
  float* act;
  float* y;
};

MlpScratch plan_mlp(Plan& plan, int64_t pairs, int64_t segments, int64_t entries, int64_t inter,
                    int64_t hidden, int nt, bool need_y) {
  MlpScratch s{};
  s.seg_offset = plan.take<int32_t>(segments + 2);
  s.pair_row = plan.take<int32_t>(pairs);
  s.pair_weight = plan.take<float>(pairs);
  s.pair_entry = plan.take<int32_t>(pairs);
  s.entry_pair = plan.take<int32_t>(entries);
  const int64_t cap = chunk_capacity(pairs, segments + 1, nt);
  s.chunk_seg = plan.take<int32_t>(cap);
  s.chunk_start = plan.take<int32_t>(cap);
  s.chunk_len = plan.take<int32_t>(cap);
  s.n_chunks = plan.take<int32_t>(1);
  s.keys = plan.take<int32_t>(entries);
  s.entry_row = plan.take<int32_t>(entries);
  s.entry_weight = plan.take<float>(entries);
  s.act = plan.take<float>(pairs * inter);
  s.y = need_y ? plan.take<float>(pairs * hidden) : nullptr;
  return s;
}

struct Tables {
  const uint64_t *gw, *gs, *uw, *us, *dw, *ds;
};

// gate/up + SwiGLU then down for every pair: act -> y (fp32 [P, H]).
int run_expert_stages(const Tables& t, const void* x, int x_dtype, const MlpScratch& s, float* y,
                      int64_t n_segments, int64_t inter, int64_t hidden, int64_t gsc, int64_t dsc, int nt,
                      bool vec, cudaStream_t stream) {
  ChunkArgs ca{s.seg_offset, static_cast<int>(n_segments), nt, s.chunk_seg, s.chunk_start, s.chunk_len, s.n_chunks};
  MOE_CUDA(launch_chunks(ca, stream), "chunk list");
  GemvArgs g1{};
  g1.w0 = t.gw; g1.s0 = t.gs; g1.w1 = t.uw; g1.s1 = t.us;
  g1.x = x; g1.pair_row = s.pair_row;
  g1.chunk_seg = s.chunk_seg; g1.chunk_start = s.chunk_start; g1.chunk_len = s.chunk_len; g1.n_chunks = s.n_chunks;
  g1.out0 = s.act; g1.N = static_cast<int>(inter); g1.K = static_cast<int>(hidden); g1.scale_cols = static_cast<int>(gsc);
  stage_mark(stream);
  MOE_CUDA(gemv(g1, x_dtype, 2, kEpiSwiglu, nt, vec, stream), "gate/up stage");
  stage_mark(stream);
  const int nt2 = std::min(nt, gemv_chunk_tokens(static_cast<int>(inter), kXF32));
  if (nt2 != nt) {
    // the down stage walks the same chunks; it needs the same chunk size
    return fail(kUnsupported, "intermediate size too large for the staged down projection");
  }
  GemvArgs g2 = g1;
  g2.w0 = t.dw; g2.s0 = t.ds; g2.w1 = nullptr; g2.s1 = nullptr;
  g2.x = s.act; g2.pair_row = nullptr; g2.out0 = y;
  g2.N = static_cast<int>(hidden); g2.K = static_cast<int>(inter); g2.scale_cols = static_cast<int>(dsc);
  const bool vec2 = vec && (inter % 16 == 0);
  MOE_CUDA(gemv(g2, kXF32, 1, kEpiStore, nt, vec2, stream), "down stage");
  stage_mark(stream);
  return kOk;
}

int pick_nt(int64_t max_rows_per_segment, int64_t K1, int64_t K2, int x_dtype) {
  int cap = std::min(gemv_chunk_tokens(static_cast<int>(K1), x_dtype), gemv_chunk_tokens(static_cast<int>(K2), kXF32));
  if (cap <= 0) return 0;
  int nt = max_rows_per_segment <= 1 ? 1 : (max_rows_per_segment <= 4 ? 4 : 8);
  while (nt > cap) nt = nt == 8 ? 4 : 1;
  return nt;
}

// Entries of the many / weighted / row-weighted calls: entry i = (item i / B,
// row i % B).  mode 0: weight 1; mode 1: route[item]; mode 2: route[i], and a
// zero weight drops the entry (the reference skips that work, fp8_linear.cpp:753-755).
__global__ void fill_entries_kernel(int32_t* keys, int32_t* rows, float* weights, int64_t n, int64_t B, int mode,
                                    const float* route) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t item = i / B;
    float w = 1.0f;
    if (mode == 1) w = route[item];
    if (mode == 2) w = route[i];
    keys[i] = (mode == 2 && w == 0.0f) ? -1 : static_cast<int32_t>(item);
    rows[i] = static_cast<int32_t>(i % B);
    weights[i] = w;
  }
}

// entry_pair [E, B] (item-major) -> row_pairs [B, E]
__global__ void transpose_entries_kernel(const int32_t* entry_pair, int32_t* row_pairs, int64_t E, int64_t B) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < E * B;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = i / B, b = i % B;
    row_pairs[b * E + e] = entry_pair[i];
  }
}

// pair index of each listed entry (in place allowed)
__global__ void map_entries_kernel(const int32_t* entries, const int32_t* entry_pair, int32_t* out, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t e = entries[i];
    out[i] = e >= 0 ? entry_pair[e] : -1;
  }
}

__global__ void i64_to_i32_kernel(const int64_t* in, int32_t* out, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = static_cast<int32_t>(in[i]);
}

__global__ void validate_pairs_kernel(const int64_t* item, const int64_t* row, int64_t n, int64_t items,
                                      int64_t rows, int32_t* bad) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    if (item[i] < 0 || item[i] >= items || row[i] < 0 || row[i] >= rows) atomicExch(bad, 1);
}

// Shared body of the many / weighted / row-weighted MLP entry points.
// Entry i = (item i / batch, row i % batch) in item-major order; every row's
// combine then walks its entries in item order, as the reference sums them.
int mlp_items(const Tables& t, const float* hidden, const float* route, int route_mode, float* out,
              bool per_expert_out, int64_t E, int64_t B, int64_t I, int64_t H, int64_t gsc, int64_t dsc,
              void* workspace, int64_t ws_bytes, cudaStream_t stream) {
  const int64_t entries = E * B;
  const int nt = pick_nt(B, H, I, kXF32);
  if (nt == 0) return fail(kUnsupported, "hidden/intermediate size too large for the staged GEMV");
  Plan sizing;
  plan_mlp(sizing, entries, E, entries, I, H, nt, !per_expert_out);
  Scratch scratch(workspace, ws_bytes, sizing.used(), stream);
  if (!scratch.ok()) return fail(kNoMemory, "workspace too small or allocation failed");
  Plan plan(scratch.base());
  MlpScratch s = plan_mlp(plan, entries, E, entries, I, H, nt, !per_expert_out);
  fill_entries_kernel<<<grid_for(entries), 256, 0, stream>>>(s.keys, s.entry_row, s.entry_weight, entries, B,
                                                               route ? (route_mode == 1 ? 2 : 1) : 0, route);
  MOE_CUDA(cudaGetLastError(), "entries");
  BucketArgs ba{};
  ba.keys = s.keys; ba.rows = s.entry_row; ba.weights = s.entry_weight;
  ba.n = static_cast<int>(entries); ba.k = 1; ba.key_lo = 0; ba.n_buckets = static_cast<int>(E);
  ba.bucket_offset = s.seg_offset; ba.pair_row = s.pair_row; ba.pair_weight = s.pair_weight;
  ba.pair_entry = s.pair_entry; ba.entry_pair = s.entry_pair;
  MOE_CUDA(launch_bucket(ba, stream), "bucket");
  const bool vec = H % 16 == 0 && I % 16 == 0 && aligned16(hidden);
  float* y = per_expert_out ? out : s.y;
  int code = run_expert_stages(t, hidden, kXF32, s, y, E, I, H, gsc, dsc, nt, vec, stream);
  if (code != kOk) return code;
  if (!per_expert_out) {
    // row b's entries are e * B + b for e in item order: stride-1 lists via row_ptr = null,
    // built as a transposed view of entry_pair
    CombineArgs c{};
    c.y = s.y;
    c.row_ptr = nullptr;
    c.stride = static_cast<int>(E);
    int32_t* row_pairs = s.keys;  // reuse: [B, E]
    transpose_entries_kernel<<<grid_for(entries), 256, 0, stream>>>(s.entry_pair, row_pairs, E, B);
    MOE_CUDA(cudaGetLastError(), "row lists");
    c.row_pairs = row_pairs;
    c.pair_weight = s.pair_weight;
    c.extra_base = -1;
    c.T = static_cast<int>(B);
    c.H = static_cast<int>(H);
    c.out_f32 = out;
    MOE_CUDA(launch_combine(c, stream), "combine");
  }
  return kOk;
}

}  // namespace

int moe::route_impl(const void* hidden, int hd, const void* w, int wd, const float* bias, int64_t T, int64_t H,
                      int64_t E, int64_t n_group, int64_t topk_group, int64_t k, int scoring, int renorm,
                      int fp64, float scale, int round_bf16, int64_t* ids64, int32_t* ids32, float* wf32,
                      uint16_t* wbf16, float* logits, cudaStream_t stream) {
  // prefill-sized batches on the tensor cores (split-K partials, summed in
  // part order by the selection); otherwise the fp32 GEMV / tiled kernels
  int nparts = 1;
  cudaError_t cerr = cudaErrorNotSupported;
  if (T <= 256) {
    // decode-sized batches: one cluster-reduced tensor-core pass when the operands allow it
    cerr = launch_router_logits_cluster(hidden, hd, w, wd, logits, static_cast<int>(T), static_cast<int>(H),
                                        static_cast<int>(E), stream);
    if (cerr != cudaErrorNotSupported) MOE_CUDA(cerr, "router logits");
  }
  if (T > 256) {
    // prefill-sized batches: the tcgen05 GEMM when both operands are 16-bit of one type
    cerr = launch_router_logits_tc(hidden, hd, w, wd, logits, T, H, E, &nparts, stream);
    if (cerr != cudaErrorNotSupported) MOE_CUDA(cerr, "router logits");
  }
  if (cerr != cudaErrorNotSupported) {
    // done
  } else if (T > 256 && router_split_is_mma(hidden, hd, w, wd, static_cast<int>(H))) {
    MOE_CUDA(launch_router_logits_split(hidden, hd, w, wd, logits, static_cast<int>(T), static_cast<int>(H),
                                        static_cast<int>(E), stream),
             "router logits");
    nparts = router_split_parts(static_cast<int>(H));
  } else {
    MOE_CUDA(launch_router_logits(hidden, hd, w, wd, logits, static_cast<int>(T), static_cast<int>(H),
                                  static_cast<int>(E), stream),
             "router logits");
  }
  RouterSelectParams p{};
  p.tokens = static_cast<int>(T);
  p.experts = static_cast<int>(E);
  p.top_k = static_cast<int>(k);
  p.n_group = static_cast<int>(n_group);
  p.topk_group = static_cast<int>(topk_group);
  p.scoring = scoring;
  p.renorm = renorm || scoring == kScoreSigmoid;
  p.softmax_fp64 = fp64;
  p.round_bf16 = round_bf16;
  p.route_scale = scale;
  MOE_CUDA(launch_router_select(logits, bias, p, ids64, ids32, wf32, reinterpret_cast<__nv_bfloat16*>(wbf16),
                                stream, nparts, T * E),
           "router select");
  return kOk;
}

int moe::check_route(int64_t T, int64_t H, int64_t E, int64_t n_group, int64_t topk_group, int64_t k) {
  if (T <= 0 || H <= 0 || E <= 0 || k <= 0 || k > E) return fail(kBadDims, "bad dimensions");
  if (k > 32) return fail(kUnsupported, "top_k > 32");
  if (E > 2048) return fail(kUnsupported, "more than 2048 experts");
  if (n_group < 1 || n_group > 32 || E % n_group != 0) return fail(kBadDims, "n_group must divide num_experts (<= 32)");
  if (topk_group < 1) return fail(kBadDims, "topk_group < 1");
  return kOk;
}

// Destination rank of each (token, slot) entry under a contiguous expert
// partition: rank = expert / experts_per_rank.
__global__ void ep_rank_keys_kernel(const int64_t* ids, int64_t n, int64_t per_rank, int64_t world, int32_t* keys) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = ids[i] / per_rank;
    keys[i] = (ids[i] >= 0 && r < world) ? static_cast<int32_t>(r) : -1;
  }
}

// send_rows[p] = hidden[pos_token[p]], send_expert[p] = expert id local to its rank; one warp per row.
__global__ void ep_gather_kernel(const uint16_t* hidden, const int64_t* ids, const int32_t* keys,
                                 const int32_t* pos_token, const int32_t* pos_entry, int64_t n, int64_t H,
                                 int64_t per_rank, int64_t vec, uint16_t* send_rows, int32_t* send_expert) {
  const int lane = threadIdx.x % 32;
  for (int64_t p = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) / 32; p < n;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x / 32) {
    const int32_t e = pos_entry[p];
    if (e < 0) continue;
    const uint16_t* src = hidden + static_cast<int64_t>(pos_token[p]) * H;
    uint16_t* dst = send_rows + p * H;
    if (vec) {
      for (int64_t i = lane; i < H / 8; i += 32)
        reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
    } else {
      for (int64_t i = lane; i < H; i += 32) dst[i] = src[i];
    }
    if (lane == 0) send_expert[p] = static_cast<int32_t>(ids[e] - keys[e] * per_rank);
  }
}

// Expert-parallel exchange over NVLink peer memory.  Per-destination-rank
// entry counts of this rank's (token, slot) entries.
__global__ void ep_count_kernel(const int64_t* ids, int64_t n, int64_t per_rank, int world, int32_t* counts) {
  extern __shared__ int32_t c[];
  for (int r = threadIdx.x; r < world; r += blockDim.x) c[r] = 0;
  __syncthreads();
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const int64_t r = ids[i] / per_rank;
    if (ids[i] >= 0 && r < world) atomicAdd(&c[r], 1);
  }
  __syncthreads();
  for (int r = threadIdx.x; r < world; r += blockDim.x) counts[r] = c[r];
}

// Barrier of the expert-parallel ranks over peer memory.  Each rank's signal
// buffer holds one 32-bit slot per rank: the last barrier epoch that rank
// reached (epochs only grow, so one slot per rank serves every barrier).
// One CTA; thread r < world serves peer r: (optionally) this rank's payload
// row into row `rank` of peer r's payload buffer, a system-scope fence (every
// store this rank made to peer memory before, this launch's and earlier
// launches', is visible first), this rank's epoch into peer r's slot [rank]
// (release), then a wait for peer r's epoch in this rank's slot [r]
// (acquire), for at most limit_ns of %globaltimer.  A wait that runs out sets
// code 256 and gives up; while that code is set, barriers do not wait (the
// host reads it with moe_b200_device_error).
MOE_D void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
MOE_D uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__global__ void ep_barrier_kernel(const uint64_t* peer_sig, int world, int rank, uint32_t* epoch, int64_t limit_ns,
                                  const int32_t* payload, int payload_n, const uint64_t* peer_payload) {
  __shared__ uint32_t e_s;
  if (threadIdx.x == 0) e_s = *epoch + 1u;
  __syncthreads();
  const uint32_t e = e_s;
  const int r = threadIdx.x;
  if (r < world) {
    if (payload) {
      int32_t* dst = reinterpret_cast<int32_t*>(peer_payload[r]) + static_cast<int64_t>(rank) * payload_n;
      for (int i = 0; i < payload_n; ++i) dst[i] = payload[i];
    }
    __threadfence_system();
    st_release_sys_u32(reinterpret_cast<uint32_t*>(peer_sig[r]) + rank, e);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(peer_sig[rank]) + r;
    const bool skip = (*reinterpret_cast<volatile int*>(&g_ep_error) & kEpWaitError) != 0;
    const uint64_t start = global_timer_ns();
    while (!skip && static_cast<int32_t>(ld_acquire_sys_u32(mine) - e) < 0) {
      if (global_timer_ns() - start > static_cast<uint64_t>(limit_ns)) {
        atomicOr(&g_ep_error, kEpWaitError);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *epoch = e;
}

// The wait half of a barrier for thread r < world: rank r's epoch >= e in this rank's slot [r].
MOE_D void ep_wait_peer(const uint64_t* peer_sig, int rank, int r, uint32_t e, int64_t limit_ns) {
  const uint32_t* mine = reinterpret_cast<const uint32_t*>(peer_sig[rank]) + r;
  if (*reinterpret_cast<volatile int*>(&g_ep_error) & kEpWaitError) return;
  const uint64_t start = global_timer_ns();
  while (static_cast<int32_t>(ld_acquire_sys_u32(mine) - e) < 0) {
    if (global_timer_ns() - start > static_cast<uint64_t>(limit_ns)) {
      atomicOr(&g_ep_error, kEpWaitError);
      return;
    }
    __nanosleep(64);
  }
}
MOE_D int32_t ld_relaxed_sys_s32(const int32_t* p) {
  int32_t v;
  asm volatile("ld.relaxed.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// The send side of one decode step of the peer exchange in one CTA, in
// place of the selection, rank count, receive-slot reset, counts all-gather,
// rank bucketing, row scatter and the two barriers around it (eleven
// launches): (1) warp t selects token t's experts from the router logits
// (select_token, as the router's selection kernel does); (2) this rank's
// receive slots are reset (expert -1) and its own tokens' shared-expert rows
// written after them (rows C + t, expert n_local, source entry T * top_k +
// t); (3) each entry's destination rank and its position among this rank's
// entries bound there, in entry order (a bitmask per rank); (4) barrier 1,
// carrying this rank's counts row into every peer's counts matrix; (5) every
// entry's receive slot = the entries of lower ranks bound for the same rank
// + its position, range-checked (code 64); warps write each token row and
// its expert and source codes into the destination's buffers with 16-byte
// NVLink stores; (6) a system fence, barrier 2.  Barriers as
// ep_barrier_kernel (the epoch grows by two).  Up to 128 tokens, 1024
// entries, 256 experts, 32 ranks; 1024 threads.
constexpr int kEpSendThreads = 1024;
constexpr int kEpSendWarps = kEpSendThreads / 32;
constexpr int kEpSendMaxRanks = 32;
struct EpSendArgs {
  const float* logits;   // [T, E]
  const float* bias;
  RouterSelectParams sel;
  const uint16_t* x;     // [T, H] bf16
  int64_t H;
  int world, rank, n_local;
  int64_t capacity, src_stride;
  const uint64_t* peer_rows;
  const uint64_t* peer_expert;
  const uint64_t* peer_src;
  const uint64_t* peer_matrix;
  const uint64_t* peer_sig;
  uint32_t* epoch;
  int64_t limit_ns;
  int64_t* ids64;
  float* weights_f32;
};
__global__ void __launch_bounds__(kEpSendThreads) ep_send_decode_kernel(EpSendArgs a) {
  extern __shared__ float sel_scratch[];  // [warps][2 * E]
  __shared__ uint32_t masks[kEpSendMaxRanks][kEpSendThreads / 32];
  __shared__ int32_t counts[kEpSendMaxRanks], base[kEpSendMaxRanks];
  __shared__ int32_t keys[kEpSendThreads], posv[kEpSendThreads];
  __shared__ uint32_t e_s;
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  const int T = a.sel.tokens, k = a.sel.top_k, E = a.sel.experts, n = T * k, W = a.world;
  const int64_t H = a.H, C = a.capacity;
  if (tid == 0) e_s = *a.epoch;
  // 1. selection
  for (int t = warp; t < T; t += kEpSendWarps)
    select_token(a.logits, 1, 0, a.bias, a.sel, t, sel_scratch + warp * 2 * E, sel_scratch + warp * 2 * E + E,
                 a.ids64, nullptr, a.weights_f32, nullptr);
  // 2. this rank's receive slots; its own shared-expert rows after them
  int32_t* own_expert = reinterpret_cast<int32_t*>(a.peer_expert[a.rank]);
  int32_t* own_src = reinterpret_cast<int32_t*>(a.peer_src[a.rank]);
  uint16_t* own_rows = reinterpret_cast<uint16_t*>(a.peer_rows[a.rank]);
  for (int64_t i = tid; i < C; i += kEpSendThreads) own_expert[i] = -1;
  for (int t = warp; t < T; t += kEpSendWarps) {
    const uint4* src = reinterpret_cast<const uint4*>(a.x + static_cast<int64_t>(t) * H);
    uint4* dst = reinterpret_cast<uint4*>(own_rows + (C + t) * H);
    for (int64_t i = lane; i < H / 8; i += kWarp) dst[i] = __ldg(src + i);
    if (lane == 0) {
      own_expert[C + t] = a.n_local;
      own_src[C + t] = static_cast<int32_t>(a.rank * a.src_stride + n + t);
    }
  }
  for (int i = tid; i < kEpSendMaxRanks * (kEpSendThreads / 32); i += kEpSendThreads) (&masks[0][0])[i] = 0;
  if (tid < kEpSendMaxRanks) counts[tid] = 0;
  __syncthreads();  // the selections (global) and the cleared masks are visible to the CTA
  // 3. destinations and positions
  int key = -1;
  if (tid < n) {
    const int64_t id = a.ids64[tid];
    const int64_t q = id / a.n_local;
    key = (id >= 0 && q < W) ? static_cast<int>(q) : -1;
    if (key < 0) atomicOr(&g_ep_error, kEpRangeError);
  }
  keys[tid] = key;
  if (key >= 0) {
    atomicOr(&masks[key][tid / 32], 1u << (tid % 32));
    atomicAdd(&counts[key], 1);
  }
  __syncthreads();
  if (key >= 0) {
    int pos = __popc(masks[key][tid / 32] & ((1u << (tid % 32)) - 1u));
    for (int w = 0; w < tid / 32; ++w) pos += __popc(masks[key][w]);
    posv[tid] = pos;
  }
  // 4. barrier 1 with this rank's counts row
  const uint32_t e1 = e_s + 1u, e2 = e_s + 2u;
  if (tid < W) {
    int32_t* dst = reinterpret_cast<int32_t*>(a.peer_matrix[tid]) + static_cast<int64_t>(a.rank) * W;
    for (int q = 0; q < W; ++q) dst[q] = counts[q];
    __threadfence_system();  // the reset slots, the own rows and the counts are visible before the signal
    st_release_sys_u32(reinterpret_cast<uint32_t*>(a.peer_sig[tid]) + a.rank, e1);
    ep_wait_peer(a.peer_sig, a.rank, tid, e1, a.limit_ns);
  }
  __syncthreads();
  // 5. receive slots, then the rows
  if (tid < W) {
    const int32_t* m = reinterpret_cast<const int32_t*>(a.peer_matrix[a.rank]);
    int b = 0;
    for (int r = 0; r < a.rank; ++r) b += ld_relaxed_sys_s32(m + static_cast<int64_t>(r) * W + tid);
    base[tid] = b;
  }
  __syncthreads();
  for (int e = warp; e < n; e += kEpSendWarps) {
    const int q = keys[e];
    if (q < 0) continue;
    const int64_t slot = static_cast<int64_t>(base[q]) + posv[e];
    if (slot < 0 || slot >= C) {  // counts that disagree with the rows sent: recorded, never stored
      if (lane == 0) atomicOr(&g_ep_error, kEpRangeError);
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(a.x + static_cast<int64_t>(e / k) * H);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(a.peer_rows[q]) + slot * H);
    for (int64_t i = lane; i < H / 8; i += kWarp) dst[i] = __ldg(src + i);
    if (lane == 0) {
      reinterpret_cast<int32_t*>(a.peer_expert[q])[slot] =
          static_cast<int32_t>(a.ids64[e] - static_cast<int64_t>(q) * a.n_local);
      reinterpret_cast<int32_t*>(a.peer_src[q])[slot] = static_cast<int32_t>(a.rank * a.src_stride + e);
    }
  }
  __threadfence_system();
  __syncthreads();
  // 6. barrier 2: every rank's rows have landed
  if (tid < W) {
    st_release_sys_u32(reinterpret_cast<uint32_t*>(a.peer_sig[tid]) + a.rank, e2);
    ep_wait_peer(a.peer_sig, a.rank, tid, e2, a.limit_ns);
  }
  __syncthreads();
  if (tid == 0) *a.epoch = e2;
}

// Rows to their experts' ranks: send position p (grouped by destination q,
// token order inside) goes to row O(q) + p - send_offset[q] of rank q's
// receive buffers, O(q) = the entries of ranks before this one bound for q
// (count_matrix [world][world], row = source rank).  One warp per entry;
// 16-byte stores straight into the peer's memory.
__global__ void ep_p2p_scatter_kernel(const uint16_t* hidden, const int64_t* ids, const int32_t* keys,
                                      const int32_t* pos_token, const int32_t* pos_entry, const int32_t* send_offset,
                                      const int32_t* count_matrix, int64_t n, int64_t H, int64_t per_rank, int world,
                                      int rank, int64_t capacity, int64_t src_stride, const uint64_t* peer_rows,
                                      const uint64_t* peer_expert, const uint64_t* peer_src, int vec) {
  const int lane = threadIdx.x % 32;
  for (int64_t p = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) / 32; p < n;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x / 32) {
    const int32_t e = pos_entry[p];
    if (e < 0) continue;
    const int q = keys[e];
    if (q < 0 || q >= world || e >= n) {  // a destination rank or entry outside this step
      if (lane == 0) atomicOr(&g_ep_error, kEpRangeError);
      continue;
    }
    int64_t slot = p - send_offset[q];
    for (int r = 0; r < rank; ++r) slot += count_matrix[r * world + q];
    // counts exchanged by the all-gather place every row inside the receive buffer; a slot
    // outside it (counts that disagree with the rows sent) is recorded, never stored
    if (slot < 0 || slot >= capacity) {
      if (lane == 0) atomicOr(&g_ep_error, kEpRangeError);
      continue;
    }
    const uint16_t* src = hidden + static_cast<int64_t>(pos_token[p]) * H;
    uint16_t* dst = reinterpret_cast<uint16_t*>(peer_rows[q]) + slot * H;
    if (vec) {
      for (int64_t i = lane; i < H / 8; i += 32)
        reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
    } else {
      for (int64_t i = lane; i < H; i += 32) dst[i] = src[i];
    }
    if (lane == 0) {
      reinterpret_cast<int32_t*>(peer_expert[q])[slot] = static_cast<int32_t>(ids[e] - q * per_rank);
      reinterpret_cast<int32_t*>(peer_src[q])[slot] = static_cast<int32_t>(rank * src_stride + e);
    }
  }
  __threadfence_system();
}

// fp32 -> bf16 of four values (round to nearest even), as 8 bytes
MOE_D uint2 bf16x4(const float4& f) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(f.x, f.y), hi = __floats2bfloat162_rn(f.z, f.w);
  return make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}

// Expert outputs home: received row j (valid: expert >= 0) came from entry
// e of rank r (src = r * src_stride + e); its output row goes, rounded to
// bf16, to row e of rank r's return buffer.  One warp per row.
__global__ void ep_p2p_return_kernel(const float* y, int64_t rows, const int32_t* recv_expert, const int32_t* recv_src,
                                     int64_t H, int64_t src_stride, int world, int64_t home_rows,
                                     const uint64_t* peer_yback, int vec) {
  const int lane = threadIdx.x % 32;
  for (int64_t j = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) / 32; j < rows;
       j += static_cast<int64_t>(gridDim.x) * blockDim.x / 32) {
    if (recv_expert[j] < 0) continue;
    const int32_t s = recv_src[j];
    const int64_t r = s / src_stride, e = s % src_stride;
    // src codes are written by the peers' dispatch: check them before storing into a peer's memory
    if (s < 0 || r >= world || e >= home_rows) {
      if (lane == 0) atomicOr(&g_ep_error, kEpRangeError);
      continue;
    }
    const float* src = y + j * H;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(peer_yback[r]) + e * H;
    if (vec) {
      for (int64_t i = lane; i < H / 4; i += 32)
        reinterpret_cast<uint2*>(dst)[i] = bf16x4(__ldcs(reinterpret_cast<const float4*>(src) + i));
    } else {
      for (int64_t i = lane; i < H; i += 32) dst[i] = __float2bfloat16_rn(src[i]);
    }
  }
  __threadfence_system();
}

// Home rows of the received rows' outputs: pair p (received row j =
// pair_entry[p], sent by rank r as its entry e: row_src[j] = r * src_stride +
// e) -> row e of rank r's return buffer.
// A src code outside [0, world * src_stride) or a row at or past home_rows is
// recorded in the error word and its pair is sent to `sink` (one row of this
// rank's own workspace) instead: the stores that follow -- the down GEMM's
// epilogue or ep_pairs_home_kernel -- then never leave this GPU for it.
__global__ void ep_pair_home_kernel(const int32_t* pair_entry, const int32_t* n_pairs, const int32_t* row_src,
                                    int64_t src_stride, int world, int64_t home_rows, const uint64_t* peer_yback,
                                    int64_t H, uint64_t* pair_dst, int64_t cap, float* sink) {
  const int64_t n = min(static_cast<int64_t>(*n_pairs), cap);
  for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < n;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t j = pair_entry[p];
    const int32_t s = (j >= 0 && j < cap) ? row_src[j] : -1;
    const int64_t r = s / src_stride, e = s % src_stride;
    if (s < 0 || r >= world || e >= home_rows) {
      atomicOr(&g_ep_error, kEpRangeError);
      pair_dst[p] = reinterpret_cast<uint64_t>(sink);
      continue;
    }
    pair_dst[p] = peer_yback[r] + static_cast<uint64_t>(e * H) * sizeof(__nv_bfloat16);
  }
}

// Pair p's fp32 output row y[p], rounded to bf16, to its home row
// pair_dst[p] (another GPU's memory or this one's).  One warp per pair.
__global__ void ep_pairs_home_kernel(const float* y, const int32_t* n_pairs, const uint64_t* pair_dst, int64_t H,
                                     int64_t cap, int vec) {
  const int lane = threadIdx.x % 32;
  const int64_t n = min(static_cast<int64_t>(*n_pairs), cap);
  for (int64_t p = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) / 32; p < n;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x / 32) {
    const float* src = y + p * H;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(pair_dst[p]);
    if (vec) {
      for (int64_t i = lane; i < H / 4; i += 32)
        reinterpret_cast<uint2*>(dst)[i] = bf16x4(__ldcs(reinterpret_cast<const float4*>(src) + i));
    } else {
      for (int64_t i = lane; i < H; i += 32) dst[i] = __float2bfloat16_rn(src[i]);
    }
  }
  __threadfence_system();
}

namespace {

// The shared expert's chunk list for the side stream: its pairs first .. first
// + T - 1 (token t's is first + t) in chunks of <= 8, and their token rows.
__global__ void shared_chunks_kernel(int32_t* seg, int32_t* start, int32_t* len, int32_t* n, int32_t* rows,
                                     int shared_index, int first, int T) {
  const int nch = (T + 7) / 8;
  for (int i = threadIdx.x; i < nch; i += blockDim.x) {
    seg[i] = shared_index;
    start[i] = first + 8 * i;
    len[i] = min(8, T - 8 * i);
  }
  for (int i = threadIdx.x; i < T; i += blockDim.x) rows[i] = i;
  if (threadIdx.x == 0) *n = nch;
}

// A non-blocking side stream and its fork / join events, one set per device,
// created on first use (the first call on a device should come before any
// stream capture).
struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
std::mutex g_side_mutex;
SideStream g_side[64];

int side_stream(SideStream** out) {
  int dev = 0;
  MOE_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(kUnsupported, "side stream: device index beyond 64");
  std::lock_guard<std::mutex> lock(g_side_mutex);
  SideStream& sd = g_side[dev];
  if (!sd.s) {
    MOE_CUDA(cudaStreamCreateWithFlags(&sd.s, cudaStreamNonBlocking), "side stream");
    MOE_CUDA(cudaEventCreateWithFlags(&sd.fork, cudaEventDisableTiming), "fork event");
    MOE_CUDA(cudaEventCreateWithFlags(&sd.join, cudaEventDisableTiming), "join event");
  }
  *out = &sd;
  return kOk;
}

}  // namespace

extern "C" {

int moe_b200_abi_version(void) { return MOE_B200_ABI_VERSION; }

const char* moe_b200_last_error(void) { return g_last_error; }

// ---------------------------------------------------------------------------
// FP8 linears
// ---------------------------------------------------------------------------

static int linear_common(const uint8_t* wa, const float* sa, const uint8_t* wb, const float* sb, const float* x,
                         float* oa, float* ob, int64_t batch, int64_t rows, int64_t cols, int64_t scols,
                         cudaStream_t stream) {
  if (batch <= 0 || rows <= 0 || cols <= 0 || scols <= 0) return fail(kBadDims, "bad dimensions");
  if (scols != ceil_div(cols, kBlock)) return fail(kBadDims, "scale_cols != ceil(in_cols / 128)");
  const bool dual = wb != nullptr;
  const int nt = pick_nt(batch, cols, 16, kXF32);
  if (nt == 0) return fail(kUnsupported, "in_cols too large for the staged GEMV");
  // one segment holding every row of `hidden`
  Plan sizing;
  const int64_t cap = chunk_capacity(batch, 1, nt);
  sizing.take<uint64_t>(4);
  sizing.take<int32_t>(3);
  sizing.take<int32_t>(cap * 3 + 1);
  Scratch scratch(nullptr, 0, sizing.used(), stream);
  if (!scratch.ok()) return fail(kNoMemory, "allocation failed");
  Plan plan(scratch.base());
  uint64_t* tab = plan.take<uint64_t>(4);
  int32_t* seg = plan.take<int32_t>(3);
  int32_t* chunks = plan.take<int32_t>(cap * 3 + 1);
  const uint64_t host_tab[4] = {reinterpret_cast<uint64_t>(wa), reinterpret_cast<uint64_t>(sa),
                                reinterpret_cast<uint64_t>(wb), reinterpret_cast<uint64_t>(sb)};
  const int32_t host_seg[3] = {0, static_cast<int32_t>(batch), 0};
  MOE_CUDA(cudaMemcpyAsync(tab, host_tab, sizeof host_tab, cudaMemcpyHostToDevice, stream), "tables");
  MOE_CUDA(cudaMemcpyAsync(seg, host_seg, sizeof host_seg, cudaMemcpyHostToDevice, stream), "segments");
  ChunkArgs ca{seg, 1, nt, chunks, chunks + cap, chunks + 2 * cap, chunks + 3 * cap};
  MOE_CUDA(launch_chunks(ca, stream), "chunk list");
  GemvArgs g{};
  g.w0 = tab; g.s0 = tab + 1; g.w1 = tab + 2; g.s1 = tab + 3;
  g.x = x; g.pair_row = nullptr;
  g.chunk_seg = ca.chunk_seg; g.chunk_start = ca.chunk_start; g.chunk_len = ca.chunk_len; g.n_chunks = ca.n_chunks;
  g.out0 = oa; g.out1 = ob; g.N = static_cast<int>(rows); g.K = static_cast<int>(cols); g.scale_cols = static_cast<int>(scols);
  const bool vec = cols % 16 == 0 && aligned16(x) && aligned16(wa) && (!dual || aligned16(wb));
  MOE_CUDA(gemv(g, kXF32, dual ? 2 : 1, dual ? kEpiStoreBoth : kEpiStore, nt, vec, stream), "linear");
  return kOk;
}

int moe_fp8_e4m3_block_linear_f32(const uint8_t* fp8_weight, const float* scale_inv, const float* hidden,
                                  float* out, int64_t batch, int64_t out_rows, int64_t in_cols,
                                  int64_t scale_cols, void* stream) {
  if (!fp8_weight || !scale_inv || !hidden || !out) return fail(kNullPointer, "null pointer");
  return linear_common(fp8_weight, scale_inv, nullptr, nullptr, hidden, out, nullptr, batch, out_rows, in_cols,
                       scale_cols, as_stream(stream));
}

int moe_fp8_e4m3_block_dual_linear_f32(const uint8_t* wa, const float* sa, const uint8_t* wb, const float* sb,
                                       const float* hidden, float* out_a, float* out_b, int64_t batch,
                                       int64_t out_rows, int64_t in_cols, int64_t scale_cols, void* stream) {
  if (!wa || !sa || !wb || !sb || !hidden || !out_a || !out_b) return fail(kNullPointer, "null pointer");
  return linear_common(wa, sa, wb, sb, hidden, out_a, out_b, batch, out_rows, in_cols, scale_cols,
                       as_stream(stream));
}

// ---------------------------------------------------------------------------
// FP8 expert MLPs
// ---------------------------------------------------------------------------

static int check_mlp_dims(int64_t E, int64_t B, int64_t I, int64_t H, int64_t gsc, int64_t dsc) {
  if (E <= 0 || B <= 0 || I <= 0 || H <= 0 || gsc <= 0 || dsc <= 0) return fail(kBadDims, "bad dimensions");
  if (gsc != ceil_div(H, kBlock) || dsc != ceil_div(I, kBlock))
    return fail(kBadDims, "scale columns do not match the 128x128 block layout");
  if (E > kMaxBuckets) return fail(kUnsupported, "too many experts in one call");
  if (B > INT32_MAX || I > INT32_MAX || H > INT32_MAX) return fail(kUnsupported, "dimension beyond int32");
  if (E * B > (int64_t(1) << 30)) return fail(kUnsupported, "too many (expert, row) pairs");
  // keeps every workspace size (pairs x max(I, H) x 4 bytes and the like) far from int64 overflow
  if (E * B * std::max(I, H) > (int64_t(1) << 50)) return fail(kUnsupported, "problem too large");
  return kOk;
}

int64_t moe_fp8_mlp_workspace_bytes(int64_t pairs, int64_t segments, int64_t batch, int64_t I, int64_t H) {
  Plan p;
  plan_mlp(p, pairs, segments, std::max(pairs, segments * batch), I, H, 1, true);
  p.take<uint64_t>(6 * segments);
  return static_cast<int64_t>(p.used());
}

int moe_fp8_e4m3_block_mlp_f32(const uint8_t* gate_weight, const float* gate_scale_inv, const uint8_t* up_weight,
                               const float* up_scale_inv, const uint8_t* down_weight, const float* down_scale_inv,
                               const float* hidden, float* out, int64_t batch, int64_t I, int64_t H,
                               int64_t gsc, int64_t dsc, void* workspace, int64_t workspace_bytes, void* stream) {
  if (!gate_weight || !gate_scale_inv || !up_weight || !up_scale_inv || !down_weight || !down_scale_inv ||
      !hidden || !out)
    return fail(kNullPointer, "null pointer");
  int code = check_mlp_dims(1, batch, I, H, gsc, dsc);
  if (code != kOk) return code;
  cudaStream_t s = as_stream(stream);
  // a one-entry device table of the six pointers, then the many_f32 path (E = 1: out is [1, B, H])
  uint64_t* tab = nullptr;
  MOE_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&tab), 6 * sizeof(uint64_t), s), "table alloc");
  const uint64_t host[6] = {reinterpret_cast<uint64_t>(gate_weight), reinterpret_cast<uint64_t>(gate_scale_inv),
                            reinterpret_cast<uint64_t>(up_weight),   reinterpret_cast<uint64_t>(up_scale_inv),
                            reinterpret_cast<uint64_t>(down_weight), reinterpret_cast<uint64_t>(down_scale_inv)};
  cudaError_t err = cudaMemcpyAsync(tab, host, sizeof host, cudaMemcpyHostToDevice, s);
  if (err != cudaSuccess) {
    cudaFreeAsync(tab, s);
    return cuda_fail(err, "table copy");
  }
  Tables t{tab, tab + 1, tab + 2, tab + 3, tab + 4, tab + 5};
  code = mlp_items(t, hidden, nullptr, 0, out, true, 1, batch, I, H, gsc, dsc, workspace, workspace_bytes, s);
  cudaFreeAsync(tab, s);
  return code;
}

#define MOE_TABLES_OK(g, gs, u, us, d, ds) ((g) && (gs) && (u) && (us) && (d) && (ds))

int moe_fp8_e4m3_block_mlp_many_f32(const uint64_t* gw, const uint64_t* gs, const uint64_t* uw, const uint64_t* us,
                                    const uint64_t* dw, const uint64_t* ds, const float* hidden, float* out,
                                    int64_t E, int64_t B, int64_t I, int64_t H, int64_t gsc, int64_t dsc,
                                    void* workspace, int64_t workspace_bytes, void* stream) {
  if (!MOE_TABLES_OK(gw, gs, uw, us, dw, ds) || !hidden || !out) return fail(kNullPointer, "null pointer");
  int code = check_mlp_dims(E, B, I, H, gsc, dsc);
  if (code != kOk) return code;
  Tables t{gw, gs, uw, us, dw, ds};
  return mlp_items(t, hidden, nullptr, 0, out, true, E, B, I, H, gsc, dsc, workspace, workspace_bytes,
                   as_stream(stream));
}

int moe_fp8_e4m3_block_mlp_many_weighted_f32(const uint64_t* gw, const uint64_t* gs, const uint64_t* uw,
                                             const uint64_t* us, const uint64_t* dw, const uint64_t* ds,
                                             const float* hidden, const float* route, float* out, int64_t E,
                                             int64_t B, int64_t I, int64_t H, int64_t gsc, int64_t dsc,
                                             void* workspace, int64_t workspace_bytes, void* stream) {
  if (!MOE_TABLES_OK(gw, gs, uw, us, dw, ds) || !hidden || !route || !out) return fail(kNullPointer, "null pointer");
  int code = check_mlp_dims(E, B, I, H, gsc, dsc);
  if (code != kOk) return code;
  Tables t{gw, gs, uw, us, dw, ds};
  return mlp_items(t, hidden, route, 0, out, false, E, B, I, H, gsc, dsc, workspace, workspace_bytes,
                   as_stream(stream));
}

int moe_fp8_e4m3_block_mlp_many_row_weighted_f32(const uint64_t* gw, const uint64_t* gs, const uint64_t* uw,
                                                 const uint64_t* us, const uint64_t* dw, const uint64_t* ds,
                                                 const float* hidden, const float* route, float* out, int64_t E,
                                                 int64_t B, int64_t I, int64_t H, int64_t gsc, int64_t dsc,
                                                 void* workspace, int64_t workspace_bytes, void* stream) {
  if (!MOE_TABLES_OK(gw, gs, uw, us, dw, ds) || !hidden || !route || !out) return fail(kNullPointer, "null pointer");
  int code = check_mlp_dims(E, B, I, H, gsc, dsc);
  if (code != kOk) return code;
  Tables t{gw, gs, uw, us, dw, ds};
  return mlp_items(t, hidden, route, 1, out, false, E, B, I, H, gsc, dsc, workspace, workspace_bytes,
                   as_stream(stream));
}

int moe_fp8_e4m3_block_mlp_many_pair_weighted_f32(const uint64_t* gw, const uint64_t* gs, const uint64_t* uw,
                                                  const uint64_t* us, const uint64_t* dw, const uint64_t* ds,
                                                  const float* hidden, const int64_t* pair_item,
                                                  const int64_t* pair_row, const float* pair_w, float* out,
                                                  int64_t E, int64_t P, int64_t B, int64_t I, int64_t H,
                                                  int64_t gsc, int64_t dsc, void* workspace,
                                                  int64_t workspace_bytes, void* stream) {
  if (!MOE_TABLES_OK(gw, gs, uw, us, dw, ds) || !hidden || !pair_item || !pair_row || !pair_w || !out)
    return fail(kNullPointer, "null pointer");
  if (P < 0) return fail(kBadDims, "bad dimensions");
  int code = check_mlp_dims(E, B, I, H, gsc, dsc);
  if (code != kOk) return code;
  if (B > kMaxBuckets) return fail(kUnsupported, "batch too large for the pair combine");
  cudaStream_t s = as_stream(stream);
  MOE_CUDA(cudaMemsetAsync(out, 0, static_cast<size_t>(B * H) * sizeof(float), s), "clear out");
  if (P == 0) return kOk;
  const int nt = pick_nt(P, H, I, kXF32);
  if (nt == 0) return fail(kUnsupported, "hidden/intermediate size too large for the staged GEMV");
  Plan sizing;
  plan_mlp(sizing, P, E, P, I, H, nt, true);
  sizing.take<int32_t>(P);           // rows32
  sizing.take<int32_t>(B + 2);       // row_ptr
  sizing.take<int32_t>(P);           // row_pairs (pair entry order per row)
  sizing.take<int32_t>(P);           // row pair rows (unused)
  sizing.take<int32_t>(1);           // bad flag
  Scratch scratch(workspace, workspace_bytes, sizing.used(), s);
  if (!scratch.ok()) return fail(kNoMemory, "workspace too small or allocation failed");
  Plan plan(scratch.base());
  MlpScratch m = plan_mlp(plan, P, E, P, I, H, nt, true);
  int32_t* rows32 = plan.take<int32_t>(P);
  int32_t* row_ptr = plan.take<int32_t>(B + 2);
  int32_t* row_entries = plan.take<int32_t>(P);
  int32_t* row_rows = plan.take<int32_t>(P);
  int32_t* bad = plan.take<int32_t>(1);
  // reject out-of-range indices (fp8_linear.cpp:873-880 returns -4)
  MOE_CUDA(cudaMemsetAsync(bad, 0, sizeof(int32_t), s), "clear flag");
  validate_pairs_kernel<<<grid_for(P), 256, 0, s>>>(pair_item, pair_row, P, E, B, bad);
  int32_t host_bad = 0;
  MOE_CUDA(cudaMemcpyAsync(&host_bad, bad, sizeof host_bad, cudaMemcpyDeviceToHost, s), "flag copy");
  MOE_CUDA(cudaStreamSynchronize(s), "flag sync");
  if (host_bad) return fail(kBadIndex, "pair index out of range");
  i64_to_i32_kernel<<<grid_for(P), 256, 0, s>>>(pair_item, m.keys, P);
  i64_to_i32_kernel<<<grid_for(P), 256, 0, s>>>(pair_row, rows32, P);
  MOE_CUDA(cudaGetLastError(), "index copy");
  BucketArgs ba{};
  ba.keys = m.keys; ba.rows = rows32; ba.weights = pair_w; ba.n = static_cast<int>(P); ba.k = 1;
  ba.key_lo = 0; ba.n_buckets = static_cast<int>(E);
  ba.bucket_offset = m.seg_offset; ba.pair_row = m.pair_row; ba.pair_weight = m.pair_weight;
  ba.pair_entry = m.pair_entry; ba.entry_pair = m.entry_pair;
  MOE_CUDA(launch_bucket(ba, s), "bucket by item");
  Tables t{gw, gs, uw, us, dw, ds};
  const bool vec = H % 16 == 0 && I % 16 == 0 && aligned16(hidden);
  code = run_expert_stages(t, hidden, kXF32, m, m.y, E, I, H, gsc, dsc, nt, vec, s);
  if (code != kOk) return code;
  // per-row lists in pair order: bucket the entries by row, then map entry -> pair
  BucketArgs br{};
  br.keys = rows32; br.rows = nullptr; br.weights = nullptr; br.n = static_cast<int>(P); br.k = 1;
  br.key_lo = 0; br.n_buckets = static_cast<int>(B);
  br.bucket_offset = row_ptr; br.pair_row = row_rows; br.pair_entry = row_entries;
  MOE_CUDA(launch_bucket(br, s), "bucket by row");
  map_entries_kernel<<<grid_for(P), 256, 0, s>>>(row_entries, m.entry_pair, row_entries, P);
  MOE_CUDA(cudaGetLastError(), "row lists");
  CombineArgs c{};
  c.y = m.y; c.row_ptr = row_ptr; c.stride = 0; c.row_pairs = row_entries; c.pair_weight = m.pair_weight;
  c.extra_base = -1; c.T = static_cast<int>(B); c.H = static_cast<int>(H); c.out_f32 = out;
  MOE_CUDA(launch_combine(c, s), "combine");
  return kOk;
}

// ---------------------------------------------------------------------------
// Dequant
// ---------------------------------------------------------------------------

static int dequant_common(const uint8_t* w, const float* s, uint16_t* out, int64_t rows, int64_t cols,
                          int64_t scols, bool bf16, void* stream) {
  if (!w || !s || !out) return fail(kNullPointer, "null pointer");
  if (rows <= 0 || cols <= 0 || scols <= 0) return fail(kBadDims, "bad dimensions");
  if (scols != ceil_div(cols, kBlock)) return fail(-3, "scale_cols != ceil(cols / 128)");  // fp8_dequant.cpp:133-136
  MOE_CUDA(launch_fp8_dequant(w, s, out, rows, cols, scols, bf16, as_stream(stream)), "dequant");
  return kOk;
}

int moe_fp8_e4m3_dequant_to_fp16(const uint8_t* w, const float* s, uint16_t* out, int64_t rows, int64_t cols,
                                 int64_t scols, void* stream) {
  return dequant_common(w, s, out, rows, cols, scols, false, stream);
}

int moe_fp8_e4m3_dequant_to_bf16(const uint8_t* w, const float* s, uint16_t* out, int64_t rows, int64_t cols,
                                 int64_t scols, void* stream) {
  return dequant_common(w, s, out, rows, cols, scols, true, stream);
}

// ---------------------------------------------------------------------------
// Routers
// ---------------------------------------------------------------------------

int64_t moe_route_topk_workspace_bytes(int64_t tokens, int64_t experts) {
  Plan p;
  // above 256 tokens the logits may come as up to kMaxRouterParts split-K partials
  p.take<float>((tokens > 256 ? kMaxRouterParts : 1) * tokens * experts);
  return static_cast<int64_t>(p.used());
}

int moe_route_topk(const void* hidden, int hidden_dtype, const void* router_weight, int router_dtype,
                   const float* bias, int64_t T, int64_t H, int64_t E, int64_t n_group, int64_t topk_group,
                   int64_t k, int scoring, int renorm, float route_scale, int round_bf16, int64_t* out_ids,
                   float* out_weights_f32, uint16_t* out_weights_bf16, void* workspace, int64_t workspace_bytes,
                   void* stream) {
  if (!hidden || !router_weight) return fail(kNullPointer, "null pointer");
  int code = check_route(T, H, E, n_group, topk_group, k);
  if (code != kOk) return code;
  cudaStream_t s = as_stream(stream);
  Scratch scratch(workspace, workspace_bytes, moe_route_topk_workspace_bytes(T, E), s);
  if (!scratch.ok()) return fail(kNoMemory, "workspace too small or allocation failed");
  return route_impl(hidden, hidden_dtype, router_weight, router_dtype, bias, T, H, E, n_group, topk_group, k,
                    scoring, renorm, 0, route_scale, round_bf16, out_ids, nullptr, out_weights_f32,
                    out_weights_bf16, reinterpret_cast<float*>(scratch.base()), s);
}

int moe_ds_router_topk_u16(const uint16_t* hidden_u16, const uint16_t* router_u16, int64_t H, int64_t E,
                           int64_t k, int64_t dtype_code, int64_t* out_ids, float* out_weights, void* stream) {
  if (!hidden_u16 || !router_u16 || !out_ids || !out_weights) return 1;       // ds_forward.cpp:889-894
  if (H <= 0 || E <= 0 || k <= 0 || k > E) return 2;                          // :895-897
  if (k > 32 || E > 2048) return fail(kUnsupported, "k > 32 or more than 2048 experts");
  cudaStream_t s = as_stream(stream);
  Scratch scratch(nullptr, 0, moe_route_topk_workspace_bytes(1, E), s);
  if (!scratch.ok()) return fail(kNoMemory, "allocation failed");
  const int dt = dtype_code == 1 ? kDtypeBF16 : kDtypeF16;
  return route_impl(hidden_u16, dt, router_u16, dt, nullptr, 1, H, E, 1, 1, k, kScoreSoftmax, 1, 1, 1.0f, 0,
                    out_ids, nullptr, out_weights, nullptr, reinterpret_cast<float*>(scratch.base()), s);
}

// ---------------------------------------------------------------------------
// Whole DeepSeek-V3 layer
// ---------------------------------------------------------------------------

struct LayerPlan {
  float* logits;
  int32_t* ids32;
  float* wts;
  MlpScratch m;
  __half* x16;
  float* xscale;
  __half* act16;
  float* ascale;
  // register-fed MMA kernel k-split: partial fragments + per-task counters
  int ksplit1, ksplit2;    // gate/up, down
  int64_t tasks1, tasks2;  // upper bounds on tasks (chunks x row tiles)
  float* partial;
  int32_t* counters;       // [tasks1] gate/up then [tasks2] down, then [2 x chunks] (fused decode); zeroed by
                           // the x staging of every forward
  int64_t n_counters;
  int64_t chunks;          // upper bound on the chunk list's length
  int64_t comb_tiles;      // 32-column tiles of a hidden row (the folded combine's counters)
  // the shared expert on a side stream (decode layers): its staged x rows, chunk list, split-K state
  __half* sh_x16;
  float* sh_xscale;
  int32_t* sh_rows;        // [T] token of the shared pair first + t: t
  int32_t* sh_chunk_seg;
  int32_t* sh_chunk_start;
  int32_t* sh_chunk_len;
  int32_t* sh_n_chunks;
  float* sh_partial;
  int32_t* sh_counters;    // [sh_tasks1 + sh_tasks2], zeroed by the side stream's x staging
  int64_t sh_tasks1, sh_tasks2, sh_n_counters;
  int sh_ks1, sh_ks2;
  int64_t sh_ctas;
  float* partial_fused;    // fused decode: [2 phases][2 x fused_warps][32 x 8] piece slots
  int fused_warps;
  // prefill (tcgen05 grouped GEMM): pair-ordered fp16 activations, their
  // scales, and the per-expert m-tile prefix
  __half* a16;
  float* a16scale;
  int32_t* mprefix;
  int32_t* bucket_scratch;  // multi-CTA dispatch: per-block bucket counts
};

// Token counts from which the whole-layer call runs the prefill GEMM (when
// the weights are tiled and the shapes allow): from ~16 pairs per expert on,
// one 128-row tile of tensor-core work beats re-streaming the weights per
// chunk of 8 pairs.
constexpr int64_t kPrefillMinTokens = 512;

// lean: the caller runs the tcgen05 GEMM with its outputs stored through a
// row table -- no warp-MMA buffers (x16, k-split partials) and no pair-order y.
static LayerPlan plan_layer(Plan& p, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k, int shared, int nt,
                            bool router = true, bool lean = false) {
  LayerPlan l{};
  if (router)
    l.logits = p.take<float>(static_cast<int64_t>(std::max(1, router_split_parts(static_cast<int>(H)))) * T * E);
  l.ids32 = p.take<int32_t>(T * k);
  l.wts = p.take<float>(T * k);
  l.bucket_scratch = p.take<int32_t>(bucket_scratch_ints(T * k, static_cast<int>(E)));
  const int64_t pairs = T * k + (shared ? T : 0);
  l.m = plan_mlp(p, pairs, E + 1, T * k, I, H, nt, !lean);
  if (!lean) {
    l.x16 = p.take<__half>(T * H);
    l.xscale = p.take<float>(T);
  }
  l.act16 = p.take<__half>(pairs * I);
  l.ascale = p.take<float>(pairs);
  const int64_t chunks = std::min(pairs, chunk_capacity(pairs, E + (shared ? 1 : 0), 8));
  l.tasks1 = chunks * ceil_div(I, mma_task_rows(2));
  l.tasks2 = chunks * ceil_div(H, mma_task_rows(1));
  // the k-split depends on the feed's resident warps; size for either feed
  const int ks_regs1 = mma_gemv_ksplit(l.tasks1, static_cast<int>(H));
  const int ks_regs2 = mma_gemv_ksplit(l.tasks2, static_cast<int>(I));
  const int forced = std::min(g_force_ksplit, kMaxMmaKSplit);
  const int ks_async1 = forced > 0 ? forced : async_gemv_ksplit(l.tasks1, static_cast<int>(H));
  const int ks_async2 = forced > 0 ? forced : async_gemv_ksplit(l.tasks2, static_cast<int>(I));
  const bool async = g_mma_feed == 2;
  l.ksplit1 = async ? ks_async1 : ks_regs1;
  l.ksplit2 = async ? ks_async2 : ks_regs2;
  const int64_t frag = 32 * 8;
  const int64_t part = std::max({l.tasks1 * std::max(ks_regs1, ks_async1), l.tasks2 * std::max(ks_regs2, ks_async2),
                                 int64_t{1}});
  l.chunks = chunks;
  if (!lean) {
    l.partial = p.take<float>(part * frag);
    // + the combine's per-(token, 32-column tile) arrivals when this is a whole layer
    l.comb_tiles = ceil_div(H, 32);
    l.n_counters = l.tasks1 + l.tasks2 + 2 * chunks + (router ? T * l.comb_tiles : 0);
    l.counters = p.take<int32_t>(l.n_counters);
    l.fused_warps = decode_fused_warps();
    l.partial_fused = p.take<float>(static_cast<int64_t>(2) * 2 * l.fused_warps * frag);
    if (router && shared) {
      const int64_t sh_chunks = ceil_div(T, 8);
      l.sh_x16 = p.take<__half>(T * H);
      l.sh_xscale = p.take<float>(T);
      l.sh_rows = p.take<int32_t>(T);
      l.sh_chunk_seg = p.take<int32_t>(sh_chunks);
      l.sh_chunk_start = p.take<int32_t>(sh_chunks);
      l.sh_chunk_len = p.take<int32_t>(sh_chunks);
      l.sh_n_chunks = p.take<int32_t>(1);
      l.sh_tasks1 = sh_chunks * ceil_div(I, mma_task_rows(2));
      l.sh_tasks2 = sh_chunks * ceil_div(H, mma_task_rows(1));
      l.sh_ctas = static_cast<int64_t>(gemv_grid_ctas()) *
                  std::min(kSharedSideCtasPerSm, std::max(1, async_gemv_ctas_per_sm() - 1));
      l.sh_ks1 = async_gemv_ksplit_for(l.sh_tasks1, static_cast<int>(H), l.sh_ctas);
      l.sh_ks2 = async_gemv_ksplit_for(l.sh_tasks2, static_cast<int>(I), l.sh_ctas);
      l.sh_partial = p.take<float>(std::max(l.sh_tasks1 * l.sh_ks1, l.sh_tasks2 * l.sh_ks2) * frag);
      l.sh_n_counters = l.sh_tasks1 + l.sh_tasks2;
      l.sh_counters = p.take<int32_t>(l.sh_n_counters);
    }
  }
  // the tcgen05 GEMM's pair rows: layers (router) and expert-parallel experts (rows) alike
  if (T >= kPrefillMinTokens) {
    l.a16 = p.take<__half>(pairs * H);
    l.a16scale = p.take<float>(pairs);
    l.mprefix = p.take<int32_t>(E + 2);
  }
  return l;
}

// The expert stages on the tcgen05 grouped GEMM (tiled weights): gather the
// pairs' fp16 rows, gate/up + SwiGLU, stage the activations, down.
// y16: the down GEMM stores bf16 rows into m.y's memory (the whole layer's path, whose combine reads
// them); otherwise fp32 rows, or rows through out_row.
static int run_expert_stages_prefill(const Tables& t, const void* x, bool x_bf16, int64_t k, bool shared,
                                     const LayerPlan& l, int64_t T,
                                     int64_t pairs, int64_t n_segments, int64_t I, int64_t H, const uint8_t* nan_free,
                                     cudaStream_t s, const uint64_t* out_row = nullptr, bool y16 = false) {
  const MlpScratch& m = l.m;
  // each token's row staged once and written to its pairs' rows (the shared pairs follow the routed ones)
  cudaError_t serr = launch_scatter_rows(x, x_bf16 ? kDtypeBF16 : kDtypeF32, T, H, m.entry_pair, static_cast<int>(k),
                                         shared ? m.seg_offset + (n_segments - 1) : nullptr, l.a16, l.a16scale, s);
  if (serr == cudaErrorNotSupported) {
    if (!l.x16) return fail(kUnsupported, "rows must be 16-byte aligned and at most 16 KiB");
    MOE_CUDA(launch_rows_to_f16(x, x_bf16, static_cast<int>(T), static_cast<int>(H), nullptr, l.x16, l.xscale,
                                nullptr, 0, s),
             "stage x");
    MOE_CUDA(launch_gather_rows(l.x16, l.xscale, m.pair_row, pairs, H, l.a16, l.a16scale, s), "gather pairs");
  } else {
    MOE_CUDA(serr, "stage pairs");
  }
  MOE_CUDA(launch_prefill_tiles(m.seg_offset, static_cast<int>(n_segments), l.mprefix, s), "tile map");
  stage_mark(s);
  const int64_t mtiles_bound = pairs / 128 + n_segments;
  PrefillArgs g1{};
  g1.w0 = t.gw; g1.s0 = t.gs; g1.w1 = t.uw; g1.s1 = t.us;
  g1.a16 = l.a16; g1.ascale = l.a16scale; g1.rows_a = pairs;
  g1.seg_offset = m.seg_offset; g1.mprefix = l.mprefix; g1.n_segments = static_cast<int>(n_segments);
  g1.out = m.act; g1.N = static_cast<int>(I); g1.K = static_cast<int>(H);
  g1.scale_cols = static_cast<int>(ceil_div(H, kBlock)); g1.nanfix = 1; g1.nan_free = nan_free;
  MOE_CUDA(launch_prefill_gemm(g1, true, mtiles_bound * (I / 128), s), "gate/up GEMM");
  stage_mark(s);
  // rows past the last segment (pairs routed nowhere) are neither staged nor read
  MOE_CUDA(launch_rows_to_f16(m.act, false, static_cast<int>(pairs), static_cast<int>(I),
                              m.seg_offset + n_segments, l.act16, l.ascale, nullptr, 0, s),
           "stage activations");
  stage_mark(s);
  PrefillArgs g2 = g1;
  g2.w0 = t.dw; g2.s0 = t.ds; g2.w1 = nullptr; g2.s1 = nullptr;
  g2.a16 = l.act16; g2.ascale = l.ascale;
  g2.out = m.y; g2.out_row = out_row; g2.N = static_cast<int>(H); g2.K = static_cast<int>(I);
  g2.out_row_bf16 = out_row ? 1 : 0;  // rows stored home through the table are the return buffer's bf16 rows
  if (y16 && !out_row) {
    g2.out16 = reinterpret_cast<__nv_bfloat16*>(m.y);
    g2.out = nullptr;
  }
  g2.scale_cols = static_cast<int>(ceil_div(I, kBlock));
  MOE_CUDA(launch_prefill_gemm(g2, false, mtiles_bound * (H / 256), s), "down GEMM");
  stage_mark(s);
  return kOk;
}

// The expert stages on the warp-MMA kernel: x and the SwiGLU activations are
// staged as f16 rows with power-of-two scales.
// The whole layer's combine, for the down stage to fold in.
struct LayerCombine {
  __nv_bfloat16* out;
  int64_t tokens, k;
  bool shared;
};

// x_staged: l.x16 / l.xscale already hold the staged rows and the counters are
// zero (the decode prologue did both).  comb: the layer's combine, folded into
// the down stage when the epilogue folds are on (*combined set true then).
static int run_expert_stages_mma(const Tables& t, const void* x, bool x_bf16, const LayerPlan& l, int64_t T,
                                 int64_t pairs, int64_t n_segments, int64_t I, int64_t H, bool chunks_ready,
                                 const uint8_t* nan_free, cudaStream_t s, int tiled = 0, bool x_staged = false,
                                 const LayerCombine* comb = nullptr, bool* combined = nullptr) {
  const MlpScratch& m = l.m;
  if (!chunks_ready) {
    ChunkArgs ca{m.seg_offset, static_cast<int>(n_segments), 8, m.chunk_seg, m.chunk_start, m.chunk_len, m.n_chunks};
    MOE_CUDA(launch_chunks(ca, s), "chunk list");
  }
  if (!x_staged)
    MOE_CUDA(launch_rows_to_f16(x, x_bf16, static_cast<int>(T), static_cast<int>(H), nullptr, l.x16, l.xscale,
                                l.counters, l.n_counters, s),
             "stage x");
  stage_mark(s);
  MmaArgs g1{};
  g1.w0 = t.gw; g1.s0 = t.gs; g1.w1 = t.uw; g1.s1 = t.us;
  g1.x16 = l.x16; g1.xscale = l.xscale; g1.pair_row = m.pair_row;
  g1.chunk_seg = m.chunk_seg; g1.chunk_start = m.chunk_start; g1.chunk_len = m.chunk_len; g1.n_chunks = m.n_chunks;
  g1.out0 = m.act; g1.N = static_cast<int>(I); g1.K = static_cast<int>(H);
  g1.scale_cols = static_cast<int>(ceil_div(H, kBlock)); g1.nanfix = 1;
  g1.ksplit = l.ksplit1; g1.partial = l.partial; g1.counters = l.counters; g1.nan_free = nan_free;
  g1.tiled = tiled;
  g1.kb_rotate = g_kb_rotate;
  if (g_fused_decode && g_mma_feed == 2 && l.partial_fused && l.fused_warps > 0) {
    // one persistent launch: gate/up + SwiGLU, activation staging, down
    DecodeFusedArgs f{};
    f.up = g1;
    f.up.ksplit = 1;
    f.down = g1;
    f.down.w0 = t.dw; f.down.s0 = t.ds; f.down.w1 = nullptr; f.down.s1 = nullptr;
    f.down.x16 = l.act16; f.down.xscale = l.ascale; f.down.pair_row = nullptr;
    f.down.out0 = m.y; f.down.N = static_cast<int>(H); f.down.K = static_cast<int>(I);
    f.down.scale_cols = static_cast<int>(ceil_div(I, kBlock)); f.down.ksplit = 1;
    f.partial = l.partial_fused;
    f.partial_warps = l.fused_warps;
    f.cnt_up = l.counters;
    f.cnt_down = l.counters + l.tasks1;
    f.chunk_up = l.counters + l.tasks1 + l.tasks2;
    f.chunk_ready = f.chunk_up + l.chunks;
    MOE_CUDA(launch_decode_fused(f, s), "fused decode experts");
    stage_mark(s);
    return kOk;
  }
  // the cp.async kernel can stage the activations and combine the tokens itself (last-arriving warps)
  const bool fold = g_fold_epilogues && g_mma_feed == 2 && l.counters;
  if (fold) {
    g1.stage_x16 = l.act16;
    g1.stage_scale = l.ascale;
    g1.chunk_done = l.counters + l.tasks1 + l.tasks2;
  }
  MOE_CUDA(g_mma_feed == 1   ? launch_tma_mma_gemv(g1, 2, kEpiSwiglu, s)
           : g_mma_feed == 2 ? launch_async_mma_gemv(g1, 2, kEpiSwiglu, l.tasks1, s)
                             : launch_mma_gemv(g1, 2, kEpiSwiglu, l.tasks1, s),
           "gate/up stage");
  stage_mark(s);
  if (!fold) {
    MOE_CUDA(launch_rows_to_f16(m.act, false, static_cast<int>(pairs), static_cast<int>(I), nullptr, l.act16,
                                l.ascale, nullptr, 0, s),
             "stage activations");
    stage_mark(s);
  }
  MmaArgs g2 = g1;
  g2.w0 = t.dw; g2.s0 = t.ds; g2.w1 = nullptr; g2.s1 = nullptr;
  g2.x16 = l.act16; g2.xscale = l.ascale; g2.pair_row = nullptr;
  g2.out0 = m.y; g2.N = static_cast<int>(H); g2.K = static_cast<int>(I);
  g2.scale_cols = static_cast<int>(ceil_div(I, kBlock));
  g2.ksplit = l.ksplit2;
  g2.counters = l.counters + l.tasks1;
  g2.stage_x16 = nullptr; g2.stage_scale = nullptr; g2.chunk_done = nullptr;
  if (fold && comb && comb->out && l.comb_tiles > 0 &&
      l.n_counters >= l.tasks1 + l.tasks2 + 2 * l.chunks + comb->tokens * l.comb_tiles) {
    g2.comb_out = comb->out;
    g2.comb_cnt = l.counters + l.tasks1 + l.tasks2 + 2 * l.chunks;
    g2.pair_token = m.pair_row;
    g2.entry_pair = m.entry_pair;
    g2.pair_weight = m.pair_weight;
    g2.comb_k = static_cast<int>(comb->k);
    g2.comb_shared_base = comb->shared ? static_cast<int>(comb->tokens * comb->k) : -1;
    g2.comb_need = static_cast<int>(comb->k) + (comb->shared ? 1 : 0);
    if (combined) *combined = true;
  }
  MOE_CUDA(g_mma_feed == 1   ? launch_tma_mma_gemv(g2, 1, kEpiStore, s)
           : g_mma_feed == 2 ? launch_async_mma_gemv(g2, 1, kEpiStore, l.tasks2, s)
                             : launch_mma_gemv(g2, 1, kEpiStore, l.tasks2, s),
           "down stage");
  stage_mark(s);
  return kOk;
}

// The shared expert of a decode layer on the side stream: x staging, its chunk
// list, gate/up + SwiGLU, activation staging and down for its pairs
// T*k .. T*k + T - 1, on kSharedSideCtasPerSm CTAs per SM, with a k-split
// sized for that grid (so its sums group the k-blocks differently from a
// launch over the whole GPU).  It forks from `s` where the layer starts and is
// joined before the combine.  Concurrent layers on one device share the side
// stream: their shared-expert work runs in the order the layers forked.
static int run_shared_side(const Tables& t, const void* x, bool x_bf16, const LayerPlan& l, int64_t T, int64_t k,
                           int64_t E, int64_t I, int64_t H, const uint8_t* nan_free, int tiled, cudaStream_t s,
                           SideStream* side) {
  const MlpScratch& m = l.m;
  const int64_t first = T * k;
  {
    // record and wait as one step: another host thread's layer records the same fork event
    std::lock_guard<std::mutex> lock(g_side_mutex);
    MOE_CUDA(cudaEventRecord(side->fork, s), "fork");
    MOE_CUDA(cudaStreamWaitEvent(side->s, side->fork, 0), "fork wait");
  }
  cudaStream_t ss = side->s;
  MOE_CUDA(launch_rows_to_f16(x, x_bf16, static_cast<int>(T), static_cast<int>(H), nullptr, l.sh_x16, l.sh_xscale,
                              l.sh_counters, l.sh_n_counters, ss),
           "shared x");
  shared_chunks_kernel<<<1, 64, 0, ss>>>(l.sh_chunk_seg, l.sh_chunk_start, l.sh_chunk_len, l.sh_n_chunks, l.sh_rows,
                                         static_cast<int>(E), static_cast<int>(first), static_cast<int>(T));
  MOE_CUDA(cudaGetLastError(), "shared chunks");
  MmaArgs g1{};
  g1.w0 = t.gw; g1.s0 = t.gs; g1.w1 = t.uw; g1.s1 = t.us;
  // pair first + t reads x row t: the pair-row table is indexed from `first` on (only valid pairs read it)
  g1.x16 = l.sh_x16; g1.xscale = l.sh_xscale;
  g1.pair_row = reinterpret_cast<const int32_t*>(reinterpret_cast<uintptr_t>(l.sh_rows) - first * sizeof(int32_t));
  g1.chunk_seg = l.sh_chunk_seg; g1.chunk_start = l.sh_chunk_start; g1.chunk_len = l.sh_chunk_len;
  g1.n_chunks = l.sh_n_chunks;
  g1.out0 = m.act; g1.N = static_cast<int>(I); g1.K = static_cast<int>(H);
  g1.scale_cols = static_cast<int>(ceil_div(H, kBlock)); g1.nanfix = 1;
  g1.ksplit = l.sh_ks1; g1.partial = l.sh_partial; g1.counters = l.sh_counters; g1.nan_free = nan_free;
  g1.tiled = tiled;
  MOE_CUDA(launch_async_mma_gemv(g1, 2, kEpiSwiglu, l.sh_tasks1, ss, l.sh_ctas), "shared gate/up");
  MOE_CUDA(launch_rows_to_f16(m.act + first * I, false, static_cast<int>(T), static_cast<int>(I), nullptr,
                              l.act16 + first * I, l.ascale + first, nullptr, 0, ss),
           "shared activations");
  MmaArgs g2 = g1;
  g2.w0 = t.dw; g2.s0 = t.ds; g2.w1 = nullptr; g2.s1 = nullptr;
  g2.x16 = l.act16; g2.xscale = l.ascale; g2.pair_row = nullptr;
  g2.out0 = m.y; g2.N = static_cast<int>(H); g2.K = static_cast<int>(I);
  g2.scale_cols = static_cast<int>(ceil_div(I, kBlock));
  g2.ksplit = l.sh_ks2; g2.counters = l.sh_counters + l.sh_tasks1;
  MOE_CUDA(launch_async_mma_gemv(g2, 1, kEpiStore, l.sh_tasks2, ss, l.sh_ctas), "shared down");
  MOE_CUDA(cudaEventRecord(side->join, ss), "join");
  return kOk;
}

int64_t moe_ds_moe_layer_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k, int shared) {
  Plan p;
  plan_layer(p, T, H, I, E, k, shared, 1);
  return static_cast<int64_t>(p.used());
}

int moe_ds_moe_layer_fp8(const void* hidden, int hidden_dtype, int64_t T, int64_t H, int64_t I,
                         const void* router_weight, int router_dtype, const float* router_bias, int64_t E,
                         int64_t n_group, int64_t topk_group, int64_t k, int scoring, float route_scale,
                         const uint64_t* tables, int has_shared, const uint8_t* nan_free, int weight_layout,
                         uint16_t* out_bf16, int64_t* out_ids, uint16_t* out_weights_bf16, void* workspace,
                         int64_t workspace_bytes, void* stream) {
  if (!hidden || !router_weight || !tables || !out_bf16) return fail(kNullPointer, "null pointer");
  if (weight_layout != 0 && weight_layout != 1) return fail(kBadDims, "weight_layout must be 0 or 1");
  int code = check_route(T, H, E, n_group, topk_group, k);
  if (code != kOk) return code;
  if (I <= 0) return fail(kBadDims, "bad dimensions");
  if (hidden_dtype != kDtypeBF16 && hidden_dtype != kDtypeF32) return fail(kUnsupported, "hidden must be bf16 or fp32");
  if (E + 1 > kMaxBuckets) return fail(kUnsupported, "too many experts");
  const int xd = hidden_dtype == kDtypeBF16 ? kXBF16 : kXF32;
  const int nt = pick_nt(T, H, I, xd);
  if (nt == 0) return fail(kUnsupported, "hidden/intermediate size too large for the staged GEMV");
  cudaStream_t s = as_stream(stream);
  Plan sizing;
  plan_layer(sizing, T, H, I, E, k, has_shared, nt);
  Scratch scratch(workspace, workspace_bytes, sizing.used(), s);
  if (!scratch.ok()) return fail(kNoMemory, "workspace too small or allocation failed");
  Plan plan(scratch.base());
  LayerPlan l = plan_layer(plan, T, H, I, E, k, has_shared, nt);
  g_marks = 0;
  stage_mark(s);
  const int64_t S = E + (has_shared ? 1 : 0);
  const bool use_mma = g_gemv_impl == 0 && mma_gemv_supported(static_cast<int>(H), static_cast<int>(I)) &&
                       mma_gemv_supported(static_cast<int>(I), static_cast<int>(H));
  if (weight_layout == 1 && !(use_mma && g_mma_feed == 2))
    return fail(kUnsupported, "tiled weights need the cp.async warp-MMA GEMV (hidden, intermediate % 128 == 0)");
  const int chunk = use_mma ? 8 : nt;
  // the shared expert on the side stream (decode batches on the cp.async warp-MMA GEMV)
  SideStream* side = nullptr;
  if (g_shared_side && !g_fused_decode && !g_fold_epilogues && use_mma && g_mma_feed == 2 && weight_layout == 1 &&
      has_shared && l.sh_x16 && T < kPrefillMinTokens && (hidden_dtype == kDtypeBF16 || hidden_dtype == kDtypeF32)) {
    code = side_stream(&side);
    if (code != kOk) return code;
    Tables st{tables, tables + S, tables + 2 * S, tables + 3 * S, tables + 4 * S, tables + 5 * S};
    code = run_shared_side(st, hidden, hidden_dtype == kDtypeBF16, l, T, k, E, I, H, nan_free, weight_layout, s, side);
    if (code != kOk) return code;
  }
  // the main stream's expert segments: the routed experts, plus the shared one unless the side stream has it
  const int64_t S_main = side ? S - 1 : S;
  BucketArgs ba{};
  ba.keys = l.ids32; ba.rows = nullptr; ba.weights = l.wts; ba.n = static_cast<int>(T * k);
  ba.k = static_cast<int>(k); ba.key_lo = 0; ba.n_buckets = static_cast<int>(E);
  ba.bucket_offset = l.m.seg_offset; ba.pair_row = l.m.pair_row; ba.pair_weight = l.m.pair_weight;
  ba.pair_entry = l.m.pair_entry; ba.entry_pair = l.m.entry_pair; ba.tail = has_shared ? static_cast<int>(T) : 0;
  ba.block_counts = l.bucket_scratch;
  ChunkArgs ca{l.m.seg_offset, static_cast<int>(S_main), chunk, l.m.chunk_seg, l.m.chunk_start, l.m.chunk_len,
               l.m.n_chunks};
  bool chunks_ready = false, x_staged = false, combined = false;
  if (T <= 256 && route_dispatch_smem_bytes(static_cast<int>(T), static_cast<int>(E)) <= 200 * 1024) {
    // decode batches: logits (cluster-reduced, else split-K partials), then
    // selection + dispatch + chunk list in one CTA
    int nparts = 1;
    const bool prologue = g_decode_prologue && use_mma && l.x16 &&
                          decode_prologue_supported(static_cast<int>(T), static_cast<int>(E), static_cast<int>(k),
                                                    static_cast<int>(H), hidden_dtype, hidden, static_cast<int>(S_main));
    // the router launch stages x with a cluster of its own, off the prologue's path
    bool router_staged = prologue && g_router_stages_x && hidden_dtype == kDtypeBF16;
    cudaError_t lerr = launch_router_logits_cluster(hidden, hidden_dtype, router_weight, router_dtype, l.logits,
                                                    static_cast<int>(T), static_cast<int>(H), static_cast<int>(E), s,
                                                    router_staged ? l.x16 : nullptr,
                                                    router_staged ? l.xscale : nullptr);
    if (lerr == cudaErrorNotSupported) {
      router_staged = false;
      lerr = launch_router_logits_split(hidden, hidden_dtype, router_weight, router_dtype, l.logits,
                                        static_cast<int>(T), static_cast<int>(H), static_cast<int>(E), s);
      nparts = router_split_parts(static_cast<int>(H));
    }
    MOE_CUDA(lerr, "router logits");
    RouteDispatchArgs rd{};
    rd.partial = l.logits;
    rd.nparts = nparts;
    rd.part_stride = T * E;
    rd.bias = router_bias;
    rd.select.tokens = static_cast<int>(T);
    rd.select.experts = static_cast<int>(E);
    rd.select.top_k = static_cast<int>(k);
    rd.select.n_group = static_cast<int>(n_group);
    rd.select.topk_group = static_cast<int>(topk_group);
    rd.select.scoring = scoring;
    rd.select.renorm = scoring == kScoreSigmoid;
    rd.select.softmax_fp64 = 0;
    rd.select.round_bf16 = hidden_dtype == kDtypeBF16;
    rd.select.route_scale = route_scale;
    rd.ids64 = out_ids;
    rd.weights_bf16 = reinterpret_cast<__nv_bfloat16*>(out_weights_bf16);
    rd.bucket.keys_out = l.ids32;
    rd.bucket.weights_out = l.wts;
    rd.bucket.args = ba;
    rd.chunks = ca;
    if (prologue && nparts == 1) {
      // selection, dispatch, chunk list, x staging (unless the router staged x) and counter reset in one CTA
      DecodePrologueArgs dp{};
      dp.rd = rd;
      dp.x = hidden;
      dp.hidden = static_cast<int>(H);
      dp.x16 = l.x16;
      dp.xscale = l.xscale;
      dp.stage_x = router_staged ? 0 : 1;
      dp.zero = l.counters;
      dp.zero_n = l.n_counters;
      MOE_CUDA(launch_decode_prologue(dp, hidden_dtype, s), "decode prologue");
      x_staged = true;
    } else {
      MOE_CUDA(launch_route_dispatch(rd, s), "route + dispatch");
    }
    chunks_ready = true;
  } else {
    // 1. route (weights rounded through bf16 like fp8_source.py:1547 when hidden is bf16)
    code = route_impl(hidden, hidden_dtype, router_weight, router_dtype, router_bias, T, H, E, n_group, topk_group,
                      k, scoring, 0, 0, route_scale, hidden_dtype == kDtypeBF16, out_ids, l.ids32, l.wts,
                      out_weights_bf16, l.logits, s);
    if (code != kOk) return code;
    // 2. dispatch: expert-contiguous pairs, ascending token order inside an expert, shared expert last
    MOE_CUDA(launch_bucket(ba, s), "dispatch");
  }
  // 3. experts
  Tables t{tables, tables + S, tables + 2 * S, tables + 3 * S, tables + 4 * S, tables + 5 * S};
  const bool vec = H % 16 == 0 && I % 16 == 0 && aligned16(hidden);
  const bool prefill = weight_layout == 1 && T >= kPrefillMinTokens && l.a16 != nullptr &&
                       prefill_supported(H, I, true) && prefill_supported(I, H, false);
  if (prefill) {
    // each expert's output rounded to bf16 by the down GEMM (the reference rounds it there too,
    // fp8_source.py:1839-1847): half the bytes written and read back by the combine
    code = run_expert_stages_prefill(t, hidden, hidden_dtype == kDtypeBF16, k, has_shared != 0, l, T,
                                     T * k + (has_shared ? T : 0), S, I,
                                     H, nan_free, s, nullptr, true);
  } else if (use_mma) {
    const LayerCombine lc{reinterpret_cast<__nv_bfloat16*>(out_bf16), T, k, has_shared != 0};
    // with the side stream, the main stream stages only the routed pairs' activations
    code = run_expert_stages_mma(t, hidden, hidden_dtype == kDtypeBF16, l, T,
                                 T * k + (has_shared && !side ? T : 0), S_main, I, H, chunks_ready, nan_free, s,
                                 weight_layout, x_staged, &lc, &combined);
  } else {
    code = run_expert_stages(t, hidden, xd, l.m, l.m.y, S, I, H, ceil_div(H, kBlock), ceil_div(I, kBlock), nt, vec, s);
  }
  if (code != kOk) return code;
  if (combined) return kOk;  // the down stage combined the tokens
  if (side) MOE_CUDA(cudaStreamWaitEvent(s, side->join, 0), "join wait");  // the shared expert's rows
  // 4. combine: routed slots in top-k order, then the shared expert; one bf16 rounding
  CombineArgs c{};
  c.y = l.m.y; c.row_ptr = nullptr; c.stride = static_cast<int>(k); c.row_pairs = l.m.entry_pair;
  if (prefill) {
    c.y = nullptr;
    c.y16 = reinterpret_cast<const __nv_bfloat16*>(l.m.y);
  }
  c.pair_weight = l.m.pair_weight; c.extra_base = has_shared ? static_cast<int>(T * k) : -1;
  c.T = static_cast<int>(T); c.H = static_cast<int>(H);
  c.out_bf16 = reinterpret_cast<__nv_bfloat16*>(out_bf16);
  MOE_CUDA(launch_combine(c, s), "combine");
  stage_mark(s);
  return kOk;
}

// ---------------------------------------------------------------------------
// Expert parallelism: dispatch packing, grouped experts over received rows,
// home combine (the exchange itself is the caller's all-to-all)
// ---------------------------------------------------------------------------

// ranks up to which the dispatch workspace holds the multi-CTA bucket counts
constexpr int kEpMaxScratchRanks = 64;

int64_t moe_ep_dispatch_workspace_bytes(int64_t tokens, int64_t top_k) {
  if (tokens <= 0 || top_k <= 0) return -1;
  Plan p;
  p.take<int32_t>(tokens * top_k);
  p.take<int32_t>(tokens * top_k);
  p.take<int32_t>(tokens * top_k);
  p.take<int32_t>(bucket_scratch_ints(tokens * top_k, kEpMaxScratchRanks));
  return static_cast<int64_t>(p.used());
}

int moe_ep_dispatch_pack(const int64_t* ids, const float* weights, const uint16_t* hidden_bf16, int64_t tokens,
                         int64_t hidden_dim, int64_t top_k, int64_t num_experts, int64_t world,
                         uint16_t* send_rows, int32_t* send_expert, int32_t* send_offsets, int32_t* entry_pos,
                         float* pos_weight, void* workspace, int64_t workspace_bytes, void* stream) {
  if (!ids || !weights || !hidden_bf16 || !send_rows || !send_expert || !send_offsets || !entry_pos || !pos_weight)
    return fail(kNullPointer, "null pointer");
  if (tokens <= 0 || hidden_dim <= 0 || top_k <= 0 || world <= 0 || num_experts <= 0 || num_experts % world != 0)
    return fail(kBadDims, "bad dimensions (num_experts must be a multiple of world)");
  if (world > kMaxBuckets) return fail(kUnsupported, "world too large");
  const int64_t n = tokens * top_k;
  cudaStream_t s = as_stream(stream);
  Scratch scratch(workspace, workspace_bytes, moe_ep_dispatch_workspace_bytes(tokens, top_k), s);
  if (!scratch.ok()) return fail(kNoMemory, "workspace too small or allocation failed");
  Plan plan(scratch.base());
  int32_t* keys = plan.take<int32_t>(n);
  int32_t* pos_token = plan.take<int32_t>(n);
  int32_t* pos_entry = plan.take<int32_t>(n);
  int32_t* block_counts = plan.take<int32_t>(bucket_scratch_ints(n, kEpMaxScratchRanks));
  ep_rank_keys_kernel<<<grid_for(n), 256, 0, s>>>(ids, n, num_experts / world, world, keys);
  MOE_CUDA(cudaGetLastError(), "rank keys");
  BucketArgs ba{};
  ba.keys = keys; ba.rows = nullptr; ba.weights = weights; ba.n = static_cast<int>(n); ba.k = static_cast<int>(top_k);
  ba.key_lo = 0; ba.n_buckets = static_cast<int>(world); ba.bucket_offset = send_offsets; ba.pair_row = pos_token;
  ba.pair_weight = pos_weight; ba.pair_entry = pos_entry; ba.entry_pair = entry_pos; ba.tail = 0;
  ba.block_counts = world <= kEpMaxScratchRanks ? block_counts : nullptr;
  MOE_CUDA(launch_bucket(ba, s), "rank buckets");
  const int64_t vec = hidden_dim % 8 == 0 && aligned16(hidden_bf16) && aligned16(send_rows) ? 1 : 0;
  ep_gather_kernel<<<grid_for(n * 32, 256), 256, 0, s>>>(hidden_bf16, ids, keys, pos_token, pos_entry, n, hidden_dim,
                                                         num_experts / world, vec, send_rows, send_expert);
  MOE_CUDA(cudaGetLastError(), "gather send rows");
  return kOk;
}

int moe_ep_barrier_p2p(const uint64_t* peer_sig, int64_t world, int64_t rank, uint32_t* epoch,
                       const int32_t* payload, int64_t payload_n, const uint64_t* peer_payload, int64_t limit_us,
                       void* stream) {
  if (!peer_sig || !epoch) return fail(kNullPointer, "null pointer");
  if (world <= 0 || world > 1024 || rank < 0 || rank >= world || limit_us <= 0 || limit_us > 600000000 ||
      payload_n < 0 || payload_n > 4096)
    return fail(kBadDims, "bad dimensions");
  if ((payload == nullptr) != (peer_payload == nullptr) || (payload && payload_n == 0))
    return fail(kBadDims, "payload and peer_payload go together, with payload_n > 0");
  const int threads = static_cast<int>(ceil_div(world, 32) * 32);
  ep_barrier_kernel<<<1, threads, 0, as_stream(stream)>>>(peer_sig, static_cast<int>(world), static_cast<int>(rank),
                                                          epoch, limit_us * 1000, payload,
                                                          static_cast<int>(payload_n), peer_payload);
  MOE_CUDA(cudaGetLastError(), "ep barrier");
  return kOk;
}

int64_t moe_ep_route_dispatch_p2p_workspace_bytes(int64_t tokens, int64_t num_experts) {
  return std::max<int64_t>(1, tokens) * std::max<int64_t>(1, num_experts) * static_cast<int64_t>(sizeof(float)) + 256;
}

int moe_ep_route_dispatch_p2p(const uint16_t* hidden_bf16, const void* router_weight, int router_dtype,
                              const float* bias, int64_t tokens, int64_t hidden_dim, int64_t num_experts,
                              int64_t n_group, int64_t topk_group, int64_t top_k, float route_scale, int64_t world,
                              int64_t rank, int64_t capacity, int64_t src_stride, const uint64_t* peer_rows,
                              const uint64_t* peer_expert, const uint64_t* peer_src, const uint64_t* peer_matrix,
                              const uint64_t* peer_sig, uint32_t* epoch, int64_t limit_us, int64_t* out_ids,
                              float* out_weights_f32, void* workspace, int64_t workspace_bytes, void* stream) {
  if (!router_weight || !peer_rows || !peer_expert || !peer_src || !peer_matrix || !peer_sig || !epoch)
    return fail(kNullPointer, "null pointer");
  if (tokens > 0 && (!hidden_bf16 || !out_ids || !out_weights_f32)) return fail(kNullPointer, "null pointer");
  if (tokens < 0 || hidden_dim <= 0 || hidden_dim % 8 != 0 || world <= 0 || rank < 0 || rank >= world ||
      num_experts <= 0 || num_experts % world != 0 || capacity <= 0 || limit_us <= 0 || limit_us > 600000000 ||
      top_k <= 0 || src_stride < tokens * (top_k + 1) || capacity + tokens > INT32_MAX ||
      world * src_stride > INT32_MAX)
    return fail(kBadDims, "bad dimensions");
  if (tokens > 0) {
    int code = check_route(tokens, hidden_dim, num_experts, n_group, topk_group, top_k);
    if (code != kOk) return code;
  }
  if (tokens > kEpSendThreads / 8 || tokens * top_k > kEpSendThreads || num_experts > 256 ||
      world > kEpSendMaxRanks)
    return fail(kUnsupported, "more than 128 tokens, 1024 entries, 256 experts or 32 ranks");
  if ((reinterpret_cast<uintptr_t>(hidden_bf16) & 15u) != 0) return fail(kUnsupported, "rows must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  Scratch scratch(workspace, workspace_bytes, moe_ep_route_dispatch_p2p_workspace_bytes(tokens, num_experts), s);
  if (!scratch.ok()) return fail(kNoMemory, "workspace too small or allocation failed");
  float* logits = reinterpret_cast<float*>(scratch.base());
  if (tokens > 0) {
    // the logits as the router's own path computes them for decode sizes (route_impl)
    cudaError_t cerr = launch_router_logits_cluster(hidden_bf16, kDtypeBF16, router_weight, router_dtype, logits,
                                                    static_cast<int>(tokens), static_cast<int>(hidden_dim),
                                                    static_cast<int>(num_experts), s);
    if (cerr == cudaErrorNotSupported)
      cerr = launch_router_logits(hidden_bf16, kDtypeBF16, router_weight, router_dtype, logits,
                                  static_cast<int>(tokens), static_cast<int>(hidden_dim),
                                  static_cast<int>(num_experts), s);
    MOE_CUDA(cerr, "router logits");
  }
  EpSendArgs a{};
  a.logits = logits;
  a.bias = bias;
  a.sel.tokens = static_cast<int>(tokens);
  a.sel.experts = static_cast<int>(num_experts);
  a.sel.top_k = static_cast<int>(top_k);
  a.sel.n_group = static_cast<int>(n_group);
  a.sel.topk_group = static_cast<int>(topk_group);
  a.sel.scoring = kScoreSigmoid;
  a.sel.renorm = 1;
  a.sel.softmax_fp64 = 0;
  a.sel.round_bf16 = 1;
  a.sel.route_scale = route_scale;
  a.x = hidden_bf16;
  a.H = hidden_dim;
  a.world = static_cast<int>(world);
  a.rank = static_cast<int>(rank);
  a.n_local = static_cast<int>(num_experts / world);
  a.capacity = capacity;
  a.src_stride = src_stride;
  a.peer_rows = peer_rows; a.peer_expert = peer_expert; a.peer_src = peer_src;
  a.peer_matrix = peer_matrix; a.peer_sig = peer_sig;
  a.epoch = epoch;
  a.limit_ns = limit_us * 1000;
  a.ids64 = out_ids;
  a.weights_f32 = out_weights_f32;
  const size_t smem = static_cast<size_t>(kEpSendWarps) * 2 * std::max<int64_t>(1, num_experts) * sizeof(float);
  MOE_CUDA(cudaFuncSetAttribute(ep_send_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem)),
           "send attributes");
  ep_send_decode_kernel<<<1, kEpSendThreads, smem, s>>>(a);
  MOE_CUDA(cudaGetLastError(), "ep send");
  return kOk;
}

int moe_ep_count_ranks(const int64_t* ids, int64_t tokens, int64_t top_k, int64_t num_experts, int64_t world,
                       int32_t* counts, void* stream) {
  if (!ids || !counts) return fail(kNullPointer, "null pointer");
  if (tokens <= 0 || top_k <= 0 || world <= 0 || num_experts <= 0 || num_experts % world != 0 || world > 1024)
    return fail(kBadDims, "bad dimensions (num_experts must be a multiple of world)");
  ep_count_kernel<<<1, 256, static_cast<size_t>(world) * sizeof(int32_t), as_stream(stream)>>>(
      ids, tokens * top_k, num_experts / world, static_cast<int>(world), counts);
  MOE_CUDA(cudaGetLastError(), "count ranks");
  return kOk;
}

int moe_ep_dispatch_p2p(const int64_t* ids, const uint16_t* hidden_bf16, int64_t tokens, int64_t hidden_dim,
                        int64_t top_k, int64_t num_experts, int64_t world, int64_t rank, const int32_t* count_matrix,
                        int64_t capacity, int64_t src_stride, const uint64_t* peer_rows, const uint64_t* peer_expert,
                        const uint64_t* peer_src, void* workspace, int64_t workspace_bytes, void* stream) {
  if (!ids || !hidden_bf16 || !count_matrix || !peer_rows || !peer_expert || !peer_src)
    return fail(kNullPointer, "null pointer");
  if (tokens <= 0 || hidden_dim <= 0 || top_k <= 0 || world <= 0 || num_experts <= 0 || num_experts % world != 0 ||
      rank < 0 || rank >= world || capacity <= 0 || src_stride < tokens * top_k)
    return fail(kBadDims, "bad dimensions");
  if (world > kMaxBuckets) return fail(kUnsupported, "world too large");
  if (world * src_stride > INT32_MAX) return fail(kUnsupported, "world * src_stride must fit in int32 src codes");
  const int64_t n = tokens * top_k;
  cudaStream_t s = as_stream(stream);
  Plan sizing;
  sizing.take<int32_t>(n);
  sizing.take<int32_t>(n);
  sizing.take<int32_t>(n);
  sizing.take<int32_t>(bucket_scratch_ints(n, kEpMaxScratchRanks));
  sizing.take<int32_t>(world + 1);
  Scratch scratch(workspace, workspace_bytes, static_cast<int64_t>(sizing.used()), s);
  if (!scratch.ok()) return fail(kNoMemory, "workspace too small or allocation failed");
  Plan plan(scratch.base());
  int32_t* keys = plan.take<int32_t>(n);
  int32_t* pos_token = plan.take<int32_t>(n);
  int32_t* pos_entry = plan.take<int32_t>(n);
  int32_t* block_counts = plan.take<int32_t>(bucket_scratch_ints(n, kEpMaxScratchRanks));
  int32_t* offsets = plan.take<int32_t>(world + 1);
  ep_rank_keys_kernel<<<grid_for(n), 256, 0, s>>>(ids, n, num_experts / world, world, keys);
  MOE_CUDA(cudaGetLastError(), "rank keys");
  BucketArgs ba{};
  ba.keys = keys; ba.rows = nullptr; ba.weights = nullptr; ba.n = static_cast<int>(n); ba.k = static_cast<int>(top_k);
  ba.key_lo = 0; ba.n_buckets = static_cast<int>(world); ba.bucket_offset = offsets; ba.pair_row = pos_token;
  ba.pair_weight = nullptr; ba.pair_entry = pos_entry; ba.entry_pair = nullptr; ba.tail = 0;
  ba.block_counts = world <= kEpMaxScratchRanks ? block_counts : nullptr;
  MOE_CUDA(launch_bucket(ba, s), "rank buckets");
  const int vec = hidden_dim % 8 == 0 && aligned16(hidden_bf16) ? 1 : 0;
  ep_p2p_scatter_kernel<<<grid_for(n * 32, 256), 256, 0, s>>>(
      hidden_bf16, ids, keys, pos_token, pos_entry, offsets, count_matrix, n, hidden_dim, num_experts / world,
      static_cast<int>(world), static_cast<int>(rank), capacity, src_stride, peer_rows, peer_expert, peer_src, vec);
  MOE_CUDA(cudaGetLastError(), "scatter to peers");
  return kOk;
}

int64_t moe_ep_dispatch_p2p_workspace_bytes(int64_t tokens, int64_t top_k, int64_t world) {
  if (tokens <= 0 || top_k <= 0 || world <= 0) return -1;
  const int64_t n = tokens * top_k;
  Plan p;
  p.take<int32_t>(n);
  p.take<int32_t>(n);
  p.take<int32_t>(n);
  p.take<int32_t>(bucket_scratch_ints(n, kEpMaxScratchRanks));
  p.take<int32_t>(world + 1);
  return static_cast<int64_t>(p.used());
}

int moe_ep_return_p2p(const float* y, int64_t rows, const int32_t* recv_expert, const int32_t* recv_src,
                      int64_t hidden_dim, int64_t src_stride, int64_t world, int64_t home_rows,
                      const uint64_t* peer_yback, void* stream) {
  if (!y || !recv_expert || !recv_src || !peer_yback) return fail(kNullPointer, "null pointer");
  if (rows <= 0 || hidden_dim <= 0 || src_stride <= 0 || world <= 0 || world > kMaxBuckets || home_rows <= 0 ||
      home_rows > src_stride)
    return fail(kBadDims, "bad dimensions");
  const int vec = hidden_dim % 4 == 0 && aligned16(y) ? 1 : 0;
  ep_p2p_return_kernel<<<grid_for(rows * 32, 256), 256, 0, as_stream(stream)>>>(
      y, rows, recv_expert, recv_src, hidden_dim, src_stride, static_cast<int>(world), home_rows, peer_yback, vec);
  MOE_CUDA(cudaGetLastError(), "return to peers");
  return kOk;
}

int64_t moe_ep_experts_workspace_bytes(int64_t rows, int64_t hidden_dim, int64_t intermediate, int64_t num_local) {
  if (rows <= 0 || hidden_dim <= 0 || intermediate <= 0 || num_local <= 0) return -1;
  Plan p;
  plan_layer(p, rows, hidden_dim, intermediate, num_local, 1, 0, 8, false);
  return static_cast<int64_t>(p.used());
}

// The local experts over received rows (moe_ep_experts_fp8 and
// moe_ep_experts_return_p2p): outputs either in row order (out) or, with
// home != null, straight to their home rows.
struct EpHome {
  const int32_t* row_src;
  int64_t src_stride;
  int world;
  int64_t home_rows;  // rows of every rank's return buffer
  const uint64_t* peer_yback;
};

// Tiled weights and ~16 valid rows per expert or more (the layer's prefill
// threshold): the tcgen05 grouped GEMM.  `valid` = the rows expected to carry a
// local expert (a receive buffer sized for the worst case holds far fewer);
// 0 or more than R means all R.
static bool ep_use_gemm(int weight_layout, int64_t R, int64_t valid, int64_t H, int64_t I, int64_t S) {
  const int64_t v = valid > 0 ? std::min(valid, R) : R;
  return weight_layout == 1 && v >= kPrefillMinTokens && v >= 16 * S && prefill_supported(H, I, true) &&
         prefill_supported(I, H, false);
}

static void plan_ep_experts(Plan& p, int64_t R, int64_t H, int64_t I, int64_t S, bool home, bool gemm, LayerPlan* l,
                            uint64_t** pair_dst, float** sink) {
  LayerPlan lp = plan_layer(p, R, H, I, S, 1, 0, 8, false, home && gemm);
  uint64_t* pd = home ? p.take<uint64_t>(R) : nullptr;
  float* sk = home ? p.take<float>(H) : nullptr;  // where a row with a bad home goes
  if (l) *l = lp;
  if (pair_dst) *pair_dst = pd;
  if (sink) *sink = sk;
}

static int ep_experts(const uint16_t* rows_bf16, const int32_t* row_expert, int64_t rows, int64_t valid_rows,
                      int64_t hidden_dim,
                      int64_t intermediate, const uint64_t* tables, int64_t num_local, const uint8_t* nan_free,
                      int weight_layout, float* out, const EpHome* home, void* workspace, int64_t workspace_bytes,
                      void* stream) {
  if (!rows_bf16 || !row_expert || !tables || (!out && !home)) return fail(kNullPointer, "null pointer");
  if (weight_layout != 0 && weight_layout != 1) return fail(kBadDims, "weight_layout must be 0 or 1");
  if (weight_layout == 1 && !(g_gemv_impl == 0 && g_mma_feed == 2))
    return fail(kUnsupported, "tiled weights need the cp.async warp-MMA GEMV");
  if (rows <= 0 || hidden_dim <= 0 || intermediate <= 0 || num_local <= 0) return fail(kBadDims, "bad dimensions");
  if (num_local > kMaxBuckets) return fail(kUnsupported, "too many local experts");
  if (!mma_gemv_supported(static_cast<int>(hidden_dim), static_cast<int>(intermediate)) ||
      !mma_gemv_supported(static_cast<int>(intermediate), static_cast<int>(hidden_dim)))
    return fail(kUnsupported, "hidden and intermediate sizes must be multiples of 128");
  const int64_t H = hidden_dim, I = intermediate, S = num_local, R = rows;
  cudaStream_t s = as_stream(stream);
  const bool gemm = ep_use_gemm(weight_layout, R, valid_rows, H, I, S);
  Plan sizing;
  plan_ep_experts(sizing, R, H, I, S, home != nullptr, gemm, nullptr, nullptr, nullptr);
  Scratch scratch(workspace, workspace_bytes, sizing.used(), s);
  if (!scratch.ok()) return fail(kNoMemory, "workspace too small or allocation failed");
  Plan plan(scratch.base());
  LayerPlan l{};
  uint64_t* pair_dst = nullptr;
  float* sink = nullptr;
  plan_ep_experts(plan, R, H, I, S, home != nullptr, gemm, &l, &pair_dst, &sink);
  BucketArgs ba{};
  ba.keys = row_expert; ba.rows = nullptr; ba.weights = nullptr; ba.n = static_cast<int>(R); ba.k = 1;
  ba.key_lo = 0; ba.n_buckets = static_cast<int>(S); ba.bucket_offset = l.m.seg_offset; ba.pair_row = l.m.pair_row;
  ba.pair_weight = l.m.pair_weight; ba.pair_entry = l.m.pair_entry; ba.entry_pair = l.m.entry_pair; ba.tail = 0;
  ba.block_counts = l.bucket_scratch;
  MOE_CUDA(launch_bucket(ba, s), "expert buckets");
  const int32_t* n_pairs = l.m.seg_offset + S;  // rows routed to a local expert
  if (home) {
    ep_pair_home_kernel<<<grid_for(R), 256, 0, s>>>(l.m.pair_entry, n_pairs, home->row_src, home->src_stride,
                                                    home->world, home->home_rows, home->peer_yback, H, pair_dst, R,
                                                    sink);
    MOE_CUDA(cudaGetLastError(), "home rows");
  }
  Tables t{tables, tables + S, tables + 2 * S, tables + 3 * S, tables + 4 * S, tables + 5 * S};
  // the GEMM's down epilogue stores each row at its home
  int code = gemm ? run_expert_stages_prefill(t, rows_bf16, true, 1, false, l, R, R, S, I, H, nan_free, s, pair_dst)
                  : run_expert_stages_mma(t, rows_bf16, true, l, R, R, S, I, H, false, nan_free, s, weight_layout);
  if (code != kOk) return code;
  if (home) {
    if (!gemm) {
      const int vec = H % 4 == 0;
      ep_pairs_home_kernel<<<grid_for(R * 32, 256), 256, 0, s>>>(l.m.y, n_pairs, pair_dst, H, R, vec);
      MOE_CUDA(cudaGetLastError(), "rows home");
    }
    return kOk;
  }
  // back to row order (a row routed nowhere -- key out of range -- comes back zero)
  CombineArgs c{};
  c.y = l.m.y; c.row_ptr = nullptr; c.stride = 1; c.row_pairs = l.m.entry_pair; c.pair_weight = nullptr;
  c.extra_base = -1; c.T = static_cast<int>(R); c.H = static_cast<int>(H); c.out_f32 = out;
  MOE_CUDA(launch_combine(c, s), "row order");
  return kOk;
}

int moe_ep_experts_fp8(const uint16_t* rows_bf16, const int32_t* row_expert, int64_t rows, int64_t hidden_dim,
                       int64_t intermediate, const uint64_t* tables, int64_t num_local, const uint8_t* nan_free,
                       int weight_layout, float* out, void* workspace, int64_t workspace_bytes, void* stream) {
  if (!out) return fail(kNullPointer, "null pointer");
  return ep_experts(rows_bf16, row_expert, rows, rows, hidden_dim, intermediate, tables, num_local, nan_free,
                    weight_layout, out, nullptr, workspace, workspace_bytes, stream);
}

int64_t moe_ep_experts_return_p2p_workspace_bytes(int64_t rows, int64_t valid_rows, int64_t hidden_dim,
                                                  int64_t intermediate, int64_t num_local, int weight_layout) {
  if (rows <= 0 || hidden_dim <= 0 || intermediate <= 0 || num_local <= 0) return -1;
  Plan p;
  plan_ep_experts(p, rows, hidden_dim, intermediate, num_local, true,
                  ep_use_gemm(weight_layout, rows, valid_rows, hidden_dim, intermediate, num_local), nullptr, nullptr,
                  nullptr);
  return static_cast<int64_t>(p.used());
}

int moe_ep_experts_return_p2p(const uint16_t* rows_bf16, const int32_t* row_expert, const int32_t* row_src,
                              int64_t rows, int64_t valid_rows, int64_t hidden_dim, int64_t intermediate, const uint64_t* tables,
                              int64_t num_local, const uint8_t* nan_free, int weight_layout, int64_t src_stride,
                              int64_t world, int64_t home_rows, const uint64_t* peer_yback, void* workspace,
                              int64_t workspace_bytes, void* stream) {
  if (!row_src || !peer_yback) return fail(kNullPointer, "null pointer");
  if (src_stride <= 0 || world <= 0 || world > kMaxBuckets || home_rows <= 0 || home_rows > src_stride)
    return fail(kBadDims, "bad dimensions");
  if (hidden_dim % 4 != 0) return fail(kUnsupported, "hidden size must be a multiple of 4");
  const EpHome home{row_src, src_stride, static_cast<int>(world), home_rows, peer_yback};
  return ep_experts(rows_bf16, row_expert, rows, valid_rows, hidden_dim, intermediate, tables, num_local, nan_free,
                    weight_layout, nullptr, &home, workspace, workspace_bytes, stream);
}

int moe_ep_combine(const void* y, int y_dtype, const int32_t* entry_pos, const float* pos_weight, int64_t tokens,
                   int64_t top_k, int64_t hidden_dim, int has_shared, uint16_t* out_bf16, void* stream) {
  if (!y || !entry_pos || !pos_weight || !out_bf16) return fail(kNullPointer, "null pointer");
  if (tokens <= 0 || top_k <= 0 || hidden_dim <= 0) return fail(kBadDims, "bad dimensions");
  if (y_dtype != kDtypeBF16 && y_dtype != kDtypeF32) return fail(kUnsupported, "y_dtype must be bf16 or fp32");
  CombineArgs c{};
  if (y_dtype == kDtypeBF16) c.y16 = static_cast<const __nv_bfloat16*>(y);
  else c.y = static_cast<const float*>(y);
  c.row_ptr = nullptr; c.stride = static_cast<int>(top_k); c.row_pairs = entry_pos;
  c.pair_weight = pos_weight; c.extra_base = has_shared ? static_cast<int>(tokens * top_k) : -1;
  c.T = static_cast<int>(tokens); c.H = static_cast<int>(hidden_dim);
  c.out_bf16 = reinterpret_cast<__nv_bfloat16*>(out_bf16);
  MOE_CUDA(launch_combine(c, as_stream(stream)), "combine");
  return kOk;
}

// ---------------------------------------------------------------------------
// Stage timing
// ---------------------------------------------------------------------------

int moe_b200_stage_timing(int enable) {
  if (enable && !g_events[0]) {
    for (auto& e : g_events) MOE_CUDA(cudaEventCreate(&e), "event create");
  }
  g_timing = enable != 0;
  g_marks = 0;
  return kOk;
}

int moe_b200_fused_decode(int enable) {
  if (enable != 0 && enable != 1) return fail(kBadDims, "enable must be 0 or 1");
  g_fused_decode = enable != 0;
  return kOk;
}

int moe_b200_fused_decode_enabled(void) { return g_fused_decode ? 1 : 0; }

int moe_b200_decode_prologue(int enable) {
  if (enable != 0 && enable != 1) return fail(kBadDims, "enable must be 0 or 1");
  g_decode_prologue = enable != 0;
  return kOk;
}

int moe_b200_kb_rotate(int enable) {
  if (enable != 0 && enable != 1) return fail(kBadDims, "enable must be 0 or 1");
  g_kb_rotate = enable;
  return kOk;
}

int moe_b200_fold_epilogues(int enable) {
  if (enable != 0 && enable != 1) return fail(kBadDims, "enable must be 0 or 1");
  g_fold_epilogues = enable != 0;
  return kOk;
}

int moe_b200_router_stages_x(int enable) {
  if (enable != 0 && enable != 1) return fail(kBadDims, "enable must be 0 or 1");
  g_router_stages_x = enable != 0;
  return kOk;
}

int moe_b200_shared_side(int enable) {
  if (enable != 0 && enable != 1) return fail(kBadDims, "enable must be 0 or 1");
  g_shared_side = enable != 0;
  return kOk;
}

int moe_b200_force_ksplit(int ksplit) {
  if (ksplit < 0 || ksplit > kMaxMmaKSplit) return fail(kBadDims, "ksplit must be 0 to 8");
  g_force_ksplit = ksplit;
  return kOk;
}

int moe_b200_selected_gemv(void) { return g_gemv_impl != 0 ? g_gemv_impl : (g_mma_feed == 0 ? 3 : g_mma_feed == 1 ? 4 : 0); }

int moe_b200_select_gemv(int impl) {
  if (impl < 0 || impl > 5) return fail(kBadDims, "impl must be 0 to 5");
  g_gemv_impl = impl >= 3 ? 0 : impl;
  g_mma_feed = impl == 3 ? 0 : impl == 4 ? 1 : 2;
  return kOk;
}

int64_t moe_fp8_tiled_bytes(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0 || cols % kBlock != 0) return -1;
  return fp8_tiled_bytes(rows, cols);
}

int moe_fp8_tile_weights(const uint8_t* weight, uint8_t* tiled, int64_t rows, int64_t cols, void* stream) {
  if (!weight || !tiled) return fail(kNullPointer, "null pointer");
  if (rows <= 0 || cols <= 0 || cols % kBlock != 0) return fail(kBadDims, "cols must be a positive multiple of 128");
  if (!aligned16(weight) || !aligned16(tiled)) return fail(kUnsupported, "weights must be 16-byte aligned");
  MOE_CUDA(launch_fp8_tile(weight, tiled, rows, cols, as_stream(stream)), "tile weights");
  return kOk;
}

int moe_fp8_nan_free_flags(const uint64_t* tables, int64_t num_experts, int64_t intermediate, int64_t hidden_dim,
                           uint8_t* flags, void* stream) {
  if (!tables || !flags) return fail(kNullPointer, "null pointer");
  if (num_experts <= 0 || intermediate <= 0 || hidden_dim <= 0) return fail(kBadDims, "bad dimensions");
  MOE_CUDA(launch_nan_free_flags(tables, static_cast<int>(num_experts), intermediate, hidden_dim, flags,
                                 as_stream(stream)),
           "nan-free scan");
  return kOk;
}

int moe_b200_device_error(void* stream) {
  const int a = read_and_clear_device_error(as_stream(stream));
  const int b = read_and_clear_mma_device_error(as_stream(stream));
  const int c = read_and_clear_prefill_device_error(as_stream(stream));
  const int d = read_and_clear_ep_error(as_stream(stream));
  return (a < 0 || b < 0 || c < 0 || d < 0) ? -1 : (a | b | c | d);
}

int moe_b200_stage_times(float* ms, int max_n) {
  if (!ms) return fail(kNullPointer, "null pointer");
  if (g_marks < 2) return 0;
  MOE_CUDA(cudaEventSynchronize(g_events[g_marks - 1]), "event sync");
  const int n = std::min(max_n, g_marks - 1);
  for (int i = 0; i < n; ++i) MOE_CUDA(cudaEventElapsedTime(&ms[i], g_events[i], g_events[i + 1]), "elapsed");
  return n;
}

// ---------------------------------------------------------------------------
// Sessions
// ---------------------------------------------------------------------------

struct DsSession {
  int64_t num_layers, hidden_dim, num_experts, top_k;
  int64_t monolithic_calls = 0;
  int64_t expert_invocations = 0;
  int64_t layers_executed = 0;
  int64_t attention_invocations = 0;
  int64_t fused_attention_invocations = 0;
};

void* moe_ds_session_create(int64_t num_layers, int64_t hidden_dim, int64_t num_experts, int64_t top_k) {
  if (num_layers <= 0 || hidden_dim <= 0 || num_experts < 0 || top_k < 0) return nullptr;  // ds_forward.cpp:200-202
  DsSession* s = new (std::nothrow) DsSession();
  if (!s) return nullptr;
  s->num_layers = num_layers;
  s->hidden_dim = hidden_dim;
  s->num_experts = num_experts;
  s->top_k = top_k;
  return s;
}

void moe_ds_session_destroy(void* handle) { delete static_cast<DsSession*>(handle); }

int64_t moe_ds_monolithic_call_counter(void* h) { return h ? static_cast<DsSession*>(h)->monolithic_calls : -1; }
int64_t moe_ds_expert_invocation_count(void* h) { return h ? static_cast<DsSession*>(h)->expert_invocations : -1; }
int64_t moe_ds_layers_executed_count(void* h) { return h ? static_cast<DsSession*>(h)->layers_executed : -1; }
int64_t moe_ds_attention_invocation_count(void* h) {
  return h ? static_cast<DsSession*>(h)->attention_invocations : -1;
}
int64_t moe_ds_fused_attention_invocation_count(void* h) {
  return h ? static_cast<DsSession*>(h)->fused_attention_invocations : -1;
}

// ---------------------------------------------------------------------------
// MLA attention (mla.cu)
// ---------------------------------------------------------------------------

int64_t moe_mla_attention_workspace_bytes(int64_t num_heads, int64_t cache_len, int64_t qk_nope_dim,
                                          int64_t qk_rope_dim, int64_t kv_lora_rank, int64_t v_head_dim) {
  const MlaDims d{num_heads, cache_len, qk_nope_dim, qk_rope_dim, kv_lora_rank, v_head_dim};
  if (num_heads <= 0 || cache_len <= 0 || qk_nope_dim < 0 || qk_rope_dim < 0 || kv_lora_rank <= 0 ||
      v_head_dim <= 0 || mla_supported(d) != kOk)
    return -1;
  return mla_core_workspace_bytes(d);
}

int moe_mla_attention_flash_forward(const float* q_nope, const float* q_pe, const float* kv_cache,
                                    const float* pe_cache, const float* wkv_b, float* output_heads, int64_t num_heads,
                                    int64_t cache_len, int64_t qk_nope_dim, int64_t qk_rope_dim, int64_t kv_lora_rank,
                                    int64_t v_head_dim, float softmax_scale, void* workspace, int64_t workspace_bytes,
                                    void* stream) {
  if (!q_nope || !q_pe || !kv_cache || !pe_cache || !wkv_b || !output_heads) return 1;  // ds_forward.cpp:531-536
  if (num_heads <= 0 || cache_len <= 0 || qk_nope_dim < 0 || qk_rope_dim < 0 || kv_lora_rank <= 0 ||
      v_head_dim <= 0)
    return 2;  // :537-543
  const MlaDims d{num_heads, cache_len, qk_nope_dim, qk_rope_dim, kv_lora_rank, v_head_dim};
  int code = mla_supported(d);
  if (code != kOk) return code;
  cudaStream_t s = as_stream(stream);
  Scratch scratch(workspace, workspace_bytes, static_cast<size_t>(mla_core_workspace_bytes(d)), s);
  if (!scratch.ok()) return fail(kNoMemory, "workspace too small or allocation failed");
  return mla_core_run(d, q_nope, qk_nope_dim, q_pe, qk_rope_dim, nullptr, nullptr, kv_cache, pe_cache, wkv_b,
                      output_heads, softmax_scale, scratch.base(), s);
}

int64_t moe_ds_attention_block_workspace_bytes(int64_t hidden_dim, int64_t q_lora_rank, int64_t kv_lora_rank,
                                               int64_t num_heads, int64_t qk_nope_dim, int64_t qk_rope_dim,
                                               int64_t v_head_dim, int64_t previous_len) {
  const MlaDims d{num_heads, previous_len + 1, qk_nope_dim, qk_rope_dim, kv_lora_rank, v_head_dim};
  if (hidden_dim <= 0 || q_lora_rank <= 0 || kv_lora_rank <= 0 || num_heads <= 0 || qk_nope_dim < 0 ||
      qk_rope_dim < 0 || v_head_dim <= 0 || previous_len < 0 || mla_supported(d) != kOk)
    return -1;
  return mla_block_workspace_bytes(d, q_lora_rank);
}

int moe_ds_attention_block_forward_f32(void* handle, const float* hidden_in, const float* q_a_weight,
                                       const float* q_b_weight, const float* kv_a_weight, const float* kv_b_weight,
                                       const float* o_weight, const float* q_norm_weight, const float* kv_norm_weight,
                                       const float* previous_kv_cache, const float* previous_pe_cache,
                                       const float* rope_cos, const float* rope_sin, float* next_kv_cache,
                                       float* next_pe_cache, float* hidden_out, int64_t hidden_dim,
                                       int64_t q_lora_rank, int64_t kv_lora_rank, int64_t num_heads,
                                       int64_t qk_nope_dim, int64_t qk_rope_dim, int64_t v_head_dim,
                                       int64_t previous_len, float rms_eps, float softmax_scale, void* workspace,
                                       int64_t workspace_bytes, void* stream) {
  DsSession* session = static_cast<DsSession*>(handle);
  if (!session || !hidden_in || !q_a_weight || !q_b_weight || !kv_a_weight || !kv_b_weight || !o_weight ||
      !q_norm_weight || !kv_norm_weight || !rope_cos || !rope_sin || !next_kv_cache || !next_pe_cache ||
      !hidden_out)
    return 1;  // ds_forward.cpp:673-680
  if (hidden_dim <= 0 || q_lora_rank <= 0 || kv_lora_rank <= 0 || num_heads <= 0 || qk_nope_dim < 0 ||
      qk_rope_dim < 0 || v_head_dim <= 0 || previous_len < 0)
    return 2;  // :681-686
  if (previous_len > 0 && (!previous_kv_cache || !previous_pe_cache)) return 3;  // :687-689
  const MlaDims d{num_heads, previous_len + 1, qk_nope_dim, qk_rope_dim, kv_lora_rank, v_head_dim};
  int code = mla_supported(d);
  if (code != kOk) return code;
  // the new cache either is the previous one (append in place) or does not overlap it (copied)
  auto overlaps = [](const float* a, const float* b, int64_t n) {
    return a != b && a < b + n && b < a + n;
  };
  if (previous_len > 0 && (overlaps(next_kv_cache, previous_kv_cache, previous_len * kv_lora_rank) ||
                           overlaps(next_pe_cache, previous_pe_cache, previous_len * qk_rope_dim)))
    return fail(kBadDims, "next caches partly overlap the previous ones (equal pointers append in place)");
  cudaStream_t s = as_stream(stream);
  Scratch scratch(workspace, workspace_bytes, static_cast<size_t>(mla_block_workspace_bytes(d, q_lora_rank)), s);
  if (!scratch.ok()) return fail(kNoMemory, "workspace too small or allocation failed");
  MlaBlockArgs a{};
  a.hidden = hidden_in; a.q_a = q_a_weight; a.q_b = q_b_weight; a.kv_a = kv_a_weight; a.kv_b = kv_b_weight;
  a.o_w = o_weight; a.q_norm = q_norm_weight; a.kv_norm = kv_norm_weight;
  a.prev_kv = previous_kv_cache; a.prev_pe = previous_pe_cache; a.rope_cos = rope_cos; a.rope_sin = rope_sin;
  a.next_kv = next_kv_cache; a.next_pe = next_pe_cache; a.out = hidden_out;
  a.H = hidden_dim; a.q_rank = q_lora_rank; a.prev_len = previous_len;
  a.eps = rms_eps; a.softmax_scale = softmax_scale;
  code = mla_block_run(d, a, scratch.base(), s);
  if (code != kOk) return code;
  session->monolithic_calls += 1;  // :778-780
  session->attention_invocations += 1;
  session->fused_attention_invocations += 1;
  return 0;
}

__global__ void combine_dense_kernel(const float* outputs, const float* route, int64_t E, int64_t width, float* out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < width;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float acc = 0.0f;
    for (int64_t e = 0; e < E; ++e) acc = fmaf(route[e], outputs[e * width + i], acc);
    out[i] = acc;
  }
}

int moe_ds_moe_layer_forward_f32(void* handle, const float* expert_outputs, const float* route, int64_t E,
                                 int64_t B, int64_t H, float* out, void* stream) {
  DsSession* session = static_cast<DsSession*>(handle);
  if (!session || !expert_outputs || !route || !out) return 1;  // ds_forward.cpp:347-352
  if (E <= 0 || B <= 0 || H <= 0) return 2;                     // :353-355
  combine_dense_kernel<<<grid_for(B * H), 256, 0, as_stream(stream)>>>(expert_outputs, route, E, B * H, out);
  MOE_CUDA(cudaGetLastError(), "combine");
  session->monolithic_calls += 1;
  session->expert_invocations += E;
  return 0;
}

int moe_ds_moe_layer_forward_fp8_f32(void* handle, const uint64_t* gw, const uint64_t* gs, const uint64_t* uw,
                                     const uint64_t* us, const uint64_t* dw, const uint64_t* ds,
                                     const float* hidden, const float* route, int64_t E, int64_t B, int64_t I,
                                     int64_t H, int64_t gsc, int64_t dsc, float* out, void* workspace,
                                     int64_t workspace_bytes, void* stream) {
  DsSession* session = static_cast<DsSession*>(handle);
  if (!session || !MOE_TABLES_OK(gw, gs, uw, us, dw, ds) || !hidden || !route || !out) return 1;  // :803-809
  if (E <= 0 || B <= 0 || I <= 0 || H <= 0 || gsc <= 0 || dsc <= 0) return 2;                   // :810-815
  const int code = moe_fp8_e4m3_block_mlp_many_weighted_f32(gw, gs, uw, us, dw, ds, hidden, route, out, E, B, I, H,
                                                            gsc, dsc, workspace, workspace_bytes, stream);
  if (code != 0) return 100 + code;  // :858-860
  session->monolithic_calls += 1;
  session->expert_invocations += E;
  return 0;
}

}  // extern "C"

