// extern "C" entry points for the reference's non-FP8 expert paths
// (declared in include/moe_b200.h): Q4 dequant and Q4 MoE
// (src/pcketlm/native/q4_dequant.cpp), the row8 packer and GEMV
// (fp16_packed_gemv.cpp) and the 16-bit dense MoE (fp16_moe.cpp).
//
// Every MoE entry point runs the same pipeline: (token, expert) pairs grouped
// by expert (a dense route matrix, or router top-k bucketed by expert), a
// chunk list of <= 8 pairs per expert, gate/up + SwiGLU and down projections
// on the grouped GEMV of dense_gemv.cu, then the weighted combine in the
// reference's summation order (selected-expert order, fp32).
#include <cstring>

#include "../../include/moe_b200.h"
#include "dense_gemv.cuh"
#include "dispatch.cuh"
#include "fp8_gemv.cuh"
#include "plan.cuh"
#include "prefill_gemm.cuh"
#include "route_host.cuh"
#include "router.cuh"
#include "status.cuh"

using namespace moe;

namespace {

struct DensePlan {
  // pairs grouped by segment (expert) and their chunk list
  int32_t* seg_offset;
  int32_t* pair_row;
  float* pair_weight;
  int32_t* pair_entry;
  int32_t* row_pairs;   // combine list: pair of each (token, slot)
  int32_t* chunk_seg;
  int32_t* chunk_start;
  int32_t* chunk_len;
  int32_t* n_chunks;
  // routing (router entry points)
  int32_t* ids32;
  float* wts;
  float* logits;
  uint64_t* tables;     // [6][S] built from stacked weights
  // activations
  uint16_t* x_st;
  float* x_scale;
  uint16_t* a_st;
  float* a_scale;
  float* xf;            // fp32 copy of x (shapes the MMA kernel does not take)
  float* act;
  float* y;
  // k-split of the MMA kernel
  int ks1, ks2;
  int64_t tasks1, tasks2;
  float* partial;
  int32_t* counters;
  int64_t n_counters;
  bool mma;
  // tensor-core prefill (Q4 tiled weights): natural-order fp16 rows with
  // power-of-two scales, the pair-ordered A rows and the m-tile map
  __half* x16;
  float* x16scale;
  __half* a16;
  float* a16scale;
  __half* act16;
  float* act16scale;
  int32_t* mprefix;
  int32_t* bucket_scratch;  // multi-CTA dispatch of large batches
};

DensePlan plan_dense(Plan& p, int kind, int64_t rows_x, int64_t pairs, int64_t segments, int64_t entries,
                     int64_t H, int64_t I, int64_t router_logits, bool tables, bool prefill = false) {
  DensePlan d{};
  d.seg_offset = p.take<int32_t>(segments + 2);
  d.pair_row = p.take<int32_t>(pairs);
  d.pair_weight = p.take<float>(pairs);
  d.pair_entry = p.take<int32_t>(pairs);
  d.row_pairs = p.take<int32_t>(entries);
  const int64_t cap = chunk_capacity(pairs, segments + 1, 8);
  d.chunk_seg = p.take<int32_t>(cap);
  d.chunk_start = p.take<int32_t>(cap);
  d.chunk_len = p.take<int32_t>(cap);
  d.n_chunks = p.take<int32_t>(1);
  if (router_logits > 0) {
    d.ids32 = p.take<int32_t>(entries);
    d.wts = p.take<float>(entries);
    // above 256 tokens the router may produce up to kMaxRouterParts split-K partials
    d.logits = p.take<float>((rows_x > 256 ? kMaxRouterParts : 1) * router_logits);
  }
  if (tables) d.tables = p.take<uint64_t>(6 * segments);
  d.mma = dense_mma_supported(kind, static_cast<int>(H)) && dense_mma_supported(kind, static_cast<int>(I));
  const int planes = kind == kWBF16 ? 2 : 1;
  if (d.mma) {
    d.x_st = p.take<uint16_t>(planes * rows_x * H);
    d.x_scale = p.take<float>(rows_x);
    d.a_st = p.take<uint16_t>(planes * pairs * I);
    d.a_scale = p.take<float>(pairs);
    const int64_t chunks = std::min(pairs, cap);
    d.tasks1 = chunks * ceil_div(I, dense_task_rows(2));
    d.tasks2 = chunks * ceil_div(H, dense_task_rows(1));
    d.ks1 = dense_mma_ksplit(kind, d.tasks1, static_cast<int>(H));
    d.ks2 = dense_mma_ksplit(kind, d.tasks2, static_cast<int>(I));
    const int64_t part = std::max(d.ks1 > 1 ? d.tasks1 * d.ks1 : 0, d.ks2 > 1 ? d.tasks2 * d.ks2 : 0);
    d.partial = part > 0 ? p.take<float>(part * 32 * 8) : nullptr;
    d.n_counters = (d.ks1 > 1 ? d.tasks1 : 0) + (d.ks2 > 1 ? d.tasks2 : 0);
    d.counters = d.n_counters > 0 ? p.take<int32_t>(d.n_counters) : nullptr;
  } else {
    d.xf = p.take<float>(rows_x * H);
    d.ks1 = d.ks2 = 1;
  }
  d.act = p.take<float>(pairs * I);
  d.y = p.take<float>(pairs * H);
  if (prefill) {
    d.x16 = p.take<__half>(rows_x * H);
    d.x16scale = p.take<float>(rows_x);
    d.a16 = p.take<__half>(pairs * H);
    d.a16scale = p.take<float>(pairs);
    d.act16 = p.take<__half>(pairs * I);
    d.act16scale = p.take<float>(pairs);
    d.mprefix = p.take<int32_t>(segments + 2);
    d.bucket_scratch = p.take<int32_t>(bucket_scratch_ints(entries, static_cast<int>(segments)));
  }
  return d;
}

// Q4 shapes the tensor-core prefill GEMM takes (Q4 tiled weights: K % 64; the
// GEMM's tiles: K % 128, gate/up rows % 128, down rows % 256).
bool q4_prefill_supported(int64_t H, int64_t I) {
  return prefill_supported(H, I, true) && prefill_supported(I, H, false);
}

// Dense route matrix [T, S]: pair p = s * T + t (expert-major), weight
// route[t, s]; the combine walks token t's pairs in expert order.
__global__ void dense_route_kernel(int32_t* seg_offset, int32_t* pair_row, float* pair_weight, int32_t* row_pairs,
                                   const float* route, int64_t T, int64_t S) {
  const int64_t n = S * T;
  for (int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; p < n;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t s = p / T, t = p % T;
    pair_row[p] = static_cast<int32_t>(t);
    pair_weight[p] = route[t * S + s];
    row_pairs[t * S + s] = static_cast<int32_t>(p);
  }
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i <= S;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    seg_offset[i] = static_cast<int32_t>(i * T);
}

struct DenseTables {
  const uint64_t *gw, *gs, *uw, *us, *dw, *ds;
};

// Chunk list, gate/up + SwiGLU, down: d.y[p] = down(silu(gate x) * up x) for
// every pair p, x = row pair_row[p] of `x` (x_dtype: Dtype).
int run_dense_pipeline(int kind, const DenseTables& t, const void* x, int x_dtype, int64_t rows_x, int64_t pairs,
                       int64_t S, int64_t H, int64_t I, const DensePlan& d, cudaStream_t s) {
  ChunkArgs ca{d.seg_offset, static_cast<int>(S), 8, d.chunk_seg, d.chunk_start, d.chunk_len, d.n_chunks};
  MOE_CUDA(launch_chunks(ca, s), "chunk list");
  DenseArgs g1{};
  g1.w0 = t.gw; g1.s0 = t.gs; g1.w1 = t.uw; g1.s1 = t.us;
  g1.pair_row = d.pair_row;
  g1.chunk_seg = d.chunk_seg; g1.chunk_start = d.chunk_start; g1.chunk_len = d.chunk_len; g1.n_chunks = d.n_chunks;
  g1.out0 = d.act; g1.N = static_cast<int>(I); g1.K = static_cast<int>(H);
  DenseArgs g2 = g1;
  g2.w0 = t.dw; g2.s0 = t.ds; g2.w1 = nullptr; g2.s1 = nullptr;
  g2.pair_row = nullptr; g2.out0 = d.y; g2.N = static_cast<int>(H); g2.K = static_cast<int>(I);
  const int mode = stage_mode_for(kind);
  if (d.mma) {
    // the inputs convert exactly or with the reference's own rounding (to
    // fp16 for Q4): no row scaling; the fp32 activations are scaled
    MOE_CUDA(launch_stage_rows(x, x_dtype, static_cast<int>(rows_x), static_cast<int>(H), nullptr, mode, false,
                               d.x_st, d.x_scale, rows_x * H, d.counters, d.n_counters, s),
             "stage hidden");
    g1.xs = d.x_st; g1.xscale = d.x_scale; g1.plane = rows_x * H;
    g1.ksplit = d.ks1; g1.partial = d.partial; g1.counters = d.counters;
    MOE_CUDA(launch_dense_mma_gemv(g1, kind, 2, kEpiSwiglu, d.tasks1, s), "gate/up stage");
    MOE_CUDA(launch_stage_rows(d.act, kDtypeF32, static_cast<int>(pairs), static_cast<int>(I), nullptr, mode, true,
                               d.a_st, d.a_scale, pairs * I, nullptr, 0, s),
             "stage activations");
    g2.xs = d.a_st; g2.xscale = d.a_scale; g2.plane = pairs * I;
    g2.ksplit = d.ks2; g2.partial = d.partial;
    g2.counters = d.counters ? d.counters + (d.ks1 > 1 ? d.tasks1 : 0) : nullptr;
    MOE_CUDA(launch_dense_mma_gemv(g2, kind, 1, kEpiStore, d.tasks2, s), "down stage");
  } else {
    MOE_CUDA(launch_to_f32(x, x_dtype, rows_x * H, d.xf, s), "hidden to fp32");
    g1.x = d.xf;
    MOE_CUDA(launch_dense_generic_gemv(g1, kind, 2, kEpiSwiglu, pairs, s), "gate/up stage");
    g2.x = d.act;
    MOE_CUDA(launch_dense_generic_gemv(g2, kind, 1, kEpiStore, pairs, s), "down stage");
  }
  return kOk;
}

// out[t] = sum over token t's slots of weight * y[pair], in slot order.
int dense_combine(const DensePlan& d, int64_t T, int64_t H, int64_t slots, void* out, int out_dtype,
                  bool bf16_via_f16, cudaStream_t s) {
  CombineArgs c{};
  c.y = d.y; c.row_ptr = nullptr; c.stride = static_cast<int>(slots); c.row_pairs = d.row_pairs;
  c.pair_weight = d.pair_weight; c.extra_base = -1; c.T = static_cast<int>(T); c.H = static_cast<int>(H);
  if (out_dtype == kDtypeF16) c.out_f16 = static_cast<__half*>(out);
  else if (out_dtype == kDtypeBF16) c.out_bf16 = static_cast<__nv_bfloat16*>(out);
  else c.out_f32 = static_cast<float*>(out);
  c.bf16_via_f16 = bf16_via_f16 ? 1 : 0;
  MOE_CUDA(launch_combine(c, s), "combine");
  return kOk;
}

// Bucket router picks (token, slot) by expert: pairs, weights, combine list.
int bucket_routes(const DensePlan& d, int64_t T, int64_t k, int64_t E, cudaStream_t s) {
  BucketArgs ba{};
  ba.keys = d.ids32; ba.rows = nullptr; ba.weights = d.wts; ba.n = static_cast<int>(T * k);
  ba.k = static_cast<int>(k); ba.key_lo = 0; ba.n_buckets = static_cast<int>(E);
  ba.bucket_offset = d.seg_offset; ba.pair_row = d.pair_row; ba.pair_weight = d.pair_weight;
  ba.pair_entry = d.pair_entry; ba.entry_pair = d.row_pairs; ba.tail = 0;
  ba.block_counts = d.bucket_scratch;
  MOE_CUDA(launch_bucket(ba, s), "dispatch");
  return kOk;
}

int u16_dtype(int dtype_code) { return dtype_code == 1 ? kDtypeBF16 : kDtypeF16; }

size_t selected_need(int kind, int64_t T, int64_t H, int64_t S, int64_t I) {
  Plan p;
  plan_dense(p, kind, T, S * T, S, S * T, H, I, 0, kind != kWQ4);
  return p.used();
}

int selected_forward(int kind, const DenseTables* given, const void* gate, const void* up, const void* down,
                     const void* hidden, int x_dtype, const float* route, void* out, int out_dtype, int64_t T,
                     int64_t H, int64_t S, int64_t I, void* workspace, int64_t workspace_bytes, cudaStream_t s) {
  Plan sizing;
  plan_dense(sizing, kind, T, S * T, S, S * T, H, I, 0, given == nullptr);
  Scratch scratch(workspace, workspace_bytes, sizing.used(), s);
  if (!scratch.ok()) return fail(kNoMemory, "workspace too small or allocation failed");
  Plan plan(scratch.base());
  const DensePlan d = plan_dense(plan, kind, T, S * T, S, S * T, H, I, 0, given == nullptr);
  DenseTables t{};
  if (given) {
    t = *given;
  } else {
    const int64_t gate_bytes = I * H * 2, down_bytes = H * I * 2;
    MOE_CUDA(launch_fill_table(d.tables, gate, gate_bytes, static_cast<int>(S), s), "tables");
    MOE_CUDA(launch_fill_table(d.tables + 2 * S, up, gate_bytes, static_cast<int>(S), s), "tables");
    MOE_CUDA(launch_fill_table(d.tables + 4 * S, down, down_bytes, static_cast<int>(S), s), "tables");
    t = DenseTables{d.tables, nullptr, d.tables + 2 * S, nullptr, d.tables + 4 * S, nullptr};
  }
  dense_route_kernel<<<grid_for(S * T), 256, 0, s>>>(d.seg_offset, d.pair_row, d.pair_weight, d.row_pairs, route, T, S);
  MOE_CUDA(cudaGetLastError(), "dense route");
  const int code = run_dense_pipeline(kind, t, hidden, x_dtype, T, S * T, S, H, I, d, s);
  if (code != kOk) return code;
  return dense_combine(d, T, H, S, out, out_dtype, false, s);
}

size_t routed_need(int kind, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k, bool tables,
                   bool prefill = false) {
  Plan p;
  plan_dense(p, kind, T, T * k, E, T * k, H, I, T * E, tables, prefill);
  return p.used();
}

// The Q4 expert stages on the tcgen05 grouped GEMM (prefill_gemm.cu, int4
// weights in the Q4 tiled layout): stage x as fp16 rows, gather the pairs'
// rows, gate/up + SwiGLU, stage the activations, down.  d.y gets every
// pair's output as the GEMV path leaves it.
int run_q4_prefill(const DenseTables& t, const void* x, int x_dtype, int64_t T, int64_t pairs, int64_t E, int64_t H,
                   int64_t I, const DensePlan& d, cudaStream_t s) {
  // each token's row staged once and written to its pairs' rows
  const cudaError_t serr = launch_scatter_rows(x, x_dtype, T, H, d.row_pairs, static_cast<int>(pairs / T), nullptr,
                                               d.a16, d.a16scale, s);
  if (serr == cudaErrorNotSupported) {
    if (x_dtype == kDtypeF16)
      MOE_CUDA(launch_f16_rows_to_f16(x, static_cast<int>(T), static_cast<int>(H), d.x16, d.x16scale, s), "stage x");
    else
      MOE_CUDA(launch_rows_to_f16(x, true, static_cast<int>(T), static_cast<int>(H), nullptr, d.x16, d.x16scale,
                                  nullptr, 0, s),
               "stage x");
    MOE_CUDA(launch_gather_rows(d.x16, d.x16scale, d.pair_row, pairs, H, d.a16, d.a16scale, s), "gather pairs");
  } else {
    MOE_CUDA(serr, "stage pairs");
  }
  MOE_CUDA(launch_prefill_tiles(d.seg_offset, static_cast<int>(E), d.mprefix, s), "tile map");
  const int64_t mtiles_bound = pairs / 128 + E;
  PrefillArgs g1{};
  g1.w0 = t.gw; g1.s0 = t.gs; g1.w1 = t.uw; g1.s1 = t.us;
  g1.a16 = d.a16; g1.ascale = d.a16scale; g1.rows_a = pairs;
  g1.seg_offset = d.seg_offset; g1.mprefix = d.mprefix; g1.n_segments = static_cast<int>(E);
  g1.out = d.act; g1.N = static_cast<int>(I); g1.K = static_cast<int>(H);
  g1.scale_cols = 0; g1.nanfix = 0; g1.nan_free = nullptr; g1.wformat = kPrefillQ4Row;
  MOE_CUDA(launch_prefill_gemm(g1, true, mtiles_bound * (I / 128), s), "gate/up GEMM");
  MOE_CUDA(launch_rows_to_f16(d.act, false, static_cast<int>(pairs), static_cast<int>(I), nullptr, d.act16,
                              d.act16scale, nullptr, 0, s),
           "stage activations");
  PrefillArgs g2 = g1;
  g2.w0 = t.dw; g2.s0 = t.ds; g2.w1 = nullptr; g2.s1 = nullptr;
  g2.a16 = d.act16; g2.ascale = d.act16scale;
  g2.out = d.y; g2.N = static_cast<int>(H); g2.K = static_cast<int>(I);
  MOE_CUDA(launch_prefill_gemm(g2, false, mtiles_bound * (H / 256), s), "down GEMM");
  return kOk;
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------------------
// Q4
// ---------------------------------------------------------------------------
int moe_q4_dequant_to_fp16(const uint8_t* packed, const uint16_t* scales, uint16_t* out, int64_t num_channels,
                           int64_t channel_size, void* stream) {
  if (!packed || !scales || !out) return fail(1, "null pointer");
  if (num_channels <= 0 || channel_size <= 0) return fail(2, "bad dimensions");
  MOE_CUDA(launch_q4_dequant(packed, scales, out, num_channels, channel_size, as_stream(stream)), "q4 dequant");
  return kOk;
}

int moe_q4_dequant_many_to_fp16(const uint8_t* const* packed, const uint16_t* const* scales, uint16_t* const* out,
                                const int64_t* num_channels, const int64_t* channel_sizes, int64_t count,
                                void* stream) {
  if (!packed || !scales || !out || !num_channels || !channel_sizes) return fail(1, "null pointer");  // :218-223
  if (count <= 0) return fail(2, "tensor_count <= 0");                                                 // :224-226
  for (int64_t i = 0; i < count; ++i) {
    if (!packed[i] || !scales[i] || !out[i] || num_channels[i] <= 0 || channel_sizes[i] <= 0) continue;
    MOE_CUDA(launch_q4_dequant(packed[i], scales[i], out[i], num_channels[i], channel_sizes[i], as_stream(stream)),
             "q4 dequant");
  }
  return kOk;
}

int64_t moe_q4_moe_selected_workspace_bytes(int64_t hidden_size, int64_t intermediate_size, int64_t selected) {
  if (hidden_size <= 0 || intermediate_size <= 0 || selected <= 0) return -1;
  return static_cast<int64_t>(selected_need(kWQ4, 1, hidden_size, selected, intermediate_size));
}

int moe_q4_moe_selected_forward_u16(const uint16_t* hidden, const uint64_t* gate_packed, const uint64_t* gate_scales,
                                    const uint64_t* up_packed, const uint64_t* up_scales,
                                    const uint64_t* down_packed, const uint64_t* down_scales,
                                    const float* route_weights, uint16_t* out_fp16, int64_t hidden_size,
                                    int64_t intermediate_size, int64_t selected_count, void* workspace,
                                    int64_t workspace_bytes, void* stream) {
  // q4_dequant.cpp:370-378: one code for null pointers and bad sizes
  if (!hidden || !gate_packed || !gate_scales || !up_packed || !up_scales || !down_packed || !down_scales ||
      !route_weights || !out_fp16 || hidden_size <= 0 || intermediate_size <= 0 || selected_count <= 0)
    return fail(1, "null pointer or bad dimensions");
  const DenseTables t{gate_packed, gate_scales, up_packed, up_scales, down_packed, down_scales};
  return selected_forward(kWQ4, &t, nullptr, nullptr, nullptr, hidden, kDtypeF16, route_weights, out_fp16,
                          kDtypeF16, 1, hidden_size, selected_count, intermediate_size, workspace, workspace_bytes,
                          as_stream(stream));
}

int64_t moe_q4_moe_layer_workspace_bytes(int64_t tokens, int64_t hidden_size, int64_t intermediate_size,
                                         int64_t num_experts, int64_t top_k) {
  if (tokens <= 0 || hidden_size <= 0 || intermediate_size <= 0 || num_experts <= 0 || top_k <= 0) return -1;
  // room for the tensor-core path too (weight_layout 1) where the shapes allow it
  return static_cast<int64_t>(routed_need(kWQ4, tokens, hidden_size, intermediate_size, num_experts, top_k, false,
                                          q4_prefill_supported(hidden_size, intermediate_size)));
}

int moe_q4_moe_layer_u16(const void* hidden, int hidden_dtype, int64_t tokens, int64_t hidden_size,
                         int64_t intermediate_size, const void* router_weight, int router_dtype, int64_t num_experts,
                         int64_t top_k, const uint64_t* tables, int weight_layout, void* out, int64_t* out_ids,
                         float* out_weights, void* workspace, int64_t workspace_bytes, void* stream) {
  if (!hidden || !router_weight || !tables || !out) return fail(kNullPointer, "null pointer");
  if (hidden_dtype != kDtypeBF16 && hidden_dtype != kDtypeF16) return fail(kUnsupported, "hidden must be bf16 or fp16");
  if (weight_layout != 0 && weight_layout != 1) return fail(kBadDims, "weight_layout must be 0 or 1");
  if (weight_layout == 1 && !q4_prefill_supported(hidden_size, intermediate_size))
    return fail(kUnsupported, "Q4 tiled weights need hidden % 256 == 0 and intermediate % 128 == 0");
  int code = check_route(tokens, hidden_size, num_experts, 1, 1, top_k);
  if (code != kOk) return code;
  if (intermediate_size <= 0) return fail(kBadDims, "bad dimensions");
  if (num_experts > kMaxBuckets) return fail(kUnsupported, "too many experts");
  const int64_t T = tokens, H = hidden_size, I = intermediate_size, E = num_experts, k = top_k;
  cudaStream_t s = as_stream(stream);
  const bool prefill = q4_prefill_supported(H, I);
  Scratch scratch(workspace, workspace_bytes, routed_need(kWQ4, T, H, I, E, k, false, prefill), s);
  if (!scratch.ok()) return fail(kNoMemory, "workspace too small or allocation failed");
  Plan plan(scratch.base());
  const DensePlan d = plan_dense(plan, kWQ4, T, T * k, E, T * k, H, I, T * E, false, prefill);
  // softmax over fp32 logits, top-k, renormalised (layer_bridge.py:2682-2689)
  code = route_impl(hidden, hidden_dtype, router_weight, router_dtype, nullptr, T, H, E, 1, 1, k, kScoreSoftmax, 1,
                    0, 1.0f, 0, out_ids, d.ids32, d.wts, nullptr, d.logits, s);
  if (code != kOk) return code;
  if (out_weights) MOE_CUDA(cudaMemcpyAsync(out_weights, d.wts, T * k * sizeof(float), cudaMemcpyDeviceToDevice, s),
                            "weights out");
  code = bucket_routes(d, T, k, E, s);
  if (code != kOk) return code;
  const DenseTables t{tables, tables + E, tables + 2 * E, tables + 3 * E, tables + 4 * E, tables + 5 * E};
  code = weight_layout == 1 ? run_q4_prefill(t, hidden, hidden_dtype, T, T * k, E, H, I, d, s)
                            : run_dense_pipeline(kWQ4, t, hidden, hidden_dtype, T, T * k, E, H, I, d, s);
  if (code != kOk) return code;
  // q4_moe_selected_forward_u16 returns fp16 per token; a bf16 caller gets that value as bf16
  return dense_combine(d, T, H, k, out, hidden_dtype, hidden_dtype == kDtypeBF16, s);
}

int64_t moe_q4_tiled_bytes(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0 || cols % 64 != 0) return -1;
  return q4_tiled_bytes(rows, cols);
}

int moe_q4_tile_weights(const uint8_t* packed, uint8_t* tiled, int64_t rows, int64_t cols, void* stream) {
  if (!packed || !tiled) return fail(kNullPointer, "null pointer");
  if (rows <= 0 || cols <= 0 || cols % 64 != 0) return fail(kBadDims, "cols must be a positive multiple of 64");
  MOE_CUDA(launch_q4_tile(packed, tiled, rows, cols, as_stream(stream)), "q4 tile");
  return kOk;
}

// ---------------------------------------------------------------------------
// row8
// ---------------------------------------------------------------------------
int moe_pack_u16_rows8(const uint16_t* weight, uint16_t* packed, int64_t rows, int64_t cols, void* stream) {
  if (!weight || !packed) return fail(1, "null pointer");  // fp16_packed_gemv.cpp:58-60
  if (rows < 0 || cols < 0) return fail(2, "bad dimensions");  // :61-63
  MOE_CUDA(launch_pack_rows8(weight, packed, rows, cols, as_stream(stream)), "pack rows8");
  return kOk;
}

int moe_packed_gemv_rows8(const uint16_t* hidden, const uint16_t* packed, float* out, int64_t rows, int64_t cols,
                          int dtype_code, void* stream) {
  if (!hidden || !packed || !out) return fail(1, "null pointer");  // :87-89
  if (rows < 0 || cols < 0 || (dtype_code != 0 && dtype_code != 1)) return fail(2, "bad dimensions or dtype");
  if (rows == 0) return kOk;
  if (cols == 0) {
    MOE_CUDA(cudaMemsetAsync(out, 0, rows * sizeof(float), as_stream(stream)), "zero output");
    return kOk;
  }
  MOE_CUDA(launch_rows8_gemv(hidden, packed, out, rows, cols, u16_dtype(dtype_code), as_stream(stream)),
           "rows8 gemv");
  return kOk;
}

// ---------------------------------------------------------------------------
// 16-bit dense MoE
// ---------------------------------------------------------------------------
int64_t moe_moe_selected_forward_workspace_bytes(int64_t seq_len, int64_t hidden_size, int64_t selected_count,
                                                 int64_t intermediate_size, int dtype_code) {
  if (seq_len <= 0 || hidden_size <= 0 || selected_count <= 0 || intermediate_size <= 0) return -1;
  return static_cast<int64_t>(selected_need(dtype_code == 1 ? kWBF16 : kWF16, seq_len, hidden_size, selected_count,
                                            intermediate_size));
}

int moe_moe_selected_forward_u16(const uint16_t* hidden, const uint16_t* gate_weight, const uint16_t* up_weight,
                                 const uint16_t* down_weight, const float* route_weights, uint16_t* out,
                                 int64_t seq_len, int64_t hidden_size, int64_t selected_count,
                                 int64_t intermediate_size, int dtype_code, void* workspace, int64_t workspace_bytes,
                                 void* stream) {
  if (!hidden || !gate_weight || !up_weight || !down_weight || !route_weights || !out)
    return fail(1, "null pointer");  // fp16_moe.cpp:213-218
  if (seq_len <= 0 || hidden_size <= 0 || selected_count <= 0 || intermediate_size <= 0)
    return fail(2, "bad dimensions");  // :219-221
  if (dtype_code != 0 && dtype_code != 1) return fail(3, "dtype_code must be 0 (fp16) or 1 (bf16)");  // :222-224
  const int kind = dtype_code == 1 ? kWBF16 : kWF16;
  const int dt = u16_dtype(dtype_code);
  return selected_forward(kind, nullptr, gate_weight, up_weight, down_weight, hidden, dt, route_weights, out, dt,
                          seq_len, hidden_size, selected_count, intermediate_size, workspace, workspace_bytes,
                          as_stream(stream));
}

int64_t moe_moe_forward_fp16_workspace_bytes(int64_t seq_len, int64_t hidden_size, int64_t num_experts,
                                             int64_t top_k, int64_t intermediate_size) {
  if (seq_len <= 0 || hidden_size <= 0 || num_experts <= 0 || top_k <= 0 || intermediate_size <= 0) return -1;
  return static_cast<int64_t>(
      routed_need(kWF16, seq_len, hidden_size, intermediate_size, num_experts, top_k, true));
}

int moe_moe_forward_fp16(const uint16_t* hidden, const uint16_t* router_weight, const uint16_t* gate_weight,
                         const uint16_t* up_weight, const uint16_t* down_weight, uint16_t* out,
                         int64_t* selected_experts, float* selected_weights, int64_t seq_len, int64_t hidden_size,
                         int64_t num_experts, int64_t top_k, int64_t intermediate_size, int normalize_topk,
                         void* workspace, int64_t workspace_bytes, void* stream) {
  if (!hidden || !router_weight || !gate_weight || !up_weight || !down_weight || !out)
    return fail(1, "null pointer");  // fp16_moe.cpp:106-111
  if (seq_len <= 0 || hidden_size <= 0 || num_experts <= 0 || top_k <= 0 || intermediate_size <= 0)
    return fail(2, "bad dimensions");  // :112-114
  if (top_k > num_experts) return fail(3, "top_k > num_experts");  // :115-117
  if (top_k > 32 || num_experts > kMaxBuckets) return fail(kUnsupported, "top_k > 32 or too many experts");
  const int64_t T = seq_len, H = hidden_size, I = intermediate_size, E = num_experts, k = top_k;
  cudaStream_t s = as_stream(stream);
  Scratch scratch(workspace, workspace_bytes, routed_need(kWF16, T, H, I, E, k, true), s);
  if (!scratch.ok()) return fail(kNoMemory, "workspace too small or allocation failed");
  Plan plan(scratch.base());
  const DensePlan d = plan_dense(plan, kWF16, T, T * k, E, T * k, H, I, T * E, true);
  // softmax with an fp32 denominator, top-k (ties to the lower id), optional renorm (:129-165)
  int code = route_impl(hidden, kDtypeF16, router_weight, kDtypeF16, nullptr, T, H, E, 1, 1, k, kScoreSoftmax,
                        normalize_topk ? 1 : 0, 0, 1.0f, 0, selected_experts, d.ids32, d.wts, nullptr, d.logits, s);
  if (code != kOk) return code;
  if (selected_weights)
    MOE_CUDA(cudaMemcpyAsync(selected_weights, d.wts, T * k * sizeof(float), cudaMemcpyDeviceToDevice, s),
             "weights out");
  code = bucket_routes(d, T, k, E, s);
  if (code != kOk) return code;
  const int64_t gate_bytes = I * H * 2, down_bytes = H * I * 2;
  MOE_CUDA(launch_fill_table(d.tables, gate_weight, gate_bytes, static_cast<int>(E), s), "tables");
  MOE_CUDA(launch_fill_table(d.tables + 2 * E, up_weight, gate_bytes, static_cast<int>(E), s), "tables");
  MOE_CUDA(launch_fill_table(d.tables + 4 * E, down_weight, down_bytes, static_cast<int>(E), s), "tables");
  const DenseTables t{d.tables, nullptr, d.tables + 2 * E, nullptr, d.tables + 4 * E, nullptr};
  code = run_dense_pipeline(kWF16, t, hidden, kDtypeF16, T, T * k, E, H, I, d, s);
  if (code != kOk) return code;
  return dense_combine(d, T, H, k, out, kDtypeF16, false, s);
}

}  // extern "C"
