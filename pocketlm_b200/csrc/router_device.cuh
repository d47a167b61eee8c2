// Device-side router selection, shared by the router kernels (router.cu) and
// the fused small-batch route + dispatch kernel (dispatch.cu).
#pragma once
#include "common.cuh"
#include "router.cuh"

namespace moe {

MOE_D float to_float_any(float v) { return v; }
MOE_D float to_float_any(__nv_bfloat16 v) { return __bfloat162float(v); }
MOE_D float to_float_any(__half v) { return __half2float(v); }

constexpr int kSelectWarps = 4;

// Selection for token t by one warp.  The logits are the sum of `nparts`
// partial rows spaced `part_stride` floats apart (1 part: a plain [T, E]
// logits matrix).  probs/choice: per-warp shared scratch of E floats each.
static __device__ void select_token(const float* __restrict__ logits, int nparts, int64_t part_stride,
                             const float* __restrict__ bias, const RouterSelectParams& p, int t, float* probs,
                             float* choice, int64_t* __restrict__ ids64, int32_t* __restrict__ ids32,
                             float* __restrict__ weights_f32, __nv_bfloat16* __restrict__ weights_bf16) {
  const int lane = threadIdx.x % kWarp;
  const int E = p.experts;
  const float* row = logits + static_cast<int64_t>(t) * E;
  for (int e = lane; e < E; e += kWarp) {
    float v = row[e];
    for (int q = 1; q < nparts; ++q) v += row[q * part_stride + e];
    choice[e] = v;  // raw logits for now
  }
  __syncwarp();

  // scores: sigmoid, or softmax (max-subtracted)
  if (p.scoring == kScoreSigmoid) {
    for (int e = lane; e < E; e += kWarp) probs[e] = 1.0f / (1.0f + expf(-choice[e]));
  } else {
    float m = -INFINITY;
    for (int e = lane; e < E; e += kWarp) m = fmaxf(m, choice[e]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    for (int e = lane; e < E; e += kWarp) probs[e] = expf(choice[e] - m);
    __syncwarp();
    if (p.softmax_fp64) {
      // ds_router_topk_u16: fp64 denominator, summed in expert order
      // (ds_forward.cpp:913-924)
      double denom = 0.0;
      if (lane == 0)
        for (int e = 0; e < E; ++e) denom += static_cast<double>(probs[e]);
      denom = __shfl_sync(0xFFFFFFFFu, denom, 0);
      for (int e = lane; e < E; e += kWarp) probs[e] = static_cast<float>(static_cast<double>(probs[e]) / denom);
    } else {
      float s = 0.0f;
      for (int e = lane; e < E; e += kWarp) s += probs[e];
      s = warp_sum(s);
      for (int e = lane; e < E; e += kWarp) probs[e] = probs[e] / s;
    }
  }
  __syncwarp();
  for (int e = lane; e < E; e += kWarp) choice[e] = bias ? probs[e] + bias[e] : probs[e];
  __syncwarp();
  // group-limited selection (fp8_source.py:5125-5140)
  if (p.n_group > 1) {
    const int G = E / p.n_group;
    float gscore = -INFINITY;
    if (lane < p.n_group) {
      float best = -INFINITY, second = -INFINITY;
      for (int i = 0; i < G; ++i) {
        const float v = choice[lane * G + i];
        if (v > best) {
          second = best;
          best = v;
        } else if (v > second) {
          second = v;
        }
      }
      gscore = bias ? best + second : best;
    }
    uint32_t keep = 0;
    const int kg = max(1, min(p.topk_group, p.n_group));
    for (int j = 0; j < kg; ++j) {
      float v = (keep >> lane) & 1u ? -INFINITY : gscore;
      int idx = lane < p.n_group ? lane : 0x7FFFFFFF;
      if ((keep >> lane) & 1u) idx = 0x7FFFFFFF;
      warp_argmax(v, idx);
      if (idx < kWarp) keep |= 1u << idx;
    }
    for (int e = lane; e < E; e += kWarp)
      if (!((keep >> (e / G)) & 1u)) choice[e] = -INFINITY;
    __syncwarp();
  }

  // top-k, ties to the lower expert id
  const int k = p.top_k;
  int my_id = -1;      // lane j < k holds the j-th pick
  float my_prob = 0.0f;
  for (int j = 0; j < k; ++j) {
    float v = -INFINITY;
    int idx = 0x7FFFFFFF;
    for (int e = lane; e < E; e += kWarp) {
      const float c = choice[e];
      if (c > v || (c == v && e < idx)) {
        v = c;
        idx = e;
      }
    }
    warp_argmax(v, idx);
    if (idx == 0x7FFFFFFF) idx = 0;  // every remaining score is -inf / NaN
    if (lane == j) {
      my_id = idx;
      my_prob = probs[idx];
    }
    __syncwarp();
    // a picked expert becomes NaN: every comparison with it is false, so it
    // is never picked again even when the remaining scores are all -inf
    if (lane == 0) choice[idx] = __int_as_float(0x7FC00000);
    __syncwarp();
  }

  float w = my_prob;
  if (p.renorm) {
    if (p.softmax_fp64) {
      double s = 0.0;
      for (int j = 0; j < k; ++j) s += static_cast<double>(__shfl_sync(0xFFFFFFFFu, my_prob, j));
      w = static_cast<float>(static_cast<double>(my_prob) / s);
    } else {
      float s = 0.0f;
      for (int j = 0; j < k; ++j) s += __shfl_sync(0xFFFFFFFFu, my_prob, j);
      w = my_prob / fmaxf(s, 1e-12f);
    }
  }
  w = w * p.route_scale;
  if (lane < k) {
    const int64_t o = static_cast<int64_t>(t) * k + lane;
    if (p.round_bf16) w = __bfloat162float(__float2bfloat16_rn(w));
    if (ids64) ids64[o] = my_id;
    if (ids32) ids32[o] = my_id;
    if (weights_f32) weights_f32[o] = w;
    if (weights_bf16) weights_bf16[o] = __float2bfloat16_rn(w);
  }
}


}  // namespace moe
