// Router kernels: fp32 router logits and top-k expert selection.
//
// Replaces the router math of run_fp8_router
// (src/pcketlm/core/runtime/fp8_source.py:1522-1547) with its group mask
// _mask_deepseek_route_groups (fp8_source.py:5125-5140), the native softmax
// router ds_router_topk_u16 (src/pcketlm/native/ds_forward.cpp:879-955) and
// the Mixtral softmax top-k (core/runtime/layer_bridge.py:2682-2689).
//
// Logits are dot products in fp32 of the hidden state with each router row
// (the reference computes F.linear(x.float(), W.float())); only the
// summation order differs, so selections agree except at score ties.
#include "common.cuh"
#include "router.cuh"
#include "router_device.cuh"

#include <cooperative_groups.h>

#include <algorithm>
#include <type_traits>

namespace moe {


template <typename T>
MOE_D void load8(const T* p, float* out);

template <>
MOE_D void load8<float>(const float* p, float* out) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
  out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
}

template <>
MOE_D void load8<__nv_bfloat16>(const __nv_bfloat16* p, float* out) {
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = __uint_as_float(w[i] << 16);
    out[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

template <>
MOE_D void load8<__half>(const __half* p, float* out) {
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}


// ---------------------------------------------------------------------------
// Logits, small token counts: one CTA per pair of experts, 4 warps per expert
// each summing a quarter of the hidden dimension.  The router weight streams
// from HBM once; the activations are re-read from L1/L2.
// ---------------------------------------------------------------------------
constexpr int kGemvExpertsPerCta = 2;
constexpr int kGemvSplit = 4;
constexpr int kGemvTokens = 8;

template <typename XT, typename WT>
__global__ void __launch_bounds__(256) router_logits_gemv_kernel(
    const XT* __restrict__ x, const WT* __restrict__ w, float* __restrict__ logits,
    int tokens, int hidden, int experts, int vec_ok) {
  __shared__ float partial[kGemvExpertsPerCta][kGemvSplit][kGemvTokens];
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int local_e = warp / kGemvSplit, part = warp % kGemvSplit;
  const int e = blockIdx.x * kGemvExpertsPerCta + local_e;
  const int per_part = static_cast<int>(ceil_div(ceil_div(hidden, 8), kGemvSplit)) * 8;
  const int k_lo = part * per_part;
  const int k_hi = min(hidden, k_lo + per_part);
  for (int t0 = 0; t0 < tokens; t0 += kGemvTokens) {
    const int nt = min(kGemvTokens, tokens - t0);
    float acc[kGemvTokens];
#pragma unroll
    for (int t = 0; t < kGemvTokens; ++t) acc[t] = 0.0f;
    if (e < experts) {
      const WT* wrow = w + static_cast<int64_t>(e) * hidden;
      if (vec_ok) {
        for (int k = k_lo + lane * 8; k < k_hi; k += kWarp * 8) {
          float wv[8];
          load8<WT>(wrow + k, wv);
#pragma unroll
          for (int t = 0; t < kGemvTokens; ++t) {
            if (t < nt) {
              float xv[8];
              load8<XT>(x + static_cast<int64_t>(t0 + t) * hidden + k, xv);
#pragma unroll
              for (int i = 0; i < 8; ++i) acc[t] = fmaf(xv[i], wv[i], acc[t]);
            }
          }
        }
      } else {
        for (int k = k_lo + lane; k < k_hi; k += kWarp) {
          const float wv = to_float_any(wrow[k]);
          for (int t = 0; t < nt; ++t) {
            acc[t] = fmaf(to_float_any(x[static_cast<int64_t>(t0 + t) * hidden + k]), wv, acc[t]);
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < kGemvTokens; ++t) {
      const float s = warp_sum(acc[t]);
      if (lane == 0) partial[local_e][part][t] = s;
    }
    __syncthreads();
    if (threadIdx.x < kGemvExpertsPerCta * kGemvTokens) {
      const int le = threadIdx.x / kGemvTokens, t = threadIdx.x % kGemvTokens;
      const int ee = blockIdx.x * kGemvExpertsPerCta + le;
      if (ee < experts && t < nt) {
        float s = 0.0f;
#pragma unroll
        for (int p = 0; p < kGemvSplit; ++p) s += partial[le][p][t];
        logits[static_cast<int64_t>(t0 + t) * experts + ee] = s;
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Logits, large token counts: 64x64 output tiles, 4x4 per thread, k-tiles of
// 32 staged through shared memory (row-major copies of x and w tiles).
// ---------------------------------------------------------------------------
constexpr int kTileM = 64, kTileN = 64, kTileK = 32;

// blockIdx.z selects a K part of `kpart` columns; its sums go to
// logits + z * tokens * experts (partials summed later in part order).
template <typename XT, typename WT>
__global__ void __launch_bounds__(256) router_logits_tiled_kernel(
    const XT* __restrict__ x, const WT* __restrict__ w, float* __restrict__ logits,
    int tokens, int hidden, int experts, int kpart) {
  __shared__ float xs[kTileK][kTileM + 4];
  __shared__ float ws[kTileK][kTileN + 4];
  const int tm = blockIdx.y * kTileM, tn = blockIdx.x * kTileN;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int k_lo = blockIdx.z * kpart, k_hi = min(hidden, k_lo + kpart);
  logits += static_cast<int64_t>(blockIdx.z) * tokens * experts;
  float acc[4][4] = {};
  for (int k0 = k_lo; k0 < k_hi; k0 += kTileK) {
    for (int i = threadIdx.x; i < kTileM * kTileK; i += 256) {
      const int r = i / kTileK, c = i % kTileK;
      const int gr = tm + r, gc = k0 + c;
      xs[c][r] = (gr < tokens && gc < k_hi) ? to_float_any(x[static_cast<int64_t>(gr) * hidden + gc]) : 0.0f;
      const int er = tn + r;
      ws[c][r] = (er < experts && gc < k_hi) ? to_float_any(w[static_cast<int64_t>(er) * hidden + gc]) : 0.0f;
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < kTileK; ++k) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = xs[k][ty * 4 + i];
        b[i] = ws[k][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = tm + ty * 4 + i;
    if (r >= tokens) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = tn + tx * 4 + j;
      if (c < experts) logits[static_cast<int64_t>(r) * experts + c] = acc[i][j];
    }
  }
}

// ---------------------------------------------------------------------------
// Split-K logits for decode batches: partial[q][t][e] = sum over the q-th
// k-range of x[t, k] * w[e, k].  The k-ranges are multiples of kSpan long, so
// every range starts 16-byte aligned.
// ---------------------------------------------------------------------------
constexpr int kSpan = 32;
constexpr int kMmaRouterWarps = 4;
constexpr int kPartWarps = 8;

template <typename T>
MOE_D void mma_16816_t(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1);

template <>
MOE_D void mma_16816_t<__nv_bfloat16>(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                      uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <>
MOE_D void mma_16816_t<__half>(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// x and w of the same 16-bit type (bf16 or f16): products are exact in fp32
// as in the reference's fp32 F.linear; the tensor pipe accumulates in fp32.
// A warp owns 16 experts (A rows) of one k-range and up to 64 tokens (eight
// 8-column B tiles) at a time.  Lane (g, c) loads 8 consecutive elements
// [8c, 8c + 8) of a 32-element span for rows g and g + 8 and token g; words
// 0/1 of those loads feed one m16n8k16 and words 2/3 another: physical
// k = 8c + {0,1} plays logical k = 2c + {0,1}, 8c + {2,3} plays 2c + 8 + {0,1}
// (and 8c + 4.. the same in the second MMA), identically in A and B, so each
// span's 32 products are each summed once.
template <typename T>
__global__ void __launch_bounds__(kMmaRouterWarps * kWarp) router_logits_mma_kernel(
    const T* __restrict__ x, const T* __restrict__ w, float* __restrict__ partial, int tokens, int hidden,
    int experts, int kpart) {
  const int lane = threadIdx.x % kWarp, g = lane / 4, c = lane % 4;
  const int e0 = (blockIdx.x * kMmaRouterWarps + threadIdx.x / kWarp) * 16;
  if (e0 >= experts) return;
  const int k_lo = blockIdx.y * kpart, k_hi = min(hidden, k_lo + kpart);
  const T* wa = w + static_cast<int64_t>(min(e0 + g, experts - 1)) * hidden + 8 * c;
  const T* wb = w + static_cast<int64_t>(min(e0 + g + 8, experts - 1)) * hidden + 8 * c;
  float* out = partial + static_cast<int64_t>(blockIdx.y) * tokens * experts;
  for (int t0 = blockIdx.z * 64; t0 < tokens; t0 += gridDim.z * 64) {
    const int ntiles = min(8, static_cast<int>(ceil_div(tokens - t0, 8)));
    float acc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
#pragma unroll 2
    for (int k = k_lo; k < k_hi; k += kSpan) {
      const uint4 a_lo = __ldg(reinterpret_cast<const uint4*>(wa + k));
      const uint4 a_hi = __ldg(reinterpret_cast<const uint4*>(wb + k));
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        if (n < ntiles) {
          const int tok = t0 + 8 * n + g;
          const uint4 b = tok < tokens ? __ldg(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(tok) * hidden +
                                                                             k + 8 * c))
                                       : make_uint4(0, 0, 0, 0);
          mma_16816_t<T>(acc[n], a_lo.x, a_hi.x, a_lo.y, a_hi.y, b.x, b.y);
          mma_16816_t<T>(acc[n], a_lo.z, a_hi.z, a_lo.w, a_hi.w, b.z, b.w);
        }
      }
    }
    // acc[n]: (expert e0 + g, tokens 2c, 2c + 1), (expert e0 + g + 8, same tokens)
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      if (n >= ntiles) continue;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int tok = t0 + 8 * n + 2 * c + (i & 1);
        const int e = e0 + g + (i >= 2 ? 8 : 0);
        if (tok < tokens && e < experts) out[static_cast<int64_t>(tok) * experts + e] = acc[n][i];
      }
    }
  }
}

// Decode-batch logits in one pass, no partials: a cluster of kClusterParts
// CTAs shares one 16-expert tile, each CTA a contiguous k-range split over its
// 4 warps.  Fragments and the lane mapping are those of
// router_logits_mma_kernel.  Each warp holds up to 8 spans of its weight rows
// in registers while it walks the token tiles, the warps' sums meet in shared
// memory, and after a cluster barrier each CTA adds 1/kClusterParts of the
// tile's (expert, token) sums over the cluster's CTAs in rank order through
// distributed shared memory -- a fixed order -- and writes the logits.
constexpr int kClusterParts = 8;
constexpr int kClusterWarps = 4;
constexpr int kClusterTokens = 64;
constexpr int kWarpSpans = 8;

constexpr int kStageGroup = 8;        // tokens per register batch of the x staging
constexpr int kStageMaxTokens = 256;

// The staging cluster (the launch's last cluster row, when x16 is given):
// x rows -> f16 with a power-of-two row scale, the rows_to_f16 staging
// (2^(floor(log2 amax) - 13); 1 for a row without a finite nonzero maximum),
// each CTA converting the k-range it would reduce in a logits cluster.  The
// CTAs' slice maxima meet in distributed shared memory.  `sm` is the CTA's
// reduction buffer (2 * kStageMaxTokens + kStageGroup * kClusterWarps floats).
template <typename T>
MOE_D void cluster_stage_x(cooperative_groups::cluster_group& cluster, int rank, const T* __restrict__ x, int tokens,
                           int hidden, int kpart, __half* __restrict__ x16, float* __restrict__ xscale, float* sm) {
  constexpr int V = 16 / sizeof(T);
  float* part = sm;                          // [kStageMaxTokens] this slice's maxima (read by the peers)
  float* rowmax = sm + kStageMaxTokens;      // [kStageMaxTokens] the rows' maxima
  float* wred = sm + 2 * kStageMaxTokens;    // [kStageGroup][kClusterWarps]
  const int lo = min(hidden, rank * kpart), hi = min(hidden, lo + kpart);
  const int n = (hi - lo) / V;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  auto piece = [&](int t, int i) { return reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t) * hidden + lo) + i; };
  for (int t0 = 0; t0 < tokens; t0 += kStageGroup) {
    float m[kStageGroup];
#pragma unroll
    for (int g = 0; g < kStageGroup; ++g) m[g] = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      uint4 v[kStageGroup];
#pragma unroll
      for (int g = 0; g < kStageGroup; ++g) v[g] = t0 + g < tokens ? __ldg(piece(t0 + g, i)) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int g = 0; g < kStageGroup; ++g) {
        float f[V];
        unpack16<T>(v[g], f);
#pragma unroll
        for (int j = 0; j < V; ++j) m[g] = fmaxf(m[g], fabsf(f[j]));
      }
    }
#pragma unroll
    for (int g = 0; g < kStageGroup; ++g) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m[g] = fmaxf(m[g], __shfl_xor_sync(0xFFFFFFFFu, m[g], o));
      if (lane == 0) wred[g * kClusterWarps + warp] = m[g];
    }
    __syncthreads();
    if (threadIdx.x < kStageGroup && t0 + static_cast<int>(threadIdx.x) < tokens) {
      float v = wred[threadIdx.x * kClusterWarps];
#pragma unroll
      for (int q = 1; q < kClusterWarps; ++q) v = fmaxf(v, wred[threadIdx.x * kClusterWarps + q]);
      part[t0 + threadIdx.x] = v;
    }
    __syncthreads();  // wred is rewritten by the next group
  }
  cluster.sync();  // every slice's maxima are visible to the cluster
  for (int t = threadIdx.x; t < tokens; t += blockDim.x) {
    float v = 0.0f;
    for (int q = 0; q < kClusterParts; ++q) v = fmaxf(v, cluster.map_shared_rank(part, q)[t]);
    rowmax[t] = v;
  }
  __syncthreads();
  for (int t0 = 0; t0 < tokens; t0 += kStageGroup) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      uint4 v[kStageGroup];
#pragma unroll
      for (int g = 0; g < kStageGroup; ++g) v[g] = t0 + g < tokens ? __ldg(piece(t0 + g, i)) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int g = 0; g < kStageGroup; ++g) {
        if (t0 + g >= tokens) break;
        const float amax = rowmax[t0 + g];
        const float inv = 1.0f / ((amax > 0.0f && isfinite(amax)) ? ldexpf(1.0f, ilogbf(amax) - 13) : 1.0f);
        float f[V];
        unpack16<T>(v[g], f);
        __align__(16) __half h[V];
#pragma unroll
        for (int j = 0; j < V; ++j) h[j] = __float2half_rn(f[j] * inv);
        __half* dst = x16 + static_cast<int64_t>(t0 + g) * hidden + lo + i * V;
        if (V == 8) *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(h);
        else *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(h);
      }
    }
  }
  if (rank == 0)
    for (int t = threadIdx.x; t < tokens; t += blockDim.x) {
      const float amax = rowmax[t];
      xscale[t] = (amax > 0.0f && isfinite(amax)) ? ldexpf(1.0f, ilogbf(amax) - 13) : 1.0f;
    }
  cluster.sync();  // the peers' reads of part[] are done before this CTA exits
}

template <typename T>
__global__ void __cluster_dims__(kClusterParts, 1, 1) __launch_bounds__(kClusterWarps * kWarp)
    router_logits_cluster_kernel(const T* __restrict__ x, const T* __restrict__ w, float* __restrict__ logits,
                                 int tokens, int hidden, int experts, int kpart, __half* __restrict__ x16,
                                 float* __restrict__ xscale) {
  __shared__ float red[kClusterWarps][16][kClusterTokens];
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  if (x16 != nullptr && blockIdx.y == gridDim.y - 1) {
    cluster_stage_x<T>(cluster, rank, x, tokens, hidden, kpart, x16, xscale, &red[0][0][0]);
    return;
  }
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp, g = lane / 4, c = lane % 4;
  const int e0 = blockIdx.y * 16;
  const int wpart = kpart / kClusterWarps;
  const int k_lo = min(hidden, rank * kpart + warp * wpart), k_hi = min(hidden, k_lo + wpart);
  const T* wa = w + static_cast<int64_t>(min(e0 + g, experts - 1)) * hidden + 8 * c;
  const T* wb = w + static_cast<int64_t>(min(e0 + g + 8, experts - 1)) * hidden + 8 * c;
  for (int t0 = 0; t0 < tokens; t0 += kClusterTokens) {
    const int ntiles = min(kClusterTokens / 8, static_cast<int>(ceil_div(tokens - t0, 8)));
    float acc[kClusterTokens / 8][4];
#pragma unroll
    for (int n = 0; n < kClusterTokens / 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
    for (int kc = k_lo; kc < k_hi; kc += kWarpSpans * kSpan) {
      uint4 a_lo[kWarpSpans], a_hi[kWarpSpans];
#pragma unroll
      for (int s = 0; s < kWarpSpans; ++s) {
        const int k = kc + s * kSpan;
        a_lo[s] = k < k_hi ? __ldg(reinterpret_cast<const uint4*>(wa + k)) : make_uint4(0, 0, 0, 0);
        a_hi[s] = k < k_hi ? __ldg(reinterpret_cast<const uint4*>(wb + k)) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int n = 0; n < kClusterTokens / 8; ++n) {
        if (n >= ntiles) break;
        const int tok = t0 + 8 * n + g;
        const T* xr = x + static_cast<int64_t>(min(tok, tokens - 1)) * hidden + 8 * c;
        uint4 b[kWarpSpans];
#pragma unroll
        for (int s = 0; s < kWarpSpans; ++s) {
          const int k = kc + s * kSpan;
          b[s] = (tok < tokens && k < k_hi) ? __ldg(reinterpret_cast<const uint4*>(xr + k)) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int s = 0; s < kWarpSpans; ++s) {
          mma_16816_t<T>(acc[n], a_lo[s].x, a_hi[s].x, a_lo[s].y, a_hi[s].y, b[s].x, b[s].y);
          mma_16816_t<T>(acc[n], a_lo[s].z, a_hi[s].z, a_lo[s].w, a_hi[s].w, b[s].z, b[s].w);
        }
      }
    }
    // acc[n]: (expert e0 + g (+8), tokens 8n + 2c, 8n + 2c + 1)
#pragma unroll
    for (int n = 0; n < kClusterTokens / 8; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) red[warp][g + (i >= 2 ? 8 : 0)][8 * n + 2 * c + (i & 1)] = acc[n][i];
    __syncthreads();
    for (int j = threadIdx.x; j < 16 * kClusterTokens; j += blockDim.x) {
      float* cell = &red[0][0][0] + j;
      float s = cell[0];
#pragma unroll
      for (int q = 1; q < kClusterWarps; ++q) s += cell[q * 16 * kClusterTokens];
      cell[0] = s;
    }
    cluster.sync();
    // this CTA's share of the tile: entries [rank * per, (rank + 1) * per)
    constexpr int kPer = 16 * kClusterTokens / kClusterParts;
    for (int j = rank * kPer + threadIdx.x; j < (rank + 1) * kPer; j += blockDim.x) {
      const int le = j / kClusterTokens, lt = j % kClusterTokens;
      float s = 0.0f;
      for (int q = 0; q < kClusterParts; ++q) s += cluster.map_shared_rank(&red[0][0][0], q)[j];
      const int e = e0 + le, t = t0 + lt;
      if (e < experts && t < tokens) logits[static_cast<int64_t>(t) * experts + e] = s;
    }
    cluster.sync();  // remote reads done before red[] is rewritten or the CTA exits
  }
}

// Any other dtype pair: one warp per expert and k-range, fp32 FMAs.
template <typename XT, typename WT>
__global__ void __launch_bounds__(kPartWarps * kWarp) router_logits_part_kernel(
    const XT* __restrict__ x, const WT* __restrict__ w, float* __restrict__ partial, int tokens, int hidden,
    int experts, int kpart, int vec_ok) {
  const int lane = threadIdx.x % kWarp;
  const int e = blockIdx.x * kPartWarps + threadIdx.x / kWarp;
  if (e >= experts) return;
  const int k_lo = blockIdx.y * kpart, k_hi = min(hidden, k_lo + kpart);
  const WT* wrow = w + static_cast<int64_t>(e) * hidden;
  float* out = partial + static_cast<int64_t>(blockIdx.y) * tokens * experts + e;
  for (int t = 0; t < tokens; ++t) {
    const XT* xr = x + static_cast<int64_t>(t) * hidden;
    float acc = 0.0f;
    if (vec_ok) {
      for (int k = k_lo + lane * 8; k < k_hi; k += kWarp * 8) {
        float wv[8], xv[8];
        load8<WT>(wrow + k, wv);
        load8<XT>(xr + k, xv);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc = fmaf(xv[i], wv[i], acc);
      }
    } else {
      for (int k = k_lo + lane; k < k_hi; k += kWarp) acc = fmaf(to_float_any(xr[k]), to_float_any(wrow[k]), acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) out[static_cast<int64_t>(t) * experts] = acc;
  }
}

// ---------------------------------------------------------------------------
// Selection: one warp per token.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kSelectWarps * kWarp) router_select_kernel(
    const float* __restrict__ logits, int nparts, int64_t part_stride, const float* __restrict__ bias,
    RouterSelectParams p, int64_t* __restrict__ ids64, int32_t* __restrict__ ids32,
    float* __restrict__ weights_f32, __nv_bfloat16* __restrict__ weights_bf16) {
  extern __shared__ float smem[];
  const int warp = threadIdx.x / kWarp;
  const int t = blockIdx.x * kSelectWarps + warp;
  if (t >= p.tokens) return;
  float* probs = smem + warp * 2 * p.experts;
  select_token(logits, nparts, part_stride, bias, p, t, probs, probs + p.experts, ids64, ids32, weights_f32,
               weights_bf16);
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
template <typename XT, typename WT>
static cudaError_t launch_logits_t(const void* x, const void* w, float* logits, int tokens, int hidden,
                                   int experts, cudaStream_t stream) {
  const XT* xp = static_cast<const XT*>(x);
  const WT* wp = static_cast<const WT*>(w);
  if (tokens <= 256) {
    const bool vec_ok = hidden % 8 == 0 && (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                        (reinterpret_cast<uintptr_t>(w) % 16 == 0) &&
                        (sizeof(XT) == 4 ? (hidden % 4 == 0) : true);
    dim3 grid(static_cast<unsigned>(ceil_div(experts, kGemvExpertsPerCta)));
    router_logits_gemv_kernel<XT, WT><<<grid, 256, 0, stream>>>(xp, wp, logits, tokens, hidden, experts,
                                                                  vec_ok ? 1 : 0);
  } else {
    dim3 grid(static_cast<unsigned>(ceil_div(experts, kTileN)), static_cast<unsigned>(ceil_div(tokens, kTileM)));
    router_logits_tiled_kernel<XT, WT><<<grid, 256, 0, stream>>>(xp, wp, logits, tokens, hidden, experts, hidden);
  }
  return cudaGetLastError();
}

template <typename XT>
static cudaError_t launch_logits_w(const void* x, int w_dtype, const void* w, float* logits, int tokens,
                                   int hidden, int experts, cudaStream_t stream) {
  switch (w_dtype) {
    case kDtypeF32: return launch_logits_t<XT, float>(x, w, logits, tokens, hidden, experts, stream);
    case kDtypeBF16: return launch_logits_t<XT, __nv_bfloat16>(x, w, logits, tokens, hidden, experts, stream);
    case kDtypeF16: return launch_logits_t<XT, __half>(x, w, logits, tokens, hidden, experts, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <typename XT, typename WT>
static cudaError_t launch_split_t(const void* x, const void* w, float* partial, int tokens, int hidden, int experts,
                                  cudaStream_t stream) {
  const int parts = router_split_parts(hidden);
  const int kpart = router_split_kpart(hidden);
  const bool aligned = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (reinterpret_cast<uintptr_t>(w) % 16 == 0);
  constexpr bool kPair = (std::is_same<XT, __nv_bfloat16>::value && std::is_same<WT, __nv_bfloat16>::value) ||
                         (std::is_same<XT, __half>::value && std::is_same<WT, __half>::value);
  if constexpr (kPair) {
    if (aligned && hidden % kSpan == 0) {
      dim3 grid(static_cast<unsigned>(ceil_div(ceil_div(experts, 16), kMmaRouterWarps)),
                static_cast<unsigned>(parts), static_cast<unsigned>(std::min<int64_t>(ceil_div(tokens, 64), 1024)));
      router_logits_mma_kernel<XT><<<grid, kMmaRouterWarps * kWarp, 0, stream>>>(
          static_cast<const XT*>(x), static_cast<const XT*>(w), partial, tokens, hidden, experts, kpart);
      return cudaGetLastError();
    }
  }
  dim3 grid(static_cast<unsigned>(ceil_div(experts, kPartWarps)), static_cast<unsigned>(parts));
  const bool vec_ok = aligned && hidden % 8 == 0;
  router_logits_part_kernel<XT, WT><<<grid, kPartWarps * kWarp, 0, stream>>>(
      static_cast<const XT*>(x), static_cast<const WT*>(w), partial, tokens, hidden, experts, kpart, vec_ok ? 1 : 0);
  return cudaGetLastError();
}

template <typename XT>
static cudaError_t launch_split_w(const void* x, int w_dtype, const void* w, float* partial, int tokens, int hidden,
                                  int experts, cudaStream_t stream) {
  switch (w_dtype) {
    case kDtypeF32: return launch_split_t<XT, float>(x, w, partial, tokens, hidden, experts, stream);
    case kDtypeBF16: return launch_split_t<XT, __nv_bfloat16>(x, w, partial, tokens, hidden, experts, stream);
    case kDtypeF16: return launch_split_t<XT, __half>(x, w, partial, tokens, hidden, experts, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_router_logits_cluster(const void* x, int x_dtype, const void* w, int w_dtype, float* logits,
                                         int tokens, int hidden, int experts, cudaStream_t stream, __half* x16,
                                         float* xscale) {
  if (tokens <= 0) return cudaSuccess;
  const bool aligned = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (reinterpret_cast<uintptr_t>(w) % 16 == 0);
  if (x_dtype != w_dtype || (x_dtype != kDtypeBF16 && x_dtype != kDtypeF16) || !aligned || hidden % kSpan != 0)
    return cudaErrorNotSupported;
  if (x16 && (!xscale || tokens > kStageMaxTokens || (reinterpret_cast<uintptr_t>(x16) % 16) != 0))
    return cudaErrorNotSupported;
  const int kpart = static_cast<int>(ceil_div(ceil_div(hidden, kClusterParts), kSpan * kClusterWarps)) *
                    kSpan * kClusterWarps;
  // one more cluster row stages x when asked
  dim3 grid(kClusterParts, static_cast<unsigned>(ceil_div(experts, 16) + (x16 ? 1 : 0)));
  if (x_dtype == kDtypeBF16)
    router_logits_cluster_kernel<__nv_bfloat16><<<grid, kClusterWarps * kWarp, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w), logits, tokens, hidden, experts,
        kpart, x16, xscale);
  else
    router_logits_cluster_kernel<__half><<<grid, kClusterWarps * kWarp, 0, stream>>>(
        static_cast<const __half*>(x), static_cast<const __half*>(w), logits, tokens, hidden, experts, kpart, x16,
        xscale);
  return cudaGetLastError();
}

bool router_split_is_mma(const void* x, int x_dtype, const void* w, int w_dtype, int hidden) {
  const bool aligned = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (reinterpret_cast<uintptr_t>(w) % 16 == 0);
  return aligned && hidden % kSpan == 0 && x_dtype == w_dtype && (x_dtype == kDtypeBF16 || x_dtype == kDtypeF16);
}

int router_split_parts(int hidden) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(kMaxRouterParts, ceil_div(hidden, 448))));
}

int router_split_kpart(int hidden) {
  return static_cast<int>(ceil_div(ceil_div(hidden, router_split_parts(hidden)), kSpan) * kSpan);
}

cudaError_t launch_router_logits_split(const void* x, int x_dtype, const void* w, int w_dtype, float* partial,
                                       int tokens, int hidden, int experts, cudaStream_t stream) {
  if (tokens <= 0) return cudaSuccess;
  switch (x_dtype) {
    case kDtypeF32: return launch_split_w<float>(x, w_dtype, w, partial, tokens, hidden, experts, stream);
    case kDtypeBF16: return launch_split_w<__nv_bfloat16>(x, w_dtype, w, partial, tokens, hidden, experts, stream);
    case kDtypeF16: return launch_split_w<__half>(x, w_dtype, w, partial, tokens, hidden, experts, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_router_logits(const void* x, int x_dtype, const void* w, int w_dtype, float* logits,
                                 int tokens, int hidden, int experts, cudaStream_t stream) {
  if (tokens <= 0) return cudaSuccess;
  switch (x_dtype) {
    case kDtypeF32: return launch_logits_w<float>(x, w_dtype, w, logits, tokens, hidden, experts, stream);
    case kDtypeBF16: return launch_logits_w<__nv_bfloat16>(x, w_dtype, w, logits, tokens, hidden, experts, stream);
    case kDtypeF16: return launch_logits_w<__half>(x, w_dtype, w, logits, tokens, hidden, experts, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_router_select(const float* logits, const float* bias, const RouterSelectParams& p,
                                 int64_t* ids64, int32_t* ids32, float* weights_f32,
                                 __nv_bfloat16* weights_bf16, cudaStream_t stream, int nparts, int64_t part_stride) {
  if (p.tokens <= 0) return cudaSuccess;
  const size_t smem = static_cast<size_t>(kSelectWarps) * 2 * p.experts * sizeof(float);
  const unsigned grid = static_cast<unsigned>(ceil_div(p.tokens, kSelectWarps));
  if (smem > 48 * 1024) {
    cudaError_t err = cudaFuncSetAttribute(router_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
    if (err != cudaSuccess) return err;
  }
  router_select_kernel<<<grid, kSelectWarps * kWarp, smem, stream>>>(logits, nparts, part_stride, bias, p, ids64,
                                                                      ids32, weights_f32, weights_bf16);
  return cudaGetLastError();
}

}  // namespace moe
