// Grouped GEMV for the reference's non-FP8 expert formats, plus the Q4
// dequant and row8 kernels.
//
// Replaces the expert loops of native_moe_forward_fp16 and
// native_moe_selected_forward_u16 (src/pcketlm/native/fp16_moe.cpp:90-267:
// 16-bit dense weights, fp32 accumulation), q4_moe_selected_forward_u16
// (q4_dequant.cpp:357-476: signed int4, one fp16 scale per output row), the
// Q4 dequant (q4_dequant.cpp:171-286) and the row8 packer / GEMV
// (fp16_packed_gemv.cpp:52-116).
//
// The GEMV runs on the warp MMA pipe like the FP8 one (fp8_mma.cu): a warp
// task is a chunk of <= 8 (token, expert) pairs times 16 output rows of two
// matrices (gate + up) or 32 rows of one; lane (g = lane/4, c = lane%4)
// streams 16 bytes of rows g and g+8 per 64-byte row span, and the four
// lanes c of a row cover the span.
//
//  * 16-bit weights: a lane's 16 bytes are 8 consecutive weights k0..k7;
//    words 0/1 feed one m16n8k16 (k0 k1 as logical 2c, 2c+1; k2 k3 as
//    2c+8, 2c+9) and words 2/3 another, against the same 8 activations of
//    token g loaded as 16 bytes.  Products are exact in fp32.  bf16 weights
//    multiply bf16 activations, split as hi = bf16(x) and lo = bf16(x - hi)
//    (two MMAs) so fp32 activations keep 16 bits of mantissa.
//  * int4: a lane's 16 bytes are 32 weights; each 32-bit word holds 8 codes
//    n0..n7 (n0 in the low nibble).  w & 0x000F000F pairs nibbles (n0, n4);
//    xor-ing 0x64086408 makes each half 1024 + (n ^ 8), i.e. 1032 + code
//    exactly, and subtracting 1032 leaves the signed code as an exact f16
//    (the magic-number int4 -> f16 conversion of Kim et al., "Who Says
//    Elephants Can't Run", 2022).  The high nibbles (n1, n5) are masked in
//    place (w & 0x00F000F0, 16x the value) and brought down by one
//    multiply-add; w >> 8 gives (n2, n6) and (n3, n7) the same way.  The resulting
//    pairs (n0,n4) (n1,n5) | (n2,n6) (n3,n7) feed two MMAs; the activations
//    are staged with every group of 8 stored as k0 k4 k1 k5 k2 k6 k3 k7
//    so one 16-byte load gives the matching B pairs.  Codes times f16
//    activations are exact; the row scale multiplies the fp32 sum.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "dense_gemv.cuh"
#include "fp8_gemv.cuh"

namespace moe {

constexpr int kDenseCtaWarps = 4;
constexpr int kDenseSpanBytes = 64;  // bytes of one row per 4 lanes c

// weights per row span: 32 16-bit values or 128 int4 codes
inline int span_weights(int kind) { return kind == kWQ4 ? 128 : 32; }

template <int T>
MOE_D void mma_m16n8k16(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1);

template <>
MOE_D void mma_m16n8k16<0>(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                           uint32_t b1) {  // f16
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <>
MOE_D void mma_m16n8k16<1>(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                           uint32_t b1) {  // bf16
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

MOE_D uint32_t word_at(const uint4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// int4 word -> the four f16 pairs (n0,n4) (n1,n5) (n2,n6) (n3,n7) as exact
// signed codes, one shift per word: the low nibbles of each byte pair are
// masked in place and biased to 1024 + (n ^ 8) (minus 1032: the code), the high
// nibbles masked in place and biased to 1024 + 16 (n ^ 8), brought down by one
// multiply-add (x / 16 - 72: the code).  Every step is exact in f16.
MOE_D void q4_word_to_f16x2(uint32_t w, uint32_t (&h)[4]) {
  const __half2 bias_lo = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));  // 1032
  const __half2 sixteenth = __halves2half2(__float2half(0.0625f), __float2half(0.0625f));
  const __half2 bias_hi = __halves2half2(__float2half(-72.0f), __float2half(-72.0f));
  const uint32_t w8 = w >> 8;
  const uint32_t v0 = (w & 0x000F000Fu) ^ 0x64086408u;   // n0, n4
  const uint32_t v1 = (w & 0x00F000F0u) ^ 0x64806480u;   // n1, n5 (x 16)
  const uint32_t v2 = (w8 & 0x000F000Fu) ^ 0x64086408u;  // n2, n6
  const uint32_t v3 = (w8 & 0x00F000F0u) ^ 0x64806480u;  // n3, n7 (x 16)
  const __half2 r0 = __hsub2(*reinterpret_cast<const __half2*>(&v0), bias_lo);
  const __half2 r1 = __hfma2(*reinterpret_cast<const __half2*>(&v1), sixteenth, bias_hi);
  const __half2 r2 = __hsub2(*reinterpret_cast<const __half2*>(&v2), bias_lo);
  const __half2 r3 = __hfma2(*reinterpret_cast<const __half2*>(&v3), sixteenth, bias_hi);
  h[0] = *reinterpret_cast<const uint32_t*>(&r0);
  h[1] = *reinterpret_cast<const uint32_t*>(&r1);
  h[2] = *reinterpret_cast<const uint32_t*>(&r2);
  h[3] = *reinterpret_cast<const uint32_t*>(&r3);
}

MOE_D uint4 ld_weights(const uint8_t* p) { return __ldcs(reinterpret_cast<const uint4*>(p)); }

template <int KIND, int NS, int EPI>
__global__ void __launch_bounds__(kDenseCtaWarps * kWarp) dense_mma_gemv_kernel(DenseArgs a) {
  constexpr int kMmaType = KIND == kWBF16 ? 1 : 0;
  constexpr int kTaskRows = NS == 2 ? 16 : 32;
  const int lane = threadIdx.x % kWarp;
  const int g = lane / 4, c = lane % 4;
  const int K = a.K, N = a.N;
  const int64_t row_bytes = KIND == kWQ4 ? K / 2 : static_cast<int64_t>(K) * 2;
  const int nspans = static_cast<int>(row_bytes / kDenseSpanBytes);
  const int row_tiles = static_cast<int>(ceil_div(N, kTaskRows));
  const int ksplit = a.ksplit;
  const int64_t tasks = static_cast<int64_t>(*a.n_chunks) * row_tiles;
  const int64_t units = tasks * ksplit;
  const int64_t warp_global = static_cast<int64_t>(blockIdx.x) * kDenseCtaWarps + threadIdx.x / kWarp;
  const int64_t warp_count = static_cast<int64_t>(gridDim.x) * kDenseCtaWarps;

  for (int64_t unit = warp_global; unit < units; unit += warp_count) {
    const int64_t task = unit / ksplit;
    const int ks = static_cast<int>(unit % ksplit);
    const int sp0 = static_cast<int>(static_cast<int64_t>(ks) * nspans / ksplit);
    const int sp1 = static_cast<int>(static_cast<int64_t>(ks + 1) * nspans / ksplit);
    const int ch = static_cast<int>(task / row_tiles);
    const int r0 = static_cast<int>(task % row_tiles) * kTaskRows;
    const int seg = a.chunk_seg[ch], p0 = a.chunk_start[ch], len = a.chunk_len[ch];
    const uint8_t* w0 = reinterpret_cast<const uint8_t*>(a.w0[seg]);
    const uint8_t* w1 = NS == 2 ? reinterpret_cast<const uint8_t*>(a.w1[seg]) : w0;
    const __half* s0 = KIND == kWQ4 ? reinterpret_cast<const __half*>(a.s0[seg]) : nullptr;
    const __half* s1 = KIND == kWQ4 ? (NS == 2 ? reinterpret_cast<const __half*>(a.s1[seg]) : s0) : nullptr;
    const bool present = w0 && w1 && (KIND != kWQ4 || (s0 && s1)) &&
                         ((reinterpret_cast<uintptr_t>(w0) | reinterpret_cast<uintptr_t>(w1)) & 15u) == 0;

    const uint8_t* arow[2][2];
#pragma unroll
    for (int st = 0; st < 2; ++st) {
      const int base = NS == 2 ? r0 : r0 + 16 * st;
      const uint8_t* w = st == 0 ? w0 : w1;
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int row = min(base + g + 8 * rr, N - 1);
        arow[st][rr] = present ? w + static_cast<int64_t>(row) * row_bytes + 16 * c : nullptr;
      }
    }
    const bool bvalid = g < len;
    const int64_t brow = bvalid ? (a.pair_row ? a.pair_row[p0 + g] : static_cast<int64_t>(p0 + g)) : 0;
    const uint16_t* xb = a.xs + brow * K;

    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    if (present && sp0 < sp1) {
      auto load = [&](uint4 (&buf)[2][2][2], int sp) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int s = min(sp + h, sp1 - 1);  // a clamped repeat is loaded but never used
#pragma unroll
          for (int st = 0; st < 2; ++st)
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) buf[h][st][rr] = ld_weights(arow[st][rr] + s * kDenseSpanBytes);
        }
      };
      auto compute = [&](const uint4 (&a4)[2][2], int sp) {
        const int k0 = sp * (KIND == kWQ4 ? 128 : 32);
        if (KIND == kWQ4) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 b = bvalid ? __ldg(reinterpret_cast<const uint4*>(xb + k0 + 32 * c + 8 * j))
                                   : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int st = 0; st < 2; ++st) {
              uint32_t hg[4], hh[4];
              q4_word_to_f16x2(word_at(a4[st][0], j), hg);
              q4_word_to_f16x2(word_at(a4[st][1], j), hh);
              mma_m16n8k16<0>(acc[st], hg[0], hh[0], hg[1], hh[1], b.x, b.y);
              mma_m16n8k16<0>(acc[st], hg[2], hh[2], hg[3], hh[3], b.z, b.w);
            }
          }
        } else {
          const uint4 b = bvalid ? __ldg(reinterpret_cast<const uint4*>(xb + k0 + 8 * c)) : make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int st = 0; st < 2; ++st) {
            mma_m16n8k16<kMmaType>(acc[st], a4[st][0].x, a4[st][1].x, a4[st][0].y, a4[st][1].y, b.x, b.y);
            mma_m16n8k16<kMmaType>(acc[st], a4[st][0].z, a4[st][1].z, a4[st][0].w, a4[st][1].w, b.z, b.w);
          }
          if (KIND == kWBF16) {
            const uint4 lo = bvalid ? __ldg(reinterpret_cast<const uint4*>(xb + a.plane + k0 + 8 * c))
                                    : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int st = 0; st < 2; ++st) {
              mma_m16n8k16<kMmaType>(acc[st], a4[st][0].x, a4[st][1].x, a4[st][0].y, a4[st][1].y, lo.x, lo.y);
              mma_m16n8k16<kMmaType>(acc[st], a4[st][0].z, a4[st][1].z, a4[st][0].w, a4[st][1].w, lo.z, lo.w);
            }
          }
        }
      };
      // ping-pong buffers of two spans each: the next two spans' weight loads
      // are in flight while the current two are multiplied
      uint4 bufA[2][2][2], bufB[2][2][2];
      load(bufA, sp0);
      for (int sp = sp0; sp < sp1; sp += 4) {
        if (sp + 2 < sp1) load(bufB, sp + 2);
        compute(bufA[0], sp);
        if (sp + 1 < sp1) compute(bufA[1], sp + 1);
        if (sp + 2 < sp1) {
          if (sp + 4 < sp1) load(bufA, sp + 4);
          compute(bufB[0], sp + 2);
          if (sp + 3 < sp1) compute(bufB[1], sp + 3);
        }
      }
    }

    if (ksplit > 1) {
      float4* part = reinterpret_cast<float4*>(a.partial + (task * ksplit + ks) * (kWarp * 8) + lane * 8);
      __stcg(part, make_float4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]));
      __stcg(part + 1, make_float4(acc[1][0], acc[1][1], acc[1][2], acc[1][3]));
      __threadfence();
      __syncwarp();
      int last = 0;
      if (lane == 0) last = atomicAdd(a.counters + task, 1) == ksplit - 1;
      last = __shfl_sync(0xFFFFFFFFu, last, 0);
      if (!last) continue;
      __threadfence();
#pragma unroll
      for (int st = 0; st < 2; ++st)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[st][i] = 0.0f;
      const float4* parts = reinterpret_cast<const float4*>(a.partial + task * ksplit * (kWarp * 8) + lane * 8);
      for (int r = 0; r < ksplit; ++r) {
        const float4 v0 = __ldcg(parts + r * (kWarp * 2));
        const float4 v1 = __ldcg(parts + r * (kWarp * 2) + 1);
        acc[0][0] += v0.x; acc[0][1] += v0.y; acc[0][2] += v0.z; acc[0][3] += v0.w;
        acc[1][0] += v1.x; acc[1][1] += v1.y; acc[1][2] += v1.z; acc[1][3] += v1.w;
      }
      if (lane == 0) a.counters[task] = 0;
    }

    // epilogue: lane holds rows (g, g+8) x tokens (2c, 2c+1) per stream
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int tok = 2 * c + j;
      if (tok >= len) continue;
      const int64_t tr = a.pair_row ? a.pair_row[p0 + tok] : static_cast<int64_t>(p0 + tok);
      const float xs = a.xscale[tr];
      const int64_t p = p0 + tok;
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int i = rr * 2 + j;
        if (NS == 2) {
          const int row = r0 + g + 8 * rr;
          if (row < N) {
            float gv = acc[0][i] * xs, uv = acc[1][i] * xs;
            if (KIND == kWQ4 && present) {
              gv *= __half2float(s0[row]);
              uv *= __half2float(s1[row]);
            }
            const float silu = gv / (1.0f + expf(-gv));
            a.out0[p * N + row] = EPI == kEpiSwiglu ? silu * uv : gv;
          }
        } else {
#pragma unroll
          for (int st = 0; st < 2; ++st) {
            const int row = r0 + 16 * st + g + 8 * rr;
            if (row < N) {
              float v = acc[st][i] * xs;
              if (KIND == kWQ4 && present) v *= __half2float(s0[row]);
              a.out0[p * N + row] = v;
            }
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Any shape: one warp per (chunk slot, output row), fp32 activations.
// ---------------------------------------------------------------------------
template <int KIND>
MOE_D float weight_at(const uint8_t* w, int64_t idx) {
  if (KIND == kWQ4) {
    const uint8_t byte = w[idx >> 1];
    const int nib = (idx & 1) ? (byte >> 4) : (byte & 0xF);
    return static_cast<float>(nib >= 8 ? nib - 16 : nib);
  } else if (KIND == kWBF16) {
    return __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(w)[idx]) << 16);
  } else {
    return __half2float(__ushort_as_half(reinterpret_cast<const uint16_t*>(w)[idx]));
  }
}

template <int KIND, int NS, int EPI>
__global__ void __launch_bounds__(256) dense_generic_gemv_kernel(DenseArgs a) {
  const int lane = threadIdx.x % kWarp;
  const int K = a.K, N = a.N;
  const int64_t tasks = static_cast<int64_t>(*a.n_chunks) * 8 * N;
  const int64_t warp_global = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / kWarp;
  const int64_t warp_count = static_cast<int64_t>(gridDim.x) * blockDim.x / kWarp;
  for (int64_t t = warp_global; t < tasks; t += warp_count) {
    const int ch = static_cast<int>(t / (8 * static_cast<int64_t>(N)));
    const int slot = static_cast<int>((t / N) % 8);
    const int row = static_cast<int>(t % N);
    const int len = a.chunk_len[ch];
    if (slot >= len) continue;
    const int seg = a.chunk_seg[ch];
    const int64_t p = a.chunk_start[ch] + slot;
    const int64_t xr = a.pair_row ? a.pair_row[p] : p;
    const float* x = a.x + xr * K;
    const uint8_t* w0 = reinterpret_cast<const uint8_t*>(a.w0[seg]);
    const uint8_t* w1 = NS == 2 ? reinterpret_cast<const uint8_t*>(a.w1[seg]) : nullptr;
    const __half* s0 = KIND == kWQ4 ? reinterpret_cast<const __half*>(a.s0[seg]) : nullptr;
    const __half* s1 = KIND == kWQ4 && NS == 2 ? reinterpret_cast<const __half*>(a.s1[seg]) : nullptr;
    const bool present = w0 && (NS == 1 || w1) && (KIND != kWQ4 || (s0 && (NS == 1 || s1)));
    float d0 = 0.0f, d1 = 0.0f;
    if (present) {
      const int64_t base = static_cast<int64_t>(row) * K;
      for (int k = lane; k < K; k += kWarp) {
        const float xv = x[k];
        d0 = fmaf(xv, weight_at<KIND>(w0, base + k), d0);
        if (NS == 2) d1 = fmaf(xv, weight_at<KIND>(w1, base + k), d1);
      }
    }
    d0 = warp_sum(d0);
    if (NS == 2) d1 = warp_sum(d1);
    if (lane == 0) {
      if (KIND == kWQ4 && present) {
        d0 *= __half2float(s0[row]);
        if (NS == 2) d1 *= __half2float(s1[row]);
      }
      float v = d0;
      if (NS == 2 && EPI == kEpiSwiglu) v = d0 / (1.0f + expf(-d0)) * d1;
      a.out0[p * N + row] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// Activation staging
// ---------------------------------------------------------------------------
template <typename T>
MOE_D float src_at(const T* p, int64_t i);
template <>
MOE_D float src_at<float>(const float* p, int64_t i) { return p[i]; }
template <>
MOE_D float src_at<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) { return __bfloat162float(p[i]); }
template <>
MOE_D float src_at<__half>(const __half* p, int64_t i) { return __half2float(p[i]); }

template <typename T, int MODE>
__global__ void __launch_bounds__(256) stage_rows_kernel(const T* __restrict__ src, int rows, int K,
                                                         const int32_t* __restrict__ n_rows_dev, int scaled,
                                                         uint16_t* __restrict__ dst, float* __restrict__ scale,
                                                         int64_t plane, int32_t* __restrict__ zero, int64_t zero_n) {
  __shared__ float red[8];
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < zero_n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    zero[i] = 0;
  const int n_rows = n_rows_dev ? min(rows, *n_rows_dev) : rows;
  for (int r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const T* s = src + static_cast<int64_t>(r) * K;
    float sc = 1.0f;
    if (scaled && MODE != kStageBF16HiLo) {
      float amax = 0.0f;
      for (int k = threadIdx.x; k < K; k += blockDim.x) amax = fmaxf(amax, fabsf(src_at<T>(s, k)));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
      if (threadIdx.x % kWarp == 0) red[threadIdx.x / kWarp] = amax;
      __syncthreads();
      if (threadIdx.x < kWarp) {
        float v = threadIdx.x < blockDim.x / kWarp ? red[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
        if (threadIdx.x == 0) red[0] = v;
      }
      __syncthreads();
      amax = red[0];
      sc = (amax > 0.0f && isfinite(amax)) ? ldexpf(1.0f, ilogbf(amax) - 13) : 1.0f;
    }
    const float inv = 1.0f / sc;  // exact: a power of two
    uint16_t* d = dst + static_cast<int64_t>(r) * K;
    if (MODE == kStageF16Perm8) {
      // K % 8 == 0: group q of 8 stored as k0 k4 k1 k5 k2 k6 k3 k7
      for (int q = threadIdx.x; q < K / 8; q += blockDim.x) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = src_at<T>(s, 8 * q + i);
        constexpr int kOrder[8] = {0, 4, 1, 5, 2, 6, 3, 7};
        __align__(16) uint16_t h[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = __half_as_ushort(__float2half_rn(v[kOrder[i]] * inv));
        *reinterpret_cast<uint4*>(d + 8 * q) = *reinterpret_cast<const uint4*>(h);
      }
    } else if (MODE == kStageBF16HiLo) {
      for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const float v = src_at<T>(s, k);
        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
        const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
        d[k] = __bfloat16_as_ushort(hi);
        d[plane + k] = __bfloat16_as_ushort(lo);
      }
    } else {
      for (int k = threadIdx.x; k < K; k += blockDim.x) d[k] = __half_as_ushort(__float2half_rn(src_at<T>(s, k) * inv));
    }
    if (threadIdx.x == 0) scale[r] = sc;
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Q4 dequant, row8 pack and row8 GEMV
// ---------------------------------------------------------------------------
__global__ void q4_dequant_kernel(const uint8_t* __restrict__ pk, const __half* __restrict__ sc,
                                  uint16_t* __restrict__ o, int64_t channels, int64_t size) {
  const int64_t n = channels * size;
  for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x * 8) {
    __align__(16) uint16_t h[8];
    const int cnt = static_cast<int>(n - i < 8 ? n - i : 8);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j < cnt) {
        const int64_t idx = i + j;
        const uint8_t byte = pk[idx >> 1];
        const int nib = (idx & 1) ? (byte >> 4) : (byte & 0xF);
        const float code = static_cast<float>(nib >= 8 ? nib - 16 : nib);
        h[j] = __half_as_ushort(__float2half_rn(code * __half2float(sc[idx / size])));
      }
    }
    if (cnt == 8 && (reinterpret_cast<uintptr_t>(o + i) & 15u) == 0) {
      *reinterpret_cast<uint4*>(o + i) = *reinterpret_cast<const uint4*>(h);
    } else {
      for (int j = 0; j < cnt; ++j) o[i + j] = h[j];
    }
  }
}

__global__ void pack_rows8_kernel(const uint16_t* __restrict__ w, uint16_t* __restrict__ packed, int64_t rows,
                                  int64_t cols) {
  const int64_t groups = ((rows + 7) / 8) * cols;
  for (int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; q < groups;
       q += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t blk = q / cols, col = q % cols;
    __align__(16) uint16_t v[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) {
      const int64_t r = blk * 8 + l;
      v[l] = r < rows ? w[r * cols + col] : 0;
    }
    *reinterpret_cast<uint4*>(packed + q * 8) = *reinterpret_cast<const uint4*>(v);
  }
}

template <int DT>  // kDtypeBF16 or kDtypeF16
MOE_D float u16_to_float(uint16_t v) {
  return DT == 1 ? __uint_as_float(static_cast<uint32_t>(v) << 16) : __half2float(__ushort_as_half(v));
}

template <int DT>
__global__ void __launch_bounds__(256) rows8_gemv_kernel(const uint16_t* __restrict__ x,
                                                        const uint16_t* __restrict__ packed, float* __restrict__ out,
                                                        int64_t rows, int64_t cols) {
  const int lane = threadIdx.x % kWarp;
  const int64_t blocks = (rows + 7) / 8;
  const int64_t warp_global = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / kWarp;
  const int64_t warp_count = static_cast<int64_t>(gridDim.x) * blockDim.x / kWarp;
  for (int64_t blk = warp_global; blk < blocks; blk += warp_count) {
    const uint4* src = reinterpret_cast<const uint4*>(packed + blk * cols * 8);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int64_t c = lane; c < cols; c += kWarp) {
      const uint4 v = __ldcs(src + c);
      const float xc = u16_to_float<DT>(x[c]);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] = fmaf(xc, u16_to_float<DT>(static_cast<uint16_t>(w[i] & 0xFFFFu)), acc[2 * i]);
        acc[2 * i + 1] = fmaf(xc, u16_to_float<DT>(static_cast<uint16_t>(w[i] >> 16)), acc[2 * i + 1]);
      }
    }
#pragma unroll
    for (int l = 0; l < 8; ++l) acc[l] = warp_sum(acc[l]);
    if (lane < 8) {
      const int64_t r = blk * 8 + lane;
      float mine = acc[0];
#pragma unroll
      for (int l = 1; l < 8; ++l)
        if (lane == l) mine = acc[l];
      if (r < rows) out[r] = mine;
    }
  }
}

template <typename T>
__global__ void to_f32_kernel(const T* __restrict__ src, int64_t n, float* __restrict__ dst) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = src_at<T>(src, i);
}

__global__ void fill_table_kernel(uint64_t* table, uint64_t base, int64_t stride, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    table[i] = base + static_cast<uint64_t>(static_cast<int64_t>(i) * stride);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
bool dense_mma_supported(int kind, int K) {
  if (K <= 0) return false;
  return kind == kWQ4 ? K % span_weights(kWQ4) == 0 : K % span_weights(kWF16) == 0;
}

template <int KIND>
static int dense_ctas_per_sm() {
  static int per_sm = 0;
  if (per_sm == 0) {
    int a = 0, b = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&a, dense_mma_gemv_kernel<KIND, 2, kEpiSwiglu>,
                                                  kDenseCtaWarps * kWarp, 0);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, dense_mma_gemv_kernel<KIND, 1, kEpiStore>,
                                                  kDenseCtaWarps * kWarp, 0);
    per_sm = std::max(1, std::min(a, b));
  }
  return per_sm;
}

static int dense_ctas_per_sm_of(int kind) {
  return kind == kWQ4 ? dense_ctas_per_sm<kWQ4>() : kind == kWBF16 ? dense_ctas_per_sm<kWBF16>()
                                                                   : dense_ctas_per_sm<kWF16>();
}

int dense_mma_ksplit(int kind, int64_t tasks_bound, int K) {
  const int64_t warps = static_cast<int64_t>(gemv_grid_ctas()) * dense_ctas_per_sm_of(kind) * kDenseCtaWarps;
  if (tasks_bound <= 0 || tasks_bound >= warps) return 1;
  const int64_t spans = (kind == kWQ4 ? K / 2 : static_cast<int64_t>(K) * 2) / kDenseSpanBytes;
  const int64_t want = ceil_div(warps, tasks_bound);
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>({want, spans / 8, kMaxMmaKSplit})));
}

template <int KIND>
static cudaError_t launch_dense_kind(const DenseArgs& a, int ns, int epi, unsigned grid, cudaStream_t stream) {
  const unsigned threads = kDenseCtaWarps * kWarp;
  if (ns == 2 && epi == kEpiSwiglu) dense_mma_gemv_kernel<KIND, 2, kEpiSwiglu><<<grid, threads, 0, stream>>>(a);
  else if (ns == 1 && epi == kEpiStore) dense_mma_gemv_kernel<KIND, 1, kEpiStore><<<grid, threads, 0, stream>>>(a);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t launch_dense_mma_gemv(const DenseArgs& a, int kind, int ns, int epi, int64_t tasks_bound,
                                  cudaStream_t stream) {
  if (!dense_mma_supported(kind, a.K) || a.ksplit < 1 || a.ksplit > kMaxMmaKSplit ||
      (a.ksplit > 1 && (!a.partial || !a.counters)) || !a.xs || !a.xscale)
    return cudaErrorInvalidValue;
  const int64_t full = static_cast<int64_t>(gemv_grid_ctas()) * dense_ctas_per_sm_of(kind);
  const int64_t need = ceil_div(std::max<int64_t>(1, tasks_bound) * a.ksplit, kDenseCtaWarps);
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min(full, need)));
  switch (kind) {
    case kWF16: return launch_dense_kind<kWF16>(a, ns, epi, grid, stream);
    case kWBF16: return launch_dense_kind<kWBF16>(a, ns, epi, grid, stream);
    case kWQ4: return launch_dense_kind<kWQ4>(a, ns, epi, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <int KIND>
static cudaError_t launch_generic_kind(const DenseArgs& a, int ns, int epi, unsigned grid, cudaStream_t stream) {
  if (ns == 2 && epi == kEpiSwiglu) dense_generic_gemv_kernel<KIND, 2, kEpiSwiglu><<<grid, 256, 0, stream>>>(a);
  else if (ns == 1 && epi == kEpiStore) dense_generic_gemv_kernel<KIND, 1, kEpiStore><<<grid, 256, 0, stream>>>(a);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t launch_dense_generic_gemv(const DenseArgs& a, int kind, int ns, int epi, int64_t pairs,
                                      cudaStream_t stream) {
  if (!a.x) return cudaErrorInvalidValue;
  const int64_t warps = std::max<int64_t>(1, pairs) * a.N;
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(warps, 8),
                                                                                      gemv_grid_ctas() * 16)));
  switch (kind) {
    case kWF16: return launch_generic_kind<kWF16>(a, ns, epi, grid, stream);
    case kWBF16: return launch_generic_kind<kWBF16>(a, ns, epi, grid, stream);
    case kWQ4: return launch_generic_kind<kWQ4>(a, ns, epi, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
static cudaError_t launch_stage_t(const void* src, int rows, int K, const int32_t* n_rows_dev, int mode,
                                  bool scaled, uint16_t* dst, float* scale, int64_t plane, int32_t* zero,
                                  int64_t zero_n, unsigned grid, cudaStream_t stream) {
  const T* s = static_cast<const T*>(src);
  switch (mode) {
    case kStageF16:
      stage_rows_kernel<T, kStageF16><<<grid, 256, 0, stream>>>(s, rows, K, n_rows_dev, scaled, dst, scale, plane,
                                                                  zero, zero_n);
      break;
    case kStageF16Perm8:
      if (K % 8 != 0) return cudaErrorInvalidValue;
      stage_rows_kernel<T, kStageF16Perm8><<<grid, 256, 0, stream>>>(s, rows, K, n_rows_dev, scaled, dst, scale,
                                                                       plane, zero, zero_n);
      break;
    case kStageBF16HiLo:
      stage_rows_kernel<T, kStageBF16HiLo><<<grid, 256, 0, stream>>>(s, rows, K, n_rows_dev, scaled, dst, scale,
                                                                       plane, zero, zero_n);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_stage_rows(const void* src, int src_dtype, int rows, int K, const int32_t* n_rows_dev,
                              int mode, bool scaled, uint16_t* dst, float* scale, int64_t plane,
                              int32_t* zero, int64_t zero_n, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  if (zero_n > 0 && !zero) return cudaErrorInvalidValue;
  const unsigned grid = static_cast<unsigned>(std::min(rows, gemv_grid_ctas() * 8));
  switch (src_dtype) {
    case 0: return launch_stage_t<float>(src, rows, K, n_rows_dev, mode, scaled, dst, scale, plane, zero, zero_n, grid,
                                         stream);
    case 1: return launch_stage_t<__nv_bfloat16>(src, rows, K, n_rows_dev, mode, scaled, dst, scale, plane, zero,
                                                 zero_n, grid, stream);
    case 2: return launch_stage_t<__half>(src, rows, K, n_rows_dev, mode, scaled, dst, scale, plane, zero, zero_n,
                                          grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_to_f32(const void* src, int src_dtype, int64_t n, float* dst, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(ceil_div(n, 256), gemv_grid_ctas() * 8));
  switch (src_dtype) {
    case 0: to_f32_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float*>(src), n, dst); break;
    case 1: to_f32_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(src), n, dst); break;
    case 2: to_f32_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<const __half*>(src), n, dst); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_fill_table(uint64_t* table, const void* base, int64_t stride_bytes, int n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  fill_table_kernel<<<static_cast<unsigned>(ceil_div(n, 256)), 256, 0, stream>>>(
      table, reinterpret_cast<uint64_t>(base), stride_bytes, n);
  return cudaGetLastError();
}

cudaError_t launch_q4_dequant(const uint8_t* packed, const uint16_t* scales, uint16_t* out, int64_t channels,
                              int64_t size, cudaStream_t stream) {
  const int64_t n = channels * size;
  if (n <= 0) return cudaSuccess;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(ceil_div(ceil_div(n, 8), 256), gemv_grid_ctas() * 8));
  q4_dequant_kernel<<<grid, 256, 0, stream>>>(packed, reinterpret_cast<const __half*>(scales), out, channels, size);
  return cudaGetLastError();
}

cudaError_t launch_pack_rows8(const uint16_t* w, uint16_t* packed, int64_t rows, int64_t cols, cudaStream_t stream) {
  const int64_t groups = ((rows + 7) / 8) * cols;
  if (groups <= 0) return cudaSuccess;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(ceil_div(groups, 256), gemv_grid_ctas() * 16));
  pack_rows8_kernel<<<grid, 256, 0, stream>>>(w, packed, rows, cols);
  return cudaGetLastError();
}

cudaError_t launch_rows8_gemv(const uint16_t* x, const uint16_t* packed, float* out, int64_t rows, int64_t cols,
                              int dtype, cudaStream_t stream) {
  const int64_t blocks = (rows + 7) / 8;
  if (blocks <= 0) return cudaSuccess;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(ceil_div(blocks, 8), gemv_grid_ctas() * 16));
  if (dtype == 1) rows8_gemv_kernel<1><<<grid, 256, 0, stream>>>(x, packed, out, rows, cols);
  else if (dtype == 2) rows8_gemv_kernel<2><<<grid, 256, 0, stream>>>(x, packed, out, rows, cols);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace moe
