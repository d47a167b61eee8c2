// Multi-head latent attention (MLA) for one decode token: the attention block
// of the reference's DeepSeek forward (src/pcketlm/native/ds_forward.cpp),
//   ds_mla_attention_flash_forward  :517-597  (absorbed attention core)
//   ds_attention_block_forward_f32  :647-782  (q / kv projections, RMSNorm,
//                                              RoPE, cache append, core, o_proj)
// in fp32 like the reference.  At one token every part is HBM- or
// latency-bound (the DeepSeek-V3 shapes stream 750 MB of fp32 weights), so
// the work is laid out for bandwidth:
//  * projections (q_a and kv_a in one launch, q_b, o_proj): one warp per
//    output row (2 or 4 per row when rows are few), eight 16-byte streaming
//    loads in flight per lane;
//  * RMSNorm of q_low and of the new latent row, RoPE of the new pe row: one
//    CTA each (the mean square needs the whole vector);
//  * absorbed queries q_abs[h] = W_UK[h]^T q_nope[h] (and q_pe's RoPE): one
//    CTA per (head, 128 latent columns), coalesced over the latent axis;
//  * attention: the cache split over positions (at most 64 splits), each CTA
//    taking 16 heads of one split in steps of 16 positions staged in shared
//    memory.  Per step: the 256 scores (q_abs . kv + q_pe . pe) * scale, the
//    running max and sum of the reference's online softmax (advanced a step
//    at a time instead of a position at a time: the same quantities up to
//    rounding), and the unnormalised latent sums; a split's (max, sum,
//    latent sums) per head go to the workspace;
//  * merge: one CTA per (head, 256 latent columns) folds the splits with
//    weights exp(m_s - M) and divides by the total (0 when it is not
//    positive, like the reference); W_UV[h] . latent[h] then runs as the
//    projection GEMV over per-head row blocks of wkv_b.
#include <math.h>

#include <algorithm>

#include "fp8_gemv.cuh"
#include "mla.cuh"
#include "plan.cuh"
#include "status.cuh"

namespace moe {
namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvUnroll = 8;
constexpr int kNormThreads = 256;
constexpr int kQabsThreads = 128;
constexpr int kAttnThreads = 256;
constexpr int kAttnHeads = 16;  // heads per attention CTA
constexpr int kAttnPos = 16;    // cache positions per step
constexpr int64_t kMaxSplits = 64;
constexpr int kMergeThreads = 256;

MOE_D float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// y[r] = W[r, :] . x for rows0 rows of w0 (-> y0), then rows1 rows of w1
// (-> y1, with x).  w0's rows come in groups of `group`: row r is at
// w0 + (r / group) * group_stride + (r % group) * cols and multiplies
// x + (r / group) * x_stride (one group and strides 0 for a plain matrix;
// per-head blocks of a [heads, rows, cols] tensor otherwise).
struct GemvRows {
  const float* w0;
  int64_t rows0, group, group_stride, x_stride;
  const float* w1;
  int64_t rows1, cols;
  const float* x;
  float* y0;
  float* y1;
  int vec;
};

// SPLIT warps share a row (its columns in SPLIT contiguous pieces) when there
// are too few rows to keep every SM streaming; their sums are added in piece
// order through shared memory.  Every warp of a CTA runs the same number of
// row blocks, so the barriers are reached by all of them.
template <int SPLIT>
__global__ void __launch_bounds__(kGemvThreads) mla_gemv_kernel(GemvRows a) {
  constexpr int kWarps = kGemvThreads / kWarp, kRowsPerCta = kWarps / SPLIT;
  __shared__ float part[kWarps];
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
  const int slot = warp / SPLIT, piece = warp % SPLIT;
  const int64_t rows = a.rows0 + a.rows1, cols = a.cols;
  const int64_t blocks = (rows + kRowsPerCta - 1) / kRowsPerCta;
  for (int64_t rb = blockIdx.x; rb < blocks; rb += gridDim.x) {
    const int64_t r = rb * kRowsPerCta + slot;
    float sum = 0.0f;
    if (r < rows) {
      const float* w;
      const float* x = a.x;
      if (r < a.rows0) {
        const int64_t grp = r / a.group;
        w = a.w0 + grp * a.group_stride + (r - grp * a.group) * cols;
        x += grp * a.x_stride;
      } else {
        w = a.w1 + (r - a.rows0) * cols;
      }
      float acc0 = 0.0f, acc1 = 0.0f;
      if (a.vec) {
        const float4* w4 = reinterpret_cast<const float4*>(w);
        const float4* x4 = reinterpret_cast<const float4*>(x);
        const int64_t n4 = cols / 4, i1 = (piece + 1) * n4 / SPLIT;
        int64_t i = piece * n4 / SPLIT + lane;
        for (; i + (kGemvUnroll - 1) * kWarp < i1; i += kGemvUnroll * kWarp) {
          float4 wv[kGemvUnroll];
#pragma unroll
          for (int u = 0; u < kGemvUnroll; ++u) wv[u] = __ldcs(w4 + i + u * kWarp);
#pragma unroll
          for (int u = 0; u < kGemvUnroll; u += 2) {
            const float4 xa = __ldg(x4 + i + u * kWarp), xb = __ldg(x4 + i + (u + 1) * kWarp);
            acc0 = fmaf(wv[u].x, xa.x, acc0);
            acc1 = fmaf(wv[u + 1].x, xb.x, acc1);
            acc0 = fmaf(wv[u].y, xa.y, acc0);
            acc1 = fmaf(wv[u + 1].y, xb.y, acc1);
            acc0 = fmaf(wv[u].z, xa.z, acc0);
            acc1 = fmaf(wv[u + 1].z, xb.z, acc1);
            acc0 = fmaf(wv[u].w, xa.w, acc0);
            acc1 = fmaf(wv[u + 1].w, xb.w, acc1);
          }
        }
        // the rest (fewer than 8 float4 per lane): all loads issued before the multiply-adds
        float4 wv[kGemvUnroll - 1], xv[kGemvUnroll - 1];
#pragma unroll
        for (int u = 0; u < kGemvUnroll - 1; ++u) {
          const bool in = i + u * kWarp < i1;
          wv[u] = in ? __ldcs(w4 + i + u * kWarp) : make_float4(0.f, 0.f, 0.f, 0.f);
          xv[u] = in ? __ldg(x4 + i + u * kWarp) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < kGemvUnroll - 1; ++u) {
          float& acc = (u % 2) ? acc1 : acc0;
          acc = fmaf(wv[u].x, xv[u].x, acc);
          acc = fmaf(wv[u].y, xv[u].y, acc);
          acc = fmaf(wv[u].z, xv[u].z, acc);
          acc = fmaf(wv[u].w, xv[u].w, acc);
        }
      } else {
        const int64_t c1 = (piece + 1) * cols / SPLIT;
        for (int64_t c = piece * cols / SPLIT + lane; c < c1; c += kWarp) acc0 = fmaf(__ldcs(w + c), __ldg(x + c), acc0);
      }
      sum = warp_sum(acc0 + acc1);
    }
    if (SPLIT == 1) {
      if (r < rows && lane == 0) {
        if (r < a.rows0) a.y0[r] = sum;
        else a.y1[r - a.rows0] = sum;
      }
      continue;
    }
    if (lane == 0) part[warp] = sum;
    __syncthreads();
    if (piece == 0 && lane == 0 && r < rows) {
      float total = part[warp];
#pragma unroll
      for (int k = 1; k < SPLIT; ++k) total += part[warp + k];
      if (r < a.rows0) a.y0[r] = total;
      else a.y1[r - a.rows0] = total;
    }
    __syncthreads();
  }
}

// RoPE of one rope-wide group (ds_forward.cpp:622-645): pairs (2p, 2p + 1)
// rotated by (cos[p], sin[p]); an odd width is left as it is.  Products and
// sums rounded one at a time, as the reference (built without contraction) does.
MOE_D void rope_group(const float* in, float* out, int64_t rope, const float* cos_v, const float* sin_v, int t,
                      int nt) {
  if (cos_v && rope % 2 == 0) {
    for (int64_t p = t; p < rope / 2; p += nt) {
      const float x0 = in[2 * p], x1 = in[2 * p + 1], c = cos_v[p], s = sin_v[p];
      out[2 * p] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
      out[2 * p + 1] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
  } else {
    for (int64_t i = t; i < rope; i += nt) out[i] = in[i];
  }
}

// CTA 0: q_low <- RMSNorm(q_low) * q_norm in place.  CTA 1: kv_out <-
// RMSNorm(kvr[0, R)) * kv_norm, pe_out <- RoPE(kvr[R, R + rope))
// (ds_forward.cpp:606-620, 746-756).
__global__ void __launch_bounds__(kNormThreads) mla_norm_rope_kernel(float* q_low, const float* __restrict__ q_norm,
                                                                     int64_t q_rank, const float* kvr,
                                                                     const float* __restrict__ kv_norm, int64_t R,
                                                                     int64_t rope, const float* __restrict__ cos_v,
                                                                     const float* __restrict__ sin_v, float* kv_out,
                                                                     float* pe_out, float eps) {
  __shared__ float red[kNormThreads / kWarp];
  const bool is_q = blockIdx.x == 0;
  const float* src = is_q ? q_low : kvr;
  const float* w = is_q ? q_norm : kv_norm;
  float* dst = is_q ? q_low : kv_out;
  const int64_t n = is_q ? q_rank : R;
  float ss = 0.0f;
  for (int64_t i = threadIdx.x; i < n; i += kNormThreads) ss = fmaf(src[i], src[i], ss);
  ss = warp_sum(ss);
  if (threadIdx.x % kWarp == 0) red[threadIdx.x / kWarp] = ss;
  __syncthreads();
  float total = 0.0f;
#pragma unroll
  for (int i = 0; i < kNormThreads / kWarp; ++i) total += red[i];
  const float inv = 1.0f / sqrtf(total / static_cast<float>(n) + eps);
  // each thread rewrites only the elements it read above (q_low is normalised in place)
  for (int64_t i = threadIdx.x; i < n; i += kNormThreads) dst[i] = __fmul_rn(__fmul_rn(src[i], inv), w[i]);
  if (!is_q && rope > 0) rope_group(kvr + R, pe_out, rope, cos_v, sin_v, threadIdx.x, kNormThreads);
}

// q_abs[h, c] = sum_d q_nope[h, d] * wkv_b[h, d, c]  (ds_forward.cpp:550-557); the
// y == 0 CTAs also write q_pe[h] (rotated when cos/sin are given) to q_pe_out.
__global__ void __launch_bounds__(kQabsThreads) mla_qabs_kernel(const float* __restrict__ q_nope, int64_t nope_stride,
                                                                const float* __restrict__ q_pe, int64_t pe_stride,
                                                                const float* __restrict__ wkv_b, int64_t nope,
                                                                int64_t rope, int64_t R, int64_t v_dim,
                                                                const float* __restrict__ cos_v,
                                                                const float* __restrict__ sin_v,
                                                                float* __restrict__ q_abs,
                                                                float* __restrict__ q_pe_out) {
  extern __shared__ float qs[];  // [nope]
  const int64_t h = blockIdx.x;
  for (int64_t d = threadIdx.x; d < nope; d += kQabsThreads) qs[d] = q_nope[h * nope_stride + d];
  __syncthreads();
  const int64_t c = static_cast<int64_t>(blockIdx.y) * kQabsThreads + threadIdx.x;
  if (c < R) {
    const float* w = wkv_b + h * (nope + v_dim) * R + c;
    constexpr int kU = 32;  // loads in flight per thread
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    int64_t d = 0;
    for (; d + kU <= nope; d += kU) {
      float wv[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) wv[u] = __ldcs(w + (d + u) * R);
#pragma unroll
      for (int u = 0; u < kU; u += 4) {
        a0 = fmaf(qs[d + u], wv[u], a0);
        a1 = fmaf(qs[d + u + 1], wv[u + 1], a1);
        a2 = fmaf(qs[d + u + 2], wv[u + 2], a2);
        a3 = fmaf(qs[d + u + 3], wv[u + 3], a3);
      }
    }
    for (; d < nope; ++d) a0 = fmaf(qs[d], __ldcs(w + d * R), a0);
    q_abs[h * R + c] = (a0 + a1) + (a2 + a3);
  }
  if (blockIdx.y == 0 && rope > 0)
    rope_group(q_pe + h * pe_stride, q_pe_out + h * rope, rope, cos_v, sin_v, threadIdx.x, kQabsThreads);
}

struct AttnArgs {
  const float* q_abs;  // [heads, R]
  const float* q_pe;   // [heads, rope]
  const float* kv;     // [L, R]
  const float* pe;     // [L, rope]
  float* part_acc;     // [splits, heads, R]: unnormalised latent sums
  float* part_ml;      // [splits, heads, 2]: running max, running sum
  int64_t heads, L, R, rope, per_split;
  int nbuf;            // cache-step buffers in shared memory: 2 (the next step copied during this one) or 1
  float scale;
};

MOE_HD int64_t round4(int64_t n) { return (n + 3) / 4 * 4; }
// Shared-memory row strides (floats): whole float4 rows.  The score loop reads
// 8 consecutive float4 of one row per 8 lanes, the latent loop consecutive
// floats of one row per warp: neither needs padding against bank conflicts.
MOE_HD int64_t attn_rs(int64_t R) { return round4(R); }
MOE_HD int64_t attn_ps(int64_t rope) { return round4(rope); }
MOE_HD int64_t attn_smem_floats(int64_t R, int64_t rope, int nbuf) {
  return (1 + nbuf) * kAttnHeads * (attn_rs(R) + attn_ps(rope)) + 2 * kAttnPos * kAttnHeads + 3 * kAttnHeads;
}

MOE_D void cp_async16(float* smem, const float* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
               "l"(gmem)
               : "memory");
}
MOE_D void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
MOE_D void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// VEC: R and rope multiples of 4 and 16-byte aligned sources -- the queries and
// each step's 16 cache rows arrive by 16-byte asynchronous copies (the next
// step's while this one computes, with two buffers); otherwise element by element.
template <bool VEC, int COLS>
__global__ void __launch_bounds__(kAttnThreads) mla_attention_kernel(AttnArgs a) {
  extern __shared__ __align__(16) float sm[];
  // shared-memory indices in 32 bits (R <= 1024, rope <= 256); global ones in 64
  const int R = static_cast<int>(a.R), rope = static_cast<int>(a.rope);
  const int RS = static_cast<int>(attn_rs(R)), PS = static_cast<int>(attn_ps(rope));
  const int R4 = static_cast<int>(round4(R)), P4 = static_cast<int>(round4(rope));
  const int nbuf = VEC ? a.nbuf : 1;
  float* qa_s = sm;                              // [16][RS]
  float* qp_s = qa_s + kAttnHeads * RS;          // [16][PS]
  float* kv_b = qp_s + kAttnHeads * PS;          // [nbuf][16][RS]
  float* pe_b = kv_b + nbuf * kAttnPos * RS;     // [nbuf][16][PS]
  float* pt_s = pe_b + nbuf * kAttnPos * PS;     // [16 positions][16 heads]: probabilities
  float* sc_s = pt_s + kAttnPos * kAttnHeads;    // [16 heads][16 positions]: scores
  float* alpha_s = sc_s + kAttnPos * kAttnHeads;
  float* m_s = alpha_s + kAttnHeads;
  float* l_s = m_s + kAttnHeads;

  const int t = threadIdx.x;
  const int64_t h0 = static_cast<int64_t>(blockIdx.x) * kAttnHeads;
  const int nh = static_cast<int>(a.heads - h0 < kAttnHeads ? a.heads - h0 : kAttnHeads);
  const int64_t split = blockIdx.y;
  const int64_t start = split * a.per_split;
  const int64_t end = start + a.per_split < a.L ? start + a.per_split : a.L;
  const int nsteps = static_cast<int>((end - start + kAttnPos - 1) / kAttnPos);

  // step k's cache rows into buffer k % nbuf (VEC: asynchronous, not committed here)
  auto fetch = [&](int k) {
    const int64_t p0 = start + static_cast<int64_t>(k) * kAttnPos;
    const int np = static_cast<int>(end - p0 < kAttnPos ? end - p0 : kAttnPos);
    float* kv_s = kv_b + (k % nbuf) * kAttnPos * RS;
    float* pe_s = pe_b + (k % nbuf) * kAttnPos * PS;
    if (VEC) {
      const int r4 = R / 4, e4 = rope / 4;
      for (int i = t; i < np * r4; i += kAttnThreads) {
        const int q = i / r4, c = 4 * (i - q * r4);
        cp_async16(kv_s + q * RS + c, a.kv + (p0 + q) * a.R + c);
      }
      for (int i = t; i < np * e4; i += kAttnThreads) {
        const int q = i / e4, c = 4 * (i - q * e4);
        cp_async16(pe_s + q * PS + c, a.pe + (p0 + q) * a.rope + c);
      }
    } else {
      for (int q = 0; q < kAttnPos; ++q) {
        const bool live = q < np;
        for (int c = t; c < R4; c += kAttnThreads)
          kv_s[q * RS + c] = (live && c < R) ? a.kv[(p0 + q) * a.R + c] : 0.0f;
        for (int c = t; c < P4; c += kAttnThreads)
          pe_s[q * PS + c] = (live && c < rope) ? a.pe[(p0 + q) * a.rope + c] : 0.0f;
      }
    }
  };

  // the CTA's queries (rows of heads past nh are never read)
  if (VEC) {
    const int r4 = R / 4, e4 = rope / 4;
    for (int i = t; i < nh * r4; i += kAttnThreads) {
      const int hl = i / r4, c = 4 * (i - hl * r4);
      cp_async16(qa_s + hl * RS + c, a.q_abs + (h0 + hl) * a.R + c);
    }
    for (int i = t; i < nh * e4; i += kAttnThreads) {
      const int hl = i / e4, c = 4 * (i - hl * e4);
      cp_async16(qp_s + hl * PS + c, a.q_pe + (h0 + hl) * a.rope + c);
    }
    if (nbuf == 2) fetch(0);
    cp_async_commit();
  } else {
    for (int hl = 0; hl < kAttnHeads; ++hl) {
      for (int c = t; c < R4; c += kAttnThreads)
        qa_s[hl * RS + c] = (hl < nh && c < R) ? a.q_abs[(h0 + hl) * a.R + c] : 0.0f;
      for (int c = t; c < P4; c += kAttnThreads)
        qp_s[hl * PS + c] = (hl < nh && c < rope) ? a.q_pe[(h0 + hl) * a.rope + c] : 0.0f;
    }
  }
  if (t < kAttnHeads) {
    m_s[t] = -INFINITY;
    l_s[t] = 0.0f;
  }

  float acc[COLS][kAttnHeads];
#pragma unroll
  for (int j = 0; j < COLS; ++j)
#pragma unroll
    for (int h = 0; h < kAttnHeads; ++h) acc[j][h] = 0.0f;

  const int hl = t / kAttnPos, pp = t % kAttnPos;  // this thread's score
  for (int k = 0; k < nsteps; ++k) {
    const int64_t p0 = start + static_cast<int64_t>(k) * kAttnPos;
    const int np = static_cast<int>(end - p0 < kAttnPos ? end - p0 : kAttnPos);
    // the buffer written next is no longer read (and the queries / m_s / l_s are set)
    __syncthreads();
    if (VEC) {
      if (nbuf == 2) {
        if (k + 1 < nsteps) {
          fetch(k + 1);
          cp_async_commit();
          cp_async_wait<1>();  // all but the group just issued: step k (and the queries) landed
        } else {
          cp_async_wait<0>();
        }
      } else {
        fetch(k);
        cp_async_commit();
        cp_async_wait<0>();
      }
    } else {
      fetch(k);
    }
    __syncthreads();
    const float* kv_s = kv_b + (k % nbuf) * kAttnPos * RS;
    const float* pe_s = pe_b + (k % nbuf) * kAttnPos * PS;

    // scores (ds_forward.cpp:565-570): thread (tile, kk) sums the 4 heads x 4
    // positions of block `tile` over the float4 columns kk, kk + 16, ...; the
    // 16 lanes of a tile (half a warp) then add up their partial sums
    {
      const int tile = t / 16, kk = t % 16;
      const int hb = 4 * (tile / 4), pb = 4 * (tile % 4);
      float sc[4][4];
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) sc[x][y] = 0.0f;
      auto block_dot = [&](const float* qs, const float* ks, int stride, int n4) {
        for (int i = kk; i < n4; i += 16) {
          float4 qv[4], kv4[4];
#pragma unroll
          for (int x = 0; x < 4; ++x) qv[x] = reinterpret_cast<const float4*>(qs + (hb + x) * stride)[i];
#pragma unroll
          for (int y = 0; y < 4; ++y) kv4[y] = reinterpret_cast<const float4*>(ks + (pb + y) * stride)[i];
#pragma unroll
          for (int x = 0; x < 4; ++x)
#pragma unroll
            for (int y = 0; y < 4; ++y) {
              sc[x][y] = fmaf(qv[x].x, kv4[y].x, sc[x][y]);
              sc[x][y] = fmaf(qv[x].y, kv4[y].y, sc[x][y]);
              sc[x][y] = fmaf(qv[x].z, kv4[y].z, sc[x][y]);
              sc[x][y] = fmaf(qv[x].w, kv4[y].w, sc[x][y]);
            }
        }
      };
      block_dot(qa_s, kv_s, RS, R4 / 4);
      block_dot(qp_s, pe_s, PS, P4 / 4);
      float mine = 0.0f;
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) {
          float v = sc[x][y];
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
          if (x * 4 + y == kk) mine = v;
        }
      const int h = hb + kk / 4, q = pb + kk % 4;
      sc_s[h * kAttnPos + q] = (h < nh && q < np) ? mine * a.scale : -INFINITY;
    }
    __syncthreads();
    const float s = sc_s[hl * kAttnPos + pp];
    // the 16 threads of a head are 16 consecutive lanes of one warp
    float bm = s;
#pragma unroll
    for (int o = kAttnPos / 2; o > 0; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xFFFFFFFFu, bm, o));
    const float m_old = m_s[hl];
    const float m_new = fmaxf(m_old, bm);
    const float p = s == -INFINITY ? 0.0f : expf(s - m_new);
    float bsum = p;
#pragma unroll
    for (int o = kAttnPos / 2; o > 0; o >>= 1) bsum += __shfl_xor_sync(0xFFFFFFFFu, bsum, o);
    // ds_forward.cpp:571-579: the old sum and latent sums scaled by exp(old max - new max), 0 at the start
    const float alpha = m_old == -INFINITY ? 0.0f : expf(m_old - m_new);
    pt_s[pp * kAttnHeads + hl] = p;
    __syncthreads();  // every read of m_s is done
    if (pp == 0) {
      alpha_s[hl] = alpha;
      m_s[hl] = m_new;
      l_s[hl] = l_s[hl] * alpha + bsum;
    }
    __syncthreads();

    // latent sums: columns c = t + 256 j of every head (columns past R stay 0 and are not stored)
    {
      const float4* al4 = reinterpret_cast<const float4*>(alpha_s);
#pragma unroll
      for (int g = 0; g < kAttnHeads / 4; ++g) {
        const float4 al = al4[g];
#pragma unroll
        for (int j = 0; j < COLS; ++j) {
          acc[j][4 * g] *= al.x;
          acc[j][4 * g + 1] *= al.y;
          acc[j][4 * g + 2] *= al.z;
          acc[j][4 * g + 3] *= al.w;
        }
      }
      for (int q = 0; q < np; ++q) {
        const float4* p4 = reinterpret_cast<const float4*>(pt_s + q * kAttnHeads);
        float4 pv[kAttnHeads / 4];
#pragma unroll
        for (int g = 0; g < kAttnHeads / 4; ++g) pv[g] = p4[g];
#pragma unroll
        for (int j = 0; j < COLS; ++j) {
          const int c = t + kAttnThreads * j;
          const float kvv = c < R ? kv_s[q * RS + c] : 0.0f;
#pragma unroll
          for (int g = 0; g < kAttnHeads / 4; ++g) {
            acc[j][4 * g] = fmaf(pv[g].x, kvv, acc[j][4 * g]);
            acc[j][4 * g + 1] = fmaf(pv[g].y, kvv, acc[j][4 * g + 1]);
            acc[j][4 * g + 2] = fmaf(pv[g].z, kvv, acc[j][4 * g + 2]);
            acc[j][4 * g + 3] = fmaf(pv[g].w, kvv, acc[j][4 * g + 3]);
          }
        }
      }
    }
  }
  __syncthreads();

#pragma unroll
  for (int j = 0; j < COLS; ++j) {
    const int c = t + kAttnThreads * j;
    if (c < R) {
#pragma unroll
      for (int h = 0; h < kAttnHeads; ++h)
        if (h < nh) a.part_acc[(split * a.heads + h0 + h) * a.R + c] = acc[j][h];
    }
  }
  if (t < nh) {
    a.part_ml[(split * a.heads + h0 + t) * 2] = m_s[t];
    a.part_ml[(split * a.heads + h0 + t) * 2 + 1] = l_s[t];
  }
}

// latent[h, c] = sum_s exp(m_s - M) acc_s[h, c] / sum_s exp(m_s - M) l_s[h]
// (the splits folded; 0 when the total is not positive, ds_forward.cpp:581-585).
// One CTA per (head, 256 latent columns); the splits in ascending order.
__global__ void __launch_bounds__(kMergeThreads) mla_merge_kernel(const float* __restrict__ part_acc,
                                                                  const float* __restrict__ part_ml, int64_t splits,
                                                                  int64_t heads, int64_t R,
                                                                  float* __restrict__ latent) {
  __shared__ float wsp[kMaxSplits];
  const int64_t h = blockIdx.x;
  float M = -INFINITY;
  for (int64_t s = 0; s < splits; ++s) M = fmaxf(M, part_ml[(s * heads + h) * 2]);
  for (int64_t s = threadIdx.x; s < splits; s += kMergeThreads) {
    const float m = part_ml[(s * heads + h) * 2];
    wsp[s] = m == -INFINITY ? 0.0f : expf(m - M);
  }
  __syncthreads();
  float total = 0.0f;
  for (int64_t s = 0; s < splits; ++s) total = fmaf(wsp[s], part_ml[(s * heads + h) * 2 + 1], total);
  const float inv = total > 0.0f ? 1.0f / total : 0.0f;
  const int64_t c = static_cast<int64_t>(blockIdx.y) * kMergeThreads + threadIdx.x;
  if (c >= R) return;
  constexpr int kU = 16;  // loads in flight per thread: every batch whole, the splits past the end predicated off
  float acc = 0.0f;
  for (int64_t s0 = 0; s0 < splits; s0 += kU) {
    float v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) v[u] = s0 + u < splits ? __ldcg(part_acc + ((s0 + u) * heads + h) * R + c) : 0.0f;
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (s0 + u < splits) acc = fmaf(wsp[s0 + u], v[u], acc);
  }
  latent[h * R + c] = acc * inv;
}

struct Split {
  int64_t per_split, splits;
};
// Positions per split: a multiple of the step, at most kMaxSplits splits (the
// workspace holds that many); fewer when `want` splits are asked for.
Split split_for(int64_t L, int64_t want = kMaxSplits) {
  want = std::max<int64_t>(1, std::min<int64_t>(want, kMaxSplits));
  int64_t per = std::max<int64_t>(kAttnPos, ceil_div(L, want));
  per = ceil_div(per, kAttnPos) * kAttnPos;
  return {per, ceil_div(L, per)};
}

struct CoreLayout {
  float* q_abs;
  float* q_pe;
  float* part_acc;
  float* part_ml;
  float* latent;
};
CoreLayout core_layout(Plan& p, const MlaDims& d) {
  const Split sp = split_for(d.L);
  CoreLayout l{};
  l.q_abs = p.take<float>(d.heads * d.R);
  l.q_pe = p.take<float>(d.heads * std::max<int64_t>(d.rope, 1));
  l.part_acc = p.take<float>(sp.splits * d.heads * d.R);
  l.part_ml = p.take<float>(sp.splits * d.heads * 2);
  l.latent = p.take<float>(d.heads * d.R);
  return l;
}

struct BlockLayout {
  float* q_low;
  float* kvr;
  float* q;
  float* heads_out;
  CoreLayout core;
};
BlockLayout block_layout(Plan& p, const MlaDims& d, int64_t q_rank) {
  BlockLayout l{};
  l.q_low = p.take<float>(q_rank);
  l.kvr = p.take<float>(d.R + d.rope);
  l.q = p.take<float>(d.heads * (d.nope + d.rope));
  l.heads_out = p.take<float>(d.heads * d.v);
  l.core = core_layout(p, d);
  return l;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

cudaError_t launch_gemv(GemvRows g, cudaStream_t s) {
  g.vec = g.cols % 4 == 0 && g.group_stride % 4 == 0 && g.x_stride % 4 == 0 && aligned16(g.w0) &&
          (g.rows1 == 0 || aligned16(g.w1)) && aligned16(g.x);
  const int64_t rows = g.rows0 + g.rows1, sms = gemv_grid_ctas();
  // warps per row: enough rows for 24 streaming warps per SM take one each, fewer share
  const int split = rows >= sms * 24 ? 1 : rows >= sms * 6 ? 2 : 4;
  const int64_t ctas = std::max<int64_t>(1, std::min<int64_t>(ceil_div(rows * split, kGemvThreads / kWarp), sms * 8));
  if (split == 1) mla_gemv_kernel<1><<<static_cast<unsigned>(ctas), kGemvThreads, 0, s>>>(g);
  else if (split == 2) mla_gemv_kernel<2><<<static_cast<unsigned>(ctas), kGemvThreads, 0, s>>>(g);
  else mla_gemv_kernel<4><<<static_cast<unsigned>(ctas), kGemvThreads, 0, s>>>(g);
  return cudaGetLastError();
}

// A plain [rows, cols] matrix (and optionally a second one sharing x).
GemvRows plain_rows(const float* w0, int64_t rows0, int64_t cols, const float* x, float* y0,
                    const float* w1 = nullptr, int64_t rows1 = 0, float* y1 = nullptr) {
  GemvRows g{};
  g.w0 = w0; g.rows0 = rows0; g.group = std::max<int64_t>(rows0, 1); g.group_stride = 0; g.x_stride = 0;
  g.w1 = w1; g.rows1 = rows1; g.cols = cols; g.x = x; g.y0 = y0; g.y1 = y1;
  return g;
}

}  // namespace

int mla_supported(const MlaDims& d) {
  if (d.R > kMlaMaxLatent) return fail(kUnsupported, "kv_lora_rank above 1024");
  if (d.rope > kMlaMaxRope) return fail(kUnsupported, "qk_rope_dim above 256");
  if (d.nope > kMlaMaxNope) return fail(kUnsupported, "qk_nope_dim above 8192");
  if (d.heads > (int64_t(1) << 24) || d.v > (int64_t(1) << 24) || d.L > INT32_MAX)
    return fail(kUnsupported, "dimension too large");  // grid sizes and the kernels' 32-bit step counts
  return kOk;
}

int64_t mla_core_workspace_bytes(const MlaDims& d) {
  Plan p;
  core_layout(p, d);
  return static_cast<int64_t>(p.used());
}

int64_t mla_block_workspace_bytes(const MlaDims& d, int64_t q_rank) {
  Plan p;
  block_layout(p, d, q_rank);
  return static_cast<int64_t>(p.used());
}

static int core_launch(const MlaDims& d, const CoreLayout& l, const float* q_nope, int64_t nope_stride,
                       const float* q_pe, int64_t pe_stride, const float* rope_cos, const float* rope_sin,
                       const float* kv_cache, const float* pe_cache, const float* wkv_b, float* out,
                       float softmax_scale, cudaStream_t s) {
  const dim3 qgrid(static_cast<unsigned>(d.heads), static_cast<unsigned>(ceil_div(d.R, kQabsThreads)));
  mla_qabs_kernel<<<qgrid, kQabsThreads, std::max<int64_t>(d.nope, 1) * sizeof(float), s>>>(
      q_nope, nope_stride, q_pe, pe_stride, wkv_b, d.nope, d.rope, d.R, d.v, rope_cos, rope_sin, l.q_abs, l.q_pe);
  MOE_CUDA(cudaGetLastError(), "mla absorbed queries");

  AttnArgs a{};
  a.q_abs = l.q_abs; a.q_pe = l.q_pe; a.kv = kv_cache; a.pe = pe_cache;
  a.part_acc = l.part_acc; a.part_ml = l.part_ml;
  a.heads = d.heads; a.L = d.L; a.R = d.R; a.rope = d.rope;
  a.scale = softmax_scale;
  const bool vec = d.R % 4 == 0 && d.rope % 4 == 0 && aligned16(l.q_abs) && aligned16(l.q_pe) &&
                   aligned16(kv_cache) && aligned16(pe_cache);
  // two step buffers while two CTAs still fit an SM (about 113 KB each), else one
  a.nbuf = vec && attn_smem_floats(d.R, d.rope, 2) * sizeof(float) <= 113 * 1024 ? 2 : 1;
  const size_t smem = static_cast<size_t>(attn_smem_floats(d.R, d.rope, a.nbuf)) * sizeof(float);
  const bool wide = d.R > 512;  // 4 latent columns per thread, else 2
  auto kernel = vec ? (wide ? mla_attention_kernel<true, 4> : mla_attention_kernel<true, 2>)
                    : (wide ? mla_attention_kernel<false, 4> : mla_attention_kernel<false, 2>);
  MOE_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)),
           "mla attention smem");
  // as many splits as fill the resident CTAs once (at most the workspace's kMaxSplits)
  int per_sm = 0;
  MOE_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kAttnThreads, smem), "mla occupancy");
  const int64_t groups = ceil_div(d.heads, kAttnHeads);
  const Split sp = split_for(d.L, std::max<int64_t>(1, std::max(per_sm, 1) * gemv_grid_ctas() / groups));
  a.per_split = sp.per_split;
  const dim3 agrid(static_cast<unsigned>(groups), static_cast<unsigned>(sp.splits));
  kernel<<<agrid, kAttnThreads, smem, s>>>(a);
  MOE_CUDA(cudaGetLastError(), "mla attention");

  const dim3 mgrid(static_cast<unsigned>(d.heads), static_cast<unsigned>(ceil_div(d.R, kMergeThreads)));
  mla_merge_kernel<<<mgrid, kMergeThreads, 0, s>>>(l.part_acc, l.part_ml, sp.splits, d.heads, d.R, l.latent);
  MOE_CUDA(cudaGetLastError(), "mla merge");
  // out[h, :] = W_UV[h] . latent[h] (:587-595): rows (h, j) of wkv_b[h, nope + j, :]
  GemvRows g{};
  g.w0 = wkv_b + d.nope * d.R; g.rows0 = d.heads * d.v; g.group = d.v; g.group_stride = (d.nope + d.v) * d.R;
  g.x_stride = d.R; g.cols = d.R; g.x = l.latent; g.y0 = out;
  MOE_CUDA(launch_gemv(g, s), "mla W_UV");
  return kOk;
}

int mla_core_run(const MlaDims& d, const float* q_nope, int64_t nope_stride, const float* q_pe, int64_t pe_stride,
                 const float* rope_cos, const float* rope_sin, const float* kv_cache, const float* pe_cache,
                 const float* wkv_b, float* out, float softmax_scale, char* workspace, cudaStream_t stream) {
  Plan p(workspace);
  const CoreLayout l = core_layout(p, d);
  return core_launch(d, l, q_nope, nope_stride, q_pe, pe_stride, rope_cos, rope_sin, kv_cache, pe_cache, wkv_b, out,
                     softmax_scale, stream);
}

int mla_block_run(const MlaDims& d, const MlaBlockArgs& a, char* workspace, cudaStream_t s) {
  Plan p(workspace);
  const BlockLayout l = block_layout(p, d, a.q_rank);
  // the new cache: the previous rows (ds_forward.cpp:727-742), unless the caller appends in place
  if (a.prev_len > 0 && a.next_kv != a.prev_kv)
    MOE_CUDA(cudaMemcpyAsync(a.next_kv, a.prev_kv, static_cast<size_t>(a.prev_len * d.R) * sizeof(float),
                             cudaMemcpyDeviceToDevice, s),
             "kv cache copy");
  if (a.prev_len > 0 && d.rope > 0 && a.next_pe != a.prev_pe)
    MOE_CUDA(cudaMemcpyAsync(a.next_pe, a.prev_pe, static_cast<size_t>(a.prev_len * d.rope) * sizeof(float),
                             cudaMemcpyDeviceToDevice, s),
             "pe cache copy");
  // q_low = q_a . hidden and the new kv_a row (:709, :743-755), in one launch
  MOE_CUDA(launch_gemv(plain_rows(a.q_a, a.q_rank, a.H, a.hidden, l.q_low, a.kv_a, d.R + d.rope, l.kvr), s),
           "q_a / kv_a");
  float* new_kv = a.next_kv + a.prev_len * d.R;
  float* new_pe = a.next_pe + a.prev_len * d.rope;
  mla_norm_rope_kernel<<<2, kNormThreads, 0, s>>>(l.q_low, a.q_norm, a.q_rank, l.kvr, a.kv_norm, d.R, d.rope,
                                                  a.rope_cos, a.rope_sin, new_kv, new_pe, a.eps);
  MOE_CUDA(cudaGetLastError(), "rms norm / rope");
  // q = q_b . q_low as [heads, nope + rope] (:712-724)
  MOE_CUDA(launch_gemv(plain_rows(a.q_b, d.heads * (d.nope + d.rope), a.q_rank, l.q_low, l.q), s), "q_b");
  // the core on the new cache, q_pe rotated on the way (:725-726, :758-775)
  const int code = core_launch(d, l.core, l.q, d.nope + d.rope, l.q + d.nope, d.nope + d.rope, a.rope_cos,
                               a.rope_sin, a.next_kv, a.next_pe, a.kv_b, l.heads_out, a.softmax_scale, s);
  if (code != kOk) return code;
  // hidden_out = o_proj . heads (:777)
  MOE_CUDA(launch_gemv(plain_rows(a.o_w, a.H, d.heads * d.v, l.heads_out, a.out), s), "o_proj");
  return kOk;
}

}  // namespace moe
