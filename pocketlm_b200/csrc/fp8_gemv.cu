// Grouped FP8 block-scaled GEMV (decode-sized batches) and the weighted combine.
//
// One kernel template covers every FP8 expert product of the reference's
// fp8_linear.cpp (src/pcketlm/native/): the gate/up projections with SwiGLU
// (:309-336), the down projection (:338-357), and the plain and dual linears
// (:50-210).  Work is a list of chunks -- up to NT pairs (token rows) of one
// segment (one expert) -- times 64-row output tiles.  A CTA stages the chunk's
// activation rows in shared memory once, then every warp streams its weight
// rows from HBM exactly once with 16-byte loads and multiplies them against
// all NT staged rows, so an expert's weights are read once per chunk however
// many tokens it serves.
//
// Numerics follow the reference: e4m3 codes decode exactly (0x7F/0xFF as +0,
// fp8_linear.cpp:31-33), products and sums are fp32, and each lane's 16-column
// partial sum (which lies inside one 128-column scale block) is multiplied by
// that block's scale before it is accumulated -- the reference's
// "sum the block, then scale" (fp8_linear.cpp:103-112) at a finer grain.
#include "common.cuh"
#include "fp8_gemv.cuh"

namespace moe {

constexpr int kGemvWarps = 16;
constexpr int kGemvThreads = kGemvWarps * kWarp;
constexpr int kRowsPerWarp = 4;
constexpr int kTileRows = kGemvWarps * kRowsPerWarp;  // 64 output rows per work item

MOE_D uint4 ld_stream16(const uint8_t* p) {
  // weights are touched once per chunk: stream them past L1
  return __ldcs(reinterpret_cast<const uint4*>(p));
}

template <typename XT>
MOE_D void smem_load4(const XT* p, float* out) {
  load4<XT>(p, out);
}

MOE_D float silu_mul(float g, float u) {
  const float silu = g / (1.0f + expf(-g));
  return silu * u;
}

// NS = weight streams per output row (1: linear/down, 2: gate+up or dual).
// Each warp step handles RS = 4 / NS rows, i.e. always 4 weight streams.
template <typename XT, int NT, int NS, int EPI, bool VEC>
__global__ void __launch_bounds__(kGemvThreads, 1) grouped_gemv_kernel(GemvArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  XT* xs = reinterpret_cast<XT*>(smem_raw);  // [NT][K]
  constexpr int RS = 4 / NS;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int K = a.K, N = a.N;
  const int n_chunks = *a.n_chunks;
  const int row_tiles = static_cast<int>(ceil_div(N, kTileRows));
  const int64_t work = static_cast<int64_t>(n_chunks) * row_tiles;
  const int64_t w_lo = work * blockIdx.x / gridDim.x;
  const int64_t w_hi = work * (blockIdx.x + 1) / gridDim.x;
  int staged = -1;

  for (int64_t wi = w_lo; wi < w_hi; ++wi) {
    const int c = static_cast<int>(wi / row_tiles);
    const int rt = static_cast<int>(wi % row_tiles);
    const int seg = a.chunk_seg[c], p0 = a.chunk_start[c], len = a.chunk_len[c];
    if (c != staged) {
      __syncthreads();
      // stage the chunk's activation rows (zero-filled past len)
      for (int t = 0; t < NT; ++t) {
        XT* dst = xs + static_cast<int64_t>(t) * K;
        if (t < len) {
          const int64_t src_row = a.pair_row ? a.pair_row[p0 + t] : static_cast<int64_t>(p0 + t);
          const XT* src = static_cast<const XT*>(a.x) + src_row * K;
          if (VEC) {
            const int n16 = K * static_cast<int>(sizeof(XT)) / 16;
            for (int i = threadIdx.x; i < n16; i += kGemvThreads)
              reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
          } else {
            for (int i = threadIdx.x; i < K; i += kGemvThreads) dst[i] = src[i];
          }
        } else {
          for (int i = threadIdx.x; i < K; i += kGemvThreads) dst[i] = XT(0.0f);
        }
      }
      __syncthreads();
      staged = c;
    }

    const uint8_t* w0 = reinterpret_cast<const uint8_t*>(a.w0[seg]);
    const float* s0 = reinterpret_cast<const float*>(a.s0[seg]);
    const uint8_t* w1 = NS == 2 ? reinterpret_cast<const uint8_t*>(a.w1[seg]) : nullptr;
    const float* s1 = NS == 2 ? reinterpret_cast<const float*>(a.s1[seg]) : nullptr;
    // an absent expert (null table entry) contributes zeros, as the reference
    // skips it (fp8_linear.cpp:410-415, :449-451)
    const bool present = w0 && s0 && (NS == 1 || (w1 && s1));
    // 16-byte vector loads need 16-byte aligned weight rows; otherwise take the byte path
    const bool wal = ((reinterpret_cast<uintptr_t>(w0) | reinterpret_cast<uintptr_t>(w1) |
                       static_cast<uintptr_t>(K)) & 15u) == 0;

    for (int step = 0; step < kRowsPerWarp / RS; ++step) {
      const int r0 = rt * kTileRows + warp * kRowsPerWarp + step * RS;
      if (r0 >= N) break;
      // stream q (0..3) -> row r0 + q / NS, weight matrix q % NS
      const uint8_t* wp[4];
      const float* sp[4];
      bool live[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int r = r0 + q / NS;
        live[q] = r < N;
        const int rr = live[q] ? r : r0;
        const uint8_t* wbase = (q % NS) == 0 ? w0 : w1;
        const float* sbase = (q % NS) == 0 ? s0 : s1;
        wp[q] = wbase ? wbase + static_cast<int64_t>(rr) * K : nullptr;
        sp[q] = sbase ? sbase + static_cast<int64_t>(rr / kBlock) * a.scale_cols : nullptr;
      }
      float acc[4][NT];
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[q][t] = 0.0f;

      if (!present) {
        // acc stays zero
      } else if (VEC && wal) {
        const int nk = K / 16;
#pragma unroll 2
        for (int kc = lane; kc < nk; kc += kWarp) {
          uint4 raw[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) raw[q] = ld_stream16(wp[q] + kc * 16);
          float sc[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) sc[q] = __ldg(sp[q] + (kc >> 3));
          float part[4][NT];
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int t = 0; t < NT; ++t) part[q][t] = 0.0f;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float wv[4][4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint32_t word = j == 0 ? raw[q].x : j == 1 ? raw[q].y : j == 2 ? raw[q].z : raw[q].w;
              e4m3x4_to_float4(word, wv[q]);
            }
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              if (t < len) {
                float xv[4];
                smem_load4<XT>(xs + static_cast<int64_t>(t) * K + kc * 16 + j * 4, xv);
#pragma unroll
                for (int q = 0; q < 4; ++q)
#pragma unroll
                  for (int i = 0; i < 4; ++i) part[q][t] = fmaf(xv[i], wv[q][i], part[q][t]);
              }
            }
          }
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[q][t] = fmaf(part[q][t], sc[q], acc[q][t]);
        }
      } else {
        for (int k = lane; k < K; k += kWarp) {
          float sc[4], wv[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            sc[q] = sp[q][k / kBlock];
            wv[q] = e4m3_to_float_zero_nan(wp[q][k]);
          }
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if (t < len) {
              const float xv = to_float<XT>(xs[static_cast<int64_t>(t) * K + k]);
#pragma unroll
              for (int q = 0; q < 4; ++q) acc[q][t] = fmaf(xv * wv[q], sc[q], acc[q][t]);
            }
          }
        }
      }

      // reduce across the warp; lane t keeps token t's sums
      float mine[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) mine[q] = 0.0f;
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const float s = warp_sum(acc[q][t]);
          if (lane == t) mine[q] = s;
        }
      if (lane < len) {
        const int64_t p = p0 + lane;
#pragma unroll
        for (int i = 0; i < RS; ++i) {
          const int r = r0 + i;
          if (!live[i * NS]) continue;
          if (EPI == kEpiSwiglu) {
            a.out0[p * N + r] = silu_mul(mine[i * 2], mine[i * 2 + 1]);
          } else if (EPI == kEpiStore) {
            a.out0[p * N + r] = mine[i];
          } else {  // kEpiStoreBoth
            a.out0[p * N + r] = mine[i * 2];
            a.out1[p * N + r] = mine[i * 2 + 1];
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Weighted combine: out[t] = sum_j weight[p_j] * y[p_j], pairs of row t taken
// in list order (the reference's summation order: fp8_linear.cpp:557-585 for
// table order, :964-975 for pair order).
// ---------------------------------------------------------------------------
// W values of row p from column h (W = 8: bf16 rows, 16-byte loads; 4: fp32 or bf16; 1: any)
template <int W>
MOE_D void load_y(const CombineArgs& a, int64_t p, int h, float (&v)[W]) {
  if (a.y16) {
    const __nv_bfloat16* yp = a.y16 + p * a.H + h;
    if constexpr (W == 8) {
      const uint4 u = *reinterpret_cast<const uint4*>(yp);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
      }
    } else if constexpr (W == 4) {
      const uint2 u = *reinterpret_cast<const uint2*>(yp);
      v[0] = __uint_as_float(u.x << 16); v[1] = __uint_as_float(u.x & 0xFFFF0000u);
      v[2] = __uint_as_float(u.y << 16); v[3] = __uint_as_float(u.y & 0xFFFF0000u);
    } else {
      v[0] = __bfloat162float(yp[0]);
    }
    return;
  }
  const float* yp = a.y + p * a.H + h;
  if constexpr (W == 4) {
    const float4 f = *reinterpret_cast<const float4*>(yp);
    v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
  } else {
#pragma unroll
    for (int i = 0; i < W; ++i) v[i] = yp[i];
  }
}

template <int W>
__global__ void combine_kernel(CombineArgs a) {
  const int h = (blockIdx.x * blockDim.x + threadIdx.x) * W;
  if (h >= a.H) return;
  for (int t = blockIdx.y; t < a.T; t += gridDim.y) {  // rows past grid.y's limit of 65535 loop
    const int lo = a.row_ptr ? a.row_ptr[t] : t * a.stride;
    const int hi = a.row_ptr ? a.row_ptr[t + 1] : lo + a.stride;
    float acc[W];
#pragma unroll
    for (int i = 0; i < W; ++i) acc[i] = 0.0f;
#pragma unroll 8
    for (int j = lo; j < hi; ++j) {
      const int p = a.row_pairs ? a.row_pairs[j] : j;
      if (p < 0) continue;
      const float w = a.pair_weight ? a.pair_weight[p] : 1.0f;
      float v[W];
      load_y<W>(a, p, h, v);
#pragma unroll
      for (int i = 0; i < W; ++i) acc[i] = fmaf(w, v[i], acc[i]);
    }
    if (a.extra_base >= 0) {
      float v[W];
      load_y<W>(a, a.extra_base + t, h, v);
#pragma unroll
      for (int i = 0; i < W; ++i) acc[i] += v[i];
    }
    const int64_t o = static_cast<int64_t>(t) * a.H + h;
#pragma unroll
    for (int i = 0; i < W; ++i) {
      if (a.out_f32) a.out_f32[o + i] = acc[i];
      if (a.out_f16) a.out_f16[o + i] = __float2half_rn(acc[i]);
      if (a.out_bf16)
        a.out_bf16[o + i] = __float2bfloat16_rn(a.bf16_via_f16 ? __half2float(__float2half_rn(acc[i])) : acc[i]);
    }
  }
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
int gemv_grid_ctas() {
  static int ctas = 0;
  if (ctas == 0) {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    ctas = sms > 0 ? sms : 148;
  }
  return ctas;
}

template <typename XT, int NT, int NS, int EPI>
static cudaError_t launch_t(const GemvArgs& a, bool vec, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(NT) * a.K * sizeof(XT);
  auto kernel = vec ? grouped_gemv_kernel<XT, NT, NS, EPI, true> : grouped_gemv_kernel<XT, NT, NS, EPI, false>;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  kernel<<<gemv_grid_ctas(), kGemvThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

template <typename XT, int NS, int EPI>
static cudaError_t launch_nt(const GemvArgs& a, int nt, bool vec, cudaStream_t stream) {
  switch (nt) {
    case 1: return launch_t<XT, 1, NS, EPI>(a, vec, stream);
    case 4: return launch_t<XT, 4, NS, EPI>(a, vec, stream);
    case 8: return launch_t<XT, 8, NS, EPI>(a, vec, stream);
    default: return cudaErrorInvalidValue;
  }
}

int gemv_chunk_tokens(int K, int x_dtype) {
  const size_t budget = 200 * 1024;
  const size_t row = static_cast<size_t>(K) * (x_dtype == kXF32 ? 4 : 2);
  if (x_dtype != kXF32 && 8 * row <= budget) return 8;
  if (4 * row <= budget) return 4;
  if (row <= budget) return 1;
  return 0;
}

cudaError_t launch_grouped_gemv(const GemvArgs& a, int x_dtype, int ns, int epi, int nt, bool vec,
                                cudaStream_t stream) {
  if (x_dtype == kXBF16) {
    if (ns == 2 && epi == kEpiSwiglu) return launch_nt<__nv_bfloat16, 2, kEpiSwiglu>(a, nt, vec, stream);
    if (ns == 1 && epi == kEpiStore) return launch_nt<__nv_bfloat16, 1, kEpiStore>(a, nt, vec, stream);
    if (ns == 2 && epi == kEpiStoreBoth) return launch_nt<__nv_bfloat16, 2, kEpiStoreBoth>(a, nt, vec, stream);
  } else {
    if (ns == 2 && epi == kEpiSwiglu) return launch_nt<float, 2, kEpiSwiglu>(a, nt, vec, stream);
    if (ns == 1 && epi == kEpiStore) return launch_nt<float, 1, kEpiStore>(a, nt, vec, stream);
    if (ns == 2 && epi == kEpiStoreBoth) return launch_nt<float, 2, kEpiStoreBoth>(a, nt, vec, stream);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_combine(const CombineArgs& a, cudaStream_t stream) {
  if (a.T <= 0) return cudaSuccess;
  // bf16 rows: 8 columns per thread (one 16-byte load per pair); fp32: 4
  const bool y16_aligned = a.y16 && (reinterpret_cast<uintptr_t>(a.y16) & 15u) == 0;
  const int per_thread = (y16_aligned && a.H % 8 == 0) ? 8 : (a.H % 4) == 0 ? 4 : 1;
  const int threads = 64;
  dim3 grid(static_cast<unsigned>(ceil_div(ceil_div(a.H, per_thread), threads)),
            static_cast<unsigned>(std::min(a.T, 65535)));
  if (per_thread == 8) combine_kernel<8><<<grid, threads, 0, stream>>>(a);
  else if (per_thread == 4) combine_kernel<4><<<grid, threads, 0, stream>>>(a);
  else combine_kernel<1><<<grid, threads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace moe
