// Warp-specialised grouped FP8 GEMV: bulk-copy (TMA) weight ring + FMA warps.
//
// Same work and numerics as grouped_gemv_kernel (fp8_gemv.cu) -- chunks of up
// to NT token rows of one expert times row tiles, e4m3 decoded exactly (codes
// 0x7F/0xFF as +0, fp8_linear.cpp:31-33 of the reference), fp32 products, each
// 16-column partial scaled by its 128x128 block scale -- but the weights reach
// the FMA warps through shared memory:
//
//   warp 0      producer: per (row tile, 1 KiB k-slice) it issues one
//               cp.async.bulk per (row, stream) into a ring stage and arms the
//               stage's "full" mbarrier with the byte count;
//   warps 1..8  consumers: wait "full", multiply the slice against the staged
//               activation rows, release the stage through its "empty"
//               mbarrier.
//
// With 4-6 stages of 32 KiB the SM keeps 128-192 KiB of weight reads in
// flight without spending registers on them, which is what a 148-SM part
// needs to stream HBM at full rate.  Each CTA walks a contiguous range of
// work items, so the staged activation rows change only at chunk boundaries.
#include <algorithm>

#include "async_copy.cuh"
#include "common.cuh"
#include "fp8_gemv.cuh"

namespace moe {

constexpr int kConsumerWarps = 8;
constexpr int kStreamThreads = (kConsumerWarps + 1) * kWarp;
constexpr int kSlice = 1024;  // bytes of one weight row per ring stage
constexpr size_t kSmemBudget = 225 * 1024;

MOE_HD size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

MOE_D float silu_mul_s(float g, float u) {
  const float silu = g / (1.0f + expf(-g));
  return silu * u;
}

template <typename XT, int NT, int NS, int EPI>
__global__ void __launch_bounds__(kStreamThreads, 1) stream_gemv_kernel(GemvArgs a, int stages) {
  constexpr int RW = 4 / NS;                    // rows per consumer warp
  constexpr int R = kConsumerWarps * RW;        // rows per work item
  constexpr size_t kStageBytes = static_cast<size_t>(R) * NS * kSlice;
  extern __shared__ __align__(128) unsigned char smem[];
  const int K = a.K, N = a.N;
  XT* xs = reinterpret_cast<XT*>(smem);
  unsigned char* ring = smem + align_up(static_cast<size_t>(NT) * K * sizeof(XT), 128);
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + stages * kStageBytes);
  uint64_t* empty = full + stages;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  const int n_chunks = *a.n_chunks;
  const int row_tiles = static_cast<int>(ceil_div(N, R));
  const int nslice = static_cast<int>(ceil_div(K, kSlice));
  const int64_t work = static_cast<int64_t>(n_chunks) * row_tiles;
  const int64_t w_lo = work * blockIdx.x / gridDim.x;
  const int64_t w_hi = work * (blockIdx.x + 1) / gridDim.x;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    uint32_t it = 0;
    bool ok = true;
    for (int64_t wi = w_lo; wi < w_hi && ok; ++wi) {
      const int c = static_cast<int>(wi / row_tiles);
      const int r0 = static_cast<int>(wi % row_tiles) * R;
      const int seg = a.chunk_seg[c];
      const uint8_t* wb0 = reinterpret_cast<const uint8_t*>(a.w0[seg]);
      const uint8_t* wb1 = NS == 2 ? reinterpret_cast<const uint8_t*>(a.w1[seg]) : nullptr;
      bool present = wb0 && a.s0[seg] && (NS == 1 || (wb1 && a.s1[seg]));
      if (present && ((reinterpret_cast<uintptr_t>(wb0) | reinterpret_cast<uintptr_t>(wb1)) & 15u) != 0) {
        // bulk copies need 16-byte aligned sources: refuse loudly, compute nothing
        if (lane == 0) atomicOr(&g_device_error, 8);
        present = false;
      }
      const int rows_valid = min(R, N - r0);
      for (int s = 0; s < nslice; ++s, ++it) {
        const uint32_t stage = it % stages, use = it / stages;
        if (!mbar_wait(&empty[stage], (use & 1u) ^ 1u, 1)) {
          ok = false;
          break;
        }
        const int k0 = s * kSlice;
        const int sl = min(kSlice, K - k0);
        const uint32_t bytes = present ? static_cast<uint32_t>(rows_valid * NS * sl) : 0u;
        if (lane == 0) {
          if (bytes) mbar_arrive_expect_tx(&full[stage], bytes);
          else mbar_arrive(&full[stage]);
        }
        __syncwarp();
        if (present && lane < R * NS) {
          const int row = r0 + lane / NS;
          if (row < N) {
            const uint8_t* src = ((lane % NS) == 0 ? wb0 : wb1) + static_cast<int64_t>(row) * K + k0;
            bulk_copy_g2s(ring + stage * kStageBytes + static_cast<size_t>(lane) * kSlice, src,
                          static_cast<uint32_t>(sl), &full[stage]);
          }
        }
      }
    }
    if (!ok) {
      // a consumer stopped: let the copies already issued land before exiting
      const uint32_t first = it > static_cast<uint32_t>(stages) ? it - stages : 0u;
      for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % stages], (j / stages) & 1u, 4);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int cw = warp - 1;
  const int ctid = threadIdx.x - kWarp;
  constexpr int kConsumerThreads = kConsumerWarps * kWarp;
  uint32_t it = 0;
  int staged = -1;
  for (int64_t wi = w_lo; wi < w_hi; ++wi) {
    const int c = static_cast<int>(wi / row_tiles);
    const int rt = static_cast<int>(wi % row_tiles);
    const int seg = a.chunk_seg[c], p0 = a.chunk_start[c], len = a.chunk_len[c];
    if (c != staged) {
      named_barrier_sync(1, kConsumerThreads);
      for (int t = 0; t < NT; ++t) {
        XT* dst = xs + static_cast<int64_t>(t) * K;
        if (t < len) {
          const int64_t src_row = a.pair_row ? a.pair_row[p0 + t] : static_cast<int64_t>(p0 + t);
          const uint4* src = reinterpret_cast<const uint4*>(static_cast<const XT*>(a.x) + src_row * K);
          const int n16 = K * static_cast<int>(sizeof(XT)) / 16;
          for (int i = ctid; i < n16; i += kConsumerThreads) reinterpret_cast<uint4*>(dst)[i] = __ldg(src + i);
        } else {
          for (int i = ctid; i < K; i += kConsumerThreads) dst[i] = XT(0.0f);
        }
      }
      named_barrier_sync(1, kConsumerThreads);
      staged = c;
    }
    const bool present = a.w0[seg] && a.s0[seg] && (NS == 1 || (a.w1[seg] && a.s1[seg])) &&
                         ((a.w0[seg] | (NS == 2 ? a.w1[seg] : 0ull)) & 15ull) == 0;
    const float* sb0 = reinterpret_cast<const float*>(a.s0[seg]);
    const float* sb1 = NS == 2 ? reinterpret_cast<const float*>(a.s1[seg]) : nullptr;
    const int rbase = rt * R + cw * RW;
    // stream q: row rbase + q / NS, matrix q % NS, ring slot (cw * RW + q / NS) * NS + q % NS
    const float* sp[4];
    bool live[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int row = rbase + q / NS;
      live[q] = row < N;
      const float* sb = (q % NS) == 0 ? sb0 : sb1;
      sp[q] = (sb && live[q]) ? sb + static_cast<int64_t>(row / kBlock) * a.scale_cols : nullptr;
    }
    float acc[4][NT];
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[q][t] = 0.0f;

    bool ok = true;
    for (int s = 0; s < nslice; ++s, ++it) {
      const uint32_t stage = it % stages, use = it / stages;
      if (!mbar_wait(&full[stage], use & 1u, 2)) {
        ok = false;
        break;
      }
      if (present) {
        const unsigned char* st = ring + stage * kStageBytes;
#pragma unroll
        for (int jj = 0; jj < kSlice / 16 / kWarp; ++jj) {
          const int j = lane + jj * kWarp;
          const int kbyte = s * kSlice + j * 16;
          if (kbyte < K) {
            uint4 raw[4];
            float sc[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int slot = (cw * RW + q / NS) * NS + q % NS;
              raw[q] = *reinterpret_cast<const uint4*>(st + static_cast<size_t>(slot) * kSlice + j * 16);
              sc[q] = sp[q] ? __ldg(sp[q] + kbyte / kBlock) : 0.0f;
            }
            float part[4][NT];
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
              for (int t = 0; t < NT; ++t) part[q][t] = 0.0f;
#pragma unroll
            for (int w4 = 0; w4 < 4; ++w4) {
              float wv[4][4];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const uint32_t word = w4 == 0 ? raw[q].x : w4 == 1 ? raw[q].y : w4 == 2 ? raw[q].z : raw[q].w;
                e4m3x4_to_float4(word, wv[q]);
              }
#pragma unroll
              for (int t = 0; t < NT; ++t) {
                if (t < len) {
                  float xv[4];
                  load4<XT>(xs + static_cast<int64_t>(t) * K + kbyte + w4 * 4, xv);
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
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
    }
    if (!ok) return;

    float mine[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const float v = warp_sum(acc[q][t]);
        if (lane == t) mine[q] = v;
      }
    if (lane < len) {
      const int64_t p = p0 + lane;
#pragma unroll
      for (int i = 0; i < RW; ++i) {
        const int r = rbase + i;
        if (!live[i * NS]) continue;
        if (EPI == kEpiSwiglu) {
          a.out0[p * N + r] = silu_mul_s(mine[i * 2], mine[i * 2 + 1]);
        } else if (EPI == kEpiStore) {
          a.out0[p * N + r] = mine[i];
        } else {
          a.out0[p * N + r] = mine[i * 2];
          a.out1[p * N + r] = mine[i * 2 + 1];
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

template <typename XT, int NT, int NS>
static size_t stream_smem(int K, int stages) {
  constexpr int R = kConsumerWarps * (4 / NS);
  return align_up(static_cast<size_t>(NT) * K * sizeof(XT), 128) + static_cast<size_t>(stages) * R * NS * kSlice +
         2 * sizeof(uint64_t) * stages;
}

template <typename XT, int NT, int NS, int EPI>
static cudaError_t stream_launch_t(const GemvArgs& a, cudaStream_t stream) {
  constexpr int R = kConsumerWarps * (4 / NS);
  const size_t per_stage = static_cast<size_t>(R) * NS * kSlice + 2 * sizeof(uint64_t);
  const size_t fixed = align_up(static_cast<size_t>(NT) * a.K * sizeof(XT), 128);
  if (fixed + 2 * per_stage > kSmemBudget) return cudaErrorInvalidValue;
  const int stages = static_cast<int>(std::min<size_t>(6, (kSmemBudget - fixed) / per_stage));
  const size_t smem = stream_smem<XT, NT, NS>(a.K, stages);
  auto kernel = stream_gemv_kernel<XT, NT, NS, EPI>;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  kernel<<<gemv_grid_ctas(), kStreamThreads, smem, stream>>>(a, stages);
  return cudaGetLastError();
}

template <typename XT, int NS, int EPI>
static cudaError_t stream_launch_nt(const GemvArgs& a, int nt, cudaStream_t stream) {
  switch (nt) {
    case 1: return stream_launch_t<XT, 1, NS, EPI>(a, stream);
    case 4: return stream_launch_t<XT, 4, NS, EPI>(a, stream);
    case 8: return stream_launch_t<XT, 8, NS, EPI>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

bool stream_gemv_supported(int K, int x_dtype, int nt) {
  if (K % 16 != 0) return false;
  const size_t xb = static_cast<size_t>(nt) * K * (x_dtype == kXF32 ? 4 : 2);
  return align_up(xb, 128) + 2 * (32 * kSlice + 16) <= kSmemBudget;
}

cudaError_t launch_stream_gemv(const GemvArgs& a, int x_dtype, int ns, int epi, int nt, cudaStream_t stream) {
  if (x_dtype == kXBF16) {
    if (ns == 2 && epi == kEpiSwiglu) return stream_launch_nt<__nv_bfloat16, 2, kEpiSwiglu>(a, nt, stream);
    if (ns == 1 && epi == kEpiStore) return stream_launch_nt<__nv_bfloat16, 1, kEpiStore>(a, nt, stream);
    if (ns == 2 && epi == kEpiStoreBoth) return stream_launch_nt<__nv_bfloat16, 2, kEpiStoreBoth>(a, nt, stream);
  } else {
    if (ns == 2 && epi == kEpiSwiglu) return stream_launch_nt<float, 2, kEpiSwiglu>(a, nt, stream);
    if (ns == 1 && epi == kEpiStore) return stream_launch_nt<float, 1, kEpiStore>(a, nt, stream);
    if (ns == 2 && epi == kEpiStoreBoth) return stream_launch_nt<float, 2, kEpiStoreBoth>(a, nt, stream);
  }
  return cudaErrorInvalidValue;
}

int read_and_clear_device_error(cudaStream_t stream) { return read_and_clear_local_error(stream); }

}  // namespace moe
