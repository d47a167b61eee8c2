// Grouped FP8 GEMV on the warp MMA pipe (decode batches, layer path).
//
// The decode GEMV is bound by HBM, but decoding e4m3 and multiplying on the
// FMA pipe costs about three instructions per weight byte, which is as much
// issue bandwidth as an SM has at 6.5 TB/s.  Here every warp streams 16 (or
// 32) weight rows with 16-byte loads, turns each e4m3 pair into an f16 pair
// with one exact conversion, and lets mma.m16n8k16 (fp32 accumulate) do the
// products against up to 8 token rows: about one instruction per weight byte,
// whatever the number of tokens up to 8.  The tensor pipe is idle otherwise;
// its throughput is not what this kernel needs.
//
// Fragment trick: a dot product is invariant under any permutation of k
// applied to both operands.  Lane (g = lane/4, c = lane%4) loads bytes
// [16c, 16c+16) of a 64-byte k-span of rows g and g+8; in k-step s it feeds
// word s of that load as its A fragment (low byte pair -> logical k 2c, 2c+1,
// high pair -> 2c+8, 2c+9) and the matching activations x[16c+4s .. +3] of
// token g as its B fragment, so the four k-steps of a span cover its 64
// physical columns exactly once.
//
// Scales: the two spans of a 128-column k-block accumulate into a fresh
// fp32 fragment, which is then multiplied by that block's weight scale and
// added to the running sums -- the reference's "sum the block, then scale"
// (fp8_linear.cpp:103-112).  Activations are staged as f16 divided by a
// per-row power of two (rows_to_f16_kernel), undone in the epilogue, so any
// fp32/bf16 magnitude survives and bf16 inputs stay exact.
#include <cuda_fp16.h>

#include <algorithm>

#include "async_copy.cuh"
#include "common.cuh"
#include "fp8_gemv.cuh"

namespace moe {

constexpr int kMmaCtaWarps = 4;

MOE_D void mma_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

MOE_D uint4 ldg_stream(const void* p) { return __ldcs(reinterpret_cast<const uint4*>(p)); }

MOE_D uint32_t word_of(const uint4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// One 128-column k-block of operands for one lane.
struct KBlock {
  uint4 a[2][2][2];  // [span][stream][row g, row g+8]
  uint4 b[2][2];     // [span][lo 8 halfs, hi 8 halfs] of the lane's token row
};

// Activation rows -> f16 with a per-row power-of-two scale:
// dst[r, k] = src[r, k] / scale[r], scale = 2^(floor(log2(amax)) - 13) so the
// largest magnitude lands in [2^13, 2^14) (1 for an all-zero row).

// Activation rows -> f16 with a per-row power-of-two scale:
// dst[r, k] = src[r, k] / scale[r], scale = 2^(floor(log2(amax)) - 13) so the
// largest magnitude lands in [2^13, 2^14) (1 for an all-zero row).  One CTA
// per row, 16-byte loads (K * sizeof(T) must be a multiple of 16).
// The same for rows of at most P x 256 x 16 bytes (P <= 16: K <= 16384 fp32 or
// 32768 16-bit values): each thread keeps its P 16-byte pieces in registers
// between the max and the conversion, so a row is read once.
template <typename T, int P>
__global__ void __launch_bounds__(256) rows_to_f16_regs_kernel(const T* __restrict__ src, int rows, int K,
                                                               const int32_t* __restrict__ n_rows_dev,
                                                               __half* __restrict__ dst, float* __restrict__ scale,
                                                               int32_t* __restrict__ zero, int64_t zero_n) {
  constexpr int V = 16 / sizeof(T);
  __shared__ float red[8];
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < zero_n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    zero[i] = 0;
  const int n_rows = n_rows_dev ? min(rows, *n_rows_dev) : rows;
  const int n16 = K / V;
  for (int r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const uint4* s = reinterpret_cast<const uint4*>(src + static_cast<int64_t>(r) * K);
    uint4 v[P];
    float amax = 0.0f;
#pragma unroll
    for (int q = 0; q < P; ++q) {
      const int i = threadIdx.x + q * 256;
      v[q] = i < n16 ? __ldg(s + i) : make_uint4(0, 0, 0, 0);
      float f[V];
      unpack16<T>(v[q], f);
#pragma unroll
      for (int j = 0; j < V; ++j) amax = fmaxf(amax, fabsf(f[j]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    if (threadIdx.x % kWarp == 0) red[threadIdx.x / kWarp] = amax;
    __syncthreads();
    if (threadIdx.x < kWarp) {
      float w = threadIdx.x < blockDim.x / kWarp ? red[threadIdx.x] : 0.0f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) w = fmaxf(w, __shfl_xor_sync(0xFFFFFFFFu, w, o));
      if (threadIdx.x == 0) red[0] = w;
    }
    __syncthreads();
    amax = red[0];
    const float sc = (amax > 0.0f && isfinite(amax)) ? ldexpf(1.0f, ilogbf(amax) - 13) : 1.0f;
    const float inv = 1.0f / sc;  // exact: power of two
    __half* d = dst + static_cast<int64_t>(r) * K;
#pragma unroll
    for (int q = 0; q < P; ++q) {
      const int i = threadIdx.x + q * 256;
      if (i >= n16) continue;
      float f[V];
      unpack16<T>(v[q], f);
      __align__(16) __half h[V];
#pragma unroll
      for (int j = 0; j < V; ++j) h[j] = __float2half_rn(f[j] * inv);
      if (V == 8) {
        *reinterpret_cast<uint4*>(d + i * V) = *reinterpret_cast<const uint4*>(h);
      } else {
        *reinterpret_cast<uint2*>(d + i * V) = *reinterpret_cast<const uint2*>(h);
      }
    }
    if (threadIdx.x == 0) scale[r] = sc;
    __syncthreads();
  }
}

template <typename T>
__global__ void __launch_bounds__(256) rows_to_f16_kernel(const T* __restrict__ src, int rows, int K,
                                                          const int32_t* __restrict__ n_rows_dev,
                                                          __half* __restrict__ dst, float* __restrict__ scale,
                                                          int32_t* __restrict__ zero, int64_t zero_n) {
  constexpr int V = 16 / sizeof(T);
  __shared__ float red[8];
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < zero_n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    zero[i] = 0;
  const int n_rows = n_rows_dev ? min(rows, *n_rows_dev) : rows;
  const int n16 = K / V;
  for (int r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const uint4* s = reinterpret_cast<const uint4*>(src + static_cast<int64_t>(r) * K);
    float amax = 0.0f;
#pragma unroll 4
    for (int i = threadIdx.x; i < n16; i += blockDim.x) {
      float v[V];
      unpack16<T>(__ldg(s + i), v);
#pragma unroll
      for (int j = 0; j < V; ++j) amax = fmaxf(amax, fabsf(v[j]));
    }
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
    const float sc = (amax > 0.0f && isfinite(amax)) ? ldexpf(1.0f, ilogbf(amax) - 13) : 1.0f;
    const float inv = 1.0f / sc;  // exact: power of two
    __half* d = dst + static_cast<int64_t>(r) * K;
#pragma unroll 4
    for (int i = threadIdx.x; i < n16; i += blockDim.x) {
      float v[V];
      unpack16<T>(__ldg(s + i), v);
      __align__(16) __half h[V];
#pragma unroll
      for (int j = 0; j < V; ++j) h[j] = __float2half_rn(v[j] * inv);
      if (V == 8) {
        *reinterpret_cast<uint4*>(d + i * V) = *reinterpret_cast<const uint4*>(h);
      } else {
        *reinterpret_cast<uint2*>(d + i * V) = *reinterpret_cast<const uint2*>(h);
      }
    }
    if (threadIdx.x == 0) scale[r] = sc;
    __syncthreads();
  }
}

// A task is (chunk of <= 8 pairs, row tile): 16 rows of two matrices (gate +
// up, SwiGLU epilogue) when NS == 2, 32 rows of one matrix as two 16-row tiles
// when NS == 1.  Each warp streams the k-blocks [kb0, kb1) of one task with
// ping-pong register buffers.  With a.ksplit == 1 that range is all of K and
// the warp writes the outputs itself.  With a.ksplit > 1 (too few tasks to
// occupy every warp, e.g. one-token batches) a task's k-blocks are cut into
// ksplit ranges taken by different warps: each writes its fp32 fragment to
// a.partial, and the warp arriving last at the task's counter adds the
// partials in range order -- the same order whoever arrives last -- runs the
// epilogue and resets the counter to zero for the next launch.
template <int NS, int EPI>
__global__ void __launch_bounds__(kMmaCtaWarps * kWarp) mma_gemv_kernel(MmaArgs a) {
  const int lane = threadIdx.x % kWarp;
  const int g = lane / 4, c = lane % 4;
  const int K = a.K, N = a.N;
  constexpr int kTaskRows = NS == 2 ? 16 : 32;
  const int row_tiles = static_cast<int>(ceil_div(N, kTaskRows));
  const int ksplit = a.ksplit;
  const int64_t tasks = static_cast<int64_t>(*a.n_chunks) * row_tiles;
  const int64_t units = tasks * ksplit;
  const int64_t warp_global = static_cast<int64_t>(blockIdx.x) * kMmaCtaWarps + threadIdx.x / kWarp;
  const int64_t warp_count = static_cast<int64_t>(gridDim.x) * kMmaCtaWarps;
  const int nkb = K / kBlock;

  for (int64_t unit = warp_global; unit < units; unit += warp_count) {
    const int64_t task = unit / ksplit;
    const int ks = static_cast<int>(unit % ksplit);
    const int kb0 = static_cast<int>(static_cast<int64_t>(ks) * nkb / ksplit);
    const int kb1 = static_cast<int>(static_cast<int64_t>(ks + 1) * nkb / ksplit);
    const int ch = static_cast<int>(task / row_tiles);
    const int r0 = static_cast<int>(task % row_tiles) * kTaskRows;
    const int seg = a.chunk_seg[ch], p0 = a.chunk_start[ch], len = a.chunk_len[ch];
    const uint8_t* w0 = reinterpret_cast<const uint8_t*>(a.w0[seg]);
    const float* s0 = reinterpret_cast<const float*>(a.s0[seg]);
    const uint8_t* w1 = NS == 2 ? reinterpret_cast<const uint8_t*>(a.w1[seg]) : w0;
    const float* s1 = NS == 2 ? reinterpret_cast<const float*>(a.s1[seg]) : s0;
    const bool present = w0 && s0 && w1 && s1 &&
                         ((reinterpret_cast<uintptr_t>(w0) | reinterpret_cast<uintptr_t>(w1)) & 15u) == 0;

    // A rows of this lane: stream st, row half rr
    const uint8_t* arow[2][2];
    const float* srow[2];
#pragma unroll
    for (int st = 0; st < 2; ++st) {
      const int base = NS == 2 ? r0 : r0 + 16 * st;
      const uint8_t* w = st == 0 ? w0 : w1;
      const float* sc = st == 0 ? s0 : s1;
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int row = min(base + g + 8 * rr, N - 1);
        arow[st][rr] = present ? w + static_cast<int64_t>(row) * K + 16 * c : nullptr;
      }
      srow[st] = present ? sc + static_cast<int64_t>(min(base, N - 1) / kBlock) * a.scale_cols : nullptr;
    }
    // B row: token g of the chunk
    const bool bvalid = g < len;
    const int64_t brow = bvalid ? (a.pair_row ? a.pair_row[p0 + g] : static_cast<int64_t>(p0 + g)) : 0;
    const __half* xb = a.x16 + brow * K + 16 * c;

    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    if (present && kb0 < kb1) {
      auto load = [&](KBlock& kb, int kbi) {
#pragma unroll
        for (int sp = 0; sp < 2; ++sp) {
          const int off = kbi * kBlock + sp * 64;
#pragma unroll
          for (int st = 0; st < 2; ++st)
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) kb.a[sp][st][rr] = ldg_stream(arow[st][rr] + off);
          if (bvalid) {
            kb.b[sp][0] = __ldg(reinterpret_cast<const uint4*>(xb + off));
            kb.b[sp][1] = __ldg(reinterpret_cast<const uint4*>(xb + off + 8));
          } else {
            kb.b[sp][0] = make_uint4(0, 0, 0, 0);
            kb.b[sp][1] = make_uint4(0, 0, 0, 0);
          }
        }
      };
      auto compute = [&](const KBlock& kb, int kbi) {
        float t[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int sp = 0; sp < 2; ++sp) {
          const uint32_t bw[8] = {kb.b[sp][0].x, kb.b[sp][0].y, kb.b[sp][0].z, kb.b[sp][0].w,
                                  kb.b[sp][1].x, kb.b[sp][1].y, kb.b[sp][1].z, kb.b[sp][1].w};
#pragma unroll
          for (int s = 0; s < 4; ++s) {
#pragma unroll
            for (int st = 0; st < 2; ++st) {
              uint32_t wg = word_of(kb.a[sp][st][0], s);
              uint32_t wh = word_of(kb.a[sp][st][1], s);
              if (a.nanfix) {
                wg = e4m3x4_nan_to_zero(wg);
                wh = e4m3x4_nan_to_zero(wh);
              }
              uint32_t g0, g1, h0, h1;
              e4m3x4_to_f16x2x2(wg, g0, g1);
              e4m3x4_to_f16x2x2(wh, h0, h1);
              mma_16816(t[st], g0, h0, g1, h1, bw[2 * s], bw[2 * s + 1]);
            }
          }
        }
#pragma unroll
        for (int st = 0; st < 2; ++st) {
          const float sc = __ldg(srow[st] + kbi);
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[st][i] = fmaf(t[st][i], sc, acc[st][i]);
        }
      };
      // ping-pong register buffers, one k-block of loads in flight ahead of the math
      KBlock buf0, buf1;
      load(buf0, kb0);
      for (int kbi = kb0; kbi < kb1; kbi += 2) {
        if (kbi + 1 < kb1) load(buf1, kbi + 1);
        compute(buf0, kbi);
        if (kbi + 1 < kb1) {
          if (kbi + 2 < kb1) load(buf0, kbi + 2);
          compute(buf1, kbi + 1);
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
            const float gv = acc[0][i] * xs, uv = acc[1][i] * xs;
            const float silu = gv / (1.0f + expf(-gv));
            a.out0[p * N + row] = EPI == kEpiSwiglu ? silu * uv : gv;
          }
        } else {
#pragma unroll
          for (int st = 0; st < 2; ++st) {
            const int row = r0 + 16 * st + g + 8 * rr;
            if (row < N) a.out0[p * N + row] = acc[st][i] * xs;
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// The same tasks with the operands staged through shared memory by cp.async:
// every warp owns a ring of kAsyncStages k-blocks; lane l copies its own
// 8 x 16 bytes of weights and 4 x 16 bytes of activations of a k-block (the
// bytes it multiplies) to slots (i * 32 + l) * 16 of a stage and later reads
// exactly those bytes back, so the ring needs no barrier -- only the lane's
// own cp.async groups (commit / wait_group).  kAsyncStages - 1 k-blocks of
// every lane stay in flight without holding registers, and the block scales
// are loaded one k-block ahead.  Experts flagged NaN-free skip the 0x7F/0xFF
// fix-up (a warp-uniform choice per task).
// ---------------------------------------------------------------------------
constexpr int kAsyncWarps = 4;
constexpr int kAsyncStages = 3;
constexpr int kAsyncStageBytes = kWarp * 12 * 16;  // 6 KiB: a k-block of the warp's 32 row streams + its activations
constexpr int kAsyncSmem = kAsyncWarps * kAsyncStages * kAsyncStageBytes;
// Fragment-native ("tiled") weight layout: tiled_offset (fp8_gemv.cuh).  A
// row tile's k-block is two 1 KiB halves (sp) 8 KiB apart; consecutive
// k-blocks of a row tile are 16 KiB apart.
constexpr int kTileKBlockStride = 2 * kTileRunBytes;

MOE_D void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem)), "l"(gmem) : "memory");
}
// src_bytes < 16 zero-fills the rest of the 16-byte destination (0: all zeros, nothing read)
MOE_D void cp_async16_zfill(void* smem, const void* gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(smem)), "l"(gmem), "r"(src_bytes)
               : "memory");
}
MOE_D void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
MOE_D void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// One warp unit's operand addresses: a task's k-range [kb0, kb1) (empty when
// the expert is absent).  TILED: the weights are in the fragment-native layout
// of fp8_tile_kernel (tbase[st] = this lane's 16 bytes of piece rr = 0, half
// sp = 0 of k-block 0 of stream st's 16-row tile); otherwise row-major
// (arow[st][rr] = row g + 8 rr at column 16 c).
struct UnitOperands {
  const uint8_t* arow[2][2];
  const uint8_t* tbase[2];
  const float* srow[2];
  const __half* xb;
  bool bvalid;
  int kb0, kb1;
  int rot;  // the unit's k-blocks are streamed from kb0 + rot, wrapping to kb0 (0: in order)
};

// acc += this lane's share of W[k-blocks kb0..kb1) . x for unit u.  The warp's
// ring is one pipeline across its units: step j of u sits in stage (step0 + j)
// % kAsyncStages, the first `primed` steps of u were issued by the previous
// unit, and in its last k-blocks this unit issues the first steps of the next
// unit `nx` (returned: how many), so the ring does not drain between units.
// Every iteration commits one cp.async group (possibly empty) and the prologue
// kAsyncStages - 1 - primed, so kAsyncStages - 1 newer groups always follow
// the one being waited for.  Each lane reads only its own ring slots.
template <bool FIX, bool TILED>
MOE_D int async_accumulate(float (&acc)[2][4], unsigned char* ring, const UnitOperands& u, const UnitOperands& nx,
                           uint32_t step0, int primed, int lane) {
  auto slot = [&](uint32_t stage, int i) { return ring + stage * kAsyncStageBytes + (i * kWarp + lane) * 16; };
  // slots 0-7: this lane's weight pieces (span, stream, row half); 8-11: its
  // activation pieces (span, half); an absent token row is zero-filled
  auto issue = [&](const UnitOperands& o, int kbi, uint32_t step) {
    const uint32_t stage = step % kAsyncStages;
#pragma unroll
    for (int sp = 0; sp < 2; ++sp) {
#pragma unroll
      for (int st = 0; st < 2; ++st)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr)
          cp_async16(slot(stage, (sp * 2 + st) * 2 + rr),
                     TILED ? o.tbase[st] + static_cast<int64_t>(kbi) * kTileKBlockStride + sp * kTileRunBytes + rr * (kWarp * 16)
                           : o.arow[st][rr] + kbi * kBlock + sp * 64);
#pragma unroll
      for (int h = 0; h < 2; ++h)
        cp_async16_zfill(slot(stage, 8 + sp * 2 + h), o.xb + kbi * kBlock + sp * 64 + h * 8, o.bvalid ? 16 : 0);
    }
  };
  const int kb0 = u.kb0, kb1 = u.kb1, n = kb1 - kb0;
  const int nx_steps = nx.kb1 - nx.kb0;
  // k-block of step j of a unit (its rotation applied)
  auto kb_of = [](const UnitOperands& o, int j) {
    const int m = o.kb1 - o.kb0;
    const int r = j + o.rot;
    return o.kb0 + (r >= m ? r - m : r);
  };
  int nx_issued = 0;
  for (int j = primed; j < kAsyncStages - 1; ++j) {
    if (j < n) issue(u, kb_of(u, j), step0 + j);
    cp_async_commit();
  }
  float sc0 = __ldg(u.srow[0] + kb_of(u, 0)), sc1 = __ldg(u.srow[1] + kb_of(u, 0));
  for (int j = 0; j < n; ++j) {
    const int ahead = j + kAsyncStages - 1;  // step of u (or beyond: of nx) to issue now
    if (ahead < n) {
      issue(u, kb_of(u, ahead), step0 + ahead);
    } else if (nx_issued < nx_steps && nx_issued < kAsyncStages - 1) {
      issue(nx, kb_of(nx, nx_issued), step0 + n + nx_issued);
      ++nx_issued;
    }
    cp_async_commit();
    // next k-block's scales load while this one is multiplied
    const int kn = kb_of(u, min(j + 1, n - 1));
    const float nsc0 = __ldg(u.srow[0] + kn), nsc1 = __ldg(u.srow[1] + kn);
    cp_async_wait<kAsyncStages - 1>();  // this lane's copies of step j have landed
    const uint32_t stage = (step0 + j) % kAsyncStages;
    float t[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int sp = 0; sp < 2; ++sp) {
      uint4 av[2][2];
#pragma unroll
      for (int st = 0; st < 2; ++st)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr)
          av[st][rr] = *reinterpret_cast<const uint4*>(slot(stage, (sp * 2 + st) * 2 + rr));
      const uint4 b0 = *reinterpret_cast<const uint4*>(slot(stage, 8 + sp * 2));
      const uint4 b1 = *reinterpret_cast<const uint4*>(slot(stage, 8 + sp * 2 + 1));
      const uint32_t bw[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int s = 0; s < 4; ++s) {
#pragma unroll
        for (int st = 0; st < 2; ++st) {
          uint32_t wg = word_of(av[st][0], s);
          uint32_t wh = word_of(av[st][1], s);
          if (FIX) {
            wg = e4m3x4_nan_to_zero(wg);
            wh = e4m3x4_nan_to_zero(wh);
          }
          uint32_t g0, g1, h0, h1;
          e4m3x4_to_f16x2x2(wg, g0, g1);
          e4m3x4_to_f16x2x2(wh, h0, h1);
          mma_16816(t[st], g0, h0, g1, h1, bw[2 * s], bw[2 * s + 1]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc[0][i] = fmaf(t[0][i], sc0, acc[0][i]);
      acc[1][i] = fmaf(t[1][i], sc1, acc[1][i]);
    }
    sc0 = nsc0;
    sc1 = nsc1;
  }
  return nx_issued;
}

// Rows [p0, p0 + len) of src (N fp32 each) -> f16 with a power-of-two row
// scale, by one warp: rows_to_f16_kernel's arithmetic (the same bits).  The
// rows were written by other warps of this launch: read from L2.
MOE_D void stage_rows_f16_warp(const float* src, int p0, int len, int N, __half* dst16, float* scale, int lane) {
  const int n4 = N / 4;
  for (int p = p0; p < p0 + len; ++p) {
    const float4* row = reinterpret_cast<const float4*>(src + static_cast<int64_t>(p) * N);
    float amax = 0.0f;
    for (int i0 = lane; i0 < n4; i0 += 8 * kWarp) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = i0 + u * kWarp < n4 ? __ldcg(row + i0 + u * kWarp) : make_float4(0, 0, 0, 0);
#pragma unroll
      for (int u = 0; u < 8; ++u)
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    const float sc = (amax > 0.0f && isfinite(amax)) ? ldexpf(1.0f, ilogbf(amax) - 13) : 1.0f;
    const float inv = 1.0f / sc;  // exact: power of two
    __half* dst = dst16 + static_cast<int64_t>(p) * N;
    for (int i = lane; i < n4; i += kWarp) {
      const float4 v = __ldcg(row + i);
      __align__(8) __half h[4] = {__float2half_rn(v.x * inv), __float2half_rn(v.y * inv),
                                  __float2half_rn(v.z * inv), __float2half_rn(v.w * inv)};
      *reinterpret_cast<uint2*>(dst + 4 * i) = *reinterpret_cast<const uint2*>(h);
    }
    if (lane == 0) scale[p] = sc;
  }
}

// Columns [c0, c0 + 32) of token t's combined row, one column per lane:
// combine_kernel's arithmetic.  The pair rows were written by other warps of
// this launch: read from L2.
MOE_D void combine_tile_warp(const MmaArgs& a, const float* y, int t, int c0, int lane) {
  const int col = c0 + lane;
  if (col >= a.N) return;
  float acc = 0.0f;
  for (int s = 0; s < a.comb_k; ++s) {
    const int p = a.entry_pair[static_cast<int64_t>(t) * a.comb_k + s];
    if (p < 0) continue;
    acc = fmaf(a.pair_weight[p], __ldcg(y + static_cast<int64_t>(p) * a.N + col), acc);
  }
  if (a.comb_shared_base >= 0) acc += __ldcg(y + static_cast<int64_t>(a.comb_shared_base + t) * a.N + col);
  a.comb_out[static_cast<int64_t>(t) * a.N + col] = __float2bfloat16_rn(acc);
}

template <int NS, int EPI, bool TILED>
__global__ void __launch_bounds__(kAsyncWarps * kWarp) mma_gemv_async_kernel(MmaArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int g = lane / 4, c = lane % 4;
  const int K = a.K, N = a.N;
  unsigned char* ring = smem + warp * kAsyncStages * kAsyncStageBytes;
  constexpr int kTaskRows = NS == 2 ? 16 : 32;
  const int row_tiles = static_cast<int>(ceil_div(N, kTaskRows));
  const int ksplit = a.ksplit;
  const int64_t tasks = static_cast<int64_t>(*a.n_chunks) * row_tiles;
  const int64_t units = tasks * ksplit;
  const int64_t warp_global = static_cast<int64_t>(blockIdx.x) * kAsyncWarps + warp;
  const int64_t warp_count = static_cast<int64_t>(gridDim.x) * kAsyncWarps;
  const int nkb = K / kBlock;

  // operand addresses of a unit (an empty k-range when out of range or the expert is absent)
  auto operands = [&](int64_t unit, UnitOperands& o, bool& fix) {
    o.kb0 = o.kb1 = 0;
    o.rot = 0;
    fix = false;
    if (unit >= units) return;
    const int64_t task = unit / ksplit;
    const int ks = static_cast<int>(unit % ksplit);
    const int ch = static_cast<int>(task / row_tiles);
    const int r0 = static_cast<int>(task % row_tiles) * kTaskRows;
    const int seg = a.chunk_seg[ch], p0 = a.chunk_start[ch], len = a.chunk_len[ch];
    const uint8_t* w0 = reinterpret_cast<const uint8_t*>(a.w0[seg]);
    const float* s0 = reinterpret_cast<const float*>(a.s0[seg]);
    const uint8_t* w1 = NS == 2 ? reinterpret_cast<const uint8_t*>(a.w1[seg]) : w0;
    const float* s1 = NS == 2 ? reinterpret_cast<const float*>(a.s1[seg]) : s0;
    const bool present = w0 && s0 && w1 && s1 &&
                         ((reinterpret_cast<uintptr_t>(w0) | reinterpret_cast<uintptr_t>(w1)) & 15u) == 0;
    if (!present) return;
#pragma unroll
    for (int st = 0; st < 2; ++st) {
      const int base = NS == 2 ? r0 : r0 + 16 * st;
      const uint8_t* w = st == 0 ? w0 : w1;
      const float* sc = st == 0 ? s0 : s1;
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int row = min(base + g + 8 * rr, N - 1);
        o.arow[st][rr] = w + static_cast<int64_t>(row) * K + 16 * c;
      }
      o.srow[st] = sc + static_cast<int64_t>(min(base, N - 1) / kBlock) * a.scale_cols;
      const int64_t tile = NS == 2 ? r0 / 16 : r0 / 16 + st;
      o.tbase[st] = w + tiled_offset(tile, 0, 0, nkb) + lane * 16;
    }
    o.bvalid = g < len;
    const int64_t brow = o.bvalid ? (a.pair_row ? a.pair_row[p0 + g] : static_cast<int64_t>(p0 + g)) : 0;
    o.xb = a.x16 + brow * K + 16 * c;
    o.kb0 = static_cast<int>(static_cast<int64_t>(ks) * nkb / ksplit);
    o.kb1 = static_cast<int>(static_cast<int64_t>(ks + 1) * nkb / ksplit);
    // staggered start: concurrent units do not walk the k-blocks in lockstep
    if (a.kb_rotate && o.kb1 > o.kb0) o.rot = static_cast<int>((unit * 37) % (o.kb1 - o.kb0));
    fix = a.nanfix && !(a.nan_free && a.nan_free[seg]);
  };

  UnitOperands cur, nxt;
  bool cur_fix, nxt_fix;
  operands(warp_global, cur, cur_fix);
  uint32_t step0 = 0;  // ring steps (k-blocks) of this warp's earlier units
  int primed = 0;      // k-blocks of `cur` already issued by the previous unit
  for (int64_t unit = warp_global; unit < units; unit += warp_count) {
    const int64_t task = unit / ksplit;
    const int ks = static_cast<int>(unit % ksplit);
    const int ch = static_cast<int>(task / row_tiles);
    const int r0 = static_cast<int>(task % row_tiles) * kTaskRows;
    const int p0 = a.chunk_start[ch], len = a.chunk_len[ch];
    operands(unit + warp_count, nxt, nxt_fix);

    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    const int n = cur.kb1 - cur.kb0;
    int nx_primed = 0;
    if (n > 0) {
      nx_primed = cur_fix ? async_accumulate<true, TILED>(acc, ring, cur, nxt, step0, primed, lane)
                          : async_accumulate<false, TILED>(acc, ring, cur, nxt, step0, primed, lane);
    }
    step0 += n;
    primed = nx_primed;
    cur = nxt;
    cur_fix = nxt_fix;

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
            const float gv = acc[0][i] * xs, uv = acc[1][i] * xs;
            const float silu = gv / (1.0f + expf(-gv));
            a.out0[p * N + row] = EPI == kEpiSwiglu ? silu * uv : gv;
          }
        } else {
#pragma unroll
          for (int st = 0; st < 2; ++st) {
            const int row = r0 + 16 * st + g + 8 * rr;
            if (row < N) a.out0[p * N + row] = acc[st][i] * xs;
          }
        }
      }
    }
    // folded follow-ups: the activation staging of a finished chunk (gate/up), the combine of
    // the token tiles this task completed (down)
    if (NS == 2 && a.chunk_done) {
      __threadfence();
      __syncwarp();
      int last = 0;
      if (lane == 0) last = atomicAdd(a.chunk_done + ch, 1) == row_tiles - 1;
      if (__shfl_sync(0xFFFFFFFFu, last, 0)) {
        __threadfence();
        stage_rows_f16_warp(a.out0, p0, len, N, a.stage_x16, a.stage_scale, lane);
      }
    } else if (NS == 1 && a.comb_out) {
      __threadfence();
      __syncwarp();
      const int tile = r0 / 32, tiles = static_cast<int>(ceil_div(N, 32));
      for (int j = 0; j < len; ++j) {
        const int t = a.pair_token[p0 + j];
        int last = 0;
        if (lane == 0) last = atomicAdd(a.comb_cnt + static_cast<int64_t>(t) * tiles + tile, 1) == a.comb_need - 1;
        if (__shfl_sync(0xFFFFFFFFu, last, 0)) {
          __threadfence();
          combine_tile_warp(a, a.out0, t, r0, lane);
        }
      }
    }
  }
  cp_async_wait<0>();  // no copy of this warp in flight when it exits
}

// ---------------------------------------------------------------------------
// Fused decode experts (tiled weights): gate/up + SwiGLU, the f16 staging of
// the SwiGLU activations and the down projection in ONE persistent launch of
// every resident warp -- the work of mma_gemv_async_kernel<2>,
// rows_to_f16_kernel<float> and mma_gemv_async_kernel<1> without two launch
// gaps and without the ramp and tail of three grids.
//
// Work split (per phase, "stream-K"): a phase's work is tasks x k-blocks
// "steps" (a task = chunk of <= 8 pairs x 16 rows of gate + up, or x 32 rows
// of down); warp w of the W used takes steps [w S / W, (w + 1) S / W), so every
// warp streams the same weight bytes.  A task whose steps fall to several
// warps has each piece written to a partial slot of its warp (2 per warp and
// phase: its first task, its last) and the warp adding the last piece sums
// the pieces in warp order -- the same order whoever arrives last -- then runs
// the epilogue.  Every warp does its gate/up range, then its down range.
//
// Dependency: when a chunk's last gate/up task is written, the warp that
// wrote it stages the chunk's activation rows to f16 with a power-of-two row
// scale (rows_to_f16_kernel's arithmetic, so the staged rows are the same
// bits) and publishes the chunk's ready flag (release).  A down piece of a
// chunk waits for that flag (acquire; bounded by kWaitLimitNs, after which
// the piece is skipped and kDecodeWaitError is recorded).  The wait always
// ends: every CTA is resident (the grid is the occupancy of this kernel),
// gate/up pieces never wait, and every warp finishes its gate/up range first.
// The counters and flags must be zero on entry (the x staging kernel clears
// them each forward).
// ---------------------------------------------------------------------------
constexpr int kDecodeWaitError = 128;

MOE_D int ld_acquire_gpu(const int32_t* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
MOE_D void st_release_gpu(int32_t* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// One phase's geometry on the device.
struct DecodePhase {
  int rows, row_tiles, nkb;
  int64_t tasks, steps, warps;  // warps: W used by this phase (0: no work)
  MOE_D int64_t lo(int64_t w) const { return w * steps / warps; }
  MOE_D int64_t hi(int64_t w) const { return (w + 1) * steps / warps; }
  // the warp whose range holds step s
  MOE_D int64_t warp_of(int64_t s) const { return ((s + 1) * warps - 1) / steps; }
};

MOE_D DecodePhase decode_phase(int N, int K, int ns, int n_chunks, int64_t W) {
  DecodePhase p;
  p.rows = ns == 2 ? 16 : 32;
  p.row_tiles = static_cast<int>(ceil_div(N, p.rows));
  p.nkb = K / kBlock;
  p.tasks = static_cast<int64_t>(n_chunks) * p.row_tiles;
  p.steps = p.tasks * p.nkb;
  // at least a quarter of a task per warp keeps the pieces of a task to five or fewer, and at most one
  // warp per step keeps every warp's range non-empty (a task's pieces then come from every warp between
  // the first and the last that hold its steps, which is what the arrival count expects)
  p.warps = p.steps > 0 ? max(int64_t{1}, min(min(W, p.steps), 4 * p.steps / max(p.nkb, 1))) : 0;
  return p;
}

// A warp's piece: task `task` of phase `ph`, k-blocks [kb0, kb1).
struct DecodeSeg {
  int ph;
  int64_t task;
  int kb0, kb1;
};

template <int PH>
MOE_D const MmaArgs& decode_args(const DecodeFusedArgs& a) {
  if constexpr (PH == 0) return a.up;
  else return a.down;
}

// Operand addresses of a piece of phase PH (an empty k-range when the expert is absent).
template <int PH>
MOE_D void decode_operands(const DecodeFusedArgs& a, const DecodePhase& P, const DecodeSeg& sg, int lane,
                           UnitOperands& o, bool& fix) {
  constexpr int NS = PH == 0 ? 2 : 1;
  const MmaArgs& m = decode_args<PH>(a);
  const int g = lane / 4, c = lane % 4;
  o.kb0 = o.kb1 = 0;
  o.rot = 0;
  fix = false;
  const int ch = static_cast<int>(sg.task / P.row_tiles);
  const int r0 = static_cast<int>(sg.task % P.row_tiles) * P.rows;
  const int seg = m.chunk_seg[ch], p0 = m.chunk_start[ch], len = m.chunk_len[ch];
  const uint8_t* w0 = reinterpret_cast<const uint8_t*>(m.w0[seg]);
  const float* s0 = reinterpret_cast<const float*>(m.s0[seg]);
  const uint8_t* w1 = NS == 2 ? reinterpret_cast<const uint8_t*>(m.w1[seg]) : w0;
  const float* s1 = NS == 2 ? reinterpret_cast<const float*>(m.s1[seg]) : s0;
  const bool present = w0 && s0 && w1 && s1 &&
                       ((reinterpret_cast<uintptr_t>(w0) | reinterpret_cast<uintptr_t>(w1)) & 15u) == 0;
  if (!present) return;
#pragma unroll
  for (int st = 0; st < 2; ++st) {
    const int base = NS == 2 ? r0 : r0 + 16 * st;
    const uint8_t* w = st == 0 ? w0 : w1;
    const float* sc = st == 0 ? s0 : s1;
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int row = min(base + g + 8 * rr, m.N - 1);
      o.arow[st][rr] = w + static_cast<int64_t>(row) * m.K + 16 * c;
    }
    o.srow[st] = sc + static_cast<int64_t>(min(base, m.N - 1) / kBlock) * m.scale_cols;
    const int64_t tile = NS == 2 ? r0 / 16 : r0 / 16 + st;
    o.tbase[st] = w + tiled_offset(tile, 0, 0, P.nkb) + lane * 16;
  }
  o.bvalid = g < len;
  const int64_t brow = o.bvalid ? (m.pair_row ? m.pair_row[p0 + g] : static_cast<int64_t>(p0 + g)) : 0;
  o.xb = m.x16 + brow * m.K + 16 * c;
  o.kb0 = sg.kb0;
  o.kb1 = sg.kb1;
  if (m.kb_rotate && sg.kb1 > sg.kb0) o.rot = static_cast<int>((sg.task * 37) % (sg.kb1 - sg.kb0));
  fix = m.nanfix && !(m.nan_free && m.nan_free[seg]);
}

// A finished task's outputs: SwiGLU of gate and up (PH 0, act) or the down rows (PH 1, y).
template <int PH>
MOE_D void decode_epilogue(const DecodeFusedArgs& a, const DecodePhase& P, const DecodeSeg& sg, int lane,
                           const float (&acc)[2][4], bool known_staged) {
  const MmaArgs& m = decode_args<PH>(a);
  const int g = lane / 4, c = lane % 4;
  const int ch = static_cast<int>(sg.task / P.row_tiles);
  const int r0 = static_cast<int>(sg.task % P.row_tiles) * P.rows;
  const int p0 = m.chunk_start[ch], len = m.chunk_len[ch];
  // the down phase's row scales are written in this launch: read from L2 once the chunk is published
  // (never, after a timed-out wait: its outputs are then written as zeros)
  int staged = 1;
  if (PH == 1 && !known_staged) {
    if (lane == 0) staged = ld_acquire_gpu(a.chunk_ready + ch);
    staged = __shfl_sync(0xFFFFFFFFu, staged, 0);
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int tok = 2 * c + j;
    if (tok >= len) continue;
    const int64_t tr = m.pair_row ? m.pair_row[p0 + tok] : static_cast<int64_t>(p0 + tok);
    const float xs = PH == 0 ? m.xscale[tr] : (staged ? __ldcg(m.xscale + tr) : 0.0f);
    const int64_t p = p0 + tok;
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int i = rr * 2 + j;
      if (PH == 0) {
        const int row = r0 + g + 8 * rr;
        if (row < m.N) {
          const float gv = acc[0][i] * xs, uv = acc[1][i] * xs;
          m.out0[p * m.N + row] = gv / (1.0f + expf(-gv)) * uv;
        }
      } else {
#pragma unroll
        for (int st = 0; st < 2; ++st) {
          const int row = r0 + 16 * st + g + 8 * rr;
          if (row < m.N) m.out0[p * m.N + row] = acc[st][i] * xs;
        }
      }
    }
  }
}

// Chunk ch's activation rows -> f16 with a power-of-two row scale, by one
// warp (rows_to_f16_kernel's arithmetic: the same bits).
MOE_D void decode_stage_chunk(const DecodeFusedArgs& a, int ch, int lane) {
  const int p0 = a.up.chunk_start[ch], len = a.up.chunk_len[ch];
  const int I = a.up.N;
  const int n4 = I / 4;
  for (int p = p0; p < p0 + len; ++p) {
    const float4* row = reinterpret_cast<const float4*>(a.up.out0 + static_cast<int64_t>(p) * I);
    float amax = 0.0f;
    for (int i0 = lane; i0 < n4; i0 += 8 * kWarp) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = i0 + u * kWarp < n4 ? __ldcg(row + i0 + u * kWarp) : make_float4(0, 0, 0, 0);
#pragma unroll
      for (int u = 0; u < 8; ++u)
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    const float sc = (amax > 0.0f && isfinite(amax)) ? ldexpf(1.0f, ilogbf(amax) - 13) : 1.0f;
    const float inv = 1.0f / sc;  // exact: power of two
    __half* dst = const_cast<__half*>(a.down.x16) + static_cast<int64_t>(p) * I;
    for (int i = lane; i < n4; i += kWarp) {
      const float4 v = __ldcg(row + i);
      __align__(8) __half h[4] = {__float2half_rn(v.x * inv), __float2half_rn(v.y * inv),
                                  __float2half_rn(v.z * inv), __float2half_rn(v.w * inv)};
      *reinterpret_cast<uint2*>(dst + 4 * i) = *reinterpret_cast<const uint2*>(h);
    }
    if (lane == 0) const_cast<float*>(a.down.xscale)[p] = sc;
  }
}

template <bool TILED>
__global__ void __launch_bounds__(kAsyncWarps * kWarp) decode_fused_kernel(DecodeFusedArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  unsigned char* ring = smem + warp * kAsyncStages * kAsyncStageBytes;
  const int64_t W = min(static_cast<int64_t>(gridDim.x) * kAsyncWarps, static_cast<int64_t>(a.partial_warps));
  const int64_t wg = static_cast<int64_t>(blockIdx.x) * kAsyncWarps + warp;
  if (wg >= W) return;
  const int n_chunks = *a.up.n_chunks;
  const DecodePhase ph0 = decode_phase(a.up.N, a.up.K, 2, n_chunks, W);
  const DecodePhase ph1 = decode_phase(a.down.N, a.down.K, 1, n_chunks, W);

  // the warp's pieces in order: its gate/up range, then its down range
  int cur_ph = 0;
  int64_t s_at = 0, s_end = 0;
  if (wg < ph0.warps) {
    s_at = ph0.lo(wg);
    s_end = ph0.hi(wg);
  }
  auto next_seg = [&](DecodeSeg& sg) -> bool {
    while (s_at >= s_end) {
      if (cur_ph == 1) return false;
      cur_ph = 1;
      s_at = s_end = 0;
      if (wg < ph1.warps) {
        s_at = ph1.lo(wg);
        s_end = ph1.hi(wg);
      }
    }
    const int nkb = cur_ph ? ph1.nkb : ph0.nkb;
    sg.ph = cur_ph;
    sg.task = s_at / nkb;
    sg.kb0 = static_cast<int>(s_at - sg.task * nkb);
    sg.kb1 = static_cast<int>(min(s_end - sg.task * nkb, static_cast<int64_t>(nkb)));
    s_at = (sg.task + 1) * nkb;
    return true;
  };
  auto operands = [&](const DecodeSeg& sg, UnitOperands& o, bool& fix) {
    if (sg.ph == 0) decode_operands<0>(a, ph0, sg, lane, o, fix);
    else decode_operands<1>(a, ph1, sg, lane, o, fix);
  };
  auto chunk_of = [&](const DecodeSeg& sg) {
    return static_cast<int>(sg.task / (sg.ph ? ph1.row_tiles : ph0.row_tiles));
  };
  // the last chunk this warp saw published (flags only go from 0 to 1 within a launch)
  int known_ready = -1;
  // whether a down piece's activations are staged (gate/up pieces need nothing)
  auto ready = [&](const DecodeSeg& sg) -> bool {
    if (sg.ph == 0) return true;
    const int ch = chunk_of(sg);
    if (ch == known_ready) return true;
    int v = 0;
    if (lane == 0) v = ld_acquire_gpu(a.chunk_ready + ch);
    v = __shfl_sync(0xFFFFFFFFu, v, 0);
    if (v) known_ready = ch;
    return v != 0;
  };
  auto wait_ready = [&](const DecodeSeg& sg) -> bool {
    if (chunk_of(sg) == known_ready) return true;
    int ok = 0;
    if (lane == 0) {
      const int32_t* flag = a.chunk_ready + chunk_of(sg);
      const uint64_t t0 = global_timer_ns();
      while (true) {
        if (ld_acquire_gpu(flag)) {
          ok = 1;
          break;
        }
        if (global_timer_ns() - t0 > kWaitLimitNs) {
          atomicOr(&g_device_error, kDecodeWaitError);
          break;
        }
        __nanosleep(128);
      }
    }
    ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
    if (ok) known_ready = chunk_of(sg);
    return ok != 0;
  };
  // a gate/up task is complete: count it; the chunk's last one stages and publishes the activations
  auto complete_up = [&](const DecodeSeg& sg) {
    const int ch = chunk_of(sg);
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = atomicAdd(a.chunk_up + ch, 1) == ph0.row_tiles - 1;
    if (!__shfl_sync(0xFFFFFFFFu, last, 0)) return;
    __threadfence();
    decode_stage_chunk(a, ch, lane);
    __threadfence();
    __syncwarp();
    if (lane == 0) st_release_gpu(a.chunk_ready + ch, 1);
  };
  auto finish = [&](const DecodeSeg& sg, const float (&acc)[2][4]) {
    if (sg.ph == 0) {
      decode_epilogue<0>(a, ph0, sg, lane, acc, true);
      complete_up(sg);
    } else {
      decode_epilogue<1>(a, ph1, sg, lane, acc, chunk_of(sg) == known_ready);
    }
  };

  DecodeSeg cur, nxt;
  bool have = next_seg(cur);
  UnitOperands cu, nu;
  bool cfix = false, nfix = false;
  if (have) operands(cur, cu, cfix);
  uint32_t step0 = 0;
  int primed = 0;
  while (have) {
    const bool have_n = next_seg(nxt);
    UnitOperands nx_issue;  // what may be prefetched of the next piece: nothing until its activations exist
    nx_issue.kb0 = nx_issue.kb1 = 0;
    nx_issue.rot = 0;
    if (have_n) {
      operands(nxt, nu, nfix);
      if (ready(nxt)) nx_issue = nu;
    }
    // a down piece waits for its chunk's activations (absent experts too: their zero rows need the
    // chunk's scale); after a timeout it is skipped and its rows come out zero (error recorded)
    bool run = cu.kb1 > cu.kb0;
    if (cur.ph == 1 && primed == 0 && !wait_ready(cur)) run = false;
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    int nx_primed = 0;
    if (run) {
      nx_primed = cfix ? async_accumulate<true, TILED>(acc, ring, cu, nx_issue, step0, primed, lane)
                       : async_accumulate<false, TILED>(acc, ring, cu, nx_issue, step0, primed, lane);
      step0 += cu.kb1 - cu.kb0;
    }
    primed = nx_primed;

    const DecodePhase P = cur.ph ? ph1 : ph0;
    if (cur.kb0 == 0 && cur.kb1 == P.nkb) {
      finish(cur, acc);
    } else {
      // a piece: park it in this warp's slot; the last arriving piece sums them in warp order
      const int64_t first_task = P.lo(wg) / P.nkb;
      float* slots = a.partial + static_cast<int64_t>(cur.ph) * 2 * a.partial_warps * (kWarp * 8);
      float4* mine = reinterpret_cast<float4*>(slots + (2 * wg + (cur.task == first_task ? 0 : 1)) * (kWarp * 8) +
                                               lane * 8);
      __stcg(mine, make_float4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]));
      __stcg(mine + 1, make_float4(acc[1][0], acc[1][1], acc[1][2], acc[1][3]));
      __threadfence();
      __syncwarp();
      const int64_t w_lo = P.warp_of(cur.task * P.nkb), w_hi = P.warp_of((cur.task + 1) * P.nkb - 1);
      int32_t* counter = (cur.ph ? a.cnt_down : a.cnt_up) + cur.task;
      int last = 0;
      if (lane == 0) last = atomicAdd(counter, 1) == static_cast<int>(w_hi - w_lo);
      if (__shfl_sync(0xFFFFFFFFu, last, 0)) {
        __threadfence();
        float sum[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        for (int64_t w = w_lo; w <= w_hi; ++w) {
          const int64_t wf = P.lo(w) / P.nkb;
          const float4* part = reinterpret_cast<const float4*>(
              slots + (2 * w + (cur.task == wf ? 0 : 1)) * (kWarp * 8) + lane * 8);
          const float4 v0 = __ldcg(part), v1 = __ldcg(part + 1);
          sum[0][0] += v0.x; sum[0][1] += v0.y; sum[0][2] += v0.z; sum[0][3] += v0.w;
          sum[1][0] += v1.x; sum[1][1] += v1.y; sum[1][2] += v1.z; sum[1][3] += v1.w;
        }
        finish(cur, sum);
      }
    }
    cur = nxt;
    cu = nu;
    cfix = nfix;
    have = have_n;
  }
  cp_async_wait<0>();  // no copy of this warp in flight when it exits
}

// flags[s] = 1 when expert s's three weight matrices hold no 0x7F / 0xFF byte.
__global__ void nan_free_kernel(const uint64_t* __restrict__ tables, int S, int64_t inter, int64_t hidden,
                                uint8_t* __restrict__ flags) {
  __shared__ int found;
  const int s = blockIdx.y;
  if (threadIdx.x == 0) found = 0;
  __syncthreads();
  const int64_t sizes[3] = {inter * hidden, inter * hidden, hidden * inter};
  const uint64_t ptrs[3] = {tables[s], tables[2 * S + s], tables[4 * S + s]};
  int hit = 0;
  for (int m = 0; m < 3 && !hit; ++m) {
    const uint8_t* w = reinterpret_cast<const uint8_t*>(ptrs[m]);
    if (!w) continue;
    const int64_t n = sizes[m];
    const bool vec = (reinterpret_cast<uintptr_t>(w) & 15u) == 0;
    const int64_t n16 = vec ? n / 16 : 0;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n16 && !hit;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const uint4 v = __ldcs(reinterpret_cast<const uint4*>(w) + i);
      const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) hit |= (((words[j] & 0x7F7F7F7Fu) + 0x01010101u) & 0x80808080u) != 0;
    }
    for (int64_t i = n16 * 16 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
      hit |= (w[i] & 0x7F) == 0x7F;
  }
  if (hit) found = 1;
  __syncthreads();
  // flags start at 1 (launcher); any CTA that saw a NaN code clears it
  if (threadIdx.x == 0 && found) flags[s] = 0;
}

// row-major e4m3 [rows, cols] -> fragment-native tiles (tiled_offset); rows
// past `rows` (up to a multiple of 128) are zero.  Thread q writes the q-th
// 16 bytes of the destination: (group, kb, sp, row tile j, piece rr, lane).
__global__ void fp8_tile_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t rows,
                                int64_t cols) {
  const int64_t nkb = cols / kBlock;
  const int64_t units = fp8_tiled_bytes_dev(rows, cols) / 16;
  for (int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; q < units;
       q += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int lane = static_cast<int>(q % kWarp);
    const int rr = static_cast<int>((q / kWarp) % 2);
    const int j = static_cast<int>((q / (2 * kWarp)) % 8);
    const int sp = static_cast<int>((q / (16 * kWarp)) % 2);
    const int64_t kb = (q / (32 * kWarp)) % nkb;
    const int64_t group = q / (32 * kWarp * nkb);
    const int g = lane / 4, c = lane % 4;
    const int64_t row = group * kTileGroupRows + j * 16 + g + 8 * rr;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < rows) v = *reinterpret_cast<const uint4*>(src + row * cols + kb * kBlock + sp * 64 + 16 * c);
    *reinterpret_cast<uint4*>(dst + q * 16) = v;
  }
}

// ---------------------------------------------------------------------------
// The same tasks fed by TMA: every warp owns a ring of kTmaStages shared-memory
// stages; lane l bulk-copies (cp.async.bulk) a 512-byte slice (4 k-blocks) of
// its row-stream l (stream l / 16, row l % 16 of the task) into slot l of a
// stage, completing on the stage's mbarrier.  Slots are 576 bytes apart (an
// odd multiple of 64) so that the eight lanes of each shared-memory phase
// (rows g, g+1, all four c) hit 32 distinct banks.  With three stages a warp
// keeps up to 32 KiB of weight reads in flight without holding them in
// registers, and each row is read in 512-byte runs.
// ---------------------------------------------------------------------------
constexpr int kTmaWarps = 4;
constexpr int kTmaStages = 3;
constexpr int kSliceBlocks = 4;                    // k-blocks per stage: 512 contiguous bytes per row
constexpr int kSliceBytes = kSliceBlocks * kBlock;
constexpr int kSlotBytes = kSliceBytes + 64;       // odd 64-byte offset keeps the fragment reads conflict-free
constexpr int kStageBytes = 32 * kSlotBytes;
constexpr size_t kTmaSmem = static_cast<size_t>(kTmaWarps) * kTmaStages * kStageBytes +
                            static_cast<size_t>(kTmaWarps) * kTmaStages * sizeof(uint64_t);

template <int NS, int EPI>
__global__ void __launch_bounds__(kTmaWarps * kWarp) tma_mma_gemv_kernel(MmaArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int g = lane / 4, c = lane % 4;
  const int K = a.K, N = a.N;
  unsigned char* ring = smem + static_cast<size_t>(warp) * kTmaStages * kStageBytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(kTmaWarps) * kTmaStages * kStageBytes) +
                  warp * kTmaStages;
  if (lane == 0) {
    for (int s = 0; s < kTmaStages; ++s) mbar_init(&bar[s], 1);
    fence_barrier_init();
  }
  __syncwarp();

  constexpr int kTaskRows = NS == 2 ? 16 : 32;
  const int row_tiles = static_cast<int>(ceil_div(N, kTaskRows));
  const int64_t tasks = static_cast<int64_t>(*a.n_chunks) * row_tiles;
  const int64_t warp_global = static_cast<int64_t>(blockIdx.x) * kTmaWarps + warp;
  const int64_t warp_count = static_cast<int64_t>(gridDim.x) * kTmaWarps;
  const int nkb = K / kBlock;
  uint32_t issued = 0, consumed = 0;

  for (int64_t task = warp_global; task < tasks; task += warp_count) {
    const int ch = static_cast<int>(task / row_tiles);
    const int r0 = static_cast<int>(task % row_tiles) * kTaskRows;
    const int seg = a.chunk_seg[ch], p0 = a.chunk_start[ch], len = a.chunk_len[ch];
    const uint8_t* w0 = reinterpret_cast<const uint8_t*>(a.w0[seg]);
    const float* s0 = reinterpret_cast<const float*>(a.s0[seg]);
    const uint8_t* w1 = NS == 2 ? reinterpret_cast<const uint8_t*>(a.w1[seg]) : w0;
    const float* s1 = NS == 2 ? reinterpret_cast<const float*>(a.s1[seg]) : s0;
    const bool present = w0 && s0 && w1 && s1 &&
                         ((reinterpret_cast<uintptr_t>(w0) | reinterpret_cast<uintptr_t>(w1)) & 15u) == 0;
    // row-stream of this lane's copies: stream lane / 16, row lane % 16 of that stream's 16-row tile
    const int my_st = lane / 16;
    const int my_row = min((NS == 2 ? r0 : r0 + 16 * my_st) + lane % 16, N - 1);
    const uint8_t* my_src = present ? (my_st == 0 ? w0 : w1) + static_cast<int64_t>(my_row) * K : nullptr;
    const float* srow[2];
#pragma unroll
    for (int st = 0; st < 2; ++st) {
      const int base = NS == 2 ? r0 : r0 + 16 * st;
      srow[st] = present ? (st == 0 ? s0 : s1) + static_cast<int64_t>(min(base, N - 1) / kBlock) * a.scale_cols
                         : nullptr;
    }
    const bool bvalid = g < len;
    const int64_t brow = bvalid ? (a.pair_row ? a.pair_row[p0 + g] : static_cast<int64_t>(p0 + g)) : 0;
    const __half* xb = a.x16 + brow * K + 16 * c;

    const int nslices = static_cast<int>(ceil_div(nkb, kSliceBlocks));
    auto issue = [&](int sl) {
      const uint32_t stage = issued % kTmaStages;
      const int blocks = min(kSliceBlocks, nkb - sl * kSliceBlocks);
      if (lane == 0) mbar_arrive_expect_tx(&bar[stage], 32u * blocks * kBlock);
      __syncwarp();
      bulk_copy_g2s(ring + stage * kStageBytes + lane * kSlotBytes,
                    my_src + static_cast<int64_t>(sl) * kSliceBytes, blocks * kBlock, &bar[stage]);
      ++issued;
    };
    auto load_b = [&](uint4 (&b)[2][2], int kbi) {
#pragma unroll
      for (int sp = 0; sp < 2; ++sp) {
        const int off = kbi * kBlock + sp * 64;
        if (bvalid) {
          b[sp][0] = __ldg(reinterpret_cast<const uint4*>(xb + off));
          b[sp][1] = __ldg(reinterpret_cast<const uint4*>(xb + off + 8));
        } else {
          b[sp][0] = make_uint4(0, 0, 0, 0);
          b[sp][1] = make_uint4(0, 0, 0, 0);
        }
      }
    };

    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    if (present) {
      for (int j = 0; j < min(kTmaStages, nslices); ++j) issue(j);
      uint4 bcur[2][2], bnxt[2][2];
      load_b(bcur, 0);
      for (int sl = 0; sl < nslices; ++sl) {
        const uint32_t stage = consumed % kTmaStages;
        if (!mbar_wait(&bar[stage], (consumed / kTmaStages) & 1u, 16)) {
          // error word set; let the copies still in flight land (bounded) before the CTA exits
          for (uint32_t q = consumed + 1; q < issued; ++q) mbar_wait(&bar[q % kTmaStages], (q / kTmaStages) & 1u, 16);
          return;
        }
        ++consumed;
        const unsigned char* st_base = ring + stage * kStageBytes;
        const int blocks = min(kSliceBlocks, nkb - sl * kSliceBlocks);
        for (int bi = 0; bi < blocks; ++bi) {
          const int kbi = sl * kSliceBlocks + bi;
          uint4 af[2][2][2];  // [span][stream][row g, row g + 8]
#pragma unroll
          for (int sp = 0; sp < 2; ++sp)
#pragma unroll
            for (int st = 0; st < 2; ++st)
#pragma unroll
              for (int rr = 0; rr < 2; ++rr)
                af[sp][st][rr] = *reinterpret_cast<const uint4*>(st_base + (st * 16 + g + 8 * rr) * kSlotBytes +
                                                                 bi * kBlock + sp * 64 + 16 * c);
          if (kbi + 1 < nkb) load_b(bnxt, kbi + 1);
          if (bi == blocks - 1) {
            // the whole slice is in registers now: hand the stage back to the async proxy
            fence_proxy_async_shared();
            __syncwarp();
            if (sl + kTmaStages < nslices) issue(sl + kTmaStages);
          }
          float t[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
          for (int sp = 0; sp < 2; ++sp) {
            const uint32_t bw[8] = {bcur[sp][0].x, bcur[sp][0].y, bcur[sp][0].z, bcur[sp][0].w,
                                    bcur[sp][1].x, bcur[sp][1].y, bcur[sp][1].z, bcur[sp][1].w};
#pragma unroll
            for (int s = 0; s < 4; ++s) {
#pragma unroll
              for (int st = 0; st < 2; ++st) {
                uint32_t wg = word_of(af[sp][st][0], s);
                uint32_t wh = word_of(af[sp][st][1], s);
                if (a.nanfix) {
                  wg = e4m3x4_nan_to_zero(wg);
                  wh = e4m3x4_nan_to_zero(wh);
                }
                uint32_t g0, g1, h0, h1;
                e4m3x4_to_f16x2x2(wg, g0, g1);
                e4m3x4_to_f16x2x2(wh, h0, h1);
                mma_16816(t[st], g0, h0, g1, h1, bw[2 * s], bw[2 * s + 1]);
              }
            }
          }
#pragma unroll
          for (int st = 0; st < 2; ++st) {
            const float sc = __ldg(srow[st] + kbi);
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[st][i] = fmaf(t[st][i], sc, acc[st][i]);
          }
          if (kbi + 1 < nkb) {
#pragma unroll
            for (int sp = 0; sp < 2; ++sp) {
              bcur[sp][0] = bnxt[sp][0];
              bcur[sp][1] = bnxt[sp][1];
            }
          }
        }
      }
    }

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
            const float gv = acc[0][i] * xs, uv = acc[1][i] * xs;
            const float silu = gv / (1.0f + expf(-gv));
            a.out0[p * N + row] = EPI == kEpiSwiglu ? silu * uv : gv;
          }
        } else {
#pragma unroll
          for (int st = 0; st < 2; ++st) {
            const int row = r0 + 16 * st + g + 8 * rr;
            if (row < N) a.out0[p * N + row] = acc[st][i] * xs;
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

bool mma_gemv_supported(int K, int N) { return K % kBlock == 0 && K > 0 && N > 0; }

// rows of at most 4 x 256 16-byte pieces go through the single-read kernel
template <typename T>
static void launch_rows_to_f16_t(const T* src, int rows, int K, const int32_t* n_rows_dev, __half* dst, float* scale,
                                 int32_t* zero, int64_t zero_n, unsigned grid, cudaStream_t stream) {
  const int pieces = static_cast<int>(ceil_div(static_cast<int64_t>(K) * sizeof(T), 16));
  if (pieces <= 256)
    rows_to_f16_regs_kernel<T, 1><<<grid, 256, 0, stream>>>(src, rows, K, n_rows_dev, dst, scale, zero, zero_n);
  else if (pieces <= 512)
    rows_to_f16_regs_kernel<T, 2><<<grid, 256, 0, stream>>>(src, rows, K, n_rows_dev, dst, scale, zero, zero_n);
  else if (pieces <= 1024)
    rows_to_f16_regs_kernel<T, 4><<<grid, 256, 0, stream>>>(src, rows, K, n_rows_dev, dst, scale, zero, zero_n);
  else if (pieces <= 2048)
    rows_to_f16_regs_kernel<T, 8><<<grid, 256, 0, stream>>>(src, rows, K, n_rows_dev, dst, scale, zero, zero_n);
  else if (pieces <= 4096)
    rows_to_f16_regs_kernel<T, 16><<<grid, 256, 0, stream>>>(src, rows, K, n_rows_dev, dst, scale, zero, zero_n);
  else
    rows_to_f16_kernel<T><<<grid, 256, 0, stream>>>(src, rows, K, n_rows_dev, dst, scale, zero, zero_n);
}

cudaError_t launch_f16_rows_to_f16(const void* src, int rows, int K, __half* dst, float* scale, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const unsigned grid = static_cast<unsigned>(std::min(rows, gemv_grid_ctas() * 8));
  launch_rows_to_f16_t(static_cast<const __half*>(src), rows, K, nullptr, dst, scale, nullptr, 0, grid, stream);
  return cudaGetLastError();
}

cudaError_t launch_rows_to_f16(const void* src, bool src_bf16, int rows, int K, const int32_t* n_rows_dev,
                               __half* dst, float* scale, int32_t* zero, int64_t zero_n, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  if (zero_n > 0 && !zero) return cudaErrorInvalidValue;
  const unsigned grid = static_cast<unsigned>(std::min(rows, gemv_grid_ctas() * 8));
  if (src_bf16)
    launch_rows_to_f16_t(static_cast<const __nv_bfloat16*>(src), rows, K, n_rows_dev, dst, scale, zero, zero_n, grid,
                         stream);
  else
    launch_rows_to_f16_t(static_cast<const float*>(src), rows, K, n_rows_dev, dst, scale, zero, zero_n, grid, stream);
  return cudaGetLastError();
}

cudaError_t launch_tma_mma_gemv(const MmaArgs& a, int ns, int epi, cudaStream_t stream) {
  const unsigned grid = static_cast<unsigned>(gemv_grid_ctas());  // one 4-warp CTA per SM (216 KiB of rings)
  auto k2 = tma_mma_gemv_kernel<2, kEpiSwiglu>;
  auto k1 = tma_mma_gemv_kernel<1, kEpiStore>;
  if (ns == 2 && epi == kEpiSwiglu) {
    cudaError_t err = cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kTmaSmem));
    if (err != cudaSuccess) return err;
    k2<<<grid, kTmaWarps * kWarp, kTmaSmem, stream>>>(a);
  } else if (ns == 1 && epi == kEpiStore) {
    cudaError_t err = cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kTmaSmem));
    if (err != cudaSuccess) return err;
    k1<<<grid, kTmaWarps * kWarp, kTmaSmem, stream>>>(a);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

int read_and_clear_mma_device_error(cudaStream_t stream) { return read_and_clear_local_error(stream); }

static int async_ctas_per_sm() {
  static int per_sm = 0;
  if (per_sm == 0) {
    int a = 0, b = 0;
    cudaFuncSetAttribute(mma_gemv_async_kernel<2, kEpiSwiglu, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kAsyncSmem);
    cudaFuncSetAttribute(mma_gemv_async_kernel<1, kEpiStore, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kAsyncSmem);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&a, mma_gemv_async_kernel<2, kEpiSwiglu, false>,
                                                  kAsyncWarps * kWarp, kAsyncSmem);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, mma_gemv_async_kernel<1, kEpiStore, false>,
                                                  kAsyncWarps * kWarp, kAsyncSmem);
    per_sm = std::max(1, std::min(a, b));
  }
  return per_sm;
}

// K-split of the warp tasks when there are fewer tasks than resident warps:
// enough k-ranges to cover the warps (at least four k-blocks each), then one
// more if that packs the round-robin (task, k-range) units into fewer
// rounds per task (1152 tasks on 1776 warps: 2 -> 2 rounds of half a task,
// 3 -> 2 rounds of a third).  Each k-range costs a partial write and a
// reduction, so batches with a task per warp or more are not split.
static int balanced_ksplit(int64_t tasks, int64_t warps, int K) {
  if (tasks <= 0 || tasks >= warps) return 1;
  const int nkb = K / kBlock;
  const int cap = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(nkb / 4, kMaxMmaKSplit)));
  const int want = static_cast<int>(std::min<int64_t>(ceil_div(warps, tasks), cap));
  auto per_task = [&](int ks) { return static_cast<double>(ceil_div(tasks * ks, warps)) / ks; };
  return (want + 1 <= cap && per_task(want + 1) < per_task(want)) ? want + 1 : std::max(1, want);
}

int async_gemv_ksplit(int64_t tasks_bound, int K) {
  const int64_t warps = static_cast<int64_t>(gemv_grid_ctas()) * async_ctas_per_sm() * kAsyncWarps;
  return balanced_ksplit(tasks_bound, warps, K);
}

int async_gemv_ctas_per_sm() { return async_ctas_per_sm(); }

int async_gemv_ksplit_for(int64_t tasks_bound, int K, int64_t ctas) {
  return balanced_ksplit(tasks_bound, std::max<int64_t>(1, ctas) * kAsyncWarps, K);
}

cudaError_t launch_async_mma_gemv(const MmaArgs& a, int ns, int epi, int64_t tasks_bound, cudaStream_t stream,
                                  int64_t max_ctas) {
  if (a.ksplit < 1 || a.ksplit > kMaxMmaKSplit || (a.ksplit > 1 && (!a.partial || !a.counters)))
    return cudaErrorInvalidValue;
  int64_t full = static_cast<int64_t>(gemv_grid_ctas()) * async_ctas_per_sm();
  if (max_ctas > 0) full = std::min(full, max_ctas);
  const int64_t need = ceil_div(std::max<int64_t>(1, tasks_bound) * a.ksplit, kAsyncWarps);
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min(full, need)));
  auto kernel = ns == 2 ? (a.tiled ? mma_gemv_async_kernel<2, kEpiSwiglu, true> : mma_gemv_async_kernel<2, kEpiSwiglu, false>)
                        : (a.tiled ? mma_gemv_async_kernel<1, kEpiStore, true> : mma_gemv_async_kernel<1, kEpiStore, false>);
  if (!((ns == 2 && epi == kEpiSwiglu) || (ns == 1 && epi == kEpiStore))) return cudaErrorInvalidValue;
  // per device context, so set on every launch (a host-side call; graphs do not record it)
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAsyncSmem);
  if (err != cudaSuccess) return err;
  kernel<<<grid, kAsyncWarps * kWarp, kAsyncSmem, stream>>>(a);
  return cudaGetLastError();
}

static int decode_fused_ctas_per_sm() {
  static int per_sm = 0;
  if (per_sm == 0) {
    int a = 0, b = 0;
    cudaFuncSetAttribute(decode_fused_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kAsyncSmem);
    cudaFuncSetAttribute(decode_fused_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kAsyncSmem);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&a, decode_fused_kernel<true>, kAsyncWarps * kWarp, kAsyncSmem);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, decode_fused_kernel<false>, kAsyncWarps * kWarp, kAsyncSmem);
    per_sm = std::max(1, std::min(a, b));
  }
  return per_sm;
}

int decode_fused_warps() { return gemv_grid_ctas() * decode_fused_ctas_per_sm() * kAsyncWarps; }

cudaError_t launch_decode_fused(const DecodeFusedArgs& a, cudaStream_t stream) {
  if (!a.partial || a.partial_warps <= 0 || !a.cnt_up || !a.cnt_down || !a.chunk_up || !a.chunk_ready ||
      a.up.tiled != a.down.tiled || a.up.K % kBlock != 0 || a.down.K % kBlock != 0)
    return cudaErrorInvalidValue;
  // every CTA resident at once: the down pieces wait for gate/up pieces of other CTAs
  const int ctas = std::min(gemv_grid_ctas() * decode_fused_ctas_per_sm(),
                            static_cast<int>(ceil_div(a.partial_warps, kAsyncWarps)));
  auto kernel = a.up.tiled ? decode_fused_kernel<true> : decode_fused_kernel<false>;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAsyncSmem);
  if (err != cudaSuccess) return err;
  kernel<<<static_cast<unsigned>(std::max(1, ctas)), kAsyncWarps * kWarp, kAsyncSmem, stream>>>(a);
  return cudaGetLastError();
}

int64_t fp8_tiled_bytes(int64_t rows, int64_t cols) { return fp8_tiled_bytes_dev(rows, cols); }

cudaError_t launch_fp8_tile(const uint8_t* src, uint8_t* dst, int64_t rows, int64_t cols, cudaStream_t stream) {
  if (rows <= 0 || cols <= 0) return cudaSuccess;
  if (cols % kBlock != 0 || (reinterpret_cast<uintptr_t>(src) & 15u) || (reinterpret_cast<uintptr_t>(dst) & 15u))
    return cudaErrorInvalidValue;
  const int64_t pieces = fp8_tiled_bytes(rows, cols) / 16;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(ceil_div(pieces, 256), gemv_grid_ctas() * 16));
  fp8_tile_kernel<<<grid, 256, 0, stream>>>(src, dst, rows, cols);
  return cudaGetLastError();
}

cudaError_t launch_nan_free_flags(const uint64_t* tables, int S, int64_t inter, int64_t hidden, uint8_t* flags,
                                  cudaStream_t stream) {
  if (S <= 0) return cudaSuccess;
  cudaError_t err = cudaMemsetAsync(flags, 1, static_cast<size_t>(S), stream);
  if (err != cudaSuccess) return err;
  dim3 grid(64, static_cast<unsigned>(S));
  nan_free_kernel<<<grid, 256, 0, stream>>>(tables, S, inter, hidden, flags);
  return cudaGetLastError();
}

// Resident 4-warp CTAs per SM of the register-fed kernel (register-limited).
static int mma_ctas_per_sm() {
  static int per_sm = 0;
  if (per_sm == 0) {
    int a = 0, b = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&a, mma_gemv_kernel<2, kEpiSwiglu>, kMmaCtaWarps * kWarp, 0);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, mma_gemv_kernel<1, kEpiStore>, kMmaCtaWarps * kWarp, 0);
    per_sm = std::max(1, std::min(a, b));
  }
  return per_sm;
}

int mma_gemv_ksplit(int64_t tasks_bound, int K) {
  const int64_t warps = static_cast<int64_t>(gemv_grid_ctas()) * mma_ctas_per_sm() * kMmaCtaWarps;
  return balanced_ksplit(tasks_bound, warps, K);
}

cudaError_t launch_mma_gemv(const MmaArgs& a, int ns, int epi, int64_t tasks_bound, cudaStream_t stream) {
  if (a.ksplit < 1 || a.ksplit > kMaxMmaKSplit || (a.ksplit > 1 && (!a.partial || !a.counters)))
    return cudaErrorInvalidValue;
  const int64_t full = static_cast<int64_t>(gemv_grid_ctas()) * mma_ctas_per_sm();
  const int64_t need = ceil_div(std::max<int64_t>(1, tasks_bound) * a.ksplit, kMmaCtaWarps);
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min(full, need)));
  if (ns == 2 && epi == kEpiSwiglu) mma_gemv_kernel<2, kEpiSwiglu><<<grid, kMmaCtaWarps * kWarp, 0, stream>>>(a);
  else if (ns == 1 && epi == kEpiStore) mma_gemv_kernel<1, kEpiStore><<<grid, kMmaCtaWarps * kWarp, 0, stream>>>(a);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace moe
