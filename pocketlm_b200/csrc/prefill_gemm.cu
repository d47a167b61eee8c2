// Grouped FP8-weight GEMM for prefill batches on the 5th-generation tensor
// cores (tcgen05 + TMEM + TMA), sm_100a.
//
// The per-expert products of run_fp8_moe (fp8_source.py:1569-1884) for large
// token counts: for every expert e with M_e (token, expert) pairs,
//   gate/up:  act[p, n] = silu(x_p . gate_e[n]) * (x_p . up_e[n])
//   down:     y[p, h]   = act_p . down_e[h]
// with 128 x 128 fp32 block scales on the e4m3 weights (fp8_linear.cpp:103-112).
//
// Operands.  A is the pairs' activation rows in fp16, each row divided by a
// power of two (exact; undone in the epilogue), expert-contiguous [P, K] and
// loaded by TMA (128B swizzle, 128 rows x 64 columns per box, two boxes per
// 256-pair tile).  B is the
// expert's weights in the fragment-native tiled layout (fp8_mma.cu), brought
// in by 1-D bulk copies of 8 KiB runs and converted by eight converter warps
// to fp16 with the k-block's scale folded in -- the exact e4m3 value times
// the scale rounded to fp16, product rounded to fp16: a relative error of
// at most about 2^-10 per weight -- written in the same 128B-swizzled
// K-major layout.  A tile is 256 pairs x 256 weight rows (128 gate + 128 up
// rows for the fused gate/up GEMM): two M = 128 MMAs per K = 16 step share
// the converted weights, so each converted byte feeds twice the tensor work
// of a 128-pair tile.  D accumulates in fp32 in tensor memory (2 x 256
// columns).  K = 64 per pipeline stage; three load stages (two A sub-tiles +
// raw weights, 48 KiB) feed two converted-weight buffers (32 KiB).  A tile of
// at most 128 pairs loads and multiplies one sub-tile.
//
// Warp roles (608 threads): warps 0-7 epilogue (warp w: TMEM lanes
// 32 (w % 4) .. + 31 of sub-tile w / 4), warps 8-15 converter, warp 16 TMA
// producer, warp 17 MMA issuer, warp 18 TMEM allocator.  A persistent CTA
// walks tiles (expert m-tile, n-tile) in order; the epilogue drains a tile's
// accumulators before the next tile's first MMA.  Every wait is bounded (2 s of %globaltimer): on
// expiry the CTA records an error code, every role leaves its loop, the
// producer waits (bounded) for the copies it issued, and TMEM is freed.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "async_copy.cuh"
#include "common.cuh"
#include "fp8_gemv.cuh"
#include "prefill_gemm.cuh"
#include "router.cuh"

namespace moe {
namespace {

constexpr int kBM = 256;              // pairs per tile: two 128-row MMA sub-tiles sharing B
constexpr int kSubM = 128;            // pairs per MMA (M of tcgen05.mma, cta_group::1)
constexpr int kBN = 256;              // weight rows per tile (128 gate + 128 up for the gate/up GEMM)
constexpr int kBK = 64;               // k per stage (half a scale block)
constexpr int kStages = 3;            // load stages: two A sub-tiles + raw e4m3 weights
constexpr int kConvBufs = 2;          // converted fp16 weight buffers
constexpr int kATileBytes = kSubM * kBK * 2;     // 16 KiB per sub-tile, fp16, 128B-swizzled (TMA)
constexpr int kRawBytes = kBN * kBK;             // 16 KiB e4m3: two 8 KiB runs of 8 row tiles
constexpr int kLoadBytes = 2 * kATileBytes + kRawBytes;  // 48 KiB per stage
constexpr int kBTileBytes = kBN * kBK * 2;       // 32 KiB, fp16, 128B-swizzled (converter)
constexpr int kTmemCols = 2 * kBN;               // the two sub-tiles' accumulators (512 columns)
constexpr int kEpiWarps = 8, kConvWarps = 8;
constexpr int kConvThreads = kConvWarps * kWarp;
constexpr int kProducerWarp = kEpiWarps + kConvWarps, kMmaWarp = kProducerWarp + 1, kAllocWarp = kProducerWarp + 2;
constexpr int kThreads = (kAllocWarp + 1) * kWarp;
constexpr int kCodeWait = 32;
constexpr int kPrefetchStages = 4;  // weight runs requested into L2 this many stages ahead
constexpr int kScaleRegs = 4;  // converter scale cache: registers per lane and half

struct Barriers {
  uint64_t full[kStages];      // producer -> converter, MMA: A + raw weights landed (tx bytes)
  uint64_t empty[kStages];     // MMA -> producer: the stage's MMAs completed (tcgen05.commit)
  uint64_t cfull[kConvBufs];   // converter -> MMA: fp16 weights written (4 arrivals)
  uint64_t cempty[kConvBufs];  // MMA -> converter: buffer consumed (tcgen05.commit)
  uint64_t tfull;              // MMA -> epilogue: tile accumulators complete
  uint64_t tempty;             // epilogue -> MMA: accumulators drained (one arrival per epilogue warp)
  uint64_t drain;              // MMA issuer's last commit: all of its MMAs complete
  uint32_t tmem_base;
  int abort;
};
constexpr int kStageBytes = kWarp * 16 * 4;  // epilogue staging per warp: 32 rows x 16 fp32
constexpr size_t kSmemBytes = 1024 /* alignment slack */ + static_cast<size_t>(kStages) * kLoadBytes +
                              static_cast<size_t>(kConvBufs) * kBTileBytes +
                              static_cast<size_t>(kEpiWarps) * kStageBytes + sizeof(Barriers);
static_assert(kSmemBytes <= 232448, "shared memory per block");

// ---------------------------------------------------------------- PTX

MOE_D void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)), "r"(ncols)
               : "memory");
}
MOE_D void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
MOE_D void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
MOE_D void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MOE_D void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

MOE_D void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
MOE_D void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
// 16 columns of this warp's 32 TMEM lanes; the registers are valid after tmem_ld_wait().
MOE_D void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// explicit shared-space accesses (the aligned smem base is a generic pointer)
MOE_D uint4 ld_shared_v4(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(smem_addr(p)));
  return v;
}
MOE_D void st_shared_v4(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(smem_addr(p)), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
// warm L2 with a weight run a few stages ahead of its bulk copy (no shared memory held)
MOE_D void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
MOE_D void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
MOE_D void tma_load_2d(void* dst, const CUtensorMap* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// K-major, 128B-swizzled operand tile: rows of 128 bytes, 8-row atoms 1024 B apart.
MOE_D uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(16 >> 4) << 16;    // leading byte offset (unused with 128B swizzle)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;  // stride byte offset: next 8-row atom
  d |= static_cast<uint64_t>(1) << 46;          // descriptor version for tcgen05
  d |= static_cast<uint64_t>(2) << 61;          // 128B swizzle
  return d;
}
// kind::f16 instruction descriptor: fp32 D, fp16 A and B, both K-major.
constexpr uint32_t kIdesc = (1u << 4) | (static_cast<uint32_t>(kBN >> 3) << 17) | (static_cast<uint32_t>(kSubM >> 4) << 24);

// Bounded wait that also gives up when another role aborted.  Between checks
// the thread sleeps in try_wait (woken when the phase completes), so waiting
// roles take no issue slots from the converter warps.
constexpr uint32_t kSuspendHintNs = 20000;
MOE_D bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (!mbar_try_wait_sleep(bar, parity, kSuspendHintNs)) {
    if (*abort) return false;
    if (global_timer_ns() - start > kWaitLimitNs) {
      atomicOr(&g_device_error, kCodeWait);
      *abort = 1;
      return false;
    }
  }
  return true;
}

// ------------------------------------------------------------ tile map
// tile t -> (segment, first pair, pairs in the segment from there, n-tile)
struct TileRef {
  int seg, row0, rows, nt;
};
MOE_D TileRef tile_at(int64_t t, const int32_t* mprefix, const int32_t* seg_offset, int n_segments, int n_tiles) {
  const int m = static_cast<int>(t / n_tiles);
  TileRef r;
  r.nt = static_cast<int>(t % n_tiles);
  int lo = 0, hi = n_segments;  // largest s with mprefix[s] <= m
  while (hi - lo > 1) {
    const int mid = (lo + hi) / 2;
    if (mprefix[mid] <= m) lo = mid;
    else hi = mid;
  }
  r.seg = lo;
  r.row0 = seg_offset[lo] + (m - mprefix[lo]) * kBM;
  r.rows = min(kBM, seg_offset[lo + 1] - r.row0);
  return r;
}

// mprefix[s] = m-tiles of segments before s; mprefix[n_segments] = all of them.
__global__ void prefill_tiles_kernel(const int32_t* seg_offset, int n_segments, int32_t* mprefix) {
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  int acc = 0;
  for (int s = 0; s < n_segments; ++s) {
    mprefix[s] = acc;
    const int rows = seg_offset[s + 1] - seg_offset[s];
    acc += (rows + kBM - 1) / kBM;
  }
  mprefix[n_segments] = acc;
}

// A rows of the gate/up GEMM: xa[p] = x16[pair_row[p]], ascale[p] = xscale[pair_row[p]].
__global__ void gather_rows_kernel(const __half* x16, const float* xscale, const int32_t* pair_row, int64_t P,
                                   int64_t K, __half* xa, float* ascale) {
  const int lane = threadIdx.x % kWarp;
  for (int64_t p = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / kWarp; p < P;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x / kWarp) {
    const int64_t r = pair_row[p];
    const uint4* src = reinterpret_cast<const uint4*>(x16 + r * K);
    uint4* dst = reinterpret_cast<uint4*>(xa + p * K);
    for (int64_t i = lane; i < K / 8; i += kWarp) dst[i] = __ldg(src + i);
    if (lane == 0) ascale[p] = xscale[r];
  }
}

// Row-major packed int4 [rows, K / 2] -> the Q4 tiled layout; thread q writes
// the q-th 16 bytes of the destination (run, row, half of its 32 bytes).
__global__ void q4_tile_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t rows, int64_t K) {
  const int64_t nkblk = K / 64, row_bytes = K / 2;
  const int64_t units = (rows + 127) / 128 * nkblk * 256;
  for (int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; q < units;
       q += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t run = q / 256;
    const int w = static_cast<int>(q % 256);
    const int64_t group = run / nkblk, kblk = run % nkblk;
    const int64_t row = group * 128 + w / 2;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < rows) v = *reinterpret_cast<const uint4*>(src + row * row_bytes + kblk * 32 + (w % 2) * 16);
    *reinterpret_cast<uint4*>(dst + q * 16) = v;
  }
}

// 16 bytes of activations -> floats
template <typename T>
MOE_D void piece_to_float(const uint4& v, float* out);
template <>
MOE_D void piece_to_float<float>(const uint4& v, float* out) {
  out[0] = __uint_as_float(v.x); out[1] = __uint_as_float(v.y);
  out[2] = __uint_as_float(v.z); out[3] = __uint_as_float(v.w);
}
template <>
MOE_D void piece_to_float<__nv_bfloat16>(const uint4& v, float* out) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = __uint_as_float(w[i] << 16);
    out[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
template <>
MOE_D void piece_to_float<__half>(const uint4& v, float* out) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}

// The pairs' A rows straight from the tokens: token t's row (read once, kept
// in registers) -> fp16 / power-of-two scale (the rows_to_f16 staging:
// 2^(floor(log2 amax) - 13), 1 for an all-zero row), written to the row of
// each of its pairs: entry_pair[t * k + j] (>= 0), then, with a shared
// expert, pair *tail_first + t.  One CTA per token; a token with no pair is
// not read.
template <typename T, int P>
__global__ void __launch_bounds__(256) scatter_rows_kernel(const T* __restrict__ x, int T_, int K,
                                                           const int32_t* __restrict__ entry_pair, int k,
                                                           const int32_t* __restrict__ tail_first,
                                                           __half* __restrict__ a16, float* __restrict__ ascale) {
  constexpr int V = 16 / sizeof(T);
  __shared__ float red[8];
  const int n16 = K / V;
  for (int t = blockIdx.x; t < T_; t += gridDim.x) {
    bool any = tail_first != nullptr;  // the same for every thread of the CTA
    for (int j = 0; j < k; ++j) any |= entry_pair[static_cast<int64_t>(t) * k + j] >= 0;
    if (!any) continue;
    const uint4* s = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t) * K);
    uint4 v[P];
    float amax = 0.0f;
#pragma unroll
    for (int q = 0; q < P; ++q) {
      const int i = threadIdx.x + q * 256;
      v[q] = i < n16 ? __ldg(s + i) : make_uint4(0, 0, 0, 0);
      float f[V];
      piece_to_float<T>(v[q], f);
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
    // fp16 pieces: V values each (8 halves = 16 bytes, or 4 halves = 8 bytes for fp32 input)
    uint4 h16[P];
#pragma unroll
    for (int q = 0; q < P; ++q) {
      float f[V];
      piece_to_float<T>(v[q], f);
      __align__(16) __half h[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) h[j] = __float2half_rn(j < V ? f[j] * inv : 0.0f);
      h16[q] = *reinterpret_cast<const uint4*>(h);
    }
    const int n_out = k + (tail_first ? 1 : 0);
    for (int j = 0; j < n_out; ++j) {
      const int p = j < k ? entry_pair[static_cast<int64_t>(t) * k + j] : *tail_first + t;
      if (p < 0) continue;
      __half* d = a16 + static_cast<int64_t>(p) * K;
#pragma unroll
      for (int q = 0; q < P; ++q) {
        const int i = threadIdx.x + q * 256;
        if (i >= n16) continue;
        if (V == 8) *reinterpret_cast<uint4*>(d + i * V) = h16[q];
        else *reinterpret_cast<uint2*>(d + i * V) = make_uint2(h16[q].x, h16[q].y);
      }
      if (threadIdx.x == 0) ascale[p] = sc;
    }
    __syncthreads();
  }
}

// --------------------------------------------------------------- kernel
template <bool GATEUP, int WF>
__global__ void __launch_bounds__(kThreads, 1) prefill_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                                                    const __grid_constant__ CUtensorMap tmap_a64,
                                                                    const __grid_constant__ CUtensorMap tmap_a32,
                                                                    PrefillArgs a) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto a_tile = [&](int s, int h) { return smem + s * kLoadBytes + h * kATileBytes; };
  auto raw_tile = [&](int s) { return smem + s * kLoadBytes + 2 * kATileBytes; };
  auto b_tile = [&](int b) { return smem + kStages * kLoadBytes + b * kBTileBytes; };
  unsigned char* stage_buf = smem + kStages * kLoadBytes + kConvBufs * kBTileBytes;  // epilogue staging
  Barriers* bars = reinterpret_cast<Barriers*>(stage_buf + kEpiWarps * kStageBytes);
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  volatile int* abort = &bars->abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < kConvBufs; ++b) {
      mbar_init(&bars->cfull[b], kConvWarps);
      mbar_init(&bars->cempty[b], 1);
    }
    mbar_init(&bars->tfull, 1);
    mbar_init(&bars->tempty, kEpiWarps);
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == kAllocWarp) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  const int K = a.K, N = a.N;
  const int n_tiles = GATEUP ? N / (kBN / 2) : N / kBN;
  const int64_t tiles = static_cast<int64_t>(a.mprefix[a.n_segments]) * n_tiles;
  const int nkh = K / kBK;  // pipeline stages per tile
  const int nkb = K / 128;  // k-blocks (scale columns, tiled-layout blocks)
  constexpr uint32_t kRunBytes = WF == kPrefillQ4Row ? 4096 : kTileRunBytes;  // per matrix half and stage
  // an expert without (16-byte aligned) weights and scales is skipped by every
  // role alike; the epilogue writes its pairs' rows as zeros
  auto present = [&](int seg) {
    const uint64_t w0 = a.w0[seg], w1 = GATEUP ? a.w1[seg] : w0;
    return w0 && w1 && a.s0[seg] && (!GATEUP || a.s1[seg]) && ((w0 | w1) & 15u) == 0;
  };

  if (warp == kProducerWarp) {
    if (lane == 0) {
      uint32_t it = 0;
      for (int64_t t = blockIdx.x; t < tiles && !*abort; t += gridDim.x) {
        const TileRef tr = tile_at(t, a.mprefix, a.seg_offset, a.n_segments, n_tiles);
        if (!present(tr.seg)) continue;
        // two 128-row groups (8 row tiles each, one 8 KiB run per k-step):
        // gate/up = group nt of each matrix, down = groups 2 nt, 2 nt + 1
        const uint8_t* w0 = reinterpret_cast<const uint8_t*>(a.w0[tr.seg]);
        const uint8_t* wbase[2] = {w0, GATEUP ? reinterpret_cast<const uint8_t*>(a.w1[tr.seg]) : w0};
        const int64_t tile0[2] = {GATEUP ? tr.nt * 8 : tr.nt * 16, GATEUP ? tr.nt * 8 : tr.nt * 16 + 8};
        // the stage's run of matrix half h: 8 KiB of e4m3 (k-block kq / 2, half kq % 2)
        // or 4 KiB of int4 codes (64-code k-block kq)
        auto run_at = [&](int h, int kq) {
          return WF == kPrefillQ4Row ? wbase[h] + q4_tiled_offset(tile0[h] / 8, kq, nkh)
                                     : wbase[h] + tiled_offset(tile0[h], kq / 2, kq % 2, nkb);
        };
        auto prefetch = [&](int kq) {
#pragma unroll
          for (int h = 0; h < 2; ++h) bulk_prefetch_l2(run_at(h, kq), kRunBytes);
        };
        for (int kq = 0; kq < kPrefetchStages && kq < nkh; ++kq) prefetch(kq);
        for (int kh = 0; kh < nkh && !*abort; ++kh, ++it) {
          const int s = it % kStages;
          if (kh + kPrefetchStages < nkh) prefetch(kh + kPrefetchStages);
          if (it >= kStages && !wait_or_abort(&bars->empty[s], ((it / kStages) - 1) & 1, abort)) break;
          // the second sub-tile only when the tile has more than 128 pairs
          const bool two = tr.rows > kSubM;
          // a sub-tile of <= 32 / 64 pairs loads that many rows (the rest of the
          // 128-row tile keeps stale data; its results are never stored)
          const int rows0 = min(tr.rows, kSubM), rows1 = tr.rows - kSubM;
          auto a_box = [&](int rows) { return rows <= 32 ? &tmap_a32 : rows <= 64 ? &tmap_a64 : &tmap_a; };
          auto a_bytes = [&](int rows) { return rows <= 32 ? kATileBytes / 4 : rows <= 64 ? kATileBytes / 2 : kATileBytes; };
          mbar_arrive_expect_tx(&bars->full[s], a_bytes(rows0) + (two ? a_bytes(rows1) : 0) + 2 * kRunBytes);
          tma_load_2d(a_tile(s, 0), a_box(rows0), kh * kBK, tr.row0, &bars->full[s]);
          if (two) tma_load_2d(a_tile(s, 1), a_box(rows1), kh * kBK, tr.row0 + kSubM, &bars->full[s]);
#pragma unroll
          for (int h = 0; h < 2; ++h) bulk_copy_g2s(raw_tile(s) + h * kRunBytes, run_at(h, kh), kRunBytes, &bars->full[s]);
        }
      }
      // every copy issued lands before the CTA may exit
      for (uint32_t j = it > kStages ? it - kStages : 0; j < it; ++j)
        mbar_wait(&bars->full[j % kStages], (j / kStages) & 1, kCodeWait);
    }
  } else if (WF == kPrefillQ4Row && warp >= kEpiWarps && warp < kEpiWarps + kConvWarps) {
    // converter, int4 codes: thread ct owns tile row n = ct (run n / 128, row
    // n % 128 of it): its 32 bytes hold k 0..63 of the stage, converted
    // exactly to fp16 integers -8..7 (the row scale is applied in the
    // epilogue) and written as one 128-byte swizzled row
    const int n = threadIdx.x - kEpiWarps * kWarp;  // 0 .. 255
    const __half2 mul = __halves2half2(__float2half(1.0f), __float2half(0.0625f));
    const __half2 add = __halves2half2(__float2half(-1032.0f), __float2half(-72.0f));
    uint32_t it = 0;
    for (int64_t t = blockIdx.x; t < tiles && !*abort; t += gridDim.x) {
      const TileRef tr = tile_at(t, a.mprefix, a.seg_offset, a.n_segments, n_tiles);
      if (!present(tr.seg)) continue;
      bool ok = true;
      for (int kh = 0; kh < nkh; ++kh, ++it) {
        const int s = it % kStages, b = it % kConvBufs;
        if (!wait_or_abort(&bars->full[s], (it / kStages) & 1, abort) ||
            (it >= kConvBufs && !wait_or_abort(&bars->cempty[b], ((it / kConvBufs) - 1) & 1, abort))) {
          ok = false;
          break;
        }
        const unsigned char* src = raw_tile(s) + (n / 128) * kRunBytes + (n % 128) * 32;
        unsigned char* bt = b_tile(b);
        const uint4 lo = ld_shared_v4(src), hi = ld_shared_v4(src + 16);
        const uint32_t words[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          // word c = codes k 8c .. 8c + 7, two per byte (even k low): byte j -> (k 8c+2j, 8c+2j+1)
          uint32_t h[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t v;
            asm("prmt.b32 %0, %1, 0, %2;" : "=r"(v) : "r"(words[c]), "r"(0x4040 + 0x0101 * j));
            // halves 1024 + (lo ^ 8) and 1024 + 16 (hi ^ 8), then x (1, 1/16) - (1032, 72): the signed codes
            v = (v & 0x00F0000Fu) ^ 0x64806408u;
            const __half2 r = __hfma2(*reinterpret_cast<const __half2*>(&v), mul, add);
            h[j] = *reinterpret_cast<const uint32_t*>(&r);
          }
          st_shared_v4(bt + (n / 8) * 1024 + (n % 8) * 128 + ((c ^ (n % 8)) * 16), h[0], h[1], h[2], h[3]);
        }
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->cfull[b]);
      }
      if (!ok) break;
    }
  } else if (WF == kPrefillFp8Block && warp >= kEpiWarps && warp < kEpiWarps + kConvWarps) {
    // converter: e4m3 runs x block scale -> fp16, 128B-swizzled K-major
    const int ct = threadIdx.x - kEpiWarps * kWarp;  // 0 .. kConvThreads - 1
    uint32_t it = 0;
    for (int64_t t = blockIdx.x; t < tiles && !*abort; t += gridDim.x) {
      const TileRef tr = tile_at(t, a.mprefix, a.seg_offset, a.n_segments, n_tiles);
      if (!present(tr.seg)) continue;
      const bool fix = a.nanfix && !(a.nan_free && a.nan_free[tr.seg]);
      // scale rows of the two 128-row halves of the tile
      const float* sb0 = reinterpret_cast<const float*>(a.s0[tr.seg]);
      const float* sb1 = GATEUP ? reinterpret_cast<const float*>(a.s1[tr.seg]) : sb0;
      sb0 += static_cast<int64_t>(GATEUP ? tr.nt : 2 * tr.nt) * a.scale_cols;
      sb1 += static_cast<int64_t>(GATEUP ? tr.nt : 2 * tr.nt + 1) * a.scale_cols;
      // the tile's block scales, k-block kb in lane kb % 32 of register kb / 32
      // (read once per tile; K up to kScaleRegs * 32 * 128, else per stage)
      const bool cached = nkb <= kScaleRegs * kWarp;
      auto scale_at = [&](const float* sb, int i) {
        const int kbi = lane + i * kWarp;
        return (cached && kbi < nkb) ? __ldg(sb + kbi) : 0.0f;
      };
      // four named registers per half (an indexed array would live in local memory)
      const float g0 = scale_at(sb0, 0), g1 = scale_at(sb0, 1), g2 = scale_at(sb0, 2), g3 = scale_at(sb0, 3);
      const float u0 = scale_at(sb1, 0), u1 = scale_at(sb1, 1), u2 = scale_at(sb1, 2), u3 = scale_at(sb1, 3);
      bool ok = true;
      for (int kh = 0; kh < nkh; ++kh, ++it) {
        const int s = it % kStages, b = it % kConvBufs;
        const int kb = kh / 2;
        // the block scales as fp16 pairs: w * s is rounded once more, to fp16
        float sf0, sf1;
        if (cached) {
          const int r = kb / kWarp;
          const float v0 = r == 0 ? g0 : r == 1 ? g1 : r == 2 ? g2 : g3;
          const float v1 = r == 0 ? u0 : r == 1 ? u1 : r == 2 ? u2 : u3;
          sf0 = __shfl_sync(0xffffffffu, v0, kb % kWarp);
          sf1 = __shfl_sync(0xffffffffu, v1, kb % kWarp);
        } else {
          sf0 = __ldg(sb0 + kb);
          sf1 = __ldg(sb1 + kb);
        }
        const __half2 sc_lo = __float2half2_rn(sf0), sc_hi = __float2half2_rn(sf1);
        if (!wait_or_abort(&bars->full[s], (it / kStages) & 1, abort) ||
            (it >= kConvBufs && !wait_or_abort(&bars->cempty[b], ((it / kConvBufs) - 1) & 1, abort))) {
          ok = false;
          break;
        }
        const unsigned char* raw = raw_tile(s);
        unsigned char* bt = b_tile(b);
#pragma unroll
        for (int q = 0; q < kRawBytes / 16 / kConvThreads; ++q) {
          const int u = ct + q * kConvThreads;  // 16-byte unit: run u / 64, row half, lane
          const int run = u / 64, rr = (u / kWarp) % 2, ul = u % kWarp;
          const int g = ul / 4, c = ul % 4;
          const int n = 16 * run + g + 8 * rr;  // tile row 0..255
          uint4 v = ld_shared_v4(raw + u * 16);
          if (fix) {
            v.x = e4m3x4_nan_to_zero(v.x);
            v.y = e4m3x4_nan_to_zero(v.y);
            v.z = e4m3x4_nan_to_zero(v.z);
            v.w = e4m3x4_nan_to_zero(v.w);
          }
          const __half2 scale = q * kConvThreads >= kRawBytes / 32 ? sc_hi : sc_lo;  // runs 8-15: second half
          const uint32_t words[4] = {v.x, v.y, v.z, v.w};
          uint32_t h[8];
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            e4m3x4_to_f16x2x2(words[w], h[2 * w], h[2 * w + 1]);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const __half2 hv = __hmul2(*reinterpret_cast<const __half2*>(&h[2 * w + hh]), scale);
              h[2 * w + hh] = *reinterpret_cast<const uint32_t*>(&hv);
            }
          }
          // k 16c .. 16c + 15 of this stage = 16-byte chunks 2c, 2c + 1 of row n
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int chunk = 2 * c + j;
            unsigned char* dst = bt + (n / 8) * 1024 + (n % 8) * 128 + ((chunk ^ (n % 8)) * 16);
            st_shared_v4(dst, h[4 * j], h[4 * j + 1], h[4 * j + 2], h[4 * j + 3]);
          }
        }
        fence_proxy_async_shared();  // generic-proxy writes -> visible to the tensor core (async proxy)
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->cfull[b]);
      }
      if (!ok) break;
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      uint32_t it = 0, ti = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < tiles && ok && !*abort; t += gridDim.x) {
        const TileRef tr = tile_at(t, a.mprefix, a.seg_offset, a.n_segments, n_tiles);
        if (!present(tr.seg)) continue;
        const bool two = tr.rows > kSubM;
        // the epilogue has drained the previous tile's accumulators
        if (ti >= 1 && !wait_or_abort(&bars->tempty, (ti - 1) & 1, abort)) break;
        tc_fence_after();
        for (int kh = 0; kh < nkh; ++kh, ++it) {
          const int s = it % kStages, b = it % kConvBufs;
          if (!wait_or_abort(&bars->full[s], (it / kStages) & 1, abort) ||
              !wait_or_abort(&bars->cfull[b], (it / kConvBufs) & 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa0 = smem_addr(a_tile(s, 0)), sa1 = smem_addr(a_tile(s, 1)), sbt = smem_addr(b_tile(b));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t bdesc = sw128_desc(sbt + k * 32);
            umma_f16(tmem, sw128_desc(sa0 + k * 32), bdesc, kIdesc, (kh | k) != 0);
            if (two) umma_f16(tmem + kBN, sw128_desc(sa1 + k * 32), bdesc, kIdesc, (kh | k) != 0);
          }
          umma_commit(&bars->empty[s]);   // A + raw stage free once these MMAs complete
          umma_commit(&bars->cempty[b]);  // and the converted buffer
        }
        if (ok) umma_commit(&bars->tfull);
        ++ti;
      }
      // every MMA this thread issued has completed before TMEM is released
      umma_commit(&bars->drain);
      mbar_wait(&bars->drain, 0, kCodeWait);
    }
  } else if (warp < kEpiWarps) {
    // warp w drains TMEM lanes 32 (w % 4) .. + 31 of sub-tile w / 4 (columns 256 (w / 4) ..)
    uint32_t ti = 0;
    const int half = warp / 4, quad = warp % 4;
    unsigned char* stage = stage_buf + warp * kStageBytes;
    const int row_in_tile = half * kSubM + quad * kWarp + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * kWarp) << 16;
    for (int64_t t = blockIdx.x; t < tiles && !*abort; t += gridDim.x) {
      const TileRef tr = tile_at(t, a.mprefix, a.seg_offset, a.n_segments, n_tiles);
      if (!present(tr.seg)) {
        // absent expert: its pairs' output rows are zero
        if (row_in_tile < tr.rows) {
          const int64_t pz = tr.row0 + row_in_tile;
          if (!GATEUP && (a.out16 || (a.out_row && a.out_row_bf16))) {
            __nv_bfloat16* row16 =
                a.out16 ? a.out16 + pz * N : reinterpret_cast<__nv_bfloat16*>(a.out_row[pz]);
            uint4* out = reinterpret_cast<uint4*>(row16 + tr.nt * kBN);
            for (int j = 0; j < kBN / 8; ++j) out[j] = make_uint4(0u, 0u, 0u, 0u);
          } else {
            float* row = !GATEUP && a.out_row ? reinterpret_cast<float*>(a.out_row[pz]) : a.out + pz * N;
            float4* out = reinterpret_cast<float4*>(row + tr.nt * (GATEUP ? kBN / 2 : kBN));
            for (int j = 0; j < (GATEUP ? kBN / 2 : kBN) / 4; ++j) out[j] = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
        continue;
      }
      if (!wait_or_abort(&bars->tfull, ti & 1, abort)) break;
      tc_fence_after();
      // the second sub-tile's accumulator was not written for tiles of <= 128 pairs
      const bool live = half == 0 || tr.rows > kSubM;
      const uint32_t taddr = tmem + half * kBN + lane_off;
      const bool valid = row_in_tile < tr.rows;
      const int64_t p = tr.row0 + row_in_tile;
      const float xs = valid ? a.ascale[p] : 0.0f;
      // int4 weights: fp16 scale of each output column (weight row), else none
      const __half* csc0 = WF == kPrefillQ4Row ? reinterpret_cast<const __half*>(a.s0[tr.seg]) +
                                                     static_cast<int64_t>(tr.nt) * (GATEUP ? kBN / 2 : kBN)
                                               : nullptr;
      const __half* csc1 = WF == kPrefillQ4Row && GATEUP
                               ? reinterpret_cast<const __half*>(a.s1[tr.seg]) + static_cast<int64_t>(tr.nt) * (kBN / 2)
                               : nullptr;
      // down (256 fp32 per row): 16 columns of the warp's 32 rows at a time
      // leave through its 2 KiB staging buffer -- lane = row on the way in,
      // four lanes per row (64 contiguous bytes) on the way out; 16-byte
      // slots XOR-swizzled by row so both phases are free of bank conflicts
      const int row_base = half * kSubM + quad * kWarp;  // the warp's first row in the tile
      // the output rows this lane stores in emit64: rows lane / 4 + 8 i of the warp's 32 (byte addresses of
      // the tile's first column: fp32 rows, or bf16 rows with out16)
      const bool y16 = !GATEUP && (a.out16 != nullptr || (a.out_row && a.out_row_bf16));
      unsigned char* out_row[4] = {nullptr, nullptr, nullptr, nullptr};
      if (!GATEUP) {
        unsigned char* mine = nullptr;
        if (valid)
          mine = y16 ? reinterpret_cast<unsigned char*>(
                           (a.out16 ? a.out16 + p * N : reinterpret_cast<__nv_bfloat16*>(a.out_row[p])) + tr.nt * kBN)
                     : reinterpret_cast<unsigned char*>(
                           (a.out_row ? reinterpret_cast<float*>(a.out_row[p]) : a.out + p * N) + tr.nt * kBN);
        const uint64_t m64 = reinterpret_cast<uint64_t>(mine);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int src = lane / 4 + 8 * i;
          const uint32_t lo = __shfl_sync(0xFFFFFFFFu, static_cast<uint32_t>(m64), src);
          const uint32_t hi = __shfl_sync(0xFFFFFFFFu, static_cast<uint32_t>(m64 >> 32), src);
          out_row[i] = reinterpret_cast<unsigned char*>((static_cast<uint64_t>(hi) << 32) | lo);
        }
      }
      // 64 bytes of each of the warp's rows (16 fp32 or 32 bf16 columns) starting at byte b0 of the tile
      auto emit64 = [&](const uint32_t (&v)[16], int b0) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          st_shared_v4(stage + lane * 64 + ((j ^ ((lane >> 1) & 3)) * 16), v[4 * j], v[4 * j + 1], v[4 * j + 2],
                       v[4 * j + 3]);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int rr = lane / 4 + 8 * i, j = lane % 4;
          const uint4 w = ld_shared_v4(stage + rr * 64 + ((j ^ ((rr >> 1) & 3)) * 16));
          if (row_base + rr < tr.rows) *reinterpret_cast<uint4*>(out_row[i] + b0 + 16 * j) = w;
        }
        __syncwarp();
      };
      if (!live) {
      } else if (GATEUP) {
        // 128 SwiGLU outputs per row: direct 16-byte stores from each row's lane
        float* out = a.out + p * N + tr.nt * (kBN / 2);
#pragma unroll 1
        for (int c0 = 0; c0 < kBN / 2; c0 += 16) {
          uint32_t gr[16], ur[16];
          tmem_ld16(taddr + c0, gr);
          tmem_ld16(taddr + kBN / 2 + c0, ur);
          tmem_ld_wait();
          if (valid) {
#pragma unroll
            for (int j = 0; j < 16; j += 4) {
              float4 o;
              float* op = &o.x;
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                float g = __uint_as_float(gr[j + q]) * xs, u = __uint_as_float(ur[j + q]) * xs;
                if (WF == kPrefillQ4Row) {
                  g *= __half2float(csc0[c0 + j + q]);
                  u *= __half2float(csc1[c0 + j + q]);
                }
                op[q] = g / (1.0f + expf(-g)) * u;
              }
              *reinterpret_cast<float4*>(out + c0 + j) = o;
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c0 = 0; c0 < kBN; c0 += 32) {
          uint32_t d0[16], d1[16];
          tmem_ld16(taddr + c0, d0);
          tmem_ld16(taddr + c0 + 16, d1);
          tmem_ld_wait();
          float o0[16], o1[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            o0[q] = __uint_as_float(d0[q]) * xs * (WF == kPrefillQ4Row ? __half2float(csc0[c0 + q]) : 1.0f);
            o1[q] = __uint_as_float(d1[q]) * xs * (WF == kPrefillQ4Row ? __half2float(csc0[c0 + 16 + q]) : 1.0f);
          }
          uint32_t w[16];
          if (y16) {
            // 32 columns rounded to bf16, two per word
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const __nv_bfloat162 lo = __floats2bfloat162_rn(o0[2 * q], o0[2 * q + 1]);
              const __nv_bfloat162 hi = __floats2bfloat162_rn(o1[2 * q], o1[2 * q + 1]);
              w[q] = *reinterpret_cast<const uint32_t*>(&lo);
              w[8 + q] = *reinterpret_cast<const uint32_t*>(&hi);
            }
            emit64(w, c0 * 2);
          } else {
#pragma unroll
            for (int q = 0; q < 16; ++q) w[q] = __float_as_uint(o0[q]);
            emit64(w, c0 * 4);
#pragma unroll
            for (int q = 0; q < 16; ++q) w[q] = __float_as_uint(o1[q]);
            emit64(w, (c0 + 16) * 4);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->tempty);
      ++ti;
    }
  }

  // rows stored to another GPU's memory are visible there once this grid ends
  if (!GATEUP && a.out_row && warp < kEpiWarps) __threadfence_system();
  // all roles done; the MMA issuer saw its last commit arrive (drain)
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kAllocWarp) tmem_dealloc(tmem, kTmemCols);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// ------------------------------------------------------- router logits
// Prefill-sized router GEMM on tcgen05: partial[z][t][e] = sum over the z-th
// k-range of x[t, k] * w[e, k], x and w both bf16 or both f16 (products
// exact in fp32, fp32 accumulation in tensor memory) -- the reference's fp32
// F.linear of the gate (fp8_source.py:1547) up to the order of the sums.
// One CTA per (128-token tile, expert tile of <= 256, k-range): TMA loads
// both operands (128B swizzle, 64 columns per stage, four stages), one
// thread issues M = 128 x N MMAs, four warps drain TMEM to the partials.
constexpr int kRStages = 4;
constexpr int kRATile = 128 * 64 * 2;   // 16 KiB
constexpr int kRBTile = 256 * 64 * 2;   // 32 KiB (up to 256 experts)
constexpr int kRThreads = 6 * kWarp;    // warps 0-3 epilogue, 4 producer, 5 MMA + TMEM
struct RBarriers {
  uint64_t full[kRStages];
  uint64_t empty[kRStages];
  uint64_t tfull;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};
constexpr size_t kRSmemBytes = 1024 + static_cast<size_t>(kRStages) * (kRATile + kRBTile) + sizeof(RBarriers);
static_assert(kRSmemBytes <= 232448, "shared memory per block");

template <bool BF16>
__global__ void __launch_bounds__(kRThreads, 1) router_tc_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                                 const __grid_constant__ CUtensorMap tmap_w,
                                                                 float* partial, int tokens, int experts, int ncols,
                                                                 int n_tiles, int nkh, int parts) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto a_tile = [&](int s) { return smem + s * (kRATile + kRBTile); };
  auto b_tile = [&](int s) { return smem + s * (kRATile + kRBTile) + kRATile; };
  RBarriers* bars = reinterpret_cast<RBarriers*>(smem + kRStages * (kRATile + kRBTile));
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  volatile int* abort = &bars->abort;
  const int m0 = (blockIdx.x / n_tiles) * 128, n0 = (blockIdx.x % n_tiles) * ncols;
  const int z = blockIdx.y;
  const int kh0 = static_cast<int>(static_cast<int64_t>(z) * nkh / parts);
  const int kh1 = static_cast<int>(static_cast<int64_t>(z + 1) * nkh / parts);
  const uint32_t b_bytes = static_cast<uint32_t>(ncols) * 64 * 2;
  const uint32_t idesc = (1u << 4) | (BF16 ? (1u << 7) | (1u << 10) : 0u) |
                         (static_cast<uint32_t>(ncols >> 3) << 17) | (static_cast<uint32_t>(128 >> 4) << 24);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->tfull, 1);
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(&bars->tmem_base, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 4) {
    if (lane == 0) {
      uint32_t it = 0;
      for (int kh = kh0; kh < kh1 && !*abort; ++kh, ++it) {
        const int s = it % kRStages;
        if (it >= kRStages && !wait_or_abort(&bars->empty[s], ((it / kRStages) - 1) & 1, abort)) break;
        mbar_arrive_expect_tx(&bars->full[s], kRATile + b_bytes);
        tma_load_2d(a_tile(s), &tmap_x, kh * 64, m0, &bars->full[s]);
        tma_load_2d(b_tile(s), &tmap_w, kh * 64, n0, &bars->full[s]);
      }
      for (uint32_t j = it > kRStages ? it - kRStages : 0; j < it; ++j)
        mbar_wait(&bars->full[j % kRStages], (j / kRStages) & 1, kCodeWait);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int kh = kh0; kh < kh1; ++kh, ++it) {
        const int s = it % kRStages;
        if (!wait_or_abort(&bars->full[s], (it / kRStages) & 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_addr(a_tile(s)), sb = smem_addr(b_tile(s));
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16(tmem, sw128_desc(sa + k * 32), sw128_desc(sb + k * 32), idesc, (it | k) != 0);
        umma_commit(&bars->empty[s]);
      }
      if (ok) umma_commit(&bars->tfull);
      umma_commit(&bars->drain);
      mbar_wait(&bars->drain, 0, kCodeWait);
    }
  } else {
    // epilogue: warp w drains TMEM lanes 32w .. 32w + 31 (tokens m0 + 32w + lane)
    if (wait_or_abort(&bars->tfull, 0, abort)) {
      tc_fence_after();
      const int t = m0 + warp * kWarp + lane;
      float* row = partial + (static_cast<int64_t>(z) * tokens + t) * experts + n0;
      const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * kWarp) << 16);
      const bool vec = experts % 4 == 0;
#pragma unroll 1
      for (int c0 = 0; c0 < ncols; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(taddr + c0, r);
        tmem_ld_wait();
        if (t < tokens) {
          if (vec && n0 + c0 + 16 <= experts) {
#pragma unroll
            for (int j = 0; j < 16; j += 4)
              *reinterpret_cast<float4*>(row + c0 + j) = make_float4(
                  __uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (n0 + c0 + j < experts) row[c0 + j] = __uint_as_float(r[j]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem, 256);
}

}  // namespace

size_t prefill_smem_bytes() { return kSmemBytes; }

bool prefill_supported(int64_t K, int64_t N, bool gateup) {
  return K > 0 && N > 0 && K % 128 == 0 && (gateup ? N % (kBN / 2) == 0 : N % kBN == 0);
}

cudaError_t launch_prefill_tiles(const int32_t* seg_offset, int n_segments, int32_t* mprefix, cudaStream_t stream) {
  prefill_tiles_kernel<<<1, 32, 0, stream>>>(seg_offset, n_segments, mprefix);
  return cudaGetLastError();
}

cudaError_t launch_gather_rows(const __half* x16, const float* xscale, const int32_t* pair_row, int64_t P, int64_t K,
                               __half* xa, float* ascale, cudaStream_t stream) {
  if (P <= 0) return cudaSuccess;
  if (K % 8 != 0) return cudaErrorInvalidValue;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(ceil_div(P * kWarp, 256), gemv_grid_ctas() * 16));
  gather_rows_kernel<<<grid, 256, 0, stream>>>(x16, xscale, pair_row, P, K, xa, ascale);
  return cudaGetLastError();
}

cudaError_t launch_prefill_gemm(const PrefillArgs& a, bool gateup, int64_t max_tiles, cudaStream_t stream) {
  if (!prefill_supported(a.K, a.N, gateup) || a.rows_a <= 0) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.a16) & 15u) != 0) return cudaErrorInvalidValue;
  // outputs: rows of out, or (down GEMM only) the row table
  if (gateup ? (!a.out || a.out_row || a.out16) : (!a.out && !a.out_row && !a.out16)) return cudaErrorInvalidValue;
  if (a.out16 && (a.out_row || (reinterpret_cast<uintptr_t>(a.out16) & 15u) != 0 || a.N % 8 != 0))
    return cudaErrorInvalidValue;
  auto encode = encode_fn();
  if (!encode) return cudaErrorNotSupported;
  // A boxes of 128, 64 and 32 rows (the smaller ones for small tiles)
  CUtensorMap tmap[3];
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(a.K), static_cast<cuuint64_t>(a.rows_a)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.K) * 2};
  const cuuint32_t estr[2] = {1, 1};
  for (int i = 0; i < 3; ++i) {
    const cuuint32_t box[2] = {kBK, static_cast<cuuint32_t>(kSubM >> i)};
    if (encode(&tmap[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(a.a16), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  const bool q4 = a.wformat == kPrefillQ4Row;
  auto kernel = gateup ? (q4 ? prefill_gemm_kernel<true, kPrefillQ4Row> : prefill_gemm_kernel<true, kPrefillFp8Block>)
                       : (q4 ? prefill_gemm_kernel<false, kPrefillQ4Row> : prefill_gemm_kernel<false, kPrefillFp8Block>);
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes));
  if (err != cudaSuccess) return err;
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(gemv_grid_ctas(), max_tiles)));
  kernel<<<grid, kThreads, kSmemBytes, stream>>>(tmap[0], tmap[1], tmap[2], a);
  return cudaGetLastError();
}

int router_tc_parts(int64_t tokens, int64_t hidden, int64_t experts) {
  const int64_t ncols = experts >= 256 ? 256 : (experts + 15) / 16 * 16;
  const int64_t tiles = ceil_div(tokens, 128) * ceil_div(experts, ncols);
  const int64_t nkh = hidden / 64;
  // fill the SMs with k-ranges of at least eight stages, at most kMaxRouterTcParts ranges
  int64_t parts = std::max<int64_t>(1, gemv_grid_ctas() / std::max<int64_t>(1, tiles));
  // (and no more than the split-K router's parts, which size the callers' partial buffers)
  parts = std::min<int64_t>({parts, kMaxRouterTcParts, std::max<int64_t>(1, nkh / 8),
                             std::max<int64_t>(1, router_split_parts(static_cast<int>(hidden)))});
  return static_cast<int>(parts);
}

cudaError_t launch_router_logits_tc(const void* x, int xdtype, const void* w, int wdtype, float* partial,
                                    int64_t tokens, int64_t hidden, int64_t experts, int* nparts,
                                    cudaStream_t stream) {
  // both operands bf16 or both f16, 16-byte aligned rows, whole 64-column stages
  if (xdtype != wdtype || (xdtype != kDtypeBF16 && xdtype != kDtypeF16)) return cudaErrorNotSupported;
  if (hidden % 64 != 0 || tokens <= 0 || experts <= 0 || experts > 2048) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15u) return cudaErrorNotSupported;
  auto encode = encode_fn();
  if (!encode) return cudaErrorNotSupported;
  const bool bf16 = xdtype == kDtypeBF16;
  const int ncols = experts >= 256 ? 256 : static_cast<int>((experts + 15) / 16 * 16);
  const int n_tiles = static_cast<int>(ceil_div(experts, ncols));
  const int parts = router_tc_parts(tokens, hidden, experts);
  const CUtensorMapDataType dt = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tx, tw;
  const cuuint32_t estr[2] = {1, 1};
  const cuuint64_t xdims[2] = {static_cast<cuuint64_t>(hidden), static_cast<cuuint64_t>(tokens)};
  const cuuint64_t wdims[2] = {static_cast<cuuint64_t>(hidden), static_cast<cuuint64_t>(experts)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(hidden) * 2};
  const cuuint32_t xbox[2] = {64, 128};
  const cuuint32_t wbox[2] = {64, static_cast<cuuint32_t>(ncols)};
  if (encode(&tx, dt, 2, const_cast<void*>(x), xdims, strides, xbox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
          CUDA_SUCCESS ||
      encode(&tw, dt, 2, const_cast<void*>(w), wdims, strides, wbox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
          CUDA_SUCCESS)
    return cudaErrorNotSupported;
  auto kernel = bf16 ? router_tc_kernel<true> : router_tc_kernel<false>;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kRSmemBytes));
  if (err != cudaSuccess) return err;
  dim3 grid(static_cast<unsigned>(ceil_div(tokens, 128) * n_tiles), static_cast<unsigned>(parts));
  kernel<<<grid, kRThreads, kRSmemBytes, stream>>>(tx, tw, partial, static_cast<int>(tokens), static_cast<int>(experts),
                                                   ncols, n_tiles, static_cast<int>(hidden / 64), parts);
  *nparts = parts;
  return cudaGetLastError();
}

int64_t q4_tiled_bytes(int64_t rows, int64_t K) { return (rows + 127) / 128 * 128 * (K / 2); }

cudaError_t launch_q4_tile(const uint8_t* packed, uint8_t* tiled, int64_t rows, int64_t K, cudaStream_t stream) {
  if (rows <= 0 || K <= 0) return cudaSuccess;
  if (K % 64 != 0 || (reinterpret_cast<uintptr_t>(packed) & 15u) || (reinterpret_cast<uintptr_t>(tiled) & 15u))
    return cudaErrorInvalidValue;
  const int64_t units = q4_tiled_bytes(rows, K) / 16;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(ceil_div(units, 256), gemv_grid_ctas() * 16));
  q4_tile_kernel<<<grid, 256, 0, stream>>>(packed, tiled, rows, K);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_scatter_t(const void* x, int64_t T_, int64_t K, const int32_t* entry_pair, int k,
                                    const int32_t* tail_first, __half* a16, float* ascale, cudaStream_t stream) {
  const int64_t pieces = K * static_cast<int64_t>(sizeof(T)) / 16;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(T_, gemv_grid_ctas() * 8));
  const T* xs = static_cast<const T*>(x);
  if (pieces <= 256)
    scatter_rows_kernel<T, 1><<<grid, 256, 0, stream>>>(xs, static_cast<int>(T_), static_cast<int>(K), entry_pair, k,
                                                        tail_first, a16, ascale);
  else if (pieces <= 512)
    scatter_rows_kernel<T, 2><<<grid, 256, 0, stream>>>(xs, static_cast<int>(T_), static_cast<int>(K), entry_pair, k,
                                                        tail_first, a16, ascale);
  else if (pieces <= 1024)
    scatter_rows_kernel<T, 4><<<grid, 256, 0, stream>>>(xs, static_cast<int>(T_), static_cast<int>(K), entry_pair, k,
                                                        tail_first, a16, ascale);
  else
    return cudaErrorNotSupported;
  return cudaGetLastError();
}

cudaError_t launch_scatter_rows(const void* x, int x_dtype, int64_t T_, int64_t K, const int32_t* entry_pair, int k,
                                const int32_t* tail_first, __half* a16, float* ascale, cudaStream_t stream) {
  if (T_ <= 0) return cudaSuccess;
  if (K % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15u)) return cudaErrorNotSupported;
  switch (x_dtype) {
    case kDtypeBF16: return launch_scatter_t<__nv_bfloat16>(x, T_, K, entry_pair, k, tail_first, a16, ascale, stream);
    case kDtypeF16: return launch_scatter_t<__half>(x, T_, K, entry_pair, k, tail_first, a16, ascale, stream);
    case kDtypeF32: return launch_scatter_t<float>(x, T_, K, entry_pair, k, tail_first, a16, ascale, stream);
    default: return cudaErrorNotSupported;
  }
}

int read_and_clear_prefill_device_error(cudaStream_t stream) { return read_and_clear_local_error(stream); }

}  // namespace moe
