// moe_fp8_e4m3_block_mlp_f32_noalloc: the FP8 expert MLP without any device
// allocation.
//
// Some callers of this library cannot call cudaMalloc, or let a library call
// it for them: a serving process that reserves the whole GPU for its own
// memory arena at start-up (so any further allocation fails or fragments the
// arena), a host whose hot path must not take the CUDA allocator's locks or
// risk the implicit device synchronisation of cudaMalloc/cudaFree, or a thin
// binding (ctypes, cgo, JNI) that only passes device pointers it already owns
// and has no allocator from which to hand out scratch space.  This entry point
// takes only their inputs and outputs; its intermediate buffers (the expert
// pointer table, the chunk list and the fp32 SwiGLU activations) live in one
// fixed-size device array compiled into the library.
#include <algorithm>
#include <mutex>

#include "../../include/moe_b200.h"
#include "dispatch.cuh"
#include "fp8_gemv.cuh"
#include "status.cuh"

namespace moe {
namespace {

constexpr size_t kNoAllocBytes = MOE_B200_NOALLOC_SCRATCH_BYTES;

// The scratch.  Every GPU that loads the library holds one copy until the
// process exits.  In host code this name is only a host-side stand-in, not a
// device address: it must never be passed to a kernel.  noalloc_scratch()
// resolves the real address on the current device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch on the current device, looked up once per
// device with that device current (cudaGetSymbolAddress).  Because that
// first lookup happens inside the first call on a device, the first call on
// each device should come before any stream capture.
int noalloc_scratch(void** out) {
  int dev = 0;
  MOE_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(kUnsupported, "no-alloc scratch: device index beyond 64");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    MOE_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(no-alloc scratch)");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return kOk;
}

size_t round256(size_t n) { return (n + 255) & ~size_t(255); }

struct Layout {
  size_t table, seg, n_chunks, chunk_seg, chunk_start, chunk_len, act, total;
};

Layout layout_for(int64_t batch, int64_t inter, int nt) {
  const int64_t cap = chunk_capacity(batch, 2, nt);
  Layout l{};
  size_t at = 0;
  l.table = at;       at += round256(6 * sizeof(uint64_t));
  l.seg = at;         at += round256(2 * sizeof(int32_t));
  l.n_chunks = at;    at += round256(sizeof(int32_t));
  l.chunk_seg = at;   at += round256(cap * sizeof(int32_t));
  l.chunk_start = at; at += round256(cap * sizeof(int32_t));
  l.chunk_len = at;   at += round256(cap * sizeof(int32_t));
  l.act = at;         at += round256(static_cast<size_t>(batch) * inter * sizeof(float));
  l.total = at;
  return l;
}

// Writes the one-expert pointer table and the single segment [0, batch).
// Everything else the calls read is rewritten by each call before use, so
// nothing left over from a previous call is ever read.
__global__ void noalloc_setup_kernel(uint64_t* table, int32_t* seg, uint64_t g, uint64_t gs, uint64_t u,
                                     uint64_t us, uint64_t d, uint64_t ds, int32_t batch) {
  table[0] = g;
  table[1] = gs;
  table[2] = u;
  table[3] = us;
  table[4] = d;
  table[5] = ds;
  seg[0] = 0;
  seg[1] = batch;
}

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" int moe_fp8_e4m3_block_mlp_f32_noalloc(const uint8_t* gate_weight, const float* gate_scale_inv,
                                                  const uint8_t* up_weight, const float* up_scale_inv,
                                                  const uint8_t* down_weight, const float* down_scale_inv,
                                                  const float* hidden, float* out, int64_t batch, int64_t I,
                                                  int64_t H, int64_t gsc, int64_t dsc, void* stream) {
  if (!gate_weight || !gate_scale_inv || !up_weight || !up_scale_inv || !down_weight || !down_scale_inv ||
      !hidden || !out)
    return fail(kNullPointer, "null pointer");
  if (batch <= 0 || I <= 0 || H <= 0 || gsc <= 0 || dsc <= 0) return fail(kBadDims, "bad dimensions");
  if (gsc != ceil_div(H, kBlock) || dsc != ceil_div(I, kBlock))
    return fail(kBadDims, "scale columns do not match the 128x128 block layout");
  // sizes checked before any product is formed: the kernels take int dimensions, and the activations
  // (batch x I fp32) alone must fit the static scratch
  if (I > INT32_MAX || H > INT32_MAX) return fail(kUnsupported, "no-alloc MLP: dimension beyond int32");
  if (batch > static_cast<int64_t>(kNoAllocBytes / sizeof(float)) / I) {
    static thread_local char msg[256];
    std::snprintf(msg, sizeof msg,
                  "no-alloc MLP needs more than %zu bytes of scratch for batch=%lld intermediate=%lld; the static "
                  "limit is %zu bytes (MOE_B200_NOALLOC_SCRATCH_BYTES)",
                  kNoAllocBytes, static_cast<long long>(batch), static_cast<long long>(I), kNoAllocBytes);
    return fail(kNoMemory, msg);
  }
  int nt = batch <= 1 ? 1 : (batch <= 4 ? 4 : 8);
  const int cap = std::min(gemv_chunk_tokens(static_cast<int>(H), kXF32), gemv_chunk_tokens(static_cast<int>(I), kXF32));
  if (cap <= 0) return fail(kUnsupported, "hidden/intermediate size too large for the staged GEMV");
  while (nt > cap) nt = nt == 8 ? 4 : 1;
  const Layout l = layout_for(batch, I, nt);
  if (l.total > kNoAllocBytes) {
    static thread_local char msg[256];
    std::snprintf(msg, sizeof msg,
                  "no-alloc MLP needs %zu bytes of scratch for batch=%lld intermediate=%lld; the static limit is "
                  "%zu bytes (MOE_B200_NOALLOC_SCRATCH_BYTES)",
                  l.total, static_cast<long long>(batch), static_cast<long long>(I), kNoAllocBytes);
    return fail(kNoMemory, msg);
  }
  void* base_v = nullptr;
  const int code = noalloc_scratch(&base_v);
  if (code != kOk) return code;
  char* base = static_cast<char*>(base_v);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint64_t* table = reinterpret_cast<uint64_t*>(base + l.table);
  int32_t* seg = reinterpret_cast<int32_t*>(base + l.seg);
  noalloc_setup_kernel<<<1, 1, 0, s>>>(table, seg, reinterpret_cast<uint64_t>(gate_weight),
                                       reinterpret_cast<uint64_t>(gate_scale_inv), reinterpret_cast<uint64_t>(up_weight),
                                       reinterpret_cast<uint64_t>(up_scale_inv), reinterpret_cast<uint64_t>(down_weight),
                                       reinterpret_cast<uint64_t>(down_scale_inv), static_cast<int32_t>(batch));
  MOE_CUDA(cudaGetLastError(), "no-alloc setup");
  ChunkArgs ca{seg, 1, nt,
               reinterpret_cast<int32_t*>(base + l.chunk_seg), reinterpret_cast<int32_t*>(base + l.chunk_start),
               reinterpret_cast<int32_t*>(base + l.chunk_len), reinterpret_cast<int32_t*>(base + l.n_chunks)};
  MOE_CUDA(launch_chunks(ca, s), "no-alloc chunk list");
  float* act = reinterpret_cast<float*>(base + l.act);
  const bool vec = H % 16 == 0 && I % 16 == 0 && (reinterpret_cast<uintptr_t>(hidden) & 15u) == 0;
  GemvArgs g1{};
  g1.w0 = table;
  g1.s0 = table + 1;
  g1.w1 = table + 2;
  g1.s1 = table + 3;
  g1.x = hidden;
  g1.pair_row = nullptr;
  g1.chunk_seg = ca.chunk_seg;
  g1.chunk_start = ca.chunk_start;
  g1.chunk_len = ca.chunk_len;
  g1.n_chunks = ca.n_chunks;
  g1.out0 = act;
  g1.N = static_cast<int>(I);
  g1.K = static_cast<int>(H);
  g1.scale_cols = static_cast<int>(gsc);
  MOE_CUDA(launch_grouped_gemv(g1, kXF32, 2, kEpiSwiglu, nt, vec, s), "no-alloc gate/up");
  GemvArgs g2 = g1;
  g2.w0 = table + 4;
  g2.s0 = table + 5;
  g2.w1 = nullptr;
  g2.s1 = nullptr;
  g2.x = act;
  g2.out0 = out;
  g2.N = static_cast<int>(H);
  g2.K = static_cast<int>(I);
  g2.scale_cols = static_cast<int>(dsc);
  MOE_CUDA(launch_grouped_gemv(g2, kXF32, 1, kEpiStore, nt, I % 16 == 0, s), "no-alloc down");
  return kOk;
}
