// mbarrier + bulk-copy (TMA, non-tensor) helpers for sm_90+/sm_100a, in
// inline PTX.  Every wait is bounded: after kWaitLimitNs of %globaltimer the
// wait gives up, records `code` in the device error word and returns false.
#pragma once
#include "common.cuh"

namespace moe {

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Device error word: nonzero after a bounded wait gave up (moe_b200_device_error).
// Defined per translation unit (no relocatable device code); only
// fp8_stream.cu includes this header and reads the word back.
static __device__ int g_device_error = 0;

// Host: read this translation unit's error word, clear it, return it (-1 if unreadable).
static inline int read_and_clear_local_error(cudaStream_t stream) {
  int host = 0;
  if (cudaMemcpyFromSymbolAsync(&host, g_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return -1;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return -1;
  if (host) {
    const int zero = 0;
    cudaMemcpyToSymbolAsync(g_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    cudaStreamSynchronize(stream);
  }
  return host;
}

// Order this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) writes to the same shared memory.
MOE_D void fence_proxy_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

MOE_D uint32_t smem_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

MOE_D uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

MOE_D void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Make barrier initialisation visible to the async (TMA) proxy.
MOE_D void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

MOE_D void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_addr(bar))
               : "memory");
}

MOE_D void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(
                   smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

MOE_D bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps (issuing nothing) until
// the phase completes or about `hint_ns` pass, instead of spinning.
MOE_D bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Wait until the phase with the given parity has completed; false on timeout.
MOE_D bool mbar_wait(uint64_t* bar, uint32_t parity, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - start > kWaitLimitNs) {
      atomicOr(&g_device_error, code);
      return false;
    }
  }
  return true;
}

// 1-D bulk copy global -> shared of this CTA, completing on `bar` (tx bytes).
// Both addresses 16-byte aligned, `bytes` a multiple of 16.
MOE_D void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

MOE_D void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace moe
