// Scratch planning shared by the C entry points: a bump allocator over one
// workspace block, and the caller's workspace or a stream-ordered allocation.
#pragma once
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "common.cuh"

namespace moe {

// Bump allocator over one workspace block; sizes round up to 256 bytes.
class Plan {
 public:
  explicit Plan(char* base = nullptr) : base_(base) {}
  template <typename T>
  T* take(int64_t count) {
    const size_t bytes = (static_cast<size_t>(count > 0 ? count : 1) * sizeof(T) + 255) & ~size_t(255);
    T* p = base_ ? reinterpret_cast<T*>(base_ + used_) : nullptr;
    used_ += bytes;
    return p;
  }
  size_t used() const { return used_; }

 private:
  char* base_;
  size_t used_ = 0;
};

// Either the caller's workspace or a stream-ordered allocation freed at scope end.
class Scratch {
 public:
  Scratch(void* workspace, int64_t bytes, size_t need, cudaStream_t stream) : stream_(stream) {
    if (workspace) {
      ok_ = bytes >= static_cast<int64_t>(need);
      base_ = static_cast<char*>(workspace);
    } else {
      ok_ = cudaMallocAsync(reinterpret_cast<void**>(&base_), need > 0 ? need : 256, stream) == cudaSuccess;
      owned_ = ok_;
    }
  }
  ~Scratch() {
    if (owned_) cudaFreeAsync(base_, stream_);
  }
  bool ok() const { return ok_; }
  char* base() const { return base_; }

 private:
  cudaStream_t stream_;
  char* base_ = nullptr;
  bool ok_ = false;
  bool owned_ = false;
};

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

inline unsigned grid_for(int64_t n, int threads = 256) {
  return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, threads), 4096)));
}

}  // namespace moe
