// FP8 e4m3 128x128 block dequantisation to fp16 / bf16.
//
// Replaces fp8_e4m3_dequant_to_fp16 / _to_bf16
// (src/pcketlm/native/fp8_dequant.cpp:119-204): out = round(e4m3(w) * scale)
// with round-to-nearest-even.  The all-ones codes are NaN there, with fixed
// payloads: the fp16 path yields 0x7F80 / 0xFF80 (the F16C conversion of the
// NaN the reference builds, fp8_dequant.cpp:22-27) and the bf16 path 0xFFFF
// (fp8_dequant.cpp:109-111).  This kernel reproduces those bits exactly.
// HBM-bound: one pass, 1 byte in and 2 bytes out per element.
#include "common.cuh"
#include "dequant.cuh"
#include <algorithm>

namespace moe {

template <bool BF16>
MOE_D uint16_t dequant_one(uint8_t code, float scale) {
  if ((code & 0x7Fu) == 0x7Fu) {
    if (BF16) return 0xFFFFu;
    return (code & 0x80u) ? 0xFF80u : 0x7F80u;
  }
  const float v = e4m3x2_to_float2(code).x * scale;
  return BF16 ? float_to_bf16_bits(v) : float_to_f16_bits(v);
}

// Vector path: each thread converts 16 consecutive codes of one row
// (cols % 16 == 0, 16-byte aligned rows).
template <bool BF16>
__global__ void dequant_vec_kernel(const uint8_t* __restrict__ w, const float* __restrict__ s,
                                   uint16_t* __restrict__ out, int64_t rows, int64_t cols, int64_t scale_cols) {
  const int64_t n16 = rows * (cols / 16);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n16;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / (cols / 16), c = (i % (cols / 16)) * 16;
    const float scale = __ldg(s + (r / kBlock) * scale_cols + c / kBlock);
    const uint4 raw = __ldcs(reinterpret_cast<const uint4*>(w + r * cols + c));
    const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
    uint32_t packed[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t wd = words[j];
      uint16_t h[4];
#pragma unroll
      for (int b = 0; b < 4; ++b) h[b] = dequant_one<BF16>(static_cast<uint8_t>(wd >> (8 * b)), scale);
      packed[2 * j] = h[0] | (static_cast<uint32_t>(h[1]) << 16);
      packed[2 * j + 1] = h[2] | (static_cast<uint32_t>(h[3]) << 16);
    }
    uint4* dst = reinterpret_cast<uint4*>(out + r * cols + c);
    __stcs(dst, make_uint4(packed[0], packed[1], packed[2], packed[3]));
    __stcs(dst + 1, make_uint4(packed[4], packed[5], packed[6], packed[7]));
  }
}

template <bool BF16>
__global__ void dequant_scalar_kernel(const uint8_t* __restrict__ w, const float* __restrict__ s,
                                      uint16_t* __restrict__ out, int64_t rows, int64_t cols, int64_t scale_cols) {
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    out[i] = dequant_one<BF16>(w[i], s[(r / kBlock) * scale_cols + c / kBlock]);
  }
}

cudaError_t launch_fp8_dequant(const uint8_t* w, const float* s, uint16_t* out, int64_t rows, int64_t cols,
                               int64_t scale_cols, bool bf16, cudaStream_t stream) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const bool vec = cols % 16 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(out) % 16 == 0;
  const int threads = 256;
  const int64_t items = vec ? rows * (cols / 16) : rows * cols;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(ceil_div(items, threads), int64_t(sms) * 8));
  if (grid == 0) return cudaSuccess;
  if (vec) {
    if (bf16) dequant_vec_kernel<true><<<grid, threads, 0, stream>>>(w, s, out, rows, cols, scale_cols);
    else dequant_vec_kernel<false><<<grid, threads, 0, stream>>>(w, s, out, rows, cols, scale_cols);
  } else {
    if (bf16) dequant_scalar_kernel<true><<<grid, threads, 0, stream>>>(w, s, out, rows, cols, scale_cols);
    else dequant_scalar_kernel<false><<<grid, threads, 0, stream>>>(w, s, out, rows, cols, scale_cols);
  }
  return cudaGetLastError();
}

}  // namespace moe
