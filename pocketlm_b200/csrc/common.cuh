// Shared device helpers for the sm_100a MoE kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define MOE_HD __host__ __device__ __forceinline__
#define MOE_D __device__ __forceinline__

namespace moe {

constexpr int kBlock = 128;  // FP8 scale block edge (128x128)
constexpr int kWarp = 32;

// Return codes shared by every C entry point (the reference uses small
// negative codes for argument errors, fp8_linear.cpp:60-65).
enum Status : int {
  kOk = 0,
  kNullPointer = -1,
  kBadDims = -2,
  kNoMemory = -3,
  kBadIndex = -4,
  kUnsupported = -5,
  kCudaError = -100,  // kCudaError - cudaError_t
};

MOE_HD int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------------------
// FP8 e4m3 decode
// ---------------------------------------------------------------------------

// Clear the all-ones codes 0x7F / 0xFF of four packed e4m3 bytes.  The
// reference's linear/MLP kernels decode those codes as +0.0
// (fp8_linear.cpp:31-33) where the hardware conversion yields NaN; clearing
// the byte to 0x00 gives exactly +0.0.
MOE_D uint32_t e4m3x4_nan_to_zero(uint32_t w) {
  // (byte & 0x7F) + 1 reaches bit 7 exactly when byte & 0x7F == 0x7F (no
  // carry crosses a byte); prmt's sign mode spreads each bit 7 over its byte
  const uint32_t s = (w & 0x7F7F7F7Fu) + 0x01010101u;
  uint32_t mask;
  asm("prmt.b32 %0, %1, 0, 0xBA98;" : "=r"(mask) : "r"(s));
  return w & ~mask;
}

// Four e4m3 bytes -> two fp16x2 words (exact): lo = bytes 0, 1; hi = bytes 2, 3.
// The 32-bit word is split into its 16-bit halves inside the asm, so no
// extract / repack instructions surround the two conversions.
MOE_D void e4m3x4_to_f16x2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("{\n .reg .b16 l, h;\n mov.b32 {l, h}, %2;\n cvt.rn.f16x2.e4m3x2 %0, l;\n cvt.rn.f16x2.e4m3x2 %1, h;\n}"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}

// Two e4m3 bytes (low half of `pair`) -> two floats (exact).
MOE_D float2 e4m3x2_to_float2(uint16_t pair) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(pair), __NV_E4M3);
  return __half22float2(*reinterpret_cast<__half2*>(&h));
}

// Four e4m3 bytes -> four floats, NaN codes decoded as +0.0.
MOE_D void e4m3x4_to_float4(uint32_t w, float* out) {
  w = e4m3x4_nan_to_zero(w);
  const float2 lo = e4m3x2_to_float2(static_cast<uint16_t>(w & 0xFFFFu));
  const float2 hi = e4m3x2_to_float2(static_cast<uint16_t>(w >> 16));
  out[0] = lo.x;
  out[1] = lo.y;
  out[2] = hi.x;
  out[3] = hi.y;
}

// One e4m3 byte -> float with the reference's linear semantics.
MOE_D float e4m3_to_float_zero_nan(uint8_t b) {
  if ((b & 0x7Fu) == 0x7Fu) return 0.0f;
  return e4m3x2_to_float2(b).x;
}

// ---------------------------------------------------------------------------
// 16-bit float helpers
// ---------------------------------------------------------------------------

MOE_D float bf16_bits_to_float(uint16_t v) { return __uint_as_float(static_cast<uint32_t>(v) << 16); }

MOE_D float f16_bits_to_float(uint16_t v) { return __half2float(__ushort_as_half(v)); }

// dtype_code: 0 = fp16, 1 = bf16 (the reference's u16 storage code,
// native/__init__.py:141-146).
MOE_D float u16_to_float(uint16_t v, int dtype_code) {
  return dtype_code == 1 ? bf16_bits_to_float(v) : f16_bits_to_float(v);
}

MOE_D uint16_t float_to_bf16_bits(float v) { return __bfloat16_as_ushort(__float2bfloat16_rn(v)); }

MOE_D uint16_t float_to_f16_bits(float v) { return __half_as_ushort(__float2half_rn(v)); }

MOE_D uint16_t float_to_u16(float v, int dtype_code) {
  return dtype_code == 1 ? float_to_bf16_bits(v) : float_to_f16_bits(v);
}

// Load 4 consecutive activations of type T as floats.
template <typename T>
MOE_D void load4(const T* p, float* out);

template <>
MOE_D void load4<float>(const float* p, float* out) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  out[0] = v.x;
  out[1] = v.y;
  out[2] = v.z;
  out[3] = v.w;
}

template <>
MOE_D void load4<__nv_bfloat16>(const __nv_bfloat16* p, float* out) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  out[0] = __uint_as_float(v.x << 16);
  out[1] = __uint_as_float(v.x & 0xFFFF0000u);
  out[2] = __uint_as_float(v.y << 16);
  out[3] = __uint_as_float(v.y & 0xFFFF0000u);
}

template <typename T>
MOE_D float to_float(T v);
template <>
MOE_D float to_float<float>(float v) { return v; }
template <>
MOE_D float to_float<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// ---------------------------------------------------------------------------
// Warp reductions
// ---------------------------------------------------------------------------

MOE_D float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// Arg-max over the warp; ties go to the lower index (the tie rule of the
// reference's partial_sort comparator, ds_forward.cpp:931-943).
MOE_D void warp_argmax(float& v, int& idx) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xFFFFFFFFu, v, o);
    const int oi = __shfl_xor_sync(0xFFFFFFFFu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
}

// 16 bytes of activations -> floats (4 fp32, or 8 bf16 / f16 values), exactly.
template <typename T>
MOE_D void unpack16(const uint4& v, float* out);

template <>
MOE_D void unpack16<float>(const uint4& v, float* out) {
  out[0] = __uint_as_float(v.x);
  out[1] = __uint_as_float(v.y);
  out[2] = __uint_as_float(v.z);
  out[3] = __uint_as_float(v.w);
}

template <>
MOE_D void unpack16<__nv_bfloat16>(const uint4& v, float* out) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = __uint_as_float(w[i] << 16);
    out[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

template <>
MOE_D void unpack16<__half>(const uint4& v, float* out) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}

}  // namespace moe
