// fp4terms.cuh -- device helpers for carrying activations as sums of NVFP4
// terms on the block-scaled tensor cores (prefill_fp4.cu, decode_stack_fp4.cu):
// the UE4M3 scale rounding up and the hardware E2M1 pair conversions.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"

namespace nvfp4 {

// Smallest E4M3 magnitude >= v (v >= 0, v <= 448).
__device__ __forceinline__ uint32_t e4m3_ceil(float v) {
  uint32_t b = e4m3_encode(v) & 0x7Fu;
  if (scale_to_f32(b) < v && b < 0x7Eu) b++;
  return b;
}

// The same for 0 <= v <= 448, branch-free above 2^-6: below 2^-6 the
// subnormal steps k * 2^-9 (k = ceil(v * 2^9), 8 meaning 2^-6); from 2^-6 up the
// float's mantissa rounded up to 3 bits (a carry moves into the exponent) and
// the exponent rebased from bias 127 to bias 7; saturated at 0x7E (448).
__device__ __forceinline__ uint32_t e4m3_ceil_fast(float v) {
  if (v < 0.015625f) return (uint32_t)ceilf(v * 512.0f);
  const uint32_t r = ((__float_as_uint(v) + 0xFFFFFu) >> 20) - (120u << 3);
  return min(r, 0x7Eu);
}

// Two values -> one byte of E2M1 codes, rounded to nearest even and saturated
// at +-6 by the hardware converter (first operand in the high nibble), and the
// byte back to the two exact values.
__device__ __forceinline__ uint32_t e2m1_pair(float lo, float hi) {
  uint32_t r;
  asm("{\n.reg .b8 t;\ncvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\ncvt.u32.u8 %0, t;\n}"
      : "=r"(r)
      : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ float2 e2m1_pair_value(uint32_t byte) {
  uint32_t h;
  asm("{\n.reg .b8 t;\ncvt.u8.u32 t, %1;\ncvt.rn.f16x2.e2m1x2 %0, t;\n}" : "=r"(h) : "r"(byte));
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

}  // namespace nvfp4
