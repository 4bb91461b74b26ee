// common.cuh -- shared device helpers for the NVFP4 MoE kernels (sm_100a).
//
// NVFP4 storage format (the reference's MLX "nvfp4" mode, group 16):
//   * codes: 8 E2M1 nibbles per uint32, element k of a row at bits 4*(k%8) of
//     word k/8 (low nibble first); nibble bit 3 is the sign
//     (backend/cpu/quantized.cpp:31-47, ops.cpp:4958-4962).
//   * scales: one byte per 16 consecutive elements of a row, decoded as MLX's
//     FromFP8 does (backend/cpu/unary_ops.h:154-172): the bits (b & 0x7F) << 7
//     read as an IEEE half, times 256, sign from bit 7.  Byte 0x7F decodes to
//     480 (not NaN as in OCP E4M3), so the hardware e4m3 converter is NOT used
//     for scales.
// Every product LUT[code] * scale has <= 6 significant bits and lies in
// [2^-10, 2880], so it is exact in f16: dequantisation to f16 is bit-exact.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace nvfp4 {

// ---------------------------------------------------------------------------
// dtype tags shared with the C ABI (include/nvfp4moe.h).
enum DType : int { kBF16 = 0, kF16 = 1, kF32 = 2 };

__device__ __forceinline__ float load_as_f32(const void* p, int dtype, int64_t i) {
  if (dtype == kBF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == kF16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_from_f32(void* p, int dtype, int64_t i, float v) {
  if (dtype == kBF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else if (dtype == kF16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

// ---------------------------------------------------------------------------
// E2M1 pairs -> f16x2.  One hardware conversion per byte: the low nibble
// lands in the low half.  Four bytes of a 32-bit word give four f16x2.
__device__ __forceinline__ void e2m1x8_to_f16x2x4(uint32_t w, uint32_t (&h)[4]) {
  asm(
      "{\n"
      ".reg .b8 b0, b1, b2, b3;\n"
      "mov.b32 {b0, b1, b2, b3}, %4;\n"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n"
      "}\n"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
}

// One E2M1 code -> f32 (exact), arithmetically: magnitude code m is
// 0.5*m for m < 2, else (1 + (m&1)/2) * 2^(m/2 - 1); bit 3 is the sign.
__device__ __forceinline__ float fp4_to_f32(uint32_t code) {
  const uint32_t m = code & 7u;
  const float mag = m < 2u ? 0.5f * (float)m : ldexpf(1.0f + 0.5f * (float)(m & 1u), (int)(m >> 1) - 1);
  return (code & 8u) ? -mag : mag;
}

// Scale byte pair (lo byte -> low half) -> f16x2 of the MLX E4M3 decode.
__device__ __forceinline__ uint32_t scale2_to_f16x2(uint32_t two_bytes) {
  const uint32_t b0 = two_bytes & 0xFFu, b1 = (two_bytes >> 8) & 0xFFu;
  const uint32_t h0 = ((b0 & 0x7Fu) << 7) | ((b0 & 0x80u) << 8);
  const uint32_t h1 = ((b1 & 0x7Fu) << 7) | ((b1 & 0x80u) << 8);
  uint32_t packed = h0 | (h1 << 16);
  __half2 v = *reinterpret_cast<__half2*>(&packed);
  v = __hmul2(v, __half2half2(__float2half_rn(256.0f)));
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float scale_to_f32(uint32_t b) {
  const uint32_t h = ((b & 0x7Fu) << 7);
  const float v = __half2float(__ushort_as_half((unsigned short)h)) * 256.0f;
  return (b & 0x80u) ? -v : v;
}

// f32 -> E4M3 byte as MLX's ToFP8 rounds it (backend/cpu/unary_ops.h:120-151):
// round-to-nearest-even on the bit pattern, subnormals through a float add,
// saturation at 0x7E, the sign copied.
__device__ __forceinline__ uint32_t e4m3_encode(float f) {
  uint32_t bits = __float_as_uint(f);
  const uint32_t sign = bits & 0x80000000u;
  bits ^= sign;
  uint32_t r;
  if (bits >= (543u << 21)) {
    r = 0x7Eu;
  } else if (bits < (121u << 23)) {
    const uint32_t magic = 141u << 23;
    r = (__float_as_uint(__fadd_rn(__uint_as_float(bits), __uint_as_float(magic))) - magic) &
        0xFFu;
  } else {
    const uint32_t odd = (bits >> 20) & 1u;
    r = ((bits + ((uint32_t)(7 - 127) << 23) + 0x7FFFFu + odd) >> 20) & 0xFFu;
  }
  return r | (sign >> 24);
}

// MLX to_fp4_e2m1: round to the nearest E2M1 magnitude with ties to the even
// code, saturating at 6; NaN -> +6 (code 7); the sign bit from signbit().
__device__ __forceinline__ uint32_t fp4_code_mlx(float v) {
  if (isnan(v)) return 0x7u;
  const uint32_t sign = signbit(v) ? 0x8u : 0u;
  const float a = fabsf(v);
  uint32_t m;
  if (a > 5.0f) m = 7;
  else if (a >= 3.5f) m = 6;
  else if (a > 2.5f) m = 5;
  else if (a >= 1.75f) m = 4;
  else if (a > 1.25f) m = 3;
  else if (a >= 0.75f) m = 2;
  else if (a > 0.25f) m = 1;
  else m = 0;
  return m | sign;
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// Broadcast the low / high half of an f16x2 to both halves.
__device__ __forceinline__ uint32_t bcast_lo(uint32_t v) { return __byte_perm(v, 0, 0x1010); }
__device__ __forceinline__ uint32_t bcast_hi(uint32_t v) { return __byte_perm(v, 0, 0x3232); }

// ---------------------------------------------------------------------------
// Warp-level m16n8k16 f16 x f16 -> f32 (accumulate in place).
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                              uint32_t a2, uint32_t a3, uint32_t b0,
                                              uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Streaming 128-bit global load that does not allocate in L1 (weights are
// read exactly once per call).
__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ldg_stream_u16(const void* p) {
  unsigned short r;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];\n" : "=h"(r) : "l"(p));
  return r;
}

// Eight consecutive activation elements (elem_off % 8 == 0, 16-byte aligned).
__device__ __forceinline__ void load8(const void* x, int dtype, int64_t elem_off, float (&f)[8]) {
  if (dtype == kF32) {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + elem_off);
    const float4 b =
        *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + elem_off + 4);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    const uint4 v = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(x) + elem_off);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      if (dtype == kBF16) {
        const float2 p = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
        f[2 * i] = p.x; f[2 * i + 1] = p.y;
      } else {
        const float2 p = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        f[2 * i] = p.x; f[2 * i + 1] = p.y;
      }
    }
  }
}

// Eight consecutive output elements (elem_off % 8 == 0, 16-byte aligned).
__device__ __forceinline__ void store8_from_f32(void* y, int dtype, int64_t elem_off,
                                                const float (&f)[8]) {
  if (dtype == kF32) {
    float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(y) + elem_off);
    d[0] = make_float4(f[0], f[1], f[2], f[3]);
    d[1] = make_float4(f[4], f[5], f[6], f[7]);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      if (dtype == kBF16) {
        const __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&b);
      } else {
        const __half2 b = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&b);
      }
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(y) + elem_off) =
        make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Power-of-two exponent e with max_abs * 2^-e in [1, 2); 0 for zero / non-finite.
// Clamped at -100 so that 2^-e stays a finite f32: a row whose largest
// magnitude is below 2^-100 stages as zeros (its products are below 2^-100 times
// the weights' norm) instead of overflowing the reciprocal to inf.
__device__ __forceinline__ int pow2_exponent(float max_abs) {
  if (!(max_abs > 0.0f) || !isfinite(max_abs)) return 0;
  int e;
  frexpf(max_abs, &e);  // max_abs = m * 2^e, m in [0.5, 1)
  return max(e - 1, -100);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// SiLU exactly as the reference composes it: g * sigmoid(g) with
// sigmoid(x) = x < 0 ? 1/(1+e^|x|) : 1 - 1/(1+e^|x|)  (backend/cpu/unary_ops.h:77-84).
// 1/(1+e^|x|) is the correctly rounded reciprocal (the same bits as the IEEE
// division 1.0f / y, without its general-operand path).
__device__ __forceinline__ float sigmoid_ref(float x) {
  const float y = __frcp_rn(1.0f + expf(fabsf(x)));
  return x < 0.0f ? y : 1.0f - y;
}
__device__ __forceinline__ float silu_ref(float g) { return g * sigmoid_ref(g); }

}  // namespace nvfp4
