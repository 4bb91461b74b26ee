// gemv.cuh -- the decode GEMV engine shared by qmv.cu and decode_stack.cu: a
// warp owns 16 weight rows x up to 8 activation columns and walks K in chunks
// of 128 codes; E2M1 pairs through the hardware converter, the group scale
// folded in with one HMUL2 (exact), mma.sync m16n8k16 f16 -> f32 into two
// independent accumulator sets.  K inside a chunk is permuted (thread t's 32
// codes are K [32t, 32t+32), MMA i takes codes 4i..4i+3) and the activation
// column in shared memory uses the same permutation plus an XOR swizzle.
#pragma once

#include "common.cuh"

namespace nvfp4 {

constexpr int kChunk = 128;       // codes per row per chunk
constexpr int kChunkBytes = 64;   // packed bytes per row per chunk
constexpr int kChunkScales = 8;   // scale bytes per row per chunk
constexpr int kXPad = 32;         // f16 padding per column: 64 B bank offset

// Physical f16 index of logical element k of a staged column.
__device__ __forceinline__ int xs_swz(int k) {
  const int c = k >> 7, r = k & 127;
  const int b = r * 2;
  const int t = b >> 6, q = (b >> 4) & 3, o = b & 15;
  return (c << 7) + (((t << 6) + ((q ^ t) << 4) + o) >> 1);
}

struct Chunk {
  uint4 lo, hi;
  uint32_t slo, shi;
};


struct Acc {
  float a[4], b[4];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int r = 0; r < 4; r++) a[r] = b[r] = 0.f;
  }
  __device__ __forceinline__ void fold(float (&out)[4]) const {
#pragma unroll
    for (int r = 0; r < 4; r++) out[r] = a[r] + b[r];
  }
};

__device__ __forceinline__ void compute_chunk(Acc& acc, const Chunk& c, const __half* xcol,
                                              int ch, int t) {
  uint32_t xb[16];
  if (xcol) {
    const uint4* base = reinterpret_cast<const uint4*>(xcol + ch * kChunk);
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const uint4 v = base[t * 4 + (q ^ t)];
      xb[4 * q + 0] = v.x;
      xb[4 * q + 1] = v.y;
      xb[4 * q + 2] = v.z;
      xb[4 * q + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int q = 0; q < 16; q++) xb[q] = 0u;
  }
  const uint32_t SL = scale2_to_f16x2(c.slo), SH = scale2_to_f16x2(c.shi);
  const uint32_t sl[2] = {bcast_lo(SL), bcast_hi(SL)};
  const uint32_t sh[2] = {bcast_lo(SH), bcast_hi(SH)};
  const uint32_t wl[4] = {c.lo.x, c.lo.y, c.lo.z, c.lo.w};
  const uint32_t wh[4] = {c.hi.x, c.hi.y, c.hi.z, c.hi.w};
#pragma unroll
  for (int j = 0; j < 4; j++) {
    uint32_t hl[4], hh[4];
    e2m1x8_to_f16x2x4(wl[j], hl);
    e2m1x8_to_f16x2x4(wh[j], hh);
    const uint32_t s_l = sl[j >> 1], s_h = sh[j >> 1];
    mma_f16_16816(acc.a, hmul2_u32(hl[0], s_l), hmul2_u32(hh[0], s_h), hmul2_u32(hl[1], s_l),
                  hmul2_u32(hh[1], s_h), xb[4 * j], xb[4 * j + 1]);
    mma_f16_16816(acc.b, hmul2_u32(hl[2], s_l), hmul2_u32(hh[2], s_h), hmul2_u32(hl[3], s_l),
                  hmul2_u32(hh[3], s_h), xb[4 * j + 2], xb[4 * j + 3]);
  }
}


// Eight f16 of one staged column, logical elements k..k+7 (k % 8 == 0): the
// swizzle moves whole 16-byte groups, so they stay contiguous.
__device__ __forceinline__ void store8_f16(__half* col, int k, const float (&f)[8], float mul) {
  uint32_t h[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const __half2 v = __floats2half2_rn(f[2 * i] * mul, f[2 * i + 1] * mul);
    h[i] = *reinterpret_cast<const uint32_t*>(&v);
  }
  *reinterpret_cast<uint4*>(col + xs_swz(k)) = make_uint4(h[0], h[1], h[2], h[3]);
}

// Max over a warp, then one shared atomic per warp and column.  Non-negative
// floats order like their bit patterns.
__device__ __forceinline__ void warp_atomic_max(int* slot, float m, bool active) {
  m = warp_max(active ? m : 0.f);
  if ((threadIdx.x & 31) == 0) atomicMax(slot, __float_as_int(m));
}


__device__ __forceinline__ int tma_row_pitch(int K) { return K / 2 + 64; }
__device__ __forceinline__ int tma_scale_pitch(int K) { return K / 16 + 16; }

// Chunk `ch` of a 16-row tile held in shared memory.
__device__ __forceinline__ void load_chunk_smem(Chunk& c, const uint8_t* tile, int rp, int sp,
                                                int g, int ch, int t) {
  c.lo = *reinterpret_cast<const uint4*>(tile + g * rp + ch * kChunkBytes + 16 * t);
  c.hi = *reinterpret_cast<const uint4*>(tile + (g + 8) * rp + ch * kChunkBytes + 16 * t);
  const uint8_t* sc = tile + 16 * rp;
  c.slo = *reinterpret_cast<const uint16_t*>(sc + g * sp + ch * kChunkScales + 2 * t);
  c.shi = *reinterpret_cast<const uint16_t*>(sc + (g + 8) * sp + ch * kChunkScales + 2 * t);
}


}  // namespace nvfp4
