// quant.cu -- NVFP4 (group 16) quantize / dequantize on sm_100a.
//
// dequantize follows fp_dequantize (ops.cpp:5120-5241): LUT[code] * e4m3(s),
// exact in every output dtype.
//
// quantize follows fp_quantize (ops.cpp:4873-4978) as it evaluates on a CPU
// stream for bf16 / f16 / f32 weights, op by op, with the rounding each op of
// that graph performs:
//   amax  = max |w| over the group                 (exact)
//   scale = round_T(amax / 6)                      (T = the weight dtype)
//   sb    = e4m3_encode(scale)                     (MLX ToFP8, saturating at 0x7E)
//   q     = round_T(w / round_T(e4m3_decode(sb)))  then widened to f32
//   code  = argmin_i |q - LUT[i]|, first minimum wins (so all-NaN -> 0)
// The E4M3 encoder restates the bit algorithm of ToFP8
// (backend/cpu/unary_ops.h:120-151): it has to round exactly like the
// reference for the scale bytes to be bit-exact.
#include "common.cuh"
#include "kernels.h"

namespace nvfp4 {
namespace {

__device__ __forceinline__ float round_to(float v, int dtype) {
  if (dtype == kBF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dtype == kF16) return __half2float(__float2half_rn(v));
  return v;
}

__device__ __forceinline__ int argmin_fp4(float q) {
  int best = 0;
  float bv = fabsf(q - fp4_to_f32(0));
#pragma unroll
  for (int i = 1; i < 16; i++) {
    const float d = fabsf(q - fp4_to_f32(i));
    if (d < bv) {
      bv = d;
      best = i;
    }
  }
  return best;
}

// One thread per group of 16 elements.
__global__ void quantize_kernel(uint8_t* wq, uint8_t* sq, const void* w, int dtype,
                                int64_t groups) {
  for (int64_t gi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; gi < groups;
       gi += (int64_t)gridDim.x * blockDim.x) {
    float v[16];
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 16; j++) {
      v[j] = load_as_f32(w, dtype, gi * 16 + j);
      amax = fmaxf(amax, fabsf(v[j]));
    }
    const float scale = round_to(__fdiv_rn(amax, 6.0f), dtype);
    const uint32_t sb = e4m3_encode(scale);
    const float sdec = round_to(scale_to_f32(sb), dtype);
    uint32_t words[2] = {0u, 0u};
#pragma unroll
    for (int j = 0; j < 16; j++) {
      const float q = round_to(__fdiv_rn(v[j], sdec), dtype);
      words[j >> 3] |= (uint32_t)argmin_fp4(q) << (4 * (j & 7));
    }
    reinterpret_cast<uint2*>(wq)[gi] = make_uint2(words[0], words[1]);
    sq[gi] = (uint8_t)sb;
  }
}

// One thread per packed word (8 outputs).
__global__ void dequantize_kernel(void* out, int dtype, const uint8_t* w, const uint8_t* s,
                                  int64_t words) {
  for (int64_t wi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; wi < words;
       wi += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t word = reinterpret_cast<const uint32_t*>(w)[wi];
    const float scale = scale_to_f32(s[wi >> 1]);
    uint32_t h[4];
    e2m1x8_to_f16x2x4(word, h);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[j]));
      store_from_f32(out, dtype, wi * 8 + 2 * j, f.x * scale);
      store_from_f32(out, dtype, wi * 8 + 2 * j + 1, f.y * scale);
    }
  }
}

unsigned grid_for(int64_t n, int threads) {
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + threads - 1) / threads, 148 * 32));
}

}  // namespace

cudaError_t launch_dequantize(void* out, int dtype, const uint8_t* w, const uint8_t* s,
                              int64_t rows, int64_t K, cudaStream_t stream) {
  const int64_t words = rows * (K / 8);
  if (words == 0) return cudaSuccess;
  dequantize_kernel<<<grid_for(words, 256), 256, 0, stream>>>(out, dtype, w, s, words);
  return cudaGetLastError();
}

cudaError_t launch_quantize(uint8_t* wq, uint8_t* sq, const void* w, int dtype, int64_t rows,
                            int64_t K, cudaStream_t stream) {
  const int64_t groups = rows * (K / 16);
  if (groups == 0) return cudaSuccess;
  quantize_kernel<<<grid_for(groups, 256), 256, 0, stream>>>(wq, sq, w, dtype, groups);
  return cudaGetLastError();
}

}  // namespace nvfp4
