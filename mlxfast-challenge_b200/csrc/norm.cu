// norm.cu -- RMSNorm of activation rows on sm_100a, the norm that feeds each
// Laguna MoE block (post_attention_layernorm, VLM/MLXLLM/Models/
// Laguna.swift:242-246) in the per-layer decode path.
//
// Semantics: MLX fast::rms_norm as the CPU evaluates it (its fallback graph,
// mlx/fast.cpp:90-108): x32 = f32(x); x32 *= rsqrt(mean(x32^2) + eps);
// x = dtype(x32); y = dtype(x * w).  One CTA per row; the sum of squares is
// f32 in a fixed order (per-thread strided sums, then a fixed tree), so the
// result is the same on every run.  r = 1 / sqrt(v) with IEEE division and
// square root.
#include "common.cuh"
#include "kernels.h"
#include "topk.cuh"

namespace nvfp4 {
namespace {

constexpr int kNormThreads = 256;

__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(NormArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ float part[kNormThreads / 32];
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t base = row * a.H;
  float s = 0.f;
  for (int64_t i = tid; i < a.H; i += kNormThreads) {
    const float v = load_as_f32(a.x, a.dtype, base + i);
    s += v * v;
  }
  s = warp_sum(s);
  if (lane == 0) part[warp] = s;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; w++) tot += part[w];
  const float r = 1.0f / sqrtf(tot / (float)a.H + a.eps);
  for (int64_t i = tid; i < a.H; i += kNormThreads) {
    const float v = round_to_dtype(load_as_f32(a.x, a.dtype, base + i) * r, a.dtype);
    const float w = a.w ? load_as_f32(a.w, a.dtype, i) : 1.0f;
    store_from_f32(a.y, a.dtype, base + i, v * w);
  }
}

}  // namespace

cudaError_t launch_rms_norm(const NormArgs& a, cudaStream_t stream, bool pdl) {
  if (a.T <= 0) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.T);
  cfg.blockDim = dim3(kNormThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, rms_norm_kernel, a);
}

}  // namespace nvfp4
