// topk.cuh -- the Laguna router's selection step on one warp, shared by the
// router kernels (router.cu) and the routed decode stack (decode_stack_fp4.cu).
//
// Semantics (VLM/MLXLLM/Models/Laguna.swift:165-180, LagunaMoEGate): from the
// logits (already rounded to the activation dtype, as the reference's matmul
// returns them) s = sigmoid(logit) (backend/cpu/unary_ops.h:77-84),
// choice = s + bias, top-k by choice (ties to the lower expert id; the
// reference's argPartition leaves them unspecified), weights s / sum(s) of
// the chosen experts when norm_topk_prob.  Slots in descending choice order.
#pragma once

#include "common.cuh"

namespace nvfp4 {

// One 64-bit key per candidate: the choice's bits made order-preserving as an
// unsigned integer, then the complement of the expert id (equal choices: the
// lower id is the larger key); 0 marks an entry already taken, padding, or a
// NaN choice (never chosen, as a NaN never compares greater).
__device__ __forceinline__ uint64_t choice_key(float c, uint32_t e) {
  if (!(c > -INFINITY)) return 0ull;  // -inf (padding) and NaN
  const uint32_t b = __float_as_uint(c + 0.0f);  // -0 as +0: equal choices tie by id
  const uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((uint64_t)o << 32) | (uint64_t)(0xFFFFFFFFu - e);
}

// Called by a whole warp.  Lane owns experts lane + 32 j, j < kPer
// (E <= 32 kPer); logit[j] is that expert's rounded logit.  Lane r < k ends
// with slot r: its expert id (0x7fffffff when fewer than k experts have a
// finite choice) and weight.  A round is a lane-local max over the lane's
// keys, the warp max of the key (two redux.sync: the high words, then the low
// words among the lanes holding that high word) and the winner's score from
// its lane.
template <int kPer>
__device__ __forceinline__ void topk_select(const float (&logit)[kPer], const float* bias, int E,
                                            int k, bool norm, int lane, uint32_t& isel,
                                            float& wsel) {
  float sc[kPer];
  uint64_t key[kPer];
#pragma unroll
  for (int j = 0; j < kPer; j++) {
    const int e = lane + 32 * j;
    const bool live = e < E;
    const float sg = sigmoid_ref(logit[j]);
    sc[j] = live ? sg : 0.f;
    key[j] = live ? choice_key(sg + (bias ? bias[e] : 0.f), (uint32_t)e) : 0ull;
  }
  float wsum = 0.f;
  wsel = 0.f;
  isel = 0;
  for (int r = 0; r < k; r++) {
    uint64_t bk = key[0];
    float bs = sc[0];
#pragma unroll
    for (int j = 1; j < kPer; j++)
      if (key[j] > bk) {
        bk = key[j];
        bs = sc[j];
      }
    const uint32_t hi = (uint32_t)(bk >> 32);
    const uint32_t mhi = __reduce_max_sync(0xffffffffu, hi);
    const uint32_t mlo = __reduce_max_sync(0xffffffffu, hi == mhi ? (uint32_t)bk : 0u);
    const uint64_t wk = ((uint64_t)mhi << 32) | mlo;
    const uint32_t bid = wk ? 0xFFFFFFFFu - (uint32_t)wk : 0x7fffffffu;
    const float ws = __shfl_sync(0xffffffffu, bs, (int)(bid & 31));
    if (wk && (int)(bid & 31) == lane) {
#pragma unroll
      for (int j = 0; j < kPer; j++)
        if (key[j] == wk) key[j] = 0ull;
    }
    const float s = wk ? ws : 0.f;
    wsum += s;
    if (lane == r) {
      wsel = s;
      isel = bid;
    }
  }
  if (norm) wsel = wsel / wsum;
}

__device__ __forceinline__ float round_to_dtype(float v, int dtype) {
  if (dtype == kBF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dtype == kF16) return __half2float(__float2half_rn(v));
  return v;
}

}  // namespace nvfp4
