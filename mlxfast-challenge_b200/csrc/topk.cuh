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

// The same selection by sorting and merging, for k <= K (K = 8 or 16), in a
// fixed number of steps instead of k dependent rounds of warp reductions: each
// lane sorts its kPer keys (a bitonic network in registers) and keeps its top
// K; five butterfly levels (lane xor 1, 2, 4, 8, 16) each merge the lane's
// list with its partner's (max of the list and the reversed partner list is
// bitonic and holds the top K of both; a half-cleaner cascade sorts it), so
// every lane ends with the warp's top K in descending key order -- the order,
// ties and NaN handling of topk_select.  score / bias: the lane's sigmoid
// scores and biases (bias 0 where there is none).  The weight sum runs over
// slots 0..k-1 in order, as topk_select's.
template <int N>
__device__ __forceinline__ void sort_keys_desc(uint64_t (&v)[N]) {
#pragma unroll
  for (int size = 2; size <= N; size <<= 1)
#pragma unroll
    for (int stride = size / 2; stride > 0; stride >>= 1)
#pragma unroll
      for (int i = 0; i < N; i++) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const uint64_t a = v[i], b = v[j];
          const bool sw = desc ? (b > a) : (b < a);
          v[i] = sw ? b : a;
          v[j] = sw ? a : b;
        }
      }
}

// Butterfly levels lane xor o, o = o_first, 2 o_first, .. < o_end, on
// descending lists of K keys (the max of the list and the reversed partner
// list is bitonic and holds the top K of both; a half-cleaner cascade sorts
// it): afterwards lanes that differ only in those bits hold the same list.
template <int K>
__device__ __forceinline__ void merge_levels(uint64_t (&t)[K], int o_first, int o_end) {
  for (int o = o_first; o < o_end; o <<= 1) {
    uint64_t p[K];
#pragma unroll
    for (int i = 0; i < K; i++) {
      const uint32_t lo = __shfl_xor_sync(0xffffffffu, (uint32_t)t[i], o);
      const uint32_t hi = __shfl_xor_sync(0xffffffffu, (uint32_t)(t[i] >> 32), o);
      p[i] = ((uint64_t)hi << 32) | lo;
    }
#pragma unroll
    for (int i = 0; i < K; i++) t[i] = t[i] > p[K - 1 - i] ? t[i] : p[K - 1 - i];
#pragma unroll
    for (int stride = K / 2; stride > 0; stride >>= 1)
#pragma unroll
      for (int i = 0; i < K; i++) {
        const int j = i ^ stride;
        if (j > i) {
          const uint64_t a = t[i], b = t[j];
          t[i] = b > a ? b : a;
          t[j] = b > a ? a : b;
        }
      }
  }
}

// Slots 0 .. k-1 of a sorted key list (the same on every lane): lane r < k
// gets slot r's expert id and weight (its score from scores[id], shared
// memory; weights / their sum in slot order when norm).
template <int K>
__device__ __forceinline__ void slots_from_keys(const uint64_t (&t)[K], const float* scores, int k,
                                                bool norm, int lane, uint32_t& isel, float& wsel) {
  float wsum = 0.f;
  wsel = 0.f;
  isel = 0;
#pragma unroll
  for (int r = 0; r < K; r++) {
    if (r >= k) break;
    const uint64_t key = t[r];
    const uint32_t id = key ? 0xFFFFFFFFu - (uint32_t)key : 0x7fffffffu;
    const float s = key ? scores[id] : 0.f;
    wsum += s;
    if (lane == r) {
      wsel = s;
      isel = id;
    }
  }
  if (norm) wsel = wsel / wsum;
}

template <int kPer, int K>
__device__ __forceinline__ void topk_merge(const float (&score)[kPer], const float (&bias)[kPer],
                                           int E, int k, bool norm, int lane, uint32_t& isel,
                                           float& wsel, float* scratch = nullptr) {
  constexpr int NS = kPer > K ? kPer : K;
  uint64_t v[NS];
#pragma unroll
  for (int j = 0; j < NS; j++) {
    const int e = lane + 32 * j;
    v[j] = (j < kPer && e < E) ? choice_key(score[j < kPer ? j : 0] + bias[j < kPer ? j : 0],
                                            (uint32_t)e)
                               : 0ull;
  }
  sort_keys_desc<NS>(v);
  uint64_t t[K];
#pragma unroll
  for (int i = 0; i < K; i++) t[i] = v[i];
  merge_levels<K>(t, 1, 32);
  // slot r = t[r]; its score from the expert's lane (id % 32, entry id / 32):
  // through `scratch` (32 kPer floats of this warp's shared memory) when
  // given, else by shuffles
  float wsum = 0.f;
  wsel = 0.f;
  isel = 0;
  if (scratch) {
#pragma unroll
    for (int j = 0; j < kPer; j++) scratch[lane + 32 * j] = score[j];
    __syncwarp();
  }
#pragma unroll
  for (int r = 0; r < K; r++) {
    if (r >= k) break;
    const uint64_t key = t[r];
    const uint32_t id = key ? 0xFFFFFFFFu - (uint32_t)key : 0x7fffffffu;
    float s = 0.f;
    if (scratch) {
      s = key ? scratch[id] : 0.f;
    } else {
#pragma unroll
      for (int j = 0; j < kPer; j++) {
        const float sj = __shfl_sync(0xffffffffu, score[j], (int)(id & 31));
        if (key && (int)(id >> 5) == j) s = sj;
      }
    }
    wsum += s;
    if (lane == r) {
      wsel = s;
      isel = id;
    }
  }
  if (scratch) __syncwarp();  // the scratch may be reused after the call
  if (norm) wsel = wsel / wsum;
}

__device__ __forceinline__ float round_to_dtype(float v, int dtype) {
  if (dtype == kBF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dtype == kF16) return __half2float(__float2half_rn(v));
  return v;
}

}  // namespace nvfp4
