// router.cu -- the Laguna MoE router on sm_100a: BF16 logits GEMV, sigmoid,
// bias-for-choice top-k and renormalisation in one launch.
//
// Semantics (VLM/MLXLLM/Models/Laguna.swift:165-180, LagunaMoEGate):
//   logits = x @ G^T            -- bf16 operands, f32 accumulation; for bf16
//                                  x the result is rounded to bf16 as the
//                                  reference's bf16 matmul returns it
//   s      = sigmoid(f32 logits) (backend/cpu/unary_ops.h:77-84)
//   choice = s + bias
//   top-k of choice             -- ties go to the lower expert id (the
//                                  reference's argPartition leaves them
//                                  unspecified)
//   w      = s[top] / sum(s[top]) when norm_topk_prob
// Slots are written in descending choice order.
//
// Layout of the launch: grid (E/16 expert tiles, ksplit K slices, ceil(T/8)
// token groups).  Each CTA computes a 16-expert x 8-token tile of partial
// logits over its K slice with mma.sync m16n8k16 bf16 (the router weights
// are bf16 already: no dequantisation) and writes it to the workspace.  The
// last CTA of a token group (one atomic ticket per group; the counter is
// reset by that CTA) sums the slices in a fixed order and selects the top-k,
// so the result is deterministic.
#include "common.cuh"
#include "kernels.h"

namespace nvfp4 {
namespace {

constexpr int kRouterWarps = 4;
constexpr int kRouterPad = 32;  // bf16 elements of padding per staged column

__global__ void __launch_bounds__(kRouterWarps * 32) router_kernel(RouterArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int Kc = (int)(a.H / a.ksplit);
  const int ldx = Kc + kRouterPad;
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem);
  __shared__ bool is_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t e0 = (int64_t)blockIdx.x * 16;
  const int ks = blockIdx.y;
  const int64_t tg = blockIdx.z;
  const int64_t t0 = tg * 8;
  const int ntok = (int)(a.T - t0 < 8 ? a.T - t0 : 8);
  const int64_t k0 = (int64_t)ks * Kc;

  // x is the preceding kernel's output (programmatic dependent launch).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // Stage x[t0 .. t0+ntok) [k0, k0+Kc) as bf16 (exact for bf16 inputs).
  for (int idx = threadIdx.x; idx < 8 * Kc; idx += blockDim.x) {
    const int c = idx / Kc, k = idx % Kc;
    float v = 0.f;
    if (c < ntok) v = load_as_f32(a.x, a.dtype, (t0 + c) * a.H + k0 + k);
    xs[c * ldx + k] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
  }
  __syncthreads();

  // Each warp covers Kc / kRouterWarps of the slice in chunks of 32.
  const int kw = Kc / kRouterWarps;
  const int kb = warp * kw;
  const int64_t r_lo = e0 + g, r_hi = e0 + g + 8;
  const uint16_t* glo = a.G + r_lo * a.H + k0;
  const uint16_t* ghi = a.G + r_hi * a.H + k0;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int c = kb; c < kb + kw; c += 32) {
    const uint4 wl = r_lo < a.E ? *reinterpret_cast<const uint4*>(glo + c + 8 * t)
                                : make_uint4(0, 0, 0, 0);
    const uint4 wh = r_hi < a.E ? *reinterpret_cast<const uint4*>(ghi + c + 8 * t)
                                : make_uint4(0, 0, 0, 0);
    const uint4 xv = *reinterpret_cast<const uint4*>(xs + g * ldx + c + 8 * t);
    mma_bf16_16816(acc, wl.x, wh.x, wl.y, wh.y, xv.x, xv.y);
    mma_bf16_16816(acc, wl.z, wh.z, wl.w, wh.w, xv.z, xv.w);
  }
  // Cross-warp reduction (fixed order) into warp 0, then store partials.
  __shared__ float red[kRouterWarps - 1][4][32];
  if (warp > 0)
    for (int r = 0; r < 4; r++) red[warp - 1][r][lane] = acc[r];
  __syncthreads();
  if (warp == 0) {
    for (int w = 1; w < kRouterWarps; w++)
      for (int r = 0; r < 4; r++) acc[r] += red[w - 1][r][lane];
    float* part = a.partial + ((tg * a.ksplit + ks) * 8) * a.E;
    for (int r = 0; r < 4; r++) {
      const int col = 2 * t + (r & 1);
      const int64_t e = (r < 2) ? r_lo : r_hi;
      if (e < a.E) part[(int64_t)col * a.E + e] = acc[r];
    }
  }
  // Ticket: the last CTA of this token group finishes the routing.
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned total = gridDim.x * gridDim.y;
    const unsigned prev = atomicAdd(&a.counters[tg], 1u);
    is_last = (prev == total - 1);
    if (is_last) a.counters[tg] = 0u;  // self-reset for the next call
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();

  // One warp per token: sum slices, sigmoid, top-k.
  const float* part0 = a.partial + (tg * a.ksplit * 8) * a.E;
  for (int c = warp; c < ntok; c += kRouterWarps) {
    const int64_t tok = t0 + c;
    // Each lane owns experts lane, lane+32, ... (E <= 32 * 16).
    float sc[16], ch[16];
    const int per = (int)((a.E + 31) / 32);
    for (int j = 0; j < 16; j++) {
      sc[j] = 0.f;
      ch[j] = -INFINITY;
    }
    for (int j = 0; j < per && j < 16; j++) {
      const int64_t e = lane + 32 * j;
      if (e >= a.E) break;
      float l = 0.f;
      for (int s = 0; s < a.ksplit; s++) l += __ldcg(part0 + ((int64_t)s * 8 + c) * a.E + e);
      if (a.dtype == kBF16) l = __bfloat162float(__float2bfloat16_rn(l));
      else if (a.dtype == kF16) l = __half2float(__float2half_rn(l));
      const float s = sigmoid_ref(l);
      sc[j] = s;
      ch[j] = s + (a.bias ? a.bias[e] : 0.f);
    }
    float wsum = 0.f;
    float wsel = 0.f;
    uint32_t isel = 0;
    for (int r = 0; r < a.k; r++) {
      // Lane-local best (highest choice, then lowest id).
      float bv = -INFINITY;
      int bj = -1;
      for (int j = 0; j < per && j < 16; j++) {
        if (lane + 32 * j >= a.E) break;
        if (ch[j] > bv) {
          bv = ch[j];
          bj = j;
        }
      }
      int bid = bj >= 0 ? lane + 32 * bj : 0x7fffffff;
      float bs = bj >= 0 ? sc[bj] : 0.f;
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oid = __shfl_xor_sync(0xffffffffu, bid, o);
        const float os = __shfl_xor_sync(0xffffffffu, bs, o);
        if (ov > bv || (ov == bv && oid < bid)) {
          bv = ov;
          bid = oid;
          bs = os;
        }
      }
      if (bid != 0x7fffffff && (bid & 31) == lane) ch[bid >> 5] = -INFINITY;
      wsum += bs;
      if (lane == r) {
        wsel = bs;
        isel = (uint32_t)bid;
      }
    }
    if (lane < a.k) {
      a.inds[tok * a.k + lane] = isel;
      a.wts[tok * a.k + lane] = a.norm ? wsel / wsum : wsel;
    }
  }
}

}  // namespace

int router_ksplit(int64_t H) {
  // K slices of at least 128 elements, each a multiple of 32 * warps.
  for (int ks : {8, 4, 2, 1})
    if (H % (ks * 32 * kRouterWarps) == 0 && H / ks >= 128) return ks;
  return (H % (32 * kRouterWarps) == 0) ? 1 : 0;
}

cudaError_t launch_router(const RouterArgs& a, cudaStream_t stream, bool pdl) {
  if (a.T == 0) return cudaSuccess;
  const int Kc = (int)(a.H / a.ksplit);
  const size_t smem = (size_t)8 * (Kc + kRouterPad) * sizeof(uint16_t);
  cudaError_t err = ensure_smem(router_kernel, smem);
  if (err != cudaSuccess) return err;
  dim3 grid((unsigned)((a.E + 15) / 16), (unsigned)a.ksplit, (unsigned)((a.T + 7) / 8));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kRouterWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = pdl ? 1 : 0;
  err = cudaLaunchKernelEx(&cfg, router_kernel, a);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

}  // namespace nvfp4
