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
// Decode (T <= 8) launch: grid (E/16 expert tiles, ksplit K slices, ceil(T/8)
// token groups).  Each CTA computes a 16-expert x 8-token tile of partial
// logits over its K slice with mma.sync m16n8k16 bf16 (the router weights
// are bf16 already: no dequantisation) and writes it to the workspace.  The
// last CTA of a token group (one atomic ticket per group; the counter is
// reset by that CTA) sums the slices in a fixed order and selects the top-k,
// so the result is deterministic.
#include "common.cuh"
#include "kernels.h"
#include "topk.cuh"

namespace nvfp4 {
namespace {

constexpr int kRouterWarps = 4;
constexpr int kRouterPad = 32;  // bf16 elements of padding per staged column

// Route one token (called by a whole warp): logit(e) = sum over `slices`
// of lg[s * stride + e], rounded to the activation dtype as the reference's
// matmul returns it, then the selection of topk.cuh (sort and merge for
// k <= 16, rounds of warp maxima beyond).  Lane owns experts
// lane + 32 j, j < kPer (E <= 32 kPer), fully unrolled so the per-lane arrays
// stay in registers.
template <int kPer>
__device__ void route_token_t(const RouterArgs& a, int64_t tok, const float* lg, int64_t stride,
                              int slices, int lane) {
  float lgt[kPer];
#pragma unroll
  for (int j = 0; j < kPer; j++) {
    const int64_t e = lane + 32 * j;
    const bool live = e < a.E;
    float l = live ? __ldcg(lg + e) : 0.f;
    for (int s = 1; s < slices; s++)
      if (live) l += __ldcg(lg + (int64_t)s * stride + e);
    lgt[j] = round_to_dtype(l, a.dtype);
  }
  uint32_t isel;
  float wsel;
  if (a.k <= 16) {
    float sc[kPer], bs[kPer];
#pragma unroll
    for (int j = 0; j < kPer; j++) {
      const int64_t e = lane + 32 * j;
      sc[j] = sigmoid_ref(lgt[j]);
      bs[j] = (a.bias && e < a.E) ? a.bias[e] : 0.f;
    }
    if (a.k <= 8) topk_merge<kPer, 8>(sc, bs, (int)a.E, a.k, a.norm != 0, lane, isel, wsel);
    else topk_merge<kPer, 16>(sc, bs, (int)a.E, a.k, a.norm != 0, lane, isel, wsel);
  } else {
    topk_select<kPer>(lgt, a.bias, (int)a.E, a.k, a.norm != 0, lane, isel, wsel);
  }
  if (lane < a.k) {
    a.inds[tok * a.k + lane] = isel;
    a.wts[tok * a.k + lane] = wsel;
  }
}

__device__ void route_token(const RouterArgs& a, int64_t tok, const float* lg, int64_t stride,
                            int slices, int lane) {
  if (a.E <= 256) route_token_t<8>(a, tok, lg, stride, slices, lane);
  else route_token_t<16>(a, tok, lg, stride, slices, lane);
}

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
  for (int c = warp; c < ntok; c += kRouterWarps)
    route_token(a, t0 + c, part0 + (int64_t)c * a.E, 8 * a.E, a.ksplit, lane);
}

// Prefill logits: grid (ceil(E/32), ceil(T/32)); warp w covers experts
// 16*(w&1).. and tokens 16*(w>>1).. of the CTA's 32 x 32 tile with mma.sync
// m16n8k16 bf16 (A = router rows, B = token rows), fragments loaded straight
// from global memory (each 32-wide K chunk uses the same element permutation
// in A and B, so the dot products are unchanged).  logits[T, E] f32.
__global__ void __launch_bounds__(128) router_logits_kernel(RouterArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t e0 = (int64_t)blockIdx.x * 32 + (warp & 1) * 16;
  const int64_t tk0 = (int64_t)blockIdx.y * 32 + (warp >> 1) * 16;
  const int64_t r_lo = e0 + g, r_hi = e0 + g + 8;
  const bool ok_lo = r_lo < a.E, ok_hi = r_hi < a.E;
  const uint16_t* glo = a.G + (ok_lo ? r_lo : 0) * a.H;
  const uint16_t* ghi = a.G + (ok_hi ? r_hi : 0) * a.H;
  int64_t tok[2];
  bool tok_ok[2];
#pragma unroll
  for (int j = 0; j < 2; j++) {
    tok[j] = tk0 + 8 * j + g;
    tok_ok[j] = tok[j] < a.T;
  }
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll 4
  for (int64_t c = 0; c < a.H; c += 32) {
    const uint4 wl = ok_lo ? *reinterpret_cast<const uint4*>(glo + c + 8 * t) : make_uint4(0, 0, 0, 0);
    const uint4 wh = ok_hi ? *reinterpret_cast<const uint4*>(ghi + c + 8 * t) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int j = 0; j < 2; j++) {
      uint4 xv = make_uint4(0, 0, 0, 0);
      if (tok_ok[j]) {
        const int64_t off = tok[j] * a.H + c + 8 * t;
        if (a.dtype == kBF16) {
          xv = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(a.x) + off);
        } else {
          float f[8];
          load8(a.x, a.dtype, off, f);
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t*>(&b);
          }
          xv = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      mma_bf16_16816(acc[j], wl.x, wh.x, wl.y, wh.y, xv.x, xv.y);
      mma_bf16_16816(acc[j], wl.z, wh.z, wl.w, wh.w, xv.z, xv.w);
    }
  }
#pragma unroll
  for (int j = 0; j < 2; j++)
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int64_t tk = tk0 + 8 * j + 2 * t + (r & 1);
      const int64_t e = (r < 2) ? r_lo : r_hi;
      if (tk < a.T && e < a.E) a.partial[tk * a.E + e] = acc[j][r];
    }
}

// Prefill logits for bf16 x: grid (ceil(E/32), ceil(T/32)), 128 threads.  The
// CTA's 32 router rows and 32 token rows stream through shared memory in
// 64-wide K chunks (cp.async, kLgStages deep; rows padded to 192 bytes so the
// 16-byte fragment reads are conflict-free); warp w computes experts
// 16*(w&1).. x tokens 16*(w>>1).. with mma.sync m16n8k16 bf16 (same K
// permutation in A and B as above).
constexpr int kLgStages = 6;
constexpr int kLgPitch = 192;                   // bytes per staged row (128 + pad)
constexpr int kLgTile = 32 * kLgPitch;          // one 32-row operand tile
__device__ __forceinline__ void cp_async16_lg(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__global__ void __launch_bounds__(128) router_logits_smem_kernel(RouterArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t eb = (int64_t)blockIdx.x * 32, tb = (int64_t)blockIdx.y * 32;
  const int nk = (int)(a.H / 64);
  const uint16_t* x = reinterpret_cast<const uint16_t*>(a.x);
  auto load_stage = [&](int st, int kc) {
    uint8_t* sg = smem + st * 2 * kLgTile;
    uint8_t* sx = sg + kLgTile;
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const int q = threadIdx.x + 128 * i;  // 256 chunks of 16 bytes per tile
      const int row = q >> 3, c = q & 7;
      const int64_t e = eb + row, tk = tb + row;
      cp_async16_lg(sg + row * kLgPitch + c * 16,
                    a.G + (e < a.E ? e : 0) * a.H + (int64_t)kc * 64 + c * 8, e < a.E);
      cp_async16_lg(sx + row * kLgPitch + c * 16,
                    x + (tk < a.T ? tk : 0) * a.H + (int64_t)kc * 64 + c * 8, tk < a.T);
    }
  };
#pragma unroll
  for (int s = 0; s < kLgStages - 1; s++) {
    if (s < nk) load_stage(s, s);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  const int erow = (warp & 1) * 16, trow = (warp >> 1) * 16;
  for (int kc = 0; kc < nk; kc++) {
    asm volatile("cp.async.wait_group %0;" ::"n"(kLgStages - 2) : "memory");
    __syncthreads();
    if (kc + kLgStages - 1 < nk) load_stage((kc + kLgStages - 1) % kLgStages, kc + kLgStages - 1);
    asm volatile("cp.async.commit_group;" ::: "memory");
    const uint8_t* sg = smem + (kc % kLgStages) * 2 * kLgTile;
    const uint8_t* sx = sg + kLgTile;
#pragma unroll
    for (int sub = 0; sub < 2; sub++) {  // two 32-wide K pieces of the chunk
      const int cb = sub * 64 + t * 16;
      const uint4 wl = *reinterpret_cast<const uint4*>(sg + (erow + g) * kLgPitch + cb);
      const uint4 wh = *reinterpret_cast<const uint4*>(sg + (erow + g + 8) * kLgPitch + cb);
#pragma unroll
      for (int j = 0; j < 2; j++) {
        const uint4 xv = *reinterpret_cast<const uint4*>(sx + (trow + 8 * j + g) * kLgPitch + cb);
        mma_bf16_16816(acc[j], wl.x, wh.x, wl.y, wh.y, xv.x, xv.y);
        mma_bf16_16816(acc[j], wl.z, wh.z, wl.w, wh.w, xv.z, xv.w);
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
#pragma unroll
  for (int j = 0; j < 2; j++)
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int64_t tk = tb + trow + 8 * j + 2 * t + (r & 1);
      const int64_t e = eb + erow + g + ((r < 2) ? 0 : 8);
      if (tk < a.T && e < a.E) a.partial[tk * a.E + e] = acc[j][r];
    }
}

// Prefill routing: one warp per token over logits[T, E].
__global__ void __launch_bounds__(256) router_topk_kernel(RouterArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const int64_t tok = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (tok < a.T) route_token(a, tok, a.partial + tok * a.E, 0, 1, lane);
}

}  // namespace

int router_ksplit(int64_t H) {
  // K slices of at least 128 elements, each a multiple of 32 * warps.
  for (int ks : {8, 4, 2, 1})
    if (H % (ks * 32 * kRouterWarps) == 0 && H / ks >= 128) return ks;
  return (H % (32 * kRouterWarps) == 0) ? 1 : 0;
}

template <typename Kern>
cudaError_t launch_plain(Kern kern, dim3 grid, dim3 block, cudaStream_t stream, bool pdl,
                         const RouterArgs& a) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t err = cudaLaunchKernelEx(&cfg, kern, a);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

// T > 8: logits GEMM then one warp per token (the partial workspace, sized
// ceil(T/8) * 8 * ksplit * E floats, holds the [T, E] logits).  T <= 8: the
// split-K single-launch kernel.
cudaError_t launch_router(const RouterArgs& a, cudaStream_t stream, bool pdl) {
  if (a.T == 0) return cudaSuccess;
  if (a.T > 8) {
    const dim3 grid((unsigned)((a.E + 31) / 32), (unsigned)((a.T + 31) / 32));
    cudaError_t err;
    const bool staged = a.dtype == kBF16 && a.H % 64 == 0 &&
                        (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 &&
                        (reinterpret_cast<uintptr_t>(a.G) & 15) == 0;
    if (staged) {
      const size_t smem = (size_t)kLgStages * 2 * kLgTile;
      err = ensure_smem(router_logits_smem_kernel, smem);
      if (err != cudaSuccess) return err;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = grid;
      cfg.blockDim = dim3(128);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = stream;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr.val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = pdl ? 1 : 0;
      err = cudaLaunchKernelEx(&cfg, router_logits_smem_kernel, a);
      if (err == cudaSuccess) err = cudaGetLastError();
    } else {
      err = launch_plain(router_logits_kernel, grid, dim3(128), stream, pdl, a);
    }
    if (err != cudaSuccess) return err;
    return launch_plain(router_topk_kernel, dim3((unsigned)((a.T + 7) / 8)), dim3(256), stream,
                        true, a);
  }
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
