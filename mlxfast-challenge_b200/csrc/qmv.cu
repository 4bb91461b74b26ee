// qmv.cu -- decode-shaped NVFP4 matmuls on sm_100a: at most 8 activation rows
// meet each weight matrix, so the work is bound by streaming the packed
// weights from HBM.
//
// Engine (shared by every kernel in this file): a warp owns a tile of 16
// weight rows and up to 8 activation columns and walks K in chunks of 128
// codes.  Per chunk each thread issues one 128-bit streaming load per row
// (rows g and g+8, g = lane/4, t = lane%4) and one 16-bit scale load per row,
// converts E2M1 pairs to f16x2 with the hardware converter, folds the group
// scale in with one HMUL2 (exact: see common.cuh) and feeds mma.sync
// m16n8k16 (f16 x f16 -> f32).  K inside a chunk is permuted: thread t's
// 32 codes are actual K [32t, 32t+32) and MMA i takes its codes 4i..4i+3;
// the activation tile in shared memory is laid out with the same permutation
// (plus an XOR swizzle that keeps the 128-bit B loads bank-conflict free).
// Activations enter as f16 scaled by a per-column power of two (max |x| is
// mapped into [1,2)), so no input range can overflow f16; the power is
// re-applied to the f32 result.  Loads run 4 chunks ahead of the MMAs.
//
// Reference semantics followed: fp_qmm_t (backend/cpu/quantized.cpp:491-533)
// for every product, fp_bs_qmm_dispatch_mode (:805-844) for the gather, the
// SwitchGLU gate/up -> silu(gate)*up -> down chain
// (VLM/MLXLMCommon/SwitchLayers.swift:532-580) and the Laguna sparse block
// combine  y = scaling * sum_j w_j * expert_j(x) + shared(x)
// (VLM/MLXLLM/Models/Laguna.swift:204-212).
#include "common.cuh"
#include "kernels.h"

namespace nvfp4 {

namespace {

constexpr int kChunk = 128;       // codes per row per chunk
constexpr int kChunkBytes = 64;   // packed bytes per row per chunk
constexpr int kChunkScales = 8;   // scale bytes per row per chunk
constexpr int kXPad = 32;         // f16 padding per column: 64 B bank offset
constexpr int kRing = 4;          // chunks in flight per warp

__device__ int g_device_error = 0;

__device__ __forceinline__ void flag_error(int code) { atomicCAS(&g_device_error, 0, code); }

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

__device__ __forceinline__ void load_chunk(Chunk& c, const uint8_t* clo, const uint8_t* chi,
                                           const uint8_t* slo, const uint8_t* shi, int ch,
                                           int t) {
  if (clo) {
    c.lo = ldg_stream_u4(clo + ch * kChunkBytes + 16 * t);
    c.slo = ldg_stream_u16(slo + ch * kChunkScales + 2 * t);
  } else {
    c.lo = make_uint4(0, 0, 0, 0);
    c.slo = 0;
  }
  if (chi) {
    c.hi = ldg_stream_u4(chi + ch * kChunkBytes + 16 * t);
    c.shi = ldg_stream_u16(shi + ch * kChunkScales + 2 * t);
  } else {
    c.hi = make_uint4(0, 0, 0, 0);
    c.shi = 0;
  }
}

__device__ __forceinline__ void compute_chunk(float (&acc)[4], const Chunk& c,
                                              const __half* xcol, int ch, int t) {
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
    mma_f16_16816(acc, hmul2_u32(hl[0], s_l), hmul2_u32(hh[0], s_h), hmul2_u32(hl[1], s_l),
                  hmul2_u32(hh[1], s_h), xb[4 * j], xb[4 * j + 1]);
    mma_f16_16816(acc, hmul2_u32(hl[2], s_l), hmul2_u32(hh[2], s_h), hmul2_u32(hl[3], s_l),
                  hmul2_u32(hh[3], s_h), xb[4 * j + 2], xb[4 * j + 3]);
  }
}

// Stage one activation column: f16(v * 2^-e) at swizzled positions, zeros in
// [K, Kpad).  Executed by one warp; returns 2^e (all lanes).
template <typename Loader>
__device__ float stage_column_warp(__half* col, int K, int Kpad, Loader ld) {
  const int lane = threadIdx.x & 31;
  float m = 0.0f;
  for (int k = lane; k < K; k += 32) m = fmaxf(m, fabsf(ld(k)));
  m = warp_max(m);
  const int e = pow2_exponent(m);
  const float inv = ldexpf(1.0f, -e);
  for (int k = lane; k < Kpad; k += 32)
    col[xs_swz(k)] = __float2half_rn(k < K ? ld(k) * inv : 0.0f);
  return ldexpf(1.0f, e);
}

// Deterministic cross-warp reduction of the MMA fragments into warp 0.
template <int WARPS>
__device__ __forceinline__ void reduce_to_warp0(float (&acc)[4], float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (WARPS > 1) {
    if (warp > 0) {
#pragma unroll
      for (int r = 0; r < 4; r++) red[((warp - 1) * 4 + r) * 32 + lane] = acc[r];
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll 1
      for (int w = 1; w < WARPS; w++)
#pragma unroll
        for (int r = 0; r < 4; r++) acc[r] += red[((w - 1) * 4 + r) * 32 + lane];
    }
  }
}

// ---------------------------------------------------------------------------
// Gather QMM (also the dense quantized_matmul with one expert and no index).
// grid = (P * mchunks, ceil(N/16)); segment = (pair p, 8-row chunk of M).
template <int WARPS>
__global__ void __launch_bounds__(WARPS * 32) qmm_gather_kernel(QmmArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int Kpad = (int)a.K;  // fast path: K % 128 == 0
  const int ldx = Kpad + kXPad;
  __half* xs = reinterpret_cast<__half*>(smem);
  float* colscale = reinterpret_cast<float*>(xs + 8 * ldx);
  float* red = colscale + 8;

  const int seg = blockIdx.x;
  const int p = seg / a.mchunks, mc = seg % a.mchunks;
  const uint32_t e = a.rhs ? a.rhs[p] : 0u;
  const uint32_t xi = a.lhs ? a.lhs[p] : (uint32_t)p;
  if (e >= (uint32_t)a.n_experts || xi >= (uint32_t)a.n_x_batches) {
    if (threadIdx.x == 0 && blockIdx.y == 0) flag_error(1);
    return;
  }
  const int ncols = min(8, a.M - mc * 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  for (int j = warp; j < ncols; j += WARPS) {
    const int64_t row = ((int64_t)xi * a.M + mc * 8 + j) * a.K;
    const float s = stage_column_warp(xs + j * ldx, (int)a.K, Kpad,
                                      [&](int k) { return load_as_f32(a.x, a.dtype, row + k); });
    if (lane == 0) colscale[j] = s;
  }
  __syncthreads();

  const int64_t n_lo = (int64_t)blockIdx.y * 16 + g, n_hi = n_lo + 8;
  const uint8_t* wbase = a.w + (int64_t)e * a.w_stride;
  const uint8_t* sbase = a.s + (int64_t)e * a.s_stride;
  const int64_t rowb = a.K / 2, rows = a.K / 16;
  const uint8_t* clo = n_lo < a.N ? wbase + n_lo * rowb : nullptr;
  const uint8_t* chi = n_hi < a.N ? wbase + n_hi * rowb : nullptr;
  const uint8_t* slo = sbase + n_lo * rows;
  const uint8_t* shi = sbase + n_hi * rows;
  const __half* xcol = g < ncols ? xs + g * ldx : nullptr;

  const int nch = Kpad / kChunk;
  const int c0 = (warp * nch) / WARPS, c1 = ((warp + 1) * nch) / WARPS;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  Chunk ring[kRing];
#pragma unroll
  for (int u = 0; u < kRing; u++)
    if (c0 + u < c1) load_chunk(ring[u], clo, chi, slo, shi, c0 + u, t);
  for (int base = c0; base < c1; base += kRing) {
#pragma unroll
    for (int u = 0; u < kRing; u++) {
      const int ch = base + u;
      if (ch < c1) {
        compute_chunk(acc, ring[u], xcol, ch, t);
        if (ch + kRing < c1) load_chunk(ring[u], clo, chi, slo, shi, ch + kRing, t);
      }
    }
  }
  reduce_to_warp0<WARPS>(acc, red);
  if (warp == 0) {
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int col = 2 * t + (r & 1);
      const int64_t n = (r < 2) ? n_lo : n_hi;
      if (col < ncols && n < a.N) {
        const int64_t orow = (int64_t)p * a.M + mc * 8 + col;
        store_from_f32(a.out, a.dtype, orow * a.N + n, acc[r] * colscale[col]);
      }
    }
  }
}

// Generic (slow) path for shapes the tiled engine does not cover (K not a
// multiple of 128, misaligned pointers): one thread per output element, f32
// accumulation in the reference's group order.
__global__ void qmm_gather_generic_kernel(QmmArgs a) {
  const int64_t total = a.P * (int64_t)a.M * a.N;
  const int64_t rowb = a.K / 2, rows = a.K / 16;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = idx % a.N;
    const int64_t m = (idx / a.N) % a.M;
    const int64_t p = idx / ((int64_t)a.N * a.M);
    const uint32_t e = a.rhs ? a.rhs[p] : 0u;
    const uint32_t xi = a.lhs ? a.lhs[p] : (uint32_t)p;
    if (e >= (uint32_t)a.n_experts || xi >= (uint32_t)a.n_x_batches) {
      flag_error(1);
      continue;
    }
    const uint8_t* wr = a.w + (int64_t)e * a.w_stride + n * rowb;
    const uint8_t* sr = a.s + (int64_t)e * a.s_stride + n * rows;
    const int64_t xrow = ((int64_t)xi * a.M + m) * a.K;
    float sum = 0.f;
    for (int64_t gidx = 0; gidx < a.K / 16; gidx++) {
      const float scale = scale_to_f32(sr[gidx]);
      float gs = 0.f;
      for (int j = 0; j < 16; j++) {
        const int64_t k = gidx * 16 + j;
        const int code = (wr[k / 2] >> (4 * (k & 1))) & 15;
        const float lut = fp4_to_f32(code);
        gs += load_as_f32(a.x, a.dtype, xrow + k) * lut;
      }
      sum += scale * gs;
    }
    store_from_f32(a.out, a.dtype, (p * a.M + m) * a.N + n, sum);
  }
}

// ---------------------------------------------------------------------------
// Routed (and shared) expert gate/up projections fused with SwiGLU.
// grid = (T * kk, ceil(Imax/8)), kk = k (+1 with a shared expert).  A warp
// tile holds gate rows i0..i0+7 in MMA rows 0..7 and the matching up rows in
// MMA rows 8..15, so every thread ends with (gate, up) of one row.
template <int WARPS>
__global__ void __launch_bounds__(WARPS * 32) moe_gateup_kernel(GateUpArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int Kpad = (int)a.H;
  const int ldx = Kpad + kXPad;
  __half* xs = reinterpret_cast<__half*>(smem);
  float* colscale = reinterpret_cast<float*>(xs + ldx);
  float* red = colscale + 4;

  const int seg = blockIdx.x;
  const int tok = seg / a.kk, slot = seg % a.kk;
  const bool routed = slot < a.k;
  const int64_t Irows = routed ? a.I : a.Is;
  const int64_t i0 = (int64_t)blockIdx.y * 8;
  if (i0 >= Irows) return;
  const uint8_t *gw, *gs, *uw, *us;
  if (routed) {
    const uint32_t e = a.inds[(int64_t)tok * a.k + slot];
    if (e >= (uint32_t)a.E) {
      if (threadIdx.x == 0) flag_error(2);
      return;
    }
    gw = a.gw + (int64_t)e * a.w_stride;
    gs = a.gs + (int64_t)e * a.s_stride;
    uw = a.uw + (int64_t)e * a.w_stride;
    us = a.us + (int64_t)e * a.s_stride;
  } else {
    gw = a.sgw;
    gs = a.sgs;
    uw = a.suw;
    us = a.sus;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  if (warp == 0) {
    const int64_t row = (int64_t)tok * a.H;
    const float s = stage_column_warp(xs, (int)a.H, Kpad,
                                      [&](int k) { return load_as_f32(a.x, a.dtype, row + k); });
    if (lane == 0) colscale[0] = s;
  }
  __syncthreads();

  const int64_t i = i0 + g;
  const int64_t rowb = a.H / 2, rows = a.H / 16;
  const uint8_t* clo = i < Irows ? gw + i * rowb : nullptr;
  const uint8_t* chi = i < Irows ? uw + i * rowb : nullptr;
  const uint8_t* slo = gs + i * rows;
  const uint8_t* shi = us + i * rows;
  const __half* xcol = g == 0 ? xs : nullptr;

  const int nch = Kpad / kChunk;
  const int c0 = (warp * nch) / WARPS, c1 = ((warp + 1) * nch) / WARPS;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  Chunk ring[kRing];
#pragma unroll
  for (int u = 0; u < kRing; u++)
    if (c0 + u < c1) load_chunk(ring[u], clo, chi, slo, shi, c0 + u, t);
  for (int base = c0; base < c1; base += kRing) {
#pragma unroll
    for (int u = 0; u < kRing; u++) {
      const int ch = base + u;
      if (ch < c1) {
        compute_chunk(acc, ring[u], xcol, ch, t);
        if (ch + kRing < c1) load_chunk(ring[u], clo, chi, slo, shi, ch + kRing, t);
      }
    }
  }
  reduce_to_warp0<WARPS>(acc, red);
  if (warp == 0 && t == 0 && i < Irows) {
    const float cs = colscale[0];
    const float gate = acc[0] * cs, up = acc[2] * cs;
    a.act[(int64_t)seg * a.act_ld + i] = silu_ref(gate) * up;
  }
}

// ---------------------------------------------------------------------------
// Down projections of every (token, slot) segment plus the shared expert,
// weighted, summed, scaled and added to the residual in one pass.
// grid = (ceil(H/16), ceil(T/8)).  Each segment is one K-range of the
// accumulation; its activation is pre-multiplied by w_j * scaling (1 for the
// shared expert) and only the owning token's MMA column is non-zero.
template <int WARPS>
__global__ void __launch_bounds__(WARPS * 32) moe_down_kernel(DownArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int Ipad = a.Ipad;
  const int ldx = Ipad + kXPad;
  const int t0 = blockIdx.y * 8;
  const int ntok = (int)(a.T - t0 < 8 ? a.T - t0 : 8);
  const int nseg = ntok * a.kk;
  __half* xs = reinterpret_cast<__half*>(smem);
  float* colscale = reinterpret_cast<float*>(xs + (size_t)nseg * ldx);
  float* red = colscale + 8;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  // Per token: power-of-two prescale over all of its weighted segments.
  for (int tl = warp; tl < ntok; tl += WARPS) {
    const int tok = t0 + tl;
    float m = 0.f;
    for (int sl = 0; sl < a.kk; sl++) {
      const bool routed = sl < a.k;
      const int64_t Iseg = routed ? a.I : a.Is;
      const float wgt = routed ? a.wts[(int64_t)tok * a.k + sl] * a.scaling : 1.0f;
      const float* src = a.act + ((int64_t)tok * a.kk + sl) * a.act_ld;
      for (int k = lane; k < Iseg; k += 32) m = fmaxf(m, fabsf(src[k] * wgt));
    }
    m = warp_max(m);
    const int e = pow2_exponent(m);
    const float inv = ldexpf(1.0f, -e);
    for (int sl = 0; sl < a.kk; sl++) {
      const bool routed = sl < a.k;
      const int64_t Iseg = routed ? a.I : a.Is;
      const float wgt = (routed ? a.wts[(int64_t)tok * a.k + sl] * a.scaling : 1.0f) * inv;
      const float* src = a.act + ((int64_t)tok * a.kk + sl) * a.act_ld;
      __half* col = xs + (size_t)(tl * a.kk + sl) * ldx;
      for (int k = lane; k < Ipad; k += 32)
        col[xs_swz(k)] = __float2half_rn(k < Iseg ? src[k] * wgt : 0.0f);
    }
    if (lane == 0) colscale[tl] = ldexpf(1.0f, e);
  }
  __syncthreads();

  const int64_t h_lo = (int64_t)blockIdx.x * 16 + g, h_hi = h_lo + 8;
  const int nch = Ipad / kChunk;
  const int nunits = nseg * nch;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};

  // Unit u -> (segment, chunk); row pointers resolved per unit.
  auto unit_ptrs = [&](int u, const uint8_t*& clo, const uint8_t*& chi, const uint8_t*& slo,
                       const uint8_t*& shi, int& ch, const __half*& xcol) {
    const int s = u / nch;
    ch = u % nch;
    const int tl = s / a.kk, sl = s % a.kk;
    const bool routed = sl < a.k;
    const int64_t Iseg = routed ? a.I : a.Is;
    const uint8_t* wb;
    const uint8_t* sb;
    if (routed) {
      uint32_t e = a.inds[(int64_t)(t0 + tl) * a.k + sl];
      if (e >= (uint32_t)a.E) {
        flag_error(3);
        e = 0;
      }
      wb = a.dw + (int64_t)e * a.w_stride;
      sb = a.ds + (int64_t)e * a.s_stride;
    } else {
      wb = a.sdw;
      sb = a.sds;
    }
    const bool chunk_ok = (int64_t)(ch + 1) * kChunk <= Iseg;
    const int64_t rowb = Iseg / 2, rows = Iseg / 16;
    clo = (chunk_ok && h_lo < a.H) ? wb + h_lo * rowb : nullptr;
    chi = (chunk_ok && h_hi < a.H) ? wb + h_hi * rowb : nullptr;
    slo = sb + h_lo * rows;
    shi = sb + h_hi * rows;
    xcol = (g == tl) ? xs + (size_t)s * ldx : nullptr;
  };

  Chunk ring[kRing];
#pragma unroll
  for (int r = 0; r < kRing; r++) {
    const int u = warp + r * WARPS;
    if (u < nunits) {
      const uint8_t *clo, *chi, *slo, *shi;
      int ch;
      const __half* xcol;
      unit_ptrs(u, clo, chi, slo, shi, ch, xcol);
      load_chunk(ring[r], clo, chi, slo, shi, ch, t);
    }
  }
  for (int base = warp; base < nunits; base += kRing * WARPS) {
#pragma unroll
    for (int r = 0; r < kRing; r++) {
      const int u = base + r * WARPS;
      if (u < nunits) {
        const uint8_t *clo, *chi, *slo, *shi;
        int ch;
        const __half* xcol;
        unit_ptrs(u, clo, chi, slo, shi, ch, xcol);
        compute_chunk(acc, ring[r], xcol, ch, t);
        const int un = u + kRing * WARPS;
        if (un < nunits) {
          unit_ptrs(un, clo, chi, slo, shi, ch, xcol);
          load_chunk(ring[r], clo, chi, slo, shi, ch, t);
        }
      }
    }
  }
  reduce_to_warp0<WARPS>(acc, red);
  if (warp == 0) {
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int col = 2 * t + (r & 1);
      const int64_t h = (r < 2) ? h_lo : h_hi;
      if (col < ntok && h < a.H) {
        const int64_t o = (int64_t)(t0 + col) * a.H + h;
        float v = acc[r] * colscale[col];
        if (a.residual) v += load_as_f32(a.residual, a.dtype, o);
        store_from_f32(a.y, a.dtype, o, v);
      }
    }
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// Host launchers.
constexpr int kQmmWarps = 4;
constexpr int kGateUpWarps = 4;
constexpr int kDownWarps = 8;

size_t qmm_smem_bytes(int64_t K) {
  return (size_t)8 * (K + kXPad) * sizeof(__half) + 8 * sizeof(float) +
         (size_t)(kQmmWarps - 1) * 4 * 32 * sizeof(float);
}

bool qmm_fast_path_ok(const QmmArgs& a) {
  return a.K % kChunk == 0 && qmm_smem_bytes(a.K) <= 200 * 1024 &&
         (reinterpret_cast<uintptr_t>(a.w) & 15) == 0 && (a.w_stride & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.s) & 1) == 0 && (a.s_stride & 1) == 0;
}

cudaError_t launch_qmm_gather(const QmmArgs& a, cudaStream_t stream) {
  if (a.P == 0 || a.M == 0 || a.N == 0) return cudaSuccess;
  if (qmm_fast_path_ok(a)) {
    const size_t smem = qmm_smem_bytes(a.K);
    auto kern = qmm_gather_kernel<kQmmWarps>;
    cudaError_t err = ensure_smem(kern, smem);
    if (err != cudaSuccess) return err;
    dim3 grid((unsigned)(a.P * a.mchunks), (unsigned)((a.N + 15) / 16));
    kern<<<grid, kQmmWarps * 32, smem, stream>>>(a);
  } else {
    const int64_t total = a.P * (int64_t)a.M * a.N;
    const int threads = 256;
    const int64_t blocks = std::min<int64_t>((total + threads - 1) / threads, 148 * 64);
    qmm_gather_generic_kernel<<<(unsigned)blocks, threads, 0, stream>>>(a);
  }
  return cudaGetLastError();
}

size_t gateup_smem_bytes(int64_t H) {
  return (size_t)(H + kXPad) * sizeof(__half) + 4 * sizeof(float) +
         (size_t)(kGateUpWarps - 1) * 4 * 32 * sizeof(float);
}

cudaError_t launch_moe_gateup(const GateUpArgs& a, cudaStream_t stream) {
  if (a.T == 0) return cudaSuccess;
  const size_t smem = gateup_smem_bytes(a.H);
  auto kern = moe_gateup_kernel<kGateUpWarps>;
  cudaError_t err = ensure_smem(kern, smem);
  if (err != cudaSuccess) return err;
  const int64_t Imax = std::max(a.I, a.Is);
  dim3 grid((unsigned)(a.T * a.kk), (unsigned)((Imax + 7) / 8));
  kern<<<grid, kGateUpWarps * 32, smem, stream>>>(a);
  return cudaGetLastError();
}

size_t down_smem_bytes(int64_t Ipad, int kk) {
  return (size_t)8 * kk * (Ipad + kXPad) * sizeof(__half) + 8 * sizeof(float) +
         (size_t)(kDownWarps - 1) * 4 * 32 * sizeof(float);
}

cudaError_t launch_moe_down(const DownArgs& a, cudaStream_t stream) {
  if (a.T == 0) return cudaSuccess;
  const size_t smem = down_smem_bytes(a.Ipad, a.kk);
  auto kern = moe_down_kernel<kDownWarps>;
  cudaError_t err = ensure_smem(kern, smem);
  if (err != cudaSuccess) return err;
  dim3 grid((unsigned)((a.H + 15) / 16), (unsigned)((a.T + 7) / 8));
  kern<<<grid, kDownWarps * 32, smem, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t read_and_clear_device_error(int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_device_error, sizeof(int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
}

}  // namespace nvfp4
