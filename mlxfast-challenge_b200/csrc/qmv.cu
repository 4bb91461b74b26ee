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
// m16n8k16 (f16 x f16 -> f32) into two independent accumulator sets.  K
// inside a chunk is permuted: thread t's 32 codes are actual K [32t, 32t+32)
// and MMA i takes its codes 4i..4i+3; the activation tile in shared memory is
// laid out with the same permutation (plus an XOR swizzle that keeps the
// 128-bit B loads bank-conflict free).  Activations enter as f16 scaled by a
// per-column power of two (max |x| is mapped into [1,2)), so no input range
// can overflow f16; the power is re-applied to the f32 result.
//
// Latency hiding: every kernel puts its weight loads in flight before it
// reads anything a preceding kernel produced, and supports programmatic
// dependent launch (PDL): it waits on the preceding grid (griddepcontrol.wait)
// only before touching that grid's outputs, and lets its own dependents
// launch right after that wait.  So in a stream / CUDA graph of these
// kernels the next kernel's weight streaming overlaps the current one.
//
// Reference semantics followed: fp_qmm_t (backend/cpu/quantized.cpp:491-533)
// for every product, fp_bs_qmm_dispatch_mode (:805-844) for the gather, the
// SwitchGLU gate/up -> silu(gate)*up -> down chain
// (VLM/MLXLMCommon/SwitchLayers.swift:532-580) and the Laguna sparse block
// combine  y = scaling * sum_j w_j * expert_j(x) + shared(x)
// (VLM/MLXLLM/Models/Laguna.swift:204-212).
#include <cooperative_groups.h>

#include "common.cuh"
#include "gemv.cuh"
#include "kernels.h"
#include "tma.cuh"

namespace cg = cooperative_groups;

namespace nvfp4 {

namespace {

constexpr int kRing = 4;          // chunks in flight per warp

__device__ int g_device_error = 0;

__device__ __forceinline__ void flag_error(int code) { atomicCAS(&g_device_error, 0, code); }

// PDL hooks (no-ops when the grid was launched without the PDL attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

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

// Block-cooperative staging of `ncols` activation columns (column j is the K
// elements at element offset off(j)), each as f16(v * 2^-e_j) with max |v| *
// 2^-e_j in [1, 2).  colscale[j] = 2^e_j.  Two passes over the (L1/L2-hot)
// activations: maxima via shared atomics, then the scaled f16 copy.  The
// items of one column are contiguous in `it`, so a warp's items belong to a
// short run of columns; the max is reduced per column of that run.
template <typename Off>
__device__ void stage_columns(__half* xs, int ldx, int ncols, int K, const void* x, int dtype,
                              Off off, float* colscale, int* colmax) {
  if (threadIdx.x < 8) colmax[threadIdx.x] = 0;
  __syncthreads();
  const int per = K / 8;
  const int items = ncols * per;
  const int rounds = (items + blockDim.x - 1) / blockDim.x;
  for (int r = 0; r < rounds; r++) {
    const int it = r * blockDim.x + threadIdx.x;
    const bool ok = it < items;
    const int j = ok ? it / per : 0;
    float m = 0.f;
    if (ok) {
      float f[8];
      load8(x, dtype, off(j) + (int64_t)(it - j * per) * 8, f);
#pragma unroll
      for (int i = 0; i < 8; i++) m = fmaxf(m, fabsf(f[i]));
    }
    const int j0 = __shfl_sync(0xffffffffu, j, 0);
    const int j1 = __shfl_sync(0xffffffffu, ok ? j : j0, 31);
    for (int jj = j0; jj <= j1; jj++) warp_atomic_max(&colmax[jj], m, ok && j == jj);
  }
  __syncthreads();
  if (threadIdx.x < ncols)
    colscale[threadIdx.x] = ldexpf(1.0f, pow2_exponent(__int_as_float(colmax[threadIdx.x])));
  __syncthreads();
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int j = it / per, v = it - j * per;
    float f[8];
    load8(x, dtype, off(j) + (int64_t)v * 8, f);
    store8_f16(xs + j * ldx, v * 8, f, 1.0f / colscale[j]);
  }
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

// Chunks [c0, c1) of one warp's tile: the first kRing loads were issued by
// the caller into `ring`; later ones are issued as slots free up.
__device__ __forceinline__ void run_chunks(Acc& acc, Chunk (&ring)[kRing], const uint8_t* clo,
                                           const uint8_t* chi, const uint8_t* slo,
                                           const uint8_t* shi, const __half* xcol, int c0,
                                           int c1, int t) {
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
}

// ---------------------------------------------------------------------------
// Gather QMM (also the dense quantized_matmul with one expert and no index).
// grid = (P * mchunks, ceil(N/16)); segment = (pair p, 8-row chunk of M).
template <int WARPS>
__global__ void __launch_bounds__(WARPS * 32) qmm_gather_kernel(QmmArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int Kpad = (int)a.K;  // fast path: K % 128 == 0
  const int ldx = Kpad + kXPad;
  __half* xs = reinterpret_cast<__half*>(smem);
  float* colscale = reinterpret_cast<float*>(xs + 8 * ldx);
  int* colmax = reinterpret_cast<int*>(colscale + 8);
  float* red = colscale + 16;

  // Indices may come from the preceding kernel: wait first.
  pdl_wait();
  pdl_trigger();
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
  Chunk ring[kRing];
#pragma unroll
  for (int u = 0; u < kRing; u++)
    if (c0 + u < c1) load_chunk(ring[u], clo, chi, slo, shi, c0 + u, t);

  const int64_t xrow0 = ((int64_t)xi * a.M + mc * 8) * a.K;
  stage_columns(xs, ldx, ncols, (int)a.K, a.x, a.dtype,
                [&](int j) { return xrow0 + (int64_t)j * a.K; }, colscale, colmax);
  __syncthreads();

  Acc acc;
  acc.zero();
  run_chunks(acc, ring, clo, chi, slo, shi, xcol, c0, c1, t);
  float d[4];
  acc.fold(d);
  reduce_to_warp0<WARPS>(d, red);
  if (warp == 0) {
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int col = 2 * t + (r & 1);
      const int64_t n = (r < 2) ? n_lo : n_hi;
      if (col < ncols && n < a.N) {
        const int64_t orow = (int64_t)p * a.M + mc * 8 + col;
        store_from_f32(a.out, a.dtype, orow * a.N + n, d[r] * colscale[col]);
      }
    }
  }
}

// Generic (slow) path for shapes the tiled engine does not cover (K not a
// multiple of 128, misaligned pointers): one thread per output element, f32
// accumulation in the reference's group order.
__global__ void qmm_gather_generic_kernel(QmmArgs a) {
  pdl_wait();
  pdl_trigger();
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
        gs += load_as_f32(a.x, a.dtype, xrow + k) * fp4_to_f32(code);
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
// MMA rows 8..15, so every thread ends with (gate, up) of one row.  The
// WARPS warps of a CTA split K.
template <int WARPS>
__global__ void __launch_bounds__(WARPS * 32) moe_gateup_kernel(GateUpArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int Kpad = (int)a.H;
  const int ldx = Kpad + kXPad;
  __half* xs = reinterpret_cast<__half*>(smem);
  float* colscale = reinterpret_cast<float*>(xs + ldx);
  int* colmax = reinterpret_cast<int*>(colscale + 8);
  float* red = colscale + 16;

  const int seg = blockIdx.x;
  const int tok = seg / a.kk, slot = seg % a.kk;
  const bool routed = slot < a.k;
  const int64_t Irows = routed ? a.I : a.Is;
  const int64_t i0 = (int64_t)blockIdx.y * 8;
  if (i0 >= Irows) {
    pdl_trigger();
    return;
  }
  // Routing produced by the preceding kernel is only read after the wait.
  if (routed && !a.inds_static) pdl_wait();
  const uint8_t *gw, *gs, *uw, *us;
  if (routed) {
    const uint32_t e = a.inds[(int64_t)tok * a.k + slot];
    if (e >= (uint32_t)a.E) {
      if (threadIdx.x == 0) flag_error(2);
      pdl_wait();
      pdl_trigger();
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
  const int64_t i = i0 + g;
  const int64_t rowb = a.H / 2, rows = a.H / 16;
  const uint8_t* clo = i < Irows ? gw + i * rowb : nullptr;
  const uint8_t* chi = i < Irows ? uw + i * rowb : nullptr;
  const uint8_t* slo = gs + i * rows;
  const uint8_t* shi = us + i * rows;
  const __half* xcol = g == 0 ? xs : nullptr;

  const int nch = Kpad / kChunk;
  const int c0 = (warp * nch) / WARPS, c1 = ((warp + 1) * nch) / WARPS;
  Chunk ring[kRing];
#pragma unroll
  for (int u = 0; u < kRing; u++)
    if (c0 + u < c1) load_chunk(ring[u], clo, chi, slo, shi, c0 + u, t);

  // x is the preceding kernel's output.
  pdl_wait();
  pdl_trigger();
  const int64_t xrow = (int64_t)tok * a.H;
  stage_columns(xs, ldx, 1, (int)a.H, a.x, a.dtype, [&](int) { return xrow; }, colscale, colmax);
  __syncthreads();

  Acc acc;
  acc.zero();
  run_chunks(acc, ring, clo, chi, slo, shi, xcol, c0, c1, t);
  float d[4];
  acc.fold(d);
  reduce_to_warp0<WARPS>(d, red);
  if (warp == 0 && t == 0 && i < Irows) {
    const float cs = colscale[0];
    const float gate = d[0] * cs, up = d[2] * cs;
    a.act[(int64_t)seg * a.act_ld + i] = silu_ref(gate) * up;
  }
}

// ---------------------------------------------------------------------------
// Down projections of every (token, slot) segment plus the shared expert,
// weighted, summed, scaled and added to the residual.
// grid = (ceil(H/16) * CL, ceil(T/8)) with thread-block clusters of CL CTAs
// along x: the CL CTAs of a cluster share one 16-row output tile and take
// every CL-th segment of its K range (segment = one expert's I-long down
// row for one token).  Each CTA stages only its own segments, pre-multiplied
// by w_j * scaling (1 for the shared expert) under one power-of-two prescale
// per token; only the owning token's MMA column is non-zero.  The CL partial
// tiles are summed in CTA rank 0 through distributed shared memory, in rank
// order (deterministic).
template <int WARPS, int CL>
__global__ void __launch_bounds__(WARPS * 32) moe_down_kernel(DownArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int Ipad = a.Ipad;
  const int ldx = Ipad + kXPad;
  const int t0 = blockIdx.y * 8;
  const int ntok = (int)(a.T - t0 < 8 ? a.T - t0 : 8);
  const int nseg_all = ntok * a.kk;
  const int nseg = nseg_all > rank ? (nseg_all - rank + CL - 1) / CL : 0;  // my segments
  __half* xs = reinterpret_cast<__half*>(smem);
  float* colscale = reinterpret_cast<float*>(xs + (size_t)a.max_seg_per_cta * ldx);
  int* colmax = reinterpret_cast<int*>(colscale + 8);
  float* segw = colscale + 16;                      // [max_seg_per_cta]
  float* red = segw + a.max_seg_per_cta;            // [(WARPS-1)*4*32]
  float* cred = red + (WARPS - 1) * 4 * 32;         // [(CL-1)*4*32], rank 0 only

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t h_lo = (int64_t)(blockIdx.x / CL) * 16 + g, h_hi = h_lo + 8;
  const int nch = Ipad / kChunk;
  const int nunits = nseg * nch;

  // Local segment ls -> global segment rank + ls*CL -> (token, slot).
  auto unit_ptrs = [&](int u, const uint8_t*& clo, const uint8_t*& chi, const uint8_t*& slo,
                       const uint8_t*& shi, int& ch, const __half*& xcol) {
    const int ls = u / nch;
    ch = u - ls * nch;
    const int s = rank + ls * CL;
    const int tl = s / a.kk, sl = s - tl * a.kk;
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
    xcol = (g == tl) ? xs + (size_t)ls * ldx : nullptr;
  };

  // The routing was written before the gate/up kernel this grid follows
  // started its own wait, so it is complete once this grid runs: the weights
  // go in flight before waiting for the gate/up output.
  if (!a.inds_static) pdl_wait();
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
  if (threadIdx.x < 8) colmax[threadIdx.x] = 0;
  for (int ls = threadIdx.x; ls < nseg; ls += blockDim.x) {
    const int s = rank + ls * CL;
    const int tl = s / a.kk, sl = s - tl * a.kk;
    segw[ls] = sl < a.k ? a.wts[(int64_t)(t0 + tl) * a.k + sl] * a.scaling : 1.0f;
  }
  pdl_wait();  // act is the preceding kernel's output
  pdl_trigger();
  __syncthreads();

  // Stage my segments: per-token max of |act * w| over my segments, then f16.
  const int per = Ipad / 8;
  const int items = nseg * per;
  const int rounds = (items + blockDim.x - 1) / blockDim.x;
  for (int r = 0; r < rounds; r++) {
    const int it = r * blockDim.x + threadIdx.x;
    const bool ok = it < items;
    int tl = 0;
    float m = 0.f;
    if (ok) {
      const int ls = it / per, v = it - ls * per;
      const int s = rank + ls * CL;
      tl = s / a.kk;
      const int sl = s - tl * a.kk;
      const int64_t Iseg = sl < a.k ? a.I : a.Is;
      if ((int64_t)v * 8 < Iseg) {
        float f[8];
        load8(a.act, kF32, ((int64_t)(t0 + tl) * a.kk + sl) * a.act_ld + (int64_t)v * 8, f);
#pragma unroll
        for (int i = 0; i < 8; i++) m = fmaxf(m, fabsf(f[i] * segw[ls]));
      }
    }
    const int j0 = __shfl_sync(0xffffffffu, tl, 0);
    const int j1 = __shfl_sync(0xffffffffu, ok ? tl : j0, 31);
    for (int jj = j0; jj <= j1; jj++) warp_atomic_max(&colmax[jj], m, ok && tl == jj);
  }
  __syncthreads();
  if (threadIdx.x < ntok)
    colscale[threadIdx.x] = ldexpf(1.0f, pow2_exponent(__int_as_float(colmax[threadIdx.x])));
  __syncthreads();
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int ls = it / per, v = it - ls * per;
    const int s = rank + ls * CL;
    const int tl = s / a.kk, sl = s - tl * a.kk;
    const int64_t Iseg = sl < a.k ? a.I : a.Is;
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if ((int64_t)v * 8 < Iseg)
      load8(a.act, kF32, ((int64_t)(t0 + tl) * a.kk + sl) * a.act_ld + (int64_t)v * 8, f);
    store8_f16(xs + (size_t)ls * ldx, v * 8, f, segw[ls] / colscale[tl]);
  }
  __syncthreads();

  Acc acc;
  acc.zero();
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
  float d[4];
  acc.fold(d);
  reduce_to_warp0<WARPS>(d, red);
  // Apply this CTA's per-token prescale, then combine the cluster in rank 0.
  if (warp == 0) {
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int col = 2 * t + (r & 1);
      d[r] = col < ntok ? d[r] * colscale[col] : 0.f;
    }
    if (rank > 0) {
      float* dst = cluster.map_shared_rank(cred, 0);
#pragma unroll
      for (int r = 0; r < 4; r++) dst[((rank - 1) * 4 + r) * 32 + lane] = d[r];
    }
  }
  cluster.sync();
  if (rank == 0 && warp == 0) {
#pragma unroll 1
    for (int q = 1; q < CL; q++)
#pragma unroll
      for (int r = 0; r < 4; r++) d[r] += cred[((q - 1) * 4 + r) * 32 + lane];
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int col = 2 * t + (r & 1);
      const int64_t h = (r < 2) ? h_lo : h_hi;
      if (col < ntok && h < a.H) {
        const int64_t o = (int64_t)(t0 + col) * a.H + h;
        float v = d[r];
        if (a.residual) v += load_as_f32(a.residual, a.dtype, o);
        store_from_f32(a.y, a.dtype, o, v);
      }
    }
  }
}


// ===========================================================================
// Bulk-copy-fed decode kernels (T <= 8).
//
// One CTA per SM-sized share of the tiles: a producer warp streams whole
// weight tiles into a ring of shared-memory slots with cp.async.bulk (one
// copy per lane: 16 code rows + 16 scale rows of a 16-row tile), completion
// tracked by an mbarrier per slot; eight consumer warps compute from shared
// memory and release the slot through a second mbarrier.  Rows are stored
// with padded pitches (codes +64 B, scales +16 B) so the consumers' 128-bit
// and 16-bit shared loads are bank-conflict free.  Many tiles are in flight
// per SM from the first cycle, independent of register pressure.  Every wait
// is bounded (tma.cuh): on expiry the kernel latches error 4 and drains.
// ===========================================================================
constexpr int kTmaConsumers = 8;
constexpr int kTmaThreads = (kTmaConsumers + 1) * 32;
constexpr int kGuSlots = 5;
constexpr int kDnSlots = 16;
constexpr int kErrTimeout = 4;

// Consumer-only staging of T activation rows (no __syncthreads: the
// producer warp does not take part).  Same numerics as stage_columns.
__device__ void stage_rows_consumers(__half* xs, int ldx, int ncols, int K, const void* x,
                                     int dtype, float* colscale, int* colmax) {
  const int nthr = kTmaConsumers * 32;
  if (threadIdx.x < 8) colmax[threadIdx.x] = 0;
  named_sync(1, nthr);
  const int per = K / 8;
  const int items = ncols * per;
  const int rounds = (items + nthr - 1) / nthr;
  for (int r = 0; r < rounds; r++) {
    const int it = r * nthr + threadIdx.x;
    const bool ok = it < items;
    const int j = ok ? it / per : 0;
    float m = 0.f;
    if (ok) {
      float f[8];
      load8(x, dtype, (int64_t)j * K + (int64_t)(it - j * per) * 8, f);
#pragma unroll
      for (int i = 0; i < 8; i++) m = fmaxf(m, fabsf(f[i]));
    }
    const int j0 = __shfl_sync(0xffffffffu, j, 0);
    const int j1 = __shfl_sync(0xffffffffu, ok ? j : j0, 31);
    for (int jj = j0; jj <= j1; jj++) warp_atomic_max(&colmax[jj], m, ok && j == jj);
  }
  named_sync(1, nthr);
  if (threadIdx.x < ncols)
    colscale[threadIdx.x] = ldexpf(1.0f, pow2_exponent(__int_as_float(colmax[threadIdx.x])));
  named_sync(1, nthr);
  for (int it = threadIdx.x; it < items; it += nthr) {
    const int j = it / per, v = it - j * per;
    float f[8];
    load8(x, dtype, (int64_t)j * K + (int64_t)v * 8, f);
    store8_f16(xs + j * ldx, v * 8, f, 1.0f / colscale[j]);
  }
  named_sync(1, nthr);
}

struct TmaSmem {
  uint64_t* full;
  uint64_t* empty;
  uint64_t* red_full;  // [2]
  uint64_t* red_free;  // [2]
};

// --------------------------- gate/up + SwiGLU -----------------------------
// Tiles: u = seg * tps + rg, seg = (token, slot), rg = group of 8 rows (gate
// rows in tile rows 0..7, up rows in 8..15).  CTA b takes u = b, b+G, ...
__global__ void __launch_bounds__(kTmaThreads, 1) moe_gateup_tma_kernel(GateUpArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int H = (int)a.H;
  const int rp = tma_row_pitch(H), sp = tma_scale_pitch(H);
  const int slot_bytes = (16 * rp + 16 * sp + 127) / 128 * 128;
  const uint32_t tile_bytes = (uint32_t)(16 * (H / 2) + 16 * (H / 16));
  const int ldx = H + kXPad;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  TmaSmem B{bars, bars + kGuSlots, bars + 2 * kGuSlots, bars + 2 * kGuSlots + 2};
  unsigned char* p = smem + 256;
  uint8_t* slots = p;
  p += kGuSlots * slot_bytes;
  __half* xs = reinterpret_cast<__half*>(p);
  p += (size_t)a.T * ldx * sizeof(__half);
  float* colscale = reinterpret_cast<float*>(p);
  int* colmax = reinterpret_cast<int*>(colscale + 8);
  float* red = colscale + 16;  // [2][kTmaConsumers-1][4][32]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tps = (int)((std::max(a.I, a.Is) + 7) / 8);
  const int ntiles = (int)a.T * a.kk * tps;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kGuSlots; i++) {
      mbar_init(&B.full[i], 1);
      mbar_init(&B.empty[i], kTmaConsumers);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&B.red_full[i], kTmaConsumers - 1);
      mbar_init(&B.red_free[i], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();

  auto tile_of = [&](int u, int& seg, int64_t& i0) {
    seg = u / tps;
    i0 = (int64_t)(u - seg * tps) * 8;
    const int slot = seg % a.kk;
    return i0 < (slot < a.k ? a.I : a.Is);
  };

  if (warp == kTmaConsumers) {
    // ---------------- producer ----------------
    if (!a.inds_static) pdl_wait();  // routing written by the preceding kernel
    int j = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < ntiles && ok; u += gridDim.x) {
      int seg;
      int64_t i0;
      if (!tile_of(u, seg, i0)) continue;
      const int s = j % kGuSlots;
      if (j >= kGuSlots && !mbar_wait_bounded(&B.empty[s], ((j / kGuSlots) - 1) & 1)) {
        if (lane == 0) flag_error(kErrTimeout);
        ok = false;
        break;
      }
      const int tok = seg / a.kk, slot = seg % a.kk;
      const uint8_t *gw, *gs, *uw, *us;
      if (slot < a.k) {
        uint32_t e = a.inds[(int64_t)tok * a.k + slot];
        if (e >= (uint32_t)a.E) {
          if (lane == 0) flag_error(2);
          e = 0;  // keep the pipeline consistent; the output is flagged invalid
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
      uint8_t* dst = slots + (size_t)s * slot_bytes;
      if (lane == 0) mbar_arrive_expect_tx(&B.full[s], tile_bytes);
      __syncwarp();
      const int r = lane & 15;
      const int64_t row = i0 + (r & 7);
      if (lane < 16) {
        const uint8_t* src = (r < 8 ? gw : uw) + row * (H / 2);
        bulk_g2s(dst + r * rp, src, (uint32_t)(H / 2), &B.full[s]);
      } else {
        const uint8_t* src = (r < 8 ? gs : us) + row * (H / 16);
        bulk_g2s(dst + 16 * rp + r * sp, src, (uint32_t)(H / 16), &B.full[s]);
      }
      j++;
    }
    pdl_wait();
    pdl_trigger();
    // Drain: never leave the CTA with copies still landing in its memory.
    for (int jj = (j > kGuSlots ? j - kGuSlots : 0); jj < j; jj++)
      if (!mbar_wait_bounded(&B.full[jj % kGuSlots], (jj / kGuSlots) & 1) && lane == 0)
        flag_error(kErrTimeout);
    return;
  }

  // ---------------- consumers ----------------
  pdl_wait();  // x is the preceding kernel's output
  pdl_trigger();
  stage_rows_consumers(xs, ldx, (int)a.T, H, a.x, a.dtype, colscale, colmax);
  const int g = lane >> 2, t = lane & 3;
  const int nch = H / kChunk;
  const int c0 = (warp * nch) / kTmaConsumers, c1 = ((warp + 1) * nch) / kTmaConsumers;
  int j = 0;
  for (int u = blockIdx.x; u < ntiles; u += gridDim.x) {
    int seg;
    int64_t i0;
    if (!tile_of(u, seg, i0)) continue;
    const int s = j % kGuSlots;
    if (!mbar_wait_bounded(&B.full[s], (j / kGuSlots) & 1)) {
      if (lane == 0) flag_error(kErrTimeout);
      break;
    }
    const int tok = seg / a.kk;
    const uint8_t* tile = slots + (size_t)s * slot_bytes;
    const __half* xcol = g == 0 ? xs + tok * ldx : nullptr;
    Acc acc;
    acc.zero();
    for (int ch = c0; ch < c1; ch++) {
      Chunk c;
      load_chunk_smem(c, tile, rp, sp, g, ch, t);
      compute_chunk(acc, c, xcol, ch, t);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&B.empty[s]);
    float d[4];
    acc.fold(d);
    const int rb = j & 1;
    float* rbuf = red + rb * (kTmaConsumers - 1) * 4 * 32;
    if (warp > 0) {
      if (j >= 2 && !mbar_wait_bounded(&B.red_free[rb], ((j >> 1) - 1) & 1)) {
        if (lane == 0) flag_error(kErrTimeout);
        break;
      }
#pragma unroll
      for (int r = 0; r < 4; r++) rbuf[((warp - 1) * 4 + r) * 32 + lane] = d[r];
      __syncwarp();
      if (lane == 0) mbar_arrive(&B.red_full[rb]);
    } else {
      if (!mbar_wait_bounded(&B.red_full[rb], (j >> 1) & 1)) {
        if (lane == 0) flag_error(kErrTimeout);
        break;
      }
#pragma unroll 1
      for (int w = 1; w < kTmaConsumers; w++)
#pragma unroll
        for (int r = 0; r < 4; r++) d[r] += rbuf[((w - 1) * 4 + r) * 32 + lane];
      __syncwarp();
      if (lane == 0) mbar_arrive(&B.red_free[rb]);
      if (t == 0) {
        const float cs = colscale[tok];
        a.act[(int64_t)seg * a.act_ld + i0 + g] = silu_ref(d[0] * cs) * (d[2] * cs);
      }
    }
    j++;
  }
}

// ------------------------------ down + combine ------------------------------
// One CTA per 16-row output tile.  Units u = 0..nseg-1 are the segments
// (token, slot) of the tile's K range; unit u's 16 rows of that expert's down
// matrix go through slot u % S.  Consumer warps 0..3 take even units, 4..7 odd
// units, warp w%4 the chunks w%4, w%4+4, ... of the unit; all accumulate in
// registers across units and reduce once at the end.
__global__ void __launch_bounds__(kTmaThreads, 1) moe_down_tma_kernel(DownArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int Ipad = a.Ipad;
  const int rp = tma_row_pitch(Ipad), sp = tma_scale_pitch(Ipad);
  const int slot_bytes = (16 * rp + 16 * sp + 127) / 128 * 128;
  const int ldx = Ipad + kXPad;
  const int ntok = (int)a.T;  // <= 8
  const int nseg = ntok * a.kk;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  TmaSmem B{bars, bars + kDnSlots, bars + 2 * kDnSlots, bars + 2 * kDnSlots + 2};
  unsigned char* p = smem + 512;
  uint8_t* slots = p;
  p += kDnSlots * slot_bytes;
  __half* xs = reinterpret_cast<__half*>(p);
  p += (size_t)nseg * ldx * sizeof(__half);
  float* colscale = reinterpret_cast<float*>(p);
  int* colmax = reinterpret_cast<int*>(colscale + 8);
  float* segw = colscale + 16;       // [nseg]
  float* red = segw + nseg;          // [kTmaConsumers-1][4][32]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t h0 = (int64_t)blockIdx.x * 16;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kDnSlots; i++) {
      mbar_init(&B.full[i], 1);
      mbar_init(&B.empty[i], kTmaConsumers / 2);
    }
    mbar_init(&B.red_full[0], kTmaConsumers - 1);
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kTmaConsumers) {
    // ---------------- producer ----------------
    // The routing is complete before this grid starts (it precedes the
    // gate/up kernel this one follows), so the weights stream immediately.
    if (!a.inds_static) pdl_wait();
    int u = 0;
    for (; u < nseg; u++) {
      const int s = u % kDnSlots;
      if (u >= kDnSlots && !mbar_wait_bounded(&B.empty[s], ((u / kDnSlots) - 1) & 1)) {
        if (lane == 0) flag_error(kErrTimeout);
        break;
      }
      const int tl = u / a.kk, sl = u - tl * a.kk;
      const bool routed = sl < a.k;
      const int Iseg = (int)(routed ? a.I : a.Is);
      const uint8_t *wb, *sb;
      if (routed) {
        uint32_t e = a.inds[(int64_t)tl * a.k + sl];
        if (e >= (uint32_t)a.E) {
          if (lane == 0) flag_error(3);
          e = 0;
        }
        wb = a.dw + (int64_t)e * a.w_stride;
        sb = a.ds + (int64_t)e * a.s_stride;
      } else {
        wb = a.sdw;
        sb = a.sds;
      }
      uint8_t* dst = slots + (size_t)s * slot_bytes;
      if (lane == 0) mbar_arrive_expect_tx(&B.full[s], (uint32_t)(16 * (Iseg / 2 + Iseg / 16)));
      __syncwarp();
      const int r = lane & 15;
      const int64_t row = h0 + r;
      if (lane < 16)
        bulk_g2s(dst + r * rp, wb + row * (Iseg / 2), (uint32_t)(Iseg / 2), &B.full[s]);
      else
        bulk_g2s(dst + 16 * rp + r * sp, sb + row * (Iseg / 16), (uint32_t)(Iseg / 16),
                 &B.full[s]);
    }
    pdl_wait();
    pdl_trigger();
    for (int jj = (u > kDnSlots ? u - kDnSlots : 0); jj < u; jj++)
      if (!mbar_wait_bounded(&B.full[jj % kDnSlots], (jj / kDnSlots) & 1) && lane == 0)
        flag_error(kErrTimeout);
    return;
  }

  // ---------------- consumers ----------------
  const int nthr = kTmaConsumers * 32;
  for (int s = threadIdx.x; s < nseg; s += nthr) {
    const int tl = s / a.kk, sl = s - tl * a.kk;
    segw[s] = sl < a.k ? a.wts[(int64_t)tl * a.k + sl] * a.scaling : 1.0f;
  }
  if (threadIdx.x < 8) colmax[threadIdx.x] = 0;
  pdl_wait();  // act is the preceding kernel's output
  pdl_trigger();
  named_sync(1, nthr);
  const int per = Ipad / 8;
  const int items = nseg * per;
  const int rounds = (items + nthr - 1) / nthr;
  for (int r = 0; r < rounds; r++) {
    const int it = r * nthr + threadIdx.x;
    const bool ok = it < items;
    int tl = 0;
    float m = 0.f;
    if (ok) {
      const int s = it / per, v = it - s * per;
      tl = s / a.kk;
      const int sl = s - tl * a.kk;
      const int64_t Iseg = sl < a.k ? a.I : a.Is;
      if ((int64_t)v * 8 < Iseg) {
        float f[8];
        load8(a.act, kF32, ((int64_t)tl * a.kk + sl) * a.act_ld + (int64_t)v * 8, f);
#pragma unroll
        for (int i = 0; i < 8; i++) m = fmaxf(m, fabsf(f[i] * segw[s]));
      }
    }
    const int j0 = __shfl_sync(0xffffffffu, tl, 0);
    const int j1 = __shfl_sync(0xffffffffu, ok ? tl : j0, 31);
    for (int jj = j0; jj <= j1; jj++) warp_atomic_max(&colmax[jj], m, ok && tl == jj);
  }
  named_sync(1, nthr);
  if (threadIdx.x < ntok)
    colscale[threadIdx.x] = ldexpf(1.0f, pow2_exponent(__int_as_float(colmax[threadIdx.x])));
  named_sync(1, nthr);
  for (int it = threadIdx.x; it < items; it += nthr) {
    const int s = it / per, v = it - s * per;
    const int tl = s / a.kk, sl = s - tl * a.kk;
    const int64_t Iseg = sl < a.k ? a.I : a.Is;
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if ((int64_t)v * 8 < Iseg)
      load8(a.act, kF32, ((int64_t)tl * a.kk + sl) * a.act_ld + (int64_t)v * 8, f);
    store8_f16(xs + (size_t)s * ldx, v * 8, f, segw[s] / colscale[tl]);
  }
  named_sync(1, nthr);

  const int g = lane >> 2, t = lane & 3;
  const int grp = warp >> 2, wq = warp & 3;
  Acc acc;
  acc.zero();
  bool alive = true;
  for (int u = grp; u < nseg; u += 2) {
    const int s = u % kDnSlots;
    if (!mbar_wait_bounded(&B.full[s], (u / kDnSlots) & 1)) {
      if (lane == 0) flag_error(kErrTimeout);
      alive = false;
      break;
    }
    const int tl = u / a.kk, sl = u - tl * a.kk;
    const int nch = (int)((sl < a.k ? a.I : a.Is) / kChunk);
    const uint8_t* tile = slots + (size_t)s * slot_bytes;
    const __half* xcol = g == tl ? xs + (size_t)u * ldx : nullptr;
    for (int ch = wq; ch < nch; ch += 4) {
      Chunk c;
      load_chunk_smem(c, tile, rp, sp, g, ch, t);
      compute_chunk(acc, c, xcol, ch, t);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&B.empty[s]);
  }
  float d[4];
  acc.fold(d);
  if (warp > 0) {
#pragma unroll
    for (int r = 0; r < 4; r++) red[((warp - 1) * 4 + r) * 32 + lane] = d[r];
    __syncwarp();
    if (lane == 0) mbar_arrive(&B.red_full[0]);
    return;
  }
  if (!alive || !mbar_wait_bounded(&B.red_full[0], 0)) {
    if (lane == 0) flag_error(kErrTimeout);
    return;
  }
#pragma unroll 1
  for (int w = 1; w < kTmaConsumers; w++)
#pragma unroll
    for (int r = 0; r < 4; r++) d[r] += red[((w - 1) * 4 + r) * 32 + lane];
#pragma unroll
  for (int r = 0; r < 4; r++) {
    const int col = 2 * t + (r & 1);
    const int64_t h = h0 + g + ((r < 2) ? 0 : 8);
    if (col < ntok && h < a.H) {
      const int64_t o = (int64_t)col * a.H + h;
      float v = d[r] * colscale[col];
      if (a.residual) v += load_as_f32(a.residual, a.dtype, o);
      store_from_f32(a.y, a.dtype, o, v);
    }
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// Host launchers.
constexpr int kQmmWarps = 4;
constexpr int kGateUpWarps = 8;
constexpr int kDownWarps = 4;
constexpr int kDownCluster = 4;

// Launch with optional programmatic dependent launch and cluster shape.
template <typename Kern, typename Args>
static cudaError_t launch_ex(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             bool pdl, int cluster_x, const Args& args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int n = 0;
  if (pdl) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    n++;
  }
  if (cluster_x > 1) {
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = cluster_x;
    attrs[n].val.clusterDim.y = 1;
    attrs[n].val.clusterDim.z = 1;
    n++;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, args);
}

size_t qmm_smem_bytes(int64_t K) {
  return (size_t)8 * (K + kXPad) * sizeof(__half) + 16 * sizeof(float) +
         (size_t)(kQmmWarps - 1) * 4 * 32 * sizeof(float);
}

bool qmm_fast_path_ok(const QmmArgs& a) {
  return a.K % kChunk == 0 && qmm_smem_bytes(a.K) <= 200 * 1024 &&
         (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.w) & 15) == 0 && (a.w_stride & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.s) & 1) == 0 && (a.s_stride & 1) == 0;
}

cudaError_t launch_qmm_gather(const QmmArgs& a, cudaStream_t stream, bool pdl) {
  if (a.P == 0 || a.M == 0 || a.N == 0) return cudaSuccess;
  if (qmm_fast_path_ok(a)) {
    const size_t smem = qmm_smem_bytes(a.K);
    auto kern = qmm_gather_kernel<kQmmWarps>;
    cudaError_t err = ensure_smem(kern, smem);
    if (err != cudaSuccess) return err;
    dim3 grid((unsigned)(a.P * a.mchunks), (unsigned)((a.N + 15) / 16));
    err = launch_ex(kern, grid, dim3(kQmmWarps * 32), smem, stream, pdl, 1, a);
    if (err != cudaSuccess) return err;
  } else {
    const int64_t total = a.P * (int64_t)a.M * a.N;
    const int threads = 256;
    const int64_t blocks = std::min<int64_t>((total + threads - 1) / threads, 148 * 64);
    cudaError_t err = launch_ex(qmm_gather_generic_kernel, dim3((unsigned)blocks), dim3(threads),
                                0, stream, pdl, 1, a);
    if (err != cudaSuccess) return err;
  }
  return cudaGetLastError();
}

size_t gateup_smem_bytes(int64_t H) {
  return (size_t)(H + kXPad) * sizeof(__half) + 16 * sizeof(float) +
         (size_t)(kGateUpWarps - 1) * 4 * 32 * sizeof(float);
}

cudaError_t launch_moe_gateup_tma(const GateUpArgs& a, cudaStream_t stream, bool pdl);
bool gateup_tma_ok(const GateUpArgs& a);

cudaError_t launch_moe_gateup(const GateUpArgs& a, cudaStream_t stream, bool pdl) {
  if (a.T == 0) return cudaSuccess;
  if (a.bulk && gateup_tma_ok(a)) return launch_moe_gateup_tma(a, stream, pdl);
  const size_t smem = gateup_smem_bytes(a.H);
  auto kern = moe_gateup_kernel<kGateUpWarps>;
  cudaError_t err = ensure_smem(kern, smem);
  if (err != cudaSuccess) return err;
  const int64_t Imax = std::max(a.I, a.Is);
  dim3 grid((unsigned)(a.T * a.kk), (unsigned)((Imax + 7) / 8));
  err = launch_ex(kern, grid, dim3(kGateUpWarps * 32), smem, stream, pdl, 1, a);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

int down_max_seg_per_cta(int kk) { return (8 * kk + kDownCluster - 1) / kDownCluster; }

size_t down_smem_bytes(int64_t Ipad, int kk) {
  const int ms = down_max_seg_per_cta(kk);
  return (size_t)ms * (Ipad + kXPad) * sizeof(__half) + (16 + ms) * sizeof(float) +
         (size_t)(kDownWarps - 1 + kDownCluster - 1) * 4 * 32 * sizeof(float);
}

cudaError_t launch_moe_down_tma(const DownArgs& a, cudaStream_t stream, bool pdl);
bool down_tma_ok(const DownArgs& a);

cudaError_t launch_moe_down(const DownArgs& a_in, cudaStream_t stream, bool pdl) {
  if (a_in.T == 0) return cudaSuccess;
  if (a_in.bulk && down_tma_ok(a_in)) return launch_moe_down_tma(a_in, stream, pdl);
  DownArgs a = a_in;
  a.max_seg_per_cta = down_max_seg_per_cta(a.kk);
  const size_t smem = down_smem_bytes(a.Ipad, a.kk);
  auto kern = moe_down_kernel<kDownWarps, kDownCluster>;
  cudaError_t err = ensure_smem(kern, smem);
  if (err != cudaSuccess) return err;
  dim3 grid((unsigned)((a.H + 15) / 16 * kDownCluster), (unsigned)((a.T + 7) / 8));
  err = launch_ex(kern, grid, dim3(kDownWarps * 32), smem, stream, pdl, kDownCluster, a);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}


// ---- bulk-copy-fed decode launchers -----------------------------------------
static int sm_count() {
  static int n[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (n[dev] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n[dev] = v > 0 ? v : 148;
  }
  return n[dev];
}

static size_t gateup_tma_smem(int64_t H, int64_t T) {
  const size_t rp = H / 2 + 64, sp = H / 16 + 16;
  const size_t slot = (16 * rp + 16 * sp + 127) / 128 * 128;
  return 256 + kGuSlots * slot + (size_t)T * (H + kXPad) * sizeof(__half) +
         (16 + 2 * (kTmaConsumers - 1) * 4 * 32) * sizeof(float);
}

static size_t down_tma_smem(int64_t Ipad, int64_t T, int kk) {
  const size_t rp = Ipad / 2 + 64, sp = Ipad / 16 + 16;
  const size_t slot = (16 * rp + 16 * sp + 127) / 128 * 128;
  const size_t nseg = (size_t)T * kk;
  return 512 + kDnSlots * slot + nseg * (Ipad + kXPad) * sizeof(__half) +
         (16 + nseg + (kTmaConsumers - 1) * 4 * 32) * sizeof(float);
}

static bool aligned16p(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

bool gateup_tma_ok(const GateUpArgs& a) {
  return a.T >= 1 && a.T <= 8 && a.H % 256 == 0 && a.I % 8 == 0 && a.Is % 8 == 0 &&
         gateup_tma_smem(a.H, a.T) <= 200 * 1024 && aligned16p(a.gw) && aligned16p(a.gs) &&
         aligned16p(a.uw) && aligned16p(a.us) &&
         (a.Is == 0 || (aligned16p(a.sgw) && aligned16p(a.sgs) && aligned16p(a.suw) &&
                        aligned16p(a.sus)));
}

bool down_tma_ok(const DownArgs& a) {
  return a.T >= 1 && a.T <= 8 && a.I % 256 == 0 && a.Is % 256 == 0 && a.H % 16 == 0 &&
         down_tma_smem(a.Ipad, a.T, a.kk) <= 200 * 1024 && aligned16p(a.dw) &&
         aligned16p(a.ds) && (a.Is == 0 || (aligned16p(a.sdw) && aligned16p(a.sds)));
}

cudaError_t launch_moe_gateup_tma(const GateUpArgs& a, cudaStream_t stream, bool pdl) {
  const size_t smem = gateup_tma_smem(a.H, a.T);
  cudaError_t err = ensure_smem(moe_gateup_tma_kernel, smem);
  if (err != cudaSuccess) return err;
  const int64_t tps = (std::max(a.I, a.Is) + 7) / 8;
  const int64_t ntiles = a.T * a.kk * tps;
  const int grid = (int)std::min<int64_t>(ntiles, sm_count());
  err = launch_ex(moe_gateup_tma_kernel, dim3(grid), dim3(kTmaThreads), smem, stream, pdl, 1, a);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

cudaError_t launch_moe_down_tma(const DownArgs& a, cudaStream_t stream, bool pdl) {
  const size_t smem = down_tma_smem(a.Ipad, a.T, a.kk);
  cudaError_t err = ensure_smem(moe_down_tma_kernel, smem);
  if (err != cudaSuccess) return err;
  err = launch_ex(moe_down_tma_kernel, dim3((unsigned)(a.H / 16)), dim3(kTmaThreads), smem,
                  stream, pdl, 1, a);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

cudaError_t read_and_clear_device_error(int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_device_error, sizeof(int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
}

}  // namespace nvfp4
