// prefill_fp4.cu -- the MoE prefill GEMMs on the block-scaled FP4 tensor
// cores (tcgen05.mma kind::mxf4nvf4): no dequantisation pass.
//
// Same semantics as prefill.cu (gather_qmm over expert-sorted slots,
// VMLX/backend/cpu/quantized.cpp:805-844; SwitchGLU, SwitchLayers.swift:
// 532-580; the Laguna combine, Laguna.swift:204-212), with the activations
// carried as a sum of four NVFP4 terms instead of 16-bit values:
//
//   x_row = sum_t fac[t] * dequant(codes_t, scales_t),
//
// term t being the NVFP4 quantisation (UE4M3 scale per group of 16, E2M1
// codes rounded to nearest even) of the row's residual after terms 0..t-1,
// under a power-of-two factor per (row, term): the row's max places its largest
// term-0 group scale in [171, 352], term t's factor is 4^-t times that (no
// term's scales overflow E4M3; groups far below the row max get subnormal
// scales in the later terms).  Each term cuts the residual by at least 6x per
// group; four terms reproduce the W4A16 product to a relative-L2 of ~1e-4
// (N(0,1) rows and SwiGLU outputs, a numpy restatement), 50x inside the
// path's 5e-3 tolerance.  The weight operand is the checkpoint's NVFP4 data as
// is (codes and E4M3 group scales used as UE4M3: the quantizer never emits a
// sign bit or 0x7F).  Every product is exact and sums in f32.
//
// rows_to_terms_kernel: one warp per source row, the row's groups spread over
//   the lanes; writes the four term rows (slot * 4 + t) of every slot the row
//   feeds (x: its k routed slots and its shared-expert slot; act: itself).
// nvfp4_gemm_fp4_kernel: one persistent CTA per SM over the tile list of
//   moe_sort (tiles of <= 32 slots of one expert), in weight-row tiles of 128
//   (mode 1: 64 gate rows + the same 64 up rows; mode 2: 128 down rows):
//     TMA warp       per 256-wide K slab: the tile's weight codes + scales and
//                    its 128 term rows (32 slots x 4 terms) + scales, into a
//                    4-deep ring (128-byte swizzled K-major);
//     scale warps    (4) copy each stage's scale bytes into tensor memory in
//                    the layout the block-scaled MMA reads (scale of row m,
//                    block j at lanes m % 32 + 32 r, r = 0..3, column m / 32,
//                    byte j);
//     MMA thread     4 tcgen05.mma per slab (M=128, N = 4 x slots, K=64) into
//                    one of three TMEM accumulators;
//     epilogue       (8 warps, two per TMEM lane quarter, alternate 32-column
//                    chunks) accumulator column 4 j + t holds term t of slot
//                    j: y = sum_t fac * D.  Mode 2 writes Y[slot][row]; mode 1
//                    passes gate and up values through shared memory (the
//                    gate rows sit in lane quarters 0-1, the up rows in 2-3)
//                    and writes act = silu(gate) * up.
// Every wait is bounded (tma.cuh): on expiry error 4 is latched and each role
// leaves its loop before TMEM is released.
#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"
#include "fp4terms.cuh"

namespace nvfp4 {
namespace {

constexpr int kT = kFp4Terms;
constexpr int kFBM = 128;                  // weight rows per tile (MMA M)
constexpr int kFTok = kFp4TileTokens;      // slots per tile
constexpr int kFRows = kT * kFTok;         // term rows per tile = max MMA N (128)
constexpr int kFStages = 4;
constexpr int kFBufs = 3;                  // accumulators: the epilogue trails the MMA by up to two tiles
constexpr int kFA = kFBM * 128;            // weight codes of one slab: 16 KB
constexpr int kFB = kFRows * 128;          // term-row codes of one slab: 16 KB
constexpr int kFSA = kFBM * 16;            // weight scales: 2 KB
constexpr int kFSB = kFRows * 16;          // term-row scales: 2 KB
constexpr int kFStage = kFA + kFB + kFSA + kFSB;  // 36 KB, 1 KB multiple
static_assert(kFStage % 1024 == 0, "stage alignment");
constexpr int kFThreads = 448;             // 0 TMA, 1 MMA, 2-5 scales, 6-13 epilogue
constexpr int kWarpTma = 0, kWarpMma = 1, kWarpEpi0 = 6;  // warps 2-5: scale factors
// Epilogue: two warps per tensor-memory lane quarter (warp w reads lanes
// 32 (w % 4) ..), each taking every other 32-column chunk of a tile.
constexpr int kEpiT = kFThreads - 32 * kWarpEpi0;  // 256
constexpr int kFAcc = 128;                 // accumulator columns (one buffer)
constexpr int kFSf = 32;                   // scale columns per stage: 16 A + 16 B
constexpr int kFTmem = 512;
static_assert(kFBufs * kFAcc + kFStages * kFSf <= kFTmem, "TMEM budget");
constexpr int kGuPitch = kFTok + 1;        // gate/up exchange rows (bank-conflict free)
constexpr int kErrTimeout = 4;
constexpr long long kDrainBudget = 200000000LL;

__device__ int g_fp4_error = 0;
__device__ __forceinline__ void fflag(int code) { atomicCAS(&g_fp4_error, 0, code); }

__device__ __forceinline__ void pdl_wait_f() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger_f() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint32_t elect_one() {
  uint32_t e;
  asm volatile("{\n.reg .pred p;\nelect.sync _|p, 0xffffffff;\nselp.u32 %0, 1, 0, p;\n}\n"
               : "=r"(e));
  return e;
}

// Named barrier over `count` threads that also ANDs a predicate across them:
// the epilogue warps leave their loop together (a warp that left alone would
// strand the others at the next barrier).
__device__ __forceinline__ bool sync_and(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n"
      ".reg .pred p, q;\n"
      "setp.ne.u32 p, %1, 0;\n"
      "bar.red.and.pred q, %2, %3, p;\n"
      "selp.u32 %0, 1, 0, q;\n"
      "}\n"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

// rows_to_terms: one CTA of K / 512 warps per source row; lane l of warp w
// owns group 32 w + l (16 consecutive values).  The row max (warp shuffle +
// shared memory across the warps) sets the factors; per term: the group's
// UE4M3 scale (the smallest >= amax * P / 6), codes by the hardware converter,
// the residual updated with the values the codes stand for.
__global__ void __launch_bounds__(128) rows_to_terms_kernel(TermsArgs a) {
  __shared__ float wmax[2][4];
  pdl_wait_f();
  pdl_trigger_f();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  const int64_t K = a.K;
  const int64_t cb = K / 2, sbytes = K / 16;  // bytes per term row
  const int grp = 32 * warp + lane;
  int it = 0;  // rows this CTA has decomposed
  for (int64_t r = blockIdx.x; r < a.rows; r += gridDim.x) {
    const bool extra = a.extra_base >= 0 && r >= a.extra_lo && r < a.extra_hi;
    if (a.dst_map && !extra) {  // a row no slot reads (expert-parallel: all foreign)
      bool any = false;
      for (int d = 0; d < a.map_count; d++) any |= a.dst_map[r * a.map_stride + d] >= 0;
      if (!any) continue;  // uniform over the CTA
    }
    float v[16];
    const int64_t e0 = r * a.src_ld + (int64_t)grp * 16;
    load8(a.src, a.src_dtype, e0, *reinterpret_cast<float(*)[8]>(&v[0]));
    load8(a.src, a.src_dtype, e0 + 8, *reinterpret_cast<float(*)[8]>(&v[8]));
    uint2 code[kT];
    uint32_t sb[kT];
    float fac[kT];
    // A row holding NaN or +-inf keeps the reference's non-finite result: its
    // terms are written with NaN factors (the row max is forced to +inf).
    bool bad = false;
#pragma unroll
    for (int j = 0; j < 16; j++) bad |= !isfinite(v[j]);
    // The row's max sets term 0's factor P = 2^(10 - floor(log2 m)) (m * P in
    // [1024, 2048): the largest group scale in [171, 352]); term t uses P * 4^t.
    // A term's residual is at most its group scale (E2M1 spacing 2 at the top,
    // no saturation as scales round up), so the next term's scales stay <= 2/3
    // of this term's bound: no E4M3 overflow, one row max instead of four.
    float m;
    {
      float a0 = 0.f;
#pragma unroll
      for (int j = 0; j < 16; j++) a0 = fmaxf(a0, fabsf(v[j]));
      m = warp_max(bad ? INFINITY : a0);
      if (nw > 1) {  // buffer by row parity: the next row's writes pass one barrier first
        if (lane == 0) wmax[it & 1][warp] = m;
        __syncthreads();
        m = wmax[it & 1][0];
        for (int w = 1; w < nw; w++) m = fmaxf(m, wmax[it & 1][w]);
      }
    }
    // Exponent arithmetic on normal floats (rows whose max is below 2^-100,
    // zero or not finite get no terms).
    const int em = (__float_as_int(m) >> 23) & 0xFF;  // biased exponent of m
    const bool live = m >= 7.9e-31f && m < INFINITY;
    float P = live ? __int_as_float((127 + 10 - (em - 127)) << 23) : 0.f;
    float f = live ? __int_as_float((127 - 10 + (em - 127)) << 23)  // 1 / P
                   : (m == INFINITY ? __int_as_float(0x7fc00000) : 0.f);
#pragma unroll
    for (int t = 0; t < kT; t++, P *= 4.0f, f *= 0.25f) {
      float amax = 0.f;
#pragma unroll
      for (int j = 0; j < 16; j++) amax = fmaxf(amax, fabsf(v[j]));
      fac[t] = f;
      const uint32_t b = live ? e4m3_ceil_fast(amax * P * (1.0f / 6.0f)) : 0u;
      const float s = scale_to_f32(b);
      // |v * inv| <= 6 up to rounding (the converter saturates there); the
      // residual below uses the exact value the code stands for
      const float inv = s > 0.f ? P * __frcp_rn(s) : 0.f;
      const float back = s > 0.f ? s * f : 0.f;  // s > 0 only for live rows
      uint32_t w[2] = {0u, 0u};
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        const uint32_t byte = e2m1_pair(v[j] * inv, v[j + 1] * inv);
        const float2 q = e2m1_pair_value(byte);
        v[j] -= q.x * back;
        v[j + 1] -= q.y * back;
        w[j >> 3] |= byte << (4 * (j & 7));
      }
      code[t] = make_uint2(w[0], w[1]);
      sb[t] = b;
    }
    it++;
    // Every destination slot of this row.
    const int nd = a.dst_map ? a.map_count : 0;
    for (int d = -1; d < nd + 1; d++) {
      int64_t slot;
      if (d < 0) {
        if (a.dst_map || a.extra_base >= 0) continue;
        slot = r;  // identity
      } else if (d < nd) {
        slot = a.dst_map[r * a.map_stride + d];
        if (slot < 0) continue;
      } else {
        if (!extra) continue;
        slot = a.extra_base + (r - a.extra_lo);
      }
#pragma unroll
      for (int t = 0; t < kT; t++) {
        const int64_t tr = slot * kT + t;
        *reinterpret_cast<uint2*>(a.codes + tr * cb + (int64_t)grp * 8) = code[t];
        a.scales[tr * sbytes + grp] = (uint8_t)sb[t];
        if (threadIdx.x == 0) a.fac[tr] = fac[t];
      }
    }
  }
}

// ---------------------------------------------------------------------------
struct FTile {
  int grp, start, count, N, m_tile, Mrows;
  bool is_shared;
};

__device__ __forceinline__ int f_total(const GemmFp4Args& a, int m_tiles) {
  return *a.ntiles * m_tiles;
}

// Tile u: tile-list entry u / m_tiles (staged in shared memory), weight-row
// tile u % m_tiles.  False when that weight-row tile lies beyond the group.
__device__ __forceinline__ bool f_tile(const GemmFp4Args& a, const int4* stiles, int u, int m_tiles,
                                       FTile& ti) {
  const int gt = u / m_tiles;
  ti.m_tile = u - gt * m_tiles;
  const int4 td = stiles[gt];
  ti.grp = td.x;
  ti.start = td.y;
  ti.count = td.z;
  ti.N = (kT * ti.count + 15) & ~15;
  ti.is_shared = ti.grp == a.shared_group;
  ti.Mrows = ti.is_shared ? a.Mrows_shared : a.Mrows;
  return ti.m_tile * (a.mode == 1 ? 64 : 128) < ti.Mrows;
}

__device__ __forceinline__ float silu_f(float x) {
  const float y = __fdividef(1.0f, 1.0f + __expf(fabsf(x)));
  return x * (x < 0.0f ? y : 1.0f - y);
}

// MODE (1 gate/up + SwiGLU, 2 down) as a template parameter: each launch runs
// only its own epilogue code.
template <int MODE>
__global__ void __launch_bounds__(kFThreads, 1)
    nvfp4_gemm_fp4_kernel(const __grid_constant__ GemmFp4Args a) {
  extern __shared__ __align__(1024) unsigned char fsmem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(fsmem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sStage = smem;                                             // [kFStages][kFStage]
  float* sG = reinterpret_cast<float*>(sStage + kFStages * kFStage);  // [64][kGuPitch]
  float* sU = sG + 64 * kGuPitch;                                     // [64][kGuPitch]
  float* sFac = sU + 64 * kGuPitch;                                   // [kFRows]
  uint64_t* full = reinterpret_cast<uint64_t*>(sFac + kFRows);
  uint64_t* empty = full + kFStages;
  uint64_t* sf_ready = empty + kFStages;
  uint64_t* acc_full = sf_ready + kFStages;
  uint64_t* acc_empty = acc_full + kFBufs;
  uint64_t* drain = acc_empty + kFBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  // [a.max_tiles] tile list, 16-byte aligned for the int4 accesses
  int4* sTiles = reinterpret_cast<int4*>(
      (reinterpret_cast<uintptr_t>(tmem_slot + 4) + 15) & ~static_cast<uintptr_t>(15));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kFStages; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
      mbar_init(&sf_ready[i], 4);
    }
    for (int i = 0; i < kFBufs; i++) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpiT / 32);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == kWarpTma && lane == 0) {
    prefetch_map(&a.mc0);
    prefetch_map(&a.ms0);
    for (int i = 0; i < 4; i++) {
      prefetch_map(&a.mb[i]);
      prefetch_map(&a.msb[i]);
    }
  }
  pdl_wait_f();  // tiles and term rows come from the preceding kernels
  pdl_trigger_f();
  const int m_tiles = MODE == 1 ? (max(a.Mrows, a.Mrows_shared) + 63) / 64
                                  : (max(a.Mrows, a.Mrows_shared) + 127) / 128;
  const int ntot = f_total(a, m_tiles);
  if ((int)blockIdx.x >= ntot) return;  // uniform per CTA, before any barrier use
  // the tile list once into shared memory: every role walks it per tile, and
  // a global read there costs ~1 us while the weight stream fills the memory
  const int nlist = min(*a.ntiles, a.max_tiles);
  for (int i = threadIdx.x; i < nlist; i += blockDim.x) sTiles[i] = a.tiles[i];
  if (warp == kWarpMma) tmem_alloc(tmem_slot, kFTmem);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tsf = tmem + kFBufs * kFAcc;  // stage s: tsf + kFSf * s
  const int nslab = a.K / 256;

  if (warp == kWarpTma) {
    // ------------------------------ TMA producer ------------------------------
    const uint32_t el = elect_one();
    uint32_t g = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < ntot && ok; u += gridDim.x) {
      FTile ti;
      if (!f_tile(a, sTiles, u, m_tiles, ti)) continue;
      const CUtensorMap* c0 = ti.is_shared ? &a.mcs0 : &a.mc0;
      const CUtensorMap* s0 = ti.is_shared ? &a.mss0 : &a.ms0;
      const CUtensorMap* c1 = ti.is_shared ? &a.mcs1 : &a.mc1;
      const CUtensorMap* s1 = ti.is_shared ? &a.mss1 : &a.ms1;
      const int row0 = (ti.is_shared ? 0 : ti.grp * a.Mrows) + ti.m_tile * (MODE == 1 ? 64 : 128);
      const int brow = ti.start * kT;
      const int hb = (ti.N + 31) / 32 - 1;  // term rows loaded: 32 (hb + 1) >= N
      const uint32_t tx = (uint32_t)(kFA + kFSA) +
                          (uint32_t)(32 * (hb + 1)) * (128 + 16);
      for (int sl = 0; sl < nslab; sl++, g++) {
        const int s = g % kFStages;
        if (g >= kFStages && !mbar_wait_bounded(&empty[s], ((g / kFStages) - 1) & 1)) {
          if (el) fflag(kErrTimeout);
          ok = false;
          break;
        }
        if (el) {
          uint8_t* st = sStage + s * kFStage;
          mbar_arrive_expect_tx(&full[s], tx);
          if (MODE == 1) {
            tma_load_2d(st, c0, sl * 128, row0, &full[s]);
            tma_load_2d(st + kFA / 2, c1, sl * 128, row0, &full[s]);
            tma_load_2d(st + kFA + kFB, s0, sl * 16, row0, &full[s]);
            tma_load_2d(st + kFA + kFB + kFSA / 2, s1, sl * 16, row0, &full[s]);
          } else {
            tma_load_2d(st, c0, sl * 128, row0, &full[s]);
            tma_load_2d(st + kFA + kFB, s0, sl * 16, row0, &full[s]);
          }
          tma_load_2d(st + kFA, &a.mb[hb], sl * 128, brow, &full[s]);
          tma_load_2d(st + kFA + kFB + kFSA, &a.msb[hb], sl * 16, brow, &full[s]);
        }
        __syncwarp();
      }
    }
    // no copy may still be landing at exit
    for (uint32_t i = 0; i < (g < (uint32_t)kFStages ? g : (uint32_t)kFStages); i++) {
      const uint32_t q = g - 1 - i;
      mbar_wait_bounded(&full[q % kFStages], (q / kFStages) & 1, kDrainBudget);
    }
  } else if (warp == kWarpMma) {
    // ------------------------------ MMA issuer ------------------------------
    const uint32_t el = elect_one();
    uint32_t g = 0;
    int j = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < ntot && ok; u += gridDim.x) {
      FTile ti;
      if (!f_tile(a, sTiles, u, m_tiles, ti)) continue;
      const int buf = j % kFBufs;
      if (j >= kFBufs && !mbar_wait_bounded(&acc_empty[buf], ((j / kFBufs) - 1) & 1)) {
        if (el) fflag(kErrTimeout);
        break;
      }
      tc_fence_after();
      const uint32_t idesc = idesc_mxf4nvf4(kFBM, ti.N);
      const uint32_t d = tmem + (uint32_t)(buf * kFAcc);
      for (int sl = 0; sl < nslab; sl++, g++) {
        const int s = g % kFStages;
        if (!mbar_wait_bounded(&sf_ready[s], (g / kFStages) & 1)) {
          if (el) fflag(kErrTimeout);
          ok = false;
          break;
        }
        tc_fence_after();
        if (el) {
          const uint32_t sa = smem_u32(sStage + s * kFStage);
          const uint32_t sb = sa + kFA;
          const uint32_t sfa = tsf + (uint32_t)(s * kFSf);
#pragma unroll
          for (int k4 = 0; k4 < 4; k4++)
            umma_mxf4nvf4(d, smem_desc_sw128(sa + 32 * k4), smem_desc_sw128(sb + 32 * k4), idesc,
                          sfa + 4 * k4, sfa + 16 + 4 * k4, (sl | k4) != 0 ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (el) umma_commit(&acc_full[buf]);
      __syncwarp();
      j++;
    }
    if (el) umma_commit(drain);
    __syncwarp();
    if (!mbar_wait_bounded(drain, 0) && el) fflag(kErrTimeout);
  } else if (warp < kWarpEpi0) {
    // ---------------------- scale factors into tensor memory ----------------------
    const int q = warp & 3;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    uint32_t g = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < ntot && ok; u += gridDim.x) {
      FTile ti;
      if (!f_tile(a, sTiles, u, m_tiles, ti)) continue;
      for (int sl = 0; sl < nslab; sl++, g++) {
        const int s = g % kFStages;
        if (!mbar_wait_bounded(&full[s], (g / kFStages) & 1)) {
          if (lane == 0) fflag(kErrTimeout);
          ok = false;
          break;
        }
        const uint8_t* st = sStage + s * kFStage;
        uint32_t ra[16], rb[16];
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const uint4 va = *reinterpret_cast<const uint4*>(st + kFA + kFB + 16 * (lane + 32 * c));
          ra[0 + c] = va.x;
          ra[4 + c] = va.y;
          ra[8 + c] = va.z;
          ra[12 + c] = va.w;
          const uint4 vb =
              *reinterpret_cast<const uint4*>(st + kFA + kFB + kFSA + 16 * (lane + 32 * c));
          rb[0 + c] = vb.x;
          rb[4 + c] = vb.y;
          rb[8 + c] = vb.z;
          rb[12 + c] = vb.w;
        }
        const uint32_t col = tsf + (uint32_t)(s * kFSf);
        tmem_st16(lane_base + col, ra);
        tmem_st16(lane_base + col + 16, rb);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sf_ready[s]);
      }
    }
  } else {
    // ------------------------------ epilogue ------------------------------
    const int q = warp & 3;  // TMEM lane quarter: rows 32 q .. 32 q + 31
    const int eh = (warp - kWarpEpi0) >> 2;       // chunks eh, eh + 2, ... of a tile
    const int et = threadIdx.x - 32 * kWarpEpi0;  // 0 .. kEpiT - 1
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    int j = 0;
    // The tile's term factors (column 4 s + t <- slot s, term t), loaded one
    // tile ahead so the global read stays off the per-tile chain.
    auto next_tile = [&](int from, FTile& nt) -> int {
      for (int v = from; v < ntot; v += gridDim.x)
        if (f_tile(a, sTiles, v, m_tiles, nt)) return v;
      return ntot;
    };
    FTile tn;
    int un = next_tile(blockIdx.x, tn);
    float fnext = (un < ntot && et < kT * tn.count) ? a.bfac[(int64_t)tn.start * kT + et] : 0.f;
    while (un < ntot) {
      const FTile ti = tn;
      const int u = un;
      const float fcur = fnext;
      un = next_tile(u + gridDim.x, tn);
      fnext = (un < ntot && et < kT * tn.count) ? a.bfac[(int64_t)tn.start * kT + et] : 0.f;
      const int buf = j % kFBufs;
      named_sync(2, kEpiT);
      if (et < kFRows) sFac[et] = fcur;
      named_sync(2, kEpiT);
      const bool got = mbar_wait_bounded(&acc_full[buf], (j / kFBufs) & 1);
      if (!got && lane == 0) fflag(kErrTimeout);
      if (!sync_and(2, kEpiT, got)) break;
      tc_fence_after();
      const int r = 32 * q + lane;  // accumulator row = TMEM lane
      // every slot of a chunk folded unconditionally (straight-line code: the
      // factors of slots past the tile are zero), then the guarded stores;
      // a slot's four factors in one 16-byte shared-memory read
      const float4* fac4 = reinterpret_cast<const float4*>(sFac);
      for (int c0 = 32 * eh; c0 < ti.N; c0 += 64) {
        uint32_t v[32];
        tmem_ld32_nowait(tmem + lane_base + (uint32_t)(buf * kFAcc + c0), v);
        tmem_wait_ld();
        float yy[8];
#pragma unroll
        for (int jj = 0; jj < 8; jj++) {
          const float4 f = fac4[c0 / kT + jj];
          float y = 0.f;
          y += f.x * __uint_as_float(v[kT * jj]);
          y += f.y * __uint_as_float(v[kT * jj + 1]);
          y += f.z * __uint_as_float(v[kT * jj + 2]);
          y += f.w * __uint_as_float(v[kT * jj + 3]);
          yy[jj] = y;
        }
#pragma unroll
        for (int jj = 0; jj < 8; jj++) {
          const int sidx = c0 / kT + jj;  // slot within the tile
          if (sidx >= ti.count) continue;
          const float y = yy[jj];
          if (MODE == 2) {
            const int row = ti.m_tile * 128 + r;
            if (row < ti.Mrows) a.out[(int64_t)(ti.start + sidx) * a.out_ld + row] = y;
          } else if (r < 64) {
            sG[r * kGuPitch + sidx] = y;
          } else {
            sU[(r - 64) * kGuPitch + sidx] = y;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      if (MODE == 1) {
        named_sync(2, kEpiT);
        const int i = et & 63;
        const int row = ti.m_tile * 64 + i;
        if (row < ti.Mrows)
          for (int sidx = et >> 6; sidx < ti.count; sidx += kEpiT / 64)
            a.out[(int64_t)(ti.start + sidx) * a.out_ld + row] =
                silu_f(sG[i * kGuPitch + sidx]) * sU[i * kGuPitch + sidx];
      }
      j++;
    }
  }
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kFTmem);
  }
}

template <typename Kern, typename... Args>
cudaError_t launch_pdl_f(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                         const Args&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

}  // namespace

size_t gemm_fp4_smem_bytes(int max_tiles) {
  return 1024 + (size_t)kFStages * kFStage + 2 * 64 * kGuPitch * sizeof(float) +
         kFRows * sizeof(float) + (3 * kFStages + 2 * kFBufs + 1) * 8 + 16 + 16 + (size_t)max_tiles * 16;
}

cudaError_t launch_rows_to_terms(const TermsArgs& a, cudaStream_t stream) {
  if (a.rows == 0) return cudaSuccess;
  if (a.K % 512 != 0 || a.K > 2048) return cudaErrorInvalidValue;
  const int threads = (int)(a.K / 512) * 32;
  const int blocks = (int)std::min<int64_t>(a.rows, 148 * 32);
  return launch_pdl_f(rows_to_terms_kernel, dim3(blocks), dim3(threads), 0, stream, a);
}

cudaError_t launch_nvfp4_gemm_fp4(const GemmFp4Args& a, int max_tiles, cudaStream_t stream) {
  if (a.max_tiles != max_tiles) return cudaErrorInvalidValue;
  const size_t smem = gemm_fp4_smem_bytes(max_tiles);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if (a.mode != 1 && a.mode != 2) return cudaErrorInvalidValue;
  auto kern = a.mode == 1 ? nvfp4_gemm_fp4_kernel<1> : nvfp4_gemm_fp4_kernel<2>;
  cudaError_t e = ensure_smem(kern, smem);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const int m_tiles = a.mode == 1 ? (std::max(a.Mrows, a.Mrows_shared) + 63) / 64
                                  : (std::max(a.Mrows, a.Mrows_shared) + 127) / 128;
  const int grid = std::max(1, std::min(sms, max_tiles * m_tiles));
  return launch_pdl_f(kern, dim3(grid), dim3(kFThreads), smem, stream, a);
}

cudaError_t read_and_clear_fp4_error(int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_fp4_error, sizeof(int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_fp4_error, &zero, sizeof(int));
}

}  // namespace nvfp4
