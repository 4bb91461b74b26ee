// prefill.cu -- the sorted-expert (grouped) NVFP4 GEMM on sm_100a tensor
// cores (tcgen05, TMEM accumulators, TMA operand feeds) and the MoE prefill
// plumbing around it.
//
// Reference semantics: gather_qmm over tokens sorted by expert
// (VMLX/backend/cpu/quantized.cpp:805-844 per pair; SwitchGLU with
// sortedIndices, VLM/MLXLMCommon/SwitchLayers.swift:532-580; gatherSort /
// scatterUnsort :385-428), the Laguna block combine (Laguna.swift:204-212).
//
// GEMM: D[weight rows, tokens] = W[rows, K] x X[tokens, K]^T in tiles of 128
// weight rows (UMMA M) by up to 64 tokens (UMMA N), K in MMA stages of 64.
// One persistent CTA per SM walks its tiles; warp roles form a pipeline that
// runs across tile boundaries:
//   weight TMA (1 thread)  per 256-wide K slab, the tile rows' packed codes
//                          (16 KB, 128-byte swizzle) and E4M3 scales (2 KB)
//                          into a 6-deep shared-memory ring;
//   dequantisers          4 groups of 4 warps; group q owns K quarter q of
//   (16 warps)            every slab, one thread per tile row (= TMEM lane):
//                          E2M1 pairs by the hardware converter times the group
//                          scale (exact in f16 / bf16), written to one of two
//                          A slabs in tensor memory (tcgen05.st);
//   activation TMA         16-row boxes of the tile's slot-ordered 16-bit
//   (1 thread)             activation rows, a whole slab at a time, into a
//                          3-deep B ring (128-byte swizzled K-major);
//   MMA issuer (1 thread)  per slab 16 tcgen05.mma kind::f16 (A from TMEM, B
//                          from shared memory) into one of two TMEM
//                          accumulators, then one commit per freed buffer.
// The MMA issue costs a fixed ~46 cycles per instruction for N <= 96, so the
// per-slab granularity keeps the issuing thread's bookkeeping off that path.
//   epilogue (4 warps)     tcgen05.ld of the finished accumulator (one TMEM
//                          sub-partition each; the accumulator is released at
//                          once), staged in shared memory one slot row per
//                          tile column, written out with coalesced 16-byte
//                          stores while the next tile runs.
// Operand type: f16 for pre-scaled activation rows (rows_to_f16: per-row power
// of two, exact for bf16 inputs, re-applied in the epilogue) and for f16
// inputs; bf16 for bf16 inputs (dense quantized_matmul, no workspace).
// Epilogue modes: 0 plain out[slot][n] = D; 1 gate/up: tile rows
// alternate blocks of 8 gate rows and the same 8 up rows, so TMEM lanes r and
// r ^ 8 pair up in one warp and act = silu(gate) * up (f32); 2 down: Y[slot][n] = D (f32, combined per token
// afterwards).  All mbarrier waits are bounded (tma.cuh): on expiry error 4 is
// latched and every role leaves its loop before TMEM is released.
#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"

#include <mutex>

#include <cudaTypedefs.h>

namespace nvfp4 {
namespace {

constexpr int kBM = 128;                     // weight rows per tile
constexpr int kBN = 64;                      // tokens per tile (max UMMA N used)
constexpr int kBK = 64;                      // K per MMA stage: one 128 B swizzle row of 16-bit
constexpr int kSlabK = 256;                  // K per weight slab (128 code bytes per row)
constexpr int kStages = 4;                   // 64-wide K stages per slab
constexpr int kASlabs = 2;                   // A slabs in TMEM
constexpr int kBSlabs = 3;                   // B (activation) slabs in shared memory
constexpr int kRawSlots = 5;                 // weight slabs in flight
constexpr int kOutPitch = 512;               // staged output: bytes per tile column (slot)
constexpr int kGroupWarps = 4;               // one dequantiser group: 128 threads = 128 rows
constexpr int kDeqWarps = kStages * kGroupWarps;
constexpr int kEpiWarps = 4;
constexpr int kWarpMma = 0, kWarpRaw = 1, kWarpAct = 2, kWarpDeq0 = 3;
constexpr int kWarpEpi0 = kWarpDeq0 + kDeqWarps;  // 19..22: TMEM sub-partitions 3,0,1,2
static_assert(kStages * kBK == kSlabK, "dequantiser group q owns stage q of each slab");
constexpr int kGemmThreads = 32 * (kWarpEpi0 + kEpiWarps);
constexpr int kStageB = kBN * kBK * 2;       // 8 KB
constexpr int kSlabB = kStages * kStageB;    // 32 KB
constexpr int kBoxB = 16 * kBK * 2;          // one 16-row activation box, 2 KB
constexpr int kRawCodes = kBM * 128;         // 16 KB
constexpr int kRawSlot = kRawCodes + kBM * 16;  // + 16 scale bytes per row
constexpr int kAccCols = 2 * kBN;            // two f32 accumulators
constexpr int kACols = kBK / 2;              // one A stage: 64 16-bit K per lane
constexpr int kASlabCols = kStages * kACols; // 128
constexpr int kTmemCols = 512;               // accumulators + A slabs, power of two
static_assert(kAccCols + kASlabs * kASlabCols <= kTmemCols, "TMEM budget");
constexpr int kErrTimeout = 4;
constexpr long long kDrainBudget = 200000000LL;  // ~0.1 s: in-flight copies on an error path

__device__ int g_prefill_error = 0;
__device__ __forceinline__ void flag(int code) { atomicCAS(&g_prefill_error, 0, code); }

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- dequantisation of 8 codes (one word) into 16 bytes of operand ----------
__device__ __forceinline__ uint4 dequant8_f16(uint32_t word, uint32_t scale_f16x2) {
  uint32_t h[4];
  e2m1x8_to_f16x2x4(word, h);
  return make_uint4(hmul2_u32(h[0], scale_f16x2), hmul2_u32(h[1], scale_f16x2),
                    hmul2_u32(h[2], scale_f16x2), hmul2_u32(h[3], scale_f16x2));
}

__device__ __forceinline__ uint4 dequant8_bf16(uint32_t word, uint32_t scale_f16x2) {
  uint32_t h[4];
  e2m1x8_to_f16x2x4(word, h);
  const float s = __half2float(__ushort_as_half((unsigned short)(scale_f16x2 & 0xFFFFu)));
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[i]));
    const __nv_bfloat162 b = __floats2bfloat162_rn(f.x * s, f.y * s);
    o[i] = *reinterpret_cast<const uint32_t*>(&b);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// ---- tile bookkeeping (identical in every role) --------------------------------
struct TileInfo {
  int grp, start, count, N, m_tile, Mrows;
  bool is_shared;
};

__device__ __forceinline__ int total_tiles(const GemmArgs& a, int m_tiles) {
  const int ngt = a.implicit_M > 0 ? (a.implicit_M + kBN - 1) / kBN : *a.ntiles;
  return ngt * m_tiles;
}

// Tile-list entry of tile u (read one tile ahead by every role: a global
// load costs ~1 us while the weight stream fills the memory system).
__device__ __forceinline__ int4 fetch_td(const GemmArgs& a, int u, int m_tiles, int ntot) {
  if (a.implicit_M > 0 || u >= ntot) return make_int4(0, 0, 0, 0);
  return a.tiles[u / m_tiles];
}

// The CTA's tile-list entries, read two tiles ahead.
struct TileStream {
  int4 td0, td1;
  __device__ __forceinline__ void start(const GemmArgs& a, int m_tiles, int ntot) {
    td0 = fetch_td(a, blockIdx.x, m_tiles, ntot);
    td1 = fetch_td(a, blockIdx.x + gridDim.x, m_tiles, ntot);
  }
  // Entry of tile u (the loop's current tile); queues the one two tiles on.
  __device__ __forceinline__ int4 next(const GemmArgs& a, int u, int m_tiles, int ntot) {
    const int4 td = td0;
    td0 = td1;
    td1 = fetch_td(a, u + 2 * gridDim.x, m_tiles, ntot);
    return td;
  }
};

// Tile u: token tile u / m_tiles, weight-row tile u % m_tiles (consecutive
// CTAs share a token tile, so its activation rows are read from L2).  Returns
// false when that weight-row tile lies beyond the group's rows.
__device__ __forceinline__ bool tile_info(const GemmArgs& a, int u, int m_tiles, int4 td,
                                          TileInfo& ti) {
  const int gt = u / m_tiles;
  ti.m_tile = u - gt * m_tiles;
  if (a.implicit_M > 0) {
    ti.grp = 0;
    ti.start = gt * kBN;
    ti.count = min(kBN, a.implicit_M - gt * kBN);
  } else {
    ti.grp = td.x;
    ti.start = td.y;
    ti.count = td.z;
  }
  ti.N = (ti.count + 15) & ~15;
  ti.is_shared = ti.grp == a.shared_group;
  ti.Mrows = ti.is_shared ? a.Mrows_shared : a.Mrows;
  return ti.m_tile * (a.mode == 1 ? 64 : 128) < ti.Mrows;
}

// silu(x) = x * sigmoid(x), sigmoid composed as the reference does
// (x < 0 ? y : 1 - y with y = 1 / (1 + e^|x|)), with the fast exponential and
// division intrinsics (a few ulp; the tolerance is 5e-3 relative-L2).
__device__ __forceinline__ float silu_fast(float x) {
  const float y = __fdividef(1.0f, 1.0f + __expf(fabsf(x)));
  return x * (x < 0.0f ? y : 1.0f - y);
}

template <bool F16>
__global__ void __launch_bounds__(kGemmThreads, 1)
    nvfp4_gemm_kernel(const __grid_constant__ GemmArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // Swizzle atoms (TMA and UMMA) need 1024-byte alignment.
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sB = smem;
  uint8_t* sRaw = sB + kBSlabs * kSlabB;
  uint8_t* sOut = sRaw + kRawSlots * kRawSlot;  // [kBN][kOutPitch]
  uint64_t* a_full = reinterpret_cast<uint64_t*>(sOut + kBN * kOutPitch);
  uint64_t* a_empty = a_full + kASlabs;
  uint64_t* b_full = a_empty + kASlabs;
  uint64_t* b_empty = b_full + kBSlabs;
  uint64_t* raw_full = b_empty + kBSlabs;
  uint64_t* raw_empty = raw_full + kRawSlots;
  uint64_t* acc_full = raw_empty + kRawSlots;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* sc_full = acc_empty + 2;
  uint64_t* sc_empty = sc_full + 2;
  uint64_t* drain = sc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  float* s_scale = reinterpret_cast<float*>(tmem_slot + 4);  // [2][kBN] per-column scales

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kASlabs; i++) {
      mbar_init(&a_full[i], kDeqWarps);    // every dequantiser warp
      mbar_init(&a_empty[i], 1);           // MMA commit
    }
    for (int i = 0; i < kBSlabs; i++) {
      mbar_init(&b_full[i], 1);            // activation TMA (with tx)
      mbar_init(&b_empty[i], 1);           // MMA commit
    }
    for (int i = 0; i < kRawSlots; i++) {
      mbar_init(&raw_full[i], 1);          // weight TMA (with tx)
      mbar_init(&raw_empty[i], kDeqWarps);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&acc_full[i], 1);          // MMA commit at the end of a tile
      mbar_init(&acc_empty[i], kEpiWarps);
      mbar_init(&sc_full[i], 1);           // activation warp: the tile's column scales
      mbar_init(&sc_empty[i], kEpiWarps);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == kWarpRaw && lane == 0) {
    prefetch_map(&a.mc0);
    prefetch_map(&a.ms0);
  }
  // Tiles, slot maps and activations come from preceding kernels.
  pdl_wait();
  pdl_trigger();
  const int m_tiles = a.mode == 1 ? (max(a.Mrows, a.Mrows_shared) + 63) / 64
                                  : (max(a.Mrows, a.Mrows_shared) + 127) / 128;
  const int ntot = total_tiles(a, m_tiles);
  if ((int)blockIdx.x >= ntot) return;  // uniform per CTA, before any barrier use
  if (warp == kWarpMma) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nslab = a.K / kSlabK;

  if (warp == kWarpMma) {
    // ------------------------------ MMA issuer ------------------------------
    uint32_t elected;
    asm volatile("{\n.reg .pred p;\nelect.sync _|p, 0xffffffff;\nselp.u32 %0, 1, 0, p;\n}\n" : "=r"(elected));
    {
      uint32_t g = 0;
      int j = 0;
      bool ok = true;
      TileStream ts;
      ts.start(a, m_tiles, ntot);
      for (int u = blockIdx.x; u < ntot && ok; u += gridDim.x) {
        TileInfo ti;
        if (!tile_info(a, u, m_tiles, ts.next(a, u, m_tiles, ntot), ti)) continue;
        const int buf = j & 1;
        if (j >= 2 && !mbar_wait_bounded(&acc_empty[buf], ((j >> 1) - 1) & 1)) {
          if (elected) flag(kErrTimeout);
          break;
        }
        tc_fence_after();
        const uint32_t idesc =
            idesc_f16_f32(kBM, ti.N) | (F16 ? 0u : ((1u << 7) | (1u << 10)));
        const uint32_t d = tmem + (uint32_t)(buf * kBN);
        for (int sl = 0; sl < nslab; sl++, g++) {
          const int as = g % kASlabs, bs = g % kBSlabs;
          if (!mbar_wait_bounded(&a_full[as], (g / kASlabs) & 1) ||
              !mbar_wait_bounded(&b_full[bs], (g / kBSlabs) & 1)) {
            if (elected) flag(kErrTimeout);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ta = tmem + (uint32_t)(kAccCols + as * kASlabCols);
          const uint64_t bd = smem_desc_sw128(smem_u32(sB + bs * kSlabB));
          if (elected) {
#pragma unroll
          for (int s = 0; s < kStages; s++)
#pragma unroll
            for (int ks = 0; ks < kBK / 16; ks++)  // 16 K: 8 TMEM columns of A, 32 bytes of B
              umma_f16_ts(d, ta + s * kACols + 8 * ks, bd + s * (kStageB >> 4) + 2 * ks, idesc,
                          (sl | s | ks) != 0);
          umma_commit(&a_empty[as]);
          umma_commit(&b_empty[bs]);
          }
          __syncwarp();
        }
        if (!ok) break;
        if (elected) umma_commit(&acc_full[buf]);
        __syncwarp();
        j++;
      }
      if (elected) umma_commit(drain);
      __syncwarp();
      if (!mbar_wait_bounded(drain, 0) && elected) flag(kErrTimeout);
    }
    __syncwarp();
  } else if (warp == kWarpRaw) {
    // ------------------------------ weight TMA ------------------------------
    uint32_t elected;
    asm volatile("{\n.reg .pred p;\nelect.sync _|p, 0xffffffff;\nselp.u32 %0, 1, 0, p;\n}\n" : "=r"(elected));
    {
      uint32_t g = 0;
      bool ok = true;
      TileStream ts;
      ts.start(a, m_tiles, ntot);
      for (int u = blockIdx.x; u < ntot && ok; u += gridDim.x) {
        TileInfo ti;
        if (!tile_info(a, u, m_tiles, ts.next(a, u, m_tiles, ntot), ti)) continue;
        const CUtensorMap* c0 = ti.is_shared ? &a.mcs0 : &a.mc0;
        const CUtensorMap* s0 = ti.is_shared ? &a.mss0 : &a.ms0;
        const CUtensorMap* c1 = ti.is_shared ? &a.mcs1 : &a.mc1;
        const CUtensorMap* s1 = ti.is_shared ? &a.mss1 : &a.ms1;
        const int row0 =
            (ti.is_shared ? 0 : ti.grp * a.Mrows) + ti.m_tile * (a.mode == 1 ? 64 : 128);
        for (int sl = 0; sl < nslab; sl++, g++) {
          const int r = g % kRawSlots;
          if (g >= kRawSlots &&
              !mbar_wait_bounded(&raw_empty[r], ((g / kRawSlots) - 1) & 1)) {
            if (elected) flag(kErrTimeout);
            ok = false;
            break;
          }
          uint8_t* slot = sRaw + r * kRawSlot;
          if (!elected) continue;
          mbar_arrive_expect_tx(&raw_full[r], kRawSlot);
          if (a.mode == 1) {
            tma_load_2d(slot, c0, sl * 128, row0, &raw_full[r]);
            tma_load_2d(slot + kRawCodes / 2, c1, sl * 128, row0, &raw_full[r]);
            tma_load_2d(slot + kRawCodes, s0, sl * 16, row0, &raw_full[r]);
            tma_load_2d(slot + kRawCodes + 64 * 16, s1, sl * 16, row0, &raw_full[r]);
          } else {
            tma_load_2d(slot, c0, sl * 128, row0, &raw_full[r]);
            tma_load_2d(slot + kRawCodes, s0, sl * 16, row0, &raw_full[r]);
          }
        }
      }
      // No copy may still be in flight when the CTA exits (immediate unless a
      // wait above gave up).
      for (uint32_t i = 0; i < min(g, (uint32_t)kRawSlots); i++) {
        const uint32_t gg = g - 1 - i;
        mbar_wait_bounded(&raw_full[gg % kRawSlots], (gg / kRawSlots) & 1, kDrainBudget);
      }
    }
    __syncwarp();
  } else if (warp == kWarpAct) {
    // ---------------------------- activation TMA ----------------------------
    // Lane 0 issues the B slabs; with pre-scaled rows the whole warp also
    // stages the tile's per-column scales (read one tile ahead) for the
    // epilogue.
    uint32_t g = 0;
    int j = 0;
    bool ok = true;
    TileStream ts;
    ts.start(a, m_tiles, ntot);
    float sc_next[2] = {1.0f, 1.0f};
    auto load_scales = [&](int4 td, int u, float (&dst)[2]) {
      TileInfo tn;
      const bool valid = u < ntot && tile_info(a, u, m_tiles, td, tn);
#pragma unroll
      for (int h2 = 0; h2 < 2; h2++) {
        const int n = 32 * h2 + lane;
        dst[h2] = (a.bscale && valid && n < tn.count) ? a.bscale[tn.start + n] : 1.0f;
      }
    };
    load_scales(ts.td0, blockIdx.x, sc_next);
    for (int u = blockIdx.x; u < ntot && ok; u += gridDim.x) {
      const int4 td = ts.next(a, u, m_tiles, ntot);
      const float sc_cur[2] = {sc_next[0], sc_next[1]};
      load_scales(ts.td0, u + gridDim.x, sc_next);
      TileInfo ti;
      if (!tile_info(a, u, m_tiles, td, ti)) continue;
      const int sb = j & 1;
      if (j >= 2 && !mbar_wait_bounded(&sc_empty[sb], ((j >> 1) - 1) & 1)) {
        if (lane == 0) flag(kErrTimeout);
        break;
      }
      s_scale[sb * kBN + lane] = sc_cur[0];
      s_scale[sb * kBN + 32 + lane] = sc_cur[1];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sc_full[sb]);
      j++;
      {
        const int nbox = ti.N / 16;
        for (int sl = 0; sl < nslab; sl++, g++) {
          const int bs = g % kBSlabs;
          if (g >= kBSlabs && !mbar_wait_bounded(&b_empty[bs], ((g / kBSlabs) - 1) & 1)) {
            if (lane == 0) flag(kErrTimeout);
            ok = false;
            break;
          }
          if (lane != 0) continue;
          mbar_arrive_expect_tx(&b_full[bs], kStages * nbox * kBoxB);
          for (int s = 0; s < kStages; s++)
            for (int b = 0; b < nbox; b++)
              tma_load_2d(sB + bs * kSlabB + s * kStageB + b * kBoxB, &a.mb,
                          (sl * kStages + s) * kBK, ti.start + 16 * b, &b_full[bs]);
        }
        __syncwarp();
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    {
      for (uint32_t i = 0; i < min(g, (uint32_t)kBSlabs); i++) {
        const uint32_t gg = g - 1 - i;
        mbar_wait_bounded(&b_full[gg % kBSlabs], (gg / kBSlabs) & 1, kDrainBudget);
      }
    }
    __syncwarp();
  } else if (warp < kWarpEpi0) {
    // ------------------------------ dequantisers ------------------------------
    // Group q, thread -> tile row r = the TMEM lane this warp may write; slab
    // row sr holds tile row r (mode 1: tile rows [16b, 16b+8) are gate rows
    // 8b.., [16b+8, 16b+16) the same up rows, and the slab has gate rows 0..63
    // then up rows 64..127).  Eight consecutive rows read eight distinct
    // 16-byte bank groups of the swizzled slab.
    const int q = (warp - kWarpDeq0) / kGroupWarps;
    const int r = 32 * (warp & 3) + lane;
    const int sr = a.mode == 1 ? (((r >> 3) & 1) * 64 + (r >> 4) * 8 + (r & 7)) : r;
    const int sw_sr = sr & 7;
    const uint32_t ta = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(kAccCols + q * kACols);
    uint32_t g = 0;
    bool ok = true;
    TileStream ts;
    ts.start(a, m_tiles, ntot);
    for (int u = blockIdx.x; u < ntot && ok; u += gridDim.x) {
      TileInfo ti;
      if (!tile_info(a, u, m_tiles, ts.next(a, u, m_tiles, ntot), ti)) continue;
      for (int sl = 0; sl < nslab; sl++, g++) {
        const int rs = g % kRawSlots;
        if (!mbar_wait_bounded(&raw_full[rs], (g / kRawSlots) & 1)) {
          flag(kErrTimeout);
          ok = false;
          break;
        }
        const uint8_t* slot = sRaw + rs * kRawSlot;
        const uint4 cw0 =
            *reinterpret_cast<const uint4*>(slot + sr * 128 + (((2 * q) ^ sw_sr) << 4));
        const uint4 cw1 =
            *reinterpret_cast<const uint4*>(slot + sr * 128 + (((2 * q + 1) ^ sw_sr) << 4));
        const uint32_t sc4 = *reinterpret_cast<const uint32_t*>(slot + kRawCodes + sr * 16 + q * 4);
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[rs]);
        const uint32_t S01 = scale2_to_f16x2(sc4 & 0xFFFFu), S23 = scale2_to_f16x2(sc4 >> 16);
        const uint32_t sc[4] = {bcast_lo(S01), bcast_hi(S01), bcast_lo(S23), bcast_hi(S23)};
        const uint32_t wds[8] = {cw0.x, cw0.y, cw0.z, cw0.w, cw1.x, cw1.y, cw1.z, cw1.w};
        uint32_t o[32];  // column c = K elements 2c, 2c+1 of the stage
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const uint4 v = F16 ? dequant8_f16(wds[j], sc[j >> 1]) : dequant8_bf16(wds[j], sc[j >> 1]);
          o[4 * j] = v.x;
          o[4 * j + 1] = v.y;
          o[4 * j + 2] = v.z;
          o[4 * j + 3] = v.w;
        }
        // Warp-uniform: tcgen05.st below is .sync.aligned.
        const int as = g % kASlabs;
        if (g >= kASlabs &&
            !__all_sync(0xffffffffu, mbar_wait_bounded(&a_empty[as], ((g / kASlabs) - 1) & 1))) {
          if (lane == 0) flag(kErrTimeout);
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_st32(ta + as * kASlabCols, o);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[as]);
      }
    }
  } else {
    // ------------------------------ epilogue --------------------------------
    const int sp = warp & 3;       // TMEM sub-partition this warp may read
    const int r = sp * 32 + lane;  // tile row = TMEM lane
    int j = 0;
    TileStream ts;
    ts.start(a, m_tiles, ntot);
    for (int u = blockIdx.x; u < ntot; u += gridDim.x) {
      TileInfo ti;
      if (!tile_info(a, u, m_tiles, ts.next(a, u, m_tiles, ntot), ti)) continue;
      const int buf = j & 1;
      // Warp-uniform decision: the TMEM loads below are .sync.aligned.
      const bool have =
          __all_sync(0xffffffffu, mbar_wait_bounded(&sc_full[buf], (j >> 1) & 1) &&
                                      mbar_wait_bounded(&acc_full[buf], (j >> 1) & 1));
      if (!have) {
        if (lane == 0) flag(kErrTimeout);
        break;
      }
      tc_fence_after();
      // Per-column scales, one column per lane, broadcast by shuffle.
      const float cs_l[2] = {s_scale[buf * kBN + lane], s_scale[buf * kBN + 32 + lane]};
      __syncwarp();
      if (lane == 0) mbar_arrive(&sc_empty[buf]);
      // The whole accumulator (N <= 64 columns) into registers; TMEM is then
      // handed back to the MMA before any output work.
      uint32_t v[2][32];
      const uint32_t taddr = tmem + ((uint32_t)(sp * 32) << 16) + (uint32_t)(buf * kBN);
      tmem_ld32_nowait(taddr, v[0]);
      if (ti.N > 32) tmem_ld32_nowait(taddr + 32, v[1]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      // Staging buffer free: every epilogue thread has copied out the
      // previous tile.
      named_sync(1, 32 * kEpiWarps);
#pragma unroll
      for (int h2 = 0; h2 < 2; h2++) {
        if (h2 == 1 && ti.N <= 32) break;  // warp-uniform
#pragma unroll
        for (int q = 0; q < 32; q++) {
          const int n = 32 * h2 + q;
          const float val = __uint_as_float(v[h2][q]) * __shfl_sync(0xffffffffu, cs_l[h2], q);
          uint8_t* row = sOut + n * kOutPitch;
          if (a.mode == 1) {
            const float other = __shfl_xor_sync(0xffffffffu, val, 8);
            if (!(r & 8))
              reinterpret_cast<float*>(row)[(r >> 4) * 8 + (r & 7)] = silu_fast(val) * other;
          } else if (a.mode == 2 || a.out_dtype == kF32) {
            reinterpret_cast<float*>(row)[r] = val;
          } else if (a.out_dtype == kBF16) {
            reinterpret_cast<__nv_bfloat16*>(row)[r] = __float2bfloat16_rn(val);
          } else {
            reinterpret_cast<__half*>(row)[r] = __float2half_rn(val);
          }
        }
      }
      const int esz = (a.mode != 0 || a.out_dtype == kF32) ? 4 : 2;
      const int row_elems = a.mode == 1 ? 64 : 128;
      const int64_t col0 = (int64_t)ti.m_tile * row_elems;
      const int et = threadIdx.x - 32 * kWarpEpi0;
      if (a.out_vec) {
        // Coalesced 16-byte copies of the staged rows (the TMA queue stays
        // with the operand loads).
        named_sync(1, 32 * kEpiWarps);
        const int chunks = row_elems * esz / 16;
        for (int idx = et; idx < ti.count * chunks; idx += 32 * kEpiWarps) {
          const int n = idx / chunks, c = idx - n * chunks;
          const uint4 v4 = *reinterpret_cast<const uint4*>(sOut + n * kOutPitch + c * 16);
          *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(a.out) +
                                    ((int64_t)(ti.start + n) * a.out_ld + col0) * esz + c * 16) = v4;
        }
      } else {
        named_sync(1, 32 * kEpiWarps);
        const int64_t rows_left = ti.Mrows - col0;
        const int ncol = rows_left < row_elems ? (int)rows_left : row_elems;
        for (int idx = et; idx < ti.count * row_elems; idx += 32 * kEpiWarps) {
          const int n = idx / row_elems, c = idx - n * row_elems;
          if (c >= ncol) continue;
          const uint8_t* src = sOut + n * kOutPitch + c * esz;
          uint8_t* dst = reinterpret_cast<uint8_t*>(a.out) +
                         ((int64_t)(ti.start + n) * a.out_ld + col0 + c) * esz;
          if (esz == 4) *reinterpret_cast<float*>(dst) = *reinterpret_cast<const float*>(src);
          else *reinterpret_cast<uint16_t*>(dst) = *reinterpret_cast<const uint16_t*>(src);
        }
      }
      j++;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kWarpMma) tmem_dealloc(tmem, kTmemCols);
}

// ---------------------------------------------------------------------------
// Activation rows -> f16(v * 2^-e) with max |v| * 2^-e in [1, 2) per row, and
// 2^e in scale[row] (exact for bf16 inputs; no input overflows f16).  dst row r
// reads src row src_map[r] (the expert-sorted slot order).  One warp per row;
// K a multiple of 8.
__global__ void rows_to_f16_kernel(RowsArgs a) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int r = warp; r < a.rows; r += nwarps) {
    const int64_t src = (int64_t)(a.src_map ? a.src_map[r] : r) * a.src_ld;
    float m = 0.f;
    for (int k = lane * 8; k < a.K; k += 256) {
      float f[8];
      load8(a.src, a.src_dtype, src + k, f);
#pragma unroll
      for (int i = 0; i < 8; i++) m = fmaxf(m, fabsf(f[i]));
    }
    m = warp_max(m);
    const int e = pow2_exponent(m);
    const float inv = ldexpf(1.0f, -e);
    for (int k = lane * 8; k < a.K; k += 256) {
      float f[8];
      load8(a.src, a.src_dtype, src + k, f);
      uint32_t hv[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const __half2 v = __floats2half2_rn(f[2 * i] * inv, f[2 * i + 1] * inv);
        hv[i] = *reinterpret_cast<const uint32_t*>(&v);
      }
      *reinterpret_cast<uint4*>(a.dst + (int64_t)r * a.dst_ld + k) =
          make_uint4(hv[0], hv[1], hv[2], hv[3]);
    }
    if (lane == 0) a.scale[r] = ldexpf(1.0f, e);
  }
}

// ---------------------------------------------------------------------------
// Sort (token, slot) pairs by expert (counting sort, SwitchLayers.swift:385-420
// gatherSort) and cut each expert's run into tiles of <= 64 tokens.  One CTA.
// Outputs: brow[slot] = token of the pair in sorted slot `slot`;
// pos[pair] = slot (the inverse permutation scatterUnsort applies);
// tiles[] = (expert, first slot, count); the shared expert, when present, is
// group E with slots P..P+T-1 = tokens 0..T-1.  Slot order inside an expert
// is the atomic arrival order; no output depends on it (every pair's row is
// computed independently and the combine reads by `pos`).
__global__ void __launch_bounds__(1024) moe_sort_kernel(SortArgs a) {
  __shared__ int cnt[1024];
  __shared__ int off[1024];
  __shared__ int toff[1025];
  __shared__ int wsum[32], wtsum[32];
  pdl_wait();
  pdl_trigger();
  const int E = a.E;
  const int tb = a.tile_tokens > 0 ? a.tile_tokens : kBN;  // tokens per tile
  const int P = a.P;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    const uint32_t e = a.inds[p] - (uint32_t)a.e_base;
    if (e < (uint32_t)E) atomicAdd(&cnt[e], 1);
    else if (!a.skip_foreign) flag(5);
  }
  __syncthreads();
  // Exclusive prefix sums over the experts (E <= 1024 = blockDim.x) of the
  // pair counts and of the tile counts: warp scans, then a scan of the warp
  // totals.
  {
    const int e = threadIdx.x;
    const int c = e < E ? cnt[e] : 0;
    const int tc = (c + tb - 1) / tb;
    int sc = c, st = tc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int vc = __shfl_up_sync(0xffffffffu, sc, o);
      const int vt = __shfl_up_sync(0xffffffffu, st, o);
      if (lane >= o) {
        sc += vc;
        st += vt;
      }
    }
    if (lane == 31) {
      wsum[warp] = sc;
      wtsum[warp] = st;
    }
    __syncthreads();
    if (warp == 0) {
      int wc = wsum[lane], wt = wtsum[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int vc = __shfl_up_sync(0xffffffffu, wc, o);
        const int vt = __shfl_up_sync(0xffffffffu, wt, o);
        if (lane >= o) {
          wc += vc;
          wt += vt;
        }
      }
      wsum[lane] = wc - wsum[lane];    // exclusive over warps
      wtsum[lane] = wt - wtsum[lane];
    }
    __syncthreads();
    if (e < E) {
      off[e] = wsum[warp] + sc - c;
      toff[e] = wtsum[warp] + st - tc;
      if (e == E - 1) {
        const int tacc = toff[e] + tc;
        toff[E] = tacc;
        const int shn = a.sh_rows > 0 ? a.sh_rows : a.T;
        const int tsh = a.with_shared ? (shn + tb - 1) / tb : 0;
        *a.ntiles = tacc + tsh;
      }
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int n = cnt[e];
    for (int t = 0; t * tb < n; t++)
      a.tiles[toff[e] + t] = make_int4(e, off[e] + t * tb, min(tb, n - t * tb), 0);
    cnt[e] = 0;  // reused as the scatter cursor
  }
  if (a.with_shared) {
    const int shn = a.sh_rows > 0 ? a.sh_rows : a.T;
    for (int t = threadIdx.x; t * tb < shn; t += blockDim.x)
      a.tiles[toff[E] + t] = make_int4(E, P + t * tb, min(tb, shn - t * tb), 0);
    for (int t = threadIdx.x; t < shn; t += blockDim.x) a.brow[P + t] = a.sh_row0 + t;
  }
  __syncthreads();
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    const uint32_t e = a.inds[p] - (uint32_t)a.e_base;
    if (e >= (uint32_t)E) {
      a.pos[p] = -1;
      continue;
    }
    const int slot = off[e] + atomicAdd(&cnt[e], 1);
    a.brow[slot] = p / a.k;
    a.pos[p] = slot;
  }
}

// y[t] = scaling * sum_j w[t][j] * Y[pos[t*k+j]] + Y[P + t] (shared) + residual
// in a fixed j order (deterministic).  Each thread owns 8 consecutive h of one
// token (H a multiple of 8): two 16-byte loads per expert row, one store.
__global__ void moe_combine_kernel(CombineArgs a) {
  pdl_wait();
  pdl_trigger();
  const int H8 = a.H / 8;
  const int64_t total = (int64_t)a.T * H8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / H8, h = (i - t * H8) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < a.k; j++) {
      const int slot = a.pos[t * a.k + j];
      if (slot < 0) continue;
      const float w = a.wts[t * a.k + j];
      const float4* src = reinterpret_cast<const float4*>(a.Y + (int64_t)slot * a.H + h);
      const float4 u = src[0], v = src[1];
      acc[0] += w * u.x; acc[1] += w * u.y; acc[2] += w * u.z; acc[3] += w * u.w;
      acc[4] += w * v.x; acc[5] += w * v.y; acc[6] += w * v.z; acc[7] += w * v.w;
    }
#pragma unroll
    for (int q = 0; q < 8; q++) acc[q] *= a.scaling;
    const int64_t ts = t - a.sh_row0;
    if (a.with_shared && ts >= 0 && ts < (a.sh_rows > 0 ? a.sh_rows : a.T)) {
      const float4* src = reinterpret_cast<const float4*>(a.Y + (int64_t)(a.P + ts) * a.H + h);
      const float4 u = src[0], v = src[1];
      acc[0] += u.x; acc[1] += u.y; acc[2] += u.z; acc[3] += u.w;
      acc[4] += v.x; acc[5] += v.y; acc[6] += v.z; acc[7] += v.w;
    }
    const int64_t off = t * a.H + h;
    if (a.residual) {
      float r[8];
      load8(a.residual, a.dtype, off, r);
#pragma unroll
      for (int q = 0; q < 8; q++) acc[q] += r[q];
    }
    store8_from_f32(a.y, a.dtype, off, acc);
  }
}

template <typename Kern, typename Args>
cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       bool pdl, const Args& args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

int gemm_sm_count() {
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

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

cudaError_t encode_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner,
                      uint64_t rows, uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows,
                      CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15) || rows == 0 || inner == 0)
    return cudaErrorInvalidValue;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace

cudaError_t map_codes(CUtensorMap* m, const void* w, int64_t rows, int64_t K, int box_rows) {
  return encode_2d(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, (uint64_t)K / 2, (uint64_t)rows,
                   (uint64_t)K / 2, 128, (uint32_t)box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

cudaError_t map_codes_k64(CUtensorMap* m, const void* w, int64_t rows, int64_t K, int box_rows) {
  return encode_2d(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, (uint64_t)K / 2, (uint64_t)rows,
                   (uint64_t)K / 2, 32, (uint32_t)box_rows, CU_TENSOR_MAP_SWIZZLE_32B);
}

cudaError_t map_scales(CUtensorMap* m, const void* s, int64_t rows, int64_t K, int box_rows) {
  return encode_2d(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, s, (uint64_t)K / 16, (uint64_t)rows,
                   (uint64_t)K / 16, 16, (uint32_t)box_rows, CU_TENSOR_MAP_SWIZZLE_NONE);
}

cudaError_t map_rows16(CUtensorMap* m, const void* b, bool bf16, int64_t rows, int64_t K,
                       int64_t ld) {
  return encode_2d(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   b, (uint64_t)K, (uint64_t)rows, (uint64_t)ld * 2, kBK, 16,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

size_t gemm_smem_bytes() {
  return 1024 + (size_t)kBSlabs * kSlabB + (size_t)kRawSlots * kRawSlot + (size_t)kBN * kOutPitch +
         (2 * kASlabs + 2 * kBSlabs + 2 * kRawSlots + 9) * 8 + 16 + 2 * kBN * sizeof(float);
}

int gemm_tile_tokens() { return kBN; }
int gemm_slab_k() { return kSlabK; }

// f16: the activation map holds f16 rows (A is dequantised to f16), else bf16.
cudaError_t launch_nvfp4_gemm(const GemmArgs& a, bool f16, int max_tiles, cudaStream_t stream,
                              bool pdl) {
  if (max_tiles <= 0) return cudaSuccess;
  if (a.K % kSlabK) return cudaErrorInvalidValue;
  const size_t smem = gemm_smem_bytes();
  auto kern = f16 ? nvfp4_gemm_kernel<true> : nvfp4_gemm_kernel<false>;
  // 16-byte output copies need 16-byte aligned rows and only whole row tiles.
  GemmArgs args = a;
  const int esz = (a.mode != 0 || a.out_dtype == kF32) ? 4 : 2;
  const int tile_rows = a.mode == 1 ? 64 : 128;
  args.out_vec = (reinterpret_cast<uintptr_t>(a.out) % 16 == 0) && (a.out_ld * esz) % 16 == 0 &&
                  a.Mrows % tile_rows == 0 && a.Mrows_shared % tile_rows == 0;
  cudaError_t e = ensure_smem(kern, smem);
  if (e != cudaSuccess) return e;
  const int mrows = std::max(a.Mrows, a.Mrows_shared);
  const int m_tiles = a.mode == 1 ? (mrows + 63) / 64 : (mrows + 127) / 128;
  const int64_t upper = (int64_t)m_tiles * max_tiles;
  const int grid = (int)std::min<int64_t>(upper, gemm_sm_count());
  return launch_pdl(kern, dim3(grid), dim3(kGemmThreads), smem, stream, pdl, args);
}

cudaError_t launch_rows_to_f16(const RowsArgs& a, cudaStream_t stream, bool pdl) {
  if (a.rows <= 0) return cudaSuccess;
  const int threads = 256;
  const int blocks = std::min(std::max(1, (a.rows + 7) / 8), gemm_sm_count() * 8);
  return launch_pdl(rows_to_f16_kernel, dim3(blocks), dim3(threads), 0, stream, pdl, a);
}

cudaError_t launch_moe_sort(const SortArgs& a, cudaStream_t stream, bool pdl) {
  return launch_pdl(moe_sort_kernel, dim3(1), dim3(1024), 0, stream, pdl, a);
}

cudaError_t launch_moe_combine(const CombineArgs& a, cudaStream_t stream, bool pdl) {
  const int64_t total = (int64_t)a.T * (a.H / 8);
  const int threads = 256;
  const int blocks = (int)std::min<int64_t>((total + threads - 1) / threads, 148 * 16);
  return launch_pdl(moe_combine_kernel, dim3(blocks), dim3(threads), 0, stream, pdl, a);
}

cudaError_t read_and_clear_prefill_error(int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_prefill_error, sizeof(int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_prefill_error, &zero, sizeof(int));
}

}  // namespace nvfp4
