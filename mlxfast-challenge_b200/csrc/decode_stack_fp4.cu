// decode_stack_fp4.cu -- serial decode (T = 1) through a stack of sparse MoE
// layers on the block-scaled FP4 tensor cores, as ONE persistent cooperative
// launch (or one per 40 layers).
//
// Reference semantics: as decode_stack.cu -- per layer the routed SwitchGLU
// gate/up -> SwiGLU -> down chain with given routing (VLM/MLXLMCommon/
// SwitchLayers.swift:532-580) and the Laguna combine y = scaling * sum_j w_j *
// expert_j(x) + shared(x) (VLM/MLXLLM/Models/Laguna.swift:204-212), the layer
// loop being the runtime's decode step over its sparse layers
// (Sources/MLXFastModel/LagunaRuntimeModel.swift:11460 -> :11030 -> :10678);
// each layer's output rounded to the activation dtype.
//
// The products run as tcgen05.mma kind::mxf4nvf4 (M = 128 weight rows, N = 16,
// K = 64): the weight operand is the checkpoint's E2M1 codes and E4M3 group
// scales as stored; the activation row is carried, as in prefill_fp4.cu, as
// four NVFP4 terms (term t = the NVFP4 quantisation of the residual after
// terms 0..t-1 under a power-of-two factor per term, UE4M3 scales rounded up,
// codes rounded to nearest even by the hardware converter), B rows 0..3;
// rows 4..15 are zero.  Sums are f32.
//
// Why: at T = 1 the mma.sync stack spends most of each layer on the CUDA
// cores, converting E2M1 pairs and multiplying group scales into every weight
// element; here the tensor core consumes codes and scales directly and a layer
// is two short dependent chains.
//
// Work of one layer over G CTAs (CTA c takes item c of each list):
//   gate/up item (segment, 64-row block b of I, K part p of nks): A = the 64
//     gate rows of block b and the same 64 up rows over K part p; B = the
//     x terms of part p.  The part is four runs (one per chain warp), each
//     decomposed with its own term factors and summed in its own TMEM
//     accumulator.  Epilogue: sum_run sum_t fac * D_run[:, t]
//     -> GUp[p][seg][gate|up][i].
//   down item (segment, 128-row block of H): A = 128 down rows over all of I;
//     B = the terms of act = silu(sum_p gate) * (sum_p up), four runs as
//     above.  Epilogue: the same fold * w_seg * scaling (1 for the shared
//     expert) -> Yp[seg][h]; the next layer's x is sum_seg Yp[seg] in segment
//     order, rounded to the activation dtype.
// Every partial has its own slot and is summed in a fixed order: results are
// the same on every run.  No grid-wide barrier: a down item waits for the
// gate/up items of its segment, a gate/up item for the previous layer's down
// items of its K part (release/acquire counters).  GUp and Yp alternate
// between two buffers by layer parity: a buffer is rewritten two layers later,
// after (through those waits) every reader of its previous contents.
//
// Routed stack (ROUTED, BASELINE config[2] at one sequence): the router runs
// inside the launch, per layer -- the Laguna gate (Laguna.swift:149-181) on
// the layer's input, then the experts it picks -- with, optionally, the
// decoder layer's residual stream and RMSNorm around the block
// (Laguna.swift:242-246: h_{l+1} = h_l + block_l(RMSNorm_l(h_l))).  Only the
// shared expert's weights can stream ahead of the chain; a routed expert's
// slabs go out the moment its layer's top-k is known.
//   Items: CTA pairs (clusters of 2).  The pair of (segment, I block b)
// computes gate/up over its two K halves (one per CTA), swaps the partials
// through distributed shared memory (remote stores and a remote mbarrier
// arrival), and each CTA computes the down projection of the block's 64 act
// values for its half of H: row tiles of 128 rows x K 64 (32-byte rows,
// 32-byte swizzle), one MMA each.  A row of the layer output is then the sum
// of kk * I / 64 partials.
//   Reducers (CTA j < H / 32, 32 rows each): with the norm, every down item
// adds its partials to one counted 64-bit fixed-point word per row (2^-24
// units, with an add count: integer sums do not depend on the order of the
// adds, so every run gives the same bits) and the reducer polls the word until
// it is complete; without the norm, f32 partials per (segment, I block)
// behind per-row-block counters, summed in a fixed order.  The reducer adds
// the residual h_l and rounds to the activation dtype -- h_{l+1} for its rows
// -- and, with the norm, publishes the rows' f32 sum of squares as its tagged
// word of the layer, reads every reducer's word and sums them in reducer order
// (the same bits on every reducer), and forms x = dtype(dtype(h * rsqrt(mean +
// eps)) * w), the reference's RMSNorm fallback (mlx/fast.cpp:90-108); x goes
// out as tagged words (the gate/up items' input); then it adds x[rows] .
// G[e, rows] for every expert e into the expert's counted logit sum (2^-28
// units).  The reducers' router rows are prefetched two layers ahead with
// cp.async.
//   Router: the last CTA, all its warps, no item: waits for the counts,
// rounds each logit to the activation dtype as the reference's bf16 matmul
// does, selects the top-k (topk.cuh) and publishes the layer's routing line;
// every CTA with an item of the layer reads it.
//
// Roles (320 threads): warp 0 TMA (this CTA's weight slabs of layer l, l+1,
// ... in consumption order into a 10-stage ring -- 8 in the routed stack, one
// layer's slabs and two more -- so the next layer's weights stream while this
// layer's chain runs), warp 1 MMA issue, warps 2-5 weight
// scales into tensor memory, warps 6-9 the chain (terms, epilogues, the
// dependency counters).  Every wait is bounded; on expiry an error is latched
// (the site code below) and each role leaves its loop (the copies and MMAs it
// issued drained) before tensor memory is released.
#include "common.cuh"
#include "fp4terms.cuh"
#include "kernels.h"
#include "topk.cuh"
#include "umma.cuh"

namespace nvfp4 {
namespace {

constexpr int kT = kFp4Terms;
constexpr int kN = 16;                    // MMA N: term rows 0..3, rows 4..15 zero
constexpr int kStages = 10;               // ring stages (8 in the routed stack)
__host__ __device__ constexpr int stages(bool routed) { return routed ? 8 : kStages; }
constexpr int kA = 128 * 128;             // weight codes of one slab (128 rows x K 256): 16 KB
constexpr int kSA = 128 * 16;             // their scale bytes: 2 KB
constexpr int kStage = kA + kSA;          // 18 KB, 1 KB multiple
static_assert(kStage % 1024 == 0, "stage alignment");
constexpr int kBSlab = kN * 128;          // term codes of one K slab: 2 KB
constexpr int kThreads = 320;
constexpr int kWarpTma = 0, kWarpMma = 1, kWarpChain0 = 6;  // warps 2-5: weight scales
constexpr int kChain = 128;
constexpr int kBarChain = 1;              // named barrier of the chain warps
// Tensor memory: gate/up accumulators (one per chain warp's K run, 16 columns
// each), down accumulators (given routing: one per run; routed stack: one per
// 128-row tile, up to 8), the weight scales of each ring stage, the x-term
// scales, the act-term scales.
constexpr uint32_t kAccGU = 0, kAccD = 64, kSfaCols = 16;
__host__ __device__ constexpr uint32_t sfa0_of(bool routed) { return routed ? 192u : 128u; }
__host__ __device__ constexpr uint32_t sfbx_of(bool routed) {
  return sfa0_of(routed) + (uint32_t)stages(routed) * kSfaCols;
}
constexpr uint32_t kTmemCols = 512;
// Routed stack down stage: up to 3 row tiles of 128 rows x K 64 (an I block):
// codes 4 KB each (32-byte rows, 32-byte swizzle) at 4 KB * j, then their
// scale bytes (16 per row, the four K steps around the block) at 12 KB + 2 KB * j.
constexpr int kRTileCodes = 128 * 32, kRTileScales = 128 * 16, kRTilesPerStage = 3;
constexpr int kRScales0 = kRTilesPerStage * kRTileCodes;
static_assert(kRScales0 + kRTilesPerStage * kRTileScales <= kStage, "routed down stage");
constexpr int kErrIndex = 2;
// A wait that expired latches 1000 * (layer in the launch + 1) + site, site:
// 41 TMA ring slot, 42 MMA x terms, 43 MMA gate/up stage, 44 MMA act terms,
// 45 MMA down stage, 46 MMA drain, 47 scale warps stage, 48 chain gate/up
// accumulator, 49 chain down accumulator, 50 a segment's gate/up items, 51 a
// K part's down items (previous layer), 52 the last layer's down items; routed
// stack: 53 the layer's router reducers, 54 a row block's down items (the
// reducer), 55 the TMA warp waiting for the layer's routing, 56 the reducers'
// sums of squares (the norm), 57 a gate/up item's tagged inputs; the routed
// stack's pairs: 50 the partner's gate/up partials.
__host__ __device__ constexpr int fs_timeout(int l, int site) { return 1000 * (l + 1) + site; }
constexpr long long kDrainBudget = 200000000LL;

__device__ int g_fs_error = 0;
__device__ __forceinline__ void fsflag(int code) { atomicCAS(&g_fs_error, 0, code); }

__device__ __forceinline__ uint32_t elect_one_fs() {
  uint32_t e;
  asm volatile("{\n.reg .pred p;\nelect.sync _|p, 0xffffffff;\nselp.u32 %0, 1, 0, p;\n}\n"
               : "=r"(e));
  return e;
}

__device__ __forceinline__ bool chain_sync_and(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n"
      ".reg .pred p, q;\n"
      "setp.ne.u32 p, %1, 0;\n"
      "bar.red.and.pred q, %2, %3, p;\n"
      "selp.u32 %0, 1, 0, q;\n"
      "}\n"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(kBarChain), "r"(kChain)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void red_release_add_fs(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_fs(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float round_to(float v, int dtype) {
  if (dtype == kBF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dtype == kF16) return __half2float(__float2half_rn(v));
  return v;
}

// Shared-memory carve-up (base 1024-byte aligned); also sizes it on the host.
struct FsSmem {
  uint8_t *stage, *bx, *ba, *scx, *sca;
  float *wmax, *facx, *faca;
  uint64_t *full, *empty, *sfr, *xready, *aready, *gufull, *dfull, *drain;
  uint32_t* tslot;
  int* bar_ok;
  volatile int* hold;  // refills wait (MMA start to the loads after the next barrier)
  volatile int* cur;   // the layer the chain is in: its stages are never held
  uint32_t* inds;
  float* wts;
  uint8_t* rsl;          // routed: [2][E <= 256][32] bf16, a reducer's router rows
  float* xs;             // routed: [32] the reducer's rows of x_{l+1}
  float* gux;            // routed: [2][128] the pair's gate/up partials (K part 0, 1)
  float* red;            // routed: [4][32] the reducer's quarter sums
  uint64_t* guready;     // routed: the partner's partials have landed in gux
  volatile int* rlayer;  // routed: layers whose routing is in inds / wts
};

__host__ __device__ inline size_t fs_carve(int H, int I, int L, bool routed, uint8_t* base,
                                           FsSmem* S) {
  const int ns = stages(routed);
  size_t o = 0;
  auto take = [&](size_t bytes, size_t align) -> uint8_t* {
    o = (o + align - 1) / align * align;
    uint8_t* p = base ? base + o : nullptr;
    o += bytes;
    return p;
  };
  FsSmem t{};
  t.stage = take((size_t)ns * kStage, 1024);
  t.bx = take((size_t)(H / 256) * kBSlab, 1024);  // bx and ba adjacent (zeroed together)
  t.ba = take((size_t)(I / 256) * kBSlab, 1024);
  t.scx = take((size_t)kT * (H / 16), 16);
  t.sca = take((size_t)kT * (I / 16), 16);
  t.wmax = reinterpret_cast<float*>(take(8 * 4, 16));
  t.facx = reinterpret_cast<float*>(take(16 * 4, 16));
  t.faca = reinterpret_cast<float*>(take(16 * 4, 16));
  t.full = reinterpret_cast<uint64_t*>(take(ns * 8, 8));
  t.empty = reinterpret_cast<uint64_t*>(take(ns * 8, 8));
  t.sfr = reinterpret_cast<uint64_t*>(take(ns * 8, 8));
  t.xready = reinterpret_cast<uint64_t*>(take(8, 8));
  t.aready = reinterpret_cast<uint64_t*>(take(8, 8));
  t.gufull = reinterpret_cast<uint64_t*>(take(8, 8));
  t.dfull = reinterpret_cast<uint64_t*>(take(8, 8));
  t.drain = reinterpret_cast<uint64_t*>(take(8, 8));
  t.tslot = reinterpret_cast<uint32_t*>(take(4, 4));
  t.bar_ok = reinterpret_cast<int*>(take(4, 4));
  t.hold = reinterpret_cast<volatile int*>(take(4, 4));
  t.cur = reinterpret_cast<volatile int*>(take(4, 4));
  t.inds = reinterpret_cast<uint32_t*>(take((size_t)L * 16 * 4, 16));
  t.wts = reinterpret_cast<float*>(take((size_t)L * 16 * 4, 16));
  if (routed) {
    t.rsl = take((size_t)2 * 256 * kFsRedRows * 2, 128);
    t.xs = reinterpret_cast<float*>(take(kFsRedRows * 4, 16));
    t.gux = reinterpret_cast<float*>(take(2 * 128 * 4, 16));
    t.red = reinterpret_cast<float*>(take(4 * 32 * 4, 16));
    t.guready = reinterpret_cast<uint64_t*>(take(8, 8));
    t.rlayer = reinterpret_cast<volatile int*>(take(4, 4));
  }
  if (S) *S = t;
  return o;
}

// 128 V values of the activation row (K positions kb .. kb + 128 V) as four
// NVFP4 terms, in the chain warps: thread ct holds the V values k0 = kb + ct *
// V .. k0 + V - 1 (a group of 16 spans 16 / V threads), so chain warp w holds
// the run of 32 V values from kb + 32 V w.  Each run is decomposed on its own
// (its own power-of-two factors: warp shuffles only; the MMAs keep one
// accumulator per run).  The run's max sets term 0's factor, which places its
// largest group scale in [171, 352]; term t's factor is 4^-t times that.  Per
// term: group max (shuffle), the group's UE4M3 scale, codes by the hardware
// converter into the B tile (row t, 128-byte swizzle), the residual updated
// with the values the codes stand for.  Writes the scale bytes sSc[t][group] (groups of the whole
// row, K / 16 per term) and the factors fac[4 w + t]; ends with a chain
// barrier.  Follows rows_to_terms_kernel (prefill_fp4.cu), over the run
// instead of the row and with the factor progression above instead of one
// max per term.
template <int V>
__device__ __forceinline__ void make_terms(float (&v)[V], int ct, int K, int kb, uint8_t* sB,
                                           uint8_t* sSc, float* fac) {
  static_assert(V == 2 || V == 4 || V == 8 || V == 16, "values per thread");
  constexpr int TPG = 16 / V;
  const int lane = ct & 31, cw = ct >> 5;
  const int k0 = kb + ct * V;
  const bool in = k0 < K;  // threads past the row (all zeros) store nothing
  const int grp = k0 / 16;
  const int byte0 = (k0 & 255) >> 1;
  const int chunk = byte0 >> 4, within = byte0 & 15;
  uint8_t* slab = sB + (k0 / 256) * kBSlab;
  bool bad = false;
#pragma unroll
  for (int j = 0; j < V; j++) bad |= !isfinite(v[j]);
  // The run's factor from its max, once: term t uses P * 4^t.  The largest
  // term-0 group scale lies in [171, 352]; a term's residual is at most its
  // group scale (E2M1 spacing 2 at the top, no saturation since scales round
  // up), so term t + 1's scales stay <= 2/3 of term t's bound (<= 240): no
  // E4M3 overflow, and 3 mantissa bits at every normal magnitude.
  float m;
  {
    float a0 = 0.f;
#pragma unroll
    for (int j = 0; j < V; j++) a0 = fmaxf(a0, fabsf(v[j]));
    m = warp_max(bad ? INFINITY : a0);
  }
  const int em = (__float_as_int(m) >> 23) & 0xFF;
  const bool live = m >= 7.9e-31f && m < INFINITY;
  float P = live ? __int_as_float((127 + 10 - (em - 127)) << 23) : 0.f;
  float f = live ? __int_as_float((127 - 10 + (em - 127)) << 23)
                 : (m == INFINITY ? __int_as_float(0x7fc00000) : 0.f);
#pragma unroll
  for (int t = 0; t < kT; t++, P *= 4.0f, f *= 0.25f) {
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < V; j++) amax = fmaxf(amax, fabsf(v[j]));
#pragma unroll
    for (int o = 1; o < TPG; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const uint32_t b = live ? e4m3_ceil_fast(amax * P * (1.0f / 6.0f)) : 0u;
    const float s = scale_to_f32(b);
    const float inv = s > 0.f ? P * __frcp_rn(s) : 0.f;
    const float back = s > 0.f ? s * f : 0.f;
    uint32_t w[(V + 7) / 8] = {};
#pragma unroll
    for (int j = 0; j < V; j += 2) {
      const uint32_t byte = e2m1_pair(v[j] * inv, v[j + 1] * inv);
      const float2 q = e2m1_pair_value(byte);
      v[j] -= q.x * back;
      v[j + 1] -= q.y * back;
      w[j >> 3] |= byte << (4 * (j & 7));
    }
    uint8_t* dst = slab + t * 128 + ((chunk ^ t) << 4) + within;
    if (in) {
      if constexpr (V == 16) *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
      else if constexpr (V == 8) *reinterpret_cast<uint32_t*>(dst) = w[0];
      else if constexpr (V == 4) *reinterpret_cast<uint16_t*>(dst) = (uint16_t)w[0];
      else *dst = (uint8_t)w[0];  // V = 2: one byte per thread
      if (ct % TPG == 0) sSc[t * (K / 16) + grp] = (uint8_t)b;
    }
    if (lane == 0) fac[4 * cw + t] = f;
  }
  named_sync(kBarChain, kChain);
}

// The term scales into tensor memory in the block-scaled MMA's layout (as the
// weight scales: row n, block j of K step s at lane n % 32 of every lane
// quarter, column 4 s + n / 32, byte j), rows 0..3 only.  Each chain warp
// writes its own lane quarter.
// Steps step0 .. step0 + nsteps - 1 (nsteps a multiple of 8) of a row of K.
__device__ __forceinline__ void store_term_scales(const uint8_t* sSc, int K, int step0, int nsteps,
                                                  uint32_t taddr, int lane) {
  const int ns = K / 64;  // K steps of the row
  const uint32_t* src = reinterpret_cast<const uint32_t*>(sSc);  // [t][ns]
  for (int blk = 0; blk < nsteps / 8; blk++) {
    uint32_t r[32];
#pragma unroll
    for (int cc = 0; cc < 32; cc++)
      r[cc] = ((cc & 3) == 0 && lane < kT) ? src[lane * ns + step0 + blk * 8 + (cc >> 2)] : 0u;
    tmem_st32(taddr + 4 * step0 + 32 * blk, r);
  }
}

// One accumulator row: sum over the 4 runs r and 4 terms t of fac[4 r + t] *
// D_r[t] (runs in order, terms in order), D_r at columns 16 r .. 16 r + 3.
__device__ __forceinline__ float fold_runs(uint32_t taddr, const float* fac) {
  uint32_t d[4][4];
#pragma unroll
  for (int r = 0; r < 4; r++)
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(d[r][0]), "=r"(d[r][1]), "=r"(d[r][2]), "=r"(d[r][3])
                 : "r"(taddr + 16 * r)
                 : "memory");
  tmem_wait_ld();
  float y = 0.f;
#pragma unroll
  for (int r = 0; r < 4; r++)
#pragma unroll
    for (int t = 0; t < kT; t++) y += fac[4 * r + t] * __uint_as_float(d[r][t]);
  return y;
}

// v[0..V) = sum over the kk segment partials of Yp at k0 .. k0 + V - 1, in
// segment order; 64 floats of loads in flight per thread per round.
template <int V>
__device__ __forceinline__ void load_segment_sum(const float* Yp, int H, int kk, int k0,
                                                 float (&v)[V]) {
  constexpr int NF = V / 4;
  constexpr int SEG = 16 / NF;
#pragma unroll
  for (int j = 0; j < V; j++) v[j] = 0.f;
  for (int s0 = 0; s0 < kk; s0 += SEG) {
    float4 b[SEG][NF];
#pragma unroll
    for (int q = 0; q < SEG; q++)
#pragma unroll
      for (int f = 0; f < NF; f++)
        b[q][f] = s0 + q < kk ? __ldcg(reinterpret_cast<const float4*>(Yp + (size_t)(s0 + q) * H +
                                                                       k0 + 4 * f))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q = 0; q < SEG; q++)
#pragma unroll
      for (int f = 0; f < NF; f++) {
        v[4 * f] += b[q][f].x;
        v[4 * f + 1] += b[q][f].y;
        v[4 * f + 2] += b[q][f].z;
        v[4 * f + 3] += b[q][f].w;
      }
  }
}

// ---- routed stack: CTA pairs (clusters of 2) ----
// The partner CTA's shared-memory address of this CTA's smem address a.
__device__ __forceinline__ uint32_t peer_smem(uint32_t a, uint32_t peer) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(peer));
  return r;
}
__device__ __forceinline__ void st_peer_f32(uint32_t a, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}
// One arrival on a barrier in the partner's shared memory, ordering this
// thread's earlier stores to the partner first.
__device__ __forceinline__ void mbar_arrive_peer(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t* bar, uint32_t parity,
                                                          long long budget) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait_cluster(bar, parity))
    if (clock64() - start > budget) return false;
  return true;
}
// Every thread of both CTAs of the pair.
__device__ __forceinline__ void cluster_sync_fs() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// ---- routed stack: router rows, logit partials, routing ----

__device__ __forceinline__ void cp_async16_fs(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit_fs() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// every group but the most recent one has landed
__device__ __forceinline__ void cp_async_wait_prev_fs() {
  asm volatile("cp.async.wait_group 1;" ::: "memory");
}

// Reducer rows [r0, r0 + 32) of every expert's router row of layer j into
// rsl[j & 1] ([e][32] bf16, 64 bytes per expert), by the 128 chain threads;
// one cp.async group per call (empty when j is past the launch).
__device__ __forceinline__ void issue_router_rows(const FsArgs& a, const FsSmem& S, int j, int r0,
                                                  int ct) {
  if (j < a.L) {
    const uint16_t* G = a.layer[j].router_w;
    uint8_t* dst = S.rsl + (size_t)(j & 1) * (256 * kFsRedRows * 2);
    for (int i = ct; i < a.E * 4; i += kChain) {
      const int e = i >> 2, q = i & 3;
      cp_async16_fs(dst + e * 64 + q * 16, G + (size_t)e * a.H + r0 + q * 8);
    }
  }
  cp_async_commit_fs();
}

// ---- routed stack: the exchange area (zeroed at launch; values carry their
// own completion, so no release / acquire pair sits in the routing chain) ----
struct Xchg {
  unsigned long long* rt;   // [kFsMaxLayers][8]: layer l's routing, slot j tagged l + 1
  unsigned long long* xin;  // [2][H / 2]: the layer inputs, two values per word, tagged
  unsigned long long* sq;   // [kFsMaxLayers][kFsMaxReducers]: sums of squares, tagged
  unsigned long long* ys;   // [L][H][kFsYsStride]: counted layer-output sums (norm on)
  unsigned long long* lg;   // [L][E][kFsLgStride]: counted logit sums
};
__device__ __forceinline__ Xchg xchg(const FsArgs& a) {
  Xchg x;
  x.rt = a.XG;
  x.xin = x.rt + (size_t)kFsMaxLayers * 8;
  x.sq = x.xin + (size_t)a.H;
  x.ys = x.sq + (size_t)kFsMaxLayers * kFsMaxReducers;
  x.lg = x.ys + (size_t)a.L * a.H * kFsYsStride;
  return x;
}

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Publishing a tagged word: an atomic exchange, performed at L2 at once (a
// relaxed store could wait in the writing SM; measured: the reducers' sums of
// squares were seen 1.8 us later with plain stores, the layer 1.9 us longer).
__device__ __forceinline__ void publish_u64(unsigned long long* p, unsigned long long v) {
  unsigned long long old;
  asm volatile("atom.relaxed.gpu.global.exch.b64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v)
               : "memory");
}

// A tagged word: bits 63..48 the tag (a layer of the launch + 1, never 0 after
// the launch's zeroing), bits 31..0 the payload.  One 8-byte store, so a
// reader sees the payload whole once it sees the tag.
__device__ __forceinline__ unsigned long long tagged(uint32_t tag, uint32_t payload) {
  return ((unsigned long long)tag << 48) | payload;
}
__device__ __forceinline__ uint32_t tag_of(unsigned long long w) { return (uint32_t)(w >> 48); }

// Counted sums: each contributor adds (q << 16) + (bad << 8) + 1 with q its
// value in 2^-F units; bits 7..0 count the adds, bits 15..8 the values that
// were not finite or beyond 2^B in magnitude (the sum is then NaN), bits
// 63..16 the sum of q (|sum| < 2^47 for fewer than 2^(47 - F - B) adds).
// Integer sums do not depend on the order of the adds, so every run gives the
// same bits.  Logits: F = 28, B = 13, 64 reducers; the routed stack's layer
// outputs: F = 24, B = 16, kk * I / 64 <= 127 down items per row.
template <int F, int B>
__device__ __forceinline__ void add_counted(unsigned long long* p, float x) {
  const bool ok = fabsf(x) < (float)(1 << B);
  const long long q = ok ? __float2ll_rn(x * (float)(1ull << F)) : 0ll;
  const unsigned long long v = ((unsigned long long)q << 16) + (ok ? 1ull : 0x101ull);
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
template <int F>
__device__ __forceinline__ float decode_counted(unsigned long long v) {
  if ((v >> 8) & 0xFF) return __int_as_float(0x7fc00000);
  return __ll2float_rn((long long)v >> 16) * (1.0f / (float)(1ull << F));
}
__device__ __forceinline__ void add_counted_logit(unsigned long long* line, float p) {
  add_counted<28, 13>(line, p);
}
__device__ __forceinline__ float decode_counted_logit(unsigned long long v) {
  return decode_counted<28>(v);
}

// Bounded poll by a whole warp: every lane's `n` words (in its registers
// after the call) until done(word) holds for all of them across the warp.
template <int N, typename Done>
__device__ __forceinline__ bool poll_words(const unsigned long long* const (&p)[N],
                                           unsigned long long (&w)[N], long long budget,
                                           Done done) {
  const long long t0 = clock64();
  for (;;) {
    bool mine = true;
#pragma unroll
    for (int i = 0; i < N; i++) {
      if (p[i]) {
        w[i] = ld_relaxed_u64(p[i]);
        mine &= done(w[i]);
      }
    }
    if (__all_sync(0xffffffffu, mine)) return true;
    if (__any_sync(0xffffffffu, clock64() - t0 > budget)) return false;  // warp-uniform
    __nanosleep(20);
  }
}

// The reducer's share of layer j's logits: for experts ct and ct + 128,
// sum over its 32 rows r (in order) of xs[r] * G_j[e, r0 + r], added to the
// experts' counted sums.
__device__ __forceinline__ void router_partials(const FsArgs& a, const FsSmem& S, const Xchg& X,
                                                int j, int ct) {
  const uint8_t* sl = S.rsl + (size_t)(j & 1) * (256 * kFsRedRows * 2);
  unsigned long long* lg = X.lg + (size_t)j * a.E * kFsLgStride;
  float p[2] = {0.f, 0.f};
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const int e = ct + 128 * h;
    if (e >= a.E) break;
    const uint4* g = reinterpret_cast<const uint4*>(sl + e * 64);
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const uint4 w = g[q];
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ws[i]));
        p[h] += S.xs[8 * q + 2 * i] * f.x;
        p[h] += S.xs[8 * q + 2 * i + 1] * f.y;
      }
    }
  }
  // both adds back to back: every expert's sum completes at about the same time
#pragma unroll
  for (int h = 0; h < 2; h++)
    if (ct + 128 * h < a.E) add_counted_logit(lg + (size_t)(ct + 128 * h) * kFsLgStride, p[h]);
}

// The router CTA, all its warps (it has no expert item): thread t < 256
// waits until all nR reducers have added to the logit sum of expert t, rounds
// the logit to the activation dtype as the reference's bf16 matmul returns
// it, scores it and ranks its key among its warp's 32 (the number of larger
// keys: keys are distinct apart from 0, topk.cuh); keys of rank < k form the
// warp's sorted list.  Warps 0-1 rank the 8 warps' list entries (one each)
// among all 64, which gives the top k in slot order; warp 0 publishes slot j
// (lane j < k) as tagged (expert id << 32 | weight bits) words of layer l's
// routing line, and into the layer's routing outputs; weights / their sum in
// slot order.  Counting compares shared-memory words instead of exchanging
// keys between lanes: no dependent chain of warp shuffles.
__device__ __forceinline__ bool route_and_publish_cta(const FsArgs& a, const FsSmem& S,
                                                      const Xchg& X, int l, int nR) {
  constexpr int kW = 8;  // warps holding one expert per lane
  const int t = threadIdx.x, w = t >> 5, lane = t & 31;
  uint64_t* wkeys = reinterpret_cast<uint64_t*>(S.rsl);                 // [8][32]
  uint64_t* lists = reinterpret_cast<uint64_t*>(S.rsl + 2048);          // [8][8]
  float* lscore = reinterpret_cast<float*>(S.rsl + 2048 + 512);         // [8][8]
  uint64_t* skey = reinterpret_cast<uint64_t*>(S.rsl + 2048 + 768);     // [8] slots
  float* sscore = reinterpret_cast<float*>(S.rsl + 2048 + 768 + 64);    // [8]
  int* okf = reinterpret_cast<int*>(S.rsl + 2048 + 768 + 96);
  const unsigned long long* lg = X.lg + (size_t)l * a.E * kFsLgStride;
  const float* b = a.layer[l].router_b;
  bool ok = true;
  if (w < kW) {
    if (lane < 8) {  // empty list entries and slots: no expert, score 0
      lists[w * 8 + lane] = 0ull;
      lscore[w * 8 + lane] = 0.f;
      if (w == 0) {
        skey[lane] = 0ull;
        sscore[lane] = 0.f;
      }
    }
    if (t == 0) *okf = 1;
    const bool live = t < a.E;
    const float bias = (b && live) ? __ldg(b + t) : 0.f;
    const unsigned long long* p[1] = {live ? lg + (size_t)t * kFsLgStride : nullptr};
    unsigned long long wv[1] = {0ull};
    ok = poll_words<1>(p, wv, a.budget, [&](unsigned long long v) { return (int)(v & 0xFF) == nR; });
    float sc = 0.f;
    uint64_t key = 0ull;
    if (live) {
      sc = sigmoid_ref(round_to_dtype(decode_counted_logit(wv[0]), a.dtype));
      key = choice_key(sc + bias, (uint32_t)t);
    }
    wkeys[t] = key;
    __syncwarp();
    int rc[4] = {0, 0, 0, 0};
    const ulonglong2* wk = reinterpret_cast<const ulonglong2*>(wkeys + w * 32);
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      const ulonglong2 q0 = wk[j], q1 = wk[j + 1];
      rc[0] += (int)(q0.x > key);
      rc[1] += (int)(q0.y > key);
      rc[2] += (int)(q1.x > key);
      rc[3] += (int)(q1.y > key);
    }
    const int r = (rc[0] + rc[1]) + (rc[2] + rc[3]);
    __syncwarp();  // the list entries' zeroing before the writes
    if (key && r < a.k) {  // a key of 0 (no expert) leaves its entry empty
      lists[w * 8 + r] = key;
      lscore[w * 8 + r] = sc;
    }
    if (!ok && lane == 0) *okf = 0;
  }
  __syncthreads();  // the eight lists visible to warps 0-1
  const bool all_ok = *okf != 0;
  if (w < 2) {
    const uint64_t u = lists[t];
    const float us = lscore[t];
    const ulonglong2* lk = reinterpret_cast<const ulonglong2*>(lists);
    int rq[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      const ulonglong2 q0 = lk[j], q1 = lk[j + 1];
      rq[0] += (int)(q0.x > u);
      rq[1] += (int)(q0.y > u);
      rq[2] += (int)(q1.x > u);
      rq[3] += (int)(q1.y > u);
    }
    const int r = (rq[0] + rq[1]) + (rq[2] + rq[3]);
    if (u && r < a.k) {
      skey[r] = u;
      sscore[r] = us;
    }
    named_sync(2, 64);  // the slots written
    if (w == 0) {
      const float4 s0 = reinterpret_cast<const float4*>(sscore)[0];
      const float4 s1 = reinterpret_cast<const float4*>(sscore)[1];
      const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
      float wsum = 0.f;
#pragma unroll
      for (int j = 0; j < 8; j++) wsum += j < a.k ? sv[j] : 0.f;
      const uint64_t kk = lane < 8 ? skey[lane] : 0ull;
      const uint32_t isel = kk ? 0xFFFFFFFFu - (uint32_t)kk : 0x7fffffffu;
      float wsel = lane < 8 ? sv[0] : 0.f;
#pragma unroll
      for (int j = 1; j < 8; j++)
        if (lane == j) wsel = sv[j];
      if (a.norm) wsel = wsel / wsum;
      if (lane < a.k) {
        const uint32_t id16 = isel < 0xFFFFu ? isel : 0xFFFFu;
        publish_u64(X.rt + (size_t)l * 8 + lane, tagged((uint32_t)(l + 1), 0u) |
                                                     ((unsigned long long)id16 << 32) |
                                                     __float_as_uint(wsel));
        if (a.layer[l].inds) a.layer[l].inds[lane] = isel;
        if (a.layer[l].wts) a.layer[l].wts[lane] = wsel;
      }
    }
  }
  __syncthreads();  // the scratch is free again
  return all_ok;
}

// Any other CTA, one warp: layer l's routing from its routing line.
__device__ __forceinline__ bool read_routing(const FsArgs& a, const Xchg& X, int l, int lane,
                                             uint32_t& isel, float& wsel) {
  const unsigned long long* p[1] = {lane < a.k ? X.rt + (size_t)l * 8 + lane : nullptr};
  unsigned long long w[1] = {0};
  const uint32_t tag = (uint32_t)(l + 1);
  const bool ok = poll_words<1>(p, w, a.budget,
                                [&](unsigned long long v) { return tag_of(v) == tag; });
  const uint32_t id16 = (uint32_t)(w[0] >> 32) & 0xFFFFu;
  isel = id16 == 0xFFFFu ? 0x7fffffffu : id16;
  wsel = __uint_as_float((uint32_t)w[0]);
  return ok;
}

// RM: 0 given routing, 1 routed stack, 2 routed stack with the norm (a.has_norm
// as a compile-time constant: each launch holds only its own reducer path).
template <int VX, int VA, int RM>
__global__ void __launch_bounds__(kThreads, 1)
    moe_decode_stack_fp4_kernel(const __grid_constant__ FsArgs a) {
  constexpr bool ROUTED = RM > 0, NORM = RM == 2;
  constexpr int NS = stages(ROUTED);
  extern __shared__ __align__(1024) unsigned char fs_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(fs_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int H = a.H, I = a.I;  // H = 128 VX nks, I = 128 VA (checked on the host)
  FsSmem S;
  fs_carve(H, I, a.L, ROUTED, base, &S);
  constexpr uint32_t kSfa0 = sfa0_of(ROUTED), kSfbx = sfbx_of(ROUTED);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, c = blockIdx.x;
  const int nb = I / 64;
  const int nGU = a.kk * nb * a.nks;
  const int nD = a.kk * (H / 128);
  const bool has_gu = c < nGU;
  const int gu_seg = has_gu ? c / (nb * a.nks) : 0;
  const int gu_rem = c - gu_seg * nb * a.nks;
  const int gu_b = gu_rem / a.nks, gu_p = gu_rem - (gu_rem / a.nks) * a.nks;
  const int KS = H / 256 / a.nks;  // K slabs of a gate/up item
  // Given routing: down item (segment, 128-row block d_rb) over all of I.
  // Routed stack: the CTA pair (cluster of 2) of one (segment, I block gu_b)
  // computes gate/up over its two K halves, exchanges the partials through
  // distributed shared memory, and each CTA computes the down projection of
  // the block's 64 act values for its half of H (DT tiles of 128 rows x K 64).
  const bool has_d = ROUTED ? has_gu : c < nD;
  const int d_seg = ROUTED ? gu_seg : (has_d ? c / (H / 128) : 0);
  const int d_rb = c - d_seg * (H / 128);
  const int DT = H / 256;
  const int DS = ROUTED ? (DT + kRTilesPerStage - 1) / kRTilesPerStage : I / 256;
  const uint32_t kSfba = kSfbx + (uint32_t)(H / 16);

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; i++) {
      mbar_init(&S.full[i], 1);
      mbar_init(&S.empty[i], 1);
      mbar_init(&S.sfr[i], 4);
    }
    mbar_init(S.xready, 4);
    mbar_init(S.aready, 4);
    mbar_init(S.gufull, 1);
    mbar_init(S.dfull, 1);
    mbar_init(S.drain, 1);
    if (ROUTED) mbar_init(S.guready, kChain);  // the partner's chain threads, one arrival each
    *S.hold = 0;
    *S.cur = 0;
    if (ROUTED) *S.rlayer = 0;
    fence_barrier_init();
  }
  // Given routing: the launch's layers into shared memory once.
  if (!ROUTED)
    for (int i = threadIdx.x; i < a.L * a.k; i += blockDim.x) {
      const int l = i / a.k, j = i - l * a.k;
      S.inds[l * 16 + j] = a.layer[l].inds[j];
      S.wts[l * 16 + j] = a.layer[l].wts[j];
    }
  // Term tiles: rows 4..15 stay zero for the whole launch.
  {
    uint4* z = reinterpret_cast<uint4*>(S.bx);
    const int n = (H / 256 + I / 256) * kBSlab / 16;
    for (int i = threadIdx.x; i < n; i += blockDim.x) z[i] = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async();
  }
  if (warp == kWarpMma) tmem_alloc(S.tslot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if constexpr (ROUTED) cluster_sync_fs();  // the partner's barriers exist before any arrival
  const uint32_t tmem = *S.tslot;

  if (ROUTED && c == G - 1) {
    // ------------------ the router CTA: every warp routes ------------------
    const Xchg XR = xchg(a);
    const int nR = H / kFsRedRows;
    for (int l = 0; l < a.L; l++) {
      const bool got = route_and_publish_cta(a, S, XR, l, nR);
      if (!got) {
        if (threadIdx.x == 0) fsflag(fs_timeout(l, 53));
        break;
      }
    }
  } else if (warp == kWarpTma) {
    // ------------------------------ TMA producer ------------------------------
    const uint32_t el = elect_one_fs();
    uint32_t g = 0;
    bool ok = true;
    auto slot = [&](int& s, int l) -> bool {
      s = (int)(g % NS);
      if (g >= (uint32_t)NS &&
          !mbar_wait_bounded(&S.empty[s], ((g / NS) - 1) & 1, a.budget)) {
        if (el) fsflag(fs_timeout(l, 41));
        return false;
      }
      // Refills for a later layer than the chain's wait while the chain's
      // MMAs, epilogue, dependency wait and the L2 loads behind it run (the hold
      // flag): a refill burst (the stages an MMA batch just released, up to
      // 72 KB per CTA) issued then queues ahead of the counters' atomics and
      // those loads.  They go out while the chain computes terms.  A stage of
      // the chain's own layer is never held (its MMA may be waiting for it).
      // Bounded: a missed release only costs time.
      if (el && *S.hold && l > *S.cur) {
        const long long h0 = clock64();
        while (*S.hold && l > *S.cur && clock64() - h0 < 40000) __nanosleep(64);
      }
      __syncwarp();
      return true;
    };
    // Routed stack: a routed segment's slabs of layer l wait for its routing.
    auto routing_known = [&](int l) -> bool {
      if (!ROUTED) return true;
      if (el && *S.rlayer <= l) {
        const long long t0 = clock64();
        while (*S.rlayer <= l) {
          if (clock64() - t0 > a.budget) {
            fsflag(fs_timeout(l, 55));
            break;
          }
          __nanosleep(32);
        }
      }
      __syncwarp();
      __threadfence_block();  // the routing written before the flag
      return *S.rlayer > l;
    };
    for (int l = 0; l < a.L && ok; l++) {
      const CUtensorMap* mp = &a.maps[l * a.mpl];
      if (has_gu) {
        const bool sh = gu_seg >= a.k;
        uint32_t e = 0;
        if (!sh) {
          if (!routing_known(l)) {
            ok = false;
            break;
          }
          e = S.inds[l * 16 + gu_seg];
          if (e >= (uint32_t)a.E) {
            if (el) fsflag(kErrIndex);
            e = 0;  // the pipeline stays consistent; the output is flagged invalid
          }
        }
        const CUtensorMap* m = sh ? mp + kFsMapsRouted : mp;
        const int row0 = (sh ? 0 : (int)e * I) + gu_b * 64;
        for (int sl = 0; sl < KS; sl++, g++) {
          int s;
          if (!slot(s, l)) {
            ok = false;
            break;
          }
          if (el) {
            uint8_t* st = S.stage + (size_t)s * kStage;
            const int xk = gu_p * KS + sl;
            mbar_arrive_expect_tx(&S.full[s], (uint32_t)kStage);
            tma_load_2d(st, m + 0, xk * 128, row0, &S.full[s]);
            tma_load_2d(st + kA / 2, m + 2, xk * 128, row0, &S.full[s]);
            tma_load_2d(st + kA, m + 1, xk * 16, row0, &S.full[s]);
            tma_load_2d(st + kA + kSA / 2, m + 3, xk * 16, row0, &S.full[s]);
          }
          __syncwarp();
        }
      }
      if (has_d && ok) {
        const bool sh = d_seg >= a.k;
        uint32_t e = 0;
        if (!sh) {
          if (!routing_known(l)) {
            ok = false;
            break;
          }
          e = S.inds[l * 16 + d_seg];
          if (e >= (uint32_t)a.E) {
            if (el) fsflag(kErrIndex);
            e = 0;
          }
        }
        const CUtensorMap* m = sh ? mp + kFsMapsRouted : mp;
        if (ROUTED) {
          // this CTA's half of H, K = the pair's I block: row tiles of 128 x 64
          // codes (32-byte rows), their scale bytes with the block's neighbours
          const int row0 = (sh ? 0 : (int)e * H) + gu_p * (H / 2);
          for (int sl = 0; sl < DS; sl++, g++) {
            int s;
            if (!slot(s, l)) {
              ok = false;
              break;
            }
            if (el) {
              uint8_t* st = S.stage + (size_t)s * kStage;
              const int t0 = sl * kRTilesPerStage;
              const int nt = DT - t0 < kRTilesPerStage ? DT - t0 : kRTilesPerStage;
              mbar_arrive_expect_tx(&S.full[s], (uint32_t)(nt * (kRTileCodes + kRTileScales)));
              for (int j = 0; j < nt; j++) {
                const int rr = row0 + (t0 + j) * 128;
                tma_load_2d(st + j * kRTileCodes, m + 4, gu_b * 32, rr, &S.full[s]);
                tma_load_2d(st + kRScales0 + j * kRTileScales, m + 5, (gu_b / 4) * 16, rr,
                            &S.full[s]);
              }
            }
            __syncwarp();
          }
        } else {
          const int row0 = (sh ? 0 : (int)e * H) + d_rb * 128;
          for (int sl = 0; sl < DS; sl++, g++) {
            int s;
            if (!slot(s, l)) {
              ok = false;
              break;
            }
            if (el) {
              uint8_t* st = S.stage + (size_t)s * kStage;
              mbar_arrive_expect_tx(&S.full[s], (uint32_t)kStage);
              tma_load_2d(st, m + 4, sl * 128, row0, &S.full[s]);
              tma_load_2d(st + kA, m + 5, sl * 16, row0, &S.full[s]);
            }
            __syncwarp();
          }
        }
      }
    }
    // no copy may still be landing at exit
    for (uint32_t i = 0; i < (g < (uint32_t)NS ? g : (uint32_t)NS); i++) {
      const uint32_t q = g - 1 - i;
      mbar_wait_bounded(&S.full[q % NS], (q / NS) & 1, kDrainBudget);
    }
  } else if (warp == kWarpMma) {
    // ------------------------------ MMA issuer ------------------------------
    const uint32_t el = elect_one_fs();
    const uint32_t idesc = idesc_mxf4nvf4(128, kN);
    const uint32_t sbx = smem_u32(S.bx), sba = smem_u32(S.ba);
    uint32_t g = 0, jx = 0, ja = 0;
    bool ok = true;
    for (int l = 0; l < a.L && ok; l++) {
      if (has_gu) {
        if (!mbar_wait_bounded(S.xready, jx & 1, a.budget)) {
          if (el) fsflag(fs_timeout(l, 42));
          break;
        }
        jx++;
        tc_fence_after();
        for (int sl = 0; sl < KS; sl++, g++) {
          const int s = (int)(g % NS);
          if (!mbar_wait_bounded(&S.sfr[s], (g / NS) & 1, a.budget)) {
            if (el) fsflag(fs_timeout(l, 43));
            ok = false;
            break;
          }
          tc_fence_after();
          if (el) {
            const uint32_t sa = smem_u32(S.stage + (size_t)s * kStage);
            const int xk = gu_p * KS + sl;
            const uint32_t sb = sbx + (uint32_t)(xk * kBSlab);
            const uint32_t sfa = tmem + kSfa0 + (uint32_t)s * kSfaCols;
            const uint32_t sfb = tmem + kSfbx + (uint32_t)(16 * xk);
#pragma unroll
            for (int k4 = 0; k4 < 4; k4++) {
              const int ks = 4 * sl + k4;  // K step in the item; run = ks / (VX / 2)
              umma_mxf4nvf4(tmem + kAccGU + 16 * (ks * 2 / VX), smem_desc_sw128(sa + 32 * k4),
                            smem_desc_sw128(sb + 32 * k4), idesc, sfa + 4 * k4, sfb + 4 * k4,
                            ks % (VX / 2) != 0 ? 1u : 0u);
            }
            umma_commit(&S.empty[s]);
          }
          __syncwarp();
        }
        if (!ok) break;
        if (el) umma_commit(S.gufull);
        __syncwarp();
      }
      if (has_d) {
        if (!mbar_wait_bounded(S.aready, ja & 1, a.budget)) {
          if (el) fsflag(fs_timeout(l, 44));
          break;
        }
        ja++;
        tc_fence_after();
        for (int sl = 0; sl < DS; sl++, g++) {
          const int s = (int)(g % NS);
          if (!mbar_wait_bounded(&S.sfr[s], (g / NS) & 1, a.budget)) {
            if (el) fsflag(fs_timeout(l, 45));
            ok = false;
            break;
          }
          tc_fence_after();
          if (ROUTED) {
            // one K = 64 step per 128-row tile: tile t into accumulator t
            if (el) {
              const uint32_t sa = smem_u32(S.stage + (size_t)s * kStage);
              const int t0 = sl * kRTilesPerStage;
              const int nt = DT - t0 < kRTilesPerStage ? DT - t0 : kRTilesPerStage;
              for (int j = 0; j < nt; j++)
                umma_mxf4nvf4(tmem + kAccD + 16 * (uint32_t)(t0 + j),
                              smem_desc_sw32(sa + (uint32_t)(j * kRTileCodes)),
                              smem_desc_sw128(sba), idesc,
                              tmem + kSfa0 + (uint32_t)s * kSfaCols + 4u * (uint32_t)j,
                              tmem + kSfba, 0u);
              umma_commit(&S.empty[s]);
            }
            __syncwarp();
            continue;
          }
          if (el) {
            const uint32_t sa = smem_u32(S.stage + (size_t)s * kStage);
            const uint32_t sb = sba + (uint32_t)(sl * kBSlab);
            const uint32_t sfa = tmem + kSfa0 + (uint32_t)s * kSfaCols;
            const uint32_t sfb = tmem + kSfba + (uint32_t)(16 * sl);
#pragma unroll
            for (int k4 = 0; k4 < 4; k4++) {
              const int ks = 4 * sl + k4;
              umma_mxf4nvf4(tmem + kAccD + 16 * (ks * 2 / VA), smem_desc_sw128(sa + 32 * k4),
                            smem_desc_sw128(sb + 32 * k4), idesc, sfa + 4 * k4, sfb + 4 * k4,
                            ks % (VA / 2) != 0 ? 1u : 0u);
            }
            umma_commit(&S.empty[s]);
          }
          __syncwarp();
        }
        if (!ok) break;
        if (el) umma_commit(S.dfull);
        __syncwarp();
      }
    }
    // every MMA issued has completed before tensor memory is released
    if (el) umma_commit(S.drain);
    __syncwarp();
    if (!mbar_wait_bounded(S.drain, 0, kDrainBudget) && el) fsflag(fs_timeout(-1, 46));
  } else if (warp < kWarpChain0) {
    // -------------------- weight scales into tensor memory --------------------
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    const int per_layer = (has_gu ? KS : 0) + (has_d ? DS : 0);
    uint32_t g = 0;
    bool ok = true;
    for (int l = 0; l < a.L && ok; l++) {
      for (int i = 0; i < per_layer; i++, g++) {
        const int s = (int)(g % NS);
        if (!mbar_wait_bounded(&S.full[s], (g / NS) & 1, a.budget)) {
          if (lane == 0) fsflag(fs_timeout(l, 47));
          ok = false;
          break;
        }
        if (ROUTED && i >= KS) {
          // routed down stage: per tile, the I block's K step (4 scale bytes)
          // of each row, columns 4 j .. 4 j + 3 of the stage's scale columns
          const int t0 = (i - KS) * kRTilesPerStage;
          const int nt = DT - t0 < kRTilesPerStage ? DT - t0 : kRTilesPerStage;
          const uint8_t* sf = S.stage + (size_t)s * kStage + kRScales0 + 4 * (gu_b & 3);
          for (int j = 0; j < nt; j++) {
            uint32_t ra[4];
#pragma unroll
            for (int cq = 0; cq < 4; cq++)
              ra[cq] = *reinterpret_cast<const uint32_t*>(sf + j * kRTileScales +
                                                          16 * (lane + 32 * cq));
            tmem_st4(tmem + lane_base + kSfa0 + (uint32_t)s * kSfaCols + 4u * (uint32_t)j, ra);
          }
        } else {
          const uint8_t* sf = S.stage + (size_t)s * kStage + kA;
          uint32_t ra[16];
#pragma unroll
          for (int cq = 0; cq < 4; cq++) {
            const uint4 va = *reinterpret_cast<const uint4*>(sf + 16 * (lane + 32 * cq));
            ra[0 + cq] = va.x;
            ra[4 + cq] = va.y;
            ra[8 + cq] = va.z;
            ra[12 + cq] = va.w;
          }
          tmem_st16(tmem + lane_base + kSfa0 + (uint32_t)s * kSfaCols, ra);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.sfr[s]);
      }
    }
  } else {
    // ------------------------------ the chain ------------------------------
    const int ct = threadIdx.x - kWarpChain0 * 32;  // 0..127
    const int q = warp & 3;                         // TMEM lane quarter
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    const int r = 32 * q + lane;                    // accumulator row = TMEM lane
    uint32_t jgu = 0, jd = 0, jpair = 0;
    // Dependency counters (zero at launch): cnt1[seg] counts the gate/up items
    // of segment seg done (nb * nks per layer); cnt2[p] the down items whose
    // rows lie in K part p done (kk * H / 128 / nks per layer) -- in the
    // routed stack cnt2[rb] the down items of 128-row block rb (kk per layer).
    // Producers: the chain's writes, a barrier, then one release add.
    // Consumers: thread 0 polls (acquire, bounded), then a barrier.
    unsigned* cnt1 = a.bar;
    unsigned* cnt2 = a.bar + 16;
    const unsigned per_seg = (unsigned)(nb * a.nks);
    const int rb_per_part = H / 128 / a.nks;
    const unsigned per_part = (unsigned)(a.kk * rb_per_part);
    auto wait_count = [&](const unsigned* ctr, unsigned target, int l, int site) -> bool {
      if (ct == 0) {
        bool ok = true;
        if (ld_acquire_fs(ctr) < target) {
          const long long start = clock64();
          while (ld_acquire_fs(ctr) < target) {
            if (clock64() - start > a.budget) {
              ok = false;
              break;
            }
            __nanosleep(32);
          }
        }
        *S.bar_ok = ok;
        if (!ok) fsflag(fs_timeout(l, site));
      }
      named_sync(kBarChain, kChain);
      return *S.bar_ok != 0;
    };
    auto signal_count = [&](unsigned* ctr) {
      named_sync(kBarChain, kChain);
      if (ct == 0) red_release_add_fs(ctr, 1u);  // orders the CTA's writes (bar.sync) first
    };
    // Routed stack, reducer c (c < nR): rows [red_r0, red_r0 + 32), one per
    // thread ct < 32 (the chain's first warp); the router: the last CTA.
    const int nR = H / kFsRedRows;
    const bool is_red = ROUTED && c < nR;
    const int red_r0 = c * kFsRedRows;
    const Xchg XC = ROUTED ? xchg(a) : Xchg{};
    float hrow = 0.f;  // reducer thread ct < 32: h_j at its row (the residual)
    // Layer j's input x_j from h_j (hrow) and its logit partials.  With the
    // norm: the rows' sum of squares as this reducer's tagged word of layer j,
    // every reducer's word (polled), their sum in reducer order -- the same
    // bits on every reducer -- and x = dtype(dtype(h * r) * w) with
    // r = 1 / sqrt(sum / H + eps).  Then x_j as tagged words (two values each)
    // and into S.xs, the counted partials of x_j[rows] . G_j[e, rows] (router
    // rows of layer j landed: issued two layers ago), and the router rows of
    // layer j + 2 into the freed buffer.
    auto route_rows = [&](int j) -> bool {
      const int row = red_r0 + ct;
      const uint32_t tag = (uint32_t)(j + 1);
      float xv = hrow;
      bool ok = true;
      if (NORM && ct < 32) {
        const float w = load_as_f32(a.layer[j].norm_w, a.dtype, row);
        const float s2 = warp_sum(hrow * hrow);
        unsigned long long* sq = XC.sq + (size_t)j * kFsMaxReducers;
        if (ct == 0) publish_u64(sq + c, tagged(tag, __float_as_uint(s2)));
        const unsigned long long* p[2] = {lane < nR ? sq + lane : nullptr,
                                          lane + 32 < nR ? sq + lane + 32 : nullptr};
        unsigned long long wv[2] = {0ull, 0ull};
        ok = poll_words<2>(p, wv, a.budget, [&](unsigned long long v) { return tag_of(v) == tag; });
        if (!ok && ct == 0) fsflag(fs_timeout(j, 56));
        const float tot = warp_sum((p[0] ? __uint_as_float((uint32_t)wv[0]) : 0.f) +
                                   (p[1] ? __uint_as_float((uint32_t)wv[1]) : 0.f));
        const float r = 1.0f / sqrtf(tot / (float)H + a.eps);
        xv = round_to(round_to(hrow * r, a.dtype) * w, a.dtype);
      }
      if (ct < 32) {
        const uint32_t bits = a.dtype == kBF16 ? (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(xv))
                                               : (uint32_t)__half_as_ushort(__float2half_rn(xv));
        const uint32_t hi = __shfl_down_sync(0xffffffffu, bits, 1);
        if ((ct & 1) == 0)
          publish_u64(XC.xin + (size_t)((a.l0 + j) & 1) * (H / 2) + (row >> 1),
                         tagged(tag, (hi << 16) | bits));
        S.xs[ct] = xv;
      }
      ok = chain_sync_and(ok);
      cp_async_wait_prev_fs();
      named_sync(kBarChain, kChain);
      router_partials(a, S, XC, j, ct);
      named_sync(kBarChain, kChain);  // every read of rsl[j & 1] done
      issue_router_rows(a, S, j + 2, red_r0, ct);
      return ok;
    };
    bool alive = true;
    if (is_red) {
      // prologue: layer 0's input and logits from this launch's h_0
      issue_router_rows(a, S, 0, red_r0, ct);
      issue_router_rows(a, S, 1, red_r0, ct);
      if (ct < kFsRedRows) {
        const int row = red_r0 + ct;
        hrow = a.first ? load_as_f32(a.x0, a.dtype, row)
                       : __ldcg(a.Hres + (size_t)(a.l0 & 1) * H + row);
      }
      alive = route_rows(0);
    }
    for (int l = 0; l < a.L && alive; l++) {
      const int lg = a.l0 + l;  // index in the stack: buffer parity
      float* Yout = a.Yp + (size_t)(lg & 1) * a.kk * (ROUTED ? nb : 1) * H;
      const float* Yin = a.Yp + (size_t)((lg + 1) & 1) * a.kk * H;
      float* GUb = a.GUp + (size_t)(lg & 1) * 2 * a.kk * 2 * I;
      if (ct == 0) *S.cur = l;

      // ---- routed stack: this layer's routing (the router CTA computes and
      // publishes it; the others read its routing line).  A gate/up CTA takes
      // it after its x terms (x does not depend on the routing and is
      // published before the logits), the others here. ----
      auto take_routing = [&]() -> bool {
        uint32_t isel = 0;
        float wsel = 0.f;
        bool got = true;
        if (ct < 32) got = read_routing(a, XC, l, lane, isel, wsel);
        if (ct < 32) {
          if (!got && lane == 0) fsflag(fs_timeout(l, 53));
          if (lane < a.k) {
            S.inds[l * 16 + lane] = isel;
            S.wts[l * 16 + lane] = wsel;
          }
          __threadfence_block();
          __syncwarp();
          // the TMA warp may issue the routed slabs (on a failed poll too: ids out
          // of range are replaced and flagged there, and the chain stops below)
          if (lane == 0) *S.rlayer = l + 1;
          if (lane == 0) *S.bar_ok = got;
        }
        named_sync(kBarChain, kChain);
        return *S.bar_ok != 0;
      };
      if (ROUTED && !has_gu && has_d && !take_routing()) {
        alive = false;
        break;
      }

      // ---- phase A: x terms, gate/up item -> GUp ----
      if (has_gu) {
        // only this item's K part of x: its 128 VX values
        float v[VX];
        const int kb = gu_p * (H / a.nks);
        const int k0 = kb + ct * VX;
        if (l == 0 && a.first && !ROUTED) {
          if constexpr (VX % 8 == 0) {
#pragma unroll
            for (int j = 0; j < VX; j += 8)
              load8(a.x0, a.dtype, k0 + j, *reinterpret_cast<float(*)[8]>(&v[j]));
          } else {  // VX = 4: the aligned 8 around k0, half of them
            float f[8];
            load8(a.x0, a.dtype, k0 & ~7, f);
#pragma unroll
            for (int i = 0; i < 4; i++) v[i] = f[(k0 & 4) + i];
          }
        } else if (ROUTED) {
          // the reducers' x_l: tagged words of two values, polled until every
          // word of this thread carries layer l's tag
          const unsigned long long* xw = XC.xin + (size_t)(lg & 1) * (H / 2) + (k0 >> 1);
          const uint32_t tag = (uint32_t)(l + 1);
          unsigned long long w[VX / 2];
          const long long t0 = clock64();
          bool ok = true;
          for (;;) {
            bool done = true;
#pragma unroll
            for (int i = 0; i < VX / 2; i += 2) {
              const ulonglong2 q = __ldcg(reinterpret_cast<const ulonglong2*>(xw + i));
              w[i] = q.x;
              w[i + 1] = q.y;
              done &= tag_of(q.x) == tag && tag_of(q.y) == tag;
            }
            if (done) break;
            if (clock64() - t0 > a.budget) {
              ok = false;
              break;
            }
            __nanosleep(20);
          }
          if (!ok) fsflag(fs_timeout(l, 57));
#pragma unroll
          for (int i = 0; i < VX / 2; i++) {
            const uint32_t lo = (uint32_t)w[i] & 0xFFFFu, hi = ((uint32_t)w[i] >> 16) & 0xFFFFu;
            if (a.dtype == kBF16) {
              v[2 * i] = __bfloat162float(__ushort_as_bfloat16((unsigned short)lo));
              v[2 * i + 1] = __bfloat162float(__ushort_as_bfloat16((unsigned short)hi));
            } else {
              v[2 * i] = __half2float(__ushort_as_half((unsigned short)lo));
              v[2 * i + 1] = __half2float(__ushort_as_half((unsigned short)hi));
            }
          }
        } else {
          // the previous layer's down items of this part (previous launch: done)
          if (l > 0 && !wait_count(&cnt2[gu_p], (unsigned)l * per_part, l, 51)) {
            alive = false;
            break;
          }
          // the previous layer's output: its segments' partials in order
          load_segment_sum<VX>(Yin, H, a.kk, k0, v);
#pragma unroll
          for (int j = 0; j < VX; j++) v[j] = round_to(v[j], a.dtype);
        }
        if (ct == 0) *S.hold = 0;
        make_terms<VX>(v, ct, H, kb, S.bx, S.scx, S.facx);
        store_term_scales(S.scx, H, kb / 64, (H / a.nks) / 64, tmem + lane_base + kSfbx, lane);
        fence_proxy_async();
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (ct == 0) *S.hold = 1;
        if (lane == 0) mbar_arrive(S.xready);
        if (ROUTED && !take_routing()) {
          alive = false;
          break;
        }
        const bool got = mbar_wait_bounded(S.gufull, jgu & 1, a.budget);
        jgu++;
        if (!got && lane == 0) fsflag(fs_timeout(l, 48));
        alive = chain_sync_and(got);
        if (!alive) break;
        tc_fence_after();
        const float y = fold_runs(tmem + lane_base + kAccGU, S.facx);
        tc_fence_before();
        if (ROUTED) {
          // the pair exchange: this K part's partial of accumulator row r into
          // gux[gu_p][r] of both CTAs, then one arrival on the partner's barrier
          // (test-only NVFP4_LAUNCH_TEST_EXPIRE: the last layer's segment 0
          // never sends, so the partner's wait runs out and reports its site)
          S.gux[gu_p * 128 + r] = y;
          if (!(a.test_skip_release && l == a.L - 1 && gu_seg == 0)) {
            const uint32_t peer = (uint32_t)(gu_p ^ 1);
            st_peer_f32(peer_smem(smem_u32(&S.gux[gu_p * 128 + r]), peer), y);
            mbar_arrive_peer(peer_smem(smem_u32(S.guready), peer));
          }
        } else if (a.test_skip_release && l == a.L - 1 && gu_seg == 0) {
          __stcg(GUb + ((size_t)(gu_p * a.kk + gu_seg) * 2 + (r >> 6)) * I + gu_b * 64 + (r & 63), y);
          // test-only (NVFP4_LAUNCH_TEST_EXPIRE): this release is never made,
          // so the waits behind it run out and report their site
          named_sync(kBarChain, kChain);
        } else {
          __stcg(GUb + ((size_t)(gu_p * a.kk + gu_seg) * 2 + (r >> 6)) * I + gu_b * 64 + (r & 63), y);
          signal_count(&cnt1[gu_seg]);
        }
      }

      // ---- phase B: act terms, down item -> Yp ----
      if (has_d && ROUTED) {
        // the partner's partials of this layer (one arrival per chain thread);
        // the barrier below also publishes this CTA's own rows of gux
        const bool gotp = mbar_wait_cluster_bounded(S.guready, jpair & 1, a.budget);
        jpair++;
        if (!gotp && ct == 0) fsflag(fs_timeout(l, 50));
        alive = chain_sync_and(gotp);
        if (!alive) break;
        // the block's 64 act values, two per thread of the first warp (the
        // other warps hold zeros and store nothing): silu(gate) * up, the K
        // parts summed in order
        float v2[2] = {0.f, 0.f};
        if (ct < 32) {
#pragma unroll
          for (int j = 0; j < 2; j++) {
            const int i = 2 * ct + j;
            v2[j] = silu_ref(S.gux[i] + S.gux[128 + i]) * (S.gux[64 + i] + S.gux[192 + i]);
          }
        }
        if (ct == 0) *S.hold = 0;
        make_terms<2>(v2, ct, 64, 0, S.ba, S.sca, S.faca);
        store_term_scales(S.sca, 64, 0, 8, tmem + lane_base + kSfba, lane);
        fence_proxy_async();
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (ct == 0) *S.hold = 1;
        if (lane == 0) mbar_arrive(S.aready);
        const bool got = mbar_wait_bounded(S.dfull, jd & 1, a.budget);
        jd++;
        if (!got && lane == 0) fsflag(fs_timeout(l, 49));
        alive = chain_sync_and(got);
        if (!alive) break;
        tc_fence_after();
        const float wseg = d_seg < a.k ? S.wts[l * 16 + d_seg] * a.scaling : 1.0f;
        // tile t of this CTA's half of H: rows gu_p * H / 2 + 128 t + r; every
        // tile's accumulator row read before one wait
        float* Yb = Yout + ((size_t)d_seg * nb + gu_b) * H + gu_p * (H / 2);
        uint32_t dt[8][4];
#pragma unroll
        for (int t = 0; t < 8; t++)
          if (t < DT)
            asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(dt[t][0]), "=r"(dt[t][1]), "=r"(dt[t][2]), "=r"(dt[t][3])
                         : "r"(tmem + lane_base + kAccD + 16u * (uint32_t)t)
                         : "memory");
        tmem_wait_ld();
        // With the norm: each row's counted sum of the 2^-24 fixed-point
        // partials (the count completes it, no counter hop); without: f32
        // partials per (segment, I block) behind the row blocks' counters.
        unsigned long long* ysl =
            XC.ys + ((size_t)l * H + gu_p * (H / 2) + r) * kFsYsStride;
#pragma unroll
        for (int t = 0; t < 8; t++)
          if (t < DT) {
            float y = 0.f;
#pragma unroll
            for (int tt = 0; tt < kT; tt++) y += S.faca[tt] * __uint_as_float(dt[t][tt]);
            if (NORM) add_counted<24, 16>(ysl + (size_t)t * 128 * kFsYsStride, y * wseg);
            else __stcg(Yb + t * 128 + r, y * wseg);
          }
        tc_fence_before();
        named_sync(kBarChain, kChain);
        if (!NORM && ct < DT) red_release_add_fs(&cnt2[gu_p * DT + ct], 1u);
      } else if (has_d) {
        if (!wait_count(&cnt1[d_seg], (unsigned)(l + 1) * per_seg, l, 50)) {
          alive = false;
          break;
        }
        float v[VA];
        const int k0 = ct * VA;
#pragma unroll
        for (int j = 0; j < VA; j += 4) {
          float4 gv = make_float4(0.f, 0.f, 0.f, 0.f), uv = gv;
#pragma unroll
          for (int p = 0; p < 2; p++) {
            if (p >= a.nks) break;
            const float* src = GUb + (size_t)(p * a.kk + d_seg) * 2 * I;
            const float4 g = __ldcg(reinterpret_cast<const float4*>(src + k0 + j));
            const float4 u = __ldcg(reinterpret_cast<const float4*>(src + I + k0 + j));
            gv.x += g.x;
            gv.y += g.y;
            gv.z += g.z;
            gv.w += g.w;
            uv.x += u.x;
            uv.y += u.y;
            uv.z += u.z;
            uv.w += u.w;
          }
          v[j] = silu_ref(gv.x) * uv.x;
          v[j + 1] = silu_ref(gv.y) * uv.y;
          v[j + 2] = silu_ref(gv.z) * uv.z;
          v[j + 3] = silu_ref(gv.w) * uv.w;
        }
        if (ct == 0) *S.hold = 0;
        make_terms<VA>(v, ct, I, 0, S.ba, S.sca, S.faca);
        store_term_scales(S.sca, I, 0, I / 64, tmem + lane_base + kSfba, lane);
        fence_proxy_async();
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (ct == 0) *S.hold = 1;
        if (lane == 0) mbar_arrive(S.aready);
        const bool got = mbar_wait_bounded(S.dfull, jd & 1, a.budget);
        jd++;
        if (!got && lane == 0) fsflag(fs_timeout(l, 49));
        alive = chain_sync_and(got);
        if (!alive) break;
        tc_fence_after();
        const float wseg = d_seg < a.k ? S.wts[l * 16 + d_seg] * a.scaling : 1.0f;
        const float y = fold_runs(tmem + lane_base + kAccD, S.faca) * wseg;
        tc_fence_before();
        __stcg(Yout + (size_t)d_seg * H + d_rb * 128 + r, y);
        signal_count(&cnt2[d_rb / rb_per_part]);
      }

      // ---- routed stack, reducer: h_{l+1} for its rows, then layer l+1's input ----
      if (is_red && NORM) {
        // the counted sums of the reducer's rows: complete when all kk * nb
        // down items have added
        bool got = true;
        float vsum = 0.f;
        if (ct < 32) {
          const unsigned long long* p[1] = {XC.ys + ((size_t)l * H + red_r0 + ct) * kFsYsStride};
          unsigned long long w[1] = {0ull};
          const unsigned want = (unsigned)(a.kk * nb);
          got = poll_words<1>(p, w, a.budget,
                              [&](unsigned long long v) { return (unsigned)(v & 0xFF) == want; });
          if (!got && lane == 0) fsflag(fs_timeout(l, 54));
          vsum = decode_counted<24>(w[0]);
        }
        alive = chain_sync_and(got);
        if (!alive) break;
        if (ct < kFsRedRows) {
          const int row = red_r0 + ct;
          float v = vsum;
          if (a.residual) v += hrow;
          hrow = round_to(v, a.dtype);
          if (l == a.L - 1) {
            if (a.last) store_from_f32(a.y, a.dtype, row, hrow);
            else __stcg(a.Hres + (size_t)((lg + 1) & 1) * H + row, hrow);  // next launch's h_0
          }
        }
        if (l + 1 < a.L && !route_rows(l + 1)) {
          alive = false;
          break;
        }
      } else if (is_red) {
        // every (segment, I block) partial of the reducer's rows: thread ct
        // sums row ct % 32 over the segments and the I blocks of quarter
        // ct / 32 (in that order, all loads in flight), the four quarters then
        // in order
        if (!wait_count(&cnt2[red_r0 / 128], (unsigned)(l + 1) * a.kk * nb, l, 54)) {
          alive = false;
          break;
        }
        {
          constexpr int BQ = VA / 2;  // I blocks of a quarter (nb / 4)
          const int qq = ct >> 5;
          const float* src = Yout + (size_t)(qq * BQ) * H + red_r0 + (ct & 31);
          float part[kFsMaxSeg][BQ];
#pragma unroll
          for (int sg = 0; sg < kFsMaxSeg; sg++)
#pragma unroll
            for (int bb = 0; bb < BQ; bb++)
              part[sg][bb] = sg < a.kk ? __ldcg(src + ((size_t)sg * nb + bb) * H) : 0.f;
          float acc = 0.f;
#pragma unroll
          for (int sg = 0; sg < kFsMaxSeg; sg++)
#pragma unroll
            for (int bb = 0; bb < BQ; bb++)
              if (sg < a.kk) acc += part[sg][bb];
          S.red[ct] = acc;
        }
        named_sync(kBarChain, kChain);
        if (ct < kFsRedRows) {
          const int row = red_r0 + ct;
          float v = ((S.red[ct] + S.red[32 + ct]) + S.red[64 + ct]) + S.red[96 + ct];
          if (a.residual) v += hrow;
          hrow = round_to(v, a.dtype);
          if (l == a.L - 1) {
            if (a.last) store_from_f32(a.y, a.dtype, row, hrow);
            else __stcg(a.Hres + (size_t)((lg + 1) & 1) * H + row, hrow);  // next launch's h_0
          }
        }
        if (l + 1 < a.L && !route_rows(l + 1)) {
          alive = false;
          break;
        }
      }
    }
    // Given routing: the stack's output, this CTA's 128-row block of the last
    // layer, once every down item of its part is done.
    if (!ROUTED && alive && a.last && c < H / 128) {
      const int lg = a.l0 + a.L - 1;
      const float* Yl = a.Yp + (size_t)(lg & 1) * a.kk * H;
      if (wait_count(&cnt2[c / rb_per_part], (unsigned)a.L * per_part, a.L - 1, 52)) {
        const int i = c * kChain + ct;
        float y = __ldcg(Yl + i);
        for (int sg = 1; sg < a.kk; sg++) y += __ldcg(Yl + (size_t)sg * H + i);
        store_from_f32(a.y, a.dtype, i, y);
      }
    }
  }
  __syncthreads();
  // the partner may still write into this CTA's shared memory until it is done
  if constexpr (ROUTED) cluster_sync_fs();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int VX, int R>
const void* pick_va(int va) {
  switch (va) {
    case 4: return reinterpret_cast<const void*>(moe_decode_stack_fp4_kernel<VX, 4, R>);
    case 8: return reinterpret_cast<const void*>(moe_decode_stack_fp4_kernel<VX, 8, R>);
    case 16: return reinterpret_cast<const void*>(moe_decode_stack_fp4_kernel<VX, 16, R>);
    default: return nullptr;
  }
}

// VX: values of x per chain thread (the K part of a gate/up item / 128).
template <int R>
const void* pick_kernel(int H, int I, int nks) {
  switch (H / nks / 128) {
    case 4: return pick_va<4, R>(I / 128);
    case 8: return pick_va<8, R>(I / 128);
    case 16: return pick_va<16, R>(I / 128);
    default: return nullptr;
  }
}

}  // namespace

static_assert(sizeof(FsArgs) <= 32764, "kernel parameters above the 32 KB limit");

int decode_stack_fp4_nks(int I, int kk, int sms) {
  if (kk * (I / 64) * 2 <= sms) return 2;
  if (kk * (I / 64) <= sms) return 1;
  return 0;
}

size_t decode_stack_fp4_smem_bytes(int H, int I, int L, bool routed) {
  return fs_carve(H, I, L, routed, nullptr, nullptr) + 1024;
}

bool decode_stack_fp4_supported(int H, int I, int kk, int sms, bool routed) {
  if (H != 1024 && H != 2048) return false;
  if (I != 512 && I != 1024 && I != 2048) return false;
  if (kk < 1 || kk > 16 || kk * (H / 128) > sms) return false;  // one down item per CTA
  if (decode_stack_fp4_nks(I, kk, sms) == 0) return false;      // one gate/up item per CTA
  if (routed) {
    // CTA pairs: both K halves of every (segment, I block), the last pair of
    // the grid (the router's) without an item; one reducer per CTA
    const int G = sms & ~1;
    // (kk * I / 64 <= 127: the counted layer-output sums stay below 2^47)
    if (kk > kFsMaxSeg || decode_stack_fp4_nks(I, kk, sms) != 2 || 2 * kk * (I / 64) > G - 2 ||
        kk * (I / 64) > 127 ||
        H / kFsRedRows > G - 1)
      return false;
    if (sfbx_of(true) + (uint32_t)(H / 16 + 32) > kTmemCols) return false;
  } else if (sfbx_of(false) + (uint32_t)(H / 16 + I / 16) > kTmemCols) {
    return false;
  }
  return decode_stack_fp4_smem_bytes(H, I, kFsMaxLayers, routed) <= 227 * 1024;
}

cudaError_t launch_decode_stack_fp4(const FsArgs& a, cudaStream_t stream) {
  const void* kern = a.nks <= 0 ? nullptr
                     : !a.routed  ? pick_kernel<0>(a.H, a.I, a.nks)
                     : a.has_norm ? pick_kernel<2>(a.H, a.I, a.nks)
                                  : pick_kernel<1>(a.H, a.I, a.nks);
  if (!kern || a.L < 1 || a.L > kFsMaxLayers || a.L * a.mpl > kFsMaxMaps)
    return cudaErrorInvalidValue;
  if (a.routed && (a.E < 1 || a.E > 256 || a.k > 8 || a.dtype == kF32 ||
                   a.H / kFsRedRows > kFsMaxReducers))
    return cudaErrorInvalidValue;
  const size_t smem = decode_stack_fp4_smem_bytes(a.H, a.I, a.L, a.routed != 0);
  cudaError_t e = ensure_smem_ptr(kern, smem);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  if (decode_stack_fp4_nks(a.I, a.kk, sms) != a.nks || a.kk * (a.H / 128) > sms ||
      !decode_stack_fp4_supported(a.H, a.I, a.kk, sms, a.routed != 0))
    return cudaErrorInvalidValue;
  // The routed stack runs as CTA pairs (clusters of 2) over an even grid.
  const int grid = a.routed ? (sms & ~1) : sms;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.routed ? 2 : 1;
  // Every CTA must be resident (CTAs wait on one another's counters): one per
  // SM (every pair co-scheduled), cooperative launch.
  if (a.routed) {
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
    if (e != cudaSuccess) return e;
    if (2 * clusters < grid) return cudaErrorCooperativeLaunchTooLarge;
  } else {
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
  }
  // dependency counters, and (routed) the exchange area behind them
  const size_t zero = kFsCounters * sizeof(unsigned) +
                      (a.routed ? fs_xchg_u64(a.H, a.E, a.L) * sizeof(unsigned long long) : 0);
  if (a.routed && reinterpret_cast<const char*>(a.XG) !=
                      reinterpret_cast<const char*>(a.bar) + kFsCounters * sizeof(unsigned))
    return cudaErrorInvalidValue;
  e = cudaMemsetAsync(a.bar, 0, zero, stream);
  if (e != cudaSuccess) return e;
  void* args[] = {const_cast<FsArgs*>(&a)};
  e = cudaLaunchKernelExC(&cfg, kern, args);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t read_and_clear_stack_fp4_error(int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_fs_error, sizeof(int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_fs_error, &zero, sizeof(int));
}

}  // namespace nvfp4
