// decode_stack.cu -- serial decode (T = 1) through a stack of sparse MoE
// layers as ONE persistent cooperative launch.
//
// Reference semantics: per layer the routed SwitchGLU gate/up -> SwiGLU ->
// down chain (VLM/MLXLMCommon/SwitchLayers.swift:532-580) with given routing
// and the Laguna combine y = scaling * sum_j w_j * expert_j(x) + shared(x)
// (VLM/MLXLLM/Models/Laguna.swift:204-212); the layer loop is the runtime's
// decode step over the sparse layers (Sources/MLXFastModel/
// LagunaRuntimeModel.swift:11460 -> :11030 -> :10678).  Products follow
// fp_qmm_t (backend/cpu/quantized.cpp:491-533) with f32 accumulation; the
// per-layer output is rounded to the activation dtype as the per-layer
// kernels do.
//
// Why one launch: a decode layer moves 14 MB of expert weights but its
// dependent chain (x -> gate/up -> act -> down -> next x) is short, so
// per-layer kernels are bound by latency, not HBM.  The weights do not depend
// on the activations (the routing is known up front), so here each CTA's
// producer warp streams its share of layer l, l+1, ... into shared-memory
// rings continuously, while the consumer warps run the dependent chain and
// meet the other CTAs at two grid barriers per layer.
//
// Per layer, CTA c owns
//   gate/up units u = c, c + G, ... of kk * I/8 (segment = routed slot or the
//     shared expert; 8 gate rows + the same 8 up rows of that expert), and
//   down items dt = c, c + G, ... of H/16 (16 output rows over all kk
//     segments, one ring unit per segment).
// Consumers: gate/up units (8 warps split K, reduced through shared memory)
// -> act[seg][i] in global memory -> grid barrier -> stage act (x w_j *
// scaling, one power-of-two scale) -> down items -> next x -> grid barrier.
// Cross-CTA data (x, act) is read with L2 loads (.cg): L1 is not coherent.
// Every wait is bounded; on expiry error 4 is latched, the CTA's consumers
// stop and tell their producer, which drains its copies before exit.
#include "common.cuh"
#include "gemv.cuh"
#include "kernels.h"
#include "tma.cuh"

namespace nvfp4 {
namespace {

constexpr int kSCons = 8;                  // consumer warps (2 per SM sub-partition)
constexpr int kSThreads = (kSCons + 1) * 32;
constexpr int kGSlots = 6;                 // gate/up units in flight
constexpr int kDSlots = 12;                // down segment units in flight
constexpr int kBatch = 4;                  // gate/up units computed together
constexpr int kDGroups = kSCons / 4;       // down: groups of 4 warps, each over every kDGroups-th segment
static_assert(kSCons % 4 == 0 && kSCons >= 8, "down groups are 4 warps (one per chunk of I=512)");
constexpr int kDAcc = 2;                   // down: accumulator sets per warp
constexpr int kXChunks = 2;                // x: 8-value chunks per consumer thread (H <= 4096)
constexpr int kAChunks = 4;                // act: chunks per thread (kk * I <= 8192)
constexpr int kErrTimeout = 4;
constexpr int kErrIndex = 2;

__device__ int g_stack_error = 0;
__device__ __forceinline__ void sflag(int code) { atomicCAS(&g_stack_error, 0, code); }

__host__ __device__ constexpr int round128(int v) { return (v + 127) / 128 * 128; }

// Eight consecutive elements from global memory through L2 only.
__device__ __forceinline__ void load8_cg(const void* x, int dtype, int64_t off, float (&f)[8]) {
  if (dtype == kF32) {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + off));
    const float4 b =
        __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + off + 4));
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    const uint4 v =
        __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(x) + off));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      float2 p;
      if (dtype == kBF16) p = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      else p = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  }
}

// Named barrier over `count` threads that also ANDs a predicate across them.
__device__ __forceinline__ bool named_sync_and(int id, int count, bool pred) {
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

__device__ __forceinline__ float round_as(float v, int dtype) {
  if (dtype == kBF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dtype == kF16) return __half2float(__float2half_rn(v));
  return v;
}

__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct StackSmem {
  uint64_t *fullG, *emptyG, *fullD, *emptyD;
  uint8_t *slotsG, *slotsD;
  __half *xs, *xa;
  float *colscale, *segw, *red, *red2;
  int* colmax;
  volatile int* abort;     // consumers -> producer: stop
  volatile int* bar_ok;    // grid-barrier outcome, thread 0 -> consumers
  volatile int* hold;      // consumers in a grid barrier: producer holds refills
  uint32_t* inds;          // [L][k] routing of every layer, staged at start
  float* wts;              // [L][k]
};

}  // namespace

// Ring units hold their rows unpadded (rows of one expert are contiguous in
// HBM, so a unit is 2-4 bulk copies instead of one per row); the fragment
// reads then see 2-way bank conflicts, cheaper than 8x the copy count.
size_t decode_stack_smem_bytes(int H, int I, int kk) {
  const int slotG = round128(16 * (H / 2) + 16 * (H / 16));
  const int slotD = round128(16 * (I / 2) + 16 * (I / 16));
  size_t b = 512;  // barriers + flags
  b += (size_t)kGSlots * slotG + (size_t)kDSlots * slotD;
  b += round128((H + kXPad) * 2) + round128(kk * (I + kXPad) * 2);
  b += 64 * 4 + (size_t)(kSCons + 1) * kBatch * 4 * 32 * 4;  // colscale/colmax/segw, red, red2
  b += (size_t)kStackMaxLayers * 16 * 8;             // routing tables
  return b;
}

namespace {

__global__ void __launch_bounds__(kSThreads, 1) moe_decode_stack_kernel(
    const __grid_constant__ StackArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int H = a.H, I = a.I, kk = a.kk;
  const int rpG = H / 2, spG = H / 16;
  const int rpD = I / 2, spD = I / 16;
  const int slotG = round128(16 * rpG + 16 * spG);
  const int slotD = round128(16 * rpD + 16 * spD);
  const uint32_t bytesG = (uint32_t)(16 * (H / 2) + 16 * (H / 16));
  const uint32_t bytesD = (uint32_t)(16 * (I / 2) + 16 * (I / 16));
  const int ldxG = H + kXPad, ldxD = I + kXPad;

  StackSmem S;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  S.fullG = bars;
  S.emptyG = S.fullG + kGSlots;
  S.fullD = S.emptyG + kGSlots;
  S.emptyD = S.fullD + kDSlots;
  S.abort = reinterpret_cast<volatile int*>(S.emptyD + kDSlots);
  S.bar_ok = S.abort + 1;
  S.hold = S.abort + 2;
  unsigned char* p = smem + 512;
  S.slotsG = p;
  p += (size_t)kGSlots * slotG;
  S.slotsD = p;
  p += (size_t)kDSlots * slotD;
  S.xs = reinterpret_cast<__half*>(p);
  p += round128(ldxG * 2);
  S.xa = reinterpret_cast<__half*>(p);
  p += round128(kk * ldxD * 2);
  S.colscale = reinterpret_cast<float*>(p);
  S.colmax = reinterpret_cast<int*>(S.colscale + 8);
  S.segw = S.colscale + 16;  // [<= 48]
  S.red = S.colscale + 64;   // [kSCons][kBatch][4][32]
  S.red2 = S.red + kSCons * kBatch * 4 * 32;  // [kBatch][4][32] sums over warps
  S.inds = reinterpret_cast<uint32_t*>(S.red2 + kBatch * 4 * 32);
  S.wts = reinterpret_cast<float*>(S.inds + kStackMaxLayers * 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tps = I / 8;              // gate/up row groups per segment
  const int nG = kk * tps;            // gate/up units per layer
  const int nD = H / 16;              // down items per layer
  const int G = gridDim.x;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kGSlots; i++) {
      mbar_init(&S.fullG[i], 1);
      mbar_init(&S.emptyG[i], kSCons);
    }
    for (int i = 0; i < kDSlots; i++) {
      mbar_init(&S.fullD[i], 1);
      mbar_init(&S.emptyD[i], 4);  // the 4 warps of the segment's group
    }
    *S.abort = 0;
    *S.hold = 0;
    fence_barrier_init();
  }
  // Every layer's routing into shared memory once: a global load costs ~1 us
  // while the weight stream fills the memory system, and the producer and the
  // combine need these values in the middle of their pipelines.
  for (int i = threadIdx.x; i < a.L * a.k; i += blockDim.x) {
    const int l = i / a.k, j = i - l * a.k;
    S.inds[l * 16 + j] = a.layer[l].inds[j];
    S.wts[l * 16 + j] = a.layer[l].wts[j];
  }
  __syncthreads();

  if (warp == kSCons) {
    // ------------------------------ producer ------------------------------
    // Streams, in consumption order, every unit this CTA will compute:
    // gate/up units of layer 0, its down units, gate/up units of layer 1, ...
    uint32_t jg = 0, jd = 0;
    bool ok = true;
    // While this CTA's consumers wait in a grid barrier, the barrier's atomics
    // and polls are the critical path; a refill burst issued at that moment
    // (the slots the finished phase released) queues ahead of them in the
    // memory system.  The refills are for units needed a layer later, so they
    // wait until the barrier has passed (bounded: a missed release only costs
    // time).
    auto hold_refills = [&]() {
      if (lane == 0) {
        const long long h0 = clock64();
        while (*S.hold && !*S.abort && clock64() - h0 < 400000) __nanosleep(64);
      }
      __syncwarp();
    };
    for (int l = 0; l < a.L && ok; l++) {
      const StackLayer& ly = a.layer[l];
      for (int u = blockIdx.x; u < nG && ok; u += G) {
        const int seg = u / tps;
        const int64_t i0 = (int64_t)(u - seg * tps) * 8;
        const int s = jg % kGSlots;
        if (*S.abort ||
            (jg >= kGSlots && !mbar_wait_bounded(&S.emptyG[s], ((jg / kGSlots) - 1) & 1))) {
          ok = false;
          break;
        }
        const uint8_t *gw, *gs, *uw, *us;
        if (seg < a.k) {
          uint32_t e = S.inds[l * 16 + seg];
          if (e >= (uint32_t)a.E) {
            if (lane == 0) sflag(kErrIndex);
            e = 0;  // keep the pipeline consistent; the output is flagged invalid
          }
          gw = ly.gw + (int64_t)e * a.gw_stride;
          gs = ly.gs + (int64_t)e * a.gs_stride;
          uw = ly.uw + (int64_t)e * a.gw_stride;
          us = ly.us + (int64_t)e * a.gs_stride;
        } else {
          gw = ly.sgw;
          gs = ly.sgs;
          uw = ly.suw;
          us = ly.sus;
        }
        hold_refills();
        uint8_t* dst = S.slotsG + (size_t)s * slotG;
        // rows 0..7 gate rows i0.., rows 8..15 the same up rows; then scales
        if (lane == 0) {
          mbar_arrive_expect_tx(&S.fullG[s], bytesG);
          bulk_g2s(dst, gw + i0 * rpG, (uint32_t)(8 * rpG), &S.fullG[s]);
          bulk_g2s(dst + 8 * rpG, uw + i0 * rpG, (uint32_t)(8 * rpG), &S.fullG[s]);
          bulk_g2s(dst + 16 * rpG, gs + i0 * spG, (uint32_t)(8 * spG), &S.fullG[s]);
          bulk_g2s(dst + 16 * rpG + 8 * spG, us + i0 * spG, (uint32_t)(8 * spG), &S.fullG[s]);
        }
        __syncwarp();
        jg++;
      }
      for (int dt = blockIdx.x; dt < nD && ok; dt += G) {
        for (int seg = 0; seg < kk; seg++) {
          const int s = jd % kDSlots;
          if (*S.abort ||
              (jd >= kDSlots && !mbar_wait_bounded(&S.emptyD[s], ((jd / kDSlots) - 1) & 1))) {
            ok = false;
            break;
          }
          const uint8_t *wb, *sb;
          if (seg < a.k) {
            uint32_t e = S.inds[l * 16 + seg];
            if (e >= (uint32_t)a.E) e = 0;  // flagged by the gate/up side
            wb = ly.dw + (int64_t)e * a.dw_stride;
            sb = ly.ds + (int64_t)e * a.ds_stride;
          } else {
            wb = ly.sdw;
            sb = ly.sds;
          }
          hold_refills();
          uint8_t* dst = S.slotsD + (size_t)s * slotD;
          if (lane == 0) {
            const int64_t row0 = (int64_t)dt * 16;
            mbar_arrive_expect_tx(&S.fullD[s], bytesD);
            bulk_g2s(dst, wb + row0 * rpD, (uint32_t)(16 * rpD), &S.fullD[s]);
            bulk_g2s(dst + 16 * rpD, sb + row0 * spD, (uint32_t)(16 * spD), &S.fullD[s]);
          }
          __syncwarp();
          jd++;
        }
      }
    }
    // Drain: no copy may still be landing in this CTA's memory at exit
    // (immediate unless the consumers stopped early).
    for (uint32_t i = 0; i < min(jg, (uint32_t)kGSlots); i++) {
      const uint32_t q = jg - 1 - i;
      mbar_wait_bounded(&S.fullG[q % kGSlots], (q / kGSlots) & 1, 200000000LL);
    }
    for (uint32_t i = 0; i < min(jd, (uint32_t)kDSlots); i++) {
      const uint32_t q = jd - 1 - i;
      mbar_wait_bounded(&S.fullD[q % kDSlots], (q / kDSlots) & 1, 200000000LL);
    }
    return;
  }

  // ------------------------------ consumers ------------------------------
  const int nthr = kSCons * 32;
  const int g = lane >> 2, t = lane & 3;
  const int nchG = H / kChunk;
  const int c0 = (warp * nchG) / kSCons, c1 = ((warp + 1) * nchG) / kSCons;
  const int nchD = I / kChunk;
  uint32_t jg = 0, jd = 0;
  unsigned phase = 0;  // grid barriers passed

  // One grid barrier: every consumer thread's global writes, then this CTA's
  // arrival; thread 0 waits (bounded) for all G CTAs.  Returns false on expiry.
  auto grid_barrier = [&](unsigned* ctr) -> bool {
    if (threadIdx.x == 0) *S.hold = 1;
    named_sync(1, nthr);
    if (threadIdx.x == 0) {
      red_release_add(ctr, 1u);  // orders this CTA's writes (bar.sync above) first
      const unsigned target = (unsigned)G * (phase / 2 + 1);
      bool ok = true;
      if (ld_acquire_gpu(ctr) < target) {
        const long long start = clock64();
        while (ld_acquire_gpu(ctr) < target) {
          if (clock64() - start > 2000000000LL) {
            ok = false;
            break;
          }
          __nanosleep(32);
        }
      }
      *S.bar_ok = ok;
      *S.hold = 0;
      if (!ok) sflag(kErrTimeout);
    }
    named_sync(1, nthr);
    phase++;
    return *S.bar_ok != 0;
  };

  auto stop = [&]() {
    if (threadIdx.x == 0) *S.abort = 1;
  };

  for (int l = 0; l < a.L; l++) {
    const StackLayer& ly = a.layer[l];
    const void* xin = l == 0 ? a.x0 : a.xb[(l - 1) & 1];
    void* xout = l == a.L - 1 ? a.y : a.xb[l & 1];

    // ---- stage x (one column, f16 x 2^-e) ----
    // Each thread keeps its chunks of x in registers; max |x| (over the
    // values as stored) comes from them, one shared-memory reduction, instead
    // of a separate global read after the barrier.
    if (threadIdx.x == 0) S.colmax[0] = 0;
    named_sync(1, nthr);
    float xv[kXChunks][8];
    {
      float m = 0.f;
#pragma unroll
      for (int c = 0; c < kXChunks; c++) {
        const int v = threadIdx.x + c * nthr;
        if (v >= H / 8) continue;
        load8_cg(xin, a.dtype, (int64_t)v * 8, xv[c]);
#pragma unroll
        for (int i = 0; i < 8; i++) m = fmaxf(m, fabsf(xv[c][i]));
      }
      warp_atomic_max(&S.colmax[0], m, true);
    }
    named_sync(1, nthr);
    const float xscale = ldexpf(1.0f, pow2_exponent(__int_as_float(S.colmax[0])));
#pragma unroll
    for (int c = 0; c < kXChunks; c++) {
      const int v = threadIdx.x + c * nthr;
      if (v < H / 8) store8_f16(S.xs, v * 8, xv[c], 1.0f / xscale);
    }
    named_sync(1, nthr);

    // ---- gate/up + SwiGLU units ----
    // Every warp takes its K range of up to kBatch of this CTA's units at once
    // (one accumulator set per unit), then one reduction serves the batch:
    // warp b sums unit b's partials in warp order 0..7.
    bool alive = true;
    const int nu = blockIdx.x < nG ? (nG - 1 - blockIdx.x) / G + 1 : 0;
    for (int ub = 0; ub < nu && alive; ub += kBatch) {
      const int nb = min(kBatch, nu - ub);
      Acc acc[kBatch];
#pragma unroll
      for (int b = 0; b < kBatch; b++) {
        acc[b].zero();
        if (b >= nb || !alive) continue;
        const uint32_t q = jg + b;
        if (!mbar_wait_bounded(&S.fullG[q % kGSlots], (q / kGSlots) & 1)) {
          if (lane == 0) sflag(kErrTimeout);
          alive = false;
        }
      }
      if (alive) {
        // units interleaved inside each chunk: kBatch independent MMA chains
        const __half* xcol = g == 0 ? S.xs : nullptr;
        for (int ch = c0; ch < c1; ch++) {
#pragma unroll
          for (int b = 0; b < kBatch; b++) {
            if (b >= nb) continue;
            const uint8_t* tile = S.slotsG + (size_t)((jg + b) % kGSlots) * slotG;
            Chunk c;
            load_chunk_smem(c, tile, rpG, spG, g, ch, t);
            compute_chunk(acc[b], c, xcol, ch, t);
          }
        }
        __syncwarp();
        if (lane == 0)
          for (int b = 0; b < nb; b++) mbar_arrive(&S.emptyG[(jg + b) % kGSlots]);
      }
      alive = named_sync_and(1, nthr, alive);
      if (!alive) break;
#pragma unroll
      for (int b = 0; b < kBatch; b++) {
        if (b >= nb) continue;
        float d[4];
        acc[b].fold(d);
#pragma unroll
        for (int r = 0; r < 4; r++) S.red[((warp * kBatch + b) * 4 + r) * 32 + lane] = d[r];
      }
      named_sync(1, nthr);
      // (unit b, fragment value r) pairs over the warps: each summed over the
      // consumer warps in order
      for (int br = warp; br < 4 * nb; br += kSCons) {
        const int b = br >> 2, r = br & 3;
        float s = S.red[((0 * kBatch + b) * 4 + r) * 32 + lane];
#pragma unroll
        for (int w = 1; w < kSCons; w++) s += S.red[((w * kBatch + b) * 4 + r) * 32 + lane];
        S.red2[(b * 4 + r) * 32 + lane] = s;
      }
      named_sync(1, nthr);
      if (warp < nb) {
        const int u = blockIdx.x + (ub + warp) * G;
        const int seg = u / tps;
        const int64_t i0 = (int64_t)(u - seg * tps) * 8;
        float d[4];
#pragma unroll
        for (int r = 0; r < 4; r++) d[r] = S.red2[(warp * 4 + r) * 32 + lane];
        const float av = silu_ref(d[0] * xscale) * (d[2] * xscale);
        if (t == 0) __stcg(a.act + (int64_t)seg * I + i0 + g, av);
      }
      named_sync(1, nthr);
      jg += nb;
    }
    if (!alive || !grid_barrier(&a.bar[0])) {
      stop();
      break;
    }

    // ---- down + combine items ----
    if (blockIdx.x < nD) {
      // act columns x (w_j * scaling) (1 for the shared expert), one scale.
      if (threadIdx.x < kk)
        S.segw[threadIdx.x] = threadIdx.x < a.k ? S.wts[l * 16 + threadIdx.x] * ly.scaling : 1.0f;
      if (threadIdx.x == 0) S.colmax[0] = 0;
      named_sync(1, nthr);
      // act of every segment into registers; max |act * w_seg| from them
      const int per = I / 8;
      float av[kAChunks][8];
      {
        float m = 0.f;
#pragma unroll
        for (int c = 0; c < kAChunks; c++) {
          const int it = threadIdx.x + c * nthr;
          if (it >= kk * per) continue;
          const int sg = it / per, v = it - sg * per;
          load8_cg(a.act, kF32, (int64_t)sg * I + (int64_t)v * 8, av[c]);
#pragma unroll
          for (int i = 0; i < 8; i++) m = fmaxf(m, fabsf(av[c][i] * S.segw[sg]));
        }
        warp_atomic_max(&S.colmax[0], m, true);
      }
      named_sync(1, nthr);
      const float ascale = ldexpf(1.0f, pow2_exponent(__int_as_float(S.colmax[0])));
#pragma unroll
      for (int c = 0; c < kAChunks; c++) {
        const int it = threadIdx.x + c * nthr;
        if (it < kk * per) {
          const int sg = it / per, v = it - sg * per;
          store8_f16(S.xa + (size_t)sg * ldxD, v * 8, av[c], S.segw[sg] / ascale);
        }
      }
      named_sync(1, nthr);

      const int grp = warp >> 2, wq = warp & 3;  // kDGroups groups of 4 warps
      for (int dt = blockIdx.x; dt < nD && alive; dt += G) {
        // this group's segments grp, grp + kDGroups, ... one at a time (wait,
        // compute, release: no ring size can stall it), alternating between
        // two accumulator sets
        Acc accd[kDAcc];
#pragma unroll
        for (int i = 0; i < kDAcc; i++) accd[i].zero();
        int ai = 0;
        for (int seg = grp; seg < kk; seg += kDGroups, ai ^= 1) {
          const uint32_t q = jd + seg;
          const int s = q % kDSlots;
          if (!mbar_wait_bounded(&S.fullD[s], (q / kDSlots) & 1)) {
            if (lane == 0) sflag(kErrTimeout);
            alive = false;
            break;
          }
          const uint8_t* tile = S.slotsD + (size_t)s * slotD;
          const __half* xcol = g == 0 ? S.xa + (size_t)seg * ldxD : nullptr;
          for (int ch = wq; ch < nchD; ch += 4) {
            Chunk c;
            load_chunk_smem(c, tile, rpD, spD, g, ch, t);
            if (ai == 0) compute_chunk(accd[0], c, xcol, ch, t);
            else compute_chunk(accd[1], c, xcol, ch, t);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&S.emptyD[s]);
        }
        jd += kk;
        alive = named_sync_and(1, nthr, alive);
        if (!alive) break;
        float d[4], e4[4];
        accd[0].fold(d);
        accd[1].fold(e4);
#pragma unroll
        for (int r = 0; r < 4; r++) d[r] += e4[r];
#pragma unroll
        for (int r = 0; r < 4; r++) S.red[(warp * 4 + r) * 32 + lane] = d[r];
        named_sync(1, nthr);
        if (warp < 4) {  // warp r sums fragment value r over the warps in order
          float s = S.red[(0 * 4 + warp) * 32 + lane];
#pragma unroll
          for (int w = 1; w < kSCons; w++) s += S.red[(w * 4 + warp) * 32 + lane];
          S.red2[warp * 32 + lane] = s;
        }
        named_sync(1, nthr);
        if (warp == 0) {
#pragma unroll
          for (int r = 0; r < 4; r++) d[r] = S.red2[r * 32 + lane];
          if (t == 0) {
            const int64_t h0 = (int64_t)dt * 16;
            store_from_f32(xout, a.dtype, h0 + g, d[0] * ascale);
            store_from_f32(xout, a.dtype, h0 + g + 8, d[2] * ascale);
          }
        }
        named_sync(1, nthr);
      }
    }
    if (!alive || !grid_barrier(&a.bar[1])) {
      stop();
      break;
    }
  }
}

}  // namespace

cudaError_t launch_decode_stack(const StackArgs& a, cudaStream_t stream) {
  const size_t smem = decode_stack_smem_bytes(a.H, a.I, a.kk);
  cudaError_t e = ensure_smem(moe_decode_stack_kernel, smem);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  // Every CTA must be resident (grid barriers): one per SM, cooperative launch.
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, moe_decode_stack_kernel, kSThreads,
                                                    smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
  // Barrier counters and the per-layer maxima start at zero (contiguous).
  e = cudaMemsetAsync(a.bar, 0, (2 + 2 * kStackMaxLayers) * sizeof(unsigned), stream);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)sms);
  cfg.blockDim = dim3(kSThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeCooperative;
  attr.val.cooperative = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, moe_decode_stack_kernel, a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t read_and_clear_stack_error(int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_stack_error, sizeof(int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_stack_error, &zero, sizeof(int));
}

}  // namespace nvfp4
