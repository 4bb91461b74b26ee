// qqmm.cu -- NVFP4 x NVFP4 matmul (MLX qqmm / QQMatmul, mode "nvfp4") on the
// block-scaled tensor cores of sm_100a.
//
// Semantics (backend/cpu/quantized.cpp:1322-1360): the activations x [M, K]
// are fake-quantised to NVFP4 per row group of 16 (fp_quantize_dequantize,
// quantized.cpp:1093-1129; to_fp4_e2m1, :1064-1091), then multiplied with the
// NVFP4 weights W [N, K] (y = xhat . dequant(W)^T, output dtype = x dtype).
// Every product xhat_k * w_k is exact in f32 (E2M1 x E2M1 x E4M3 x E4M3 has at
// most 12 significant bits), so the tensor-core result equals the exact dot
// product up to f32 accumulation order.
//
// 1. qx_quantize_kernel: one thread per 16-element group, the MLX steps in
//    f32: amax = max |x| (NaN ignored, as std::max does), scale = amax / 6,
//    sb = ToFP8(scale), s = FromFP8(sb), code_j = to_fp4_e2m1(x_j / s)
//    (0 when s == 0).  Writes packed codes [M, K/2] (low nibble first) and
//    scale bytes [M, K/16] -- the same layout as the weights.
// 2. qqmm_kernel: one CTA per (128 weight rows, bn tokens, K split).  A warp
//    issues TMA loads of 256-code K boxes (W codes, x codes, both scale
//    tiles) into a 4-stage ring; four warps copy each stage's scale bytes into
//    tensor memory in the layout the block-scaled MMA reads (scale of row m,
//    block j at lanes m%32 + 32r for r = 0..3, column m/32, byte j); one
//    thread issues tcgen05.mma kind::mxf4nvf4 (M=128, N=bn, K=64, UE4M3
//    scales per 16) into a TMEM accumulator; the same four warps read it back
//    (lane = weight row, column = token) and store y, or, with K split over
//    several CTAs, write f32 partials that the tile's last CTA sums in split
//    order (deterministic).
#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"

namespace nvfp4 {
namespace {

constexpr int kQBM = 128;        // weight rows per tile (the block-scaled MMA's M)
constexpr int kQBoxBytes = 128;  // one K box: 256 codes = 128 bytes per row
constexpr int kQStages = 4;
constexpr int kQThreads = 192;   // warp 0 TMA, warp 1 MMA, warps 2-5 scales + epilogue
constexpr int kQAccCols = 128;   // accumulator columns (bn <= 128)
constexpr int kQSfCols = 32;     // per stage: 16 SFA + 16 SFB columns
constexpr int kQTmemCols = 256;
constexpr int kErrTimeout = 4;
constexpr long long kDrainBudget = 200000000LL;

__device__ int g_qqmm_error = 0;
__device__ __forceinline__ void qflag(int code) { atomicCAS(&g_qqmm_error, 0, code); }

__global__ void qx_quantize_kernel(uint8_t* __restrict__ qx, uint8_t* __restrict__ sx,
                                   const void* __restrict__ x, int dtype, int64_t groups) {
  for (int64_t gi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; gi < groups;
       gi += (int64_t)gridDim.x * blockDim.x) {
    float v[16];
    load8(x, dtype, gi * 16, *reinterpret_cast<float(*)[8]>(&v[0]));
    load8(x, dtype, gi * 16 + 8, *reinterpret_cast<float(*)[8]>(&v[8]));
    float amax = -INFINITY;
#pragma unroll
    for (int j = 0; j < 16; j++) amax = fmaxf(amax, fabsf(v[j]));
    uint32_t sb = e4m3_encode(amax / 6.0f);
    const float s = scale_to_f32(sb);
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int j = 0; j < 16; j++) {
      const uint32_t c = fp4_code_mlx(s == 0.f ? 0.0f : v[j] / s);
      if (j < 8) w0 |= c << (4 * j);
      else w1 |= c << (4 * (j - 8));
    }
    // A negative scale byte (only an all-NaN group gets one: amax = -inf)
    // is not a UE4M3 value: code * (-s) == (-code) * s, so flip the codes'
    // signs and keep the magnitude byte.
    if (sb & 0x80u) {
      sb &= 0x7Fu;
      w0 ^= 0x88888888u;
      w1 ^= 0x88888888u;
    }
    *reinterpret_cast<uint2*>(qx + gi * 8) = make_uint2(w0, w1);
    sx[gi] = (uint8_t)sb;
  }
}

struct QSmem {
  uint8_t* stage[kQStages];
  uint64_t *full, *empty, *sf_ready, *acc_full;
  uint32_t* tmem_slot;
  int* flag;
};

__global__ void __launch_bounds__(kQThreads, 1) qqmm_kernel(const __grid_constant__ QqmmArgs a) {
  extern __shared__ __align__(1024) unsigned char qsmem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(qsmem_raw) + 1023) & ~(uintptr_t)1023);
  const int bn = a.bn;
  const uint32_t offB = kQBM * kQBoxBytes;                 // 16 KB of W codes
  const uint32_t offSA = offB + (uint32_t)bn * kQBoxBytes;  // x codes: bn x 128 B
  const uint32_t offSB = offSA + kQBM * 16;                 // W scales: 128 x 16 B
  const uint32_t stage_bytes = (offSB + (uint32_t)bn * 16 + 1023) & ~1023u;
  const uint32_t tx_bytes = offSB + (uint32_t)bn * 16;
  QSmem S;
  for (int s = 0; s < kQStages; s++) S.stage[s] = base + (size_t)s * stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + (size_t)kQStages * stage_bytes);
  S.full = bars;
  S.empty = S.full + kQStages;
  S.sf_ready = S.empty + kQStages;
  S.acc_full = S.sf_ready + kQStages;
  S.tmem_slot = reinterpret_cast<uint32_t*>(S.acc_full + 1);
  S.flag = reinterpret_cast<int*>(S.tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = a.n_tiles * a.m_tiles;
  const int tile = blockIdx.x / a.splits, split = blockIdx.x - tile * a.splits;
  const int nt = tile % a.n_tiles, mt = tile / a.n_tiles;
  const int nkb = (int)(a.K / 256);
  const int kb0 = (int)((int64_t)split * nkb / a.splits);
  const int kb1 = (int)((int64_t)(split + 1) * nkb / a.splits);
  const int nk = kb1 - kb0;
  (void)tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kQStages; s++) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
      mbar_init(&S.sf_ready[s], 4);
    }
    mbar_init(S.acc_full, 1);
    *S.flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(S.tmem_slot, kQTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *S.tmem_slot;
  const uint32_t tsf0 = tmem + kQAccCols;

  if (warp == 0) {
    // ---- TMA producer ----
    if (lane == 0) {
      prefetch_map(&a.ma);
      prefetch_map(&a.mb);
      prefetch_map(&a.msa);
      prefetch_map(&a.msb);
      int issued = 0;
      for (int i = 0; i < nk; i++) {
        const int s = i % kQStages;
        if (i >= kQStages && !mbar_wait_bounded(&S.empty[s], ((i / kQStages) - 1) & 1)) {
          qflag(kErrTimeout);
          break;
        }
        const int kb = kb0 + i;
        uint8_t* st = S.stage[s];
        mbar_arrive_expect_tx(&S.full[s], tx_bytes);
        tma_load_2d(st, &a.ma, kb * kQBoxBytes, nt * kQBM, &S.full[s]);
        tma_load_2d(st + offB, &a.mb, kb * kQBoxBytes, mt * bn, &S.full[s]);
        tma_load_2d(st + offSA, &a.msa, kb * 16, nt * kQBM, &S.full[s]);
        tma_load_2d(st + offSB, &a.msb, kb * 16, mt * bn, &S.full[s]);
        issued++;
      }
      // no copy may still be landing at exit
      for (int i = issued - 1; i >= 0 && i >= issued - kQStages; i--)
        mbar_wait_bounded(&S.full[i % kQStages], (i / kQStages) & 1, kDrainBudget);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      const uint32_t idesc = idesc_mxf4nvf4(kQBM, bn);
      for (int i = 0; i < nk; i++) {
        const int s = i % kQStages;
        if (!mbar_wait_bounded(&S.sf_ready[s], (i / kQStages) & 1)) {
          qflag(kErrTimeout);
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(S.stage[s]), sbb = smem_u32(S.stage[s] + offB);
        const uint32_t sf = tsf0 + (uint32_t)(s * kQSfCols);
#pragma unroll
        for (int k4 = 0; k4 < 4; k4++)
          umma_mxf4nvf4(tmem, smem_desc_sw128(sa + 32 * k4), smem_desc_sw128(sbb + 32 * k4), idesc,
                        sf + 4 * k4, sf + 16 + 4 * k4, (i > 0 || k4 > 0) ? 1u : 0u);
        umma_commit(&S.empty[s]);
      }
      umma_commit(S.acc_full);
    }
  } else {
    // ---- scale factors into tensor memory, then the epilogue ----
    const int q = warp & 3;  // this warp's TMEM lane quarter
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    bool ok = true;
    for (int i = 0; i < nk && ok; i++) {
      const int s = i % kQStages;
      if (!mbar_wait_bounded(&S.full[s], (i / kQStages) & 1)) {
        qflag(kErrTimeout);
        ok = false;
        break;
      }
      const uint8_t* st = S.stage[s];
      uint32_t ra[16], rb[16];
#pragma unroll
      for (int c = 0; c < 4; c++) {
        // row lane + 32c: its 16 scale bytes = four MMA steps x 4 blocks
        const uint4 va = *reinterpret_cast<const uint4*>(st + offSA + 16 * (lane + 32 * c));
        ra[0 + c] = va.x;
        ra[4 + c] = va.y;
        ra[8 + c] = va.z;
        ra[12 + c] = va.w;
        const int tok = lane + 32 * c;
        uint4 vb = make_uint4(0u, 0u, 0u, 0u);
        if (tok < bn) vb = *reinterpret_cast<const uint4*>(st + offSB + 16 * tok);
        rb[0 + c] = vb.x;
        rb[4 + c] = vb.y;
        rb[8 + c] = vb.z;
        rb[12 + c] = vb.w;
      }
      const uint32_t col = tsf0 + (uint32_t)(s * kQSfCols);
      tmem_st16(lane_base + col, ra);
      tmem_st16(lane_base + col + 16, rb);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.sf_ready[s]);
    }
    if (!mbar_wait_bounded(S.acc_full, 0)) {
      qflag(kErrTimeout);
      ok = false;
    }
    tc_fence_after();
    const int64_t n = (int64_t)nt * kQBM + 32 * q + lane;
    const int64_t m0 = (int64_t)mt * bn;
    if (ok && nk > 0) {
      if (a.splits == 1) {
        for (int c0 = 0; c0 < bn; c0 += 8) {
          float v[8];
          tmem_ld8(tmem + lane_base + (uint32_t)c0, v);
#pragma unroll
          for (int j = 0; j < 8; j++) {
            const int64_t m = m0 + c0 + j;
            if (m < a.M && n < a.N) store_from_f32(a.out, a.dtype, m * a.N + n, v[j]);
          }
        }
      } else {
        float* part = a.partial + ((size_t)tile * a.splits + split) * (size_t)bn * kQBM;
        for (int c0 = 0; c0 < bn; c0 += 8) {
          float v[8];
          tmem_ld8(tmem + lane_base + (uint32_t)c0, v);
#pragma unroll
          for (int j = 0; j < 8; j++) part[(size_t)(c0 + j) * kQBM + 32 * q + lane] = v[j];
        }
        __threadfence();
        named_sync(1, 128);
        if (warp == 2 && lane == 0) {
          const unsigned old = atomicAdd(&a.ticket[tile], 1u);
          *S.flag = (old == (unsigned)(a.splits - 1)) ? 1 : 0;
        }
        named_sync(1, 128);
        if (*S.flag) {
          __threadfence();
          const float* tp = a.partial + (size_t)tile * a.splits * (size_t)bn * kQBM;
          for (int c = 0; c < bn; c++) {
            float acc = 0.f;
            for (int sp = 0; sp < a.splits; sp++)
              acc += __ldcg(tp + ((size_t)sp * bn + c) * kQBM + 32 * q + lane);
            const int64_t m = m0 + c;
            if (m < a.M && n < a.N) store_from_f32(a.out, a.dtype, m * a.N + n, acc);
          }
        }
      }
    } else if (ok && n < a.N) {
      // empty K range: y = 0
      for (int c = 0; c < bn; c++)
        if (m0 + c < a.M) store_from_f32(a.out, a.dtype, (m0 + c) * a.N + n, 0.f);
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kQTmemCols);
  }
}

}  // namespace

int qqmm_tile_tokens(int64_t M) {
  if (M <= 8) return 8;
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  return 128;
}

size_t qqmm_smem_bytes(int bn) {
  const size_t stage = ((size_t)kQBM * kQBoxBytes + (size_t)bn * kQBoxBytes + kQBM * 16 +
                        (size_t)bn * 16 + 1023) & ~(size_t)1023;
  return 1024 + kQStages * stage + (3 * kQStages + 1) * 8 + 16;
}

void qqmm_plan(int64_t M, int64_t N, int64_t K, int sms, int* bn, int* n_tiles, int* m_tiles,
               int* splits) {
  *bn = qqmm_tile_tokens(M);
  *n_tiles = (int)((N + kQBM - 1) / kQBM);
  *m_tiles = (int)((M + *bn - 1) / *bn);
  const int tiles = *n_tiles * *m_tiles;
  const int nkb = (int)(K / 256);
  int sp = tiles >= sms ? 1 : sms / tiles;
  sp = std::max(1, std::min(sp, nkb));
  *splits = sp;
}

cudaError_t launch_qx_quantize(uint8_t* qx, uint8_t* sx, const void* x, int dtype, int64_t M,
                               int64_t K, cudaStream_t stream) {
  const int64_t groups = M * (K / 16);
  if (groups == 0) return cudaSuccess;
  const int threads = 256;
  const int blocks = (int)std::min<int64_t>((groups + threads - 1) / threads, 148 * 16);
  qx_quantize_kernel<<<blocks, threads, 0, stream>>>(qx, sx, x, dtype, groups);
  return cudaGetLastError();
}

cudaError_t launch_qqmm(const QqmmArgs& a, cudaStream_t stream) {
  const size_t smem = qqmm_smem_bytes(a.bn);
  cudaError_t e = ensure_smem(qqmm_kernel, smem);
  if (e != cudaSuccess) return e;
  if (a.splits > 1) {
    e = cudaMemsetAsync(a.ticket, 0, sizeof(unsigned) * (size_t)a.n_tiles * a.m_tiles, stream);
    if (e != cudaSuccess) return e;
  }
  const unsigned grid = (unsigned)a.n_tiles * (unsigned)a.m_tiles * (unsigned)a.splits;
  qqmm_kernel<<<grid, kQThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t read_and_clear_qqmm_error(int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_qqmm_error, sizeof(int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_qqmm_error, &zero, sizeof(int));
}

}  // namespace nvfp4
