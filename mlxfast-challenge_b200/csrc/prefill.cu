// prefill.cu -- the sorted-expert (grouped) NVFP4 GEMM on sm_100a tensor
// cores (tcgen05, TMEM accumulators) and the MoE prefill plumbing around it.
//
// Reference semantics: gather_qmm over tokens sorted by expert
// (VMLX/backend/cpu/quantized.cpp:805-844 per pair; SwitchGLU with
// sortedIndices, VLM/MLXLMCommon/SwitchLayers.swift:532-580; gatherSort /
// scatterUnsort :385-428), the Laguna block combine (Laguna.swift:204-212).
//
// GEMM shape: D[weight rows, tokens] = W[rows, K] x X[tokens, K]^T per tile of
// 128 weight rows (UMMA M) and up to 64 tokens (UMMA N), K in stages of 64.
// A three-stage pipeline per CTA: a raw-loader warp streams the packed codes
// and scales of the tile rows into an 8-deep shared ring with 16-byte
// cp.async copies (mbarrier arrivals on completion); four dequantiser warps
// turn each stage into bf16 straight in the 128-byte swizzled K-major UMMA
// layout (E2M1 pairs by the hardware converter, times the E4M3 group scale:
// exact in bf16); an activation-loader warp gathers the tile's token rows
// (through a slot -> row map, so no sorted copy of the activations is ever
// written) with cp.async into the swizzled B stage; one thread issues
// tcgen05.mma kind::f16 (bf16 x bf16 -> f32 in TMEM) and commits each stage
// back to its producers through an mbarrier.  Activations stay bf16 (exact
// for bf16 inputs, the full bf16 range).  After the K loop the dequantiser
// warps read TMEM (tcgen05.ld 32x32b) and run the epilogue:
//   mode 0 (plain)   y[row of token][n] = D                      (dense qmm)
//   mode 1 (gate/up) tile rows interleave gate row i / up row i, so adjacent
//                    TMEM lanes pair up: act = silu(gate) * up -> bf16
//   mode 2 (down)    Y[slot][n] = D  (f32, combined per token afterwards)
// All mbarrier waits are bounded (tma.cuh); on expiry error 4 is latched and
// the CTA drains before releasing TMEM.
#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"

namespace nvfp4 {
namespace {

constexpr int kBM = 128;                          // weight rows per tile
constexpr int kBN = 64;                           // tokens per tile (max UMMA N used)
constexpr int kBK = 64;                           // K per stage: one 128 B swizzle atom of bf16
constexpr int kStages = 3;                        // bf16 A/B stages fed to the MMA
constexpr int kRawSlots = 5;                      // packed-weight stages in flight (2 CTAs / SM)
constexpr int kDeqWarps = 4;
constexpr int kGemmThreads = 32 * (3 + kDeqWarps);
constexpr int kStageA = kBM * kBK * 2;            // 16 KB
constexpr int kStageB = kBN * kBK * 2;            // 8 KB
constexpr int kRawPitch = 48;                     // 32 code bytes + pad: conflict-free reads
constexpr int kRawCodes = kBM * kRawPitch;        // 6 KB
constexpr int kRawSlot = kRawCodes + kBM * 4;     // + 4 scale bytes per row
constexpr int kTmemCols = 64;
constexpr int kErrTimeout = 4;

__device__ int g_prefill_error = 0;
__device__ __forceinline__ void flag(int code) { atomicCAS(&g_prefill_error, 0, code); }

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// 8 bf16 (16 bytes) from eight E2M1 codes of one word and their f32 scale.
__device__ __forceinline__ uint4 dequant8_bf16(uint32_t word, float scale) {
  uint32_t h[4];
  e2m1x8_to_f16x2x4(word, h);
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[i]));
    const __nv_bfloat162 b = __floats2bfloat162_rn(f.x * scale, f.y * scale);
    o[i] = *reinterpret_cast<const uint32_t*>(&b);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Eight activation values of one row as bf16x8 (16 bytes).
__device__ __forceinline__ uint4 load8_as_bf16(const void* x, int dtype, int64_t off) {
  if (dtype == kBF16) return *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(x) + off);
  uint32_t o[4];
  if (dtype == kF16) {
    const uint4 v = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(x) + off);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      const __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);
      o[i] = *reinterpret_cast<const uint32_t*>(&b);
    }
  } else {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + off);
    const float4 c = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + off + 4);
    const float f[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      o[i] = *reinterpret_cast<const uint32_t*>(&b);
    }
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// cp.async helpers (16-byte L2-only copies, 4-byte copies, zero-fill).
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 4 : 0)
               : "memory");
}
// One arrival on `bar` once all of this thread's prior cp.async copies landed.
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Warp roles: 0 = TMEM owner + MMA issuer (lane 0), 1 = raw weight loader,
// 2 = activation loader, 3..6 = dequantisers, then the epilogue.
constexpr int kWarpMma = 0, kWarpRaw = 1, kWarpAct = 2, kWarpDeq0 = 3;

__global__ void __launch_bounds__(kGemmThreads, 1) nvfp4_gemm_kernel(GemmArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // UMMA swizzle atoms need 1024-byte alignment.
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + kStages * kStageA;
  uint8_t* sRaw = sB + kStages * kStageB;
  uint64_t* full = reinterpret_cast<uint64_t*>(sRaw + kRawSlots * kRawSlot);
  uint64_t* empty = full + kStages;
  uint64_t* raw_full = empty + kStages;
  uint64_t* raw_empty = raw_full + kRawSlots;
  uint64_t* done = raw_empty + kRawSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  // Tiles, token maps and activations come from preceding kernels.
  pdl_wait();
  pdl_trigger();
  const int tile = blockIdx.y;
  int4 td;
  if (a.implicit_M > 0) {
    if (tile * kBN >= a.implicit_M) return;
    td = make_int4(0, tile * kBN, min(kBN, a.implicit_M - tile * kBN), 0);
  } else {
    if (tile >= *a.ntiles) return;
    td = a.tiles[tile];
  }
  const int grp = td.x, start = td.y, count = td.z;
  const int N = (count + 15) & ~15;
  const int m_tile = blockIdx.x;
  const bool is_shared = grp == a.shared_group;
  const int Mrows = is_shared ? a.Mrows_shared : a.Mrows;
  const int row_step = a.mode == 1 ? 64 : 128;
  if (m_tile * row_step >= Mrows) return;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; i++) {
      mbar_init(&full[i], kDeqWarps + 32);  // dequant warps + activation-loader lanes
      mbar_init(&empty[i], 1);              // MMA commit
    }
    for (int i = 0; i < kRawSlots; i++) {
      mbar_init(&raw_full[i], 32);          // raw-loader lanes (cp.async arrivals)
      mbar_init(&raw_empty[i], kDeqWarps);
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == kWarpMma) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nkb = a.K / kBK;

  // Bank row behind tile row r (gate/up interleave in mode 1).
  auto bank_row = [&](int r, const uint8_t*& wb, const uint8_t*& sb, int64_t& row) {
    const uint8_t* w0 = is_shared ? a.sw0 : a.w0 + (int64_t)grp * a.w_stride;
    const uint8_t* s0 = is_shared ? a.ss0 : a.s0 + (int64_t)grp * a.s_stride;
    const uint8_t* w1 = is_shared ? a.sw1 : a.w1 + (int64_t)grp * a.w_stride;
    const uint8_t* s1 = is_shared ? a.ss1 : a.s1 + (int64_t)grp * a.s_stride;
    if (a.mode == 1) {
      row = (int64_t)m_tile * 64 + (r >> 1);
      wb = (r & 1) ? w1 : w0;
      sb = (r & 1) ? s1 : s0;
    } else {
      row = (int64_t)m_tile * 128 + r;
      wb = w0;
      sb = s0;
    }
  };

  if (warp == kWarpMma) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_f32(kBM, N) | (1u << 7) | (1u << 10);  // A, B bf16
      for (int kb = 0; kb < nkb; kb++) {
        const int s = kb % kStages;
        if (!mbar_wait_bounded(&full[s], (kb / kStages) & 1)) {
          flag(kErrTimeout);
          break;
        }
        tc_fence_after();
        const uint64_t ad = smem_desc_sw128(smem_u32(sA + s * kStageA));
        const uint64_t bd = smem_desc_sw128(smem_u32(sB + s * kStageB));
#pragma unroll
        for (int ks = 0; ks < kBK / 16; ks++)  // 16 bf16 = 32 bytes = 2 descriptor units
          umma_f16(tmem, ad + 2 * ks, bd + 2 * ks, idesc, (kb | ks) != 0);
        umma_commit(&empty[s]);
      }
      umma_commit(done);  // fires when every MMA issued above has completed
    }
    __syncwarp();
  } else if (warp == kWarpRaw) {
    // --------------------------- raw weight loader ---------------------------
    // Lane l copies rows l, l+32, l+64, l+96: 32 code bytes (two 16 B copies)
    // and 4 scale bytes per row and stage, R stages ahead of the dequantisers.
    const uint8_t* cptr[4];
    const uint8_t* sptr[4];
    bool rok[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const uint8_t *wb, *sb;
      int64_t row;
      bank_row(lane + 32 * i, wb, sb, row);
      rok[i] = row < Mrows;
      cptr[i] = rok[i] ? wb + row * (a.K / 2) : a.w0;
      sptr[i] = rok[i] ? sb + row * (a.K / 16) : a.s0;
    }
    for (int kb = 0; kb < nkb; kb++) {
      const int r = kb % kRawSlots;
      if (kb >= kRawSlots && !mbar_wait_bounded(&raw_empty[r], ((kb / kRawSlots) - 1) & 1)) {
        flag(kErrTimeout);
        break;
      }
      uint8_t* slot = sRaw + r * kRawSlot;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int tr = lane + 32 * i;
        cp_async16(slot + tr * kRawPitch, cptr[i] + kb * 32, rok[i]);
        cp_async16(slot + tr * kRawPitch + 16, cptr[i] + kb * 32 + 16, rok[i]);
        cp_async4(slot + kRawCodes + tr * 4, sptr[i] + kb * 4, rok[i]);
      }
      cp_async_arrive_noinc(&raw_full[r]);
    }
    cp_async_wait<0>();
  } else if (warp == kWarpAct) {
    // --------------------------- activation loader ---------------------------
    // Lane l copies 16-byte chunks q = l + 32 i (token n = q / 8, chunk q % 8)
    // of the tile's rows into the swizzled B stage.  Copies of stage kb are
    // one commit group; the stage is handed to the MMA (proxy fence + arrive)
    // once its group has landed, kStages - 1 stages later.
    const bool direct = a.b_dtype == kBF16;
    int64_t brow[16];
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const int n = (lane + 32 * i) >> 3;
      brow[i] = n < count ? (int64_t)(a.brow ? a.brow[start + n] : start + n) : -1;
    }
    int issued = 0, handed = 0;
    for (int kb = 0; kb < nkb; kb++) {
      const int s = kb % kStages;
      if (kb >= kStages && !mbar_wait_bounded(&empty[s], ((kb / kStages) - 1) & 1)) {
        flag(kErrTimeout);
        break;
      }
      uint8_t* stage = sB + s * kStageB;
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const int q = lane + 32 * i, n = q >> 3, c = q & 7;
        uint8_t* dst = stage + n * 128 + ((c ^ (n & 7)) << 4);
        const int64_t off = (brow[i] >= 0 ? brow[i] : 0) * a.b_ld + kb * kBK + c * 8;
        if (direct) {
          cp_async16(dst, reinterpret_cast<const uint16_t*>(a.b) + off, brow[i] >= 0);
        } else {
          *reinterpret_cast<uint4*>(dst) =
              brow[i] >= 0 ? load8_as_bf16(a.b, a.b_dtype, off) : make_uint4(0, 0, 0, 0);
        }
      }
      cp_async_commit();
      issued++;
      if (issued - handed == kStages - 1) {
        cp_async_wait<kStages - 2>();
        fence_proxy_async();
        mbar_arrive(&full[handed % kStages]);
        handed++;
      }
    }
    cp_async_wait<0>();
    fence_proxy_async();
    for (; handed < issued; handed++) mbar_arrive(&full[handed % kStages]);
  } else {
    // ------------------------------ dequantisers ------------------------------
    const int pt = threadIdx.x - 32 * kWarpDeq0;  // 0..127: this thread's A row
    for (int kb = 0; kb < nkb; kb++) {
      const int r = kb % kRawSlots, s = kb % kStages;
      if (!mbar_wait_bounded(&raw_full[r], (kb / kRawSlots) & 1)) {
        flag(kErrTimeout);
        break;
      }
      const uint8_t* slot = sRaw + r * kRawSlot;
      const uint4 cw0 = *reinterpret_cast<const uint4*>(slot + pt * kRawPitch);
      const uint4 cw1 = *reinterpret_cast<const uint4*>(slot + pt * kRawPitch + 16);
      const uint32_t sw = *reinterpret_cast<const uint32_t*>(slot + kRawCodes + pt * 4);
      __syncwarp();
      if (lane == 0) mbar_arrive(&raw_empty[r]);
      if (kb >= kStages && !mbar_wait_bounded(&empty[s], ((kb / kStages) - 1) & 1)) {
        flag(kErrTimeout);
        break;
      }
      uint8_t* arow = sA + s * kStageA + pt * 128;
      const int sw7 = pt & 7;
      const uint32_t wds[8] = {cw0.x, cw0.y, cw0.z, cw0.w, cw1.x, cw1.y, cw1.z, cw1.w};
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const float scale = scale_to_f32((sw >> (8 * (j >> 1))) & 0xFFu);
        *reinterpret_cast<uint4*>(arow + ((j ^ sw7) << 4)) = dequant8_bf16(wds[j], scale);
      }
      fence_proxy_async();  // generic-proxy smem writes -> tensor-core reads
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);
    }
    // ------------------------------ epilogue --------------------------------
    // Warp-uniform decision: the TMEM loads below are .sync.aligned.
    const bool have = __all_sync(0xffffffffu, mbar_wait_bounded(done, 0));
    if (!have && lane == 0) flag(kErrTimeout);
    tc_fence_after();
    const int sp = warp & 3;       // TMEM sub-partition this warp may read
    const int r = sp * 32 + lane;  // tile row = TMEM lane
    for (int c0 = 0; c0 < N && have; c0 += 16) {
      float v[16];
      tmem_ld16(tmem + ((uint32_t)(sp * 32) << 16) + (uint32_t)c0, v);
      if (a.mode == 1) {
        const int64_t i = (int64_t)m_tile * 64 + (r >> 1);
#pragma unroll
        for (int q = 0; q < 16; q++) {
          const float other = __shfl_xor_sync(0xffffffffu, v[q], 1);
          const int n = c0 + q;
          if (!(r & 1) && n < count && i < Mrows)
            reinterpret_cast<__nv_bfloat16*>(a.out)[(int64_t)(start + n) * a.out_ld + i] =
                __float2bfloat16_rn(silu_ref(v[q]) * other);
        }
      } else {
        const int64_t rr = (int64_t)m_tile * 128 + r;
#pragma unroll
        for (int q = 0; q < 16; q++) {
          const int n = c0 + q;
          if (n < count && rr < Mrows) {
            if (a.mode == 2)
              reinterpret_cast<float*>(a.out)[(int64_t)(start + n) * a.out_ld + rr] = v[q];
            else
              store_from_f32(a.out, a.out_dtype,
                             (int64_t)(a.brow ? a.brow[start + n] : start + n) * a.out_ld + rr,
                             v[q]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kWarpMma) tmem_dealloc(tmem, kTmemCols);
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
  pdl_wait();
  pdl_trigger();
  const int E = a.E;
  const int P = a.P;
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    const uint32_t e = a.inds[p];
    if (e < (uint32_t)E) atomicAdd(&cnt[e], 1);
    else flag(5);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0, tacc = 0;
    for (int e = 0; e < E; e++) {
      off[e] = acc;
      toff[e] = tacc;
      acc += cnt[e];
      tacc += (cnt[e] + kBN - 1) / kBN;
    }
    toff[E] = tacc;
    const int tsh = a.with_shared ? (a.T + kBN - 1) / kBN : 0;
    *a.ntiles = tacc + tsh;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int n = cnt[e];
    for (int t = 0; t * kBN < n; t++)
      a.tiles[toff[e] + t] = make_int4(e, off[e] + t * kBN, min(kBN, n - t * kBN), 0);
    cnt[e] = 0;  // reused as the scatter cursor
  }
  if (a.with_shared) {
    for (int t = threadIdx.x; t * kBN < a.T; t += blockDim.x)
      a.tiles[toff[E] + t] = make_int4(E, P + t * kBN, min(kBN, a.T - t * kBN), 0);
    for (int t = threadIdx.x; t < a.T; t += blockDim.x) a.brow[P + t] = t;
  }
  __syncthreads();
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    const uint32_t e = a.inds[p];
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
// in a fixed j order (deterministic).
__global__ void moe_combine_kernel(CombineArgs a) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = (int64_t)a.T * a.H;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / a.H, h = i - t * a.H;
    float acc = 0.f;
    for (int j = 0; j < a.k; j++) {
      const int slot = a.pos[t * a.k + j];
      if (slot >= 0) acc += a.wts[t * a.k + j] * a.Y[(int64_t)slot * a.H + h];
    }
    acc *= a.scaling;
    if (a.with_shared) acc += a.Y[(int64_t)(a.P + t) * a.H + h];
    if (a.residual) acc += load_as_f32(a.residual, a.dtype, i);
    store_from_f32(a.y, a.dtype, i, acc);
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

}  // namespace

size_t gemm_smem_bytes() {
  return 1024 + (size_t)kStages * (kStageA + kStageB) + (size_t)kRawSlots * kRawSlot +
         (2 * kStages + 2 * kRawSlots + 1) * 8 + 16;
}

int gemm_tile_tokens() { return kBN; }

cudaError_t launch_nvfp4_gemm(const GemmArgs& a, int max_tiles, cudaStream_t stream, bool pdl) {
  if (max_tiles <= 0) return cudaSuccess;
  const size_t smem = gemm_smem_bytes();
  cudaError_t e = ensure_smem(nvfp4_gemm_kernel, smem);
  if (e != cudaSuccess) return e;
  const int mrows = std::max(a.Mrows, a.Mrows_shared);
  const int m_tiles = a.mode == 1 ? (mrows + 63) / 64 : (mrows + 127) / 128;
  return launch_pdl(nvfp4_gemm_kernel, dim3(m_tiles, max_tiles), dim3(kGemmThreads), smem,
                    stream, pdl, a);
}

cudaError_t launch_moe_sort(const SortArgs& a, cudaStream_t stream, bool pdl) {
  return launch_pdl(moe_sort_kernel, dim3(1), dim3(1024), 0, stream, pdl, a);
}

cudaError_t launch_moe_combine(const CombineArgs& a, cudaStream_t stream, bool pdl) {
  const int64_t total = (int64_t)a.T * a.H;
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
