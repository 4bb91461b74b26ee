// kernels.h -- argument blocks and host launchers of the CUDA kernels.  Only
// the C ABI (api.cu) includes this; nothing here crosses the library boundary.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

namespace nvfp4 {

// Gather QMM: out[p*M + m][n] = x[lhs[p]*M + m] . dequant(W[rhs[p]])[n].
struct QmmArgs {
  void* out;
  const void* x;
  const uint8_t* w;    // [E, N, K/2] bytes
  const uint8_t* s;    // [E, N, K/16]
  const uint32_t* lhs;  // [P] or null (identity)
  const uint32_t* rhs;  // [P] or null (expert 0)
  int64_t P, N, K;
  int M, mchunks, dtype;
  int64_t w_stride, s_stride;  // bytes per expert
  int64_t n_x_batches, n_experts;
};

struct GateUpArgs {
  const void* x;  // [T, H]
  int dtype;
  int64_t T, H, I, Is, E;
  int k, kk;
  const uint32_t* inds;  // [T, k]
  const uint8_t *gw, *gs, *uw, *us;  // routed banks
  int64_t w_stride, s_stride;
  const uint8_t *sgw, *sgs, *suw, *sus;  // shared expert (null when absent)
  float* act;  // [T*kk, act_ld]
  int64_t act_ld;
  int inds_static;  // inds were not written by the immediately preceding kernel
  int bulk;         // use the bulk-copy fed kernel when the shape allows
};

struct DownArgs {
  const float* act;
  int64_t act_ld;
  int64_t T, H, I, Is, E;
  int k, kk, Ipad;
  const uint32_t* inds;
  const float* wts;
  float scaling;
  const uint8_t *dw, *ds;
  int64_t w_stride, s_stride;
  const uint8_t *sdw, *sds;
  const void* residual;
  void* y;
  int dtype;
  int inds_static;      // routing complete before this grid starts (see qmv.cu)
  int max_seg_per_cta;  // set by the launcher
  int bulk;             // use the bulk-copy fed kernel when the shape allows
};

struct RouterArgs {
  const void* x;  // [T, H]
  int dtype;
  const uint16_t* G;  // bf16 [E, H]
  const float* bias;  // [E] or null
  int64_t T, H, E;
  int k, norm, ksplit;
  float* partial;       // [ceil(T/8), ksplit, 8, E]
  unsigned* counters;   // [ceil(T/8)], zero on entry, left zero on exit
  uint32_t* inds;       // [T, k]
  float* wts;           // [T, k]
};

// Sorted-slot grouped GEMM on tcgen05 (prefill.cu).  Operands arrive by TMA through
// 2-D tensor maps: packed codes [rows, K/2] bytes (box 128 bytes x 64 or 128
// rows, 128-byte swizzle), scales [rows, K/16] bytes (box 16 x rows), and
// 16-bit activation rows in slot order [slots, K] (box 64 elements x 16 rows,
// 128-byte swizzle).  Routed banks stack the groups' rows (row = group *
// Mrows + r); the shared group has its own maps.
struct alignas(64) GemmArgs {
  CUtensorMap mc0, ms0, mc1, ms1;      // routed codes / scales (mc1, ms1: up bank, mode 1)
  CUtensorMap mcs0, mss0, mcs1, mss1;  // shared-group codes / scales
  CUtensorMap mb;                      // activation rows, slot order
  int mode;          // 0 plain (out[row of slot][n]), 1 gate/up + SwiGLU -> f32 act, 2 down -> f32 Y
  int K;             // reduction length (multiple of 256)
  int Mrows;         // rows of one routed group
  int Mrows_shared;  // rows of the shared group
  int shared_group;  // group id served by the shared maps, -1 none
  int implicit_M;    // > 0: one group, slots 0..implicit_M-1, tiles of 64 (no tile list)
  const float* bscale;  // per slot: true activation row = row * bscale[slot] (null: 1)
  const int4* tiles;    // (group, first slot, count, 0)
  const int* ntiles;
  void* out;
  int out_dtype;
  int64_t out_ld;
  int out_vec;  // set by the launcher: output rows written as 16-byte chunks
};

// Tensor maps for GemmArgs (cuTensorMapEncodeTiled through the runtime's
// driver entry point).  rows: rows of the whole bank / activation matrix.
cudaError_t map_codes(CUtensorMap* m, const void* w, int64_t rows, int64_t K, int box_rows);
cudaError_t map_scales(CUtensorMap* m, const void* s, int64_t rows, int64_t K, int box_rows);
// Codes of K = 64 steps (32-byte rows, 32-byte swizzle): the routed decode
// stack's down tiles.
cudaError_t map_codes_k64(CUtensorMap* m, const void* w, int64_t rows, int64_t K, int box_rows);
cudaError_t map_rows16(CUtensorMap* m, const void* b, bool bf16, int64_t rows, int64_t K,
                       int64_t ld);

// Rows of any activation dtype -> f16 rows scaled by a per-row power of two
// (rows_to_f16_kernel); scale[r] receives the factor that undoes it.
struct RowsArgs {
  const void* src;
  int src_dtype;
  const int* src_map;  // dst row r <- src row src_map[r] (null: r)
  int rows, K;
  int64_t src_ld;
  __half* dst;
  int64_t dst_ld;
  float* scale;
};

// Serial decode through a stack of sparse MoE layers in one persistent
// cooperative launch (decode_stack.cu).  T = 1, routing given per layer.
constexpr int kStackMaxLayers = 64;
struct StackLayer {
  const uint8_t *gw, *gs, *uw, *us, *dw, *ds;        // routed banks
  const uint8_t *sgw, *sgs, *suw, *sus, *sdw, *sds;  // shared expert (null: none)
  const uint32_t* inds;                              // [k] device
  const float* wts;                                  // [k] device
  float scaling;
};
struct StackArgs {
  int L, H, I, E, k, kk, dtype;
  int64_t gw_stride, gs_stride, dw_stride, ds_stride;  // bytes per expert
  const void* x0;   // [H] input
  void* y;          // [H] output of the last layer
  void* xb[2];      // [H] ping-pong activations between layers
  float* act;       // [kk, I] gate/up output of the current layer
  unsigned* bar;    // [2] grid-barrier counters, zero at launch
  unsigned* xmax;   // [L] max |x_l| (float bits), zero at launch
  unsigned* amax;   // [L] max |act_l * w|, zero at launch
  StackLayer layer[kStackMaxLayers];
};
size_t decode_stack_smem_bytes(int H, int I, int kk);
cudaError_t launch_decode_stack(const StackArgs& a, cudaStream_t stream);
cudaError_t read_and_clear_stack_error(int* out);

// The same stack on the block-scaled FP4 tensor cores (decode_stack_fp4.cu).
// Tensor maps travel in the kernel parameters (<= 32 KB): layers of one launch
// share kFsMaxMaps maps, 6 per layer (12 with a shared expert).
constexpr int kFsMaxLayers = 40;
constexpr int kFsMaxMaps = 240;
constexpr int kFsMapsRouted = 6;  // gate codes, gate scales, up codes, up scales, down codes, down scales
struct FsLayer {
  // Given routing: inds / wts [k] read.  Routed stack: where the layer's
  // routing is written (both nullable).
  uint32_t* inds;
  float* wts;
  const uint16_t* router_w;  // routed stack: bf16 [E, H]
  const float* router_b;     // routed stack: f32 [E] or null
  const void* norm_w;        // routed stack with the norm: RMSNorm weight [H] (dtype)
};
// Routed stack: the reducers of a layer.  Reducer j (CTA j, j < H / kFsRedRows)
// sums the segment partials of rows [j * kFsRedRows, (j + 1) * kFsRedRows) and
// adds their share of every expert's router logit.
constexpr int kFsRedRows = 32;
constexpr int kFsLgStride = 16;  // u64 per logit accumulator (one 128-byte line)
constexpr int kFsYsStride = 4;   // u64 per layer-output accumulator (a 32-byte sector)
constexpr int kFsCounters = 64;  // cnt1[16] gate/up items per segment, cnt2[16] down items
constexpr int kFsMaxReducers = 64;
constexpr int kFsMaxSeg = 9;  // routed stack: top_k <= 8 routed segments + the shared expert
// Routed stack exchange area, zeroed at every launch (its values carry their
// own completion: counts or layer tags), laid out after the counters:
//   routing lines  [kFsMaxLayers][8] u64
//   layer inputs   [2][H / 2] u64 (by stack-layer parity)
//   squares        [kFsMaxLayers][kFsMaxReducers] u64
//   layer outputs  [L][H][kFsYsStride] u64: counted sums of the down partials (norm on)
//   logits         [L][E][kFsLgStride] u64
__host__ __device__ constexpr size_t fs_xchg_u64(int H, int E, int L) {
  return (size_t)kFsMaxLayers * 8 + (size_t)H + (size_t)kFsMaxLayers * kFsMaxReducers +
         (size_t)L * H * kFsYsStride + (size_t)L * E * kFsLgStride;
}
struct alignas(64) FsArgs {
  CUtensorMap maps[kFsMaxMaps];  // layer l: maps[l * mpl + j]; j >= 6: the shared expert's
  FsLayer layer[kFsMaxLayers];
  int L;           // layers in this launch
  int first;       // 1: layer 0 of the stack (input x0 in dtype), else the previous launch's
  int last;        // 1: the launch ends the stack (writes y)
  int l0;          // stack index of this launch's first layer (buffer parity)
  int H, I, E, k, kk, nks, mpl, dtype;
  int routed;      // 1: routing computed per layer on the device (the routed stack)
  int residual;    // routed stack: h_{l+1} = h_l + block_l(x_l) (else block_l(x_l))
  int norm;        // routed stack: norm_topk_prob
  int has_norm;    // routed stack: x_l = RMSNorm(h_l; layer[l].norm_w, eps) (else x_l = h_l)
  float eps;       // the norm's epsilon
  float scaling;   // routed_scaling of every layer
  int test_skip_release;  // test only: the last layer's segment-0 gate/up items skip a release
  long long budget;       // cycles a bounded wait may take before it gives up
  const void* x0;  // [H] stack input h_0 (dtype)
  void* y;         // [H] stack output (dtype)
  float* Yp;       // [2][kk][H] a layer's output per segment (f32), by layer parity
  float* GUp;      // [2][2][kk][2][I] gate / up pre-activations per K part, by parity
  float* Hres;     // routed stack: [2][H] h at a launch boundary (the next launch's h_0)
  unsigned long long* XG;  // routed stack: the exchange area (fs_xchg_u64), after bar
  unsigned* bar;   // [kFsCounters] dependency counters; zeroed at launch with XG
};
bool decode_stack_fp4_supported(int H, int I, int kk, int sms, bool routed = false);
int decode_stack_fp4_nks(int I, int kk, int sms);
size_t decode_stack_fp4_smem_bytes(int H, int I, int L, bool routed = false);
cudaError_t launch_decode_stack_fp4(const FsArgs& a, cudaStream_t stream);
cudaError_t read_and_clear_stack_fp4_error(int* out);

// RMSNorm of T rows of H (norm.cu).
struct NormArgs {
  const void* x;  // [T, H] dtype
  const void* w;  // [H] dtype, or null (weight 1)
  void* y;        // [T, H] dtype
  int64_t T, H;
  float eps;
  int dtype;
};
cudaError_t launch_rms_norm(const NormArgs& a, cudaStream_t stream, bool pdl);

// Expert-parallel dispatch / combine (ep.cu).
struct EpPlanArgs {
  const uint32_t* inds;      // [T, k] global expert ids
  int64_t T;
  int k;
  int64_t experts_per_rank;
  int world;
  int32_t* pos;     // [T*k] slot of each pair in the send buffer (-1: none)
  int32_t* ids;     // [T*k] local expert id per send slot
  int32_t* counts;  // [world] pairs per destination rank
};
struct EpPackArgs {
  const void* x;    // [T, H]
  int64_t T;
  int k;
  int64_t H;
  int esz;          // bytes per element
  const int32_t* pos;
  void* send_x;     // [T*k, H] in destination order
};
struct EpCombineArgs {
  void* y;            // [T, H]
  const void* yp;     // [T*k, H] expert outputs in send order
  const int32_t* pos;
  const float* wts;   // [T, k]
  int64_t T;
  int k;
  int64_t H;
  float scaling;
  const void* shared;    // [T, H] or null
  const void* residual;  // [T, H] or null
  int dtype;
};
cudaError_t launch_ep_plan(const EpPlanArgs& a, cudaStream_t stream);
cudaError_t launch_ep_pack(const EpPackArgs& a, cudaStream_t stream);
cudaError_t launch_ep_combine(const EpCombineArgs& a, cudaStream_t stream);
// y[T, H] = partial (f32) + shared + residual, rounded once to dtype.
cudaError_t launch_ep_finish(void* y, const void* partial, int partial_dtype, const void* shared,
                             const void* residual, int dtype, int64_t T, int64_t H,
                             cudaStream_t stream);
cudaError_t read_and_clear_ep_error(int* out);

struct SortArgs {
  const uint32_t* inds;  // [T, k]
  int T, k, E, P, with_shared;
  int* brow;   // [P + T]
  int* pos;    // [P]
  int4* tiles;
  int* ntiles;
  int tile_tokens;  // tokens per tile (0: the f16 GEMM's 64)
  // Expert-parallel partial block: ids are global, this rank's experts are
  // [e_base, e_base + E); other ids are skipped (slot -1) without an error.
  int e_base, skip_foreign;
  // shared-expert group over rows [sh_row0, sh_row0 + sh_rows) (sh_rows 0: all T)
  int sh_row0, sh_rows;
};

// Activation rows as a sum of kFp4Terms NVFP4 terms (prefill_fp4.cu):
// term t of a row is its residual after terms 0..t-1, quantised per group of
// 16 with a UE4M3 scale, under one power-of-two factor per (row, term).
constexpr int kFp4Terms = 4;
struct TermsArgs {
  const void* src;      // [rows, K] (row r at src + r * src_ld elements)
  int src_dtype;
  int64_t rows, K, src_ld;
  // destination slot of source row r: dst_map[r * map_stride + j] for
  // j < map_count (entries < 0 skipped), plus extra_base + r when
  // extra_base >= 0; identity when dst_map is null and extra_base < 0
  const int* dst_map;
  int map_stride, map_count;
  int64_t extra_base;
  int64_t extra_lo, extra_hi;  // rows that also feed extra_base + (r - extra_lo)
  uint8_t* codes;   // [slots * 4, K/2]  (term row = slot * 4 + t)
  uint8_t* scales;  // [slots * 4, K/16]
  float* fac;       // [slots * 4]: value = fac * dequant(codes, scales)
};

// Grouped GEMM on the block-scaled tensor cores over slot-ordered term rows.
struct alignas(64) GemmFp4Args {
  CUtensorMap mc0, ms0, mc1, ms1;      // routed codes / scales (mc1, ms1: up bank, mode 1)
  CUtensorMap mcs0, mss0, mcs1, mss1;  // shared-expert codes / scales
  CUtensorMap mb[4], msb[4];           // term-row codes [S*4, K/2] / scales, boxes of 32 (i+1) rows
  const float* bfac;                   // [S*4]
  const int4* tiles;                   // (group, first slot, slots <= 32, 0)
  const int* ntiles;
  int max_tiles;                       // capacity of the tile list (shared-memory copy)
  int mode;          // 1 gate/up + SwiGLU -> act f32, 2 down -> Y f32
  int K, Mrows, Mrows_shared, shared_group;
  float* out;        // mode 1: act [S, out_ld]; mode 2: Y [S, out_ld]
  int64_t out_ld;
};

struct CombineArgs {
  const float* Y;  // [P + T, H]
  const int* pos;
  const float* wts;
  int T, k, P, H, with_shared;
  float scaling;
  const void* residual;
  void* y;
  int dtype;
  int sh_row0, sh_rows;  // shared-expert rows (sh_rows 0: all T)
};

size_t gemm_smem_bytes();
int gemm_tile_tokens();
cudaError_t launch_nvfp4_gemm(const GemmArgs& a, bool f16, int max_tiles, cudaStream_t stream,
                              bool pdl);
int gemm_slab_k();
cudaError_t launch_rows_to_f16(const RowsArgs& a, cudaStream_t stream, bool pdl);
cudaError_t launch_moe_sort(const SortArgs& a, cudaStream_t stream, bool pdl);
constexpr int kFp4TileTokens = 32;
size_t gemm_fp4_smem_bytes(int max_tiles);
cudaError_t launch_rows_to_terms(const TermsArgs& a, cudaStream_t stream);
cudaError_t launch_nvfp4_gemm_fp4(const GemmFp4Args& a, int max_tiles, cudaStream_t stream);
cudaError_t read_and_clear_fp4_error(int* out);
cudaError_t launch_moe_combine(const CombineArgs& a, cudaStream_t stream, bool pdl);
cudaError_t read_and_clear_prefill_error(int* out);

// NVFP4 x NVFP4 matmul (qqmm): y[M, N] = xhat[M, K] . dequant(W)[N, K]^T.
struct alignas(64) QqmmArgs {
  CUtensorMap ma, msa;  // W codes [N, K/2] (128 x 128 B boxes, 128 B swizzle), W scales
  CUtensorMap mb, msb;  // x codes [M, K/2] (bn x 128 B boxes), x scales
  void* out;            // [M, N], dtype
  int dtype;
  int64_t M, N, K;
  int bn, n_tiles, m_tiles, splits;
  float* partial;   // [tiles][splits][bn][128] when splits > 1
  unsigned* ticket; // [tiles] when splits > 1
};
int qqmm_tile_tokens(int64_t M);
size_t qqmm_smem_bytes(int bn);
void qqmm_plan(int64_t M, int64_t N, int64_t K, int sms, int* bn, int* n_tiles, int* m_tiles,
               int* splits);
cudaError_t launch_qx_quantize(uint8_t* qx, uint8_t* sx, const void* x, int dtype, int64_t M,
                               int64_t K, cudaStream_t stream);
cudaError_t launch_qqmm(const QqmmArgs& a, cudaStream_t stream);
cudaError_t read_and_clear_qqmm_error(int* out);

size_t qmm_smem_bytes(int64_t K);
bool qmm_fast_path_ok(const QmmArgs& a);
cudaError_t launch_qmm_gather(const QmmArgs& a, cudaStream_t stream, bool pdl);
size_t gateup_smem_bytes(int64_t H);
cudaError_t launch_moe_gateup(const GateUpArgs& a, cudaStream_t stream, bool pdl);
size_t down_smem_bytes(int64_t Ipad, int kk);
cudaError_t launch_moe_down(const DownArgs& a, cudaStream_t stream, bool pdl);
cudaError_t launch_router(const RouterArgs& a, cudaStream_t stream, bool pdl);
int router_ksplit(int64_t H);
cudaError_t launch_dequantize(void* out, int dtype, const uint8_t* w, const uint8_t* s,
                              int64_t rows, int64_t K, cudaStream_t stream);
cudaError_t launch_quantize(uint8_t* wq, uint8_t* sq, const void* w, int dtype, int64_t rows,
                            int64_t K, cudaStream_t stream);
cudaError_t read_and_clear_device_error(int* out);

// Raise a kernel's dynamic shared-memory limit once per device (the call is
// not stream-ordered, so it is kept out of the launch path and therefore out
// of CUDA-graph capture after the first eager launch).
cudaError_t ensure_smem_ptr(const void* kern, size_t bytes);
template <typename Kern>
cudaError_t ensure_smem(Kern kern, size_t bytes) {
  return ensure_smem_ptr(reinterpret_cast<const void*>(kern), bytes);
}

}  // namespace nvfp4
