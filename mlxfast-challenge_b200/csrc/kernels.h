// kernels.h -- argument blocks and host launchers of the CUDA kernels.  Only
// the C ABI (api.cu) includes this; nothing here crosses the library boundary.
#pragma once

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

// Grouped NVFP4 GEMM on tcgen05 (prefill.cu).
struct GemmArgs {
  int mode;          // 0 plain (y[brow][row]), 1 gate/up + SwiGLU -> bf16 act, 2 down -> f32 Y
  int K;             // reduction length (multiple of 64)
  int Mrows;         // rows of one bank per group
  int Mrows_shared;  // rows of the shared group's bank
  const uint8_t *w0, *s0, *w1, *s1;  // routed banks (w1/s1: the up bank in mode 1)
  int64_t w_stride, s_stride;        // bytes per group
  int shared_group;                  // group id served by the shared banks, -1 none
  const uint8_t *sw0, *ss0, *sw1, *ss1;
  const void* b;     // activation rows [*, b_ld]
  int b_dtype;
  int64_t b_ld;
  const int* brow;   // slot -> activation row (null: slot itself)
  const int4* tiles; // (group, first slot, count, 0)
  const int* ntiles;
  int implicit_M;    // > 0: one group, slots 0..implicit_M-1, tiles of 64 (no tiles/brow)
  void* out;
  int out_dtype;
  int64_t out_ld;
};

struct SortArgs {
  const uint32_t* inds;  // [T, k]
  int T, k, E, P, with_shared;
  int* brow;   // [P + T]
  int* pos;    // [P]
  int4* tiles;
  int* ntiles;
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
};

size_t gemm_smem_bytes();
int gemm_tile_tokens();
cudaError_t launch_nvfp4_gemm(const GemmArgs& a, int max_tiles, cudaStream_t stream, bool pdl);
cudaError_t launch_moe_sort(const SortArgs& a, cudaStream_t stream, bool pdl);
cudaError_t launch_moe_combine(const CombineArgs& a, cudaStream_t stream, bool pdl);
cudaError_t read_and_clear_prefill_error(int* out);

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
