// api.cu -- the C ABI (include/nvfp4moe.h): argument validation in the
// reference's terms, error reporting, workspace layout and kernel dispatch.
// No entry point allocates device memory or falls back to the CPU.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <initializer_list>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/nvfp4moe.h"
#include "kernels.h"

namespace {

thread_local std::string t_last_error;
thread_local int t_launch_flags = 0;

bool first_pdl() { return (t_launch_flags & NVFP4_LAUNCH_PDL) != 0; }
bool use_bulk() { return (t_launch_flags & NVFP4_LAUNCH_BULK_COPY) != 0; }
bool use_fp4_terms() { return (t_launch_flags & NVFP4_LAUNCH_EXACT_PREFILL) == 0; }
bool use_fp4_decode() { return (t_launch_flags & NVFP4_LAUNCH_EXACT_DECODE) == 0; }
nvfp4_error_handler g_handler = nullptr;
void* g_handler_data = nullptr;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  if (g_handler) g_handler(buf, g_handler_data);
  return code;
}

int check_cuda(cudaError_t e, const char* op) {
  if (e == cudaSuccess) return NVFP4_OK;
  return fail(NVFP4_ERR_CUDA, "[%s] CUDA error: %s", op, cudaGetErrorString(e));
}

bool valid_dtype(int d) { return d == NVFP4_BF16 || d == NVFP4_F16 || d == NVFP4_F32; }

// validate_quantized_input / extract_quantized_matmul_dims (ops.cpp:84-175)
// for nvfp4, transpose=true: K must be a whole number of 16-element groups.
int check_qdims(const char* op, int64_t N, int64_t K) {
  if (K <= 0 || N < 0)
    return fail(NVFP4_ERR_INVALID, "[%s] Invalid shape: N=%lld K=%lld.", op, (long long)N,
                (long long)K);
  if (K % 16 != 0)
    return fail(NVFP4_ERR_INVALID,
                "[%s] The last dimension of the matrix needs to be divisible by the "
                "quantization group size 16. However the provided matrix has K=%lld.",
                op, (long long)K);
  return NVFP4_OK;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

struct RouterLayout {
  size_t counters_off, partial_off, total;
  int ksplit;
};

RouterLayout router_layout(int64_t T, int64_t H, int64_t E) {
  RouterLayout L;
  L.ksplit = nvfp4::router_ksplit(H);
  const int64_t groups = (T + 7) / 8;
  L.counters_off = 0;
  L.partial_off = align_up((size_t)groups * sizeof(unsigned), 256);
  L.total = L.partial_off + (size_t)groups * std::max(L.ksplit, 1) * 8 * E * sizeof(float);
  L.total = align_up(L.total, 256);
  return L;
}

struct BlockLayout {
  RouterLayout router;
  size_t inds_off, wts_off, act_off, total;
  int64_t act_ld;
  int kk;
  // Prefill (T > 8) buffers: sorted slot maps, tile list, x rows in slot order
  // as pre-scaled f16, f32 act, act as pre-scaled f16 rows, f32 Y.
  bool prefill, fp4;
  int64_t P, S, max_tiles;
  size_t brow_off, pos_off, tiles_off, ntiles_off, x16_off, xscale_off, act32_off, act16_off,
      ascale_off, y_off;
  // FP4-terms prefill: term rows of x and of act (codes, scales, factors)
  size_t xtc_off, xts_off, xtf_off, atc_off, ats_off, atf_off;
};

// The tensor-core grouped path (expert sort, grouped GEMMs): at least
// min_tokens tokens, K slabs of 256 on both GEMMs, a shared expert (if any) as
// wide as a routed one (one K for the down GEMM), and 16-byte aligned banks
// (TMA tensor-map bases).  moe_block_forward takes it from T = 2: each
// distinct expert's weights then stream once for all the tokens that chose it
// (the GEMV engine streams them once per token and slot); measured per
// Laguna layer with norm and router, T = 2 / 4 / 8: 53 / 59 / 90 us against
// 55 / 78 / 140 us.  T = 1 keeps the GEMV engine.
constexpr int64_t kGroupedMinTokens = 2;
bool prefill_shape_ok(const moe_layer_desc* L, int64_t T, int64_t min_tokens = kGroupedMinTokens) {
  const int64_t slab = nvfp4::gemm_slab_k();
  bool ok = T >= min_tokens && L->hidden % slab == 0 && L->inter % slab == 0 &&
            (L->shared_inter == 0 || L->shared_inter == L->inter) && L->n_experts <= 1024 &&
            (int64_t)L->n_experts * std::max(L->hidden, L->inter) < (1ll << 31);
  const nvfp4_bank* banks[6] = {&L->gate, &L->up, &L->down,
                                &L->shared_gate, &L->shared_up, &L->shared_down};
  for (int i = 0; i < (L->shared_inter > 0 ? 6 : 3); i++)
    ok = ok && aligned16(banks[i]->w) && aligned16(banks[i]->scales);
  return ok;
}

BlockLayout block_layout(const moe_layer_desc* L, int64_t T,
                         int64_t grouped_min_tokens = kGroupedMinTokens) {
  BlockLayout B;
  B.router = router_layout(T, L->hidden, L->n_experts);
  B.kk = (int)L->top_k + (L->shared_inter > 0 ? 1 : 0);
  B.act_ld = align_up((size_t)std::max(L->inter, L->shared_inter), 64);
  B.inds_off = B.router.total;
  B.wts_off = align_up(B.inds_off + (size_t)T * L->top_k * sizeof(uint32_t), 256);
  B.act_off = align_up(B.wts_off + (size_t)T * L->top_k * sizeof(float), 256);
  B.total = align_up(B.act_off + (size_t)T * B.kk * B.act_ld * sizeof(float), 256);
  B.prefill = prefill_shape_ok(L, T, grouped_min_tokens);
  if (B.prefill) {
    const int64_t tile = std::min<int64_t>(nvfp4::gemm_tile_tokens(), nvfp4::kFp4TileTokens);
    B.P = T * L->top_k;
    const bool sh = L->shared_inter > 0;
    B.S = B.P + (sh ? T : 0);
    B.max_tiles = L->n_experts + (B.P + tile - 1) / tile + (sh ? (T + tile - 1) / tile : 0);
    B.brow_off = B.total;
    B.pos_off = align_up(B.brow_off + (size_t)B.S * sizeof(int), 256);
    B.tiles_off = align_up(B.pos_off + (size_t)B.P * sizeof(int), 256);
    B.ntiles_off = align_up(B.tiles_off + (size_t)B.max_tiles * 16, 256);
    B.x16_off = align_up(B.ntiles_off + 16, 256);
    B.xscale_off = align_up(B.x16_off + (size_t)B.S * L->hidden * 2, 256);
    B.act32_off = align_up(B.xscale_off + (size_t)B.S * sizeof(float), 256);
    B.act16_off = align_up(B.act32_off + (size_t)B.S * B.act_ld * sizeof(float), 256);
    B.ascale_off = align_up(B.act16_off + (size_t)B.S * B.act_ld * 2, 256);
    B.y_off = align_up(B.ascale_off + (size_t)B.S * sizeof(float), 256);
    B.total = align_up(B.y_off + (size_t)B.S * L->hidden * sizeof(float), 256);
    auto k_ok = [](int64_t K) { return K == 512 || K == 1024 || K == 2048; };
    // The FP4 GEMMs stage the whole tile list in shared memory: beyond
    // ~13.8k tokens at Laguna sizes it does not fit, and the exact path
    // (no such list) takes the batch.
    B.fp4 = k_ok(L->hidden) && k_ok(L->inter) && B.max_tiles < (1 << 20) &&
            nvfp4::gemm_fp4_smem_bytes((int)B.max_tiles) <= (size_t)227 * 1024;
    if (B.fp4) {
      const size_t rows = (size_t)B.S * nvfp4::kFp4Terms;
      B.xtc_off = B.total;
      B.xts_off = align_up(B.xtc_off + rows * (L->hidden / 2), 256);
      B.xtf_off = align_up(B.xts_off + rows * (L->hidden / 16), 256);
      B.atc_off = align_up(B.xtf_off + rows * sizeof(float), 256);
      B.ats_off = align_up(B.atc_off + rows * (L->inter / 2), 256);
      B.atf_off = align_up(B.ats_off + rows * (L->inter / 16), 256);
      B.total = align_up(B.atf_off + rows * sizeof(float), 256);
    }
  }
  return B;
}

}  // namespace

namespace nvfp4 {
// Per (kernel, device) record of the dynamic shared-memory limit already set.
cudaError_t ensure_smem_ptr(const void* kern, size_t bytes) {
  struct Entry {
    const void* kern;
    int dev;
    size_t bytes;
  };
  static Entry table[64];
  static int used = 0;
  static std::mutex mu;
  if (bytes <= 48 * 1024) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; i++)
    if (table[i].kern == kern && table[i].dev == dev && table[i].bytes >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return e;
  for (int i = 0; i < used; i++)
    if (table[i].kern == kern && table[i].dev == dev) {
      table[i].bytes = bytes;
      return cudaSuccess;
    }
  if (used < 64) table[used++] = Entry{kern, dev, bytes};
  return cudaSuccess;
}
}  // namespace nvfp4

extern "C" {

const char* nvfp4_last_error(void) { return t_last_error.c_str(); }

void nvfp4_set_error_handler(nvfp4_error_handler handler, void* data) {
  g_handler = handler;
  g_handler_data = data;
}

int nvfp4_version(void) { return 1; }

int nvfp4_set_launch_flags(int flags) {
  const int old = t_launch_flags;
  t_launch_flags = flags & (NVFP4_LAUNCH_PDL | NVFP4_LAUNCH_BULK_COPY | NVFP4_LAUNCH_EXACT_PREFILL |
                            NVFP4_LAUNCH_EXACT_DECODE | NVFP4_LAUNCH_TEST_EXPIRE);
  return old;
}

int nvfp4_device_status(void) {
  int st = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return check_cuda(e, "device_status");
  e = nvfp4::read_and_clear_device_error(&st);
  if (e != cudaSuccess) return check_cuda(e, "device_status");
  int st2 = 0;
  e = nvfp4::read_and_clear_prefill_error(&st2);
  if (e != cudaSuccess) return check_cuda(e, "device_status");
  if (st == 0) st = st2;
  int st3 = 0;
  e = nvfp4::read_and_clear_stack_error(&st3);
  if (e != cudaSuccess) return check_cuda(e, "device_status");
  if (st == 0) st = st3;
  int st4 = 0;
  e = nvfp4::read_and_clear_ep_error(&st4);
  if (e != cudaSuccess) return check_cuda(e, "device_status");
  if (st == 0) st = st4;
  int st6 = 0;
  e = nvfp4::read_and_clear_fp4_error(&st6);
  if (e != cudaSuccess) return check_cuda(e, "device_status");
  if (st == 0) st = st6;
  int st5 = 0;
  e = nvfp4::read_and_clear_qqmm_error(&st5);
  if (e != cudaSuccess) return check_cuda(e, "device_status");
  if (st == 0) st = st5;
  int st7 = 0;
  e = nvfp4::read_and_clear_stack_fp4_error(&st7);
  if (e != cudaSuccess) return check_cuda(e, "device_status");
  if (st == 0) st = st7;
  // 4 and 1000 * (layer + 1) + site: a bounded wait that expired; other codes:
  // an index out of range
  if (st == 4 || st >= 1000)
    return fail(NVFP4_ERR_DEVICE_TIMEOUT,
                "[device_status] a bounded device wait expired (kernel site %d); the call's "
                "outputs are not valid.",
                st);
  if (st != 0)
    return fail(NVFP4_ERR_DEVICE_INDEX,
                "[gather_qmm] an expert or batch index was out of range (kernel site %d); "
                "the affected outputs were not written.",
                st);
  return NVFP4_OK;
}

int nvfp4_dequantize(void* out, int out_dtype, const uint32_t* w, const uint8_t* scales,
                     int64_t rows, int64_t K, nvfp4_stream stream) {
  if (!valid_dtype(out_dtype))
    return fail(NVFP4_ERR_INVALID, "[dequantize] Only real floating types are supported.");
  if (int r = check_qdims("dequantize", rows, K)) return r;
  if (rows > 0 && (!out || !w || !scales))
    return fail(NVFP4_ERR_INVALID, "[dequantize] null pointer argument.");
  return check_cuda(nvfp4::launch_dequantize(out, out_dtype, reinterpret_cast<const uint8_t*>(w),
                                             scales, rows, K, (cudaStream_t)stream),
                    "dequantize");
}

int nvfp4_quantize(uint32_t* wq, uint8_t* scales, const void* w, int w_dtype, int64_t rows,
                   int64_t K, nvfp4_stream stream) {
  if (!valid_dtype(w_dtype))
    return fail(NVFP4_ERR_INVALID,
                "[quantize] Only real floating types can be quantized.");
  if (int r = check_qdims("quantize", rows, K)) return r;
  if (rows > 0 && (!wq || !scales || !w))
    return fail(NVFP4_ERR_INVALID, "[quantize] null pointer argument.");
  if ((reinterpret_cast<uintptr_t>(wq) & 7) != 0)
    return fail(NVFP4_ERR_INVALID, "[quantize] wq must be 8-byte aligned.");
  return check_cuda(nvfp4::launch_quantize(reinterpret_cast<uint8_t*>(wq), scales, w, w_dtype,
                                           rows, K, (cudaStream_t)stream),
                    "quantize");
}

int nvfp4_gather_qmm(void* out, const void* x, int dtype, const uint32_t* w,
                     const uint8_t* scales, const uint32_t* lhs_indices,
                     const uint32_t* rhs_indices, int64_t pairs, int64_t n_x_batches,
                     int64_t n_experts, int64_t M, int64_t N, int64_t K, int sorted_indices,
                     nvfp4_stream stream) {
  (void)sorted_indices;
  if (!valid_dtype(dtype))
    return fail(NVFP4_ERR_INVALID, "[gather_qmm] Only real floating types are supported.");
  if (int r = check_qdims("gather_qmm", N, K)) return r;
  if (pairs < 0 || M < 0 || n_x_batches < 0 || n_experts <= 0)
    return fail(NVFP4_ERR_INVALID, "[gather_qmm] Invalid batch sizes.");
  if (pairs > 0x7fffffff / 8 || M > 0x7fffffff)
    return fail(NVFP4_ERR_UNSUPPORTED, "[gather_qmm] too many pairs.");
  if (pairs == 0 || M == 0 || N == 0) return NVFP4_OK;
  if (!out || !x || !w || !scales)
    return fail(NVFP4_ERR_INVALID, "[gather_qmm] null pointer argument.");
  if (!lhs_indices && n_x_batches < pairs)
    return fail(NVFP4_ERR_INVALID,
                "[gather_qmm] without lhs_indices x must hold one batch per pair.");
  nvfp4::QmmArgs a{};
  a.out = out;
  a.x = x;
  a.w = reinterpret_cast<const uint8_t*>(w);
  a.s = scales;
  a.lhs = lhs_indices;
  a.rhs = rhs_indices;
  a.P = pairs;
  a.N = N;
  a.K = K;
  a.M = (int)M;
  a.mchunks = (int)((M + 7) / 8);
  a.dtype = dtype;
  a.w_stride = N * (K / 2);
  a.s_stride = N * (K / 16);
  a.n_x_batches = n_x_batches;
  a.n_experts = n_experts;
  if ((int64_t)a.P * a.mchunks > 65535 * 1024LL)
    return fail(NVFP4_ERR_UNSUPPORTED, "[gather_qmm] too many pairs.");
  return check_cuda(nvfp4::launch_qmm_gather(a, (cudaStream_t)stream, first_pdl()),
                    "gather_qmm");
}

int nvfp4_quantize_activations(uint32_t* xq, uint8_t* scales, const void* x, int dtype,
                               int64_t M, int64_t K, nvfp4_stream stream) {
  if (!valid_dtype(dtype))
    return fail(NVFP4_ERR_INVALID,
                "[qqmm] Only real floating types except float64 are supported.");
  if (int r = check_qdims("qqmm", M, K)) return r;
  if (M == 0) return NVFP4_OK;
  if (!xq || !scales || !x) return fail(NVFP4_ERR_INVALID, "[qqmm] null pointer argument.");
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(xq) & 7) != 0)
    return fail(NVFP4_ERR_INVALID, "[qqmm] x must be 16-byte and xq 8-byte aligned.");
  return check_cuda(nvfp4::launch_qx_quantize(reinterpret_cast<uint8_t*>(xq), scales, x, dtype,
                                              M, K, (cudaStream_t)stream),
                    "qqmm");
}

struct QqmmLayout {
  size_t qx_off, sx_off, part_off, ticket_off, total;
  int bn, n_tiles, m_tiles, splits;
};

static int device_sm_count() {
  int dev = 0, v = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
    return 148;
  return v;
}

static QqmmLayout qqmm_layout(int64_t M, int64_t N, int64_t K) {
  QqmmLayout L{};
  nvfp4::qqmm_plan(M, N, K, device_sm_count(), &L.bn, &L.n_tiles, &L.m_tiles, &L.splits);
  L.qx_off = 0;
  L.sx_off = align_up((size_t)M * (size_t)(K / 2), 256);
  L.part_off = align_up(L.sx_off + (size_t)M * (size_t)(K / 16), 256);
  const size_t tiles = (size_t)L.n_tiles * L.m_tiles;
  const size_t part = L.splits > 1 ? tiles * L.splits * (size_t)L.bn * 128 * sizeof(float) : 0;
  L.ticket_off = align_up(L.part_off + part, 256);
  L.total = align_up(L.ticket_off + tiles * sizeof(unsigned), 256);
  return L;
}

size_t nvfp4_qqmm_workspace_size(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0 || K % 256 != 0) return 0;
  return qqmm_layout(M, N, K).total;
}

int nvfp4_qqmm(void* y, const void* x, int dtype, const uint32_t* w, const uint8_t* scales,
               int64_t M, int64_t N, int64_t K, void* workspace, size_t workspace_bytes,
               nvfp4_stream stream) {
  if (!valid_dtype(dtype))
    return fail(NVFP4_ERR_INVALID,
                "[qqmm] Only real floating types except float64 are supported but first "
                "argument dtype is not.");
  if (int r = check_qdims("qqmm", N, K)) return r;
  if (M < 0) return fail(NVFP4_ERR_INVALID, "[qqmm] Invalid M.");
  if (M == 0 || N == 0) return NVFP4_OK;
  if (K % 256 != 0)
    return fail(NVFP4_ERR_UNSUPPORTED, "[qqmm] K=%lld: the tensor-core path needs K %% 256 == 0.",
                (long long)K);
  if (M >= (1ll << 31) || N >= (1ll << 31))
    return fail(NVFP4_ERR_UNSUPPORTED, "[qqmm] M and N must be below 2^31.");
  if (!y || !x || !w || !scales) return fail(NVFP4_ERR_INVALID, "[qqmm] null pointer argument.");
  if (!aligned16(x) || !aligned16(w) || !aligned16(scales))
    return fail(NVFP4_ERR_INVALID, "[qqmm] x, w and scales must be 16-byte aligned.");
  const QqmmLayout L = qqmm_layout(M, N, K);
  if (!workspace || workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(NVFP4_ERR_WORKSPACE, "[qqmm] workspace needs %zu bytes, 256-byte aligned.",
                L.total);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint8_t* qx = ws + L.qx_off;
  uint8_t* sx = ws + L.sx_off;
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = nvfp4::launch_qx_quantize(qx, sx, x, dtype, M, K, st);
  if (e != cudaSuccess) return check_cuda(e, "qqmm");
  nvfp4::QqmmArgs a{};
  if (nvfp4::map_codes(&a.ma, w, N, K, 128) != cudaSuccess ||
      nvfp4::map_scales(&a.msa, scales, N, K, 128) != cudaSuccess ||
      nvfp4::map_codes(&a.mb, qx, M, K, L.bn) != cudaSuccess ||
      nvfp4::map_scales(&a.msb, sx, M, K, L.bn) != cudaSuccess)
    return fail(NVFP4_ERR_UNSUPPORTED, "[qqmm] tensor map encoding failed.");
  a.out = y;
  a.dtype = dtype;
  a.M = M;
  a.N = N;
  a.K = K;
  a.bn = L.bn;
  a.n_tiles = L.n_tiles;
  a.m_tiles = L.m_tiles;
  a.splits = L.splits;
  a.partial = reinterpret_cast<float*>(ws + L.part_off);
  a.ticket = reinterpret_cast<unsigned*>(ws + L.ticket_off);
  return check_cuda(nvfp4::launch_qqmm(a, st), "qqmm");
}

int nvfp4_quantized_matmul(void* y, const void* x, int dtype, const uint32_t* w,
                           const uint8_t* scales, int64_t M, int64_t N, int64_t K,
                           nvfp4_stream stream) {
  if (!valid_dtype(dtype))
    return fail(NVFP4_ERR_INVALID,
                "[quantized_matmul] Only real floating types are supported.");
  if (int r = check_qdims("quantized_matmul", N, K)) return r;
  if (M < 0) return fail(NVFP4_ERR_INVALID, "[quantized_matmul] Invalid M.");
  // Many 16-bit rows: the tcgen05 GEMM streams W once per 64 rows.
  if (M > 8 && dtype != NVFP4_F32 && K % nvfp4::gemm_slab_k() == 0 && N > 0 &&
      N < (1ll << 31) && M < (1ll << 31) && x && y && w && scales && aligned16(x) &&
      aligned16(w) && aligned16(scales)) {
    nvfp4::GemmArgs g{};
    g.mode = 0;
    g.K = (int)K;
    g.Mrows = (int)N;
    g.Mrows_shared = 0;
    g.shared_group = -1;
    g.implicit_M = (int)M;
    g.out = y;
    g.out_dtype = dtype;
    g.out_ld = N;
    if (nvfp4::map_codes(&g.mc0, w, N, K, 128) == cudaSuccess &&
        nvfp4::map_scales(&g.ms0, scales, N, K, 128) == cudaSuccess &&
        nvfp4::map_rows16(&g.mb, x, dtype == NVFP4_BF16, M, K, K) == cudaSuccess) {
      const int tiles = (int)((M + nvfp4::gemm_tile_tokens() - 1) / nvfp4::gemm_tile_tokens());
      return check_cuda(nvfp4::launch_nvfp4_gemm(g, dtype == NVFP4_F16, tiles,
                                                 (cudaStream_t)stream, first_pdl()),
                        "quantized_matmul");
    }
  }
  // One "pair" whose M rows are the whole activation matrix.
  return nvfp4_gather_qmm(y, x, dtype, w, scales, nullptr, nullptr, 1, 1, 1, M, N, K, 0,
                          stream);
}

int nvfp4_rms_norm(void* y, const void* x, const void* weight, int dtype, int64_t rows,
                   int64_t dims, float eps, nvfp4_stream stream) {
  const char* op = "rms_norm";
  if (!valid_dtype(dtype))
    return fail(NVFP4_ERR_INVALID, "[%s] Received unsupported type.", op);
  if (rows < 0 || dims <= 0)
    return fail(NVFP4_ERR_INVALID, "[%s] Input must have at least 1 dimension.", op);
  if (!(eps >= 0.f)) return fail(NVFP4_ERR_INVALID, "[%s] eps must be >= 0.", op);
  if (rows == 0) return NVFP4_OK;
  if (!y || !x) return fail(NVFP4_ERR_INVALID, "[%s] null pointer argument.", op);
  nvfp4::NormArgs a{};
  a.x = x;
  a.w = weight;
  a.y = y;
  a.T = rows;
  a.H = dims;
  a.eps = eps;
  a.dtype = dtype;
  return check_cuda(nvfp4::launch_rms_norm(a, (cudaStream_t)stream, first_pdl()), op);
}

size_t moe_router_workspace_size(int64_t T, int64_t H, int64_t E) {
  return router_layout(T, H, E).total;
}

static int router_checks(const char* op, int64_t T, int64_t H, int64_t E, int k,
                         const void* x, const void* G) {
  if (T < 0 || H <= 0 || E <= 0) return fail(NVFP4_ERR_INVALID, "[%s] Invalid shape.", op);
  if (k <= 0 || k > E || k > 32)
    return fail(NVFP4_ERR_INVALID, "[%s] top_k must be in [1, min(E, 32)].", op);
  if (E > 512) return fail(NVFP4_ERR_UNSUPPORTED, "[%s] at most 512 experts.", op);
  if (nvfp4::router_ksplit(H) == 0 || H % 8 != 0)
    return fail(NVFP4_ERR_UNSUPPORTED, "[%s] hidden size must be a multiple of 128.", op);
  if (T > 0 && (!x || !G)) return fail(NVFP4_ERR_INVALID, "[%s] null pointer argument.", op);
  if (G && !aligned16(G))
    return fail(NVFP4_ERR_INVALID, "[%s] router weight must be 16-byte aligned.", op);
  return NVFP4_OK;
}

int moe_router_topk(uint32_t* inds, float* weights, const void* x, int dtype,
                    const uint16_t* gate_w_bf16, const float* bias, int64_t T, int64_t H,
                    int64_t E, int k, int norm_topk_prob, void* workspace,
                    size_t workspace_bytes, nvfp4_stream stream) {
  if (!valid_dtype(dtype))
    return fail(NVFP4_ERR_INVALID, "[router] Only real floating types are supported.");
  if (int r = router_checks("router", T, H, E, k, x, gate_w_bf16)) return r;
  if (T == 0) return NVFP4_OK;
  if (!inds || !weights) return fail(NVFP4_ERR_INVALID, "[router] null output pointer.");
  const RouterLayout L = router_layout(T, H, E);
  if (!workspace || workspace_bytes < L.total)
    return fail(NVFP4_ERR_WORKSPACE, "[router] workspace of %zu bytes required.", L.total);
  nvfp4::RouterArgs a{};
  a.x = x;
  a.dtype = dtype;
  a.G = gate_w_bf16;
  a.bias = bias;
  a.T = T;
  a.H = H;
  a.E = E;
  a.k = k;
  a.norm = norm_topk_prob;
  a.ksplit = L.ksplit;
  a.counters = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + L.counters_off);
  a.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + L.partial_off);
  a.inds = inds;
  a.wts = weights;
  return check_cuda(nvfp4::launch_router(a, (cudaStream_t)stream, first_pdl()), "router");
}

size_t moe_block_workspace_size(const moe_layer_desc* layer, int64_t T) {
  if (!layer || T < 0) return 0;
  return block_layout(layer, T).total;
}

int moe_workspace_init(void* workspace, size_t bytes, nvfp4_stream stream) {
  if (!workspace && bytes) return fail(NVFP4_ERR_INVALID, "[workspace] null pointer.");
  return check_cuda(cudaMemsetAsync(workspace, 0, bytes, (cudaStream_t)stream), "workspace");
}

static int check_layer(const char* op, const moe_layer_desc* L, int dtype, int64_t T);
static int prefill_impl(void* y, const void* x, const void* residual, int dtype, int64_t T,
                        const moe_layer_desc* L, const uint32_t* inds, const float* wts, char* ws,
                        const BlockLayout& B, nvfp4_stream stream, bool pdl_first);
static int gate_up_impl(float* act, int64_t act_ld, const void* x, int dtype, int64_t T,
                        const moe_layer_desc* L, const uint32_t* inds, nvfp4_stream stream,
                        bool pdl, bool inds_static);
static int down_impl(void* y, const float* act, int64_t act_ld, const void* residual, int dtype,
                     int64_t T, const moe_layer_desc* L, const uint32_t* inds,
                     const float* weights, nvfp4_stream stream, bool pdl);

// moe_block_forward with the grouped path from grouped_min_tokens tokens on
// (the no-alloc entry keeps the GEMV engine up to T = 8, whose workspace fits
// its static scratch).
static int block_forward_impl(const char* op, void* y, const void* x, const void* residual,
                              int dtype, int64_t T, const moe_layer_desc* L,
                              const uint32_t* inds_in, const float* weights_in,
                              uint32_t* inds_out, float* weights_out, void* workspace,
                              size_t workspace_bytes, nvfp4_stream stream,
                              int64_t grouped_min_tokens);

int moe_block_forward(void* y, const void* x, const void* residual, int dtype, int64_t T,
                      const moe_layer_desc* L, const uint32_t* inds_in, const float* weights_in,
                      uint32_t* inds_out, float* weights_out, void* workspace,
                      size_t workspace_bytes, nvfp4_stream stream) {
  return block_forward_impl("moe_block", y, x, residual, dtype, T, L, inds_in, weights_in,
                            inds_out, weights_out, workspace, workspace_bytes, stream,
                            kGroupedMinTokens);
}

static int block_forward_impl(const char* op, void* y, const void* x, const void* residual,
                              int dtype, int64_t T, const moe_layer_desc* L,
                              const uint32_t* inds_in, const float* weights_in,
                              uint32_t* inds_out, float* weights_out, void* workspace,
                              size_t workspace_bytes, nvfp4_stream stream,
                              int64_t grouped_min_tokens) {
  if (int r = check_layer(op, L, dtype, T)) return r;
  const int64_t H = L->hidden, E = L->n_experts;
  const int k = (int)L->top_k;
  if (T == 0) return NVFP4_OK;
  if (!y || !x) return fail(NVFP4_ERR_INVALID, "[%s] null activation pointer.", op);
  if (!inds_in && !L->router_w)
    return fail(NVFP4_ERR_INVALID, "[%s] either inds_in or router_w is required.", op);
  if (inds_in && !weights_in)
    return fail(NVFP4_ERR_INVALID, "[%s] weights_in is required with inds_in.", op);
  const BlockLayout B = block_layout(L, T, grouped_min_tokens);
  if (!workspace || workspace_bytes < B.total)
    return fail(NVFP4_ERR_WORKSPACE, "[%s] workspace of %zu bytes required.", op, B.total);
  char* ws = static_cast<char*>(workspace);
  cudaStream_t s = (cudaStream_t)stream;

  const uint32_t* inds = inds_in;
  const float* wts = weights_in;
  if (!inds_in) {
    if (int r = router_checks(op, T, H, E, k, x, L->router_w)) return r;
    uint32_t* ri = inds_out ? inds_out : reinterpret_cast<uint32_t*>(ws + B.inds_off);
    float* rw = weights_out ? weights_out : reinterpret_cast<float*>(ws + B.wts_off);
    nvfp4::RouterArgs ra{};
    ra.x = x;
    ra.dtype = dtype;
    ra.G = L->router_w;
    ra.bias = L->router_bias;
    ra.T = T;
    ra.H = H;
    ra.E = E;
    ra.k = k;
    ra.norm = L->norm_topk_prob;
    ra.ksplit = B.router.ksplit;
    ra.counters = reinterpret_cast<unsigned*>(ws + B.router.counters_off);
    ra.partial = reinterpret_cast<float*>(ws + B.router.partial_off);
    ra.inds = ri;
    ra.wts = rw;
    if (int r = check_cuda(nvfp4::launch_router(ra, s, first_pdl()), op)) return r;
    inds = ri;
    wts = rw;
  } else if (inds_out || weights_out) {
    if (inds_out &&
        cudaMemcpyAsync(inds_out, inds_in, T * k * sizeof(uint32_t), cudaMemcpyDeviceToDevice,
                        s) != cudaSuccess)
      return check_cuda(cudaGetLastError(), op);
    if (weights_out &&
        cudaMemcpyAsync(weights_out, weights_in, T * k * sizeof(float), cudaMemcpyDeviceToDevice,
                        s) != cudaSuccess)
      return check_cuda(cudaGetLastError(), op);
  }
  // The prefill kernels move activations 16 bytes at a time.
  if (B.prefill && aligned16(x) && aligned16(y) && (!residual || aligned16(residual))) {
    const bool routed_here = inds_in == nullptr;
    const bool copied = inds_in && (inds_out || weights_out);
    return prefill_impl(y, x, residual, dtype, T, L, inds, wts, ws, B, stream,
                        /*pdl_first=*/!copied && (routed_here || first_pdl()));
  }
  float* act = reinterpret_cast<float*>(ws + B.act_off);
  // Kernels after the first overlap their predecessor (PDL).  When the router
  // ran, the gate/up kernel reads the routing only after its dependency wait.
  const bool routed_here = inds_in == nullptr;
  const bool copied = inds_in && (inds_out || weights_out);
  if (int r = gate_up_impl(act, B.act_ld, x, dtype, T, L, inds, stream,
                           /*pdl=*/!copied && (routed_here || first_pdl()),
                           /*inds_static=*/!routed_here))
    return r;
  return down_impl(y, act, B.act_ld, residual, dtype, T, L, inds, wts, stream, /*pdl=*/true);
}

// The FP4-terms prefill after the sort: x as four NVFP4 term rows per slot,
// gate/up + SwiGLU and down on the block-scaled tensor cores, act as terms in
// between, then the same combine.
static int prefill_fp4_tail(void* y, const void* x, const void* residual, int dtype, int64_t T,
                            const moe_layer_desc* L, const float* wts, char* ws,
                            const BlockLayout& B, cudaStream_t s, int64_t x_ld, int out_dtype,
                            int64_t sh_row0, int64_t sh_rows) {
  const char* op = "moe_block";
  const int64_t H = L->hidden, I = L->inter, E = L->n_experts, Is = L->shared_inter;
  const bool sh = Is > 0;
  int* pos = reinterpret_cast<int*>(ws + B.pos_off);
  int4* tiles = reinterpret_cast<int4*>(ws + B.tiles_off);
  int* ntiles = reinterpret_cast<int*>(ws + B.ntiles_off);
  float* act32 = reinterpret_cast<float*>(ws + B.act32_off);
  float* Y = reinterpret_cast<float*>(ws + B.y_off);
  uint8_t* xtc = reinterpret_cast<uint8_t*>(ws + B.xtc_off);
  uint8_t* xts = reinterpret_cast<uint8_t*>(ws + B.xts_off);
  float* xtf = reinterpret_cast<float*>(ws + B.xtf_off);
  uint8_t* atc = reinterpret_cast<uint8_t*>(ws + B.atc_off);
  uint8_t* ats = reinterpret_cast<uint8_t*>(ws + B.ats_off);
  float* atf = reinterpret_cast<float*>(ws + B.atf_off);
  const int64_t trows = B.S * nvfp4::kFp4Terms;

  nvfp4::TermsArgs tx{};
  tx.src = x;
  tx.src_dtype = dtype;
  tx.rows = T;
  tx.K = H;
  tx.src_ld = x_ld;
  tx.dst_map = pos;  // token t feeds slots pos[t * k + j]
  tx.map_stride = (int)L->top_k;
  tx.map_count = (int)L->top_k;
  tx.extra_base = sh ? B.P : -1;  // and its shared-expert slot P + (t - sh_row0)
  tx.extra_lo = sh_row0;
  tx.extra_hi = sh_row0 + sh_rows;
  tx.codes = xtc;
  tx.scales = xts;
  tx.fac = xtf;
  if (int r = check_cuda(nvfp4::launch_rows_to_terms(tx, s), op)) return r;

  auto maps_ok = [](std::initializer_list<cudaError_t> l) {
    for (cudaError_t e : l)
      if (e != cudaSuccess) return false;
    return true;
  };
  nvfp4::GemmFp4Args g{};
  g.mode = 1;
  g.K = (int)H;
  g.Mrows = (int)I;
  g.Mrows_shared = (int)Is;
  g.shared_group = sh ? (int)E : -1;
  bool ok = maps_ok({nvfp4::map_codes(&g.mc0, L->gate.w, E * I, H, 64),
                     nvfp4::map_scales(&g.ms0, L->gate.scales, E * I, H, 64),
                     nvfp4::map_codes(&g.mc1, L->up.w, E * I, H, 64),
                     nvfp4::map_scales(&g.ms1, L->up.scales, E * I, H, 64),
                     nvfp4::map_codes(&g.mb[0], xtc, trows, H, 32),
                     nvfp4::map_scales(&g.msb[0], xts, trows, H, 32),
                     nvfp4::map_codes(&g.mb[1], xtc, trows, H, 64),
                     nvfp4::map_scales(&g.msb[1], xts, trows, H, 64),
                     nvfp4::map_codes(&g.mb[2], xtc, trows, H, 96),
                     nvfp4::map_scales(&g.msb[2], xts, trows, H, 96),
                     nvfp4::map_codes(&g.mb[3], xtc, trows, H, 128),
                     nvfp4::map_scales(&g.msb[3], xts, trows, H, 128)});
  if (sh)
    ok = ok && maps_ok({nvfp4::map_codes(&g.mcs0, L->shared_gate.w, Is, H, 64),
                        nvfp4::map_scales(&g.mss0, L->shared_gate.scales, Is, H, 64),
                        nvfp4::map_codes(&g.mcs1, L->shared_up.w, Is, H, 64),
                        nvfp4::map_scales(&g.mss1, L->shared_up.scales, Is, H, 64)});
  g.bfac = xtf;
  g.tiles = tiles;
  g.ntiles = ntiles;
  g.max_tiles = (int)B.max_tiles;
  g.out = act32;
  g.out_ld = B.act_ld;

  nvfp4::GemmFp4Args d{};
  d.mode = 2;
  d.K = (int)I;
  d.Mrows = (int)H;
  d.Mrows_shared = (int)H;
  d.shared_group = sh ? (int)E : -1;
  ok = ok && maps_ok({nvfp4::map_codes(&d.mc0, L->down.w, E * H, I, 128),
                      nvfp4::map_scales(&d.ms0, L->down.scales, E * H, I, 128),
                      nvfp4::map_codes(&d.mb[0], atc, trows, I, 32),
                      nvfp4::map_scales(&d.msb[0], ats, trows, I, 32),
                      nvfp4::map_codes(&d.mb[1], atc, trows, I, 64),
                      nvfp4::map_scales(&d.msb[1], ats, trows, I, 64),
                      nvfp4::map_codes(&d.mb[2], atc, trows, I, 96),
                      nvfp4::map_scales(&d.msb[2], ats, trows, I, 96),
                      nvfp4::map_codes(&d.mb[3], atc, trows, I, 128),
                      nvfp4::map_scales(&d.msb[3], ats, trows, I, 128)});
  if (sh)
    ok = ok && maps_ok({nvfp4::map_codes(&d.mcs0, L->shared_down.w, H, I, 128),
                        nvfp4::map_scales(&d.mss0, L->shared_down.scales, H, I, 128)});
  d.bfac = atf;
  d.tiles = tiles;
  d.ntiles = ntiles;
  d.max_tiles = (int)B.max_tiles;
  d.out = Y;
  d.out_ld = H;
  if (!ok) return fail(NVFP4_ERR_CUDA, "[%s] tensor-map encoding failed.", op);

  if (int r = check_cuda(nvfp4::launch_nvfp4_gemm_fp4(g, (int)B.max_tiles, s), op)) return r;

  nvfp4::TermsArgs ta{};
  ta.src = act32;
  ta.src_dtype = NVFP4_F32;
  ta.rows = B.S;
  ta.K = I;
  ta.src_ld = B.act_ld;
  ta.dst_map = nullptr;
  ta.extra_base = -1;  // identity: slot r
  ta.extra_lo = ta.extra_hi = 0;
  ta.codes = atc;
  ta.scales = ats;
  ta.fac = atf;
  if (int r = check_cuda(nvfp4::launch_rows_to_terms(ta, s), op)) return r;

  if (int r = check_cuda(nvfp4::launch_nvfp4_gemm_fp4(d, (int)B.max_tiles, s), op)) return r;

  nvfp4::CombineArgs c{};
  c.Y = Y;
  c.pos = pos;
  c.wts = wts;
  c.T = (int)T;
  c.k = (int)L->top_k;
  c.P = (int)B.P;
  c.H = (int)H;
  c.with_shared = sh ? 1 : 0;
  c.scaling = L->routed_scaling;
  c.residual = residual;
  c.y = y;
  c.dtype = out_dtype;
  c.sh_row0 = (int)sh_row0;
  c.sh_rows = (int)sh_rows;
  return check_cuda(nvfp4::launch_moe_combine(c, s, true), op);
}

// Prefill: sort pairs by expert, gate/up + SwiGLU and down as tcgen05
// grouped GEMMs over expert-sorted token slots (the shared expert is one more
// group holding every token), then the weighted per-token combine.  Both GEMMs
// take f16 operands: x and the intermediate go through rows_to_f16 first
// (per-row power-of-two scale, re-applied in the GEMM epilogue).
static int prefill_impl(void* y, const void* x, const void* residual, int dtype, int64_t T,
                        const moe_layer_desc* L, const uint32_t* inds, const float* wts, char* ws,
                        const BlockLayout& B, nvfp4_stream stream, bool pdl_first) {
  const char* op = "moe_block";
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t H = L->hidden, I = L->inter, E = L->n_experts;
  const bool sh = L->shared_inter > 0;
  int* brow = reinterpret_cast<int*>(ws + B.brow_off);
  int* pos = reinterpret_cast<int*>(ws + B.pos_off);
  int4* tiles = reinterpret_cast<int4*>(ws + B.tiles_off);
  int* ntiles = reinterpret_cast<int*>(ws + B.ntiles_off);
  __half* x16 = reinterpret_cast<__half*>(ws + B.x16_off);
  float* xscale = reinterpret_cast<float*>(ws + B.xscale_off);
  float* act32 = reinterpret_cast<float*>(ws + B.act32_off);
  __half* act16 = reinterpret_cast<__half*>(ws + B.act16_off);
  float* ascale = reinterpret_cast<float*>(ws + B.ascale_off);
  float* Y = reinterpret_cast<float*>(ws + B.y_off);

  nvfp4::SortArgs sa{};
  sa.inds = inds;
  sa.T = (int)T;
  sa.k = (int)L->top_k;
  sa.E = (int)E;
  sa.P = (int)B.P;
  sa.with_shared = sh ? 1 : 0;
  sa.brow = brow;
  sa.pos = pos;
  sa.tiles = tiles;
  sa.ntiles = ntiles;
  const bool fp4 = use_fp4_terms() && B.fp4;
  sa.tile_tokens = fp4 ? nvfp4::kFp4TileTokens : 0;
  if (int r = check_cuda(nvfp4::launch_moe_sort(sa, s, pdl_first), op)) return r;
  if (fp4) return prefill_fp4_tail(y, x, residual, dtype, T, L, wts, ws, B, s, H, dtype, 0, T);

  // x rows in slot order (shared-expert slots P.. hold tokens 0..T-1).
  nvfp4::RowsArgs rx{};
  rx.src = x;
  rx.src_dtype = dtype;
  rx.src_map = brow;
  rx.rows = (int)B.S;
  rx.K = (int)H;
  rx.src_ld = H;
  rx.dst = x16;
  rx.dst_ld = H;
  rx.scale = xscale;
  if (int r = check_cuda(nvfp4::launch_rows_to_f16(rx, s, true), op)) return r;

  // Tensor maps: routed banks stack E groups of rows; 64-row boxes for the
  // gate/up halves of a gate/up tile, 128-row boxes for down.
  const int64_t Is = L->shared_inter;
  auto maps_ok = [](std::initializer_list<cudaError_t> l) {
    for (cudaError_t e : l)
      if (e != cudaSuccess) return false;
    return true;
  };
  nvfp4::GemmArgs g{};
  g.mode = 1;
  g.K = (int)H;
  g.Mrows = (int)I;
  g.Mrows_shared = (int)Is;
  g.shared_group = sh ? (int)E : -1;
  bool ok = maps_ok({nvfp4::map_codes(&g.mc0, L->gate.w, E * I, H, 64),
                     nvfp4::map_scales(&g.ms0, L->gate.scales, E * I, H, 64),
                     nvfp4::map_codes(&g.mc1, L->up.w, E * I, H, 64),
                     nvfp4::map_scales(&g.ms1, L->up.scales, E * I, H, 64),
                     nvfp4::map_rows16(&g.mb, x16, false, B.S, H, H)});
  if (sh)
    ok = ok && maps_ok({nvfp4::map_codes(&g.mcs0, L->shared_gate.w, Is, H, 64),
                        nvfp4::map_scales(&g.mss0, L->shared_gate.scales, Is, H, 64),
                        nvfp4::map_codes(&g.mcs1, L->shared_up.w, Is, H, 64),
                        nvfp4::map_scales(&g.mss1, L->shared_up.scales, Is, H, 64)});
  g.bscale = xscale;
  g.tiles = tiles;
  g.ntiles = ntiles;
  g.out = act32;
  g.out_dtype = NVFP4_F32;
  g.out_ld = B.act_ld;

  nvfp4::GemmArgs d{};
  d.mode = 2;
  d.K = (int)I;
  d.Mrows = (int)H;
  d.Mrows_shared = (int)H;
  d.shared_group = sh ? (int)E : -1;
  ok = ok && maps_ok({nvfp4::map_codes(&d.mc0, L->down.w, E * H, I, 128),
                      nvfp4::map_scales(&d.ms0, L->down.scales, E * H, I, 128),
                      nvfp4::map_rows16(&d.mb, act16, false, B.S, I, B.act_ld)});
  if (sh)
    ok = ok && maps_ok({nvfp4::map_codes(&d.mcs0, L->shared_down.w, H, I, 128),
                        nvfp4::map_scales(&d.mss0, L->shared_down.scales, H, I, 128)});
  d.bscale = ascale;
  d.tiles = tiles;
  d.ntiles = ntiles;
  d.out = Y;
  d.out_dtype = NVFP4_F32;
  d.out_ld = H;
  if (!ok) return fail(NVFP4_ERR_CUDA, "[%s] tensor-map encoding failed.", op);

  if (int r = check_cuda(nvfp4::launch_nvfp4_gemm(g, true, (int)B.max_tiles, s, true), op))
    return r;

  nvfp4::RowsArgs ra{};
  ra.src = act32;
  ra.src_dtype = NVFP4_F32;
  ra.rows = (int)B.S;
  ra.K = (int)I;
  ra.src_ld = B.act_ld;
  ra.dst = act16;
  ra.dst_ld = B.act_ld;
  ra.scale = ascale;
  if (int r = check_cuda(nvfp4::launch_rows_to_f16(ra, s, true), op)) return r;

  if (int r = check_cuda(nvfp4::launch_nvfp4_gemm(d, true, (int)B.max_tiles, s, true), op))
    return r;

  nvfp4::CombineArgs c{};
  c.Y = Y;
  c.pos = pos;
  c.wts = wts;
  c.T = (int)T;
  c.k = (int)L->top_k;
  c.P = (int)B.P;
  c.H = (int)H;
  c.with_shared = sh ? 1 : 0;
  c.scaling = L->routed_scaling;
  c.residual = residual;
  c.y = y;
  c.dtype = dtype;
  return check_cuda(nvfp4::launch_moe_combine(c, s, true), op);
}

static int check_layer(const char* op, const moe_layer_desc* L, int dtype, int64_t T) {
  if (!L) return fail(NVFP4_ERR_INVALID, "[%s] null layer descriptor.", op);
  if (!valid_dtype(dtype))
    return fail(NVFP4_ERR_INVALID, "[%s] Only real floating types are supported.", op);
  const int64_t H = L->hidden, I = L->inter, E = L->n_experts, Is = L->shared_inter;
  if (T < 0 || H <= 0 || I <= 0 || E <= 0 || Is < 0 || L->top_k <= 0 || L->top_k > E)
    return fail(NVFP4_ERR_INVALID, "[%s] Invalid layer shape.", op);
  if (H % 128 || I % 128 || Is % 128)
    return fail(NVFP4_ERR_UNSUPPORTED,
                "[%s] hidden and intermediate sizes must be multiples of 128 "
                "(use nvfp4_gather_qmm for other shapes).",
                op);
  return NVFP4_OK;
}

int moe_gate_up_swiglu(float* act, int64_t act_ld, const void* x, int dtype, int64_t T,
                       const moe_layer_desc* L, const uint32_t* inds, nvfp4_stream stream) {
  return gate_up_impl(act, act_ld, x, dtype, T, L, inds, stream, first_pdl(), true);
}

static int gate_up_impl(float* act, int64_t act_ld, const void* x, int dtype, int64_t T,
                        const moe_layer_desc* L, const uint32_t* inds, nvfp4_stream stream,
                        bool pdl, bool inds_static) {
  const char* op = "moe_gate_up_swiglu";
  if (int r = check_layer(op, L, dtype, T)) return r;
  if (T == 0) return NVFP4_OK;
  if (!act || !x || !inds) return fail(NVFP4_ERR_INVALID, "[%s] null pointer argument.", op);
  if (act_ld < std::max(L->inter, L->shared_inter) || act_ld % 8)
    return fail(NVFP4_ERR_INVALID,
                "[%s] act_ld must be a multiple of 8 and >= the intermediate size.", op);
  if (!aligned16(x) || !aligned16(act))
    return fail(NVFP4_ERR_INVALID, "[%s] x and act must be 16-byte aligned.", op);
  if (!L->gate.w || !L->up.w || !L->gate.scales || !L->up.scales || !aligned16(L->gate.w) ||
      !aligned16(L->up.w))
    return fail(NVFP4_ERR_INVALID, "[%s] routed banks need 16-byte aligned codes.", op);
  const int64_t H = L->hidden, I = L->inter, Is = L->shared_inter;
  if (Is > 0 && (!L->shared_gate.w || !L->shared_up.w || !L->shared_gate.scales ||
                 !L->shared_up.scales || !aligned16(L->shared_gate.w) ||
                 !aligned16(L->shared_up.w)))
    return fail(NVFP4_ERR_INVALID, "[%s] shared banks need 16-byte aligned codes.", op);
  nvfp4::GateUpArgs ga{};
  ga.x = x;
  ga.dtype = dtype;
  ga.T = T;
  ga.H = H;
  ga.I = I;
  ga.Is = Is;
  ga.E = L->n_experts;
  ga.k = (int)L->top_k;
  ga.kk = (int)L->top_k + (Is > 0 ? 1 : 0);
  ga.inds = inds;
  ga.gw = reinterpret_cast<const uint8_t*>(L->gate.w);
  ga.gs = L->gate.scales;
  ga.uw = reinterpret_cast<const uint8_t*>(L->up.w);
  ga.us = L->up.scales;
  ga.w_stride = I * (H / 2);
  ga.s_stride = I * (H / 16);
  if (Is > 0) {
    ga.sgw = reinterpret_cast<const uint8_t*>(L->shared_gate.w);
    ga.sgs = L->shared_gate.scales;
    ga.suw = reinterpret_cast<const uint8_t*>(L->shared_up.w);
    ga.sus = L->shared_up.scales;
  }
  ga.act = act;
  ga.act_ld = act_ld;
  ga.inds_static = inds_static ? 1 : 0;
  ga.bulk = use_bulk() ? 1 : 0;
  return check_cuda(nvfp4::launch_moe_gateup(ga, (cudaStream_t)stream, pdl), op);
}

int moe_down_combine(void* y, const float* act, int64_t act_ld, const void* residual, int dtype,
                     int64_t T, const moe_layer_desc* L, const uint32_t* inds,
                     const float* weights, nvfp4_stream stream) {
  return down_impl(y, act, act_ld, residual, dtype, T, L, inds, weights, stream, first_pdl());
}

static int down_impl(void* y, const float* act, int64_t act_ld, const void* residual, int dtype,
                     int64_t T, const moe_layer_desc* L, const uint32_t* inds,
                     const float* weights, nvfp4_stream stream, bool pdl) {
  const char* op = "moe_down_combine";
  if (int r = check_layer(op, L, dtype, T)) return r;
  if (T == 0) return NVFP4_OK;
  if (!y || !act || !inds || !weights)
    return fail(NVFP4_ERR_INVALID, "[%s] null pointer argument.", op);
  const int64_t H = L->hidden, I = L->inter, Is = L->shared_inter;
  const int kk = (int)L->top_k + (Is > 0 ? 1 : 0);
  if (act_ld < std::max(I, Is) || act_ld % 8)
    return fail(NVFP4_ERR_INVALID,
                "[%s] act_ld must be a multiple of 8 and >= the intermediate size.", op);
  if (!aligned16(act)) return fail(NVFP4_ERR_INVALID, "[%s] act must be 16-byte aligned.", op);
  if (!L->down.w || !L->down.scales || !aligned16(L->down.w))
    return fail(NVFP4_ERR_INVALID, "[%s] routed banks need 16-byte aligned codes.", op);
  if (Is > 0 && (!L->shared_down.w || !L->shared_down.scales || !aligned16(L->shared_down.w)))
    return fail(NVFP4_ERR_INVALID, "[%s] shared banks need 16-byte aligned codes.", op);
  if (nvfp4::down_smem_bytes(std::max(I, Is), kk) > 220 * 1024)
    return fail(NVFP4_ERR_UNSUPPORTED, "[%s] top_k * intermediate too large.", op);
  nvfp4::DownArgs da{};
  da.act = act;
  da.act_ld = act_ld;
  da.T = T;
  da.H = H;
  da.I = I;
  da.Is = Is;
  da.E = L->n_experts;
  da.k = (int)L->top_k;
  da.kk = kk;
  da.Ipad = (int)std::max(I, Is);
  da.inds = inds;
  da.wts = weights;
  da.scaling = L->routed_scaling;
  da.dw = reinterpret_cast<const uint8_t*>(L->down.w);
  da.ds = L->down.scales;
  da.w_stride = H * (I / 2);
  da.s_stride = H * (I / 16);
  if (Is > 0) {
    da.sdw = reinterpret_cast<const uint8_t*>(L->shared_down.w);
    da.sds = L->shared_down.scales;
  }
  da.residual = residual;
  da.y = y;
  da.dtype = dtype;
  // The down kernel always follows a gate/up kernel (ours or, under
  // NVFP4_LAUNCH_PDL, by the caller's contract), which waited for whatever
  // produced the routing before letting this grid launch.
  da.inds_static = 1;
  da.bulk = use_bulk() ? 1 : 0;
  return check_cuda(nvfp4::launch_moe_down(da, (cudaStream_t)stream, pdl), op);
}

// ---------------------------------------------------------------------------
// moe_block_forward_noalloc: the same sparse MoE block for callers that can
// not allocate device memory -- hosts that embed this library behind another
// runtime's allocator or operator interface and have no way to hand it a
// separately owned workspace buffer, or that must keep a fixed device-memory
// footprint once loaded.  Its scratch is the static array below instead of a
// caller workspace; nothing here calls cudaMalloc, cudaFree or any other
// allocating routine.
//
// The array lives in every GPU that loads this library until the process
// exits.  Its device address is looked up with cudaGetSymbolAddress on the
// first call made on each device (with that device current), so that first
// call should come before any stream capture.  All calls on a device share
// the array and it keeps the last call's contents: the router's tickets,
// which must start at zero, are cleared on the stream at every call, and
// calls that overlap on the GPU (other streams, other host threads) race on
// it.  Limit: kNoAllocScratchBytes, i.e. up to T = 8 tokens at Laguna XS 2.1
// sizes (E = 256, H = 2048, top-8 + shared expert of 512).
static constexpr size_t kNoAllocScratchBytes = 256 * 1024;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
// The no-alloc block runs the GEMV engine up to T = 8 (its workspace fits the
// scratch at Laguna sizes) and the grouped path beyond, where the scratch
// rejects Laguna-sized layers.
constexpr int64_t kNoAllocGroupedMinTokens = 9;

static int noalloc_scratch(void** out) {
  static void* addr[64] = {};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return check_cuda(e, "moe_block_noalloc");
  if (dev < 0 || dev >= 64)
    return fail(NVFP4_ERR_UNSUPPORTED, "[moe_block_noalloc] device ordinal %d >= 64.", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return check_cuda(e, "moe_block_noalloc");
    addr[dev] = p;
  }
  *out = addr[dev];
  return NVFP4_OK;
}

extern "C" int moe_block_forward_noalloc(void* y, const void* x, const void* residual, int dtype,
                                         int64_t T, const moe_layer_desc* L,
                                         const uint32_t* inds_in, const float* weights_in,
                                         uint32_t* inds_out, float* weights_out,
                                         nvfp4_stream stream) {
  const char* op = "moe_block_noalloc";
  if (int r = check_layer(op, L, dtype, T)) return r;
  if (T == 0) return NVFP4_OK;
  const BlockLayout B = block_layout(L, T, kNoAllocGroupedMinTokens);
  if (B.total > kNoAllocScratchBytes)
    return fail(NVFP4_ERR_WORKSPACE,
                "[%s] T=%lld needs %zu bytes of scratch but the static scratch holds %zu "
                "(up to T=8 at Laguna sizes); use moe_block_forward with a workspace.",
                op, (long long)T, B.total, kNoAllocScratchBytes);
  void* ws = nullptr;
  if (int r = noalloc_scratch(&ws)) return r;
  // The router's tickets must start at zero; the array keeps the last call's
  // contents, so clear them on this call's stream.
  const size_t counters = (size_t)((T + 7) / 8) * sizeof(unsigned);
  cudaError_t e = cudaMemsetAsync(static_cast<char*>(ws) + B.router.counters_off, 0, counters,
                                  (cudaStream_t)stream);
  if (e != cudaSuccess) return check_cuda(e, op);
  return block_forward_impl(op, y, x, residual, dtype, T, L, inds_in, weights_in, inds_out,
                            weights_out, ws, kNoAllocScratchBytes, stream,
                            kNoAllocGroupedMinTokens);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Expert-parallel block over all ranks' tokens (gather / reduce-scatter form).
extern "C" {

size_t moe_ep_partial_workspace_size(const moe_layer_desc* L, int64_t T) {
  if (!L || T <= 0) return 0;
  return block_layout(L, T).total;
}

int moe_ep_partial_forward(float* y_partial, const void* x, int64_t x_ld, int dtype, int64_t T,
                           const moe_layer_desc* L, const uint32_t* inds, const float* weights,
                           int64_t expert_base, int64_t shared_row0, int64_t shared_rows,
                           void* workspace, size_t workspace_bytes, nvfp4_stream stream) {
  return moe_ep_partial_forward_typed(y_partial, NVFP4_F32, x, x_ld, dtype, T, L, inds, weights,
                                      expert_base, shared_row0, shared_rows, workspace,
                                      workspace_bytes, stream);
}

int moe_ep_partial_forward_typed(void* y_partial, int partial_dtype, const void* x, int64_t x_ld,
                                 int dtype, int64_t T, const moe_layer_desc* L,
                                 const uint32_t* inds, const float* weights, int64_t expert_base,
                                 int64_t shared_row0, int64_t shared_rows, void* workspace,
                                 size_t workspace_bytes, nvfp4_stream stream) {
  const char* op = "moe_ep_partial";
  if (int r = check_layer(op, L, dtype, T)) return r;
  if (partial_dtype != NVFP4_F32 && partial_dtype != NVFP4_BF16)
    return fail(NVFP4_ERR_INVALID, "[%s] partials are f32 or bf16.", op);
  if (T == 0) return NVFP4_OK;
  if (!y_partial || !x || !inds || !weights)
    return fail(NVFP4_ERR_INVALID, "[%s] null pointer argument.", op);
  if (x_ld < L->hidden || expert_base < 0)
    return fail(NVFP4_ERR_INVALID, "[%s] invalid x_ld or expert_base.", op);
  const bool sh = L->shared_inter > 0;
  if (sh && (shared_row0 < 0 || shared_rows <= 0 || shared_row0 + shared_rows > T))
    return fail(NVFP4_ERR_INVALID, "[%s] shared rows outside the batch.", op);
  const BlockLayout B = block_layout(L, T);
  const int esz = dtype == NVFP4_F32 ? 4 : 2;
  if (!B.prefill || !B.fp4 || !aligned16(x) || (x_ld * esz) % 16 || !aligned16(y_partial))
    return fail(NVFP4_ERR_UNSUPPORTED,
                "[%s] needs T > 8 tokens, Laguna-sized layers, 16-byte aligned rows and a tile "
                "list (E + T * top_k / 32 + T / 32 entries) that fits in shared memory.", op);
  if (!workspace || workspace_bytes < B.total)
    return fail(NVFP4_ERR_WORKSPACE, "[%s] workspace of %zu bytes required.", op, B.total);
  char* ws = static_cast<char*>(workspace);
  cudaStream_t s = (cudaStream_t)stream;
  nvfp4::SortArgs sa{};
  sa.inds = inds;
  sa.T = (int)T;
  sa.k = (int)L->top_k;
  sa.E = (int)L->n_experts;
  sa.P = (int)B.P;
  sa.with_shared = sh ? 1 : 0;
  sa.sh_row0 = sh ? (int)shared_row0 : 0;
  sa.sh_rows = sh ? (int)shared_rows : 0;
  sa.brow = reinterpret_cast<int*>(ws + B.brow_off);
  sa.pos = reinterpret_cast<int*>(ws + B.pos_off);
  sa.tiles = reinterpret_cast<int4*>(ws + B.tiles_off);
  sa.ntiles = reinterpret_cast<int*>(ws + B.ntiles_off);
  sa.tile_tokens = nvfp4::kFp4TileTokens;
  sa.e_base = (int)expert_base;
  sa.skip_foreign = 1;
  if (int r = check_cuda(nvfp4::launch_moe_sort(sa, s, first_pdl()), op)) return r;
  return prefill_fp4_tail(y_partial, x, nullptr, dtype, T, L, weights, ws, B, s, x_ld,
                          partial_dtype, sh ? shared_row0 : 0, sh ? shared_rows : 0);
}

int moe_ep_finish(void* y, const float* partial, const void* shared, const void* residual,
                  int dtype, int64_t T, int64_t H, nvfp4_stream stream) {
  return moe_ep_finish_typed(y, partial, NVFP4_F32, shared, residual, dtype, T, H, stream);
}

int moe_ep_finish_typed(void* y, const void* partial, int partial_dtype, const void* shared,
                        const void* residual, int dtype, int64_t T, int64_t H,
                        nvfp4_stream stream) {
  if (!valid_dtype(dtype) || !valid_dtype(partial_dtype))
    return fail(NVFP4_ERR_INVALID, "[moe_ep_finish] invalid dtype.");
  if (T < 0 || H <= 0) return fail(NVFP4_ERR_INVALID, "[moe_ep_finish] invalid shape.");
  if (T > 0 && (!y || !partial))
    return fail(NVFP4_ERR_INVALID, "[moe_ep_finish] null pointer argument.");
  return check_cuda(nvfp4::launch_ep_finish(y, partial, partial_dtype, shared, residual, dtype, T, H,
                                            (cudaStream_t)stream),
                    "moe_ep_finish");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Serial decode through a stack of sparse layers in one persistent launch.
namespace {
struct StackLayout {
  size_t act_off, xb0_off, xb1_off, bar_off, y32_off, gu_off, rbar_off, x32_off, total;
};

// act / xb: the mma.sync stack; y32 / gu: the FP4 stack's f32 partials
// (per segment -- and, routed, per I block -- and [2][2][kk][2][I] per K part,
// both by layer parity);
// bar: grid-barrier / dependency counters; rbar: the routed stack's counters
// followed by its exchange area (fs_xchg_u64 words, zeroed at each launch),
// x32 its residual stream at launch boundaries ([2][H] f32, by parity).
StackLayout stack_layout(const moe_layer_desc* L0, int dtype_bytes) {
  StackLayout S;
  const int64_t kk = L0->top_k + (L0->shared_inter > 0 ? 1 : 0);
  S.act_off = 0;
  S.xb0_off = align_up((size_t)kk * L0->inter * sizeof(float), 256);
  S.xb1_off = align_up(S.xb0_off + (size_t)L0->hidden * dtype_bytes, 256);
  S.bar_off = align_up(S.xb1_off + (size_t)L0->hidden * dtype_bytes, 256);
  S.y32_off = align_up(S.bar_off + (2 + 2 * nvfp4::kStackMaxLayers) * sizeof(unsigned), 256);
  // segment partials: [2][kk][H] for the given-routing stack, [2][kk][I / 64][H]
  // (per I block of a CTA pair) for the routed one
  S.gu_off = align_up(S.y32_off + 2 * (size_t)kk * (L0->inter / 64) * L0->hidden * sizeof(float),
                      256);
  S.rbar_off = align_up(S.gu_off + 4 * (size_t)kk * 2 * L0->inter * sizeof(float), 256);
  S.x32_off = align_up(S.rbar_off + nvfp4::kFsCounters * sizeof(unsigned) +
                           nvfp4::fs_xchg_u64((int)L0->hidden, (int)L0->n_experts,
                                              nvfp4::kFsMaxLayers) * sizeof(uint64_t),
                       256);
  S.total = align_up(S.x32_off + 2 * (size_t)L0->hidden * sizeof(float), 256);
  return S;
}

int device_sms() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return sms;
}

// Tensor maps of the FP4 stack, cached per calling thread by (stack position,
// bank pointer, shape, box): a decode step re-issues the same layers, and a map
// is a pure function of those.
struct MapKey {
  const void* p;
  int64_t rows, K;
  int box;
  int kind;
  bool operator==(const MapKey& o) const {
    return p == o.p && rows == o.rows && K == o.K && box == o.box && kind == o.kind;
  }
};
struct MapCacheEntry {
  MapKey key;
  CUtensorMap map;
  bool valid;
};
thread_local std::vector<MapCacheEntry> t_map_cache;

// kind 0: codes in 128-byte rows (K 256 per box), 1: scale bytes, 2: codes in
// 32-byte rows (K 64 per box, the routed stack's down tiles).
bool cached_map(size_t idx, CUtensorMap* out, const void* p, int64_t rows, int64_t K, int box,
                int kind) {
  if (t_map_cache.size() <= idx) t_map_cache.resize(idx + 1);
  MapCacheEntry& e = t_map_cache[idx];
  const MapKey key{p, rows, K, box, kind};
  if (!e.valid || !(e.key == key)) {
    e.valid = false;
    const cudaError_t r = kind == 1   ? nvfp4::map_scales(&e.map, p, rows, K, box)
                          : kind == 2 ? nvfp4::map_codes_k64(&e.map, p, rows, K, box)
                                      : nvfp4::map_codes(&e.map, p, rows, K, box);
    if (r != cudaSuccess) return false;
    e.key = key;
    e.valid = true;
  }
  *out = e.map;
  return true;
}

// Layers per launch of the FP4 stack (the tensor maps ride in the kernel
// parameters), 0 when the FP4 stack does not take this shape or is switched off.
int fp4_stack_layers_per_launch(const moe_layer_desc* L0, bool routed = false) {
  if (!use_fp4_decode()) return 0;
  const int kk = (int)(L0->top_k + (L0->shared_inter > 0 ? 1 : 0));
  if (L0->shared_inter > 0 && L0->shared_inter != L0->inter) return 0;
  if (L0->hidden > 4096 || L0->inter > 4096) return 0;
  if (routed && (L0->n_experts > 256 || L0->top_k > 8 ||
                 L0->hidden / nvfp4::kFsRedRows > nvfp4::kFsMaxReducers))
    return 0;
  if (!nvfp4::decode_stack_fp4_supported((int)L0->hidden, (int)L0->inter, kk, device_sms(),
                                         routed))
    return 0;
  const int mpl = L0->shared_inter > 0 ? 2 * nvfp4::kFsMapsRouted : nvfp4::kFsMapsRouted;
  return std::min(nvfp4::kFsMaxLayers, nvfp4::kFsMaxMaps / mpl);
}

// Shape checks shared by both stacks: every layer as layer 0.
int check_stack_layers(const char* op, const moe_layer_desc* layers, int64_t n_layers, int dtype) {
  if (!layers || n_layers <= 0) return fail(NVFP4_ERR_INVALID, "[%s] no layers.", op);
  if (n_layers > nvfp4::kStackMaxLayers)
    return fail(NVFP4_ERR_UNSUPPORTED, "[%s] at most %d layers per call.", op,
                nvfp4::kStackMaxLayers);
  for (int64_t l = 0; l < n_layers; l++)
    if (int r = check_layer(op, &layers[l], dtype, 1)) return r;
  const moe_layer_desc* L0 = &layers[0];
  for (int64_t l = 1; l < n_layers; l++) {
    const moe_layer_desc* Ll = &layers[l];
    if (Ll->hidden != L0->hidden || Ll->inter != L0->inter || Ll->n_experts != L0->n_experts ||
        Ll->top_k != L0->top_k || Ll->shared_inter != L0->shared_inter)
      return fail(NVFP4_ERR_UNSUPPORTED, "[%s] layers must share one shape.", op);
  }
  const int64_t H = L0->hidden, I = L0->inter, Is = L0->shared_inter;
  if (H % 256 || I % 256 || (Is != 0 && Is != I) || L0->top_k > 16 || L0->n_experts > 0x7fffffff)
    return fail(NVFP4_ERR_UNSUPPORTED, "[%s] unsupported layer shape.", op);
  return NVFP4_OK;
}

// The block-scaled FP4 stack over n_layers layers, per_launch layers per
// launch.  Given routing: inds / weights [n_layers] device pointers.  Routed:
// inds_out / wts_out (nullable, entries nullable) receive each layer's routing.
int run_fp4_stack(const char* op, void* y, const void* x, int dtype, int64_t n_layers,
                  const moe_layer_desc* layers, const uint32_t* const* inds,
                  const float* const* weights, bool routed, bool residual,
                  const void* const* norm_w, float eps, uint32_t* const* inds_out,
                  float* const* wts_out, int per_launch, const StackLayout& S, char* ws,
                  cudaStream_t s) {
  const moe_layer_desc* L0 = &layers[0];
  const int64_t H = L0->hidden, I = L0->inter, E = L0->n_experts, k = L0->top_k;
  const int64_t Is = L0->shared_inter;
  const int kk = (int)(k + (Is > 0 ? 1 : 0));
  for (int64_t l = 0; l < n_layers; l++) {
    const moe_layer_desc* Ll = &layers[l];
    const nvfp4_bank* banks[6] = {&Ll->gate, &Ll->up, &Ll->down,
                                  &Ll->shared_gate, &Ll->shared_up, &Ll->shared_down};
    for (int b = 0; b < (Is > 0 ? 6 : 3); b++)
      if (!banks[b]->w || !banks[b]->scales || !aligned16(banks[b]->w) ||
          !aligned16(banks[b]->scales))
        return fail(NVFP4_ERR_UNSUPPORTED, "[%s] banks must be 16-byte aligned.", op);
    if (Ll->routed_scaling != L0->routed_scaling)
      return fail(NVFP4_ERR_UNSUPPORTED, "[%s] layers must share routed_scaling.", op);
    if (routed) {
      if (!Ll->router_w || !aligned16(Ll->router_w))
        return fail(NVFP4_ERR_INVALID, "[%s] layer %lld needs a 16-byte aligned router weight.",
                    op, (long long)l);
      if (Ll->norm_topk_prob != L0->norm_topk_prob)
        return fail(NVFP4_ERR_UNSUPPORTED, "[%s] layers must share norm_topk_prob.", op);
      if (norm_w && !norm_w[l])
        return fail(NVFP4_ERR_INVALID, "[%s] null norm weight for layer %lld.", op,
                    (long long)l);
    } else if (!inds[l] || !weights[l]) {
      return fail(NVFP4_ERR_INVALID, "[%s] null routing for layer %lld.", op, (long long)l);
    }
  }
  static thread_local nvfp4::FsArgs F;
  const int mpl = Is > 0 ? 2 * nvfp4::kFsMapsRouted : nvfp4::kFsMapsRouted;
  F.H = (int)H;
  F.I = (int)I;
  F.E = (int)E;
  F.k = (int)k;
  F.kk = kk;
  F.nks = nvfp4::decode_stack_fp4_nks((int)I, kk, device_sms());
  F.mpl = mpl;
  F.dtype = dtype;
  F.routed = routed ? 1 : 0;
  F.residual = residual ? 1 : 0;
  F.norm = L0->norm_topk_prob ? 1 : 0;
  F.has_norm = norm_w ? 1 : 0;
  F.eps = eps;
  F.scaling = L0->routed_scaling;
  // a bounded wait gives up after ~1 s (2e9 cycles); the test flag shortens
  // it to ~1 ms and withholds one release, so the waits behind it expire
  F.test_skip_release = (t_launch_flags & NVFP4_LAUNCH_TEST_EXPIRE) ? 1 : 0;
  F.budget = F.test_skip_release ? 2000000LL : 2000000000LL;
  F.x0 = x;
  F.y = y;
  F.Yp = reinterpret_cast<float*>(ws + S.y32_off);
  F.GUp = reinterpret_cast<float*>(ws + S.gu_off);
  if (routed) {
    F.bar = reinterpret_cast<unsigned*>(ws + S.rbar_off);
    F.XG = reinterpret_cast<unsigned long long*>(ws + S.rbar_off +
                                                 nvfp4::kFsCounters * sizeof(unsigned));
    F.Hres = reinterpret_cast<float*>(ws + S.x32_off);
  } else {
    F.bar = reinterpret_cast<unsigned*>(ws + S.bar_off);
    F.XG = nullptr;
    F.Hres = nullptr;
  }
  // routed and given-routing stacks keep separate tensor-map cache entries
  const size_t cache0 = routed ? (size_t)nvfp4::kStackMaxLayers * 2 * nvfp4::kFsMapsRouted : 0;
  for (int64_t l0 = 0; l0 < n_layers; l0 += per_launch) {
    const int nl = (int)std::min<int64_t>(per_launch, n_layers - l0);
    F.L = nl;
    F.l0 = (int)l0;
    F.first = l0 == 0;
    F.last = l0 + nl == n_layers;
    bool ok = true;
    for (int li = 0; li < nl; li++) {
      const moe_layer_desc* Ll = &layers[l0 + li];
      CUtensorMap* m = &F.maps[li * mpl];
      const size_t c0 = cache0 + (size_t)(l0 + li) * 2 * nvfp4::kFsMapsRouted;
      // the routed stack's down tiles are K = 64 steps (its CTA pairs' I blocks)
      const int dk = routed ? 2 : 0;
      ok = ok && cached_map(c0 + 0, &m[0], Ll->gate.w, E * I, H, 64, 0) &&
           cached_map(c0 + 1, &m[1], Ll->gate.scales, E * I, H, 64, 1) &&
           cached_map(c0 + 2, &m[2], Ll->up.w, E * I, H, 64, 0) &&
           cached_map(c0 + 3, &m[3], Ll->up.scales, E * I, H, 64, 1) &&
           cached_map(c0 + 4, &m[4], Ll->down.w, E * H, I, 128, dk) &&
           cached_map(c0 + 5, &m[5], Ll->down.scales, E * H, I, 128, 1);
      if (Is > 0)
        ok = ok && cached_map(c0 + 6, &m[6], Ll->shared_gate.w, Is, H, 64, 0) &&
             cached_map(c0 + 7, &m[7], Ll->shared_gate.scales, Is, H, 64, 1) &&
             cached_map(c0 + 8, &m[8], Ll->shared_up.w, Is, H, 64, 0) &&
             cached_map(c0 + 9, &m[9], Ll->shared_up.scales, Is, H, 64, 1) &&
             cached_map(c0 + 10, &m[10], Ll->shared_down.w, H, I, 128, dk) &&
             cached_map(c0 + 11, &m[11], Ll->shared_down.scales, H, I, 128, 1);
      nvfp4::FsLayer& d = F.layer[li];
      if (routed) {
        d.inds = inds_out ? inds_out[l0 + li] : nullptr;
        d.wts = wts_out ? wts_out[l0 + li] : nullptr;
        d.router_w = Ll->router_w;
        d.router_b = Ll->router_bias;
        d.norm_w = norm_w ? norm_w[l0 + li] : nullptr;
      } else {
        d.inds = const_cast<uint32_t*>(inds[l0 + li]);
        d.wts = const_cast<float*>(weights[l0 + li]);
        d.router_w = nullptr;
        d.router_b = nullptr;
        d.norm_w = nullptr;
      }
    }
    if (!ok) return fail(NVFP4_ERR_CUDA, "[%s] tensor-map encoding failed.", op);
    if (int r = check_cuda(nvfp4::launch_decode_stack_fp4(F, s), op)) return r;
  }
  return NVFP4_OK;
}
}  // namespace

extern "C" size_t moe_decode_stack_workspace_size(const moe_layer_desc* layers,
                                                  int64_t n_layers) {
  if (!layers || n_layers <= 0) return 0;
  return stack_layout(&layers[0], 4).total;  // sized for the widest dtype
}

extern "C" int moe_decode_stack_uses_fp4(const moe_layer_desc* layers, int64_t n_layers) {
  if (!layers || n_layers <= 0) return 0;
  return fp4_stack_layers_per_launch(&layers[0]) > 0 ? 1 : 0;
}

extern "C" int moe_decode_stack_launches(const moe_layer_desc* layers, int64_t n_layers) {
  if (!layers || n_layers <= 0) return 0;
  const int per = fp4_stack_layers_per_launch(&layers[0]);
  return per > 0 ? (int)((n_layers + per - 1) / per) : 1;
}

extern "C" int moe_decode_stack_forward(void* y, const void* x, int dtype, int64_t n_layers,
                                        const moe_layer_desc* layers,
                                        const uint32_t* const* inds, const float* const* weights,
                                        void* workspace, size_t workspace_bytes,
                                        nvfp4_stream stream) {
  const char* op = "moe_decode_stack";
  if (int r = check_stack_layers(op, layers, n_layers, dtype)) return r;
  if (!y || !x || !inds || !weights)
    return fail(NVFP4_ERR_INVALID, "[%s] null pointer argument.", op);
  const moe_layer_desc* L0 = &layers[0];
  const int64_t H = L0->hidden, I = L0->inter, E = L0->n_experts, k = L0->top_k;
  const int64_t Is = L0->shared_inter;
  const int per_launch = fp4_stack_layers_per_launch(L0);
  // mma.sync stack: each consumer thread holds at most 2 x chunks and 4 act
  // chunks of 8 values, and its rings must fit on chip
  const int kk = (int)(k + (Is > 0 ? 1 : 0));
  if (per_launch == 0 && (H > 4096 || kk * I > 8192))
    return fail(NVFP4_ERR_UNSUPPORTED, "[%s] layer too wide for the persistent stack.", op);
  if (per_launch == 0 && nvfp4::decode_stack_smem_bytes((int)H, (int)I, kk) > 227 * 1024)
    return fail(NVFP4_ERR_UNSUPPORTED, "[%s] layer too large for the on-chip rings.", op);
  const int esz = dtype == NVFP4_F32 ? 4 : 2;
  if (!aligned16(x) || !aligned16(y))
    return fail(NVFP4_ERR_UNSUPPORTED, "[%s] x and y must be 16-byte aligned.", op);
  const StackLayout S = stack_layout(L0, esz);
  if (!workspace || workspace_bytes < S.total)
    return fail(NVFP4_ERR_WORKSPACE, "[%s] workspace of %zu bytes required.", op, S.total);
  if (per_launch > 0)
    return run_fp4_stack(op, y, x, dtype, n_layers, layers, inds, weights, false, false, nullptr,
                         0.f, nullptr, nullptr, per_launch, S, static_cast<char*>(workspace),
                         (cudaStream_t)stream);
  nvfp4::StackArgs A{};
  A.L = (int)n_layers;
  A.H = (int)H;
  A.I = (int)I;
  A.E = (int)E;
  A.k = (int)k;
  A.kk = kk;
  A.dtype = dtype;
  A.gw_stride = I * (H / 2);
  A.gs_stride = I * (H / 16);
  A.dw_stride = H * (I / 2);
  A.ds_stride = H * (I / 16);
  A.x0 = x;
  A.y = y;
  char* ws = static_cast<char*>(workspace);
  A.act = reinterpret_cast<float*>(ws + S.act_off);
  A.xb[0] = ws + S.xb0_off;
  A.xb[1] = ws + S.xb1_off;
  A.bar = reinterpret_cast<unsigned*>(ws + S.bar_off);
  A.xmax = A.bar + 2;
  A.amax = A.xmax + nvfp4::kStackMaxLayers;
  for (int64_t l = 0; l < n_layers; l++) {
    const moe_layer_desc* Ll = &layers[l];
    const nvfp4_bank* banks[6] = {&Ll->gate, &Ll->up, &Ll->down,
                                  &Ll->shared_gate, &Ll->shared_up, &Ll->shared_down};
    for (int b = 0; b < (Is > 0 ? 6 : 3); b++)
      if (!banks[b]->w || !banks[b]->scales || !aligned16(banks[b]->w) ||
          !aligned16(banks[b]->scales))
        return fail(NVFP4_ERR_UNSUPPORTED, "[%s] banks must be 16-byte aligned.", op);
    if (!inds[l] || !weights[l])
      return fail(NVFP4_ERR_INVALID, "[%s] null routing for layer %lld.", op, (long long)l);
    nvfp4::StackLayer& d = A.layer[l];
    d.gw = reinterpret_cast<const uint8_t*>(Ll->gate.w);
    d.gs = Ll->gate.scales;
    d.uw = reinterpret_cast<const uint8_t*>(Ll->up.w);
    d.us = Ll->up.scales;
    d.dw = reinterpret_cast<const uint8_t*>(Ll->down.w);
    d.ds = Ll->down.scales;
    if (Is > 0) {
      d.sgw = reinterpret_cast<const uint8_t*>(Ll->shared_gate.w);
      d.sgs = Ll->shared_gate.scales;
      d.suw = reinterpret_cast<const uint8_t*>(Ll->shared_up.w);
      d.sus = Ll->shared_up.scales;
      d.sdw = reinterpret_cast<const uint8_t*>(Ll->shared_down.w);
      d.sds = Ll->shared_down.scales;
    }
    d.inds = inds[l];
    d.wts = weights[l];
    d.scaling = Ll->routed_scaling;
  }
  return check_cuda(nvfp4::launch_decode_stack(A, (cudaStream_t)stream), op);
}

// Serial decode with the router inside the stack (the routed FP4 stack).
extern "C" int moe_decode_stack_routed_launches(const moe_layer_desc* layers, int64_t n_layers) {
  if (!layers || n_layers <= 0) return 0;
  const int per = fp4_stack_layers_per_launch(&layers[0], true);
  return per > 0 ? (int)((n_layers + per - 1) / per) : 0;
}

extern "C" int moe_decode_stack_routed_forward(void* y, const void* x, int dtype,
                                               int64_t n_layers, const moe_layer_desc* layers,
                                               int residual, const void* const* norm_w,
                                               float norm_eps, uint32_t* const* inds_out,
                                               float* const* weights_out, void* workspace,
                                               size_t workspace_bytes, nvfp4_stream stream) {
  const char* op = "moe_decode_stack_routed";
  if (int r = check_stack_layers(op, layers, n_layers, dtype)) return r;
  if (!y || !x) return fail(NVFP4_ERR_INVALID, "[%s] null pointer argument.", op);
  const moe_layer_desc* L0 = &layers[0];
  const int per_launch = fp4_stack_layers_per_launch(L0, true);
  if (per_launch == 0 || dtype == NVFP4_F32)
    return fail(NVFP4_ERR_UNSUPPORTED,
                "[%s] this layer shape, dtype or launch mode has no routed stack (bf16 or f16, "
                "hidden 1024 or 2048, inter 512 / 1024 / 2048, at most 256 experts, top_k <= 8, "
                "NVFP4_LAUNCH_EXACT_DECODE clear); use moe_block_forward per layer.",
                op);
  if (!aligned16(x) || !aligned16(y))
    return fail(NVFP4_ERR_UNSUPPORTED, "[%s] x and y must be 16-byte aligned.", op);
  const StackLayout S = stack_layout(L0, dtype == NVFP4_F32 ? 4 : 2);
  if (!workspace || workspace_bytes < S.total)
    return fail(NVFP4_ERR_WORKSPACE, "[%s] workspace of %zu bytes required.", op, S.total);
  if (norm_w && !(norm_eps >= 0.f))
    return fail(NVFP4_ERR_INVALID, "[%s] norm epsilon must be >= 0.", op);
  return run_fp4_stack(op, y, x, dtype, n_layers, layers, nullptr, nullptr, true, residual != 0,
                       norm_w, norm_eps, inds_out, weights_out, per_launch, S,
                       static_cast<char*>(workspace), (cudaStream_t)stream);
}

// ---------------------------------------------------------------------------
// Expert-parallel dispatch / combine.
extern "C" int moe_ep_dispatch(void* send_x, int32_t* send_ids, int32_t* pos,
                               int32_t* send_counts, const void* x, int dtype,
                               const uint32_t* inds, int64_t T, int k, int64_t H,
                               int64_t experts_per_rank, int world, nvfp4_stream stream) {
  const char* op = "moe_ep_dispatch";
  if (!valid_dtype(dtype))
    return fail(NVFP4_ERR_INVALID, "[%s] Only real floating types are supported.", op);
  if (T < 0 || k <= 0 || H <= 0 || experts_per_rank <= 0 || world <= 0)
    return fail(NVFP4_ERR_INVALID, "[%s] Invalid shape.", op);
  if (world > 64) return fail(NVFP4_ERR_UNSUPPORTED, "[%s] at most 64 ranks.", op);
  const int esz = dtype == NVFP4_F32 ? 4 : 2;
  if ((H * esz) % 16 || !aligned16(x) || !aligned16(send_x))
    return fail(NVFP4_ERR_UNSUPPORTED, "[%s] rows must be 16-byte aligned.", op);
  if (T == 0) {
    return check_cuda(cudaMemsetAsync(send_counts, 0, world * sizeof(int32_t),
                                      (cudaStream_t)stream),
                      op);
  }
  if (!send_x || !send_ids || !pos || !send_counts || !x || !inds)
    return fail(NVFP4_ERR_INVALID, "[%s] null pointer argument.", op);
  nvfp4::EpPlanArgs pa{};
  pa.inds = inds;
  pa.T = T;
  pa.k = k;
  pa.experts_per_rank = experts_per_rank;
  pa.world = world;
  pa.pos = pos;
  pa.ids = send_ids;
  pa.counts = send_counts;
  if (int r = check_cuda(nvfp4::launch_ep_plan(pa, (cudaStream_t)stream), op)) return r;
  nvfp4::EpPackArgs ka{};
  ka.x = x;
  ka.T = T;
  ka.k = k;
  ka.H = H;
  ka.esz = esz;
  ka.pos = pos;
  ka.send_x = send_x;
  return check_cuda(nvfp4::launch_ep_pack(ka, (cudaStream_t)stream), op);
}

extern "C" int moe_ep_combine(void* y, const void* y_pairs, const int32_t* pos,
                              const float* weights, const void* shared, const void* residual,
                              int dtype, int64_t T, int k, int64_t H, float scaling,
                              nvfp4_stream stream) {
  const char* op = "moe_ep_combine";
  if (!valid_dtype(dtype))
    return fail(NVFP4_ERR_INVALID, "[%s] Only real floating types are supported.", op);
  if (T < 0 || k <= 0 || H <= 0) return fail(NVFP4_ERR_INVALID, "[%s] Invalid shape.", op);
  if (T == 0) return NVFP4_OK;
  if (!y || !y_pairs || !pos || !weights)
    return fail(NVFP4_ERR_INVALID, "[%s] null pointer argument.", op);
  nvfp4::EpCombineArgs c{};
  c.y = y;
  c.yp = y_pairs;
  c.pos = pos;
  c.wts = weights;
  c.T = T;
  c.k = k;
  c.H = H;
  c.scaling = scaling;
  c.shared = shared;
  c.residual = residual;
  c.dtype = dtype;
  return check_cuda(nvfp4::launch_ep_combine(c, (cudaStream_t)stream), op);
}
