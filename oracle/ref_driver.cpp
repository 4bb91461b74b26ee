// ref_driver.cpp -- C entry points over the reference's OWN compiled CPU
// kernels.  TEST INFRASTRUCTURE ONLY (parity pinning and the timed CPU
// baseline); never linked into the product library.
//
// oracle/Makefile compiles this file together with the reference's
// Vendor/mlx-swift/Source/Cmlx/mlx/mlx/backend/cpu/quantized.cpp, which it
// includes in place from the read-only reference tree (nothing is copied into
// this repository).  The entry points call, unchanged:
//   fp_qmm_t<T,16,4>        backend/cpu/quantized.cpp:491-533
//   detail::FromFP8/ToFP8   backend/cpu/unary_ops.h:120-172
//   detail::Sigmoid         backend/cpu/unary_ops.h:77-84
//   to_fp4_e2m1             backend/cpu/quantized.cpp:1064-1091
//   dequantize_scale<T,16>  backend/cpu/quantized.cpp:49-62
//   _MLX_BFloat16(float)    types/bf16.h:37-58
// The gather loop mirrors fp_bs_qmm_dispatch_mode (quantized.cpp:805-844) for
// row-contiguous operands; the threaded variants only split the output rows
// of the same kernel across std::threads for the CPU baseline (MLX itself runs
// one CPU stream thread, backend/cpu/encoder.h:44-55).
#include "mlx/backend/cpu/quantized.cpp"

#include <algorithm>
#include <cstring>
#include <thread>
#include <vector>

#define REF_API extern "C" __attribute__((visibility("default")))

namespace mc = mlx::core;

REF_API void ref_qmm_f32(const float* x, const uint32_t* w, const uint8_t* s, int M,
                         int N, int K, float* y) {
  mc::fp_qmm_t<float, 16, 4>(y, x, w, s, M, N, K);
}

REF_API void ref_qmm_bf16(const uint16_t* x, const uint32_t* w, const uint8_t* s, int M,
                          int N, int K, uint16_t* y) {
  static_assert(sizeof(mc::bfloat16_t) == 2, "bf16 layout");
  mc::fp_qmm_t<mc::bfloat16_t, 16, 4>(reinterpret_cast<mc::bfloat16_t*>(y),
                                      reinterpret_cast<const mc::bfloat16_t*>(x), w, s, M,
                                      N, K);
}

REF_API void ref_gather_qmm_bf16(const uint16_t* x, const uint32_t* w, const uint8_t* s,
                                 const uint32_t* lhs, const uint32_t* rhs, int pairs, int M,
                                 int N, int K, uint16_t* out) {
  for (int i = 0; i < pairs; i++) {
    long xi = lhs ? lhs[i] : i, wi = rhs[i];
    ref_qmm_bf16(x + xi * M * K, w + wi * (long)N * (K / 8), s + wi * (long)N * (K / 16), M,
                 N, K, out + (long)i * M * N);
  }
}

REF_API void ref_gather_qmm_f32(const float* x, const uint32_t* w, const uint8_t* s,
                                const uint32_t* lhs, const uint32_t* rhs, int pairs, int M,
                                int N, int K, float* out) {
  for (int i = 0; i < pairs; i++) {
    long xi = lhs ? lhs[i] : i, wi = rhs[i];
    ref_qmm_f32(x + xi * M * K, w + wi * (long)N * (K / 8), s + wi * (long)N * (K / 16), M,
                N, K, out + (long)i * M * N);
  }
}

// Threaded bf16 qmm: thread t computes output columns [n0, n1) of every row
// with the unchanged fp_qmm_t kernel.
REF_API void ref_qmm_bf16_mt(const uint16_t* x, const uint32_t* w, const uint8_t* s, int M,
                             int N, int K, uint16_t* y, int threads) {
  threads = std::max(1, std::min(threads, N));
  std::vector<std::thread> pool;
  int chunk = (N + threads - 1) / threads;
  for (int t = 0; t < threads; t++) {
    int n0 = t * chunk, n1 = std::min(N, n0 + chunk);
    if (n0 >= n1) break;
    pool.emplace_back([=] {
      for (int m = 0; m < M; m++)
        ref_qmm_bf16(x + (long)m * K, w + (long)n0 * (K / 8), s + (long)n0 * (K / 16), 1,
                     n1 - n0, K, y + (long)m * N + n0);
    });
  }
  for (auto& th : pool) th.join();
}

// QQMatmul::eval_cpu (quantized.cpp:1322-1360) for T = float / bfloat16_t:
// fp_quantize_dequantize's group loop (quantized.cpp:1093-1129, bits 4,
// group 16) re-typed over plain pointers -- the reference's own function
// takes mlx::core::array, whose allocator is not part of this build -- calling
// the reference's ToFP8, dequantize_scale, to_fp4_e2m1 and FP4_LUT, then the
// unchanged fp_qmm_t on xhat.
template <typename T>
static void ref_fake_quant(const T* w, T* out, size_t w_size) {
  const int group_size = 16;
  size_t n_groups = w_size / group_size;
  for (size_t i = 0; i < n_groups; ++i) {
    size_t idx = i * group_size;
    float scale = -std::numeric_limits<float>::infinity();
    for (int j = 0; j < group_size; ++j) scale = std::max(scale, (float)std::abs((float)w[idx + j]));
    scale /= 6.0f;
    scale = mc::dequantize_scale<float, 16>(mc::detail::ToFP8()(scale));
    for (int j = 0; j < group_size; ++j) {
      float w_el = scale == 0 ? 0.0f : w[idx + j] / scale;
      float output = mc::FP4_LUT[mc::to_fp4_e2m1(w_el)];
      out[idx + j] = static_cast<T>(scale * output);
    }
  }
}

REF_API void ref_fake_quant_f32(const float* x, int M, int K, float* xhat) {
  ref_fake_quant<float>(x, xhat, (size_t)M * K);
}

REF_API void ref_qqmm_f32(const float* x, const uint32_t* w, const uint8_t* s, int M, int N,
                          int K, float* y) {
  std::vector<float> xhat((size_t)M * K);
  ref_fake_quant<float>(x, xhat.data(), xhat.size());
  mc::fp_qmm_t<float, 16, 4>(y, xhat.data(), w, s, M, N, K);
}

REF_API void ref_qqmm_bf16(const uint16_t* x, const uint32_t* w, const uint8_t* s, int M, int N,
                           int K, uint16_t* y) {
  std::vector<mc::bfloat16_t> xhat((size_t)M * K);
  ref_fake_quant<mc::bfloat16_t>(reinterpret_cast<const mc::bfloat16_t*>(x), xhat.data(),
                                 xhat.size());
  mc::fp_qmm_t<mc::bfloat16_t, 16, 4>(reinterpret_cast<mc::bfloat16_t*>(y), xhat.data(), w, s,
                                      M, N, K);
}

REF_API float ref_from_fp8(uint8_t b) { return mc::detail::FromFP8{}(b); }
REF_API uint8_t ref_to_fp8(float f) { return mc::detail::ToFP8{}(f); }
REF_API float ref_sigmoid(float f) { return mc::detail::Sigmoid{}(f); }
REF_API uint8_t ref_to_fp4_e2m1(float f) { return mc::to_fp4_e2m1(f); }
REF_API uint16_t ref_bf16_from_f32(float f) {
  mc::bfloat16_t b(f);
  uint16_t u;
  std::memcpy(&u, &b, 2);
  return u;
}
// bf16 arithmetic as the reference's _MLX_BFloat16 operators perform it.
REF_API uint16_t ref_bf16_mul(uint16_t a, uint16_t b) {
  mc::bfloat16_t x, y;
  std::memcpy(&x, &a, 2);
  std::memcpy(&y, &b, 2);
  mc::bfloat16_t z = x * y;
  uint16_t u;
  std::memcpy(&u, &z, 2);
  return u;
}
REF_API uint16_t ref_bf16_div(uint16_t a, uint16_t b) {
  mc::bfloat16_t x, y;
  std::memcpy(&x, &a, 2);
  std::memcpy(&y, &b, 2);
  mc::bfloat16_t z = x / y;
  uint16_t u;
  std::memcpy(&u, &z, 2);
  return u;
}
