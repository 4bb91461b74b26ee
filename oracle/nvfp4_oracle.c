/*
 * nvfp4_oracle.c -- CPU restatement of the reference's NVFP4 MoE hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference arm may load it.  The product path never calls it and has no CPU
 * fallback.
 *
 * Every routine restates one piece of Layr-Labs/mlxfast-challenge's vendored
 * MLX (paths relative to Vendor/mlx-swift/Source/Cmlx/mlx/mlx/) or of the
 * Laguna model code, and cites the lines it follows.  Parity is pinned by
 * tests/test_oracle.py against (a) the reference's own compiled CPU kernels
 * (oracle/_ref, built from the reference sources by oracle/Makefile) and
 * (b) the known-answer vectors of the reference's NVFP4 tests.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* bf16 (types/bf16.h:37-58): round-to-nearest-even on the top 16 bits;    */
/* NaN maps to 0x7FC0.  Every bf16 op computes in f32 and rounds once      */
/* (types/bf16.h:71-99).                                                    */
/* ------------------------------------------------------------------------ */
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

ORC_API uint16_t orc_bf16_from_f32(float x) {
  if (isnan(x)) return 0x7FC0;
  uint32_t u = f2u(x);
  u += ((u >> 16) & 1u) + 0x7FFFu;
  return (uint16_t)(u >> 16);
}
ORC_API float orc_bf16_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }
static inline float bfr(float x) { return orc_bf16_to_f32(orc_bf16_from_f32(x)); }

/* ------------------------------------------------------------------------ */
/* E2M1 table (backend/cpu/quantized.cpp:31-47): code bit 3 is the sign.    */
/* ------------------------------------------------------------------------ */
static const float FP4_VALUES[16] = {0.0f,  0.5f,  1.0f,  1.5f,  2.0f,  3.0f,  4.0f,  6.0f,
                                     -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};
ORC_API float orc_fp4_value(int code) { return FP4_VALUES[code & 15]; }

/* ------------------------------------------------------------------------ */
/* E4M3 decode (backend/cpu/unary_ops.h:154-172): reinterpret (b & 0x7F)<<7 */
/* as IEEE half and multiply by 256; bit 7 is the sign.  0x7F / 0xFF decode */
/* to +-480 (no NaN), the half-precision subnormal range gives the E4M3     */
/* subnormals exactly.                                                      */
/* ------------------------------------------------------------------------ */
static float half_bits_to_f32(uint16_t h) {
  int e = (h >> 10) & 0x1F, m = h & 0x3FF;
  float v;
  if (e == 0) v = ldexpf((float)m, -24);
  else if (e == 31) v = m ? NAN : INFINITY;
  else v = ldexpf((float)(m | 0x400), e - 25);
  return (h & 0x8000) ? -v : v;
}
ORC_API float orc_e4m3_decode(uint8_t b) {
  float v = half_bits_to_f32((uint16_t)((b & 0x7F) << 7)) * 256.0f;
  return (b & 0x80) ? -v : v;
}

/* E4M3 encode (backend/cpu/unary_ops.h:120-151).  Restated from the same
 * bit-level algorithm: values below 2^-6 go through an f32 add of the
 * denormal magic 2^(141-127) (which rounds to nearest even in hardware),
 * normal values are rebiased and rounded to nearest even on bit 20, and
 * anything at or above the f32 pattern 543<<21 (= 464.0) saturates to 0x7E
 * (448).  The sign is copied from bit 31. */
ORC_API uint8_t orc_e4m3_encode(float f) {
  uint32_t bits = f2u(f);
  uint32_t sign = bits & 0x80000000u;
  bits ^= sign;
  uint8_t r;
  if (bits >= (543u << 21)) {
    r = 0x7E;
  } else if (bits < (121u << 23)) {
    const uint32_t magic = 141u << 23;
    uint32_t low = f2u(u2f(bits) + u2f(magic));
    r = (uint8_t)(low - magic);
  } else {
    uint32_t odd = (bits >> 20) & 1u;
    uint32_t hi = bits + (((uint32_t)(7 - 127) << 23) + 0x7FFFFu) + odd;
    r = (uint8_t)(hi >> 20);
  }
  return (uint8_t)(r | (uint8_t)(sign >> 24));
}

/* ------------------------------------------------------------------------ */
/* Dequantize (ops.cpp:5120-5241 fp_dequantize, nvfp4 branch): element     */
/* k of row r = LUT[nibble k of the packed row, low nibble first] *         */
/* e4m3(scale[r][k/16]).  Exact in f32 and in bf16.                         */
/* ------------------------------------------------------------------------ */
ORC_API void orc_dequantize(const uint32_t *w, const uint8_t *s, int64_t rows, int64_t K,
                            float *out) {
  const int64_t kw = K / 8, kg = K / 16;
  for (int64_t r = 0; r < rows; r++)
    for (int64_t k = 0; k < K; k++) {
      uint32_t word = w[r * kw + k / 8];
      int code = (word >> (4 * (k % 8))) & 15;
      out[r * K + k] = FP4_VALUES[code] * orc_e4m3_decode(s[r * kg + k / 16]);
    }
}

/* ------------------------------------------------------------------------ */
/* Quantize (ops.cpp:4873-4978 fp_quantize, group 16, no global scale, as   */
/* run eagerly on a CPU stream).  For bf16 weights every op of the graph    */
/* rounds to bf16: scale = bf16(max|w| / 6) (ops.cpp:4917-4918), promoted   */
/* to f32 by the multiply with the f32 scale_encode 1.0 (:4923), encoded    */
/* E4M3 (:4924); q = bf16(w / bf16(e4m3(scale))) promoted to f32 (:4925-    */
/* 4926); code = argmin_i |q - bf16(LUT[i])| with strict less-than so the   */
/* first minimum wins (:4958-4959, backend/cpu/arg_reduce.cpp:41-47); 8     */
/* codes packed per uint32 low nibble first (:4960-4962).  An all-zero      */
/* group has scale 0, q = 0/0 = NaN, and argmin of an all-NaN row is 0.     */
/* in_is_bf16 = 0 runs the same graph in f32 (no intermediate rounding).    */
/* ------------------------------------------------------------------------ */
static int argmin_fp4(float q) {
  int best = 0;
  float bv = fabsf(q - FP4_VALUES[0]);
  for (int i = 1; i < 16; i++) {
    float d = fabsf(q - FP4_VALUES[i]);
    if (d < bv) { bv = d; best = i; }
  }
  return best;
}

static void quantize_rows(const float *w, int in_is_bf16, int64_t rows, int64_t K,
                          uint32_t *wq, uint8_t *sq) {
  const int64_t kw = K / 8, kg = K / 16;
  for (int64_t r = 0; r < rows; r++) {
    for (int64_t g = 0; g < kg; g++) {
      const float *src = w + r * K + g * 16;
      float amax = 0.0f;
      for (int j = 0; j < 16; j++) {
        float a = fabsf(src[j]);
        if (a > amax) amax = a; /* max of |w|: exact in bf16 */
      }
      float scale = amax / 6.0f;
      if (in_is_bf16) scale = bfr(scale);
      uint8_t sb = orc_e4m3_encode(scale);
      sq[r * kg + g] = sb;
      float sdec = orc_e4m3_decode(sb); /* exact in bf16 */
      uint32_t words[2] = {0, 0};
      for (int j = 0; j < 16; j++) {
        float q = src[j] / sdec;
        if (in_is_bf16) q = bfr(q);
        int code = argmin_fp4(q);
        words[j / 8] |= (uint32_t)code << (4 * (j % 8));
      }
      wq[r * kw + g * 2] = words[0];
      wq[r * kw + g * 2 + 1] = words[1];
    }
  }
}

ORC_API void orc_quantize_bf16(const uint16_t *w, int64_t rows, int64_t K, uint32_t *wq,
                               uint8_t *sq) {
  float *tmp = (float *)malloc(sizeof(float) * (size_t)K);
  for (int64_t r = 0; r < rows; r++) {
    for (int64_t k = 0; k < K; k++) tmp[k] = orc_bf16_to_f32(w[r * K + k]);
    quantize_rows(tmp, 1, 1, K, wq + r * (K / 8), sq + r * (K / 16));
  }
  free(tmp);
}

ORC_API void orc_quantize_f32(const float *w, int64_t rows, int64_t K, uint32_t *wq,
                              uint8_t *sq) {
  quantize_rows(w, 0, rows, K, wq, sq);
}

/* ------------------------------------------------------------------------ */
/* Quantized matmul with transposed weights (backend/cpu/quantized.cpp:     */
/* 491-533 fp_qmm_t<T, 16, 4>): y[m][n] = sum_g s[n][g] * gsum, gsum =      */
/* sum_{j<16} x[m][16g+j] * LUT[code], both sums sequential in T.           */
/* ------------------------------------------------------------------------ */
ORC_API void orc_qmm_f32(const float *x, const uint32_t *w, const uint8_t *s, int64_t M,
                         int64_t N, int64_t K, float *y) {
  const int64_t kw = K / 8, kg = K / 16;
  for (int64_t m = 0; m < M; m++)
    for (int64_t n = 0; n < N; n++) {
      const float *xr = x + m * K;
      float sum = 0.0f;
      for (int64_t g = 0; g < kg; g++) {
        float scale = orc_e4m3_decode(s[n * kg + g]);
        float gsum = 0.0f;
        for (int j = 0; j < 16; j++) {
          uint32_t word = w[n * kw + g * 2 + j / 8];
          gsum += xr[g * 16 + j] * FP4_VALUES[(word >> (4 * (j % 8))) & 15];
        }
        sum += scale * gsum;
      }
      y[m * N + n] = sum;
    }
}

/* The same loop with T = bfloat16_t: every multiply and add rounds to      */
/* bf16 (types/bf16.h:71-99).  This is what MLX runs on x86 for bf16 x,     */
/* because simd::max_size<bfloat16_t> is 1 there (backend/cpu/simd/         */
/* base_simd.h:21) and the dispatch at quantized.cpp:611-616 falls back to  */
/* fp_qmm_t.                                                                */
ORC_API void orc_qmm_bf16(const uint16_t *x, const uint32_t *w, const uint8_t *s, int64_t M,
                          int64_t N, int64_t K, uint16_t *y) {
  const int64_t kw = K / 8, kg = K / 16;
  for (int64_t m = 0; m < M; m++)
    for (int64_t n = 0; n < N; n++) {
      const uint16_t *xr = x + m * K;
      float sum = 0.0f;
      for (int64_t g = 0; g < kg; g++) {
        float scale = bfr(orc_e4m3_decode(s[n * kg + g]));
        float gsum = 0.0f;
        for (int j = 0; j < 16; j++) {
          uint32_t word = w[n * kw + g * 2 + j / 8];
          float p = bfr(orc_bf16_to_f32(xr[g * 16 + j]) *
                        FP4_VALUES[(word >> (4 * (j % 8))) & 15]);
          gsum = bfr(gsum + p);
        }
        sum = bfr(sum + bfr(scale * gsum));
      }
      y[m * N + n] = orc_bf16_from_f32(sum);
    }
}

/* ------------------------------------------------------------------------ */
/* Activation fake-quantisation for QQMatmul (backend/cpu/quantized.cpp:    */
/* 1064-1091 to_fp4_e2m1, 1093-1129 fp_quantize_dequantize, bits 4, group   */
/* 16), in f32 on the values of x:                                           */
/*   amax = std::max over |x| starting from -inf (a NaN operand never wins) */
/*   s    = FromFP8(ToFP8(amax / 6))                                        */
/*   code = to_fp4_e2m1(s == 0 ? 0 : x / s); xhat = s * LUT[code]           */
/* to_fp4_e2m1 rounds |v| to the nearest E2M1 magnitude, ties to the even   */
/* code (0.25 -> 0, 0.75 -> 1, 1.25 -> 1, 1.75 -> 2, 2.5 -> 2, 3.5 -> 4,     */
/* 5 -> 4), saturates at 6, maps NaN to code 7, and takes the sign bit.      */
/* ------------------------------------------------------------------------ */
ORC_API uint8_t orc_to_fp4_e2m1(float v) {
  if (isnan(v)) return 0x7;
  uint8_t sign = signbit(v) ? 0x8 : 0x0;
  float a = fabsf(v);
  uint8_t m;
  if (a > 5.0f) m = 7;
  else if (a >= 3.5f) m = 6;
  else if (a > 2.5f) m = 5;
  else if (a >= 1.75f) m = 4;
  else if (a > 1.25f) m = 3;
  else if (a >= 0.75f) m = 2;
  else if (a > 0.25f) m = 1;
  else m = 0;
  return (uint8_t)(m | sign);
}

/* Codes and raw scale bytes of one row group (the scale byte as MLX forms  */
/* it, sign included), and xhat.                                            */
static void qx_group(const float *v, uint8_t *codes, uint8_t *sbyte, float *xhat) {
  float amax = -INFINITY;
  for (int j = 0; j < 16; j++) {
    float a = fabsf(v[j]);
    amax = (amax < a) ? a : amax; /* std::max(amax, a) */
  }
  uint8_t sb = orc_e4m3_encode(amax / 6.0f);
  float s = orc_e4m3_decode(sb);
  for (int j = 0; j < 16; j++) {
    uint8_t c = orc_to_fp4_e2m1(s == 0.0f ? 0.0f : v[j] / s);
    codes[j] = c;
    if (xhat) xhat[j] = s * FP4_VALUES[c];
  }
  *sbyte = sb;
}

/* xhat[M, K] = fp_quantize_dequantize(x) in f32. */
ORC_API void orc_quantize_dequantize_x(const float *x, int64_t M, int64_t K, float *xhat) {
  uint8_t codes[16], sb;
  for (int64_t i = 0; i < M * (K / 16); i++) qx_group(x + i * 16, codes, &sb, xhat + i * 16);
}

/* The same groups packed like the weights: xq[M, K/8] (low nibble first),  */
/* scale bytes [M, K/16].  The one scale MLX forms with the sign set        */
/* (amax = -inf: an all-NaN group) is stored as its magnitude with every    */
/* code's sign flipped, which dequantises to the same xhat.                 */
ORC_API void orc_quantize_x(const float *x, int64_t M, int64_t K, uint32_t *xq, uint8_t *s) {
  uint8_t codes[16], sb;
  for (int64_t i = 0; i < M * (K / 16); i++) {
    qx_group(x + i * 16, codes, &sb, NULL);
    uint8_t flip = (sb & 0x80) ? 0x8 : 0x0;
    uint32_t w0 = 0, w1 = 0;
    for (int j = 0; j < 8; j++) w0 |= (uint32_t)((codes[j] ^ flip) & 15) << (4 * j);
    for (int j = 0; j < 8; j++) w1 |= (uint32_t)((codes[8 + j] ^ flip) & 15) << (4 * j);
    xq[i * 2] = w0;
    xq[i * 2 + 1] = w1;
    s[i] = (uint8_t)(sb & 0x7F);
  }
}

/* QQMatmul (quantized.cpp:1322-1360): xhat = fake-quant(x), then the qmm   */
/* of quantized.cpp:491-533 on xhat.  This is the fp32-accumulated form     */
/* (T = float); x holds the activation values widened to f32.               */
ORC_API void orc_qqmm_f32(const float *x, const uint32_t *w, const uint8_t *s, int64_t M,
                          int64_t N, int64_t K, float *y) {
  float *xhat = (float *)malloc(sizeof(float) * (size_t)(M * K));
  if (!xhat) return;
  orc_quantize_dequantize_x(x, M, K, xhat);
  orc_qmm_f32(xhat, w, s, M, N, K, y);
  free(xhat);
}

/* ------------------------------------------------------------------------ */
/* Gather QMM (backend/cpu/quantized.cpp:805-844 fp_bs_qmm_dispatch_mode):  */
/* for pair i, out[i] (M x N) = x[lhs[i]] (M x K) @ W[rhs[i]]^T.  lhs may   */
/* be NULL, meaning lhs[i] = i (ops.cpp:67-81 indices_or_default after the  */
/* broadcast of ops.cpp:5377-5379).                                         */
/* ------------------------------------------------------------------------ */
ORC_API void orc_gather_qmm_f32(const float *x, const uint32_t *w, const uint8_t *s,
                                const uint32_t *lhs, const uint32_t *rhs, int64_t pairs,
                                int64_t M, int64_t N, int64_t K, float *out) {
  for (int64_t i = 0; i < pairs; i++) {
    int64_t xi = lhs ? lhs[i] : i, wi = rhs[i];
    orc_qmm_f32(x + xi * M * K, w + wi * N * (K / 8), s + wi * N * (K / 16), M, N, K,
                out + i * M * N);
  }
}

ORC_API void orc_gather_qmm_bf16(const uint16_t *x, const uint32_t *w, const uint8_t *s,
                                 const uint32_t *lhs, const uint32_t *rhs, int64_t pairs,
                                 int64_t M, int64_t N, int64_t K, uint16_t *out) {
  for (int64_t i = 0; i < pairs; i++) {
    int64_t xi = lhs ? lhs[i] : i, wi = rhs[i];
    orc_qmm_bf16(x + xi * M * K, w + wi * N * (K / 8), s + wi * N * (K / 16), M, N, K,
                 out + i * M * N);
  }
}

/* ------------------------------------------------------------------------ */
/* Sigmoid (backend/cpu/unary_ops.h:77-84): y = 1/(1+exp(|x|)); x<0 ? y :   */
/* 1-y.                                                                     */
/* ------------------------------------------------------------------------ */
ORC_API float orc_sigmoid(float x) {
  float y = 1.0f / (1.0f + expf(fabsf(x)));
  return x < 0.0f ? y : 1.0f - y;
}
static inline float silu(float g) { return g * orc_sigmoid(g); }

/* ------------------------------------------------------------------------ */
/* RMSNorm (mlx/fast.cpp:90-108, the fallback graph the CPU evaluates):      */
/*   x32 = f32(x); x32 *= rsqrt(mean(x32^2) + eps); x = bf16(x32);          */
/*   y = bf16(x * w)   (x, w bf16 bits [T, H] / [H], w NULL = 1).           */
/* MLX sums the squares in f32 in its reduction's order; this restatement   */
/* sums in double and rounds the mean to f32 once (the two agree to an ulp  */
/* of the mean).  rsqrt is 1 / sqrt in f32.                                  */
/* ------------------------------------------------------------------------ */
ORC_API void orc_rms_norm_bf16(const uint16_t *x, const uint16_t *w, int64_t T, int64_t H,
                               float eps, uint16_t *y) {
  for (int64_t t = 0; t < T; t++) {
    double ss = 0.0;
    for (int64_t h = 0; h < H; h++) {
      const double v = orc_bf16_to_f32(x[t * H + h]);
      ss += v * v;
    }
    const float mean = (float)(ss / (double)H);
    const float r = 1.0f / sqrtf(mean + eps);
    for (int64_t h = 0; h < H; h++) {
      const float v = bfr(orc_bf16_to_f32(x[t * H + h]) * r);
      const float g = w ? orc_bf16_to_f32(w[h]) : 1.0f;
      y[t * H + h] = orc_bf16_from_f32(v * g);
    }
  }
}

/* ------------------------------------------------------------------------ */
/* Router (VLM/MLXLLM/Models/Laguna.swift:165-180 LagunaMoEGate):           */
/*   logits = x @ G^T  (bf16 matmul: f32 accumulation, result rounded to    */
/*            bf16 when round_logits is set, as MLX does for bf16 inputs),  */
/*   s = sigmoid(f32 logits), choice = s + bias,                            */
/*   top-k of choice (argPartition; this restatement breaks ties toward the */
/*   lower expert id), w = s[top] / sum(s[top]) when norm is set.           */
/* Output slots are ordered by descending choice.                           */
/* ------------------------------------------------------------------------ */
ORC_API void orc_router_topk(const uint16_t *x, const uint16_t *G, const float *bias,
                             int64_t T, int64_t H, int64_t E, int k, int norm, int round_logits,
                             uint32_t *inds, float *wts, float *logits_out) {
  float *sc = (float *)malloc(sizeof(float) * (size_t)E);
  float *ch = (float *)malloc(sizeof(float) * (size_t)E);
  char *taken = (char *)malloc((size_t)E);
  for (int64_t t = 0; t < T; t++) {
    for (int64_t e = 0; e < E; e++) {
      float acc = 0.0f;
      for (int64_t h = 0; h < H; h++)
        acc += orc_bf16_to_f32(x[t * H + h]) * orc_bf16_to_f32(G[e * H + h]);
      if (round_logits) acc = bfr(acc);
      if (logits_out) logits_out[t * E + e] = acc;
      sc[e] = orc_sigmoid(acc);
      ch[e] = sc[e] + (bias ? bias[e] : 0.0f);
      taken[e] = 0;
    }
    float sum = 0.0f;
    for (int j = 0; j < k; j++) {
      int64_t best = -1;
      for (int64_t e = 0; e < E; e++)
        if (!taken[e] && (best < 0 || ch[e] > ch[best])) best = e;
      taken[best] = 1;
      inds[t * k + j] = (uint32_t)best;
      wts[t * k + j] = sc[best];
      sum += sc[best];
    }
    if (norm)
      for (int j = 0; j < k; j++) wts[t * k + j] /= sum;
  }
  free(sc);
  free(ch);
  free(taken);
}

/* ------------------------------------------------------------------------ */
/* Sparse MoE block, f32 throughout (VLM/MLXLLM/Models/Laguna.swift:204-212 */
/* with SwitchGLU VLM/MLXLMCommon/SwitchLayers.swift:532-580 and the shared */
/* LagunaMLP Laguna.swift:138-144):                                          */
/*   y[t] = scaling * sum_j w[t][j] * down_e(silu(gate_e x) * up_e x)       */
/*          + shared_down(silu(shared_gate x) * shared_up x)  (+ residual)  */
/* x is f32 [T,H].  Routed banks: gate/up [E, I, H/8] u32 + [E, I, H/16]    */
/* u8; down [E, H, I/8] + [E, H, I/16].  Shared banks likewise with one     */
/* expert of width Is (NULL to skip).  Output f32 [T, H].                    */
/* ------------------------------------------------------------------------ */
static void expert_mlp(const float *x, int64_t H, int64_t I, const uint32_t *gw,
                       const uint8_t *gs, const uint32_t *uw, const uint8_t *us,
                       const uint32_t *dw, const uint8_t *ds, float *tmp_g, float *tmp_u,
                       float *out) {
  orc_qmm_f32(x, gw, gs, 1, I, H, tmp_g);
  orc_qmm_f32(x, uw, us, 1, I, H, tmp_u);
  for (int64_t i = 0; i < I; i++) tmp_g[i] = silu(tmp_g[i]) * tmp_u[i];
  orc_qmm_f32(tmp_g, dw, ds, 1, H, I, out);
}

ORC_API void orc_moe_block_f32(const float *x, const uint32_t *inds, const float *wts,
                               int64_t T, int64_t H, int64_t I, int k, float scaling,
                               const uint32_t *gw, const uint8_t *gs, const uint32_t *uw,
                               const uint8_t *us, const uint32_t *dw, const uint8_t *ds,
                               int64_t Is, const uint32_t *sgw, const uint8_t *sgs,
                               const uint32_t *suw, const uint8_t *sus, const uint32_t *sdw,
                               const uint8_t *sds, const float *residual, float *y) {
  int64_t Imax = I > Is ? I : Is;
  float *tg = (float *)malloc(sizeof(float) * (size_t)Imax);
  float *tu = (float *)malloc(sizeof(float) * (size_t)Imax);
  float *o = (float *)malloc(sizeof(float) * (size_t)H);
  const int64_t gstr_w = I * (H / 8), gstr_s = I * (H / 16);
  const int64_t dstr_w = H * (I / 8), dstr_s = H * (I / 16);
  for (int64_t t = 0; t < T; t++) {
    float *yt = y + t * H;
    for (int64_t h = 0; h < H; h++) yt[h] = 0.0f;
    for (int j = 0; j < k; j++) {
      int64_t e = inds[t * k + j];
      expert_mlp(x + t * H, H, I, gw + e * gstr_w, gs + e * gstr_s, uw + e * gstr_w,
                 us + e * gstr_s, dw + e * dstr_w, ds + e * dstr_s, tg, tu, o);
      float wj = wts[t * k + j];
      for (int64_t h = 0; h < H; h++) yt[h] += wj * o[h];
    }
    for (int64_t h = 0; h < H; h++) yt[h] *= scaling;
    if (sgw) {
      expert_mlp(x + t * H, H, Is, sgw, sgs, suw, sus, sdw, sds, tg, tu, o);
      for (int64_t h = 0; h < H; h++) yt[h] += o[h];
    }
    if (residual)
      for (int64_t h = 0; h < H; h++) yt[h] += residual[t * H + h];
  }
  free(tg);
  free(tu);
  free(o);
}
