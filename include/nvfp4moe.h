/*
 * nvfp4moe.h -- C ABI of the B200 (sm_100a) NVFP4 MoE library
 * (libnvfp4moe.so).
 *
 * This is the drop-in boundary for the hot path of Layr-Labs/mlxfast-challenge:
 * the NVFP4 (E2M1 codes, E4M3 group-16 scales) quantized matmuls that carry
 * Laguna XS 2.1's sparse MoE blocks, plus the BF16 router that feeds them.
 * Each entry point replaces one operator of the reference's mlx-c surface
 * (Vendor/mlx-swift/Source/Cmlx/mlx-c/mlx/c/ops.h) for mode "nvfp4",
 * group_size 16, bits 4, transpose true, or one layer of its Laguna model.
 *
 * Conventions
 *   - Every tensor argument is a DEVICE pointer to row-major, contiguous
 *     memory.  Packed weights are the reference's own layout: uint32 words of
 *     8 E2M1 codes (low nibble first) [..., N, K/8] and uint8 E4M3 scales
 *     [..., N, K/16].  Activations are bf16 (NVFP4_BF16), f16 or f32; outputs
 *     take the activation dtype (ops.cpp:4568-4572).
 *   - Work is enqueued on `stream` (a cudaStream_t; NULL = legacy default
 *     stream) and is asynchronous, as MLX evaluation is stream-ordered.
 *   - Return 0 on success.  On failure nothing is enqueued, a non-zero status
 *     is returned and nvfp4_last_error() (per calling thread) holds a message
 *     in the reference's "[op] ..." style (mlx-c returns 1 and routes the
 *     message to its error handler, mlx-c/mlx/c/error.h:15-33; the handler
 *     hook is mirrored by nvfp4_set_error_handler).
 *   - Shape checks follow the reference's validation (ops.cpp:67-175,
 *     :4549-4600, :5338-5433).  Indices live on the device, so they are
 *     range-checked on the device: an out-of-range expert or x index skips its
 *     work and latches NVFP4_ERR_DEVICE_INDEX, read by nvfp4_device_status().
 *   - No entry point allocates device memory; the MoE block takes a caller
 *     workspace sized by moe_block_workspace_size().
 *   - There is no CPU fallback: without a CUDA device every call fails.
 */
#ifndef NVFP4MOE_H
#define NVFP4MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NVFP4MOE_API __attribute__((visibility("default")))

/* Status codes. */
enum {
  NVFP4_OK = 0,
  NVFP4_ERR_INVALID = 1,      /* bad shape / dtype / argument (as mlx-c's 1) */
  NVFP4_ERR_UNSUPPORTED = 2,  /* valid for the reference, not provided here */
  NVFP4_ERR_CUDA = 3,         /* CUDA runtime error */
  NVFP4_ERR_WORKSPACE = 4,    /* workspace missing or too small */
  NVFP4_ERR_DEVICE_INDEX = 5,  /* latched by kernels: index out of range */
  NVFP4_ERR_DEVICE_TIMEOUT = 6 /* latched by kernels: a bounded wait expired */
};

/* Activation / output dtypes. */
enum { NVFP4_BF16 = 0, NVFP4_F16 = 1, NVFP4_F32 = 2 };

typedef void* nvfp4_stream; /* cudaStream_t */

NVFP4MOE_API const char* nvfp4_last_error(void);
/* mlx_set_error_handler (mlx-c/mlx/c/error.h:15-33): called with the message
 * and `data` on every failure; NULL restores the default (no callback). */
typedef void (*nvfp4_error_handler)(const char* msg, void* data);
NVFP4MOE_API void nvfp4_set_error_handler(nvfp4_error_handler handler, void* data);
NVFP4MOE_API int nvfp4_version(void);

/* Launch flags of the calling thread (no counterpart in the reference, whose
 * lazy graph schedules launches itself).  NVFP4_LAUNCH_PDL lets the FIRST
 * kernel of each following call start before the preceding kernel on the
 * stream has finished (programmatic dependent launch): it streams its weights
 * immediately and reads the call's activation input only after the
 * dependency wait.  Set it only when the preceding kernel is one of this
 * library's (e.g. a decode chain captured into a CUDA graph) and it produced
 * nothing else this call reads -- in particular not the routing passed in.
 * Later kernels inside one call always overlap their predecessor.  Returns
 * the previous flags. */
#define NVFP4_LAUNCH_PDL 1
/* NVFP4_LAUNCH_BULK_COPY selects, for the GEMV engine (moe_gate_up_swiglu /
 * moe_down_combine at T <= 8, moe_block_forward at T = 1), the decode kernels
 * fed by cp.async.bulk copies into a shared-memory ring (one producer warp,
 * eight consumer warps) instead of per-thread streaming loads.  Same results. */
#define NVFP4_LAUNCH_BULK_COPY 2
/* The grouped GEMMs of moe_block_forward (T >= 2: expert sort, each distinct
 * expert streamed once) run by default on the
 * block-scaled FP4 tensor cores (tcgen05 kind::mxf4nvf4): activations as a sum
 * of four NVFP4 terms (relative-L2 ~1e-4 from the W4A16 product, 10x below
 * bf16 output rounding), weights as stored.  NVFP4_LAUNCH_EXACT_PREFILL
 * selects the exact path instead (weights dequantised to 16-bit, kind::f16;
 * ~2.1x slower at T = 512).  The FP4 GEMMs hold the batch's tile list
 * (E + T * top_k / 32 + T / 32 entries) in shared memory; a batch whose list
 * does not fit (above ~13.8k tokens at E = 256, top-8, with a shared expert)
 * runs on the exact path.  moe_ep_partial_forward has no exact path and
 * returns NVFP4_ERR_UNSUPPORTED there: call it over row ranges of the
 * gathered batch (tokens are independent), as ep.py's gather form does. */
#define NVFP4_LAUNCH_EXACT_PREFILL 4
/* moe_decode_stack_forward runs by default on the block-scaled FP4 tensor
 * cores where the shape allows (hidden 1024 or 2048, inter 512 / 1024 / 2048,
 * one gate/up and one down item per SM): activations as four NVFP4 terms as
 * above.  NVFP4_LAUNCH_EXACT_DECODE selects the mma.sync stack instead (16-bit
 * activations, exact products). */
#define NVFP4_LAUNCH_EXACT_DECODE 8
/* Test only (no counterpart in the reference): the block-scaled FP4 decode
 * stacks (moe_decode_stack_forward, moe_decode_stack_routed_forward) give
 * every bounded wait ~1 ms instead of ~1 s and withhold one release (the
 * last layer's segment-0 gate/up items never signal), so the waits behind it
 * run out: the launch returns, nvfp4_device_status() reports
 * NVFP4_ERR_DEVICE_TIMEOUT with the site 1000 * (last layer + 1) + 40..59
 * (whichever wait behind the withheld release gave up first: a counter wait
 * 50..54 or a tensor-core wait 41..49), and the outputs are not valid.  The context stays usable.  It exercises
 * the error path of the bounded waits without faulting or hanging a GPU. */
#define NVFP4_LAUNCH_TEST_EXPIRE 16
NVFP4MOE_API int nvfp4_set_launch_flags(int flags);
/* Synchronises the device, returns and clears the latched device status:
 * NVFP4_OK, NVFP4_ERR_DEVICE_INDEX, or NVFP4_ERR_DEVICE_TIMEOUT when a kernel's
 * bounded wait (on a copy, a tensor-core commit or another CTA's counter)
 * gave up -- the kernel then returned early and its outputs are not valid;
 * the message names the kernel site.  The context stays usable. */
NVFP4MOE_API int nvfp4_device_status(void);

/* mlx_dequantize (mlx-c ops.h:359; ops.cpp:5120-5241 fp_dequantize), mode
 * "nvfp4": out[rows, K] = LUT[code] * e4m3(scale).  Bit-exact. */
NVFP4MOE_API int nvfp4_dequantize(void* out, int out_dtype, const uint32_t* w,
                                  const uint8_t* scales, int64_t rows, int64_t K,
                                  nvfp4_stream stream);

/* mlx_quantize (mlx-c ops.h:801-808; ops.cpp:4873-4978 fp_quantize), mode
 * "nvfp4", group 16, no global scale: w[rows, K] (bf16/f16/f32) ->
 * wq[rows, K/8] uint32 + scales[rows, K/16] uint8, bit-identical to the
 * reference's CPU evaluation. */
NVFP4MOE_API int nvfp4_quantize(uint32_t* wq, uint8_t* scales, const void* w, int w_dtype,
                                int64_t rows, int64_t K, nvfp4_stream stream);

/* The activation half of MLX's fp_quantize_dequantize
 * (backend/cpu/quantized.cpp:1093-1129, bits 4, group 16), which QQMatmul
 * applies to x before its matmul: per row group of 16, scale =
 * ToFP8(max|x| / 6), code = to_fp4_e2m1(x / FromFP8(scale)) (:1064-1091).
 * x[M, K] (bf16/f16/f32, 16-byte aligned) -> xq[M, K/8] uint32 (low nibble
 * first) + scales[M, K/16]; dequantising them gives MLX's xhat bit for bit.
 * (A group whose max is NaN gets scale byte ToFP8(-inf) = 0xFE in MLX; it is
 * written as 0x7E with every code's sign flipped, the same xhat.) */
NVFP4MOE_API int nvfp4_quantize_activations(uint32_t* xq, uint8_t* scales, const void* x,
                                            int dtype, int64_t M, int64_t K,
                                            nvfp4_stream stream);

/* mlx_qqmm (mlx-c ops.h:790-800; ops.cpp:4691-4757), mode "nvfp4", w
 * quantized, no global scales; QQMatmul::eval_cpu (quantized.cpp:1322-1360):
 * y[M, N] = xhat[M, K] @ dequant(w)[N, K]^T with xhat the fake-quantised x
 * above; y has x's dtype.  Runs on the block-scaled tensor cores
 * (tcgen05.mma kind::mxf4nvf4, UE4M3 scales per 16): products are exact, the
 * sum is f32.  The reference's CPU path accepts only M == 1 ("NYI for the
 * general case"); any M is accepted here, as MLX's CUDA qqmm does.
 * K % 256 == 0; x, w and scales 16-byte aligned.  Workspace:
 * nvfp4_qqmm_workspace_size(M, N, K) bytes, 256-byte aligned. */
NVFP4MOE_API size_t nvfp4_qqmm_workspace_size(int64_t M, int64_t N, int64_t K);
NVFP4MOE_API int nvfp4_qqmm(void* y, const void* x, int dtype, const uint32_t* w,
                            const uint8_t* scales, int64_t M, int64_t N, int64_t K,
                            void* workspace, size_t workspace_bytes, nvfp4_stream stream);

/* mlx_quantized_matmul (mlx-c ops.h:809-818; ops.cpp:4549-4600;
 * QuantizedMatmul::eval_cpu backend/cpu/quantized.cpp:924-964), transpose:
 * y[M, N] = x[M, K] @ dequant(w)[N, K]^T. */
NVFP4MOE_API int nvfp4_quantized_matmul(void* y, const void* x, int dtype, const uint32_t* w,
                                        const uint8_t* scales, int64_t M, int64_t N, int64_t K,
                                        nvfp4_stream stream);

/* mlx_gather_qmm (mlx-c ops.h:475-488; ops.cpp:5338-5433; GatherQMM::eval_cpu
 * backend/cpu/quantized.cpp:966-1047), transpose, lhs/rhs already broadcast
 * to `pairs` entries:
 *   out[p] (M x N) = x[lhs[p]] (M x K) @ dequant(w[rhs[p]])^T
 * x is [n_x_batches, M, K]; w is [n_experts, N, K/8]; out is [pairs, M, N].
 * lhs_indices NULL means lhs[p] = p (indices_or_default, ops.cpp:67-81);
 * rhs_indices NULL means expert 0 for every pair.  sorted_indices is the
 * reference's performance hint; results never depend on it. */
NVFP4MOE_API int nvfp4_gather_qmm(void* out, const void* x, int dtype, const uint32_t* w,
                                  const uint8_t* scales, const uint32_t* lhs_indices,
                                  const uint32_t* rhs_indices, int64_t pairs,
                                  int64_t n_x_batches, int64_t n_experts, int64_t M, int64_t N,
                                  int64_t K, int sorted_indices, nvfp4_stream stream);

/* mlx_fast_rms_norm (mlx-c fast.h:163; mlx/fast.cpp:53-108), as the CPU
 * evaluates it: y[r] = dtype(dtype(x[r] * rsqrt(mean(x[r]^2) + eps)) * weight),
 * the mean of f32 squares.  x, y [rows, dims] and weight [dims] (NULL:
 * weight 1) in dtype; y may alias x.  The norm in front of every Laguna MoE
 * block (post_attention_layernorm, Laguna.swift:242-246). */
NVFP4MOE_API int nvfp4_rms_norm(void* y, const void* x, const void* weight, int dtype,
                                int64_t rows, int64_t dims, float eps, nvfp4_stream stream);

/* LagunaMoEGate (VLM/MLXLLM/Models/Laguna.swift:149-181): logits = x @ G^T
 * (bf16 G [E, H]), sigmoid, + e_score_correction_bias for the choice, top-k
 * (ties to the lower id), weights = sigmoid scores of the chosen experts,
 * renormalised when norm_topk_prob.  inds [T, k] uint32, weights [T, k] f32.
 * Needs moe_router_workspace_size() bytes of workspace, zeroed once before
 * first use (moe_workspace_init); the kernels leave it reusable. */
NVFP4MOE_API size_t moe_router_workspace_size(int64_t T, int64_t H, int64_t E);
NVFP4MOE_API int moe_router_topk(uint32_t* inds, float* weights, const void* x, int dtype,
                                 const uint16_t* gate_w_bf16, const float* bias, int64_t T,
                                 int64_t H, int64_t E, int k, int norm_topk_prob,
                                 void* workspace, size_t workspace_bytes, nvfp4_stream stream);

/* One NVFP4 bank: packed codes and scales of [n_experts, rows, K]. */
typedef struct {
  const uint32_t* w;
  const uint8_t* scales;
} nvfp4_bank;

/* One Laguna sparse MoE layer (LagunaSparseMoeBlock, Laguna.swift:183-213;
 * runtime LagunaRuntimeSparseMoEBlock, Sources/MLXFastModel/
 * LagunaRuntimeModel.swift:10498-11002).  Routed banks: gate/up [E, I, H/8],
 * down [E, H, I/8].  Shared expert banks (LagunaMLP, Laguna.swift:126-145):
 * gate/up [Is, H/8], down [H, Is/8]; set shared_inter = 0 to omit it. */
typedef struct {
  int64_t hidden;        /* H (hidden_size) */
  int64_t inter;         /* I (moe_intermediate_size) */
  int64_t n_experts;     /* E (num_experts) */
  int64_t top_k;         /* k (num_experts_per_tok) */
  int64_t shared_inter;  /* Is (shared_expert_intermediate_size) or 0 */
  float routed_scaling;  /* moe_routed_scaling_factor */
  int norm_topk_prob;
  const uint16_t* router_w; /* bf16 [E, H] (mlp.gate.weight) */
  const float* router_bias; /* f32 [E] (e_score_correction_bias) or NULL */
  nvfp4_bank gate, up, down;
  nvfp4_bank shared_gate, shared_up, shared_down;
} moe_layer_desc;

NVFP4MOE_API size_t moe_block_workspace_size(const moe_layer_desc* layer, int64_t T);
/* Zero a workspace once after allocating it (enqueued on `stream`). */
NVFP4MOE_API int moe_workspace_init(void* workspace, size_t bytes, nvfp4_stream stream);

/* Sparse MoE block forward:
 *   y = routed_scaling * sum_j w_j * down_e(silu(gate_e x) * up_e x)
 *       + shared_down(silu(shared_gate x) * shared_up x) (+ residual)
 * x, y, residual [T, H] in `dtype`.  When inds_in is NULL the router runs
 * first (router_w required); otherwise inds_in [T, k] / weights_in [T, k]
 * are used as given.  inds_out / weights_out (nullable) receive the routing
 * that was used.  T = 1 runs the GEMV engine; T >= 2 (Laguna-shaped layers:
 * hidden and inter multiples of 256) the expert sort and grouped tensor-core
 * GEMMs, which stream each distinct expert once for all its tokens. */
NVFP4MOE_API int moe_block_forward(void* y, const void* x, const void* residual, int dtype,
                                   int64_t T, const moe_layer_desc* layer,
                                   const uint32_t* inds_in, const float* weights_in,
                                   uint32_t* inds_out, float* weights_out, void* workspace,
                                   size_t workspace_bytes, nvfp4_stream stream);

/* moe_block_forward without a workspace, for callers that cannot allocate
 * device memory (no counterpart in the reference, whose MLX runtime owns its
 * allocations): hosts that reach this library only through an operator
 * interface that passes tensor pointers, with no way to hand it a separately
 * owned workspace, or that must keep a fixed device-memory footprint.  The
 * scratch is a static 256 KB device array held by every GPU that loads the
 * library until exit: enough for T <= 8 tokens at Laguna XS 2.1 sizes;
 * larger T is rejected with NVFP4_ERR_WORKSPACE.  The first call on a device
 * looks the array up (make it before any stream capture).  All calls on a
 * device share the array: calls that overlap on the GPU race.  Arguments
 * otherwise as moe_block_forward. */
NVFP4MOE_API int moe_block_forward_noalloc(void* y, const void* x, const void* residual,
                                           int dtype, int64_t T, const moe_layer_desc* layer,
                                           const uint32_t* inds_in, const float* weights_in,
                                           uint32_t* inds_out, float* weights_out,
                                           nvfp4_stream stream);

/* The two fused phases of moe_block_forward, callable on their own.
 *
 * moe_gate_up_swiglu -- the routed (and shared) gate/up projections fused
 * with SwiGLU, as the reference runtime's lagunaRoutedSwiGLUQMV
 * (Sources/MLXFastModel/LagunaRuntimeModel.swift:7424) and SwitchGLU's
 * gate/up + compiledSwiGLU (VLM/MLXLMCommon/SwitchLayers.swift:547-571):
 *   act[t][j][i] = silu(x_t . gate_e[i]) * (x_t . up_e[i]),  e = inds[t][j]
 * for slots j < k, and slot j = k (when shared_inter > 0) for the shared
 * expert.  act is f32 [T, k(+1), act_ld], act_ld >= max(I, Is).
 *
 * moe_down_combine -- the down projections with the routed weighting,
 * scaling, shared expert and residual, as lagunaRoutedSharedDownResidual
 * (LagunaRuntimeModel.swift:8441):
 *   y_t = scaling * sum_j w[t][j] * down_e(act[t][j]) + shared_down(act[t][k])
 *         (+ residual_t) */
NVFP4MOE_API int moe_gate_up_swiglu(float* act, int64_t act_ld, const void* x, int dtype,
                                    int64_t T, const moe_layer_desc* layer,
                                    const uint32_t* inds, nvfp4_stream stream);
NVFP4MOE_API int moe_down_combine(void* y, const float* act, int64_t act_ld,
                                  const void* residual, int dtype, int64_t T,
                                  const moe_layer_desc* layer, const uint32_t* inds,
                                  const float* weights, nvfp4_stream stream);

/* Serial decode through a stack of sparse MoE layers, T = 1, routing given
 * per layer: for l = 0 .. n_layers-1
 *   x_{l+1} = moe_block(x_l; layers[l], inds[l], weights[l])   (no residual)
 * and y = x_{n_layers}.  This is the MoE part of the reference runtime's
 * decode step over the sparse layers (Sources/MLXFastModel/
 * LagunaRuntimeModel.swift:11460 -> :11030 -> :10678), which the reference
 * evaluates layer by layer; it has no single-operator counterpart.  Run as one
 * persistent cooperative launch that streams the next layers' expert weights
 * while the current layer's dependent chain runs; results equal a loop of
 * moe_gate_up_swiglu + moe_down_combine.  Requirements: every layer has the
 * same hidden / inter / n_experts / top_k (<= 16) / shared_inter / routed_scaling, shared_inter 0 or equal to
 * inter, hidden and inter multiples of 256, 16-byte aligned banks,
 * n_layers <= 64; otherwise NVFP4_ERR_UNSUPPORTED (use the per-layer calls).
 * inds[l] / weights[l] are device pointers to [top_k] entries.  The call runs
 * as many CTAs as the GPU has SMs and they wait on one another inside the
 * launch (co-residency is guaranteed by the cooperative launch); do not
 * overlap it with other work that needs whole SMs.  By default (see
 * NVFP4_LAUNCH_EXACT_DECODE) the products run on the block-scaled FP4 tensor
 * cores, up to 40 layers per launch (20 with a shared expert);
 * moe_decode_stack_launches gives the number of launches a call makes under
 * the calling thread's flags, moe_decode_stack_uses_fp4 which stack runs. */
NVFP4MOE_API size_t moe_decode_stack_workspace_size(const moe_layer_desc* layers,
                                                    int64_t n_layers);
NVFP4MOE_API int moe_decode_stack_launches(const moe_layer_desc* layers, int64_t n_layers);
/* 1 when a call runs the block-scaled FP4 stack (shape supported and
 * NVFP4_LAUNCH_EXACT_DECODE clear), 0 for the mma.sync stack. */
NVFP4MOE_API int moe_decode_stack_uses_fp4(const moe_layer_desc* layers, int64_t n_layers);
NVFP4MOE_API int moe_decode_stack_forward(void* y, const void* x, int dtype, int64_t n_layers,
                                          const moe_layer_desc* layers,
                                          const uint32_t* const* inds,
                                          const float* const* weights, void* workspace,
                                          size_t workspace_bytes, nvfp4_stream stream);

/* Serial decode through a stack of sparse MoE layers with the router inside
 * the launch, T = 1: from h_0 = x, for l = 0 .. n_layers-1
 *   x_l = RMSNorm(h_l; norm_w[l], norm_eps) when norm_w, else h_l
 *   (inds_l, w_l) = router_l(x_l)   (LagunaMoEGate, Laguna.swift:149-181)
 *   h_{l+1} = moe_block(x_l; layers[l], inds_l, w_l) (+ h_l when residual)
 * and y = h_{n_layers}.  With both, a layer is the reference's decoder layer
 * without its attention half (Laguna.swift:242-246: h + mlp(
 * postAttentionLayerNorm(h))); RMSNorm as MLX's fallback (mlx/fast.cpp:90-108):
 * x = dtype(dtype(h * rsqrt(mean(h^2) + eps)) * w), norm_w[l] a device
 * pointer to [hidden] weights in dtype.  This is the MoE part of the reference runtime's
 * decode branch over its sparse layers (Sources/MLXFastModel/
 * LagunaRuntimeModel.swift:10685-10800 for one layer: router top-k, routed
 * experts, shared expert, combine), evaluated layer by layer there; it has no
 * single-operator counterpart.  One persistent cooperative launch per up to 40
 * layers (20 with a shared expert) on the block-scaled FP4 tensor cores: a
 * layer's router runs on the device as soon as its input is complete and its
 * routed experts' weights stream from then on (only the shared expert and the
 * router weights stream ahead).  Each layer's output is rounded to dtype once:
 * sum of the experts' contributions, then the residual.  Logits are summed as
 * 64-bit fixed-point integers (2^-28 units) and the norm's squares in a fixed
 * order, so the routing and the outputs are the same bits on every run; a
 * logit partial (32 rows) beyond 8192 in magnitude, or not finite, makes the
 * logit NaN (never chosen).  inds_out / weights_out: NULL, or
 * n_layers device pointers (each NULL or [top_k] entries) that receive the
 * routing used.  Every layer has the same routed_scaling (also required by
 * moe_decode_stack_forward).  Requirements as moe_decode_stack_forward's FP4 stack (hidden
 * 1024 or 2048, inter 512 / 1024 / 2048, shared_inter 0 or inter), plus
 * n_experts <= 256, top_k <= 8, dtype bf16 or f16, router_w 16-byte aligned in every layer, one
 * norm_topk_prob for all layers, NVFP4_LAUNCH_EXACT_DECODE clear; otherwise
 * NVFP4_ERR_UNSUPPORTED (run moe_block_forward per layer).  Workspace:
 * moe_decode_stack_workspace_size() bytes.  Co-residency as for
 * moe_decode_stack_forward.  moe_decode_stack_routed_launches gives the
 * launches of a call (0: unsupported). */
NVFP4MOE_API int moe_decode_stack_routed_launches(const moe_layer_desc* layers, int64_t n_layers);
NVFP4MOE_API int moe_decode_stack_routed_forward(void* y, const void* x, int dtype,
                                                 int64_t n_layers, const moe_layer_desc* layers,
                                                 int residual, const void* const* norm_w,
                                                 float norm_eps, uint32_t* const* inds_out,
                                                 float* const* weights_out, void* workspace,
                                                 size_t workspace_bytes, nvfp4_stream stream);

/* Expert parallelism (no reference counterpart: the reference runs every
 * expert on one device; its single-device analogue is SwitchGLU's gatherSort /
 * scatterUnsort, VLM/MLXLMCommon/SwitchLayers.swift:385-428).  Rank r of
 * `world` owns experts [r * experts_per_rank, (r + 1) * experts_per_rank).
 *
 * moe_ep_dispatch -- for every (token, slot) pair p of inds [T, k]:
 *   pos[p] = its row of send_x, rows grouped by destination rank in rank
 *   order and, within a rank, in pair order; send_x[pos[p]] = x[p / k];
 *   send_ids[pos[p]] = the expert's id on its owner; send_counts[r] = rows for
 *   rank r.  An out-of-range expert gets pos -1 and is reported by
 *   nvfp4_device_status.  The host then exchanges rows with an all-to-all.
 *
 * moe_ep_combine -- after the owners' expert outputs come back in send order:
 *   y_t = scaling * sum_j w[t][j] * y_pairs[pos[t*k + j]]
 *         + shared_t + residual_t   (nullable), f32 accumulation in slot order,
 * the Laguna combine (VLM/MLXLLM/Models/Laguna.swift:204-212).
 * x / y / y_pairs / shared / residual in `dtype`; rows 16-byte aligned for
 * dispatch (H * element size a multiple of 16). */
NVFP4MOE_API int moe_ep_dispatch(void* send_x, int32_t* send_ids, int32_t* pos,
                                 int32_t* send_counts, const void* x, int dtype,
                                 const uint32_t* inds, int64_t T, int k, int64_t H,
                                 int64_t experts_per_rank, int world, nvfp4_stream stream);
NVFP4MOE_API int moe_ep_combine(void* y, const void* y_pairs, const int32_t* pos,
                                const float* weights, const void* shared, const void* residual,
                                int dtype, int64_t T, int k, int64_t H, float scaling,
                                nvfp4_stream stream);

/* Expert parallelism, gather / reduce-scatter form (the alternative to
 * moe_ep_dispatch / moe_ep_combine): every rank holds all ranks' tokens
 * (all-gathered with their routing) and computes, for every token, the
 * contribution of its own experts [expert_base, expert_base + L->n_experts):
 *   y_partial[t] = routed_scaling * sum_{j: inds[t][j] local} w[t][j] * e_j(x_t)
 *                  (+ shared(x_t) for t in [shared_row0, shared_row0 + shared_rows))
 * in f32 (inds are global expert ids; other ids are skipped).  L holds this
 * rank's routed slice and, when L->shared_inter > 0, the shared expert, which
 * this rank applies to its own rows only.  x rows are x_ld elements apart.  A
 * reduce-scatter (sum) of y_partial over the ranks then gives each rank its
 * tokens' block output; moe_ep_finish adds the residual.  T >= 2 (the grouped block-scaled FP4 path).  The
 * reference runs every expert on one device; single-device analogue:
 * moe_block_forward (Laguna.swift:204-212). */
NVFP4MOE_API size_t moe_ep_partial_workspace_size(const moe_layer_desc* layer, int64_t T);
NVFP4MOE_API int moe_ep_partial_forward(float* y_partial, const void* x, int64_t x_ld,
                                        int dtype, int64_t T, const moe_layer_desc* layer,
                                        const uint32_t* inds, const float* weights,
                                        int64_t expert_base, int64_t shared_row0,
                                        int64_t shared_rows, void* workspace,
                                        size_t workspace_bytes, nvfp4_stream stream);
/* The same with the partials written in partial_dtype: NVFP4_F32 (as
 * moe_ep_partial_forward) or NVFP4_BF16, which halves the reduce-scatter's
 * bytes; each rank's partial is then rounded to bf16 once before the sum
 * (the block output is bf16 anyway). */
NVFP4MOE_API int moe_ep_partial_forward_typed(void* y_partial, int partial_dtype, const void* x,
                                              int64_t x_ld, int dtype, int64_t T,
                                              const moe_layer_desc* layer, const uint32_t* inds,
                                              const float* weights, int64_t expert_base,
                                              int64_t shared_row0, int64_t shared_rows,
                                              void* workspace, size_t workspace_bytes,
                                              nvfp4_stream stream);
/* y[T, H] = partial (f32) + shared (or NULL) + residual (or NULL), rounded
 * once to dtype. */
NVFP4MOE_API int moe_ep_finish(void* y, const float* partial, const void* shared,
                               const void* residual, int dtype, int64_t T, int64_t H,
                               nvfp4_stream stream);
/* The same with the partial sums in partial_dtype (f32, bf16 or f16). */
NVFP4MOE_API int moe_ep_finish_typed(void* y, const void* partial, int partial_dtype,
                                     const void* shared, const void* residual, int dtype,
                                     int64_t T, int64_t H, nvfp4_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* NVFP4MOE_H */
