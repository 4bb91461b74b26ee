// ep.cu -- expert-parallel dispatch / combine for the sparse MoE block.
//
// With the 256 experts split over N ranks (rank r owns experts
// [r*E/N, (r+1)*E/N)), every rank routes its own tokens, sends each
// (token, slot) pair's activation row to the rank owning the pair's expert,
// the owner runs its local experts over the rows it received (one expert per
// row), sends the expert outputs back, and the source rank combines them as the
// Laguna block does (VLM/MLXLLM/Models/Laguna.swift:204-212):
//   y_t = scaling * sum_j w[t][j] * e_j(x_t) + shared(x_t) (+ residual_t).
// The exchange itself is an NCCL all-to-all issued by the host; these kernels
// build the send buffer in destination order and read the returned rows back.
//
// moe_ep_plan_kernel: one CTA.  A stable counting sort of the T*k pairs by
// destination rank: thread i takes a contiguous run of pairs, counts per rank,
// an exclusive scan over threads (per rank, in thread order) gives each
// thread's first slot per rank, then the thread places its pairs in order.
// Deterministic: pair p's slot depends only on the routing.
// moe_ep_pack_kernel: send_x[pos[p]] = x[p / k] (16-byte copies); the plan
// also writes ids[pos[p]] = the pair's local expert id on its owner.
// moe_ep_combine_kernel: f32 accumulation in slot order j = 0..k-1, then the
// shared output and the residual, rounded once to the activation dtype.
#include "common.cuh"
#include "kernels.h"

namespace nvfp4 {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kMaxRanks = 64;

__device__ int g_ep_error = 0;

__global__ void __launch_bounds__(kPlanThreads) moe_ep_plan_kernel(EpPlanArgs a) {
  __shared__ int cnt[kMaxRanks][kPlanThreads / 32];  // per rank, per warp
  __shared__ int base[kMaxRanks];
  const int64_t P = a.T * a.k;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t per = (P + kPlanThreads - 1) / kPlanThreads;
  const int64_t p0 = (int64_t)tid * per < P ? (int64_t)tid * per : P;
  const int64_t p1 = p0 + per < P ? p0 + per : P;
  // Per rank: this thread's pair count, scanned over the warp (thread order);
  // lane 31 holds the warp total.
  for (int r = 0; r < a.world; r++) {
    int c = 0;
    for (int64_t p = p0; p < p1; p++)
      if ((int)(a.inds[p] / (uint32_t)a.experts_per_rank) == r) c++;
    int s = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += v;
    }
    if (lane == 31) cnt[r][warp] = s;
  }
  __syncthreads();
  if (tid < a.world) {
    // exclusive scan over warps for rank tid, then totals
    int acc = 0;
    for (int w = 0; w < kPlanThreads / 32; w++) {
      const int v = cnt[tid][w];
      cnt[tid][w] = acc;
      acc += v;
    }
    a.counts[tid] = acc;
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int r = 0; r < a.world; r++) {
      base[r] = acc;
      acc += a.counts[r];
    }
  }
  __syncthreads();
  // Place: for each rank, the thread's first slot = base + warp offset +
  // exclusive lane offset (recomputed with the same scan), then its pairs in
  // order.
  for (int r = 0; r < a.world; r++) {
    int c = 0;
    for (int64_t p = p0; p < p1; p++) {
      const uint32_t e = a.inds[p];
      if ((int)(e / (uint32_t)a.experts_per_rank) == r) c++;
    }
    int s = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += v;
    }
    int slot = base[r] + cnt[r][warp] + (s - c);
    for (int64_t p = p0; p < p1; p++) {
      const uint32_t e = a.inds[p];
      if ((int)(e / (uint32_t)a.experts_per_rank) == r) {
        a.pos[p] = slot;
        a.ids[slot] = (int32_t)(e - (uint32_t)r * (uint32_t)a.experts_per_rank);
        slot++;
      }
    }
  }
  // Out-of-range experts: sent to no rank (slot -1) and flagged.
  for (int64_t p = p0; p < p1; p++)
    if (a.inds[p] / (uint32_t)a.experts_per_rank >= (uint32_t)a.world) {
      a.pos[p] = -1;
      atomicCAS(&g_ep_error, 0, 6);
    }
}

__global__ void moe_ep_pack_kernel(EpPackArgs a) {
  const int64_t P = a.T * a.k;
  const int64_t chunks = a.H * a.esz / 16;  // 16-byte pieces per row
  const int64_t total = P * chunks;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = i / chunks, c = i - p * chunks;
    const int slot = a.pos[p];
    if (slot < 0) continue;
    const uint4* src = reinterpret_cast<const uint4*>(
        reinterpret_cast<const uint8_t*>(a.x) + (p / a.k) * a.H * a.esz);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(a.send_x) +
                                          (int64_t)slot * a.H * a.esz);
    dst[c] = src[c];
  }
}

__global__ void moe_ep_combine_kernel(EpCombineArgs a) {
  const int64_t total = a.T * a.H;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / a.H, h = i - t * a.H;
    float acc = 0.f;
    for (int j = 0; j < a.k; j++) {
      const int slot = a.pos[t * a.k + j];
      if (slot >= 0) acc += a.wts[t * a.k + j] * load_as_f32(a.yp, a.dtype, (int64_t)slot * a.H + h);
    }
    acc *= a.scaling;
    if (a.shared) acc += load_as_f32(a.shared, a.dtype, i);
    if (a.residual) acc += load_as_f32(a.residual, a.dtype, i);
    store_from_f32(a.y, a.dtype, i, acc);
  }
}

__global__ void moe_ep_finish_kernel(void* y, const void* partial, int partial_dtype,
                                     const void* shared, const void* residual, int dtype,
                                     int64_t total) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    float acc = load_as_f32(partial, partial_dtype, i);
    if (shared) acc += load_as_f32(shared, dtype, i);
    if (residual) acc += load_as_f32(residual, dtype, i);
    store_from_f32(y, dtype, i, acc);
  }
}

}  // namespace

cudaError_t launch_ep_finish(void* y, const void* partial, int partial_dtype, const void* shared,
                             const void* residual, int dtype, int64_t T, int64_t H,
                             cudaStream_t stream) {
  const int64_t total = T * H;
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const int blocks = (int)std::min<int64_t>((total + threads - 1) / threads, 148 * 8);
  moe_ep_finish_kernel<<<blocks, threads, 0, stream>>>(y, partial, partial_dtype, shared, residual,
                                                       dtype, total);
  return cudaGetLastError();
}

cudaError_t launch_ep_plan(const EpPlanArgs& a, cudaStream_t stream) {
  if (a.world > kMaxRanks) return cudaErrorInvalidValue;
  moe_ep_plan_kernel<<<1, kPlanThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_ep_pack(const EpPackArgs& a, cudaStream_t stream) {
  const int64_t total = a.T * a.k * (a.H * a.esz / 16);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const int blocks = (int)std::min<int64_t>((total + threads - 1) / threads, 148 * 8);
  moe_ep_pack_kernel<<<blocks, threads, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_ep_combine(const EpCombineArgs& a, cudaStream_t stream) {
  const int64_t total = a.T * a.H;
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const int blocks = (int)std::min<int64_t>((total + threads - 1) / threads, 148 * 8);
  moe_ep_combine_kernel<<<blocks, threads, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t read_and_clear_ep_error(int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_ep_error, sizeof(int));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_ep_error, &zero, sizeof(int));
}

}  // namespace nvfp4
