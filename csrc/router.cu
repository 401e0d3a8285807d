// Mixture-of-experts router kernels (one warp per token row, E <= 256 experts,
// top-k <= 16).
//
//   router_fwd   bf16 logits -> fp32 softmax probabilities, top-k selection
//                (largest first, lowest index on ties), optional
//                renormalisation of the selected weights and the per-expert
//                route histogram, in one pass (Qwen3MoeTopKRouter semantics:
//                transformers/models/qwen3_moe/modeling_qwen3_moe.py, which the
//                reference trains unchanged).
//   router_bwd   gradient of the logits from the gradients of the
//                probabilities (the auxiliary loss reads them) and of the
//                selected weights (through the renormalisation and the softmax).
//   aux_stats    statistics of the Switch load-balancing loss over recorded
//                router probabilities p: the loss applies a second softmax
//                s = softmax(p) and takes top-k of s (HF load_balancing_loss_func,
//                also parallel/parallel/engine/model_parallel/sequence_parallel.py:
//                239-280); this kernel produces the per-expert selection counts
//                and the per-expert sums of s (block partials in shared memory,
//                one atomic per expert per block).
//   aux_stats_bwd gradient of p from the gradient of the per-expert sums of s.
#include <cuda_bf16.h>
#include <stdint.h>

#include <algorithm>

#include "host_util.h"
#include "ptx.cuh"
#include "ops.cuh"

namespace pb {
namespace {

constexpr int kMaxTopK = 16;

__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, off);
    const int oi = __shfl_xor_sync(0xffffffffu, i, off);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// Softmax of VPL values per lane (expert e = lane + 32 * i); masked entries -inf.
template <int VPL>
__device__ __forceinline__ void warp_softmax(float (&v)[VPL]) {
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < VPL; ++i) m = fmaxf(m, v[i]);
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    v[i] = __expf(v[i] - m);
    s += v[i];
  }
  s = warp_sum(s);
  const float inv = 1.f / s;
#pragma unroll
  for (int i = 0; i < VPL; ++i) v[i] *= inv;
}

// Top-k of the lane-distributed values: writes the selected values / indices
// (into lane-uniform registers) and returns the chosen-slot bit mask of this lane.
template <int VPL>
__device__ __forceinline__ uint32_t warp_topk(const float (&p)[VPL], int E, int K, int lane, float* sel_v,
                                              int* sel_i) {
  uint32_t chosen = 0;
  for (int j = 0; j < K; ++j) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !(chosen & (1u << i)) && (p[i] > best || (p[i] == best && e < bi))) {
        best = p[i];
        bi = e;
      }
    }
    warp_argmax(best, bi);
    if ((bi & 31) == lane) chosen |= 1u << (bi >> 5);
    sel_v[j] = best;
    sel_i[j] = bi;
  }
  return chosen;
}

template <int VPL>
__global__ void router_fwd_kernel(const __nv_bfloat16* __restrict__ logits, int64_t ld, int T, int E, int K,
                                  bool renorm, float* __restrict__ probs, float* __restrict__ topv,
                                  int64_t* __restrict__ topi, int* __restrict__ counts) {
  pdl_prologue();
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float p[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = lane + 32 * i;
    p[i] = e < E ? __bfloat162float(logits[(int64_t)t * ld + e]) : -INFINITY;
  }
  warp_softmax(p);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = lane + 32 * i;
    if (e < E) probs[(int64_t)t * E + e] = p[i];
  }
  float sv[kMaxTopK];
  int si[kMaxTopK];
  warp_topk(p, E, K, lane, sv, si);
  float total = 0.f;
  for (int j = 0; j < K; ++j) total += sv[j];
  const float scale = renorm ? 1.f / total : 1.f;
  // lane j writes route j
  for (int j = lane; j < K; j += 32) {
    topv[(int64_t)t * K + j] = sv[j] * scale;
    topi[(int64_t)t * K + j] = si[j];
    if (counts) atomicAdd(&counts[si[j]], 1);
  }
}

template <int VPL>
__global__ void router_bwd_kernel(const float* __restrict__ probs, const float* __restrict__ dprobs,
                                  const float* __restrict__ dtopv, const int64_t* __restrict__ topi, int T, int E,
                                  int K, bool renorm, __nv_bfloat16* __restrict__ dlogits, int64_t ld) {
  pdl_prologue();
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float p[VPL], dp[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = lane + 32 * i;
    p[i] = e < E ? probs[(int64_t)t * E + e] : 0.f;
    dp[i] = (e < E && dprobs) ? dprobs[(int64_t)t * E + e] : 0.f;
  }
  // gradient of the raw (pre-renormalisation) selected probabilities
  float s = 0.f, dot = 0.f;
  if (renorm) {
    for (int j = 0; j < K; ++j) s += probs[(int64_t)t * E + topi[(int64_t)t * K + j]];
    for (int j = 0; j < K; ++j)
      dot += dtopv[(int64_t)t * K + j] * (probs[(int64_t)t * E + topi[(int64_t)t * K + j]] / s);
  }
  for (int j = 0; j < K; ++j) {
    const int e = (int)topi[(int64_t)t * K + j];
    const float g = dtopv[(int64_t)t * K + j];
    const float graw = renorm ? (g - dot) / s : g;
    if ((e & 31) == lane) {
#pragma unroll
      for (int i = 0; i < VPL; ++i)
        if (i == (e >> 5)) dp[i] += graw;
    }
  }
  // softmax backward
  float pd = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) pd += p[i] * dp[i];
  pd = warp_sum(pd);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = lane + 32 * i;
    if (e < E) dlogits[(int64_t)t * ld + e] = __float2bfloat16(p[i] * (dp[i] - pd));
  }
}

// Block partials of the load-balancing statistics: a warp per row, a lane
// owns experts lane + 32 i (registers), the block adds its warps' partials in
// warp order and writes row blockIdx.x of parts [grid, 2E] (counts, then
// sums); sum_slices adds the blocks in block order.  No atomics: the
// statistics have the same bits on every run.
template <int VPL>
__global__ void aux_stats_kernel(const float* __restrict__ probs, int R, int E, int K, float* __restrict__ parts) {
  pdl_prologue();
  extern __shared__ float sh[];  // [warps][2E]
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  float acc_s[VPL], acc_c[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) acc_s[i] = acc_c[i] = 0.f;
  for (int t = blockIdx.x * warps + warp; t < R; t += gridDim.x * warps) {
    float s[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int e = lane + 32 * i;
      s[i] = e < E ? probs[(int64_t)t * E + e] : -INFINITY;
    }
    warp_softmax(s);
    float sv[kMaxTopK];
    int si[kMaxTopK];
    const uint32_t chosen = warp_topk(s, E, K, lane, sv, si);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      if (lane + 32 * i < E) acc_s[i] += s[i];
      if (chosen & (1u << i)) acc_c[i] += 1.f;
    }
  }
  float* mine = sh + (size_t)warp * 2 * E;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = lane + 32 * i;
    if (e < E) {
      mine[e] = acc_c[i];
      mine[E + e] = acc_s[i];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * E; i += blockDim.x) {
    float t = 0.f;
    for (int w = 0; w < warps; ++w) t += sh[(size_t)w * 2 * E + i];
    parts[(int64_t)blockIdx.x * 2 * E + i] = t;
  }
}

template <int VPL>
__global__ void aux_stats_bwd_kernel(const float* __restrict__ probs, const float* __restrict__ gsum, int R, int E,
                                     float* __restrict__ dprobs) {
  pdl_prologue();
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= R) return;
  float s[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = lane + 32 * i;
    s[i] = e < E ? probs[(int64_t)t * E + e] : -INFINITY;
  }
  warp_softmax(s);
  float g[VPL], dot = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = lane + 32 * i;
    g[i] = e < E ? gsum[e] : 0.f;
    dot += g[i] * s[i];
  }
  dot = warp_sum(dot);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = lane + 32 * i;
    if (e < E) dprobs[(int64_t)t * E + e] = s[i] * (g[i] - dot);
  }
}

int vpl_for(int E) {
  PB_CHECK(E >= 1 && E <= 256, "router: at most 256 experts");
  return E <= 32 ? 1 : E <= 64 ? 2 : E <= 128 ? 4 : 8;
}

}  // namespace

void router_fwd(const void* logits, int64_t ld, int T, int E, int K, bool renorm, float* probs, float* topv,
                int64_t* topi, int* counts, cudaStream_t s) {
  PB_CHECK(K >= 1 && K <= kMaxTopK && K <= E, "router: 1 <= top_k <= min(16, experts)");
  if (T == 0) return;
  const dim3 grid((T + 7) / 8), block(256);
  switch (vpl_for(E)) {
    case 1: launch_k(router_fwd_kernel<1>, grid, block, 0, s, (const __nv_bfloat16*)logits, ld, T, E, K, renorm, probs, topv, topi, counts); break;
    case 2: launch_k(router_fwd_kernel<2>, grid, block, 0, s, (const __nv_bfloat16*)logits, ld, T, E, K, renorm, probs, topv, topi, counts); break;
    case 4: launch_k(router_fwd_kernel<4>, grid, block, 0, s, (const __nv_bfloat16*)logits, ld, T, E, K, renorm, probs, topv, topi, counts); break;
    default: launch_k(router_fwd_kernel<8>, grid, block, 0, s, (const __nv_bfloat16*)logits, ld, T, E, K, renorm, probs, topv, topi, counts); break;
  }
  PB_CUDA_CHECK(cudaGetLastError());
}

void router_bwd(const float* probs, const float* dprobs, const float* dtopv, const int64_t* topi, int T, int E, int K,
                bool renorm, void* dlogits, int64_t ld, cudaStream_t s) {
  if (T == 0) return;
  const dim3 grid((T + 7) / 8), block(256);
  auto* dl = (__nv_bfloat16*)dlogits;
  switch (vpl_for(E)) {
    case 1: launch_k(router_bwd_kernel<1>, grid, block, 0, s, probs, dprobs, dtopv, topi, T, E, K, renorm, dl, ld); break;
    case 2: launch_k(router_bwd_kernel<2>, grid, block, 0, s, probs, dprobs, dtopv, topi, T, E, K, renorm, dl, ld); break;
    case 4: launch_k(router_bwd_kernel<4>, grid, block, 0, s, probs, dprobs, dtopv, topi, T, E, K, renorm, dl, ld); break;
    default: launch_k(router_bwd_kernel<8>, grid, block, 0, s, probs, dprobs, dtopv, topi, T, E, K, renorm, dl, ld); break;
  }
  PB_CUDA_CHECK(cudaGetLastError());
}

int aux_stats_grid(int R) { return std::max(1, std::min(2 * num_sms(), (R + 7) / 8)); }

void aux_stats(const float* probs, int R, int E, int K, float* parts, cudaStream_t s) {
  PB_CHECK(K >= 1 && K <= kMaxTopK && K <= E, "aux stats: 1 <= top_k <= min(16, experts)");
  const int blocks = aux_stats_grid(R);
  const size_t sm = 8 * 2 * (size_t)E * sizeof(float);  // 8 warps x (counts, sums)
  switch (vpl_for(E)) {
    case 1: launch_k(aux_stats_kernel<1>, blocks, 256, sm, s, probs, R, E, K, parts); break;
    case 2: launch_k(aux_stats_kernel<2>, blocks, 256, sm, s, probs, R, E, K, parts); break;
    case 4: launch_k(aux_stats_kernel<4>, blocks, 256, sm, s, probs, R, E, K, parts); break;
    default: launch_k(aux_stats_kernel<8>, blocks, 256, sm, s, probs, R, E, K, parts); break;
  }
  PB_CUDA_CHECK(cudaGetLastError());
}

void aux_stats_bwd(const float* probs, const float* gsum, int R, int E, float* dprobs, cudaStream_t s) {
  if (R == 0) return;
  const dim3 grid((R + 7) / 8), block(256);
  switch (vpl_for(E)) {
    case 1: launch_k(aux_stats_bwd_kernel<1>, grid, block, 0, s, probs, gsum, R, E, dprobs); break;
    case 2: launch_k(aux_stats_bwd_kernel<2>, grid, block, 0, s, probs, gsum, R, E, dprobs); break;
    case 4: launch_k(aux_stats_bwd_kernel<4>, grid, block, 0, s, probs, gsum, R, E, dprobs); break;
    default: launch_k(aux_stats_bwd_kernel<8>, grid, block, 0, s, probs, gsum, R, E, dprobs); break;
  }
  PB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace pb
