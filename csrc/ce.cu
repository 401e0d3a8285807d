// Cross-entropy over a bf16 logits block, forward and backward in one pass
// pair (row statistics, then the softmax-minus-onehot gradient written in
// place over the logits), plus per-row statistics for the vocab-parallel
// merge across tensor-parallel ranks.
//
// Reference semantics: HF ForCausalLMLoss (logits upcast to fp32, mean over
// labels != -100; transformers/loss/loss_utils.py) on the non-model-parallel
// path and DTensor loss_parallel cross-entropy on the vocab-sharded path
// (parallel/parallel/engine/model_parallel/loss_parallel.py:22-69).
#include <cuda_bf16.h>
#include <float.h>

#include "host_util.h"
#include "ops.cuh"
#include "ptx.cuh"

namespace pb {
namespace {

constexpr int kThreads = 512;

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -FLT_MAX) return;
  s = s * __expf(m - mn) + s2 * __expf(m2 - mn);
  m = mn;
}

__device__ __forceinline__ void block_stats(float& m, float& s) {
  __shared__ float sm[kThreads / 32], ss[kThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sm[w] = m; ss[w] = s; }
  __syncthreads();
  if (w == 0) {
    m = lane < kThreads / 32 ? sm[lane] : -FLT_MAX;
    s = lane < kThreads / 32 ? ss[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      online_merge(m, s, m2, s2);
    }
    if (lane == 0) { sm[0] = m; ss[0] = s; }
  }
  __syncthreads();
  m = sm[0];
  s = ss[0];
  __syncthreads();
}

// Local row max / sum-exp with 8-wide vector loads (V % 8 == 0 and 16-byte
// aligned rows) or a scalar fallback.
__device__ __forceinline__ void row_local_stats(const __nv_bfloat16* row, int V, bool vec, float& m,
                                                float& s) {
  m = -FLT_MAX;
  s = 0.f;
  if (vec) {
    for (int c = threadIdx.x * 8; c < V; c += kThreads * 8) {
      uint4 raw = *reinterpret_cast<const uint4*>(row + c);
      const uint32_t* p = &raw.x;
      float v[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float2 f = unpack_bf16x2(p[q]);
        v[2 * q] = f.x;
        v[2 * q + 1] = f.y;
      }
      float lm = v[0];
#pragma unroll
      for (int j = 1; j < 8; ++j) lm = fmaxf(lm, v[j]);
      float ls = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) ls += __expf(v[j] - lm);
      online_merge(m, s, lm, ls);
    }
  } else {
    for (int c = threadIdx.x; c < V; c += kThreads) online_merge(m, s, __bfloat162float(row[c]), 1.f);
  }
  block_stats(m, s);
}

__global__ void __launch_bounds__(kThreads) ce_kernel(__nv_bfloat16* __restrict__ logits, int64_t ld,
                                                     const int64_t* __restrict__ labels, int T, int V,
                                                     int64_t v0, const float* __restrict__ scale,
                                                     float* __restrict__ row_lse, bool lse_given,
                                                     float* __restrict__ row_target, bool write_grad) {
  pdl_prologue();
  const int t = blockIdx.x;
  if (t >= T) return;
  __nv_bfloat16* row = logits + (int64_t)t * ld;
  const bool vec = (V % 8 == 0) && ((reinterpret_cast<uintptr_t>(row) & 15) == 0);
  float lse;
  if (lse_given) {
    lse = row_lse[t];
  } else {
    float m, s;
    row_local_stats(row, V, vec, m, s);
    lse = m + __logf(s);
    if (threadIdx.x == 0 && row_lse) row_lse[t] = lse;
  }
  const int64_t label = labels[t];
  const bool valid = label >= 0;
  const int64_t local = label - v0;
  const bool inside = valid && local >= 0 && local < V;
  if (threadIdx.x == 0) {
    const float tgt = inside ? __bfloat162float(row[local]) : 0.f;
    if (row_target) row_target[t] = tgt;
  }
  if (!write_grad) return;
  __syncthreads();  // the target logit is read before it is overwritten
  const float sc = valid ? scale[0] : 0.f;
  if (vec) {
    for (int c = threadIdx.x * 8; c < V; c += kThreads * 8) {
      uint4 raw = *reinterpret_cast<const uint4*>(row + c);
      uint32_t* p = &raw.x;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float2 f = unpack_bf16x2(p[q]);
        float g0 = __expf(f.x - lse), g1 = __expf(f.y - lse);
        if (inside && c + 2 * q == local) g0 -= 1.f;
        if (inside && c + 2 * q + 1 == local) g1 -= 1.f;
        p[q] = pack_bf16x2(g0 * sc, g1 * sc);
      }
      *reinterpret_cast<uint4*>(row + c) = raw;
    }
  } else {
    for (int c = threadIdx.x; c < V; c += kThreads) {
      float g = __expf(__bfloat162float(row[c]) - lse);
      if (inside && c == local) g -= 1.f;
      row[c] = __float2bfloat16(g * sc);
    }
  }
}

__global__ void __launch_bounds__(kThreads) ce_stats_kernel(const __nv_bfloat16* __restrict__ logits,
                                                           int64_t ld, int T, int V,
                                                           float* __restrict__ row_max,
                                                           float* __restrict__ row_sumexp) {
  pdl_prologue();
  const int t = blockIdx.x;
  if (t >= T) return;
  const __nv_bfloat16* row = logits + (int64_t)t * ld;
  const bool vec = (V % 8 == 0) && ((reinterpret_cast<uintptr_t>(row) & 15) == 0);
  float m, s;
  row_local_stats(row, V, vec, m, s);
  if (threadIdx.x == 0) {
    row_max[t] = m;
    row_sumexp[t] = s;
  }
}

// One block of 1024 threads: thread i visits rows i, i + 1024, ..., then a
// shuffle tree and the 32 warp sums in warp order; the same order on every
// run, so the loss is reproducible (no atomics).
constexpr int kRedThreads = 1024;

__device__ __forceinline__ float block_sum_fixed(float v) {
  __shared__ float warp_part[kRedThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) warp_part[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x == 0)
    for (int w = 0; w < kRedThreads / 32; ++w) t += warp_part[w];
  return t;  // valid in thread 0
}

__global__ void __launch_bounds__(kRedThreads) ce_valid_inv_kernel(const int64_t* __restrict__ labels, int T,
                                                                   float* __restrict__ inv) {
  pdl_prologue();
  float n = 0.f;
  for (int t = threadIdx.x; t < T; t += kRedThreads) n += labels[t] >= 0 ? 1.f : 0.f;
  n = block_sum_fixed(n);
  if (threadIdx.x == 0) inv[0] = 1.f / fmaxf(n, 1.f);
}

__global__ void __launch_bounds__(kRedThreads) ce_loss_reduce_kernel(const float* __restrict__ lse,
                                                                     const float* __restrict__ tgt,
                                                                     const int64_t* __restrict__ labels, int T,
                                                                     const float* __restrict__ inv,
                                                                     float* __restrict__ out, bool accumulate) {
  pdl_prologue();
  float a = 0.f;
  for (int t = threadIdx.x; t < T; t += kRedThreads)
    if (labels[t] >= 0) a += lse[t] - tgt[t];
  a = block_sum_fixed(a);
  if (threadIdx.x == 0) out[0] = a * inv[0] + (accumulate ? out[0] : 0.f);
}

}  // namespace

void ce_valid_inv(const int64_t* labels, int T, float* inv, cudaStream_t s) {
  launch_k(ce_valid_inv_kernel, 1, kRedThreads, 0, s, labels, T, inv);
  PB_CUDA_CHECK(cudaGetLastError());
}

void ce_loss_reduce(const float* lse, const float* tgt, const int64_t* labels, int T, const float* inv, float* out,
                    bool accumulate, cudaStream_t s) {
  launch_k(ce_loss_reduce_kernel, 1, kRedThreads, 0, s, lse, tgt, labels, T, inv, out, accumulate);
  PB_CUDA_CHECK(cudaGetLastError());
}

void ce_fwd_bwd(void* logits, int64_t ld, const int64_t* labels, int T, int V, int64_t v0,
                const float* scale, float* row_lse, bool lse_given, float* row_target,
                bool write_grad, cudaStream_t s) {
  if (T == 0) return;
  PB_CHECK(!write_grad || scale != nullptr, "ce: gradient scale pointer required");
  launch_k(ce_kernel, T, kThreads, 0, s, (__nv_bfloat16*)logits, ld, labels, T, V, v0, scale, row_lse,
                                   lse_given, row_target, write_grad);
  PB_CUDA_CHECK(cudaGetLastError());
}

void ce_row_stats(const void* logits, int64_t ld, int T, int V, float* row_max, float* row_sumexp,
                  cudaStream_t s) {
  if (T == 0) return;
  launch_k(ce_stats_kernel, T, kThreads, 0, s, (const __nv_bfloat16*)logits, ld, T, V, row_max, row_sumexp);
  PB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace pb
