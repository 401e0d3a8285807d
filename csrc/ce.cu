// Cross-entropy over a bf16 logits block, forward and backward in one pass
// pair (row statistics, then the softmax-minus-onehot gradient written in
// place over the logits), plus per-row statistics for the vocab-parallel
// merge across tensor-parallel ranks.
//
// Reference semantics: HF ForCausalLMLoss (logits upcast to fp32, mean over
// labels != -100; transformers/loss/loss_utils.py) on the non-model-parallel
// path and DTensor loss_parallel cross-entropy on the vocab-sharded path
// (parallel/parallel/engine/model_parallel/loss_parallel.py:22-69).
#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <float.h>

#include <algorithm>
#include <mutex>

#include "host_util.h"
#include "ops.cuh"
#include "ptx.cuh"

namespace pb {
namespace {

constexpr int kThreads = 1024;

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -FLT_MAX) return;
  s = s * __expf(m - mn) + s2 * __expf(m2 - mn);
  m = mn;
}

template <int NT>
__device__ __forceinline__ void block_stats_n(float& m, float& s) {
  __shared__ float sm[NT / 32], ss[NT / 32];
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
    m = lane < NT / 32 ? sm[lane] : -FLT_MAX;
    s = lane < NT / 32 ? ss[lane] : 0.f;
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

__device__ __forceinline__ void block_stats(float& m, float& s) { block_stats_n<kThreads>(m, s); }

// Local row max / sum-exp with 8-wide vector loads (V % 8 == 0 and 16-byte
// aligned rows) or a scalar fallback.  Each thread keeps a running max and
// rescales its sum only when a vector raises it (rare after the first few),
// so the pass costs one exponential per element; kUnroll vectors are loaded
// before any is used.
constexpr int kUnroll = 4;

__device__ __forceinline__ void row_local_stats(const __nv_bfloat16* row, int V, bool vec, float& m,
                                                float& s) {
  m = -FLT_MAX;
  s = 0.f;
  if (vec) {
    for (int c0 = threadIdx.x * 8; c0 < V; c0 += kThreads * 8 * kUnroll) {
      uint4 raw[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int c = c0 + u * kThreads * 8;
        if (c < V) raw[u] = *reinterpret_cast<const uint4*>(row + c);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (c0 + u * kThreads * 8 >= V) break;
        const uint32_t* p = &raw[u].x;
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
        if (lm > m) {
          s *= __expf(m - lm);  // m == -FLT_MAX: s is 0 and stays 0
          m = lm;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) s += __expf(v[j] - m);
      }
    }
  } else {
    for (int c = threadIdx.x; c < V; c += kThreads) online_merge(m, s, __bfloat162float(row[c]), 1.f);
  }
  block_stats(m, s);
}

// The gradient pass re-reads the row the statistics pass just read; with
// 1024-thread CTAs two rows per SM are in flight (about 90 MB at V = 151936),
// so the re-read mostly hits L2 and the logits cross DRAM once each way.
__device__ __forceinline__ void ce_row(__nv_bfloat16* __restrict__ logits, int64_t ld,
                                       const int64_t* __restrict__ labels, int t, int V, int64_t v0,
                                       const float* __restrict__ scale, float* __restrict__ row_lse,
                                       bool lse_given, float* __restrict__ row_target, bool write_grad) {
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
    for (int c0 = threadIdx.x * 8; c0 < V; c0 += kThreads * 8 * kUnroll) {
      uint4 raw[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int c = c0 + u * kThreads * 8;
        if (c < V) raw[u] = *reinterpret_cast<const uint4*>(row + c);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int c = c0 + u * kThreads * 8;
        if (c >= V) break;
        uint32_t* p = &raw[u].x;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float2 f = unpack_bf16x2(p[q]);
          float g0 = __expf(f.x - lse), g1 = __expf(f.y - lse);
          if (inside && c + 2 * q == local) g0 -= 1.f;
          if (inside && c + 2 * q + 1 == local) g1 -= 1.f;
          p[q] = pack_bf16x2(g0 * sc, g1 * sc);
        }
        *reinterpret_cast<uint4*>(row + c) = raw[u];
      }
    }
  } else {
    for (int c = threadIdx.x; c < V; c += kThreads) {
      float g = __expf(__bfloat162float(row[c]) - lse);
      if (inside && c == local) g -= 1.f;
      row[c] = __float2bfloat16(g * sc);
    }
  }
}

// One CTA per row (a grid that walks rows also works: the shared statistics
// of a row are consumed before the next row's are written).
__global__ void __launch_bounds__(kThreads) ce_kernel(__nv_bfloat16* __restrict__ logits, int64_t ld,
                                                     const int64_t* __restrict__ labels, int T, int V,
                                                     int64_t v0, const float* __restrict__ scale,
                                                     float* __restrict__ row_lse, bool lse_given,
                                                     float* __restrict__ row_target, bool write_grad) {
  pdl_prologue();
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    ce_row(logits, ld, labels, t, V, v0, scale, row_lse, lse_given, row_target, write_grad);
    __syncthreads();
  }
}

// Cluster-resident variant for wide rows: a cluster of kClusterCtas CTAs owns
// one row, each CTA one contiguous quarter kept in its shared memory.  The
// quarter is read from DRAM once (statistics on the fly, running max), the
// CTAs exchange their (max, sum-exp) through distributed shared memory and
// merge them in rank order, and the gradient is computed from shared memory
// and written once: the logits cross DRAM once each way with no reliance on
// L2 for a second read.
constexpr int kClusterCtas = 4;
constexpr int kClusterThreads = 512;

__global__ void __cluster_dims__(kClusterCtas, 1, 1) __launch_bounds__(kClusterThreads)
    ce_cluster_kernel(__nv_bfloat16* __restrict__ logits, int64_t ld, const int64_t* __restrict__ labels, int V,
                      int64_t v0, const float* __restrict__ scale, float* __restrict__ row_lse,
                      float* __restrict__ row_target, bool write_grad) {
  pdl_prologue();
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ uint4 s_row[];          // this CTA's part of the row (16-byte vectors)
  __shared__ float2 s_stat[kClusterCtas];   // per-rank (max, sum-exp), read by every CTA of the cluster
  const int part = (int)cluster.block_rank();
  const int64_t t = blockIdx.x / kClusterCtas;
  const int nvec = V / 8 / kClusterCtas;    // vectors per part (V % (8 * kClusterCtas) == 0)
  uint4* row4 = reinterpret_cast<uint4*>(logits + t * ld) + (int64_t)part * nvec;
  float m = -FLT_MAX, s = 0.f;
  for (int i0 = threadIdx.x; i0 < nvec; i0 += kClusterThreads * kUnroll) {
    uint4 raw[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = i0 + u * kClusterThreads;
      if (i < nvec) raw[u] = row4[i];
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = i0 + u * kClusterThreads;
      if (i >= nvec) break;
      s_row[i] = raw[u];
      const uint32_t* p = &raw[u].x;
      float v[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(p[q]);
        v[2 * q] = f.x;
        v[2 * q + 1] = f.y;
      }
      float lm = v[0];
#pragma unroll
      for (int j = 1; j < 8; ++j) lm = fmaxf(lm, v[j]);
      if (lm > m) {
        s *= __expf(m - lm);
        m = lm;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) s += __expf(v[j] - m);
    }
  }
  block_stats_n<kClusterThreads>(m, s);
  if (threadIdx.x == 0) s_stat[part] = make_float2(m, s);
  cluster.sync();  // every part's statistics written (and every s_row filled)
  float gm = -FLT_MAX, gs = 0.f;
#pragma unroll
  for (int r = 0; r < kClusterCtas; ++r) {
    const float2 o = *cluster.map_shared_rank(&s_stat[r], r);
    online_merge(gm, gs, o.x, o.y);
  }
  cluster.sync();  // no CTA leaves (or reuses s_stat) while others still read it
  const float lse = gm + __logf(gs);
  const int64_t label = labels[t];
  const bool valid = label >= 0;
  const int64_t local = label - v0;
  const bool inside = valid && local >= 0 && local < V;
  const int64_t lo = (int64_t)part * nvec * 8;
  const bool mine = inside && local >= lo && local < lo + (int64_t)nvec * 8;
  if (threadIdx.x == 0) {
    if (part == 0 && row_lse) row_lse[t] = lse;
    if (row_target && (mine || (!inside && part == 0))) {
      const int64_t li = local - lo;
      row_target[t] = mine ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(s_row)[li]) : 0.f;
    }
  }
  if (!write_grad) return;
  const float sc = valid ? scale[0] : 0.f;
  for (int i = threadIdx.x; i < nvec; i += kClusterThreads) {
    uint4 raw = s_row[i];
    uint32_t* p = &raw.x;
    const int64_t c = lo + (int64_t)i * 8;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = unpack_bf16x2(p[q]);
      float g0 = __expf(f.x - lse), g1 = __expf(f.y - lse);
      if (inside && c + 2 * q == local) g0 -= 1.f;
      if (inside && c + 2 * q + 1 == local) g1 -= 1.f;
      p[q] = pack_bf16x2(g0 * sc, g1 * sc);
    }
    row4[i] = raw;
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
  const size_t part_bytes = (size_t)V * 2 / kClusterCtas;
  if (!lse_given && V % (8 * kClusterCtas) == 0 && V >= 4096 && part_bytes <= 96 * 1024 && ld % 8 == 0 &&
      (reinterpret_cast<uintptr_t>(logits) & 15) == 0 && (int64_t)T * kClusterCtas < (int64_t)INT32_MAX) {
    static std::mutex mu;
    static size_t attr_bytes[64] = {0};
    int dev = 0;
    PB_CUDA_CHECK(cudaGetDevice(&dev));
    {
      std::lock_guard<std::mutex> lk(mu);
      if (attr_bytes[dev & 63] < part_bytes) {
        PB_CUDA_CHECK(cudaFuncSetAttribute(ce_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)part_bytes));
        attr_bytes[dev & 63] = part_bytes;
      }
    }
    launch_k(ce_cluster_kernel, T * kClusterCtas, kClusterThreads, part_bytes, s, (__nv_bfloat16*)logits, ld, labels,
             V, v0, scale, row_lse, row_target, write_grad);
    PB_CUDA_CHECK(cudaGetLastError());
    return;
  }
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
