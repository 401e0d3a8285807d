// Multi-tensor AdamW and the one-pass gradient sum-of-squares / finite check.
//
// Reference semantics: torch.optim.AdamW on the (bf16) parameter shards
// (parallel/parallel/engine/engine.py:61-66) with clipping by the global norm
// (parallel/parallel/engine/model_parallel/grad_norm.py:15-82,
// parallel/parallel/engine/dp_sharded.py:453-472) and the finite check of
// engine.py:249-268.  Here the clip coefficient never leaves the device: it
// is computed by clip_coef() and multiplied into the gradient inside the
// AdamW kernel, and a non-finite flag makes the update a no-op.
#include <cuda_bf16.h>

#include <algorithm>
#include <vector>

#include "host_util.h"
#include "ops.cuh"
#include "ptx.cuh"

namespace pb {
namespace {

constexpr int kMaxSegs = 48;
constexpr int kThreads = 256;
constexpr int kChunk = 8192;  // elements per block-chunk (multiple of 8 * kThreads)

struct SegTable {
  AdamSeg seg[kMaxSegs];
  int chunk_start[kMaxSegs + 1];
  int nseg;
};

struct NormTable {
  NormSeg seg[kMaxSegs];
  int chunk_start[kMaxSegs + 1];
  int nseg;
};

template <typename T>
__device__ __forceinline__ float ldf(const void* p, int64_t i) {
  if constexpr (sizeof(T) == 4)
    return reinterpret_cast<const float*>(p)[i];
  else
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}
template <typename T>
__device__ __forceinline__ void stf(void* p, int64_t i, float v) {
  if constexpr (sizeof(T) == 4)
    reinterpret_cast<float*>(p)[i] = v;
  else
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16(v);
}

__device__ __forceinline__ int find_seg(const int* starts, int nseg, int chunk) {
  int s = 0;
  while (s + 1 < nseg && starts[s + 1] <= chunk) ++s;
  return s;
}

template <typename T>
__device__ __forceinline__ void ld8(const void* base, int64_t i, float* v) {
  if constexpr (sizeof(T) == 4) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + i);
    float4 a = p[0], b = p[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(base) + i);
    const uint32_t* q = &u.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 f = unpack_bf16x2(q[k]);
      v[2 * k] = f.x;
      v[2 * k + 1] = f.y;
    }
  }
}
template <typename T>
__device__ __forceinline__ void st8(void* base, int64_t i, const float* v) {
  if constexpr (sizeof(T) == 4) {
    float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + i);
    p[0] = make_float4(v[0], v[1], v[2], v[3]);
    p[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint4 u;
    u.x = pack_bf16x2(v[0], v[1]);
    u.y = pack_bf16x2(v[2], v[3]);
    u.z = pack_bf16x2(v[4], v[5]);
    u.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(base) + i) = u;
  }
}

__device__ __forceinline__ void adam_elem(float& p, float& m, float& v, float g, float lr, float wd, float beta1,
                                          float beta2, float eps, float step_size, float bc2_sqrt) {
  p *= 1.f - lr * wd;
  m += (g - m) * (1.f - beta1);
  v = v * beta2 + (1.f - beta2) * g * g;
  const float denom = sqrtf(v) / bc2_sqrt + eps;
  p -= step_size * m / denom;
}

template <typename GT, typename ST>
__global__ void __launch_bounds__(kThreads) adamw_kernel(SegTable tab, float lr, float beta1,
                                                         float beta2, float eps, float wd,
                                                         float bc1, float bc2_sqrt,
                                                         const float* __restrict__ gscale,
                                                         const int* __restrict__ skip,
                                                         const float* __restrict__ hyper) {
  pdl_prologue();
  if (skip && *skip) return;
  const float gs = gscale ? *gscale : 1.f;
  if (hyper) {  // {lr, 1 - beta1^t, sqrt(1 - beta2^t)} from the device (CUDA-graph replays)
    lr = hyper[0];
    bc1 = hyper[1];
    bc2_sqrt = hyper[2];
  }
  const int chunk = blockIdx.x;
  const int si = find_seg(tab.chunk_start, tab.nseg, chunk);
  const AdamSeg sg = tab.seg[si];
  const int64_t base = (int64_t)(chunk - tab.chunk_start[si]) * kChunk;
  const int64_t end = min(sg.n, base + kChunk);
  const float step_size = lr / bc1;
  const bool vec = ((reinterpret_cast<uintptr_t>(sg.p) | reinterpret_cast<uintptr_t>(sg.g) |
                     reinterpret_cast<uintptr_t>(sg.m) | reinterpret_cast<uintptr_t>(sg.v)) & 31) == 0;
  int64_t i = base;
  if (vec) {
    // 8 elements per thread per step (kChunk is a multiple of 8 * kThreads)
    const int64_t vend = base + ((end - base) / 8) * 8;
    for (int64_t j = base + threadIdx.x * 8; j < vend; j += kThreads * 8) {
      float g[8], p[8], m[8], v[8];
      ld8<GT>(sg.g, j, g);
      ld8<__nv_bfloat16>(sg.p, j, p);
      ld8<ST>(sg.m, j, m);
      ld8<ST>(sg.v, j, v);
#pragma unroll
      for (int k = 0; k < 8; ++k) adam_elem(p[k], m[k], v[k], g[k] * gs, lr, wd, beta1, beta2, eps, step_size, bc2_sqrt);
      st8<__nv_bfloat16>(sg.p, j, p);
      st8<ST>(sg.m, j, m);
      st8<ST>(sg.v, j, v);
    }
    i = vend;
  }
  for (int64_t j = i + threadIdx.x; j < end; j += kThreads) {
    float p = ldf<__nv_bfloat16>(sg.p, j), m = ldf<ST>(sg.m, j), v = ldf<ST>(sg.v, j);
    adam_elem(p, m, v, ldf<GT>(sg.g, j) * gs, lr, wd, beta1, beta2, eps, step_size, bc2_sqrt);
    stf<__nv_bfloat16>(sg.p, j, p);
    stf<ST>(sg.m, j, m);
    stf<ST>(sg.v, j, v);
  }
}

// One block per chunk: the chunk's weighted sum of squares and its non-finite
// bit go to parts[2 * (chunk_base + chunk)] / [.. + 1]; sumsq_finish adds the
// chunks in chunk order, so the norm has the same bits on every run.
template <typename GT>
__global__ void __launch_bounds__(kThreads) sumsq_kernel(NormTable tab, float* __restrict__ parts, int chunk_base) {
  pdl_prologue();
  const int chunk = blockIdx.x;
  const int si = find_seg(tab.chunk_start, tab.nseg, chunk);
  const NormSeg sg = tab.seg[si];
  const int64_t base = (int64_t)(chunk - tab.chunk_start[si]) * kChunk;
  const int64_t end = min(sg.n, base + kChunk);
  float acc = 0.f;
  bool bad = false;
  int64_t i0 = base;
  if ((reinterpret_cast<uintptr_t>(sg.g) & 31) == 0) {
    // 8 elements (one 16- or 32-byte load) per thread per step
    const int64_t vend = base + ((end - base) / 8) * 8;
    for (int64_t j = base + threadIdx.x * 8; j < vend; j += kThreads * 8) {
      float g[8];
      ld8<GT>(sg.g, j, g);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        bad |= !isfinite(g[k]);
        acc = fmaf(g[k], g[k], acc);
      }
    }
    i0 = vend;
  }
  for (int64_t i = i0 + threadIdx.x; i < end; i += kThreads) {
    const float g = ldf<GT>(sg.g, i);
    bad |= !isfinite(g);
    acc = fmaf(g, g, acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  const unsigned any_bad = __ballot_sync(0xffffffffu, bad);
  __shared__ float sacc[kThreads / 32];
  __shared__ int sbad[kThreads / 32];
  if ((threadIdx.x & 31) == 0) {
    sacc[threadIdx.x >> 5] = acc;
    sbad[threadIdx.x >> 5] = any_bad != 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    int b = 0;
    for (int w = 0; w < kThreads / 32; ++w) {
      t += sacc[w];
      b |= sbad[w];
    }
    parts[2 * (int64_t)(chunk_base + chunk)] = t * sg.weight;
    parts[2 * (int64_t)(chunk_base + chunk) + 1] = (float)b;
  }
}

constexpr int kFinishThreads = 1024;

__global__ void __launch_bounds__(kFinishThreads) sumsq_finish_kernel(const float* __restrict__ parts, int chunks,
                                                                      float* __restrict__ out, int* __restrict__ flag,
                                                                      bool accumulate) {
  pdl_prologue();
  float a = 0.f;
  float bad = 0.f;
  for (int c = threadIdx.x; c < chunks; c += kFinishThreads) {
    a += parts[2 * (int64_t)c];
    bad = fmaxf(bad, parts[2 * (int64_t)c + 1]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    bad = fmaxf(bad, __shfl_xor_sync(0xffffffffu, bad, o));
  }
  __shared__ float sa[kFinishThreads / 32], sb[kFinishThreads / 32];
  if ((threadIdx.x & 31) == 0) {
    sa[threadIdx.x >> 5] = a;
    sb[threadIdx.x >> 5] = bad;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f, b = 0.f;
    for (int w = 0; w < kFinishThreads / 32; ++w) {
      t += sa[w];
      b = fmaxf(b, sb[w]);
    }
    out[0] = t + (accumulate ? out[0] : 0.f);
    if (flag) flag[0] = (b > 0.f ? 1 : 0) | (accumulate ? flag[0] : 0);
  }
}

__global__ void clip_coef_kernel(const float* total, float max_norm, float* out) {
  pdl_prologue();
  const float n = sqrtf(*total);
  out[0] = fminf(max_norm / (n + 1e-6f), 1.f);
}

}  // namespace

void adamw_multi(const AdamSeg* segs, int nseg, float lr, float beta1, float beta2, float eps,
                 float wd, int step, const float* grad_scale_dev, const int* skip_dev, const float* hyper_dev,
                 bool grad_f32, bool state_f32, cudaStream_t s) {
  const float bc1 = 1.f - powf(beta1, (float)step);
  const float bc2_sqrt = sqrtf(1.f - powf(beta2, (float)step));
  for (int off = 0; off < nseg; off += kMaxSegs) {
    SegTable tab{};
    tab.nseg = std::min(kMaxSegs, nseg - off);
    int chunks = 0;
    for (int i = 0; i < tab.nseg; ++i) {
      tab.seg[i] = segs[off + i];
      tab.chunk_start[i] = chunks;
      chunks += (int)((segs[off + i].n + kChunk - 1) / kChunk);
    }
    tab.chunk_start[tab.nseg] = chunks;
    if (chunks == 0) continue;
    if (grad_f32 && state_f32)
      launch_k(adamw_kernel<float, float>, chunks, kThreads, 0, s, tab, lr, beta1, beta2, eps, wd, bc1,
                                                             bc2_sqrt, grad_scale_dev, skip_dev, hyper_dev);
    else if (grad_f32)
      launch_k(adamw_kernel<float, __nv_bfloat16>, chunks, kThreads, 0, s,
          tab, lr, beta1, beta2, eps, wd, bc1, bc2_sqrt, grad_scale_dev, skip_dev, hyper_dev);
    else if (state_f32)
      launch_k(adamw_kernel<__nv_bfloat16, float>, chunks, kThreads, 0, s,
          tab, lr, beta1, beta2, eps, wd, bc1, bc2_sqrt, grad_scale_dev, skip_dev, hyper_dev);
    else
      launch_k(adamw_kernel<__nv_bfloat16, __nv_bfloat16>, chunks, kThreads, 0, s,
          tab, lr, beta1, beta2, eps, wd, bc1, bc2_sqrt, grad_scale_dev, skip_dev, hyper_dev);
    PB_CUDA_CHECK(cudaGetLastError());
  }
}

int64_t sumsq_chunks(const NormSeg* segs, int nseg) {
  int64_t chunks = 0;
  for (int i = 0; i < nseg; ++i) chunks += (segs[i].n + kChunk - 1) / kChunk;
  return chunks;
}

void sumsq_multi(const NormSeg* segs, int nseg, bool f32, float* parts, float* out, int* out_flag, bool accumulate,
                 cudaStream_t s) {
  const int64_t total = sumsq_chunks(segs, nseg);
  PB_CHECK(total < (int64_t)1 << 30, "sumsq: too many chunks");
  int base = 0;
  for (int off = 0; off < nseg; off += kMaxSegs) {
    NormTable tab{};
    tab.nseg = std::min(kMaxSegs, nseg - off);
    int chunks = 0;
    for (int i = 0; i < tab.nseg; ++i) {
      tab.seg[i] = segs[off + i];
      tab.chunk_start[i] = chunks;
      chunks += (int)((segs[off + i].n + kChunk - 1) / kChunk);
    }
    tab.chunk_start[tab.nseg] = chunks;
    if (chunks == 0) continue;
    if (f32)
      launch_k(sumsq_kernel<float>, chunks, kThreads, 0, s, tab, parts, base);
    else
      launch_k(sumsq_kernel<__nv_bfloat16>, chunks, kThreads, 0, s, tab, parts, base);
    PB_CUDA_CHECK(cudaGetLastError());
    base += chunks;
  }
  launch_k(sumsq_finish_kernel, 1, kFinishThreads, 0, s, parts, (int)total, out, out_flag, accumulate);
  PB_CUDA_CHECK(cudaGetLastError());
}

void clip_coef(const float* total_sumsq, float max_norm, float* scale_out, cudaStream_t s) {
  launch_k(clip_coef_kernel, 1, 1, 0, s, total_sumsq, max_norm, scale_out);
  PB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace pb
