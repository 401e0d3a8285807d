// Elementwise / gather kernels: SwiGLU forward+backward, token embedding
// forward (vocab-slice aware, for the vocab-parallel embedding) and backward
// (fp32 atomics), casts.
//
// Reference ops replaced: HF Qwen3MLP act_fn(gate)*up and nn.Embedding /
// the TP EmbeddingParallel masked lookup (transformers/integrations/
// tensor_parallel.py, used through parallel/parallel/engine/model_parallel/
// models/qwen3.py:40).
#include <cuda_bf16.h>

#include "host_util.h"
#include "ops.cuh"
#include "ptx.cuh"

namespace pb {
namespace {

__device__ __forceinline__ float bfr(float x) { return __bfloat162float(__float2bfloat16(x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + __expf(-x)); }

// 8 bf16 per thread per step.
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dh, int64_t lddh,
                                  const __nv_bfloat16* __restrict__ gu, int64_t ldgu,
                                  __nv_bfloat16* __restrict__ dgu, int64_t lddgu, int T, int I,
                                  const int* __restrict__ tiles128) {
  pdl_prologue();
  // tiles128 (optional, device): only the first 128 * *tiles128 rows are live
  if (tiles128 != nullptr) T = min(T, *tiles128 * 128);
  const int vec_per_row = I / 8;
  const int64_t total = (int64_t)T * vec_per_row;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(idx / vec_per_row);
    const int c = (int)(idx % vec_per_row) * 8;
    uint4 hraw = *reinterpret_cast<const uint4*>(dh + (int64_t)t * lddh + c);
    uint4 graw = *reinterpret_cast<const uint4*>(gu + (int64_t)t * ldgu + c);
    uint4 uraw = *reinterpret_cast<const uint4*>(gu + (int64_t)t * ldgu + I + c);
    const uint32_t* hp = &hraw.x;
    const uint32_t* gp = &graw.x;
    const uint32_t* up = &uraw.x;
    uint4 dg_out, du_out;
    uint32_t* dgp = &dg_out.x;
    uint32_t* dup = &du_out.x;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float2 h2 = unpack_bf16x2(hp[q]), g2 = unpack_bf16x2(gp[q]), u2 = unpack_bf16x2(up[q]);
      float hv[2] = {h2.x, h2.y}, gv[2] = {g2.x, g2.y}, uv[2] = {u2.x, u2.y};
      float dg[2], du[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float sg = sigmoid_f(gv[j]);
        const float silu = gv[j] * sg;
        du[j] = hv[j] * bfr(silu);
        dg[j] = hv[j] * uv[j] * sg * (1.f + gv[j] * (1.f - sg));
      }
      dgp[q] = pack_bf16x2(dg[0], dg[1]);
      dup[q] = pack_bf16x2(du[0], du[1]);
    }
    *reinterpret_cast<uint4*>(dgu + (int64_t)t * lddgu + c) = dg_out;
    *reinterpret_cast<uint4*>(dgu + (int64_t)t * lddgu + I + c) = du_out;
  }
}

// One warp per token; H % 8 == 0.
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids,
                                     const __nv_bfloat16* __restrict__ table, int64_t ldt,
                                     __nv_bfloat16* __restrict__ out, int64_t ldo, int T, int H,
                                     int64_t v0, int64_t vrows) {
  pdl_prologue();
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  const int64_t row = ids[t] - v0;
  const bool inside = row >= 0 && row < vrows;
  __nv_bfloat16* o = out + (int64_t)t * ldo;
  for (int c = lane * 8; c < H; c += 256) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (inside) v = *reinterpret_cast<const uint4*>(table + row * ldt + c);
    *reinterpret_cast<uint4*>(o + c) = v;
  }
}

// Embedding gradient from token ids sorted by value: one warp per run of
// equal ids sums that run's dY rows in fp32 (in the stable-sort order, so the
// result is deterministic) and writes - or adds into - one bf16 gradient row.
// No full-vocabulary fp32 accumulator and no atomics.
__global__ void embedding_bwd_kernel(const int64_t* __restrict__ sid, const int64_t* __restrict__ perm,
                                     const __nv_bfloat16* __restrict__ dy, int64_t lddy,
                                     __nv_bfloat16* __restrict__ grad, int64_t ldg, int T, int H, int64_t v0,
                                     int64_t vrows, bool accumulate) {
  pdl_prologue();
  const int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (p >= T) return;
  const int64_t id = sid[p];
  if (p > 0 && sid[p - 1] == id) return;  // not the head of its run
  const int64_t row = id - v0;
  if (row < 0 || row >= vrows) return;
  int end = p + 1;
  while (end < T && sid[end] == id) ++end;
  __nv_bfloat16* dst = grad + row * ldg;
  for (int c = lane * 8; c < H; c += 256) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int q = p; q < end; ++q) {
      const uint4 raw = *reinterpret_cast<const uint4*>(dy + perm[q] * lddy + c);
      const uint32_t* w = &raw.x;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(w[e]);
        acc[2 * e] += f.x;
        acc[2 * e + 1] += f.y;
      }
    }
    uint4 o;
    uint32_t* ow = &o.x;
    if (accumulate) {
      const uint4 old = *reinterpret_cast<const uint4*>(dst + c);
      const uint32_t* w = &old.x;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(w[e]);
        ow[e] = pack_bf16x2(acc[2 * e] + f.x, acc[2 * e + 1] + f.y);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) ow[e] = pack_bf16x2(acc[2 * e], acc[2 * e + 1]);
    }
    *reinterpret_cast<uint4*>(dst + c) = o;
  }
}

// x *= *s in place (bf16), skipped entirely when *s == 1: the incoming
// gradient of a loss is almost always exactly one, and the check costs no host sync.
__global__ void scale_by_scalar_kernel(__nv_bfloat16* __restrict__ x, int64_t n, const float* __restrict__ s) {
  pdl_prologue();
  const float a = *s;
  if (a == 1.f) return;
  for (int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) * 8; i < n;
       i += (int64_t)gridDim.x * blockDim.x * 8) {
    if (i + 8 <= n) {
      uint4 raw = *reinterpret_cast<const uint4*>(x + i);
      uint32_t* w = &raw.x;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(w[e]);
        w[e] = pack_bf16x2(f.x * a, f.y * a);
      }
      *reinterpret_cast<uint4*>(x + i) = raw;
    } else {
      for (int64_t j = i; j < n; ++j) x[j] = __float2bfloat16(__bfloat162float(x[j]) * a);
    }
  }
}

__global__ void cast_f32_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst,
                                     int64_t n) {
  pdl_prologue();
  for (int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) * 4; i < n;
       i += (int64_t)gridDim.x * blockDim.x * 4) {
    if (i + 4 <= n) {
      float4 v = *reinterpret_cast<const float4*>(src + i);
      uint2 o;
      o.x = pack_bf16x2(v.x, v.y);
      o.y = pack_bf16x2(v.z, v.w);
      *reinterpret_cast<uint2*>(dst + i) = o;
    } else {
      for (int64_t j = i; j < n; ++j) dst[j] = __float2bfloat16(src[j]);
    }
  }
}

int grid_for(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace

void swiglu_bwd(const void* dh, int64_t lddh, const void* gu, int64_t ldgu, void* dgu,
                int64_t lddgu, int T, int I, cudaStream_t s, const int* tiles128) {
  PB_CHECK(I % 8 == 0, "swiglu: I must be a multiple of 8");
  launch_k(swiglu_bwd_kernel, grid_for((int64_t)T * I / 8, 256), 256, 0, s,
      (const __nv_bfloat16*)dh, lddh, (const __nv_bfloat16*)gu, ldgu, (__nv_bfloat16*)dgu, lddgu, T, I, tiles128);
  PB_CUDA_CHECK(cudaGetLastError());
}

void embedding_fwd(const int64_t* ids, const void* table, int64_t ldt, void* out, int64_t ldo,
                   int T, int H, int64_t vocab_start, int64_t vocab_rows, cudaStream_t s) {
  PB_CHECK(H % 8 == 0, "embedding: H must be a multiple of 8");
  launch_k(embedding_fwd_kernel, (T + 7) / 8, 256, 0, s, ids, (const __nv_bfloat16*)table, ldt,
                                                   (__nv_bfloat16*)out, ldo, T, H, vocab_start,
                                                   vocab_rows);
  PB_CUDA_CHECK(cudaGetLastError());
}

void embedding_bwd(const int64_t* sorted_ids, const int64_t* perm, const void* dy, int64_t lddy, void* grad,
                   int64_t ldg, int T, int H, int64_t vocab_start, int64_t vocab_rows, bool accumulate,
                   cudaStream_t s) {
  PB_CHECK(H % 8 == 0 && lddy % 8 == 0 && ldg % 8 == 0, "embedding: H and strides must be multiples of 8");
  if (T == 0) return;
  launch_k(embedding_bwd_kernel, (T + 7) / 8, 256, 0, s, sorted_ids, perm, (const __nv_bfloat16*)dy, lddy,
                                                   (__nv_bfloat16*)grad, ldg, T, H, vocab_start, vocab_rows,
                                                   accumulate);
  PB_CUDA_CHECK(cudaGetLastError());
}

void scale_by_scalar(void* x, int64_t n, const float* s_dev, cudaStream_t s) {
  if (n == 0) return;
  launch_k(scale_by_scalar_kernel, grid_for(n / 8 + 1, 256), 256, 0, s, (__nv_bfloat16*)x, n, s_dev);
  PB_CUDA_CHECK(cudaGetLastError());
}

// Few slices (split-K): a thread per 4 outputs issues one 16-byte load per
// slice, then adds them in slice order.  Many slices (block partials of a
// weight gradient): a 1024-thread block owns 32 columns, warp w adds slices
// w, w + 32, ... (one coalesced 128-byte row per load) and the 32 warp sums
// are added in warp order.  Both orders are fixed, so the sums are
// reproducible.
__device__ __forceinline__ void store4_out(void* out, bool out_bf16, bool accumulate, int64_t i, float4 a) {
  if (out_bf16) {
    uint2* o = reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(out) + i);
    if (accumulate) {
      const uint2 old = *o;
      const float2 p = unpack_bf16x2(old.x), q = unpack_bf16x2(old.y);
      a.x += p.x; a.y += p.y; a.z += q.x; a.w += q.y;
    }
    *o = make_uint2(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w));
  } else {
    float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + i);
    if (accumulate) {
      const float4 p = *o;
      a.x += p.x; a.y += p.y; a.z += p.z; a.w += p.w;
    }
    *o = a;
  }
}

__device__ __forceinline__ void store1_out(void* out, bool out_bf16, bool accumulate, int64_t i, float a) {
  if (out_bf16) {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out) + i;
    *o = __float2bfloat16(a + (accumulate ? __bfloat162float(*o) : 0.f));
  } else {
    float* o = reinterpret_cast<float*>(out) + i;
    *o = a + (accumulate ? *o : 0.f);
  }
}

constexpr int kFewSlices = 8;

__global__ void sum_slices_few_vec_kernel(const float* __restrict__ parts, int slices, int64_t len4, int64_t stride,
                                          void* __restrict__ out, bool out_bf16, bool accumulate) {
  pdl_prologue();
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < len4; v += (int64_t)gridDim.x * blockDim.x) {
    float4 x[kFewSlices];
#pragma unroll
    for (int k = 0; k < kFewSlices; ++k)
      if (k < slices) x[k] = __ldcs(reinterpret_cast<const float4*>(parts + (int64_t)k * stride) + v);
    float4 a = x[0];
#pragma unroll
    for (int k = 1; k < kFewSlices; ++k)
      if (k < slices) {
        a.x += x[k].x; a.y += x[k].y; a.z += x[k].z; a.w += x[k].w;
      }
    store4_out(out, out_bf16, accumulate, v * 4, a);
  }
}

__global__ void sum_slices_few_kernel(const float* __restrict__ parts, int slices, int64_t len, int64_t stride,
                                      void* __restrict__ out, bool out_bf16, bool accumulate) {
  pdl_prologue();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < len; i += (int64_t)gridDim.x * blockDim.x) {
    float a = 0.f;
    for (int k = 0; k < slices; ++k) a += parts[(int64_t)k * stride + i];
    store1_out(out, out_bf16, accumulate, i, a);
  }
}

__global__ void __launch_bounds__(1024) sum_slices_many_kernel(const float* __restrict__ parts, int slices,
                                                               int64_t len, int64_t stride, void* __restrict__ out,
                                                               bool out_bf16, bool accumulate) {
  pdl_prologue();
  __shared__ float part[32][33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c = (int64_t)blockIdx.x * 32 + lane;
  float a = 0.f;
  if (c < len) {
    int k = warp;
    for (; k + 96 < slices; k += 128) {  // four independent loads in flight
      const float x0 = parts[(int64_t)k * stride + c], x1 = parts[(int64_t)(k + 32) * stride + c];
      const float x2 = parts[(int64_t)(k + 64) * stride + c], x3 = parts[(int64_t)(k + 96) * stride + c];
      a += x0;
      a += x1;
      a += x2;
      a += x3;
    }
    for (; k < slices; k += 32) a += parts[(int64_t)k * stride + c];
  }
  part[warp][lane] = a;
  __syncthreads();
  if (warp == 0 && c < len) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 32; ++w) t += part[w][lane];
    store1_out(out, out_bf16, accumulate, c, t);
  }
}

void sum_slices(const float* parts, int slices, int64_t len, int64_t stride, void* out, bool out_bf16,
                bool accumulate, cudaStream_t s) {
  PB_CHECK(slices >= 1 && len >= 0 && stride >= len, "sum_slices: shapes");
  if (len == 0) return;
  if (slices <= kFewSlices) {
    const bool vec = len % 4 == 0 && stride % 4 == 0 && (reinterpret_cast<uintptr_t>(parts) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(out) & (out_bf16 ? 7 : 15)) == 0;
    if (vec)
      launch_k(sum_slices_few_vec_kernel, grid_for(len / 4, 256), 256, 0, s, parts, slices, len / 4, stride, out, out_bf16,
                                                                       accumulate);
    else
      launch_k(sum_slices_few_kernel, grid_for(len, 256), 256, 0, s, parts, slices, len, stride, out, out_bf16,
                                                               accumulate);
  } else {
    launch_k(sum_slices_many_kernel, (unsigned)((len + 31) / 32), 1024, 0, s, parts, slices, len, stride, out, out_bf16,
                                                                        accumulate);
  }
  PB_CUDA_CHECK(cudaGetLastError());
}

void cast_f32_to_bf16(const float* src, void* dst, int64_t n, cudaStream_t s) {
  launch_k(cast_f32_bf16_kernel, grid_for(n / 4 + 1, 256), 256, 0, s, src, (__nv_bfloat16*)dst, n);
  PB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace pb
