// RMSNorm and the fused per-head QK-RMSNorm + rotate-half RoPE.
//
// Numerics follow HF Qwen3 (transformers/models/qwen3/modeling_qwen3.py,
// Qwen3RMSNorm and apply_rotary_pos_emb): the normalisation runs in fp32,
// the normalised value is rounded to bf16 before the weight multiply, and the
// RoPE products / sum are rounded to bf16 the way the bf16 eager ops round.
// The reference gets these ops from HF (parallel/parallel/engine/
// model_loading.py:17-35); here each is one memory-bound pass.
#include <cuda_bf16.h>

#include "host_util.h"
#include "ops.cuh"
#include "ptx.cuh"

namespace pb {
namespace {

__device__ __forceinline__ float bfr(float x) { return __bfloat162float(__float2bfloat16(x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* v) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* v) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

// One warp per row; cols % 8 == 0.
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                   const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ y,
                                   int64_t ldy, float* __restrict__ rstd, int rows, int cols, float eps) {
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const __nv_bfloat16* xr = x + (int64_t)row * ldx;
  float ss = 0.f;
  for (int c = lane * 8; c < cols; c += 256) {
    float v[8];
    load8(xr + c, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)cols + eps);
  if (lane == 0 && rstd) rstd[row] = r;
  __nv_bfloat16* yr = y + (int64_t)row * ldy;
  for (int c = lane * 8; c < cols; c += 256) {
    float v[8], wv[8];
    load8(xr + c, v);
    load8(w + c, wv);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = wv[j] * bfr(v[j] * r);
    store8(yr + c, v);
  }
}

// Block of 8 warps handles `rows_per_block` rows; dw partials in smem.
__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, int64_t lddy,
                                   const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                   const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
                                   __nv_bfloat16* __restrict__ dx, int64_t lddx, float* __restrict__ dw,
                                   int rows, int cols, int rows_per_block) {
  extern __shared__ float sdw[];
  for (int c = threadIdx.x; c < cols; c += blockDim.x) sdw[c] = 0.f;
  __syncthreads();
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(rows, r0 + rows_per_block);
  for (int row = r0 + (threadIdx.x >> 5); row < r1; row += warps) {
    const float r = rstd[row];
    const __nv_bfloat16* xr = x + (int64_t)row * ldx;
    const __nv_bfloat16* dyr = dy + (int64_t)row * lddy;
    float dot = 0.f;
    for (int c = lane * 8; c < cols; c += 256) {
      float xv[8], gv[8], wv[8];
      load8(xr + c, xv);
      load8(dyr + c, gv);
      load8(w + c, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xh = xv[j] * r;
        dot += gv[j] * wv[j] * xh;
        atomicAdd(&sdw[c + j], gv[j] * bfr(xh));
      }
    }
    dot = warp_sum(dot) / (float)cols;
    __nv_bfloat16* dxr = dx + (int64_t)row * lddx;
    for (int c = lane * 8; c < cols; c += 256) {
      float xv[8], gv[8], wv[8], o[8];
      load8(xr + c, xv);
      load8(dyr + c, gv);
      load8(w + c, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = r * (gv[j] * wv[j] - xv[j] * r * dot);
      store8(dxr + c, o);
    }
  }
  __syncthreads();
  if (dw)
    for (int c = threadIdx.x; c < cols; c += blockDim.x) atomicAdd(&dw[c], sdw[c]);
}

// One warp per (token, head); D == 128: lane owns elements [4*lane, 4*lane+4).
// RoPE pairs element i with i +- 64, i.e. lane l with lane l ^ 16.
__global__ void qknorm_rope_fwd_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ldqkv,
                                       const __nv_bfloat16* __restrict__ qw,
                                       const __nv_bfloat16* __restrict__ kw,
                                       const __nv_bfloat16* __restrict__ cosb,
                                       const __nv_bfloat16* __restrict__ sinb,
                                       __nv_bfloat16* __restrict__ q_out, int64_t ldq,
                                       __nv_bfloat16* __restrict__ k_out, int64_t ldk,
                                       float* __restrict__ rstd, int T, int S, int nq, int nkv, float eps) {
  constexpr int D = 128;
  const int warps = blockDim.x >> 5;
  const int item = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int nh = nq + nkv;
  if (item >= T * nh) return;
  const int t = item / nh, h = item % nh;
  const bool is_q = h < nq;
  const __nv_bfloat16* src = qkv + (int64_t)t * ldqkv + (int64_t)h * D + lane * 4;
  const __nv_bfloat16* wgt = (is_q ? qw : kw) + lane * 4;
  uint2 raw = *reinterpret_cast<const uint2*>(src);
  float2 a = unpack_bf16x2(raw.x), b = unpack_bf16x2(raw.y);
  float v[4] = {a.x, a.y, b.x, b.y};
  float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)D + eps);
  if (lane == 0) rstd[(int64_t)t * nh + h] = r;
  uint2 wraw = *reinterpret_cast<const uint2*>(wgt);
  float2 wa = unpack_bf16x2(wraw.x), wb = unpack_bf16x2(wraw.y);
  float wv[4] = {wa.x, wa.y, wb.x, wb.y};
  float n[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) n[j] = bfr(wv[j] * bfr(v[j] * r));
  // partner values (i +- 64)
  float p[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) p[j] = __shfl_xor_sync(0xffffffffu, n[j], 16);
  const int pos = t % S;
  const __nv_bfloat16* cr = cosb + (int64_t)pos * D + lane * 4;
  const __nv_bfloat16* sr = sinb + (int64_t)pos * D + lane * 4;
  uint2 craw = *reinterpret_cast<const uint2*>(cr);
  uint2 sraw = *reinterpret_cast<const uint2*>(sr);
  float2 ca = unpack_bf16x2(craw.x), cb = unpack_bf16x2(craw.y);
  float2 sa = unpack_bf16x2(sraw.x), sb = unpack_bf16x2(sraw.y);
  float cv[4] = {ca.x, ca.y, cb.x, cb.y}, sv[4] = {sa.x, sa.y, sb.x, sb.y};
  const float sign = lane < 16 ? -1.f : 1.f;  // rotate_half: [-x2, x1]
  float o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) o[j] = bfr(bfr(n[j] * cv[j]) + bfr(sign * p[j] * sv[j]));
  __nv_bfloat16* dst = is_q ? q_out + (int64_t)t * ldq + (int64_t)h * D
                            : k_out + (int64_t)t * ldk + (int64_t)(h - nq) * D;
  uint2 out;
  out.x = pack_bf16x2(o[0], o[1]);
  out.y = pack_bf16x2(o[2], o[3]);
  *reinterpret_cast<uint2*>(dst + lane * 4) = out;
}

// Backward of the above.  Block = 8 warps; per-block smem partials for the
// q/k norm weight grads (2 x 128 floats).
__global__ void qknorm_rope_bwd_kernel(const __nv_bfloat16* __restrict__ dq, int64_t lddq,
                                       const __nv_bfloat16* __restrict__ dk, int64_t lddk,
                                       const __nv_bfloat16* __restrict__ qkv, int64_t ldqkv,
                                       const __nv_bfloat16* __restrict__ qw,
                                       const __nv_bfloat16* __restrict__ kw,
                                       const __nv_bfloat16* __restrict__ cosb,
                                       const __nv_bfloat16* __restrict__ sinb,
                                       const float* __restrict__ rstd,
                                       __nv_bfloat16* __restrict__ dqkv, int64_t lddqkv,
                                       float* __restrict__ dqw, float* __restrict__ dkw, int T, int S,
                                       int nq, int nkv, int items_per_block) {
  constexpr int D = 128;
  __shared__ float sdw[2][D];
  for (int i = threadIdx.x; i < 2 * D; i += blockDim.x) (&sdw[0][0])[i] = 0.f;
  __syncthreads();
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nh = nq + nkv;
  const int i0 = blockIdx.x * items_per_block;
  const int i1 = min(T * nh, i0 + items_per_block);
  float acc_q[4] = {0, 0, 0, 0}, acc_k[4] = {0, 0, 0, 0};
  for (int item = i0 + (threadIdx.x >> 5); item < i1; item += warps) {
    const int t = item / nh, h = item % nh;
    const bool is_q = h < nq;
    const __nv_bfloat16* g = is_q ? dq + (int64_t)t * lddq + (int64_t)h * D
                                  : dk + (int64_t)t * lddk + (int64_t)(h - nq) * D;
    uint2 graw = *reinterpret_cast<const uint2*>(g + lane * 4);
    float2 ga = unpack_bf16x2(graw.x), gb = unpack_bf16x2(graw.y);
    float gv[4] = {ga.x, ga.y, gb.x, gb.y};
    const int pos = t % S;
    uint2 craw = *reinterpret_cast<const uint2*>(cosb + (int64_t)pos * D + lane * 4);
    uint2 sraw = *reinterpret_cast<const uint2*>(sinb + (int64_t)pos * D + lane * 4);
    float2 ca = unpack_bf16x2(craw.x), cb = unpack_bf16x2(craw.y);
    float2 sa = unpack_bf16x2(sraw.x), sb = unpack_bf16x2(sraw.y);
    float cv[4] = {ca.x, ca.y, cb.x, cb.y}, sv[4] = {sa.x, sa.y, sb.x, sb.y};
    // dn[i] = g[i]*c[i] + (i<64 ? g[i+64]*s[i+64] : -g[i-64]*s[i-64])
    float gs[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) gs[j] = __shfl_xor_sync(0xffffffffu, gv[j] * sv[j], 16);
    const float sign = lane < 16 ? 1.f : -1.f;
    float dn[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) dn[j] = gv[j] * cv[j] + sign * gs[j];
    // norm backward
    const __nv_bfloat16* src = qkv + (int64_t)t * ldqkv + (int64_t)h * D + lane * 4;
    uint2 raw = *reinterpret_cast<const uint2*>(src);
    float2 a = unpack_bf16x2(raw.x), b = unpack_bf16x2(raw.y);
    float xv[4] = {a.x, a.y, b.x, b.y};
    uint2 wraw = *reinterpret_cast<const uint2*>((is_q ? qw : kw) + lane * 4);
    float2 wa = unpack_bf16x2(wraw.x), wb = unpack_bf16x2(wraw.y);
    float wv[4] = {wa.x, wa.y, wb.x, wb.y};
    const float r = rstd[(int64_t)t * nh + h];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) dot += dn[j] * wv[j] * xv[j] * r;
    dot = warp_sum(dot) / (float)D;
    float dx[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      dx[j] = r * (dn[j] * wv[j] - xv[j] * r * dot);
      const float contrib = dn[j] * bfr(xv[j] * r);
      if (is_q) acc_q[j] += contrib; else acc_k[j] += contrib;
    }
    __nv_bfloat16* d = dqkv + (int64_t)t * lddqkv + (int64_t)h * D + lane * 4;
    uint2 out;
    out.x = pack_bf16x2(dx[0], dx[1]);
    out.y = pack_bf16x2(dx[2], dx[3]);
    *reinterpret_cast<uint2*>(d) = out;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    atomicAdd(&sdw[0][lane * 4 + j], acc_q[j]);
    atomicAdd(&sdw[1][lane * 4 + j], acc_k[j]);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    if (dqw) atomicAdd(&dqw[i], sdw[0][i]);
    if (dkw) atomicAdd(&dkw[i], sdw[1][i]);
  }
}

}  // namespace

void rmsnorm_fwd(const void* x, int64_t ldx, const void* w, void* y, int64_t ldy, float* rstd,
                 int rows, int cols, float eps, cudaStream_t s) {
  PB_CHECK(cols % 8 == 0, "rmsnorm: cols must be a multiple of 8");
  const int warps = 8;
  rmsnorm_fwd_kernel<<<(rows + warps - 1) / warps, warps * 32, 0, s>>>(
      (const __nv_bfloat16*)x, ldx, (const __nv_bfloat16*)w, (__nv_bfloat16*)y, ldy, rstd, rows,
      cols, eps);
  PB_CUDA_CHECK(cudaGetLastError());
}

void rmsnorm_bwd(const void* dy, int64_t lddy, const void* x, int64_t ldx, const void* w,
                 const float* rstd, void* dx, int64_t lddx, float* dw_acc, int rows, int cols,
                 cudaStream_t s) {
  PB_CHECK(cols % 8 == 0, "rmsnorm: cols must be a multiple of 8");
  const int blocks = num_sms() * 2;
  const int rpb = (rows + blocks - 1) / blocks;
  const int grid = (rows + rpb - 1) / rpb;
  const size_t smem = (size_t)cols * sizeof(float);
  rmsnorm_bwd_kernel<<<grid, 256, smem, s>>>((const __nv_bfloat16*)dy, lddy, (const __nv_bfloat16*)x,
                                             ldx, (const __nv_bfloat16*)w, rstd, (__nv_bfloat16*)dx,
                                             lddx, dw_acc, rows, cols, rpb);
  PB_CUDA_CHECK(cudaGetLastError());
}

void qknorm_rope_fwd(const void* qkv, int64_t ldqkv, const void* qw, const void* kw,
                     const void* cos, const void* sin, void* q_out, int64_t ldq, void* k_out,
                     int64_t ldk, float* rstd, int T, int S, int nq, int nkv, int D, float eps,
                     cudaStream_t s) {
  PB_CHECK(D == 128, "qknorm_rope: head_dim 128 only");
  const int items = T * (nq + nkv);
  const int warps = 8;
  qknorm_rope_fwd_kernel<<<(items + warps - 1) / warps, warps * 32, 0, s>>>(
      (const __nv_bfloat16*)qkv, ldqkv, (const __nv_bfloat16*)qw, (const __nv_bfloat16*)kw,
      (const __nv_bfloat16*)cos, (const __nv_bfloat16*)sin, (__nv_bfloat16*)q_out, ldq,
      (__nv_bfloat16*)k_out, ldk, rstd, T, S, nq, nkv, eps);
  PB_CUDA_CHECK(cudaGetLastError());
}

void qknorm_rope_bwd(const void* dq, int64_t lddq, const void* dk, int64_t lddk, const void* qkv,
                     int64_t ldqkv, const void* qw, const void* kw, const void* cos,
                     const void* sin, const float* rstd, void* dqkv, int64_t lddqkv,
                     float* dqw_acc, float* dkw_acc, int T, int S, int nq, int nkv, int D,
                     cudaStream_t s) {
  PB_CHECK(D == 128, "qknorm_rope: head_dim 128 only");
  const int items = T * (nq + nkv);
  const int blocks = num_sms() * 4;
  const int ipb = (items + blocks - 1) / blocks;
  const int grid = (items + ipb - 1) / ipb;
  qknorm_rope_bwd_kernel<<<grid, 256, 0, s>>>(
      (const __nv_bfloat16*)dq, lddq, (const __nv_bfloat16*)dk, lddk, (const __nv_bfloat16*)qkv,
      ldqkv, (const __nv_bfloat16*)qw, (const __nv_bfloat16*)kw, (const __nv_bfloat16*)cos,
      (const __nv_bfloat16*)sin, rstd, (__nv_bfloat16*)dqkv, lddqkv, dqw_acc, dkw_acc, T, S, nq,
      nkv, ipb);
  PB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace pb
