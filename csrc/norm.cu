// RMSNorm and the fused per-head QK-RMSNorm + rotate-half RoPE.
//
// Numerics follow HF Qwen3 (transformers/models/qwen3/modeling_qwen3.py,
// Qwen3RMSNorm and apply_rotary_pos_emb): the normalisation runs in fp32,
// the normalised value is rounded to bf16 before the weight multiply, and the
// RoPE products / sum are rounded to bf16 the way the bf16 eager ops round.
// The reference gets these ops from HF (parallel/parallel/engine/
// model_loading.py:17-35); here each is one memory-bound pass.
#include <cuda_bf16.h>

#include <algorithm>
#include <mutex>

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
  pdl_prologue();
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

// Block of 8 warps handles `rows_per_block` rows; dw partials in a per-warp
// shared-memory slice (a lane owns its 8-column groups: no atomics), summed in
// warp order into row blockIdx.x of the block-partial matrix dw [grid, cols].
__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, int64_t lddy,
                                   const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                   const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
                                   __nv_bfloat16* __restrict__ dx, int64_t lddx, float* __restrict__ dw,
                                   int rows, int cols, int rows_per_block,
                                   const __nv_bfloat16* __restrict__ dres, int64_t lddres) {
  pdl_prologue();
  extern __shared__ float sdw_all[];  // [warps][cols]
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  float* sdw = sdw_all + (threadIdx.x >> 5) * cols;
  for (int c = lane; c < cols; c += 32) sdw[c] = 0.f;
  __syncwarp();
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
        sdw[c + j] += gv[j] * bfr(xh);
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
      if (dres) {
        float rv[8];
        load8(dres + (int64_t)row * lddres + c, rv);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] += rv[j];
      }
      store8(dxr + c, o);
    }
  }
  __syncthreads();
  if (dw)
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
      float t = 0.f;
      for (int w8 = 0; w8 < warps; ++w8) t += sdw_all[w8 * cols + c];
      dw[(int64_t)blockIdx.x * cols + c] = t;
    }
}

// Register-resident variant: cols == CH * 256; lane owns CH chunks of 8
// columns; dw partials stay in registers until one shared-memory reduction
// per warp.  Optionally adds a residual-stream gradient (dres) into dx, which
// fuses the add autograd would otherwise run for "x -> norm(x) and x -> +".
template <int CH>
__global__ void __launch_bounds__(256, 2) rmsnorm_bwd_reg_kernel(
    const __nv_bfloat16* __restrict__ dy, int64_t lddy, const __nv_bfloat16* __restrict__ x, int64_t ldx,
    const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd, const __nv_bfloat16* __restrict__ dres,
    int64_t lddres, __nv_bfloat16* __restrict__ dx, int64_t lddx, float* __restrict__ dw, int rows,
    int rows_per_block) {
  pdl_prologue();
  // One warp per row, all of the row's loads (x, dy, dres) issued before the
  // reduction and kept packed in registers, so a row costs one DRAM round
  // trip.  Weight-grad partials live in a per-warp shared-memory slice (each
  // lane owns its columns: no atomics) and are summed once per block.
  constexpr int cols = CH * 256;
  extern __shared__ float sdw[];  // [warps][cols]
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  float* mine = sdw + (threadIdx.x >> 5) * cols;
  if (dw) {
#pragma unroll
    for (int k = 0; k < CH; ++k) {
      float4* d4 = reinterpret_cast<float4*>(mine + k * 256 + lane * 8);
      d4[0] = d4[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(rows, r0 + rows_per_block);
  for (int row = r0 + (threadIdx.x >> 5); row < r1; row += warps) {
    const float r = rstd[row];
    uint4 xp[CH], gp[CH], rp[CH];
#pragma unroll
    for (int k = 0; k < CH; ++k) {
      const int c = k * 256 + lane * 8;
      xp[k] = *reinterpret_cast<const uint4*>(x + (int64_t)row * ldx + c);
      gp[k] = *reinterpret_cast<const uint4*>(dy + (int64_t)row * lddy + c);
      if (dres) rp[k] = *reinterpret_cast<const uint4*>(dres + (int64_t)row * lddres + c);
    }
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < CH; ++k) {
      const uint32_t* xu = &xp[k].x;
      const uint32_t* gu = &gp[k].x;
      const uint4 wq = __ldg(reinterpret_cast<const uint4*>(w + k * 256 + lane * 8));  // L1-resident
      const uint32_t* wu = &wq.x;
      float a[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 xv = unpack_bf16x2(xu[q]), gv = unpack_bf16x2(gu[q]), wv = unpack_bf16x2(wu[q]);
        const float xh0 = xv.x * r, xh1 = xv.y * r;
        dot += gv.x * wv.x * xh0 + gv.y * wv.y * xh1;
        a[2 * q] = gv.x * bfr(xh0);
        a[2 * q + 1] = gv.y * bfr(xh1);
      }
      if (dw) {
        float4* d4 = reinterpret_cast<float4*>(mine + k * 256 + lane * 8);
        float4 u0 = d4[0], u1 = d4[1];
        u0.x += a[0]; u0.y += a[1]; u0.z += a[2]; u0.w += a[3];
        u1.x += a[4]; u1.y += a[5]; u1.z += a[6]; u1.w += a[7];
        d4[0] = u0;
        d4[1] = u1;
      }
    }
    dot = warp_sum(dot) / (float)cols;
#pragma unroll
    for (int k = 0; k < CH; ++k) {
      const int c = k * 256 + lane * 8;
      const uint32_t* xu = &xp[k].x;
      const uint32_t* gu = &gp[k].x;
      const uint4 wq = __ldg(reinterpret_cast<const uint4*>(w + c));
      const uint32_t* wu = &wq.x;
      const uint32_t* ru = &rp[k].x;
      uint4 o;
      uint32_t* ou = &o.x;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 xv = unpack_bf16x2(xu[q]), gv = unpack_bf16x2(gu[q]), wv = unpack_bf16x2(wu[q]);
        float o0 = r * (gv.x * wv.x - xv.x * r * dot), o1 = r * (gv.y * wv.y - xv.y * r * dot);
        if (dres) {
          const float2 rv = unpack_bf16x2(ru[q]);
          o0 += rv.x;
          o1 += rv.y;
        }
        ou[q] = pack_bf16x2(o0, o1);
      }
      *reinterpret_cast<uint4*>(dx + (int64_t)row * lddx + c) = o;
    }
  }
  if (dw) {
    __syncthreads();
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
      float t = 0.f;
      for (int w8 = 0; w8 < warps; ++w8) t += sdw[w8 * cols + c];
      dw[(int64_t)blockIdx.x * cols + c] = t;  // block partial, summed in block order later
    }
  }
}

// Half a warp per (token, head); D == 128: lane owns 8 consecutive elements
// (16-byte accesses).  RoPE pairs element i with i +- 64, i.e. lane l with
// lane l ^ 8 inside the same half warp.
__device__ __forceinline__ float half_sum(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void qknorm_rope_fwd_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ldqkv,
                                       const __nv_bfloat16* __restrict__ qw,
                                       const __nv_bfloat16* __restrict__ kw,
                                       const __nv_bfloat16* __restrict__ cosb,
                                       const __nv_bfloat16* __restrict__ sinb,
                                       __nv_bfloat16* __restrict__ q_out, int64_t ldq,
                                       __nv_bfloat16* __restrict__ k_out, int64_t ldk,
                                       float* __restrict__ rstd, int T, int S, int nq, int nkv, float eps) {
  pdl_prologue();
  // A half warp per unit = (token, U consecutive heads): the token's cos / sin
  // rows are loaded once and all U input rows are issued before the first
  // reduction (one DRAM round trip per unit).  The bf16 products / sums of the
  // reference's op-by-op bf16 arithmetic run as packed bf16x2 instructions: a
  // product of two bf16 values is exact in fp32, so the packed multiply rounds
  // exactly like fp32-multiply-then-round.
  constexpr int D = 128;
  constexpr int U = 4;
  const int lane = threadIdx.x & 31;
  const int hl = lane & 15;
  const int nh = nq + nkv;
  const int groups = (nh + U - 1) / U;
  const int64_t total = (int64_t)T * groups;
  int64_t unit = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 2 + (lane >> 4);
  const bool unit_ok = unit < total;
  if (!unit_ok) unit = total - 1;  // keep all lanes in the shuffles
  const int t = (int)(unit / groups), h0 = (int)(unit % groups) * U;
  const int pos = t % S;
  uint4 xv[U];
#pragma unroll
  for (int u = 0; u < U; ++u)
    xv[u] = *reinterpret_cast<const uint4*>(qkv + (int64_t)t * ldqkv + (int64_t)min(h0 + u, nh - 1) * D + hl * 8);
  const uint4 qwv = __ldg(reinterpret_cast<const uint4*>(qw + hl * 8));
  const uint4 kwv = __ldg(reinterpret_cast<const uint4*>(kw + hl * 8));
  const uint4 cv = __ldg(reinterpret_cast<const uint4*>(cosb + (int64_t)pos * D + hl * 8));
  uint4 sv = __ldg(reinterpret_cast<const uint4*>(sinb + (int64_t)pos * D + hl * 8));
  // rotate_half: [-x2, x1] -> the first half of the lanes takes -sin
  if (hl < 8) {
    sv.x ^= 0x80008000u; sv.y ^= 0x80008000u; sv.z ^= 0x80008000u; sv.w ^= 0x80008000u;
  }
  const __nv_bfloat162* c2 = reinterpret_cast<const __nv_bfloat162*>(&cv);
  const __nv_bfloat162* s2 = reinterpret_cast<const __nv_bfloat162*>(&sv);
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int h = h0 + u;
    const bool valid = unit_ok && h < nh;
    const bool is_q = h < nq;
    const uint32_t* x32 = &xv[u].x;
    float xf[8];
    float ss = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = unpack_bf16x2(x32[q]);
      xf[2 * q] = f.x;
      xf[2 * q + 1] = f.y;
      ss += f.x * f.x + f.y * f.y;
    }
    ss = half_sum(ss);
    const float r = rsqrtf(ss / (float)D + eps);
    const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(is_q ? &qwv : &kwv);
    uint4 ov;
    uint32_t* o32 = &ov.x;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const __nv_bfloat162 xh = __floats2bfloat162_rn(xf[2 * q] * r, xf[2 * q + 1] * r);
      const __nv_bfloat162 n = __hmul2(w2[q], xh);
      const uint32_t nu = *reinterpret_cast<const uint32_t*>(&n);
      const uint32_t pu = __shfl_xor_sync(0xffffffffu, nu, 8);
      const __nv_bfloat162 pn = *reinterpret_cast<const __nv_bfloat162*>(&pu);
      const __nv_bfloat162 o = __hadd2(__hmul2(n, c2[q]), __hmul2(pn, s2[q]));
      o32[q] = *reinterpret_cast<const uint32_t*>(&o);
    }
    if (!valid) continue;
    if (hl == 0) rstd[(int64_t)t * nh + h] = r;
    __nv_bfloat16* dst = is_q ? q_out + (int64_t)t * ldq + (int64_t)h * D
                              : k_out + (int64_t)t * ldk + (int64_t)(h - nq) * D;
    *reinterpret_cast<uint4*>(dst + hl * 8) = ov;
  }
}

// Backward of the above; q/k norm weight grads: per-lane registers, one slice
// per half warp in shared memory, summed in slot order into row blockIdx.x of
// the block-partial matrix [grid, 2 * D] (q weights, then k weights).
template <int U, int MINB>
__global__ void __launch_bounds__(256, MINB) qknorm_rope_bwd_kernel(const __nv_bfloat16* __restrict__ dq, int64_t lddq,
                                       const __nv_bfloat16* __restrict__ dk, int64_t lddk,
                                       const __nv_bfloat16* __restrict__ qkv, int64_t ldqkv,
                                       const __nv_bfloat16* __restrict__ qw,
                                       const __nv_bfloat16* __restrict__ kw,
                                       const __nv_bfloat16* __restrict__ cosb,
                                       const __nv_bfloat16* __restrict__ sinb,
                                       const float* __restrict__ rstd,
                                       __nv_bfloat16* __restrict__ dqkv, int64_t lddqkv,
                                       float* __restrict__ dqw, float* __restrict__ dkw, int T, int S,
                                       int nq, int nkv, int units_per_block) {
  pdl_prologue();
  // A half warp per unit = (token, group of U consecutive heads): the token's
  // cos / sin rows are loaded once per unit and every head's gradient and
  // input rows (2 x 16 bytes per lane per head) are issued before the first
  // shuffle, so a unit costs one DRAM round trip with 2U + 2 loads in flight.
  constexpr int D = 128;
  __shared__ float sdw[16][2][D];  // [half-warp slot][q / k][column]
  const int lane = threadIdx.x & 31;
  const int hl = lane & 15;
  const int slots = (blockDim.x >> 5) * 2;
  const int slot = (threadIdx.x >> 5) * 2 + (lane >> 4);
  const int nh = nq + nkv;
  const int groups = (nh + U - 1) / U;
  const int64_t total = (int64_t)T * groups;
  const int64_t u0 = (int64_t)blockIdx.x * units_per_block;
  const int64_t u1 = min(total, u0 + units_per_block);
  float qw_r[8], kw_r[8], acc_q[8], acc_k[8];
  load8(qw + hl * 8, qw_r);
  load8(kw + hl * 8, kw_r);
#pragma unroll
  for (int j = 0; j < 8; ++j) acc_q[j] = acc_k[j] = 0.f;
  const float sign = hl < 8 ? 1.f : -1.f;
  // every lane iterates the same number of times so shuffles stay converged
  const int64_t iters = (u1 - u0 + slots - 1) / slots;
  for (int64_t it = 0; it < iters; ++it) {
    int64_t unit = u0 + it * slots + slot;
    const bool unit_ok = unit < u1;
    if (!unit_ok) unit = u1 - 1;
    const int t = (int)(unit / groups), h0 = (int)(unit % groups) * U;
    const int pos = t % S;
    const uint4 cp = *reinterpret_cast<const uint4*>(cosb + (int64_t)pos * D + hl * 8);
    const uint4 sp = *reinterpret_cast<const uint4*>(sinb + (int64_t)pos * D + hl * 8);
    uint4 gp[U], xp[U];
    float rr[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int h = min(h0 + u, nh - 1);
      const bool is_q = h < nq;
      gp[u] = *reinterpret_cast<const uint4*>(is_q ? dq + (int64_t)t * lddq + (int64_t)h * D + hl * 8
                                                   : dk + (int64_t)t * lddk + (int64_t)(h - nq) * D + hl * 8);
      xp[u] = *reinterpret_cast<const uint4*>(qkv + (int64_t)t * ldqkv + (int64_t)h * D + hl * 8);
      rr[u] = rstd[(int64_t)t * nh + h];
    }
    float cv[8], sv[8];
    {
      const uint32_t* c32 = &cp.x;
      const uint32_t* s32 = &sp.x;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 c = unpack_bf16x2(c32[q]), d = unpack_bf16x2(s32[q]);
        cv[2 * q] = c.x; cv[2 * q + 1] = c.y;
        sv[2 * q] = d.x; sv[2 * q + 1] = d.y;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int h = h0 + u;
      const bool valid = unit_ok && h < nh;
      const bool is_q = h < nq;
      float gv[8], xv[8];
      const uint32_t* g32 = &gp[u].x;
      const uint32_t* x32 = &xp[u].x;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 a = unpack_bf16x2(g32[q]), b = unpack_bf16x2(x32[q]);
        gv[2 * q] = a.x; gv[2 * q + 1] = a.y;
        xv[2 * q] = b.x; xv[2 * q + 1] = b.y;
      }
      // dn[i] = g[i]*c[i] + (i<64 ? g[i+64]*s[i+64] : -g[i-64]*s[i-64])
      float dn[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) dn[j] = gv[j] * cv[j] + sign * __shfl_xor_sync(0xffffffffu, gv[j] * sv[j], 8);
      const float* wv = is_q ? qw_r : kw_r;
      const float r = rr[u];
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) dot += dn[j] * wv[j] * xv[j] * r;
      dot = half_sum(dot) / (float)D;
      if (!valid) continue;
      float dx[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        dx[j] = r * (dn[j] * wv[j] - xv[j] * r * dot);
        const float contrib = dn[j] * bfr(xv[j] * r);
        if (is_q) acc_q[j] += contrib; else acc_k[j] += contrib;
      }
      store8(dqkv + (int64_t)t * lddqkv + (int64_t)h * D + hl * 8, dx);
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    sdw[slot][0][hl * 8 + j] = acc_q[j];
    sdw[slot][1][hl * 8 + j] = acc_k[j];
  }
  __syncthreads();
  if (dqw != nullptr) {  // dqw: block partials [grid, 2 * D]
    for (int i = threadIdx.x; i < 2 * D; i += blockDim.x) {
      float t = 0.f;
      for (int sl = 0; sl < slots; ++sl) t += sdw[sl][i / D][i % D];
      dqw[(int64_t)blockIdx.x * 2 * D + i] = t;
    }
  }
}

}  // namespace

void rmsnorm_fwd(const void* x, int64_t ldx, const void* w, void* y, int64_t ldy, float* rstd,
                 int rows, int cols, float eps, cudaStream_t s) {
  PB_CHECK(cols % 8 == 0, "rmsnorm: cols must be a multiple of 8");
  const int warps = 8;
  launch_k(rmsnorm_fwd_kernel, (rows + warps - 1) / warps, warps * 32, 0, s,
      (const __nv_bfloat16*)x, ldx, (const __nv_bfloat16*)w, (__nv_bfloat16*)y, ldy, rstd, rows,
      cols, eps);
  PB_CUDA_CHECK(cudaGetLastError());
}

int rmsnorm_bwd_grid(int rows) {
  const int blocks = num_sms() * 2;  // one wave: two 256-thread blocks per SM
  const int rpb = (std::max(rows, 1) + blocks - 1) / blocks;
  return (std::max(rows, 1) + rpb - 1) / rpb;
}

void rmsnorm_bwd(const void* dy, int64_t lddy, const void* x, int64_t ldx, const void* w,
                 const float* rstd, void* dx, int64_t lddx, float* dw_part, int rows, int cols,
                 cudaStream_t s, const void* dres, int64_t lddres) {
  PB_CHECK(cols % 8 == 0, "rmsnorm: cols must be a multiple of 8");
  const int grid = rmsnorm_bwd_grid(rows);
  const int rpb = (std::max(rows, 1) + grid - 1) / grid;
  float* dw_acc = dw_part;
  const size_t smem = (size_t)8 * cols * sizeof(float);  // per-warp partial slices
  PB_CHECK(smem <= 227 * 1024, "rmsnorm bwd: rows wider than 7264 columns");
  if (smem > 48 * 1024) {
    static std::mutex mu;
    static bool attr_set[64] = {false};
    int dev = 0;
    PB_CUDA_CHECK(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    if (!attr_set[dev & 63]) {
      PB_CUDA_CHECK(cudaFuncSetAttribute(rmsnorm_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
      attr_set[dev & 63] = true;
    }
  }
  const size_t smem_reg = (size_t)8 * cols * sizeof(float);  // per-warp partials (<= 48 KB)
  if (cols % 256 == 0 && cols <= 1536) {  // wider rows would spill: generic kernel
#define PB_RMS_BWD(CH)                                                                                     \
  case CH:                                                                                                \
    launch_k(rmsnorm_bwd_reg_kernel<CH>, grid, 256, smem_reg, s,                                                 \
        (const __nv_bfloat16*)dy, lddy, (const __nv_bfloat16*)x, ldx, (const __nv_bfloat16*)w, rstd,      \
        (const __nv_bfloat16*)dres, lddres, (__nv_bfloat16*)dx, lddx, dw_acc, rows, rpb);                 \
    break;
    switch (cols / 256) {
      PB_RMS_BWD(1) PB_RMS_BWD(2) PB_RMS_BWD(3) PB_RMS_BWD(4) PB_RMS_BWD(5) PB_RMS_BWD(6)
    }
#undef PB_RMS_BWD
    PB_CUDA_CHECK(cudaGetLastError());
    return;
  }
  launch_k(rmsnorm_bwd_kernel, grid, 256, smem, s, (const __nv_bfloat16*)dy, lddy, (const __nv_bfloat16*)x,
                                             ldx, (const __nv_bfloat16*)w, rstd, (__nv_bfloat16*)dx,
                                             lddx, dw_acc, rows, cols, rpb, (const __nv_bfloat16*)dres,
                                             lddres);
  PB_CUDA_CHECK(cudaGetLastError());
}

void qknorm_rope_fwd(const void* qkv, int64_t ldqkv, const void* qw, const void* kw,
                     const void* cos, const void* sin, void* q_out, int64_t ldq, void* k_out,
                     int64_t ldk, float* rstd, int T, int S, int nq, int nkv, int D, float eps,
                     cudaStream_t s) {
  PB_CHECK(D == 128, "qknorm_rope: head_dim 128 only");
  const int units = T * ((nq + nkv + 3) / 4);  // (token, 4 heads) units
  const int per_block = 16;                    // 8 warps x 2 half-warps
  launch_k(qknorm_rope_fwd_kernel, (units + per_block - 1) / per_block, 256, 0, s,
      (const __nv_bfloat16*)qkv, ldqkv, (const __nv_bfloat16*)qw, (const __nv_bfloat16*)kw,
      (const __nv_bfloat16*)cos, (const __nv_bfloat16*)sin, (__nv_bfloat16*)q_out, ldq,
      (__nv_bfloat16*)k_out, ldk, rstd, T, S, nq, nkv, eps);
  PB_CUDA_CHECK(cudaGetLastError());
}

// Unit width U (heads per half-warp unit) and resident blocks per SM of the
// backward.  Measured on B200 at 8192 tokens x 24 heads: 4 x 2 blocks 43.3 us;
// narrower units with more blocks spill registers and lose (2 x 3: 57.5 us,
// 2 x 4: 67.8 us, 1 x 6: 83.5 us).
struct QknBwdCfg {
  int u, blocks;
};

QknBwdCfg qknorm_bwd_cfg() { return {4, 2}; }

int qknorm_rope_bwd_grid(int T, int nq, int nkv) {
  const QknBwdCfg c = qknorm_bwd_cfg();
  const int units = std::max(1, T * ((nq + nkv + c.u - 1) / c.u));  // (token, U heads) units
  const int blocks = num_sms() * c.blocks;                          // one wave
  const int ipb = (units + blocks - 1) / blocks;
  return (units + ipb - 1) / ipb;
}

void qknorm_rope_bwd(const void* dq, int64_t lddq, const void* dk, int64_t lddk, const void* qkv,
                     int64_t ldqkv, const void* qw, const void* kw, const void* cos,
                     const void* sin, const float* rstd, void* dqkv, int64_t lddqkv,
                     float* dw_part, int T, int S, int nq, int nkv, int D, cudaStream_t s) {
  PB_CHECK(D == 128, "qknorm_rope: head_dim 128 only");
  const QknBwdCfg c = qknorm_bwd_cfg();
  const int units = T * ((nq + nkv + c.u - 1) / c.u);
  const int grid = qknorm_rope_bwd_grid(T, nq, nkv);
  const int ipb = (std::max(units, 1) + grid - 1) / grid;
  launch_k(qknorm_rope_bwd_kernel<4, 2>, grid, 256, 0, s,
      (const __nv_bfloat16*)dq, lddq, (const __nv_bfloat16*)dk, lddk, (const __nv_bfloat16*)qkv,
      ldqkv, (const __nv_bfloat16*)qw, (const __nv_bfloat16*)kw, (const __nv_bfloat16*)cos,
      (const __nv_bfloat16*)sin, rstd, (__nv_bfloat16*)dqkv, lddqkv, dw_part, nullptr, T, S, nq,
      nkv, ipb);
  PB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace pb
