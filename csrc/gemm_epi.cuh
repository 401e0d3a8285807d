// Fused GEMM epilogues shared by the one-CTA and CTA-pair GEMM kernels: one
// thread owns one output row of a tile and reads its accumulator row from
// TMEM 32 columns at a time.
#pragma once
#include <cuda_bf16.h>

#include "gemm.cuh"
#include "ptx.cuh"

namespace pb {
namespace gemm_detail {

struct EpiArgs {
  void* C;
  const void* R;
  int64_t ldc, ldr;
  float alpha;
  int epi;
  int64_t up_col;  // kEpiSwiGLU: column of the "up" half inside R
  ScatterArgs sc;  // sc.nranks > 0: kEpiStoreBf16 rows go to their owners
  int tma;         // CTA-pair kernel: stage tiles in shared memory and store them with TMA
  float* ws;       // kEpiSplitOrdered: fp32 running sums of the K slices
  int64_t ws_ld;
  int* cnt;        // kEpiSplitOrdered: per (tile, CTA) count of published epilogue warps
  int out_f32;     // kEpiSplitOrdered: C is fp32
  int accum;       // kEpiSplitOrdered: C += result
};

// TMA-store epilogue staging, per epilogue warp: three 32 x 32 bf16 boxes of
// 64-byte rows with the 64-byte swizzle (16-byte chunk q of row r sits at
// chunk q ^ ((r >> 1) & 3)), which keeps the row-per-thread writes of a warp
// free of bank conflicts.
constexpr int kEpiBox = 32;
constexpr int kEpiBoxBytes = kEpiBox * kEpiBox * 2;
// (8 KB: the SwiGLU epilogue's three bf16 boxes, or two 32 x 32 fp32 boxes)
constexpr int kEpiWarpBytes = 8192;
constexpr int kEpiBoxF32Bytes = kEpiBox * kEpiBox * 4;
static_assert(3 * kEpiBoxBytes <= kEpiWarpBytes && 2 * kEpiBoxF32Bytes <= kEpiWarpBytes, "epilogue staging");

// Output row pointer of row m for the bf16 store epilogue.
__device__ __forceinline__ __nv_bfloat16* out_row_bf16(const EpiArgs& ep, int m) {
  if (ep.sc.nranks == 0) return reinterpret_cast<__nv_bfloat16*>(ep.C) + (int64_t)m * ep.ldc;
  const int b = m / ep.sc.seq, s = m % ep.sc.seq;
  const int owner = s / ep.sc.seq_local;
  const int64_t local = (int64_t)b * ep.sc.seq_local + s % ep.sc.seq_local;
  return reinterpret_cast<__nv_bfloat16*>(ep.sc.peer[owner]) + (ep.sc.slot * ep.sc.slot_rows + local) * ep.ldc;
}

// silu(g) = g * sigmoid(g) with the fast reciprocal-based division.
__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

template <typename Fn>
__device__ __forceinline__ void for_cols(int n0, int N, Fn fn) {
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (n0 + j < N) fn(j);
}

// Store 32 consecutive values of one output row (vectorised when all 32
// columns are inside [0, N)).
__device__ __forceinline__ void store_row_bf16(__nv_bfloat16* dst, const float* v, int n0, int N) {
  if (n0 + 32 <= N) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 u;
      u.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
      u.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
      u.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
      u.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
      d4[q] = u;
    }
  } else {
    for_cols(n0, N, [&](int j) { dst[j] = __float2bfloat16(v[j]); });
  }
}

__device__ __forceinline__ void load_row_bf16(const __nv_bfloat16* src, float* v, int n0, int N) {
  if (n0 + 32 <= N) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 u = s4[q];
      float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
      v[q * 8 + 0] = a.x; v[q * 8 + 1] = a.y; v[q * 8 + 2] = b.x; v[q * 8 + 3] = b.y;
      v[q * 8 + 4] = c.x; v[q * 8 + 5] = c.y; v[q * 8 + 6] = d.x; v[q * 8 + 7] = d.y;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (n0 + j < N) ? __bfloat162float(src[j]) : 0.f;
  }
}

// Epilogue of one accumulator row: t_row = TMEM address of the row's first
// accumulator column, m = output row, n_base = first output column of the
// tile.  BN = accumulator columns (SwiGLU: [gate BN/2 | up BN/2]).
template <int BN, bool SWIGLU>
__device__ __forceinline__ void epilogue_row(const EpiArgs& ep, uint32_t t_row, int m, int M, int N, int n_base) {
  constexpr int BN_OUT = SWIGLU ? BN / 2 : BN;
  if (SWIGLU) {
#pragma unroll 1
    for (int c = 0; c < BN_OUT; c += 32) {
      float g[32], u[32];
      tmem_ld32(t_row + c, g);
      tmem_ld32(t_row + BN_OUT + c, u);
      tmem_wait_ld();
      const int n0 = n_base + c;
      if (m < M) {
        if (ep.R) {
          __nv_bfloat16* gu = reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(ep.R)) + (int64_t)m * ep.ldr;
          store_row_bf16(gu + n0, g, n0, N);
          store_row_bf16(gu + ep.up_col + n0, u, n0, N);
        }
        float h[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          // round the pre-activations to bf16 first so the forward matches a
          // bf16 gate/up GEMM followed by silu(g)*u
          const float gb = __bfloat162float(__float2bfloat16(g[j]));
          const float ub = __bfloat162float(__float2bfloat16(u[j]));
          h[j] = silu_f(gb) * ub;
        }
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(ep.C) + (int64_t)m * ep.ldc + n0;
        store_row_bf16(dst, h, n0, N);
      }
    }
    return;
  }
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    float v[32];
    tmem_ld32(t_row + c, v);
    tmem_wait_ld();
    const int n0 = n_base + c;
    if (m < M && n0 < N) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= ep.alpha;
      if (ep.epi == kEpiStoreBf16) {
        store_row_bf16(out_row_bf16(ep, m) + n0, v, n0, N);
      } else if (ep.epi == kEpiResidualBf16 || ep.epi == kEpiAccumBf16) {
        const __nv_bfloat16* src =
            ep.epi == kEpiResidualBf16
                ? reinterpret_cast<const __nv_bfloat16*>(ep.R) + (int64_t)m * ep.ldr + n0
                : reinterpret_cast<const __nv_bfloat16*>(ep.C) + (int64_t)m * ep.ldc + n0;
        float r[32];
        load_row_bf16(src, r, n0, N);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += r[j];
        store_row_bf16(reinterpret_cast<__nv_bfloat16*>(ep.C) + (int64_t)m * ep.ldc + n0, v, n0, N);
      } else if (ep.epi == kEpiAtomicF32) {
        float* dst = reinterpret_cast<float*>(ep.C) + (int64_t)m * ep.ldc + n0;
        if (n0 + 32 <= N) {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            atomicAdd(reinterpret_cast<float4*>(dst) + q, make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]));
        } else {
          for_cols(n0, N, [&](int j) { atomicAdd(dst + j, v[j]); });
        }
      } else {
        float* dst = reinterpret_cast<float*>(ep.C) + (int64_t)m * ep.ldc + n0;
        const bool accum = ep.epi == kEpiAccumF32;
        if (n0 + 32 <= N) {
          float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            float4 o = make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
            if (accum) {
              float4 p = d4[q];
              o.x += p.x; o.y += p.y; o.z += p.z; o.w += p.w;
            }
            d4[q] = o;
          }
        } else {
          for_cols(n0, N, [&](int j) { dst[j] = accum ? dst[j] + v[j] : v[j]; });
        }
      }
    }
  }
}

__device__ __forceinline__ void stage_row_swz64(uint8_t* box, int r, const float* v) {
  uint8_t* row = box + r * 64;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 u;
    u.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
    u.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
    u.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
    u.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
    *reinterpret_cast<uint4*>(row + ((q ^ ((r >> 1) & 3)) << 4)) = u;
  }
}

// TMA-store epilogue of one warp's 32 accumulator rows of a tile (the bf16
// store and SwiGLU epilogues): each 32-column chunk is read from TMEM,
// converted, written into this warp's staging boxes and stored with one TMA
// tile store per array (coalesced full lines, asynchronous).  `release` runs
// right after the tile's last TMEM read, so the MMA can reuse the
// accumulator while the stores drain.  y0 = the warp's first output row,
// n_base = the tile's first output column, N = output columns.
template <int BN, bool SWIGLU, typename Release>
__device__ __forceinline__ void epilogue_warp_tma(const EpiArgs& ep, const CUtensorMap* tmC, const CUtensorMap* tmR,
                                                  uint32_t t_row, uint8_t* stage, int lane, int y0, int M, int N,
                                                  int n_base, Release release) {
  constexpr int BN_OUT = SWIGLU ? BN / 2 : BN;
  const bool rows_in = y0 < M;
#pragma unroll 1
  for (int c = 0; c < BN_OUT; c += 32) {
    float a[32], b[32];
    tmem_ld32(t_row + c, a);
    if (SWIGLU) tmem_ld32(t_row + BN_OUT + c, b);
    tmem_wait_ld();
    if (c + 32 >= BN_OUT) release();
    const int n0 = n_base + c;
    const bool store = rows_in && n0 < N;
    uint8_t* box0;
    if (SWIGLU) {
      float h[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        // the pre-activations are stored as bf16: silu(g) * u of the rounded values
        a[j] = __bfloat162float(__float2bfloat16(a[j]));
        b[j] = __bfloat162float(__float2bfloat16(b[j]));
        h[j] = silu_f(a[j]) * b[j];
      }
      if (lane == 0) bulk_wait_group_read<0>();  // the previous chunk's stores have read the boxes
      __syncwarp();
      box0 = stage;
      if (store) {
        stage_row_swz64(stage, lane, h);
        if (ep.R) {
          stage_row_swz64(stage + kEpiBoxBytes, lane, a);
          stage_row_swz64(stage + 2 * kEpiBoxBytes, lane, b);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) a[j] *= ep.alpha;
      // two boxes alternate: chunk c may be staged while chunk c - 1 drains
      box0 = stage + ((c >> 5) & 1) * kEpiBoxBytes;
      if (lane == 0) bulk_wait_group_read<1>();
      __syncwarp();
      if (store) stage_row_swz64(box0, lane, a);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0 && store) {
      tma_store_2d(tmC, box0, n0, y0);
      if (SWIGLU && ep.R) {
        tma_store_2d(tmR, stage + kEpiBoxBytes, n0, y0);
        tma_store_2d(tmR, stage + 2 * kEpiBoxBytes, (int)ep.up_col + n0, y0);
      }
    }
    if (lane == 0) bulk_commit_group();
  }
}

// One row of a 32 x 32 fp32 box of 128-byte rows with the 128-byte swizzle:
// 16-byte chunk q of row r sits at chunk q ^ (r & 7).
__device__ __forceinline__ void stage_row_swz128_f32(uint8_t* box, int r, const float* v) {
  uint8_t* row = box + r * 128;
#pragma unroll
  for (int q = 0; q < 8; ++q)
    *reinterpret_cast<float4*>(row + ((q ^ (r & 7)) << 4)) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}

// fp32 store epilogue through TMA tile stores (ep.tma == 2): the tile of K
// slice `slab` goes to slab `slab` of the [slabs, M, ldc] output (the split-K
// partials that sum_slices adds in slice order; slab 0 of 1 otherwise).  The
// tensor map's per-slab row bound keeps the rows past M of a partial tile out
// of the next slab.
template <int BN, typename Release>
__device__ __forceinline__ void epilogue_warp_tma_f32(const EpiArgs& ep, const CUtensorMap* tmC, uint32_t t_row,
                                                      uint8_t* stage, int lane, int y0, int M, int N, int n_base,
                                                      int slab, Release release) {
  const bool rows_in = y0 < M;
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    float a[32];
    tmem_ld32(t_row + c, a);
    tmem_wait_ld();
    if (c + 32 >= BN) release();
    const int n0 = n_base + c;
    const bool store = rows_in && n0 < N;
#pragma unroll
    for (int j = 0; j < 32; ++j) a[j] *= ep.alpha;
    uint8_t* box = stage + ((c >> 5) & 1) * kEpiBoxF32Bytes;
    if (lane == 0) bulk_wait_group_read<1>();
    __syncwarp();
    if (store) stage_row_swz128_f32(box, lane, a);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0 && store) tma_store_3d(tmC, box, n0, y0, slab);
    if (lane == 0) bulk_commit_group();
  }
}

}  // namespace gemm_detail
}  // namespace pb
