// Device-resident mixture-of-experts routing: every size the expert GEMMs and
// the token exchange need is computed on the GPU, so an MoE layer runs
// without a host synchronisation (and can be captured in a CUDA graph).
//
// Layout.  The rows an expert owner receives are stored expert-major in one
// padded matrix: local expert j owns rows [off[j], off[j] + rows_j) with
// rows_j = 128 * ceil(max(cnt_j, 1) / 128), where cnt_j counts the routes of
// every source rank to j.  Within expert j, source rank s's routes come
// before rank s+1's, and each rank's routes keep their flat (token * k + slot)
// order.  Rows past cnt_j are zero.  Every expert has at least one tile, so
// the weight-gradient GEMM never meets an empty K range and every row of the
// padded matrix is written by the forward GEMMs (zeros in, zeros out).
//
//   moe_hist       route histogram of this rank over the global experts,
//                  written as row `row` of an fp32 [rows, E] matrix whose
//                  other rows are zeroed (an all-reduce then turns it into the
//                  all-gather of every rank's histogram).
//   moe_plan       one CTA: the padded layout of every owner, this rank's
//                  destination (owner, row) of each route by a stable counting
//                  sort (warp match + per-warp prefix sums, 1024 routes per
//                  pass), and this rank's own layout as an owner: counts,
//                  offsets, the K range of each expert's weight-gradient
//                  product and the tile -> expert map of the row GEMMs.
//   moe_dispatch   one warp per route: hidden row of the route's token stored
//                  into the owner's receive matrix (peer memory).
//   moe_copy_pad   padded matrix rows: valid rows copied out of the receive
//                  matrix (or left in place), padding rows zeroed.
//   moe_combine    one warp per token: out[t] = sum_k w[t,k] * Y_owner[row]
//                  read from the owners (fp32 sums; w == nullptr: plain sum),
//                  optionally keeping each pulled row for the backward.
//   moe_combine_bwd one warp per route: dw[t,k] = <dout[t], y_route>, and
//                  w[t,k] * dout[t] stored into the owner's gradient matrix.
//
// Routes that are not kept (another rank's expert in the replicated-token
// layout) get owner -1 and are skipped by every kernel.
//
// Reference counterpart: the host-synchronised sort / count exchange /
// index_select of parallel/parallel/engine/model_parallel/token_dispatch.py:
// 86-174 and the HF grouped expert path it feeds (argsort / histc / cumsum).
#include <cuda_bf16.h>
#include <stdint.h>

#include "comm.cuh"
#include "host_util.h"
#include "moe.cuh"
#include "ptx.cuh"

namespace pb {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kPlanWarps = kPlanThreads / 32;

__global__ void __launch_bounds__(1024) moe_hist_kernel(const int64_t* __restrict__ topi, int64_t n_routes, int E,
                                                        float* __restrict__ mat, int mat_rows, int row) {
  pdl_prologue();
  extern __shared__ int hist[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  for (int64_t i = threadIdx.x; i < n_routes; i += blockDim.x) {
    const int64_t e = topi[i];
    if (e >= 0 && e < E) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  for (int r = 0; r < mat_rows; ++r)
    for (int e = threadIdx.x; e < E; e += blockDim.x) mat[(int64_t)r * E + e] = r == row ? (float)hist[e] : 0.f;
}

__device__ __forceinline__ int round128(int n) { return ((max(n, 1) + 127) / 128) * 128; }

// shared layout of moe_plan (E <= kMoeMaxExperts)
struct PlanSmem {
  int base[kMoeMaxExperts + 1];          // first destination row of this rank's routes to expert e
  int running[kMoeMaxExperts + 1];       // routes to e placed so far
  int wcnt[kPlanWarps][kMoeMaxExperts + 1];
  int own_total;
};

__global__ void __launch_bounds__(kPlanThreads, 1)
    moe_plan_kernel(const int64_t* __restrict__ topi, int64_t n_routes, const float* __restrict__ mat, int mat_rows,
                    int my_row, int E, int E_loc, int ep_rank, int local_only, int32_t* __restrict__ route_owner,
                    int32_t* __restrict__ route_row, int32_t* __restrict__ own_cnt, int32_t* __restrict__ own_off,
                    int2* __restrict__ krange, int32_t* __restrict__ tile_expert, int32_t* __restrict__ n_tiles,
                    int tiles_cap, int* err) {
  pdl_prologue();
  __shared__ PlanSmem sm;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int owners = E / E_loc;
  // 1. every owner's padded layout (one thread per owner, serial over its experts)
  //    and the start of this rank's block inside each expert
  if (tid < owners) {
    const int d = tid;
    int off = 0;
    for (int j = 0; j < E_loc; ++j) {
      const int e = d * E_loc + j;
      int total = 0, before = 0;
      for (int s = 0; s < mat_rows; ++s) {
        const int c = (int)mat[(int64_t)s * E + e];
        total += c;
        if (s < my_row) before += c;
      }
      sm.base[e] = off + before;
      if (d == ep_rank) {
        own_cnt[j] = total;
        own_off[j] = off;
        krange[j] = make_int2(off, off + ((max(total, 1) + 63) / 64) * 64);
      }
      off += round128(total);
    }
    if (d == ep_rank) sm.own_total = off;
  }
  for (int e = tid; e <= E; e += kPlanThreads) sm.running[e] = 0;
  __syncthreads();
  // 2. this rank as an owner: tile -> local expert map of the padded matrix
  if (warp == 0) {
    const int tiles = sm.own_total / 128;
    if (lane == 0) {
      if (tiles > tiles_cap) record_error(err, kErrMoeCapacity);
      *n_tiles = min(tiles, tiles_cap);
    }
    for (int j = 0; j < E_loc; ++j) {
      const int t0 = own_off[j] / 128, t1 = t0 + round128(own_cnt[j]) / 128;
      for (int t = t0 + lane; t < t1 && t < tiles_cap; t += 32) tile_expert[t] = j;
    }
  }
  // 3. stable counting sort of this rank's routes by destination expert
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int64_t first = 0; first < n_routes; first += kPlanThreads) {
    for (int k = tid; k < kPlanWarps * (kMoeMaxExperts + 1); k += kPlanThreads) (&sm.wcnt[0][0])[k] = 0;
    __syncthreads();
    const int64_t i = first + tid;
    int key = E;  // bucket of routes that are not kept
    int owner = -1;
    if (i < n_routes) {
      const int64_t e = topi[i];
      if (e >= 0 && e < E) {
        owner = (int)(e / E_loc);
        if (!local_only || owner == ep_rank) key = (int)e;
        else owner = -1;
      }
    }
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    const int rank_in_warp = __popc(peers & lt_mask);
    if (rank_in_warp == 0) sm.wcnt[warp][key] = __popc(peers);
    __syncthreads();
    for (int k = tid; k <= E; k += kPlanThreads) {  // exclusive scan over the warps, per expert
      int s = sm.running[k];
      for (int w = 0; w < kPlanWarps; ++w) {
        const int c = sm.wcnt[w][k];
        sm.wcnt[w][k] = s;
        s += c;
      }
      sm.running[k] = s;
    }
    __syncthreads();
    if (i < n_routes) {
      if (key < E) {
        route_owner[i] = local_only ? 0 : owner;
        route_row[i] = sm.base[key] + sm.wcnt[warp][key] + rank_in_warp;
      } else {
        route_owner[i] = -1;
        route_row[i] = -1;
      }
    }
    __syncthreads();
  }
}

// one warp per route: the token's hidden row into the owner's receive matrix
__global__ void moe_dispatch_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int K,
                                    const int32_t* __restrict__ owner, const int32_t* __restrict__ row,
                                    PeerBases dst, int64_t ldd, int64_t vecs, int64_t n_routes) {
  pdl_prologue();
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= n_routes) return;
  const int r = owner[i];
  if (r < 0 || r >= kMaxPeers) return;
  const uint4* s4 = reinterpret_cast<const uint4*>(x + (i / K) * ldx);
  uint4* d4 = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(dst.p[r]) + (int64_t)row[i] * ldd);
  for (int64_t v = lane; v < vecs; v += 32) d4[v] = s4[v];
}

// rows of the padded matrix: blockIdx.x covers rows [16*b, 16*b + 16)
__global__ void moe_copy_pad_kernel(const __nv_bfloat16* __restrict__ src, int64_t lds, __nv_bfloat16* __restrict__ dst,
                                    int64_t ldd, int64_t vecs, const int32_t* __restrict__ tile_expert,
                                    const int32_t* __restrict__ n_tiles, const int32_t* __restrict__ own_cnt,
                                    const int32_t* __restrict__ own_off) {
  pdl_prologue();
  const int64_t row0 = (int64_t)blockIdx.x * 16;
  const int tiles = *n_tiles;
  if (row0 >= (int64_t)tiles * 128) return;
  const int j = tile_expert[row0 / 128];
  const int lo = own_off[j], hi = own_off[j] + own_cnt[j];
  const bool in_place = src == dst && lds == ldd;
  for (int q = threadIdx.y; q < 16; q += blockDim.y) {
    const int64_t r = row0 + q;
    const bool valid = r >= lo && r < hi;
    if (valid && in_place) continue;
    uint4* d4 = reinterpret_cast<uint4*>(dst + r * ldd);
    if (valid) {
      const uint4* s4 = reinterpret_cast<const uint4*>(src + r * lds);
      for (int64_t v = threadIdx.x; v < vecs; v += blockDim.x) d4[v] = s4[v];
    } else {
      for (int64_t v = threadIdx.x; v < vecs; v += blockDim.x) d4[v] = make_uint4(0, 0, 0, 0);
    }
  }
}

__device__ __forceinline__ void acc_bf16x8(float* acc, const uint4& u, float w) {
  const uint32_t* p = &u.x;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 f = unpack_bf16x2(p[q]);
    acc[2 * q] += w * f.x;
    acc[2 * q + 1] += w * f.y;
  }
}

// one warp per token
__global__ void moe_combine_kernel(__nv_bfloat16* __restrict__ out, int64_t ldo, __nv_bfloat16* __restrict__ keep,
                                   const float* __restrict__ w, const int32_t* __restrict__ owner,
                                   const int32_t* __restrict__ row, PeerBases src, int64_t lds, int K, int64_t vecs,
                                   int64_t n_tokens) {
  pdl_prologue();
  const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= n_tokens) return;
  for (int64_t v = lane; v < vecs; v += 32) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < K; ++k) {
      const int64_t i = t * K + k;
      const int r = owner[i];
      uint4 u = make_uint4(0, 0, 0, 0);
      if (r >= 0 && r < kMaxPeers) {
        u = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(src.p[r]) +
                                           (int64_t)row[i] * lds)[v];
        acc_bf16x8(acc, u, w != nullptr ? w[i] : 1.f);
      }
      if (keep != nullptr) reinterpret_cast<uint4*>(keep + i * (vecs * 8))[v] = u;
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    reinterpret_cast<uint4*>(out + t * ldo)[v] = o;
  }
}

// one warp per route
__global__ void moe_combine_bwd_kernel(const __nv_bfloat16* __restrict__ dout, int64_t ldo,
                                       const __nv_bfloat16* __restrict__ kept, const float* __restrict__ w,
                                       const int32_t* __restrict__ owner, const int32_t* __restrict__ row,
                                       PeerBases dst, int64_t ldd, int K, int64_t vecs, int64_t n_routes,
                                       float* __restrict__ dw) {
  pdl_prologue();
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= n_routes) return;
  const int r = owner[i];
  if (r < 0 || r >= kMaxPeers) {
    if (lane == 0) dw[i] = 0.f;
    return;
  }
  const float wi = w[i];
  const uint4* g4 = reinterpret_cast<const uint4*>(dout + (i / K) * ldo);
  const uint4* y4 = reinterpret_cast<const uint4*>(kept + i * (vecs * 8));
  uint4* d4 = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(dst.p[r]) + (int64_t)row[i] * ldd);
  float dot = 0.f;
  for (int64_t v = lane; v < vecs; v += 32) {
    const uint4 g = g4[v], y = y4[v];
    const uint32_t* gp = &g.x;
    const uint32_t* yp = &y.x;
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 gf = unpack_bf16x2(gp[q]), yf = unpack_bf16x2(yp[q]);
      dot += gf.x * yf.x + gf.y * yf.y;
      o[q] = pack_bf16x2(gf.x * wi, gf.y * wi);
    }
    d4[v] = make_uint4(o[0], o[1], o[2], o[3]);
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, s);
  if (lane == 0) dw[i] = dot;
}

unsigned warp_blocks(int64_t warps) { return (unsigned)((warps * 32 + 255) / 256); }

}  // namespace

void moe_hist(const int64_t* topi, int64_t n_routes, int E, float* mat, int mat_rows, int row, cudaStream_t s) {
  PB_CHECK(E >= 1 && E <= kMoeMaxExperts && row >= 0 && row < mat_rows, "moe_hist: sizes");
  launch_k(moe_hist_kernel, 1, 1024, E * sizeof(int), s, topi, n_routes, E, mat, mat_rows, row);
  PB_CUDA_CHECK(cudaGetLastError());
}

void moe_plan(const MoePlanArgs& a, cudaStream_t s) {
  PB_CHECK(a.E >= 1 && a.E <= kMoeMaxExperts && a.E_loc >= 1 && a.E % a.E_loc == 0, "moe_plan: expert counts");
  PB_CHECK(a.E / a.E_loc <= kPlanThreads && a.ep_rank >= 0 && a.ep_rank < a.E / a.E_loc, "moe_plan: owners");
  PB_CHECK(a.my_row >= 0 && a.my_row < a.mat_rows, "moe_plan: histogram row");
  int dev = 0;
  PB_CUDA_CHECK(cudaGetDevice(&dev));
  launch_k(moe_plan_kernel, 1, kPlanThreads, 0, s, a.topi, a.n_routes, a.mat, a.mat_rows, a.my_row, a.E, a.E_loc, a.ep_rank,
                                             a.local_only, a.route_owner, a.route_row, a.own_cnt, a.own_off,
                                             reinterpret_cast<int2*>(a.krange), a.tile_expert, a.n_tiles, a.tiles_cap,
                                             error_word(dev));
  PB_CUDA_CHECK(cudaGetLastError());
}

void moe_dispatch(const void* x, int64_t ldx, int K, const int32_t* owner, const int32_t* row, const PeerBases& dst,
                  int64_t ldd, int64_t cols, int64_t n_routes, cudaStream_t s) {
  PB_CHECK(cols % 8 == 0 && ldx % 8 == 0 && ldd % 8 == 0, "moe_dispatch: 16-byte rows");
  if (n_routes == 0) return;
  launch_k(moe_dispatch_kernel, warp_blocks(n_routes), 256, 0, s, reinterpret_cast<const __nv_bfloat16*>(x), ldx, K, owner,
                                                            row, dst, ldd, cols / 8, n_routes);
  PB_CUDA_CHECK(cudaGetLastError());
}

void moe_copy_pad(const void* src, int64_t lds, void* dst, int64_t ldd, int64_t cols, int tiles_cap,
                  const int32_t* tile_expert, const int32_t* n_tiles, const int32_t* own_cnt, const int32_t* own_off,
                  cudaStream_t s) {
  PB_CHECK(cols % 8 == 0 && lds % 8 == 0 && ldd % 8 == 0, "moe_copy_pad: 16-byte rows");
  if (tiles_cap == 0) return;
  launch_k(moe_copy_pad_kernel, (unsigned)(tiles_cap * 8), dim3(64, 4), 0, s,
      reinterpret_cast<const __nv_bfloat16*>(src), lds, reinterpret_cast<__nv_bfloat16*>(dst), ldd, cols / 8,
      tile_expert, n_tiles, own_cnt, own_off);
  PB_CUDA_CHECK(cudaGetLastError());
}

void moe_combine(void* out, int64_t ldo, void* keep, const float* w, const int32_t* owner, const int32_t* row,
                 const PeerBases& src, int64_t lds, int K, int64_t cols, int64_t n_tokens, cudaStream_t s) {
  PB_CHECK(cols % 8 == 0 && ldo % 8 == 0 && lds % 8 == 0, "moe_combine: 16-byte rows");
  if (n_tokens == 0) return;
  launch_k(moe_combine_kernel, warp_blocks(n_tokens), 256, 0, s, reinterpret_cast<__nv_bfloat16*>(out), ldo,
                                                           reinterpret_cast<__nv_bfloat16*>(keep), w, owner, row, src,
                                                           lds, K, cols / 8, n_tokens);
  PB_CUDA_CHECK(cudaGetLastError());
}

void moe_combine_bwd(const void* dout, int64_t ldo, const void* kept, const float* w, const int32_t* owner,
                     const int32_t* row, const PeerBases& dst, int64_t ldd, int K, int64_t cols, int64_t n_routes,
                     float* dw, cudaStream_t s) {
  PB_CHECK(cols % 8 == 0 && ldo % 8 == 0 && ldd % 8 == 0, "moe_combine_bwd: 16-byte rows");
  if (n_routes == 0) return;
  launch_k(moe_combine_bwd_kernel, warp_blocks(n_routes), 256, 0, s,
      reinterpret_cast<const __nv_bfloat16*>(dout), ldo, reinterpret_cast<const __nv_bfloat16*>(kept), w, owner, row,
      dst, ldd, K, cols / 8, n_routes, dw);
  PB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace pb
