// Device-resident MoE routing launchers (moe.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "comm.cuh"

namespace pb {

constexpr int kMoeMaxExperts = 256;

// Histogram of `topi` (int64 global expert ids, n_routes) into row `row` of the
// fp32 matrix mat [mat_rows, E]; the other rows are zeroed.
void moe_hist(const int64_t* topi, int64_t n_routes, int E, float* mat, int mat_rows, int row, cudaStream_t s);

struct MoePlanArgs {
  const int64_t* topi = nullptr;  // [n_routes] global expert of each route (token-major)
  int64_t n_routes = 0;
  const float* mat = nullptr;     // [mat_rows, E] route histograms of the source ranks
  int mat_rows = 1, my_row = 0;   // this rank's histogram row
  int E = 0, E_loc = 0;           // global experts, experts per owner
  int ep_rank = 0;                // this rank's owner index
  int local_only = 0;             // keep only routes to this rank's experts (owner index 0)
  int32_t* route_owner = nullptr; // [n_routes] out: owner (-1: not kept)
  int32_t* route_row = nullptr;   // [n_routes] out: row in the owner's padded matrix
  int32_t* own_cnt = nullptr;     // [E_loc] out: rows routed to each local expert
  int32_t* own_off = nullptr;     // [E_loc] out: first padded row of each local expert
  int32_t* krange = nullptr;      // [E_loc, 2] out: weight-gradient K range (64-row multiples)
  int32_t* tile_expert = nullptr; // [tiles_cap] out: local expert of each 128-row tile
  int32_t* n_tiles = nullptr;     // [1] out: tiles of the padded matrix
  int tiles_cap = 0;
};
void moe_plan(const MoePlanArgs& a, cudaStream_t s);

// dst[owner[i]] row row[i] <- x row (i / K)          (bf16 rows of `cols`)
void moe_dispatch(const void* x, int64_t ldx, int K, const int32_t* owner, const int32_t* row, const PeerBases& dst,
                  int64_t ldd, int64_t cols, int64_t n_routes, cudaStream_t s);
// padded rows [0, 128 * n_tiles): valid rows copied from src (left alone when
// src == dst), padding rows zeroed; the grid covers tiles_cap tiles
void moe_copy_pad(const void* src, int64_t lds, void* dst, int64_t ldd, int64_t cols, int tiles_cap,
                  const int32_t* tile_expert, const int32_t* n_tiles, const int32_t* own_cnt, const int32_t* own_off,
                  cudaStream_t s);
// out[t] = sum_k w[t,k] * src[owner][row] (w == nullptr: weight 1); keep (when
// given) receives every pulled row, [n_tokens * K, cols]
void moe_combine(void* out, int64_t ldo, void* keep, const float* w, const int32_t* owner, const int32_t* row,
                 const PeerBases& src, int64_t lds, int K, int64_t cols, int64_t n_tokens, cudaStream_t s);
// dw[i] = <dout[i / K], kept[i]>; dst[owner[i]] row row[i] <- w[i] * dout[i / K]
void moe_combine_bwd(const void* dout, int64_t ldo, const void* kept, const float* w, const int32_t* owner,
                     const int32_t* row, const PeerBases& dst, int64_t ldd, int K, int64_t cols, int64_t n_routes,
                     float* dw, cudaStream_t s);

}  // namespace pb
