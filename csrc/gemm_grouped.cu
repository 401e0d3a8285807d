// Grouped bf16 GEMM for the mixture-of-experts MLPs: one persistent launch
// runs the products of every expert from a device work table.
//
// The routed rows of each expert sit at a 128-row aligned offset of one
// matrix, separated by zero rows (built by the caller), so a 128-row tile
// never mixes experts and the zero rows make out-of-group contributions
// vanish.  Two modes:
//   rows (forward, input gradient): work item {expert e, M tile, N tile};
//     C[tile rows] = A[tile rows] x B_e, B_e from a 3-D tensor map over the
//     stacked expert weights [E][..][..] (K-major, or MN-major for the input
//     gradient); the SwiGLU epilogue takes gate rows [0, I) and up rows
//     [I, 2I) of the expert's gate/up weight.
//   k (weight gradient): work item {expert e, M tile, N tile};
//     dW_e = A^T B over the expert's row range only (krange[e], multiples of
//     64), both operands MN-major views of the row matrices, C = stacked
//     [E][M][N].  The device-resident MoE layout gives every expert at least
//     one (zero) tile, so no work item meets an empty K range.
//   rows mode can also take its items from the device: with tile_expert /
//     n_tiles set, the items are every (tile, N tile) of the first *n_tiles
//     128-row tiles (the count the routing plan wrote), so no row count has
//     to reach the host.
// Warp roles and the double-buffered TMEM accumulator follow the one-CTA
// kernel in gemm.cu; each wait is bounded.
//
// Replaces the reference's per-expert dispatch through HF's grouped expert
// path (transformers integrations/moe.py grouped_mm_experts_forward, called
// from the Qwen3-MoE experts the reference trains).
#include <cuda_bf16.h>

#include <algorithm>
#include <cstdlib>

#include "gemm.cuh"
#include "gemm_epi.cuh"
#include "host_util.h"
#include "ptx.cuh"

namespace pb {
namespace {

using gemm_detail::EpiArgs;

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;

template <int BN>
struct GCfg {
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
};

template <int BN, bool A_MN, bool B_MN, bool SWIGLU, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_grouped_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, EpiArgs ep,
                        const int4* __restrict__ work, int n_work, const int2* __restrict__ krange, int M_total,
                        int M_group, int N, int K, int b_up_row, const int* __restrict__ tile_expert,
                        const int* __restrict__ n_tiles, int ntn, int* err) {
  pdl_prologue();
  using Cfg = GCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int BN_OUT = SWIGLU ? BN / 2 : BN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sB + STAGES * Cfg::B_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], 128);
    }
    mbar_init(drain_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // device-described rows mode: every (tile, N tile) of the first *n_tiles tiles
  if (tile_expert != nullptr) n_work = *((volatile const int*)n_tiles) * ntn;
  auto item = [&](int w) -> int4 {
    if (tile_expert == nullptr) return work[w];
    const int t = w / ntn;
    return make_int4(tile_expert[t], t, w - t * ntn, 0);
  };

  // K blocks of a work item: all of K (rows mode) or the expert's rows (k mode)
  auto k_span = [&](int e, int& kb0, int& kb1) {
    if (MODE == 2) {
      const int2 kr = krange[e];
      kb0 = kr.x / BK;
      kb1 = kr.y / BK;
    } else {
      kb0 = 0;
      kb1 = (K + BK - 1) / BK;
    }
  };

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x) {
        const int4 it = item(w);
        const int e = it.x, tm = it.y, tn = it.z;
        int kb0, kb1;
        k_span(e, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, err)) { ok = false; break; }
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
          uint8_t* a_dst = sA + stage * Cfg::A_BYTES;
          uint8_t* b_dst = sB + stage * Cfg::B_BYTES;
          if (!A_MN) {
            tma_load_2d(a_dst, &tmA, &full_bar[stage], kb * BK, tm * BM);
          } else {
#pragma unroll
            for (int i = 0; i < BM / 64; ++i)
              tma_load_2d(a_dst + i * 64 * BK * 2, &tmA, &full_bar[stage], tm * BM + i * 64, kb * BK);
          }
          if (MODE == 2) {  // B: MN-major rows of the expert's range
#pragma unroll
            for (int i = 0; i < BN / 64; ++i)
              tma_load_2d(b_dst + i * 64 * BK * 2, &tmB, &full_bar[stage], tn * BN + i * 64, kb * BK);
          } else if (SWIGLU) {
            tma_load_3d(b_dst, &tmB, &full_bar[stage], kb * BK, tn * BN_OUT, e);
            tma_load_3d(b_dst + (BN / 2) * BK * 2, &tmB, &full_bar[stage], kb * BK, b_up_row + tn * BN_OUT, e);
          } else if (!B_MN) {
            tma_load_3d(b_dst, &tmB, &full_bar[stage], kb * BK, tn * BN, e);
          } else {
#pragma unroll
            for (int i = 0; i < BN / 64; ++i)
              tma_load_3d(b_dst + i * 64 * BK * 2, &tmB, &full_bar[stage], tn * BN + i * 64, kb * BK, e);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x, ++local) {
        const int e = item(w).x;
        int kb0, kb1;
        k_span(e, kb0, kb1);
        const int acc = local & 1;
        if (!mbar_wait(&tempty_bar[acc], ((local >> 1) & 1) ^ 1, err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t adesc = A_MN ? smem_desc_sw128(a_base + kk * 2048, 64 * BK * 2, 1024)
                                        : smem_desc_sw128(a_base + kk * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? smem_desc_sw128(b_base + kk * 2048, 64 * BK * 2, 1024)
                                        : smem_desc_sw128(b_base + kk * 32, 16, 1024);
            mma_bf16_ss(d_tmem, adesc, bdesc, idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
          }
          mma_commit(&empty_bar[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (ok) mma_commit(&tfull_bar[acc]);
      }
    }
  } else {
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    int local = 0;
    for (int w = blockIdx.x; w < n_work; w += gridDim.x, ++local) {
      const int4 it = item(w);
      const int e = it.x, tm = it.y, tn = it.z;
      const int acc = local & 1;
      if (!mbar_wait(&tfull_bar[acc], (local >> 1) & 1, err)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      if (MODE == 2) {
        // stacked output [E][M_group][N]; the caller routes only non-empty experts here
        const int m = e * M_group + tm * BM + row;
        const int bound = (tm * BM + row < M_group) ? M_total : 0;
        gemm_detail::epilogue_row<BN, SWIGLU>(ep, t_row, m, bound, N, tn * BN_OUT);
      } else {
        gemm_detail::epilogue_row<BN, SWIGLU>(ep, t_row, tm * BM + row, M_total, N, tn * BN_OUT);
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
    }
  }

  if (warp == 1 && lane == 0 && *((volatile int*)err) != 0) {
    mma_commit(drain_bar);
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(smem_u32(drain_bar), 0) && globaltimer() - t0 < 100000000ull) {
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

template <int BN, bool A_MN, bool B_MN, bool SWIGLU, int MODE>
void launch_grouped(const GroupedGemmParams& p, cudaStream_t stream) {
  using Cfg = GCfg<BN>;
  auto kern = gemm_grouped_kernel<BN, A_MN, B_MN, SWIGLU, MODE>;
  static bool attr_set[64] = {false};
  int dev = 0;
  PB_CUDA_CHECK(cudaGetDevice(&dev));
  if (!attr_set[dev & 63]) {
    PB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES));
    attr_set[dev & 63] = true;
  }
  CUtensorMap ta, tb;
  if (MODE == 1) {
    // A [rows, K] K-major; B stacked [E][Nb][K] (K-major) or [E][K][Nb] (MN-major)
    ta = make_tmap_2d_bf16(p.A, p.K, p.M_total, p.lda, BK, BM);
    if (!B_MN)
      tb = make_tmap_3d_bf16(p.B, p.K, p.b_rows, p.E, p.ldb, (uint64_t)p.b_rows * p.ldb, BK, SWIGLU ? BN / 2 : BN, 1);
    else
      tb = make_tmap_3d_bf16(p.B, p.N, p.K, p.E, p.ldb, (uint64_t)p.K * p.ldb, 64, BK, 1);
  } else {
    // A [rows, M_group] and B [rows, N] row matrices read MN-major
    ta = make_tmap_2d_bf16(p.A, p.M_group, p.rows, p.lda, 64, BK);
    tb = make_tmap_2d_bf16(p.B, p.N, p.rows, p.ldb, 64, BK);
  }
  EpiArgs ep{p.C, p.R, p.ldc, p.ldr, p.alpha, p.epi, SWIGLU ? p.b_up_offset : 0};
  constexpr int BN_OUT = SWIGLU ? BN / 2 : BN;
  const int ntn = (p.N + BN_OUT - 1) / BN_OUT;
  const int max_items = p.tile_expert != nullptr ? (p.M_total / BM) * ntn : p.n_work;
  const int ctas = std::max(1, std::min(num_sms(dev), max_items));
  launch_k(kern, ctas, kThreads, Cfg::SMEM_BYTES, stream, ta, tb, ep, p.work, p.n_work, p.krange, p.M_total, p.M_group,
                                                    p.N, p.K, (int)p.b_up_offset, p.tile_expert, p.n_tiles, ntn,
                                                    error_word(dev));
  PB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace

// Column width of the non-SwiGLU products.  A 128 x 256 tile brings 48 KB
// into shared memory per 64-deep k-block for 4.2 MFLOP (85 FLOP per byte)
// against 32 KB for 2.1 MFLOP (64 per byte) at 128 x 128, and halves the work
// items.  Measured on the expert layer of Qwen3-30B-A3B at EP = 4 (32 experts,
// 8,192 routes, forward + backward, 50 calls): 128-wide tiles 742.7 us,
// 256-wide 718.0 us, 256 only where N >= 1536 723.1 us; so every product wider
// than 128 columns takes 256 (mode is kept for the k-mode work tables, which
// tile N by this width).  PB_GROUPED_BN=128 / 256 forces one width (read once).
int grouped_bn(int mode, int N) {
  static const int forced = [] {
    const char* v = std::getenv("PB_GROUPED_BN");
    return v ? std::atoi(v) : 0;
  }();
  (void)mode;
  if (forced == 128 || forced == 256) return forced;
  return N > 128 ? 256 : 128;
}

void gemm_grouped(const GroupedGemmParams& p, cudaStream_t stream) {
  PB_CHECK(p.n_work >= 0 && p.E > 0 && p.N > 0 && p.K > 0, "grouped gemm: sizes");
  PB_CHECK(p.lda % 8 == 0 && p.ldb % 8 == 0 && p.ldc % 8 == 0, "grouped gemm: strides must be multiples of 8");
  PB_CHECK(p.tile_expert == nullptr || (p.mode == 1 && p.n_tiles != nullptr), "grouped gemm: device tiles need rows mode");
  if (p.n_work == 0 && p.tile_expert == nullptr) return;
  const bool wide = grouped_bn(p.mode, p.N) == 256;
  if (p.mode == 1) {
    PB_CHECK(p.M_total % BM == 0, "grouped gemm: the row matrix must be 128-row padded");
    if (p.epi == kEpiSwiGLU) return launch_grouped<256, false, false, true, 1>(p, stream);
    if (!p.b_mn)
      return wide ? launch_grouped<256, false, false, false, 1>(p, stream)
                  : launch_grouped<128, false, false, false, 1>(p, stream);
    return wide ? launch_grouped<256, false, true, false, 1>(p, stream)
                : launch_grouped<128, false, true, false, 1>(p, stream);
  }
  PB_CHECK(p.mode == 2 && p.krange != nullptr, "grouped gemm: k mode needs krange");
  PB_CHECK(p.epi == kEpiStoreBf16 || p.epi == kEpiStoreF32 || p.epi == kEpiAccumF32 || p.epi == kEpiAccumBf16,
           "grouped gemm: k mode takes store / accumulate epilogues");
  return wide ? launch_grouped<256, true, true, false, 2>(p, stream) : launch_grouped<128, true, true, false, 2>(p, stream);
}

}  // namespace pb
