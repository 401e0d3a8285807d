// Persistent, warp-specialised bf16 GEMM on the sm_100a tensor cores.
//
// One CTA per SM walks a static tile schedule.  Roles per CTA (192 threads):
//   warp 0      : TMA producer (one thread) -> STAGES-deep smem ring
//   warp 1      : TMEM allocator + tcgen05.mma issuer (one thread)
//   warps 2..5  : epilogue; warp w reads TMEM lanes 32*(w%4)..+31, i.e. one
//                 output row per thread, and applies the fused epilogue.
// The fp32 accumulator lives in TMEM and is double buffered (2 x BN columns)
// so the epilogue of tile i overlaps the main loop of tile i+1.  Operand
// tiles are 128-byte swizzled; K-major tiles are one 64-element atom wide,
// MN-major tiles are loaded as 64-wide column blocks (LBO = block size).
//
// This replaces the cuBLAS nn.Linear products the reference runs through HF
// (q/k/v/o/gate/up/down/lm_head forward and both backward products,
// reference: parallel/parallel/engine/model_loading.py:17-35 loads the HF
// modules whose Linear layers issue them).
#include <cuda_bf16.h>

#include <algorithm>

#include "gemm.cuh"
#include "gemm_epi.cuh"
#include "host_util.h"
#include "ptx.cuh"

namespace pb {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

using gemm_detail::EpiArgs;

template <int BN, bool A_MN, bool B_MN, bool SWIGLU>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                EpiArgs ep, int M, int N, int K, int b_up_row, int* err) {
  pdl_prologue();
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  // SwiGLU tiles produce BN/2 output columns from BN accumulator columns.
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

  const int tiles_m = (M + BM - 1) / BM;
  const int tiles_n = (N + BN_OUT - 1) / BN_OUT;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = (K + BK - 1) / BK;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int tm = tile % tiles_m, tn = tile / tiles_m;
        for (int kb = 0; kb < num_kb; ++kb) {
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
          if (SWIGLU) {
            // gate rows then up rows, BN/2 each (B is K-major here)
            tma_load_2d(b_dst, &tmB, &full_bar[stage], kb * BK, tn * BN_OUT);
            tma_load_2d(b_dst + (BN / 2) * BK * 2, &tmB, &full_bar[stage], kb * BK,
                        b_up_row + tn * BN_OUT);
          } else if (!B_MN) {
            tma_load_2d(b_dst, &tmB, &full_bar[stage], kb * BK, tn * BN);
          } else {
#pragma unroll
            for (int i = 0; i < BN / 64; ++i)
              tma_load_2d(b_dst + i * 64 * BK * 2, &tmB, &full_bar[stage], tn * BN + i * 64, kb * BK);
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
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
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
            mma_bf16_ss(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          mma_commit(&empty_bar[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (ok) mma_commit(&tfull_bar[acc]);
      }
    }
  } else {
    // Epilogue warps.
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int tm = tile % tiles_m, tn = tile / tiles_m;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, err)) break;
      tc_fence_after();
      const int m = tm * BM + row;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      gemm_detail::epilogue_row<BN, SWIGLU>(ep, t_row, m, M, N, tn * BN_OUT);
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
    }
  }

  // On an error path the MMA issuer may have left MMAs in flight: drain them
  // (bounded) before the accumulator columns are released.
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

template <int BN, bool A_MN, bool B_MN, bool SWIGLU>
void launch(const GemmParams& p, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_kernel<BN, A_MN, B_MN, SWIGLU>;
  static bool attr_set[64] = {false};
  int dev = 0;
  PB_CUDA_CHECK(cudaGetDevice(&dev));
  if (!attr_set[dev & 63]) {
    PB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       Cfg::SMEM_BYTES));
    attr_set[dev & 63] = true;
  }
  // A: K-major -> dims {K, M}, box {64, 128}; MN-major -> dims {M, K}, box {64, 64}
  CUtensorMap ta = A_MN ? make_tmap_2d_bf16(p.A, p.M, p.K, p.lda, 64, BK)
                        : make_tmap_2d_bf16(p.A, p.K, p.M, p.lda, BK, BM);
  CUtensorMap tb;
  int b_rows = SWIGLU ? (int)(p.b_up_offset + p.N) : p.N;
  if (SWIGLU)
    tb = make_tmap_2d_bf16(p.B, p.K, b_rows, p.ldb, BK, BN / 2);
  else
    tb = B_MN ? make_tmap_2d_bf16(p.B, p.N, p.K, p.ldb, 64, BK)
              : make_tmap_2d_bf16(p.B, p.K, p.N, p.ldb, BK, BN);
  EpiArgs ep{p.C, p.R, p.ldc, p.ldr, p.alpha, p.epi, SWIGLU ? p.b_up_offset : 0};
  const int bn_out = SWIGLU ? BN / 2 : BN;
  const int tiles = ((p.M + BM - 1) / BM) * ((p.N + bn_out - 1) / bn_out);
  int ctas = num_sms(dev);
  if (p.max_ctas > 0) ctas = std::min(ctas, p.max_ctas);
  ctas = std::max(1, std::min(ctas, tiles));
  launch_k(kern, ctas, kThreads, Cfg::SMEM_BYTES, stream, ta, tb, ep, p.M, p.N, p.K,
                                                   (int)p.b_up_offset, error_word(dev));
  PB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace

void gemm_bf16(const GemmParams& p, cudaStream_t stream) {
  PB_CHECK(p.M > 0 && p.N > 0 && p.K > 0, "gemm: empty problem");
  PB_CHECK(p.lda % 8 == 0 && p.ldb % 8 == 0, "gemm: lda/ldb must be multiples of 8 elements");
  PB_CHECK((reinterpret_cast<uintptr_t>(p.A) & 15) == 0 && (reinterpret_cast<uintptr_t>(p.B) & 15) == 0,
           "gemm: A/B must be 16-byte aligned");
  const bool f32 = p.epi == kEpiStoreF32 || p.epi == kEpiAccumF32 || p.epi == kEpiAtomicF32 ||
                   (p.epi == kEpiSplitOrdered && p.out_f32);
  PB_CHECK(p.ldc % (f32 ? 4 : 8) == 0 && (reinterpret_cast<uintptr_t>(p.C) & 15) == 0,
           "gemm: C must be 16-byte aligned with a 16-byte row stride");
  if (p.epi == kEpiSwiGLU) PB_CHECK(!p.a_mn && !p.b_mn, "gemm: SwiGLU epilogue needs K-major operands");
  // The CTA-pair kernel (256-row tiles) wins on every training shape measured
  // with M >= 256; smaller M keeps the one-CTA kernel.
  if (p.kernel == 2 || p.gather || p.scatter || p.splits > 1 || p.epi == kEpiSplitOrdered ||
      (p.kernel == 0 && p.M >= 256))
    return gemm_bf16_pair(p, stream);
  if (p.epi == kEpiSwiGLU) {
    launch<256, false, false, true>(p, stream);
    return;
  }
  // Narrow problems use 128-wide tiles so more CTAs participate.
  const bool narrow =
      p.N <= 128 || (int64_t)((p.M + 127) / 128) * ((p.N + 255) / 256) < num_sms();
  if (narrow) {
    if (!p.a_mn && !p.b_mn) return launch<128, false, false, false>(p, stream);
    if (!p.a_mn && p.b_mn) return launch<128, false, true, false>(p, stream);
    if (p.a_mn && !p.b_mn) return launch<128, true, false, false>(p, stream);
    return launch<128, true, true, false>(p, stream);
  }
  if (!p.a_mn && !p.b_mn) return launch<256, false, false, false>(p, stream);
  if (!p.a_mn && p.b_mn) return launch<256, false, true, false>(p, stream);
  if (p.a_mn && !p.b_mn) return launch<256, true, false, false>(p, stream);
  return launch<256, true, true, false>(p, stream);
}

}  // namespace pb
