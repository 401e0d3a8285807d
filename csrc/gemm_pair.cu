// CTA-pair (2-SM) persistent bf16 GEMM on tcgen05.
//
// A cluster of two CTAs computes 256 x BN output tiles with
// tcgen05.mma.cta_group::2: each CTA stages its own 128 rows of A and half of
// B's BN columns, the MMA (issued by the even CTA) reads both CTAs' shared
// memory and writes each CTA's 128 accumulator rows into its own TMEM.  Per
// 64-deep k-step a CTA moves 32 KB through shared memory instead of the 48 KB
// of a one-CTA 128 x 256 tile, which keeps the shared-memory traffic (TMA
// writes + MMA reads) under the 128 B/clk the SM provides while the tensor
// core runs at full rate.
//
// Roles per CTA (192 threads): warp 0 = TMA producer (both CTAs, each for its
// own halves; completion bytes go to the even CTA's barrier), warp 1 = TMEM
// allocator (both) + MMA issuer (even CTA), warps 2..5 = epilogue (both, one
// output row per thread, the same fused epilogues as the one-CTA kernel).
// The accumulator is double buffered in TMEM (2 x BN columns).  No load uses
// cluster multicast; only MMA completion is multicast to both CTAs.
//
// Same products as gemm.cu (the nn.Linear GEMMs of the reference's HF
// modules, parallel/parallel/engine/model_loading.py:17-35).
#include <cuda_bf16.h>

#include <algorithm>
#include <mutex>

#include "gemm.cuh"
#include "gemm_epi.cuh"
#include "host_util.h"
#include "ptx.cuh"

namespace pb {
namespace {

using gemm_detail::EpiArgs;

constexpr int BM_CTA = 128;  // rows of A per CTA (tile M = 256)
constexpr int BK = 64;
constexpr int kThreads = 192;

template <int BN>
struct PairCfg {
  static constexpr int B_HALF = BN / 2;  // B rows (N) staged per CTA
  static constexpr int A_BYTES = BM_CTA * BK * 2;
  static constexpr int B_BYTES = B_HALF * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES > 8 ? 8 : (200 * 1024) / STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int EPI_BYTES = 4 * gemm_detail::kEpiWarpBytes;  // TMA-store staging of the 4 epilogue warps
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024 + 256;
};

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Ordered split-K (kEpiSplitOrdered).  Work item (tile, slice sl) of a CTA
// waits until the 4 epilogue warps of (tile, sl - 1) on the same CTA rank have
// published their rows of the running fp32 sum (*cnt >= 4 * sl), adds its own
// product and publishes again; the last slice writes the output instead and
// the fourth of its warps to finish returns the counter to zero for the next
// launch.  The wait is bounded: on timeout the error word gets
// kErrSplitTimeout and the warp skips its rows (the host then clears the
// counters with the error word).  Waits cannot deadlock: every slice waits
// only on a lower work item, every CTA handles its items in increasing order
// and all clusters of the persistent grid are resident together.
__device__ __forceinline__ bool split_wait(const int* cnt, int target, int* err) {
  bool ok = true;
  if (target > 0) {
    const uint64_t t0 = globaltimer();
    uint32_t it = 0;
    while (ld_acquire_gpu(cnt) < target) {
      if ((++it & 63u) == 0) {
        // another role's error ends the wait only after 20 ms: an error word
        // left set by an earlier step must not make a healthy slice give up
        const uint64_t dt = globaltimer() - t0;
        if (dt > PB_SPIN_LIMIT_NS || (dt > 20000000ull && *((volatile int*)err) != 0)) {
          record_error(err, kErrSplitTimeout);
          ok = false;
          break;
        }
      }
    }
  }
  return __all_sync(0xffffffffu, ok);
}

// Running-sum rows are read one 32-column chunk ahead (the loads of chunk
// c + 1 are in flight while chunk c is added and stored), so a slice's
// epilogue is not a chain of dependent L2 round trips.
__device__ __forceinline__ bool split_prefetch(const EpiArgs& ep, int m, int M, int N, int n0, float4* dst) {
  if (m >= M || n0 + 32 > N) return false;
  const float4* w4 = reinterpret_cast<const float4*>(ep.ws + (int64_t)m * ep.ws_ld + n0);
#pragma unroll
  for (int q = 0; q < 8; ++q) dst[q] = __ldcg(w4 + q);
  return true;
}

template <int BN>
__device__ __forceinline__ void epilogue_split(const EpiArgs& ep, uint32_t t_row, int m, int M, int N, int n_base,
                                               bool first, bool last, bool ok) {
  float4 nx[8];
  bool nx_ok = !first && ok && split_prefetch(ep, m, M, N, n_base, nx);
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    float4 cu[8];
    const bool cu_ok = nx_ok;
#pragma unroll
    for (int q = 0; q < 8; ++q) cu[q] = nx[q];
    if (c + 32 < BN) nx_ok = !first && ok && split_prefetch(ep, m, M, N, n_base + c + 32, nx);
    float v[32];
    tmem_ld32(t_row + c, v);
    tmem_wait_ld();
    const int n0 = n_base + c;
    if (!ok || m >= M || n0 >= N) continue;
    const bool full = n0 + 32 <= N;
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] *= ep.alpha;
    float* wrow = ep.ws + (int64_t)m * ep.ws_ld + n0;
    if (!first) {
      if (cu_ok) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          v[q * 4] += cu[q].x; v[q * 4 + 1] += cu[q].y; v[q * 4 + 2] += cu[q].z; v[q * 4 + 3] += cu[q].w;
        }
      } else {
        gemm_detail::for_cols(n0, N, [&](int j) { v[j] += __ldcg(wrow + j); });
      }
    }
    if (!last) {
      if (full) {
        float4* w4 = reinterpret_cast<float4*>(wrow);
#pragma unroll
        for (int q = 0; q < 8; ++q) __stcg(w4 + q, make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]));
      } else {
        gemm_detail::for_cols(n0, N, [&](int j) { __stcg(wrow + j, v[j]); });
      }
    } else if (ep.out_f32) {
      float* dst = reinterpret_cast<float*>(ep.C) + (int64_t)m * ep.ldc + n0;
      if (full) {
        float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float4 o = make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
          if (ep.accum) {
            const float4 p = d4[q];
            o.x += p.x; o.y += p.y; o.z += p.z; o.w += p.w;
          }
          d4[q] = o;
        }
      } else {
        gemm_detail::for_cols(n0, N, [&](int j) { dst[j] = ep.accum ? dst[j] + v[j] : v[j]; });
      }
    } else {
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(ep.C) + (int64_t)m * ep.ldc + n0;
      if (ep.accum) {
        float r[32];
        gemm_detail::load_row_bf16(dst, r, n0, N);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += r[j];
      }
      gemm_detail::store_row_bf16(dst, v, n0, N);
    }
  }
}

__device__ __forceinline__ void split_publish(int* cnt, int sl, bool last, int lane) {
  if (!last) __threadfence();  // this warp's running-sum rows before the count
  __syncwarp();
  if (lane == 0) {
    const int old = atomicAdd(cnt, 1);
    if (last && old == 4 * sl + 3) atomicExch(cnt, 0);  // every warp of every slice has arrived
  }
}

// Copy warps of the gather variant: piece q of the pieces_per_block pieces of
// block `blk` (kGatherRowsPerPiece rows of K elements, contiguous in both the
// source shard and the gathered buffer), then publish it on flags[blk].
__device__ __forceinline__ void gather_piece(const GatherArgs& g, int K, int blk, int q, int lane) {
  const int64_t m0 = (int64_t)blk * 256 + (int64_t)q * kGatherRowsPerPiece;
  const int b = (int)(m0 / g.seq), s = (int)(m0 % g.seq);
  const int r = s / g.seq_local, sl = s % g.seq_local;
  const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(g.src[r]) +
                                                    ((int64_t)b * g.seq_local + sl) * g.src_ld);
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(g.dst) + m0 * K);
  const int64_t vecs_per_row = K / 8;
  const int64_t n = (int64_t)kGatherRowsPerPiece * vecs_per_row;
  if (g.src_ld == K) {
    constexpr int U = 8;
    for (int64_t i = lane; i < n; i += 32 * U) {
      uint4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (i + u * 32 < n) v[u] = src[i + u * 32];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (i + u * 32 < n) dst[i + u * 32] = v[u];
    }
  } else {
    for (int64_t i = lane; i < n; i += 32) {
      const int64_t row = i / vecs_per_row, c = i % vecs_per_row;
      dst[i] = src[row * (g.src_ld / 8) + c];
    }
  }
  __threadfence();
  __syncwarp();
  if (lane == 0) atomicAdd(&g.flags[blk], 1);
}

template <int BN, bool A_MN, bool B_MN, bool SWIGLU, bool GATHER>
__global__ void __launch_bounds__(GATHER ? kThreads + 64 : kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, EpiArgs ep,
                     int M, int N, int K, int b_up_row, int* err, const __grid_constant__ GatherArgs ga,
                     int splits, const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR) {
  pdl_prologue();
  using Cfg = PairCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int B_HALF = Cfg::B_HALF;
  constexpr int BN_OUT = SWIGLU ? BN / 2 : BN;
  static_assert(!SWIGLU || B_HALF == BN_OUT, "SwiGLU: the even CTA stages gate rows, the odd CTA up rows");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint8_t* sEpi = sB + STAGES * Cfg::B_BYTES;  // 1024-byte aligned (stage sizes are multiples of 1 KB)
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sEpi + Cfg::EPI_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;  // used on the even CTA (256 arrivals: both epilogues)
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], 2 * 128);
    }
    mbar_init(drain_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // barriers of both CTAs initialised before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int tiles_m = (M + 2 * BM_CTA - 1) / (2 * BM_CTA);
  const int tiles_n = (N + BN_OUT - 1) / BN_OUT;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = (K + BK - 1) / BK;
  // work item w = (tile, K slice): tile = w % num_tiles, slice = w / num_tiles
  const int kb_per = (num_kb + splits - 1) / splits;
  const int num_work = num_tiles * splits;
  const int n_clusters = gridDim.x >> 1;
  const int cid = blockIdx.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int w = cid; w < num_work && ok; w += n_clusters) {
        const int tile = w % num_tiles;
        const int kb0 = (w / num_tiles) * kb_per, kb1 = min(num_kb, kb0 + kb_per);
        const int tm = GATHER ? ga.m_order[tile % tiles_m] : tile % tiles_m, tn = tile / tiles_m;
        const int a_row = tm * 2 * BM_CTA + (int)rank * BM_CTA;
        if constexpr (GATHER) {
          // the A block of this tile must have been assembled by the copy warps
          const uint64_t t0 = globaltimer();
          uint32_t it = 0;
          while (ld_acquire_gpu(&ga.flags[tm]) - ga.target < 0) {
            if ((++it & 255u) == 0 && (*((volatile int*)err) != 0 || globaltimer() - t0 > PB_SPIN_LIMIT_NS)) {
              record_error(err, kErrPeerTimeout);
              ok = false;
              break;
            }
          }
          if (!ok) break;
          asm volatile("fence.proxy.async.global;" ::: "memory");
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, err)) { ok = false; break; }
          const uint32_t full_even = mapa_shared(smem_u32(&full_bar[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * Cfg::STAGE_BYTES);
          uint8_t* a_dst = sA + stage * Cfg::A_BYTES;
          uint8_t* b_dst = sB + stage * Cfg::B_BYTES;
          if (!A_MN) {
            tma_load_2d_pair(a_dst, &tmA, full_even, kb * BK, a_row);
          } else {
#pragma unroll
            for (int i = 0; i < BM_CTA / 64; ++i)
              tma_load_2d_pair(a_dst + i * 64 * BK * 2, &tmA, full_even, a_row + i * 64, kb * BK);
          }
          if (SWIGLU) {
            // even CTA: gate rows, odd CTA: up rows (B K-major)
            tma_load_2d_pair(b_dst, &tmB, full_even, kb * BK, (leader ? 0 : b_up_row) + tn * BN_OUT);
          } else if (!B_MN) {
            tma_load_2d_pair(b_dst, &tmB, full_even, kb * BK, tn * BN + (int)rank * B_HALF);
          } else {
#pragma unroll
            for (int i = 0; i < B_HALF / 64; ++i)
              tma_load_2d_pair(b_dst + i * 64 * BK * 2, &tmB, full_even, tn * BN + (int)rank * B_HALF + i * 64,
                               kb * BK);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(2 * BM_CTA, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int w = cid; w < num_work && ok; w += n_clusters, ++local) {
        const int kb0 = (w / num_tiles) * kb_per, kb1 = min(num_kb, kb0 + kb_per);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, err)) break;
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
            mma_bf16_ss_pair(d_tmem, adesc, bdesc, idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
          }
          mma_commit_pair(&empty_bar[stage], 0x3);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (ok) mma_commit_pair(&tfull_bar[acc], 0x3);
      }
    }
  } else if (GATHER && warp >= 6) {
    // copy warps: pieces of the blocks in the order the tiles need them
    const int pieces = 256 / kGatherRowsPerPiece;
    const int cw = (int)blockIdx.x * 2 + (warp - 6);
    for (int pi = cw; pi < ga.n_blocks * pieces; pi += (int)gridDim.x * 2)
      gather_piece(ga, K, ga.m_order[pi / pieces], pi % pieces, lane);
  } else {
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    uint8_t* stage = sEpi + quarter * gemm_detail::kEpiWarpBytes;
    int local = 0;
    for (int w = cid; w < num_work; w += n_clusters, ++local) {
      const int tile = w % num_tiles;
      const int tm = GATHER ? ga.m_order[tile % tiles_m] : tile % tiles_m, tn = tile / tiles_m;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, err)) break;
      tc_fence_after();
      const int m = tm * 2 * BM_CTA + (int)rank * BM_CTA + row;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      const uint32_t tempty = mapa_shared(smem_u32(&tempty_bar[acc]), 0);
      if (ep.epi == kEpiSplitOrdered) {
        const int sl = w / num_tiles;
        int* cnt = ep.cnt + 2 * tile + (int)rank;
        const bool ok = split_wait(cnt, 4 * sl, err);
        epilogue_split<BN>(ep, t_row, m, M, N, tn * BN_OUT, sl == 0, sl == splits - 1, ok);
        tc_fence_before();
        mbar_arrive_cluster(tempty);
        if (splits > 1) split_publish(cnt, sl, sl == splits - 1, lane);
      } else if (ep.tma == 2) {
        gemm_detail::epilogue_warp_tma_f32<BN>(ep, &tmC, t_row, stage, lane, m - lane, M, N, tn * BN_OUT,
                                               w / num_tiles, [&] {
                                                 tc_fence_before();
                                                 mbar_arrive_cluster(tempty);
                                               });
      } else if (ep.tma) {
        gemm_detail::epilogue_warp_tma<BN, SWIGLU>(ep, &tmC, &tmR, t_row, stage, lane, m - lane, M, N, tn * BN_OUT,
                                                   [&] {
                                                     tc_fence_before();
                                                     mbar_arrive_cluster(tempty);
                                                   });
      } else {
        gemm_detail::epilogue_row<BN, SWIGLU>(ep, t_row, m, M, N, tn * BN_OUT);
        tc_fence_before();
        mbar_arrive_cluster(tempty);
      }
    }
    // the tile stores must have finished before the kernel's shared memory goes
    if (ep.tma && lane == 0) bulk_wait_group<0>();
  }

  // On an error path the MMA issuer may have left MMAs in flight: drain them
  // (bounded) before the accumulator columns are released.
  if (warp == 1 && lane == 0 && leader && *((volatile int*)err) != 0) {
    mma_commit_pair(drain_bar, 0x1);
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(smem_u32(drain_bar), 0) && globaltimer() - t0 < 100000000ull) {
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the pair MMA may still read its shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

template <int BN, bool A_MN, bool B_MN, bool SWIGLU, bool GATHER = false>
void launch_pair(const GemmParams& p, cudaStream_t stream) {
  using Cfg = PairCfg<BN>;
  auto kern = gemm_pair_kernel<BN, A_MN, B_MN, SWIGLU, GATHER>;
  static std::mutex mu;
  static int max_clusters[64] = {0};
  int dev = 0;
  PB_CUDA_CHECK(cudaGetDevice(&dev));
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // pdl_prologue() (ptx.cuh)
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.blockDim = dim3(GATHER ? kThreads + 64 : kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = stream;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (max_clusters[dev & 63] == 0) {
      PB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES));
      cfg.gridDim = dim3(2 * num_sms(dev) / 2, 1, 1);
      int n = 0;
      PB_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
      PB_CHECK(n > 0, "gemm pair: no cluster of two CTAs fits on this GPU");
      max_clusters[dev & 63] = n;
    }
  }
  CUtensorMap ta = A_MN ? make_tmap_2d_bf16(p.A, p.M, p.K, p.lda, 64, BK)
                        : make_tmap_2d_bf16(p.A, p.K, p.M, p.lda, BK, BM_CTA);
  CUtensorMap tb;
  if (SWIGLU)
    tb = make_tmap_2d_bf16(p.B, p.K, p.b_up_offset + p.N, p.ldb, BK, Cfg::B_HALF);
  else
    tb = B_MN ? make_tmap_2d_bf16(p.B, p.N, p.K, p.ldb, 64, BK)
              : make_tmap_2d_bf16(p.B, p.K, p.N, p.ldb, BK, Cfg::B_HALF);
  EpiArgs ep{p.C, p.R, p.ldc, p.ldr, p.alpha, p.epi, SWIGLU ? p.b_up_offset : 0};
  if (p.epi == kEpiSplitOrdered) {
    const int64_t tiles_mn = ((p.M + 2 * BM_CTA - 1) / (2 * BM_CTA)) * ((p.N + BN - 1) / BN);
    PB_CHECK(2 * tiles_mn <= kSplitSlotInts, "gemm: ordered split-K supports at most 4096 output tiles");
    PB_CHECK(p.ws != nullptr && p.ws_ld >= p.N && p.ws_ld % 4 == 0 && (reinterpret_cast<uintptr_t>(p.ws) & 15) == 0,
             "gemm: ordered split-K needs a 16-byte aligned fp32 workspace with ld % 4 == 0");
    ep.ws = p.ws;
    ep.ws_ld = p.ws_ld;
    ep.cnt = split_counters(dev);
    ep.out_f32 = p.out_f32 ? 1 : 0;
    ep.accum = p.accumulate ? 1 : 0;
  }
  if (p.scatter) ep.sc = *p.scatter;
  // TMA-store epilogue for the bf16 store and SwiGLU epilogues into local memory
  // (16-byte aligned bases and row strides; SwiGLU: whole 32-column chunks so a
  // gate store can never spill into the up half)
  auto al16 = [](const void* ptr, int64_t ld) {
    return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && (ld * 2) % 16 == 0;
  };
  CUtensorMap tc{}, tr{};
  if (!p.scatter && p.C && al16(p.C, p.ldc) &&
      ((SWIGLU && p.N % 32 == 0 && (!p.R || al16(p.R, p.ldr))) || (!SWIGLU && p.epi == kEpiStoreBf16))) {
    tc = make_tmap_2d_bf16_swz(p.C, p.N, p.M, p.ldc, gemm_detail::kEpiBox, gemm_detail::kEpiBox, 64);
    if (SWIGLU && p.R)
      tr = make_tmap_2d_bf16_swz(p.R, p.b_up_offset + p.N, p.M, p.ldr, gemm_detail::kEpiBox, gemm_detail::kEpiBox,
                                 64);
    ep.tma = 1;
  }
  // fp32 store through TMA (and split-K into per-slice slabs [splits, M, ldc])
  if (!SWIGLU && !GATHER && !p.scatter && p.epi == kEpiStoreF32 && p.C &&
      (reinterpret_cast<uintptr_t>(p.C) & 15) == 0 && (p.ldc * 4) % 16 == 0) {
    const int slabs = std::max(1, p.splits);
    tc = make_tmap_3d_f32(p.C, p.N, p.M, slabs, p.ldc, (uint64_t)p.M * p.ldc, gemm_detail::kEpiBox,
                          gemm_detail::kEpiBox, 1, true);
    ep.tma = 2;
  }
  PB_CHECK(p.splits <= 1 || p.epi != kEpiStoreF32 || ep.tma == 2,
           "gemm: split-K into fp32 slabs needs a 16-byte aligned output with a 16-byte row stride");
  GatherArgs ga{};
  if (GATHER) ga = *p.gather;
  const int bn_out = SWIGLU ? BN / 2 : BN;
  const int tiles = ((p.M + 2 * BM_CTA - 1) / (2 * BM_CTA)) * ((p.N + bn_out - 1) / bn_out) * std::max(1, p.splits);
  int clusters = max_clusters[dev & 63];
  if (p.max_ctas > 0) clusters = std::min(clusters, std::max(1, p.max_ctas / 2));
  clusters = std::max(1, std::min(clusters, tiles));
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  PB_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, ep, p.M, p.N, p.K, (int)p.b_up_offset, error_word(dev), ga,
                                   std::max(1, p.splits), tc, tr));
}

}  // namespace

void gemm_bf16_pair(const GemmParams& p, cudaStream_t stream) {
  if (p.gather) {
    // A (the gathered activations) is K-major by construction
    PB_CHECK(!p.a_mn, "gemm: the gathered A operand is K-major");
    PB_CHECK(p.gather->seq_local % 256 == 0 && p.gather->n_blocks == (p.M + 255) / 256 && p.M % 256 == 0 &&
                 p.gather->n_blocks <= 64 && p.K % 8 == 0 && p.gather->nranks <= 8,
             "gemm: gather needs 256-row aligned shards, M % 256 == 0 and at most 64 blocks");
    if (p.epi == kEpiSwiGLU) return launch_pair<256, false, false, true, true>(p, stream);
    if (!p.b_mn) return launch_pair<256, false, false, false, true>(p, stream);
    return launch_pair<256, false, true, false, true>(p, stream);
  }
  if (p.scatter) PB_CHECK(p.epi == kEpiStoreBf16 && p.scatter->nranks <= 8, "gemm: scatter needs the bf16 store epilogue");
  PB_CHECK(p.splits <= 1 || ((p.epi == kEpiAtomicF32 || p.epi == kEpiSplitOrdered || p.epi == kEpiStoreF32) &&
                               !p.gather && !p.scatter),
           "gemm: split-K needs the atomic, the ordered or the fp32 slab epilogue");
  if (p.epi == kEpiSwiGLU) return launch_pair<256, false, false, true>(p, stream);
  if (!p.a_mn && !p.b_mn) return launch_pair<256, false, false, false>(p, stream);
  if (!p.a_mn && p.b_mn) return launch_pair<256, false, true, false>(p, stream);
  if (p.a_mn && !p.b_mn) return launch_pair<256, true, false, false>(p, stream);
  return launch_pair<256, true, true, false>(p, stream);
}

}  // namespace pb
