// Causal GQA flash-attention backward on tcgen05.
//
// One CTA owns a 128-key tile j of one (batch, kv-head) and loops over every
// query head of the GQA group and every query tile i that can see tile j.
// Per (head, i), with K_j / V_j resident in shared memory:
//   S^T  = K_j Q_i^T            -> TMEM cols [  0,128)  (lane = key)
//   dP^T = V_j dO_i^T           -> TMEM cols [128,256)
//   P^T  = exp2(S^T*scale*log2e - lse*log2e) -> smem (bf16)   [element warps]
//   dV  += P^T dO_i             -> TMEM cols [256,384)
//   dS^T = P^T (dP^T*scale - delta*scale) -> smem (same buffer, after dV read P)
//   dQ_i = dS K_j               -> TMEM cols [128,256)  (dP^T is consumed by then)
//   dK  += dS^T Q_i             -> TMEM cols [384,512)
// dQ_i leaves TMEM through a shared staging buffer and a bulk tensor
// reduce-add (the fp32 add happens in L2) issued by its own warpgroup; dK / dV
// leave TMEM once at the end.  Every operand tile is loaded once in the
// K-major 128B-swizzled layout and re-read as MN-major where a product needs
// its transpose (same bytes, different descriptor strides).
//
// Warpgroups (512 threads): 0 = TMA producer (warp 0) and MMA issuer (warp 1);
// 1 and 2 = element warps, warpgroup 1+g handling query columns [64g, 64g+64)
// of S^T / dP^T; 3 = dQ drain (TMEM -> shared stage -> bulk reduce-add).  A
// warp reads the TMEM lane quarter warp % 4.  setmaxnreg moves registers from
// warpgroups 0 and 3 to the element warpgroups.
//
// A prep kernel computes delta*scale = rowsum(dO*O)*scale and lse*log2e into
// one scratch array and zeroes the dQ accumulator; a cast kernel turns the
// accumulator into bf16 dq afterwards.
//
// Replaces the autograd of HF's SDPA call in the reference
// (parallel/parallel/engine/model_loading.py:22).
#include <cuda_bf16.h>

#include <algorithm>
#include <cstdio>
#include <exception>
#include <mutex>

#include "attention.cuh"
#include "host_util.h"
#include "ptx.cuh"

namespace pb {
namespace {

constexpr int BT = 128;   // tile rows (queries or keys)
constexpr int HD = 128;
constexpr int kThreads = 512;  // 4 warpgroups
// setmaxnreg split: 128 registers a thread at launch (65536 / 512); the sum
// over the four warpgroups must stay 4 x 128.
constexpr int kRegsCtl = 56, kRegsElem = 168, kRegsDq = 120;
static_assert(kRegsCtl + 2 * kRegsElem + kRegsDq == 4 * 128, "attention bwd: register split");
constexpr int TILE = 128 * HD * 2;   // 32 KB bf16 operand tile
constexpr int STAGE = 128 * 32 * 4;  // 16 KB of dQ staging per buffer (2 buffers)
constexpr int DQ_BOX = 32 * 32 * 4;  // 4 KB: one warp's 32 rows x 32 fp32 columns
// K, V, Q x2, dO, P/dS + two dQ stages + double-buffered lse2/delta (2 KB)
// + barriers + TMEM slot.
constexpr int SMALL_BYTES = 2048 + 24 * 8;
constexpr int SMEM_BYTES = 232448;  // the sm_100 per-block maximum
static_assert(6 * TILE + 2 * STAGE + SMALL_BYTES <= SMEM_BYTES, "attention bwd: smem budget");
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// DS_STORE: instead of producing dQ, every dS^T tile (the bf16 shared-memory
// image, already swizzled for the MMA) is stored to ds_buf for the dQ kernel.
template <bool kTrace, bool DS_STORE>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                    const __grid_constant__ CUtensorMap tmdQ, const float* __restrict__ LSE2,
                    const float* __restrict__ DELTA, __nv_bfloat16* __restrict__ dK, int64_t lddk,
                    __nv_bfloat16* __restrict__ dV, int64_t lddv, int B, int S, int nq, int nkv, float scale,
                    bool causal, int* err, long long* trace, __nv_bfloat16* __restrict__ ds_buf) {
  pdl_prologue();
  // optional per-CTA phase timing (clock64 cycles, kTrace builds only); slots
  // are documented at the use sites
  constexpr int kSlots = kTrace ? kAttnBwdTraceSlots : 1;
  long long tacc[kSlots];
#pragma unroll
  for (int i = 0; i < kSlots; ++i) tacc[i] = 0;
  auto tw = [&](int slot, uint64_t* bar, uint32_t par) -> bool {
    if constexpr (!kTrace) {
      return mbar_wait(bar, par, err);
    } else {
      const long long t0 = clock64();
      const bool r = mbar_wait(bar, par, err);
      tacc[slot] += clock64() - t0;
      return r;
    }
  };
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  // The 128B-swizzled tiles need 1024-byte alignment; the budget leaves
  // SMEM_BYTES - 6*TILE - 2*STAGE - SMALL_BYTES bytes for it.  Bail out
  // (uniformly, before any barrier or TMEM use) if the window is aligned worse.
  if ((size_t)(smem - smem_raw) + 6 * TILE + 2 * STAGE + SMALL_BYTES > (size_t)SMEM_BYTES) {
    if (threadIdx.x == 0) record_error(err, kErrBadArg);
    return;
  }
  uint8_t* sK = smem;
  uint8_t* sV = smem + TILE;
  uint8_t* sQ = smem + 2 * TILE;  // 2 stages
  uint8_t* sdO = smem + 4 * TILE;
  uint8_t* sPdS = smem + 5 * TILE;
  uint8_t* sStage = smem + 6 * TILE;  // 2 dQ staging buffers
  float* s_lse = reinterpret_cast<float*>(smem + 6 * TILE + 2 * STAGE);  // [2][128] -lse * log2e
  float* s_delta = s_lse + 256;                                          // [2][128] delta * scale
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_delta + 256);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;   // [2]
  uint64_t* q_empty = bars + 3;  // [2]
  uint64_t* do_full = bars + 5;
  uint64_t* do_empty = bars + 6;
  uint64_t* s_full = bars + 7;
  uint64_t* s_empty = bars + 8;
  uint64_t* dp_full = bars + 9;
  uint64_t* p_full = bars + 10;
  uint64_t* dv_done = bars + 11;
  uint64_t* ds_full = bars + 12;
  uint64_t* pds_free = bars + 13;
  uint64_t* dq_full = bars + 14;
  uint64_t* dq_empty = bars + 15;
  uint64_t* kv_done = bars + 16;
  uint64_t* drain = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wg = warp >> 2;
  const int n_t = (S + BT - 1) / BT;
  const int G = nq / nkv;
  const int j = blockIdx.x / (B * nkv);  // smallest key tile (most work) first
  const int bk = blockIdx.x % (B * nkv);
  const int b = bk / nkv, kvh = bk % nkv;
  const int i0 = causal ? j : 0;
  const int n_iter = G * (n_t - i0);
  constexpr int kElem = 256;  // two element warpgroups

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    mbar_init(do_full, 1);
    mbar_init(do_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(s_empty, kElem);
    mbar_init(dp_full, 1);
    mbar_init(p_full, kElem);
    mbar_init(dv_done, 1);
    mbar_init(ds_full, kElem);
    mbar_init(pds_free, DS_STORE ? 2 : 1);  // dK product done (+ dS tile stored)
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 128);
    mbar_init(kv_done, 1);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tdP = tmem + 128, tdV = tmem + 256, tdK = tmem + 384;

  if (wg == 0) {
    // ---------------------------------------------------------------- warpgroup 0: TMA (warp 0), MMA (warp 1)
    regs_decrease<kRegsCtl>();
    if (warp == 0 && lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmdO);
      mbar_arrive_expect_tx(kv_full, 2 * TILE);
      for (int a = 0; a < 2; ++a) {
        tma_load_3d(sK + a * (TILE / 2), &tmK, kv_full, kvh * HD + a * 64, j * BT, b);
        tma_load_3d(sV + a * (TILE / 2), &tmV, kv_full, kvh * HD + a * 64, j * BT, b);
      }
      for (int it = 0; it < n_iter; ++it) {
        const int h = kvh * G + it / (n_t - i0);
        const int i = i0 + it % (n_t - i0);
        const int st = it & 1;
        // slot 15: producer waiting for free buffers
        if (!tw(15, &q_empty[st], ((it >> 1) & 1) ^ 1)) break;
        mbar_arrive_expect_tx(&q_full[st], TILE + 1024);
        for (int a = 0; a < 2; ++a)
          tma_load_3d(sQ + st * TILE + a * (TILE / 2), &tmQ, &q_full[st], h * HD + a * 64, i * BT, b);
        const int64_t row0 = ((int64_t)b * nq + h) * S + (int64_t)i * BT;  // 16B aligned: S % 8 == 0
        bulk_load(s_lse + st * 128, LSE2 + row0, 512, &q_full[st]);
        bulk_load(s_delta + st * 128, DELTA + row0, 512, &q_full[st]);
        if (!tw(15, do_empty, (it & 1) ^ 1)) break;
        mbar_arrive_expect_tx(do_full, TILE);
        for (int a = 0; a < 2; ++a)
          tma_load_3d(sdO + a * (TILE / 2), &tmdO, do_full, h * HD + a * 64, i * BT, b);
      }
    } else if (warp == 1 && lane == 0) {
      constexpr uint32_t id_kk = idesc_bf16(128, 128, false, false);  // both K-major
      constexpr uint32_t id_km = idesc_bf16(128, 128, false, true);   // A K-major, B MN-major
      constexpr uint32_t id_mm = idesc_bf16(128, 128, true, true);    // both MN-major
      const uint32_t k_base = smem_u32(sK), v_base = smem_u32(sV), pds_base = smem_u32(sPdS);
      const uint32_t do_base = smem_u32(sdO);
      // S^T(it) = K Q_it^T into TMEM cols [0,128); slot 0 = waits for Q / S free
      auto issue_s = [&](int it) -> bool {
        const int st = it & 1;
        if (!tw(0, &q_full[st], (it >> 1) & 1) || !tw(0, s_empty, (it & 1) ^ 1)) return false;
        tc_fence_after();
        const uint32_t q_base = smem_u32(sQ + st * TILE);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * (TILE / 2) + (kk & 3) * 32;
          mma_bf16_ss(tS, smem_desc_sw128(k_base + off, 16, 1024), smem_desc_sw128(q_base + off, 16, 1024),
                      id_kk, kk > 0);
        }
        mma_commit(s_full);
        return true;
      };
      bool ok = mbar_wait(kv_full, 0, err) && (n_iter == 0 || issue_s(0));
      const long long t_mma0 = clock64();
      for (int it = 0; it < n_iter && ok; ++it) {
        const int st = it & 1;
        const uint32_t ph = it & 1;
        const uint32_t q_base = smem_u32(sQ + st * TILE);
        // slot 1: dQ(it-1) drained from TMEM, dO(it) loaded
        if ((!DS_STORE && !tw(1, dq_empty, ph ^ 1)) || !tw(1, do_full, ph)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // dP^T = V dO^T
          const uint32_t off = (kk >> 2) * (TILE / 2) + (kk & 3) * 32;
          mma_bf16_ss(tdP, smem_desc_sw128(v_base + off, 16, 1024), smem_desc_sw128(do_base + off, 16, 1024),
                      id_kk, kk > 0);
        }
        mma_commit(dp_full);
        if (!tw(2, p_full, ph)) { ok = false; break; }  // slot 2: P written into TMEM
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // dV += P^T dO   (K = queries; P^T read from TMEM)
          // element warpgroup g stored queries [64g, 64g+64) as 32 packed columns at 64g
          const uint32_t a_col = (kk >> 2) * 64 + (kk & 3) * 8;
          mma_bf16_ts(tdV, tS + a_col, smem_desc_sw128(do_base + kk * 2048, TILE / 2, 1024), id_km,
                      (it > 0 || kk > 0));
        }
        mma_commit(dv_done);
        mma_commit(do_empty);
        // S^T(it+1) overwrites P^T(it): issued after dV(it) (MMAs run in order)
        if (it + 1 < n_iter && !issue_s(it + 1)) { ok = false; break; }
        if (!tw(3, ds_full, ph)) { ok = false; break; }  // slot 3: dS written
        tc_fence_after();
        if constexpr (!DS_STORE) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {  // dQ = dS K   (K = keys; dS read MN-major)
            mma_bf16_ss(tdP, smem_desc_sw128(pds_base + kk * 2048, TILE / 2, 1024),
                        smem_desc_sw128(k_base + kk * 2048, TILE / 2, 1024), id_mm, kk > 0);
          }
          mma_commit(dq_full);
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // dK += dS^T Q   (K = queries)
          const uint32_t aoff = (kk >> 2) * (TILE / 2) + (kk & 3) * 32;
          mma_bf16_ss(tdK, smem_desc_sw128(pds_base + aoff, 16, 1024),
                      smem_desc_sw128(q_base + kk * 2048, TILE / 2, 1024), id_km, (it > 0 || kk > 0));
        }
        mma_commit(&q_empty[st]);
        mma_commit(pds_free);
      }
      if (kTrace) tacc[4] = clock64() - t_mma0;  // slot 4: MMA loop total
      if (ok) mma_commit(kv_done);
      else {
        mma_commit(drain);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(smem_u32(drain), 0) && globaltimer() - t0 < 100000000ull) {
        }
      }
    }
  } else if (wg <= 2) {
    // ---------------------------------------------------------------- warpgroups 1, 2: softmax gradient
    regs_increase<kRegsElem>();
    const int quarter = warp & 3;
    const int g = wg - 1;                     // element warpgroup
    const int cg = g * 64;                    // its query-column block
    const int r = quarter * 32 + lane;        // key row (S^T / dP^T TMEM lane)
    const int kpos = j * BT + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float scale_log2 = scale * kLog2e;
    uint8_t* pds_row = sPdS + g * (TILE / 2) + r * 128;  // this thread's row in atom g (dS)
    bool ok = true;
    const long long t_loop0 = clock64();
    long long tm = 0;
    for (int it = 0; it < n_iter && ok; ++it) {
      const int i = i0 + it % (n_t - i0);
      const uint32_t ph = it & 1;
      const int st = it & 1;
      // lse2 / delta of query tile i arrive with Q_i (bulk copies on q_full); slot 5
      if (!tw(5, &q_full[st], (it >> 1) & 1)) { ok = false; break; }
      const float* lse_t = s_lse + st * 128 + cg;
      const float* delta_t = s_delta + st * 128 + cg;
      if (!tw(6, s_full, ph)) { ok = false; break; }  // slot 6
      tc_fence_after();
      if (kTrace) tm = clock64();
      float p[64];
      tmem_ld32(tS + lane_off + cg, p);
      tmem_ld32(tS + lane_off + cg + 32, p + 32);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(s_empty);
      const bool masked = (causal && i == j) || (i + 1) * BT > S || (j + 1) * BT > S;
      if (!masked) {
#pragma unroll
        for (int c = 0; c < 64; c += 4) {
          const float4 l = *reinterpret_cast<const float4*>(lse_t + c);  // -lse * log2(e)
          p[c] = ex2(fmaf(p[c], scale_log2, l.x));
          p[c + 1] = ex2(fmaf(p[c + 1], scale_log2, l.y));
          p[c + 2] = ex2(fmaf(p[c + 2], scale_log2, l.z));
          p[c + 3] = ex2(fmaf(p[c + 3], scale_log2, l.w));
        }
      } else {
        const int q0 = i * BT + cg;
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float x = ex2(fmaf(p[c], scale_log2, lse_t[c]));
          const int q = q0 + c;
          p[c] = ((causal && kpos > q) || kpos >= S || q >= S) ? 0.f : x;
        }
      }
      // P^T packed to bf16 pairs (row = key, this warpgroup's 64 queries); the
      // packed copy is also what dS uses below (the same rounding dV sees).
      uint32_t pb[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) pb[e] = pack_bf16x2(p[2 * e], p[2 * e + 1]);
      if (kTrace) tacc[7] += clock64() - tm;  // slot 7: S -> P
      if (kTrace) tm = clock64();
      // P^T (packed bf16 pairs) over the first 32 of this warpgroup's own S^T
      // columns, which this thread has already read: the dV product's A operand
      tmem_st32(tS + lane_off + cg, reinterpret_cast<const float*>(pb));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_full);
      if (kTrace) tacc[9] += clock64() - tm;  // slot 9: P write
      if (!tw(10, dp_full, ph)) { ok = false; break; }  // slot 10
      tc_fence_after();
      if (kTrace) tm = clock64();
      uint32_t ds[32];  // dS^T row, packed bf16 pairs
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) {
        float dp[32];
        tmem_ld32(tdP + lane_off + cg + c2 * 32, dp);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          const float4 dl = *reinterpret_cast<const float4*>(delta_t + c2 * 32 + e);
          const int w = (c2 * 32 + e) / 2;
          const float2 p01 = unpack_bf16x2(pb[w]), p23 = unpack_bf16x2(pb[w + 1]);
          ds[w] = pack_bf16x2(p01.x * fmaf(dp[e], scale, -dl.x), p01.y * fmaf(dp[e + 1], scale, -dl.y));
          ds[w + 1] = pack_bf16x2(p23.x * fmaf(dp[e + 2], scale, -dl.z), p23.y * fmaf(dp[e + 3], scale, -dl.w));
        }
      }
      tc_fence_before();
      if (kTrace) tacc[11] += clock64() - tm;  // slot 11: dS compute
      // slot 12: the dS buffer is free (dQ / dK of the previous tile read it and,
      // with DS_STORE, it has been stored)
      if (!tw(12, pds_free, ph ^ 1)) { ok = false; break; }
#pragma unroll
      for (int ch = 0; ch < 8; ++ch)
        *reinterpret_cast<uint4*>(pds_row + ((ch ^ (r & 7)) << 4)) =
            make_uint4(ds[4 * ch], ds[4 * ch + 1], ds[4 * ch + 2], ds[4 * ch + 3]);
      fence_proxy_async_smem();
      mbar_arrive(ds_full);
    }
    if (kTrace) tacc[14] = clock64() - t_loop0;  // slot 14: element loop total
    if (ok && mbar_wait(kv_done, 0, err)) {
      tc_fence_after();
      const bool valid = kpos < S;
      __nv_bfloat16* dvr = dV + ((int64_t)b * S + kpos) * lddv + (int64_t)kvh * HD + cg;
      __nv_bfloat16* dkr = dK + ((int64_t)b * S + kpos) * lddk + (int64_t)kvh * HD + cg;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        const uint32_t col = (c < 2 ? tdV : tdK) + cg + (c & 1) * 32;
        tmem_ld32(col + lane_off, v);
        tmem_wait_ld();
        if (valid) {
          uint4* d4 = reinterpret_cast<uint4*>((c < 2 ? dvr : dkr) + (c & 1) * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 u;
            u.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
            u.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
            u.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
            u.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
            d4[q] = u;
          }
        }
      }
    }
  } else if (DS_STORE) {
    // ---------------------------------------------------------------- warpgroup 3: dS tile store
    regs_decrease<kRegsDq>();
    if (threadIdx.x == 3 * 128) {
      const int tiles_bh = causal ? n_t * (n_t + 1) / 2 : n_t * n_t;
      bool ok = true;
      for (int it = 0; it < n_iter && ok; ++it) {
        const int h = kvh * G + it / (n_t - i0);
        const int i = i0 + it % (n_t - i0);
        if (!tw(16, ds_full, it & 1)) { ok = false; break; }
        const int64_t tile = ((int64_t)b * nq + h) * tiles_bh + (causal ? (int64_t)i * (i + 1) / 2 : (int64_t)i * n_t) + j;
        bulk_store(ds_buf + tile * (TILE / 2), sPdS, TILE);
        bulk_commit_group();
        bulk_wait_group_read<0>();  // the P/dS buffer may be overwritten after this
        mbar_arrive(pds_free);
      }
      bulk_wait_group<0>();
    }
  } else {
    // ---------------------------------------------------------------- warpgroup 3: dQ drain
    // TMEM dQ (lane = query row) -> shared staging -> bulk tensor reduce-add
    // into the fp32 accumulator.  Each warp owns its 32 rows end to end: a
    // private ring of two 32 x 32 fp32 boxes (4 KB each), its own bulk groups,
    // no cross-warp handshakes; TMEM is released once all four column chunks
    // of every warp are in registers / staged.
    regs_decrease<kRegsDq>();
    const int quarter = warp & 3;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint8_t* ring = sStage + quarter * (2 * DQ_BOX);  // this warp's two boxes
    bool ok = true;
    int n = 0;  // chunks staged by this warp so far; chunk n uses box n & 1
    const long long t_loop0 = clock64();
    for (int it = 0; it < n_iter && ok; ++it) {
      const int h = kvh * G + it / (n_t - i0);
      const int i = i0 + it % (n_t - i0);
      if (!tw(16, dq_full, it & 1)) { ok = false; break; }  // slot 16
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < 4; ++c, ++n) {
        float v[32];
        tmem_ld32(tdP + lane_off + c * 32, v);
        tmem_wait_ld();
        if (c == 3) {  // all of this warp's dQ(it) columns are out of TMEM
          tc_fence_before();
          mbar_arrive(dq_empty);
        }
        uint8_t* box = ring + (n & 1) * DQ_BOX;
        if (lane == 0 && n >= 2) bulk_wait_group_read<1>();  // box n-2 has been read
        __syncwarp();
#pragma unroll
        for (int ch = 0; ch < 8; ++ch)
          *reinterpret_cast<float4*>(box + lane * 128 + ((ch ^ (lane & 7)) << 4)) =
              make_float4(v[ch * 4], v[ch * 4 + 1], v[ch * 4 + 2], v[ch * 4 + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_3d(&tmdQ, box, h * HD + c * 32, i * BT + quarter * 32, b);
          bulk_commit_group();
        }
      }
    }
    if (lane == 0) bulk_wait_group<0>();
    if (kTrace) tacc[19] = clock64() - t_loop0;  // slot 19: dQ loop total
  }
  if constexpr (kTrace) {
    if (threadIdx.x == 0 || threadIdx.x == 32 || threadIdx.x == 128 || threadIdx.x == 384) {
      long long* dst = trace + (int64_t)blockIdx.x * kAttnBwdTraceSlots;
#pragma unroll
      for (int i = 0; i < kSlots; ++i)
        if (tacc[i]) atomicAdd(reinterpret_cast<unsigned long long*>(dst + i), (unsigned long long)tacc[i]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// delta2[b, h, s] = scale * sum_d dO * O     (first half of `scratch`)
// nlse2[b, h, s]  = -lse * log2(e)           (second half)
// and, when dq_acc is given, zero the fp32 dQ accumulator.  A warp handles 16
// consecutive tokens of one (batch, head): a half warp per token row (16-byte
// loads, all issued before the reductions), contiguous delta / lse accesses.
// The two halves are padded by 128 zeros so the main kernel's 128-row bulk
// copies stay in bounds and finite.
__global__ void attn_bwd_prep_kernel(const __nv_bfloat16* __restrict__ O, int64_t ldo,
                                     const __nv_bfloat16* __restrict__ dO, int64_t lddo,
                                     const float* __restrict__ lse, float* __restrict__ scratch,
                                     float* __restrict__ dq_acc, int64_t ld_acc, int B, int S, int nq, float scale) {
  pdl_prologue();
  constexpr int kTok = 16;  // tokens per warp
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t rows = (int64_t)B * nq * S;
  float* delta2 = scratch;
  float* lse2 = scratch + rows + 128;
  if (gid < 128) {
    delta2[rows + gid] = 0.f;
    lse2[rows + gid] = 0.f;
  }
  const int lane = threadIdx.x & 31, hl = lane & 15, half = lane >> 4;
  const int64_t wid = gid >> 5;
  const int groups = (S + kTok - 1) / kTok;
  if (wid >= (int64_t)B * nq * groups) return;
  const int bh = (int)(wid / groups);
  const int s0 = (int)(wid % groups) * kTok;
  const int b = bh / nq, h = bh % nq;
  uint4 ov[kTok / 2], gv[kTok / 2];
#pragma unroll
  for (int k = 0; k < kTok / 2; ++k) {
    const int s = min(s0 + 2 * k + half, S - 1);
    const int64_t t = (int64_t)b * S + s;
    ov[k] = *reinterpret_cast<const uint4*>(O + t * ldo + h * HD + hl * 8);
    gv[k] = *reinterpret_cast<const uint4*>(dO + t * lddo + h * HD + hl * 8);
  }
  float mine = 0.f;  // lane 2k+half (k < 8) ends up holding token s0 + 2k + half
#pragma unroll
  for (int k = 0; k < kTok / 2; ++k) {
    const uint32_t* o32 = &ov[k].x;
    const uint32_t* g32 = &gv[k].x;
    float acc = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 a = unpack_bf16x2(o32[e]), c = unpack_bf16x2(g32[e]);
      acc += a.x * c.x + a.y * c.y;
    }
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    // acc: half-0 lanes hold token 2k, half-1 lanes token 2k+1; lanes 0..15
    // also receive the half-1 value
    const float other = __shfl_down_sync(0xffffffffu, acc, 16);
    if (lane == 2 * k) mine = acc;
    if (lane == 2 * k + 1) mine = other;
  }
  if (dq_acc) {
#pragma unroll
    for (int k = 0; k < kTok / 2; ++k) {
      const int s = s0 + 2 * k + half;
      if (s < S) {
        float4* z = reinterpret_cast<float4*>(dq_acc + ((int64_t)b * S + s) * ld_acc + h * HD + hl * 8);
        z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
        z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  }
  const int s = s0 + lane;
  if (lane < kTok && s < S) {
    const int64_t idx = (int64_t)bh * S + s;
    delta2[idx] = mine * scale;
    lse2[idx] = -lse[idx] * kLog2e;
  }
}

// dQ from the stored dS tiles: persistent CTAs walk the (query tile i, batch,
// head) items, heavy tiles first; dQ_i = sum_j dS_ij K_j accumulates in TMEM
// (double buffered, so the epilogue of one item overlaps the next item's
// products) and leaves as bf16 (dS already carries the softmax scale).  Warp
// 0 streams the dS tiles (1-D bulk copies of the stored shared-memory images)
// and the K tiles (TMA) through a 3-stage ring, warp 1 issues the MMAs, warps
// 2..5 write dq.
constexpr int DQ_STAGES = 3;
constexpr int DQ_SMEM = DQ_STAGES * 2 * TILE + 1024 + 256;

__global__ void __launch_bounds__(192, 1)
    attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmK, const __nv_bfloat16* __restrict__ ds_buf,
                       __nv_bfloat16* __restrict__ dq, int64_t lddq, int B, int S, int nq, int nkv, bool causal,
                       int* err) {
  pdl_prologue();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sDS = smem;                     // [stages][TILE]
  uint8_t* sKt = smem + DQ_STAGES * TILE;  // [stages][TILE]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 2 * DQ_STAGES * TILE);
  uint64_t* full = bars;                // [stages]
  uint64_t* empty = bars + DQ_STAGES;   // [stages]
  uint64_t* tfull = bars + 2 * DQ_STAGES;  // [2] accumulator ready
  uint64_t* tempty = tfull + 2;            // [2] accumulator drained
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_t = (S + BT - 1) / BT;
  const int n_items = B * nq * n_t;
  const int tiles_bh = causal ? n_t * (n_t + 1) / 2 : n_t * n_t;
  auto decode = [&](int w, int& qi, int& b, int& h) {
    qi = n_t - 1 - w / (B * nq);  // heaviest query tiles first
    const int rem = w % (B * nq);
    b = rem / nq;
    h = rem % nq;
  };
  if (threadIdx.x == 0) {
    for (int st = 0; st < DQ_STAGES; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      int n = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
        int qi, b, h;
        decode(w, qi, b, h);
        const int kvh = h / (nq / nkv);
        const int n_j = causal ? qi + 1 : n_t;
        const int64_t tile0 = ((int64_t)b * nq + h) * tiles_bh + (causal ? (int64_t)qi * (qi + 1) / 2 : (int64_t)qi * n_t);
        for (int jj = 0; jj < n_j; ++jj, ++n) {
          const int st = n % DQ_STAGES;
          if (!mbar_wait(&empty[st], ((n / DQ_STAGES) & 1) ^ 1, err)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[st], 2 * TILE);
          bulk_load(sDS + st * TILE, ds_buf + (tile0 + jj) * (TILE / 2), TILE, &full[st]);
          for (int a = 0; a < 2; ++a)
            tma_load_3d(sKt + st * TILE + a * (TILE / 2), &tmK, &full[st], kvh * HD + a * 64, jj * BT, b);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_mm = idesc_bf16(128, 128, true, true);  // both MN-major
      bool ok = true;
      int n = 0, local = 0;
      for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++local) {
        int qi, b, h;
        decode(w, qi, b, h);
        const int n_j = causal ? qi + 1 : n_t;
        const int acc = local & 1;
        if (!mbar_wait(&tempty[acc], ((local >> 1) & 1) ^ 1, err)) { ok = false; break; }
        tc_fence_after();
        for (int jj = 0; jj < n_j; ++jj, ++n) {
          const int st = n % DQ_STAGES;
          if (!mbar_wait(&full[st], (n / DQ_STAGES) & 1, err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t ds_base = smem_u32(sDS + st * TILE), k_base = smem_u32(sKt + st * TILE);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)  // dQ += dS K_j   (K = keys; dS^T image read MN-major)
            mma_bf16_ss(tmem + acc * 128, smem_desc_sw128(ds_base + kk * 2048, TILE / 2, 1024),
                        smem_desc_sw128(k_base + kk * 2048, TILE / 2, 1024), id_mm, (jj > 0 || kk > 0));
          mma_commit(&empty[st]);
        }
        if (ok) mma_commit(&tfull[acc]);
      }
      if (!ok) {
        mma_commit(drain);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(smem_u32(drain), 0) && globaltimer() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    int local = 0;
    for (int w = blockIdx.x; w < n_items; w += gridDim.x, ++local) {
      int qi, b, h;
      decode(w, qi, b, h);
      const int acc = local & 1;
      if (!mbar_wait(&tfull[acc], (local >> 1) & 1, err)) break;
      tc_fence_after();
      const int q = qi * BT + r;
      __nv_bfloat16* dst = dq + ((int64_t)b * S + q) * lddq + (int64_t)h * HD;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(tmem + acc * 128 + ((uint32_t)(quarter * 32) << 16) + c * 32, v);
        tmem_wait_ld();
        if (q < S) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 o;
            o.x = pack_bf16x2(v[u * 8 + 0], v[u * 8 + 1]);
            o.y = pack_bf16x2(v[u * 8 + 2], v[u * 8 + 3]);
            o.z = pack_bf16x2(v[u * 8 + 4], v[u * 8 + 5]);
            o.w = pack_bf16x2(v[u * 8 + 6], v[u * 8 + 7]);
            d4[u] = o;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

__global__ void cast_rows_kernel(const float* __restrict__ src, int64_t lds, __nv_bfloat16* __restrict__ dst,
                                 int64_t ldd, int rows, int cols) {
  pdl_prologue();
  const int64_t total = (int64_t)rows * cols / 4;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = idx * 4;
    const int r = (int)(e / cols), c = (int)(e % cols);
    float4 v = *reinterpret_cast<const float4*>(src + r * lds + c);
    uint2 o;
    o.x = pack_bf16x2(v.x, v.y);
    o.y = pack_bf16x2(v.z, v.w);
    *reinterpret_cast<uint2*>(dst + r * ldd + c) = o;
  }
}

}  // namespace

void attention_bwd(const AttnBwdParams& p, cudaStream_t s) {
  PB_CHECK(p.D == HD, "attention: head_dim must be 128");
  PB_CHECK(p.nq % p.nkv == 0, "attention: nq must be a multiple of nkv");
  PB_CHECK(p.S % 8 == 0, "attention bwd: sequence length must be a multiple of 8");
  // the dynamic shared-memory limit is a per-device function attribute
  {
    static std::mutex mu;
    static bool attr_set[64] = {false};
    int dev = 0;
    PB_CUDA_CHECK(cudaGetDevice(&dev));
    PB_CHECK(dev >= 0 && dev < 64, "attention bwd: device index out of range");
    std::lock_guard<std::mutex> lk(mu);
    if (!attr_set[dev]) {
      for (auto k : {attn_bwd_kernel<false, false>, attn_bwd_kernel<true, false>, attn_bwd_kernel<false, true>,
                     attn_bwd_kernel<true, true>})
        PB_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
      PB_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DQ_SMEM));
      attr_set[dev] = true;
    }
  }
  const bool ds_path = p.ds_buf != nullptr;
  PB_CHECK(ds_path || p.dq_acc != nullptr, "attention bwd: needs a dS tile buffer or a dQ accumulator");
  const int64_t T = (int64_t)p.B * p.S;
  const int64_t rows = (int64_t)p.B * p.nq * p.S;
  const int64_t ld_acc = (int64_t)p.nq * HD;
  const int64_t prep_threads = std::max<int64_t>((int64_t)p.B * p.nq * ((p.S + 15) / 16) * 32, 128);
  launch_k(attn_bwd_prep_kernel, (unsigned)((prep_threads + 255) / 256), 256, 0, s,
      (const __nv_bfloat16*)p.o, p.ldo, (const __nv_bfloat16*)p.dout, p.lddo, p.lse, p.delta,
      ds_path ? nullptr : p.dq_acc, ld_acc, p.B, p.S, p.nq, p.scale);
  PB_CUDA_CHECK(cudaGetLastError());
  const uint64_t S = p.S, B = p.B;
  CUtensorMap tq = make_tmap_3d_bf16(p.q, (uint64_t)p.nq * HD, S, B, p.ldq, S * p.ldq, 64, 128, 1);
  CUtensorMap tk = make_tmap_3d_bf16(p.k, (uint64_t)p.nkv * HD, S, B, p.ldk, S * p.ldk, 64, 128, 1);
  CUtensorMap tv = make_tmap_3d_bf16(p.v, (uint64_t)p.nkv * HD, S, B, p.ldv, S * p.ldv, 64, 128, 1);
  CUtensorMap tdo = make_tmap_3d_bf16(p.dout, (uint64_t)p.nq * HD, S, B, p.lddo, S * p.lddo, 64, 128, 1);
  CUtensorMap tdq{};
  if (!ds_path) tdq = make_tmap_3d_f32(p.dq_acc, (uint64_t)ld_acc, S, B, ld_acc, S * ld_acc, 32, 32, 1, true);
  const int n_t = (p.S + BT - 1) / BT;
  const int grid = p.B * p.nkv * n_t;
  auto kern = ds_path ? (p.trace ? attn_bwd_kernel<true, true> : attn_bwd_kernel<false, true>)
                      : (p.trace ? attn_bwd_kernel<true, false> : attn_bwd_kernel<false, false>);
  launch_k(kern, grid, kThreads, SMEM_BYTES, s, tq, tk, tv, tdo, tdq, p.delta + rows + 128, p.delta, (__nv_bfloat16*)p.dk,
                                          p.lddk, (__nv_bfloat16*)p.dv, p.lddv, p.B, p.S, p.nq, p.nkv, p.scale,
                                          p.causal, error_word(), p.trace, (__nv_bfloat16*)p.ds_buf);
  PB_CUDA_CHECK(cudaGetLastError());
  if (ds_path) {
    launch_k(attn_bwd_dq_kernel, std::min(num_sms(), p.B * p.nq * n_t), 192, DQ_SMEM, s, tk, (const __nv_bfloat16*)p.ds_buf,
                                                              (__nv_bfloat16*)p.dq, p.lddq, p.B, p.S, p.nq, p.nkv,
                                                              p.causal, error_word());
    PB_CUDA_CHECK(cudaGetLastError());
    return;
  }
  const int64_t cast_work = T * ld_acc / 4;
  int cgrid = (int)std::min<int64_t>((cast_work + 255) / 256, (int64_t)num_sms() * 16);
  launch_k(cast_rows_kernel, cgrid, 256, 0, s, p.dq_acc, ld_acc, (__nv_bfloat16*)p.dq, p.lddq, (int)T, (int)ld_acc);
  PB_CUDA_CHECK(cudaGetLastError());
}

int64_t attention_bwd_ds_elems(int B, int S, int nq, bool causal) {
  const int64_t n_t = (S + BT - 1) / BT;
  return (int64_t)B * nq * (causal ? n_t * (n_t + 1) / 2 : n_t * n_t) * (TILE / 2);
}

}  // namespace pb

// ===========================================================================
// Allocation-free entry point: pb_attention_bwd_noalloc
//
// This entry point has no counterpart in the reference.  It exists for callers
// that cannot allocate device memory on their own: code running inside a
// captured or externally owned stream with a fixed memory budget, plugins of
// other runtimes that forbid cudaMalloc after start-up, and allocation-free
// serving paths.  It computes the same dq / dk / dv as attention_bwd() (the
// launcher above, used by the Python bindings) but keeps every scratch buffer
// (the per-row delta, lse rescaled to base 2, the fp32 dq accumulator and the
// kernel's error word) in one file-scope __device__ array of fixed size,
// kNoAllocScratchBytes (8.5 MiB).  Every GPU that loads this library holds
// that array until the process exits.
//
//  * The caller passes inputs (q, k, v, o, dout, lse) and outputs (dq, dk, dv)
//    with the same layouts as attention_bwd(); lse needs no padding here.
//  * Problems whose scratch would exceed the array are rejected: the function
//    returns kNoAllocTooLarge and launches nothing.
//  * No cudaMalloc / cudaFree or allocating library routine is called.  The
//    first call on each device looks up the array's device address with
//    cudaGetSymbolAddress while that device is current and caches it; make
//    that first call outside any stream capture.
//  * All calls share the array and it keeps the last call's contents; the
//    parts that must start at zero are cleared on the caller's stream by each
//    call.  Calls that overlap on the GPU (different streams without ordering,
//    or different host threads on the same device) race on the array.
// ===========================================================================
namespace pb {
namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)(8u << 20) + (256u << 10);
static __device__ __align__(256) unsigned char g_attn_bwd_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocOk = 0;
constexpr int kNoAllocTooLarge = 1;
constexpr int kNoAllocBadArgs = 2;
constexpr int kNoAllocCudaError = 3;

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_base[kMaxDevices] = {nullptr};
bool g_noalloc_attr[kMaxDevices] = {false};
thread_local char g_noalloc_msg[256] = "";

void noalloc_set_msg(const char* m) {
  snprintf(g_noalloc_msg, sizeof(g_noalloc_msg), "%s", m);
}

size_t round256(size_t n) { return (n + 255) & ~size_t(255); }

}  // namespace
}  // namespace pb

extern "C" __attribute__((visibility("default"))) const char* pb_attention_bwd_noalloc_last_error() {
  return pb::g_noalloc_msg;
}

extern "C" __attribute__((visibility("default"))) size_t pb_attention_bwd_noalloc_scratch_bytes() {
  return pb::kNoAllocScratchBytes;
}

// Returns 0 on success, 1 if the problem needs more scratch than the fixed
// array holds, 2 on invalid arguments, 3 on a CUDA error (message available
// from pb_attention_bwd_noalloc_last_error()).
extern "C" __attribute__((visibility("default"))) int pb_attention_bwd_noalloc(
    const void* q, const void* k, const void* v, const void* o, const void* dout, const float* lse, void* dq,
    void* dk, void* dv, int64_t ldq, int64_t ldk, int64_t ldv, int64_t ldo, int64_t lddo, int64_t lddq,
    int64_t lddk, int64_t lddv, int B, int S, int nq, int nkv, int D, float scale, int causal,
    cudaStream_t stream) {
  using namespace pb;
  if (!q || !k || !v || !o || !dout || !lse || !dq || !dk || !dv || B <= 0 || S <= 0 || nq <= 0 || nkv <= 0 ||
      D != HD || nq % nkv != 0 || S % 8 != 0) {
    noalloc_set_msg("pb_attention_bwd_noalloc: invalid arguments (need head_dim 128, nq % nkv == 0, S % 8 == 0)");
    return kNoAllocBadArgs;
  }
  const int64_t T = (int64_t)B * S;
  const int64_t rows = (int64_t)B * nq * S;
  const int64_t ld_acc = (int64_t)nq * HD;
  // scratch layout: [err word 256 B][delta*scale, lse*log2e: 2 x (rows+128) f32][dq_acc T*ld_acc f32]
  const size_t off_delta = 256;
  const size_t off_acc = off_delta + round256((size_t)2 * (rows + 128) * sizeof(float));
  const size_t need = off_acc + (size_t)T * ld_acc * sizeof(float);
  if (need > kNoAllocScratchBytes) {
    char m[256];
    snprintf(m, sizeof(m),
             "pb_attention_bwd_noalloc: problem needs %zu scratch bytes, the fixed array holds %zu "
             "(reduce B*S*nq)",
             need, kNoAllocScratchBytes);
    noalloc_set_msg(m);
    return kNoAllocTooLarge;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    noalloc_set_msg("pb_attention_bwd_noalloc: cudaGetDevice failed");
    return kNoAllocCudaError;
  }
  unsigned char* base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_base[dev]) {
      void* ptr = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&ptr, g_attn_bwd_scratch);
      if (e != cudaSuccess || ptr == nullptr) {
        char m[256];
        snprintf(m, sizeof(m), "pb_attention_bwd_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
        noalloc_set_msg(m);
        return kNoAllocCudaError;
      }
      g_noalloc_base[dev] = ptr;
    }
    if (!g_noalloc_attr[dev]) {
      if (cudaFuncSetAttribute(attn_bwd_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
          cudaSuccess) {
        noalloc_set_msg("pb_attention_bwd_noalloc: cudaFuncSetAttribute failed");
        return kNoAllocCudaError;
      }
      g_noalloc_attr[dev] = true;
    }
    base = static_cast<unsigned char*>(g_noalloc_base[dev]);
  }
  int* err = reinterpret_cast<int*>(base);
  float* delta = reinterpret_cast<float*>(base + off_delta);
  float* dq_acc = reinterpret_cast<float*>(base + off_acc);
  try {
    // the prep kernel zeroes the dq accumulator and the scratch padding
    PB_CUDA_CHECK(cudaMemsetAsync(err, 0, 256, stream));
    const int64_t prep_threads = std::max<int64_t>((int64_t)B * nq * ((S + 15) / 16) * 32, 128);
    launch_k(attn_bwd_prep_kernel, (unsigned)((prep_threads + 255) / 256), 256, 0, stream,
        (const __nv_bfloat16*)o, ldo, (const __nv_bfloat16*)dout, lddo, lse, delta, dq_acc, ld_acc, B, S, nq, scale);
    PB_CUDA_CHECK(cudaGetLastError());
    const uint64_t uS = S, uB = B;
    CUtensorMap tq = make_tmap_3d_bf16(q, (uint64_t)nq * HD, uS, uB, ldq, uS * ldq, 64, 128, 1);
    CUtensorMap tk = make_tmap_3d_bf16(k, (uint64_t)nkv * HD, uS, uB, ldk, uS * ldk, 64, 128, 1);
    CUtensorMap tv = make_tmap_3d_bf16(v, (uint64_t)nkv * HD, uS, uB, ldv, uS * ldv, 64, 128, 1);
    CUtensorMap tdo = make_tmap_3d_bf16(dout, (uint64_t)nq * HD, uS, uB, lddo, uS * lddo, 64, 128, 1);
    CUtensorMap tdq = make_tmap_3d_f32(dq_acc, (uint64_t)ld_acc, uS, uB, ld_acc, uS * ld_acc, 32, 32, 1, true);
    const int n_t = (S + BT - 1) / BT;
    launch_k(attn_bwd_kernel<false, false>, B * nkv * n_t, kThreads, SMEM_BYTES, stream,
        tq, tk, tv, tdo, tdq, delta + rows + 128, delta, (__nv_bfloat16*)dk, lddk, (__nv_bfloat16*)dv, lddv, B, S,
        nq, nkv, scale, causal != 0, err, nullptr, nullptr);
    PB_CUDA_CHECK(cudaGetLastError());
    int sms = 0;
    PB_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int64_t cast_work = T * ld_acc / 4;
    const int cgrid = (int)std::min<int64_t>((cast_work + 255) / 256, (int64_t)sms * 16);
    launch_k(cast_rows_kernel, cgrid, 256, 0, stream, dq_acc, ld_acc, (__nv_bfloat16*)dq, lddq, (int)T, (int)ld_acc);
    PB_CUDA_CHECK(cudaGetLastError());
  } catch (const std::exception& ex) {
    noalloc_set_msg(ex.what());
    return kNoAllocCudaError;
  }
  noalloc_set_msg("");
  return kNoAllocOk;
}

// Bounded-wait status of the last call on this device (reads the error word
// kept in the scratch array; synchronises the device first).
extern "C" __attribute__((visibility("default"))) int pb_attention_bwd_noalloc_device_status() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= pb::kMaxDevices) return -1;
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lk(pb::g_noalloc_mu);  // the first call on a device writes it under the lock
    base = pb::g_noalloc_base[dev];
  }
  if (base == nullptr) return -1;
  int v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpy(&v, base, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  return v;
}
