// Causal GQA flash-attention forward on tcgen05.
//
// One CTA computes one 128-query tile for a pair of query heads that share a
// kv head (GQA groups of even size; one head per CTA otherwise), so every K / V
// tile it loads feeds two tiles of work.  Roles (384 threads, 3 warpgroups):
//   warpgroup 0, warp 0 : TMA producer - Q (both heads) once, K_j / V_j rings
//   warpgroup 0, warp 1 : TMEM allocator + MMA issuer
//   warpgroup 1 + t     : softmax of query tile t, one query row per thread
// TMEM (512 columns): S_t in [128t, 128t+128), O_t in [256 + 128t, ...).
// Per key tile j and query tile t:
//   S_t  = Q_t K_j^T            (A, B from shared memory)
//   P_t  = exp2(S_t*scale*log2e - m_t), packed bf16 into the first 64
//          columns of S_t by the softmax warps (tcgen05.st)
//   O_t += P_t V_j              (A = P_t read from TMEM, B = V_j from shared)
// The MMA warp alternates the two tiles (PV_0(j), S_0(j+1), PV_1(j),
// S_1(j+1)) so the tensor core works on one tile while the other tile's
// softmax runs, and P never touches shared memory.  MMAs of one thread run in
// issue order, so S_t(j+1) (which overwrites P_t(j)) follows PV_t(j) safely,
// and observing S_t(j+1) complete implies PV_t(j) is complete.
// The running max moves lazily (only when a row's max grew by more than 2^8);
// the final O / l does not depend on the reference max, so the result is exact.
//
// Replaces the SDPA call HF makes for every layer in the reference
// (attn_implementation="sdpa", parallel/parallel/engine/model_loading.py:22).
#include <cuda_bf16.h>

#include <algorithm>
#include <mutex>

#include "attention.cuh"
#include "host_util.h"
#include "ptx.cuh"

namespace pb {
namespace {

constexpr int BQ = 128;   // queries per tile
constexpr int BKV = 128;  // keys per tile
constexpr int HD = 128;   // head dim
constexpr int kThreads = 384;
// setmaxnreg split: 168 registers a thread at launch (65536 / 384, rounded
// down to a multiple of 8); the sum over the three warpgroups stays 3 x 168.
constexpr int kRegsCtl = 56, kRegsSoftmax = 224;
static_assert(kRegsCtl + 2 * kRegsSoftmax == 3 * 168, "attention fwd: register split");
constexpr int TILE_BYTES = 128 * HD * 2;  // 32 KB: 128 rows x 128 bf16
constexpr int SMEM_BYTES = TILE_BYTES * 6 + 1024 + 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool kTrace>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ O, int64_t ldo,
                    float* __restrict__ LSE, int B, int S, int nq, int nkv, float scale_log2, bool causal,
                    int* err, long long* trace) {
  pdl_prologue();
  // optional per-CTA phase timing (clock64 cycles, kTrace builds only)
  constexpr int kSlots = kTrace ? 16 : 1;
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
  uint8_t* sQ = smem;                    // [2 tiles]
  uint8_t* sK = smem + 2 * TILE_BYTES;   // 2 stages
  uint8_t* sV = smem + 4 * TILE_BYTES;   // 2 stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * TILE_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2 stages]
  uint64_t* k_empty = bars + 3;  // [2 stages]
  uint64_t* v_full = bars + 5;   // [2 stages]
  uint64_t* v_empty = bars + 7;  // [2 stages]
  uint64_t* s_full = bars + 9;   // [2 tiles]
  uint64_t* p_full = bars + 11;  // [2 tiles]
  uint64_t* o_full = bars + 13;
  uint64_t* drain = bars + 14;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wg = warp >> 2;
  const int G = nq / nkv;
  const int tpc = (G % 2 == 0) ? 2 : 1;  // query tiles (heads) per CTA
  const int n_hg = nq / tpc;
  const int n_qt = (S + BQ - 1) / BQ;
  const int n_kt = (S + BKV - 1) / BKV;
  const int qi = n_qt - 1 - blockIdx.x / (B * n_hg);  // heaviest tiles first
  const int rem = blockIdx.x % (B * n_hg);
  const int b = rem / n_hg;
  const int h0 = (rem % n_hg) * tpc;
  const int kvh = h0 / G;
  const int n_kv = causal ? min(qi + 1, n_kt) : n_kt;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
    }
    mbar_init(o_full, 1);
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

  if (wg == 0) {
    regs_decrease<kRegsCtl>();
    if (warp == 0 && lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, tpc * TILE_BYTES);
      for (int t = 0; t < tpc; ++t)
        for (int a = 0; a < 2; ++a)
          tma_load_3d(sQ + t * TILE_BYTES + a * (TILE_BYTES / 2), &tmQ, q_full, (h0 + t) * HD + a * 64, qi * BQ, b);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j & 1;
        const uint32_t ph = ((j >> 1) & 1) ^ 1;
        if (!tw(0, &k_empty[st], ph)) break;
        mbar_arrive_expect_tx(&k_full[st], TILE_BYTES);
        uint8_t* kd = sK + st * TILE_BYTES;
        tma_load_3d(kd, &tmK, &k_full[st], kvh * HD, j * BKV, b);
        tma_load_3d(kd + TILE_BYTES / 2, &tmK, &k_full[st], kvh * HD + 64, j * BKV, b);
        if (!tw(0, &v_empty[st], ph)) break;
        mbar_arrive_expect_tx(&v_full[st], TILE_BYTES);
        uint8_t* vd = sV + st * TILE_BYTES;
        // MN-major V: [d-block (16 KB)][key-block (8 KB)] of {64 d x 64 keys}
        for (int db = 0; db < 2; ++db)
          for (int kb = 0; kb < 2; ++kb)
            tma_load_3d(vd + db * 16384 + kb * 8192, &tmV, &v_full[st], kvh * HD + db * 64,
                        j * BKV + kb * 64, b);
      }
    } else if (warp == 1 && lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16(128, 128, false, false);
      constexpr uint32_t idesc_o = idesc_bf16(128, 128, false, true);
      bool ok = mbar_wait(q_full, 0, err);
      // S_t(j) = Q_t K_j^T
      auto issue_s = [&](int t, int j) -> bool {
        const int st = j & 1;
        if (!tw(1, &k_full[st], (j >> 1) & 1)) return false;
        tc_fence_after();
        const uint32_t q_base = smem_u32(sQ + t * TILE_BYTES);
        const uint32_t k_base = smem_u32(sK + st * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (TILE_BYTES / 2) + (kk & 3) * 32;
          mma_bf16_ss(tmem + t * 128, smem_desc_sw128(q_base + off, 16, 1024),
                      smem_desc_sw128(k_base + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[t]);
        return true;
      };
      const long long t_mma0 = clock64();
      for (int t = 0; t < tpc && ok; ++t) ok = issue_s(t, 0);
      if (ok) mma_commit(&k_empty[0]);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j & 1;
        if (!tw(2, &v_full[st], (j >> 1) & 1)) { ok = false; break; }
        const uint32_t v_base = smem_u32(sV + st * TILE_BYTES);
        for (int t = 0; t < tpc; ++t) {
          if (!tw(3, &p_full[t], j & 1)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk)  // O_t += P_t V_j, P_t from TMEM
            mma_bf16_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8,
                        smem_desc_sw128(v_base + kk * 2048, 16384, 1024), idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
          if (j + 1 < n_kv && !issue_s(t, j + 1)) { ok = false; break; }
        }
        if (!ok) break;
        mma_commit(&v_empty[st]);
        if (j + 1 < n_kv) mma_commit(&k_empty[(j + 1) & 1]);
      }
      if (kTrace) tacc[4] = clock64() - t_mma0;  // slot 4: MMA loop total
      if (ok) mma_commit(o_full);
      else {
        mma_commit(drain);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(smem_u32(drain), 0) && globaltimer() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    regs_increase<kRegsSoftmax>();
    const int t = wg - 1;  // query tile (head h0 + t)
    if (t < tpc) {
      const int h = h0 + t;
      const int quarter = warp & 3;
      const int row = quarter * 32 + lane;
      const int qpos = qi * BQ + row;
      const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
      const uint32_t tS = tmem + t * 128 + lane_off;
      const uint32_t tO = tmem + 256 + t * 128 + lane_off;
      float m_ref = -INFINITY, l = 0.f;
      bool ok = true;
      const long long t_sm0 = clock64();
      long long tm = 0;
      for (int j = 0; j < n_kv; ++j) {
        if (!tw(5, &s_full[t], j & 1)) { ok = false; break; }  // slot 5
        tc_fence_after();
        if (kTrace) tm = clock64();
        float s[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, s + c * 32);
        tmem_wait_ld();
        if (kTrace) { tacc[9] += clock64() - tm; tm = clock64(); }  // slot 9: S load
        const int kbase = j * BKV;
        const bool diag = (causal && kbase + BKV - 1 > qi * BQ) || kbase + BKV > S;
        if (diag) {
#pragma unroll
          for (int c = 0; c < 128; ++c) {
            const int kpos = kbase + c;
            if ((causal && kpos > qpos) || kpos >= S) s[c] = -INFINITY;
          }
        }
        // row max as 8 independent chains (a single 127-deep chain is latency bound)
        float m8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) m8[u] = s[u];
#pragma unroll
        for (int c = 8; c < 128; c += 8)
#pragma unroll
          for (int u = 0; u < 8; ++u) m8[u] = fmaxf(m8[u], s[c + u]);
        float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])), fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
        mx *= scale_log2;
        // lazy rescale: move the reference max only when it grew by > 2^8
        const bool need = mx > m_ref + kRescaleThreshold;
        float alpha = 1.f;
        if (need) {
          alpha = (m_ref == -INFINITY) ? 0.f : ex2(m_ref - mx);
          m_ref = mx;
        }
        const float mu = (m_ref == -INFINITY) ? 0.f : m_ref;
        float r4[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t pk[64];
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float a0 = ex2(fmaf(s[2 * c], scale_log2, -mu)), a1 = ex2(fmaf(s[2 * c + 1], scale_log2, -mu));
          r4[c & 3] += a0 + a1;
          pk[c] = pack_bf16x2(a0, a1);
        }
        const float rs = (r4[0] + r4[1]) + (r4[2] + r4[3]);
        l = l * alpha + rs;
        if (kTrace) { tacc[10] += clock64() - tm; tm = clock64(); }  // slot 10: max + exp
        // O_t rescale: PV_t(j-1) is complete (S_t(j) was issued after it)
        if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(tO + c * 32, o);
          }
        }
        if (kTrace) { tacc[7] += clock64() - tm; tm = clock64(); }  // slot 7: O rescale
        // P_t (bf16 pairs) over the first 64 columns of S_t
        tmem_st32(tS, reinterpret_cast<const float*>(pk));
        tmem_st32(tS + 32, reinterpret_cast<const float*>(pk + 32));
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[t]);
        if (kTrace) tacc[11] += clock64() - tm;  // slot 11: P store
      }
      if (kTrace) tacc[8] = clock64() - t_sm0;  // slot 8: softmax loop total
      if (ok && mbar_wait(o_full, 0, err)) {
        tc_fence_after();
        const float inv_l = l > 0.f ? 1.f / l : 0.f;
        const bool valid = qpos < S;
        __nv_bfloat16* orow = O + ((int64_t)b * S + qpos) * ldo + (int64_t)h * HD;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
          if (valid) {
            uint4* d4 = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 u;
              u.x = pack_bf16x2(o[q * 8 + 0] * inv_l, o[q * 8 + 1] * inv_l);
              u.y = pack_bf16x2(o[q * 8 + 2] * inv_l, o[q * 8 + 3] * inv_l);
              u.z = pack_bf16x2(o[q * 8 + 4] * inv_l, o[q * 8 + 5] * inv_l);
              u.w = pack_bf16x2(o[q * 8 + 6] * inv_l, o[q * 8 + 7] * inv_l);
              d4[q] = u;
            }
          }
        }
        if (valid && LSE)
          LSE[((int64_t)b * nq + h) * S + qpos] = (m_ref + __log2f(l)) * 0.6931471805599453f;
      }
    }
  }
  if constexpr (kTrace) {
    if (threadIdx.x == 0 || threadIdx.x == 32 || threadIdx.x == 128) {
      long long* dst = trace + (int64_t)blockIdx.x * 16;
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

}  // namespace

void attention_fwd(const AttnParams& p, cudaStream_t s) {
  PB_CHECK(p.D == HD, "attention: head_dim must be 128");
  PB_CHECK(p.nq % p.nkv == 0, "attention: nq must be a multiple of nkv");
  // the dynamic shared-memory limit is a per-device function attribute
  {
    static std::mutex mu;
    static bool attr_set[64] = {false};
    int dev = 0;
    PB_CUDA_CHECK(cudaGetDevice(&dev));
    PB_CHECK(dev >= 0 && dev < 64, "attention fwd: device index out of range");
    std::lock_guard<std::mutex> lk(mu);
    if (!attr_set[dev]) {
      for (auto k : {attn_fwd_kernel<false>, attn_fwd_kernel<true>})
        PB_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
      attr_set[dev] = true;
    }
  }
  const uint64_t S = p.S, B = p.B;
  CUtensorMap tq = make_tmap_3d_bf16(p.q, (uint64_t)p.nq * HD, S, B, p.ldq, S * p.ldq, 64, 128, 1);
  CUtensorMap tk = make_tmap_3d_bf16(p.k, (uint64_t)p.nkv * HD, S, B, p.ldk, S * p.ldk, 64, 128, 1);
  CUtensorMap tv = make_tmap_3d_bf16(p.v, (uint64_t)p.nkv * HD, S, B, p.ldv, S * p.ldv, 64, 64, 1);
  const int G = p.nq / p.nkv;
  const int tpc = (G % 2 == 0) ? 2 : 1;
  const int n_qt = (p.S + BQ - 1) / BQ;
  const int grid = p.B * (p.nq / tpc) * n_qt;
  auto kern = p.trace ? attn_fwd_kernel<true> : attn_fwd_kernel<false>;
  launch_k(kern, grid, kThreads, SMEM_BYTES, s, tq, tk, tv, (__nv_bfloat16*)p.o, p.ldo, p.lse, p.B, p.S, p.nq, p.nkv,
                                          p.scale * kLog2e, p.causal, error_word(), p.trace);
  PB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace pb
