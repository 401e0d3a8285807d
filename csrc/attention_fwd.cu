// Causal GQA flash-attention forward on tcgen05.
//
// One CTA computes a 128-query tile of one (batch, head).  Roles (192 thr):
//   warp 0     : TMA producer - Q once, then K_j / V_j into 2-deep rings
//   warp 1     : TMEM allocator + MMA issuer:  S_j = Q K_j^T (TMEM, double
//                buffered), O += P_j V_j (TMEM accumulator)
//   warps 2..5 : softmax - one query row per thread; reads S_j from TMEM,
//                keeps the running max / sum in registers, writes P_j (bf16,
//                128B-swizzled) to shared memory for the PV MMA, and rescales
//                O in TMEM only when a row's max grew by more than 2^8
//                (exact: the final O / l does not depend on the reference max)
// S_{j+1} is issued before PV_j so the tensor core overlaps the softmax.
//
// Replaces the SDPA call HF makes for every layer in the reference
// (attn_implementation="sdpa", parallel/parallel/engine/model_loading.py:22).
#include <cuda_bf16.h>

#include <algorithm>

#include "attention.cuh"
#include "host_util.h"
#include "ptx.cuh"

namespace pb {
namespace {

constexpr int BQ = 128;       // queries per CTA
constexpr int BKV = 128;      // keys per tile
constexpr int HD = 128;       // head dim
constexpr int kThreads = 192;
constexpr int TILE_BYTES = 128 * HD * 2;  // 32 KB: 128 rows x 128 bf16
constexpr int SMEM_BYTES = TILE_BYTES * 6 + 1024 + 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ O, int64_t ldo,
                    float* __restrict__ LSE, int B, int S, int nq, int nkv, float scale_log2, bool causal,
                    int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + TILE_BYTES;       // 2 stages
  uint8_t* sV = smem + 3 * TILE_BYTES;   // 2 stages
  uint8_t* sP = smem + 5 * TILE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * TILE_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* s_empty = bars + 11; // [2]
  uint64_t* p_full = bars + 13;
  uint64_t* p_empty = bars + 14;
  uint64_t* o_full = bars + 15;
  uint64_t* drain = bars + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (S + BQ - 1) / BQ;
  const int bh = blockIdx.x % (B * nq);
  const int qi = n_qt - 1 - blockIdx.x / (B * nq);  // heaviest tiles first
  const int b = bh / nq, h = bh % nq;
  const int kvh = h / (nq / nkv);
  const int n_kv = causal ? min(qi + 1, (S + BKV - 1) / BKV) : (S + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(p_empty, 1);
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
  const uint32_t tS = tmem;        // 2 x 128 columns
  const uint32_t tO = tmem + 256;  // 128 columns

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, TILE_BYTES);
      tma_load_3d(sQ, &tmQ, q_full, h * HD, qi * BQ, b);
      tma_load_3d(sQ + TILE_BYTES / 2, &tmQ, q_full, h * HD + 64, qi * BQ, b);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j & 1;
        const uint32_t ph = ((j >> 1) & 1) ^ 1;
        if (!mbar_wait(&k_empty[st], ph, err)) break;
        mbar_arrive_expect_tx(&k_full[st], TILE_BYTES);
        uint8_t* kd = sK + st * TILE_BYTES;
        tma_load_3d(kd, &tmK, &k_full[st], kvh * HD, j * BKV, b);
        tma_load_3d(kd + TILE_BYTES / 2, &tmK, &k_full[st], kvh * HD + 64, j * BKV, b);
        if (!mbar_wait(&v_empty[st], ph, err)) break;
        mbar_arrive_expect_tx(&v_full[st], TILE_BYTES);
        uint8_t* vd = sV + st * TILE_BYTES;
        // MN-major V: [d-block (16 KB)][key-block (8 KB)] of {64 d x 64 keys}
        for (int db = 0; db < 2; ++db)
          for (int kb = 0; kb < 2; ++kb)
            tma_load_3d(vd + db * 16384 + kb * 8192, &tmV, &v_full[st], kvh * HD + db * 64,
                        j * BKV + kb * 64, b);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16(128, 128, false, false);
      constexpr uint32_t idesc_o = idesc_bf16(128, 128, false, true);
      const uint32_t q_base = smem_u32(sQ);
      const uint32_t p_base = smem_u32(sP);
      bool ok = mbar_wait(q_full, 0, err);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(&k_full[st], (j >> 1) & 1, err)) return false;
        if (!mbar_wait(&s_empty[st], ((j >> 1) & 1) ^ 1, err)) return false;
        tc_fence_after();
        const uint32_t k_base = smem_u32(sK + st * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (TILE_BYTES / 2) + (kk & 3) * 32;
          mma_bf16_ss(tS + st * 128, smem_desc_sw128(q_base + off, 16, 1024),
                      smem_desc_sw128(k_base + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
        mma_commit(&k_empty[st]);
        mma_commit(&s_full[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < n_kv && ok; ++j) {
        if (j + 1 < n_kv && !issue_s(j + 1)) { ok = false; break; }
        const int st = j & 1;
        if (!mbar_wait(p_full, j & 1, err)) { ok = false; break; }
        if (!mbar_wait(&v_full[st], (j >> 1) & 1, err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t v_base = smem_u32(sV + st * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
          const uint32_t poff = (kk >> 2) * (TILE_BYTES / 2) + (kk & 3) * 32;
          mma_bf16_ss(tO, smem_desc_sw128(p_base + poff, 16, 1024),
                      smem_desc_sw128(v_base + kk * 2048, 16384, 1024), idesc_o,
                      (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&v_empty[st]);
        mma_commit(p_empty);
      }
      if (ok) mma_commit(o_full);
      else {
        mma_commit(drain);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(smem_u32(drain), 0) && globaltimer() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    // softmax warps: thread owns query row `row` of the tile
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int qpos = qi * BQ + row;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int st = j & 1;
      if (!mbar_wait(&s_full[st], (j >> 1) & 1, err)) { ok = false; break; }
      tc_fence_after();
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + lane_off + st * 128 + c * 32, s + c * 32);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_empty[st]);
      const int kbase = j * BKV;
      const bool diag = (causal && kbase + BKV - 1 > qi * BQ) || kbase + BKV > S;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        float x = s[c] * scale_log2;
        if (diag) {
          const int kpos = kbase + c;
          if ((causal && kpos > qpos) || kpos >= S) x = -INFINITY;
        }
        s[c] = x;
        mx = fmaxf(mx, x);
      }
      // lazy rescale: move the reference max only when it grew by > 2^8
      const bool need = mx > m_ref + kRescaleThreshold;
      float alpha = 1.f;
      if (need) {
        alpha = (m_ref == -INFINITY) ? 0.f : ex2(m_ref - mx);
        m_ref = mx;
      }
      const float mu = (m_ref == -INFINITY) ? 0.f : m_ref;
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        s[c] = ex2(s[c] - mu);
        rs += s[c];
      }
      l = l * alpha + rs;
      if (j > 0) {
        if (!mbar_wait(p_empty, (j - 1) & 1, err)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float o[32];
            tmem_ld32(tO + lane_off + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(tO + lane_off + c * 32, o);
          }
          tmem_wait_st();
        }
      }
      // P (bf16) -> smem, K-major 128B swizzle: atom (64 keys) x row x 16B chunk
#pragma unroll
      for (int a = 0; a < 2; ++a) {
        uint8_t* rowp = sP + a * (TILE_BYTES / 2) + row * 128;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const float* pv = s + a * 64 + ch * 8;
          uint4 u;
          u.x = pack_bf16x2(pv[0], pv[1]);
          u.y = pack_bf16x2(pv[2], pv[3]);
          u.z = pack_bf16x2(pv[4], pv[5]);
          u.w = pack_bf16x2(pv[6], pv[7]);
          *reinterpret_cast<uint4*>(rowp + ((ch ^ (row & 7)) << 4)) = u;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && mbar_wait(o_full, 0, err)) {
      tc_fence_after();
      const float inv_l = l > 0.f ? 1.f / l : 0.f;
      const bool valid = qpos < S;
      __nv_bfloat16* orow = O + ((int64_t)b * S + qpos) * ldo + (int64_t)h * HD;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float o[32];
        tmem_ld32(tO + lane_off + c * 32, o);
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
      if (valid && LSE) LSE[(int64_t)bh * S + qpos] = (m_ref + __log2f(l)) * 0.6931471805599453f;
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
  static bool attr = false;
  if (!attr) {
    PB_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       SMEM_BYTES));
    attr = true;
  }
  const uint64_t S = p.S, B = p.B;
  CUtensorMap tq = make_tmap_3d_bf16(p.q, (uint64_t)p.nq * HD, S, B, p.ldq, S * p.ldq, 64, 128, 1);
  CUtensorMap tk = make_tmap_3d_bf16(p.k, (uint64_t)p.nkv * HD, S, B, p.ldk, S * p.ldk, 64, 128, 1);
  CUtensorMap tv = make_tmap_3d_bf16(p.v, (uint64_t)p.nkv * HD, S, B, p.ldv, S * p.ldv, 64, 64, 1);
  const int n_qt = (p.S + BQ - 1) / BQ;
  const int grid = p.B * p.nq * n_qt;
  attn_fwd_kernel<<<grid, kThreads, SMEM_BYTES, s>>>(tq, tk, tv, (__nv_bfloat16*)p.o, p.ldo, p.lse, p.B,
                                                     p.S, p.nq, p.nkv, p.scale * kLog2e, p.causal,
                                                     error_word());
  PB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace pb
