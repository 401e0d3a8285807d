// Causal GQA flash-attention backward on tcgen05.
//
// One CTA owns a 128-key tile j of one (batch, kv-head) and loops over every
// query head of the GQA group and every query tile i that can see tile j.
// Per (head, i), with K_j / V_j resident in shared memory:
//   S^T  = K_j Q_i^T            -> TMEM cols [  0,128)  (lane = key)
//   dP^T = V_j dO_i^T           -> TMEM cols [128,256)
//   P^T  = exp(S^T*scale - lse) -> smem (bf16)              [elementwise warps]
//   dV  += P^T dO_i             -> TMEM cols [256,384)
//   dS^T = P^T (dP^T - delta) * scale -> smem (same buffer, after dV read P)
//   dK  += dS^T Q_i             -> TMEM cols [384,512)
//   dQ_i = dS K_j               -> TMEM cols [128,256)  (dP^T is consumed by then)
// dQ_i is added into an fp32 accumulator with vector atomics; dK / dV leave
// TMEM once at the end.  Every operand tile is loaded once in the K-major
// 128B-swizzled layout and re-read as MN-major where a product needs its
// transpose (same bytes, different descriptor strides).
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
constexpr int kThreads = 192;
constexpr int TILE = 128 * HD * 2;  // 32 KB
// 7 tiles + double-buffered lse/delta (2 x 1 KB) + 21 barriers + TMEM slot.
constexpr int SMALL_BYTES = 2048 + 22 * 8;
constexpr int SMEM_BYTES = 232448;  // the sm_100 per-block maximum
static_assert(7 * TILE + SMALL_BYTES <= SMEM_BYTES, "attention bwd: smem budget");
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                    const float* __restrict__ LSE, const float* __restrict__ DELTA,
                    float* __restrict__ dq_acc, int64_t ld_dqacc, __nv_bfloat16* __restrict__ dK,
                    int64_t lddk, __nv_bfloat16* __restrict__ dV, int64_t lddv, int B, int S, int nq,
                    int nkv, float scale, bool causal, int* err, long long* trace) {
  // optional per-CTA phase timing (clock64 cycles), slots documented at the use sites
  long long tacc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) tacc[i] = 0;
  auto tw = [&](int slot, uint64_t* bar, uint32_t par) -> bool {
    if (!trace) return mbar_wait(bar, par, err);
    const long long t0 = clock64();
    const bool r = mbar_wait(bar, par, err);
    tacc[slot] += clock64() - t0;
    return r;
  };
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  // The 128B-swizzled tiles need 1024-byte alignment; the budget leaves
  // SMEM_BYTES - 7*TILE - SMALL_BYTES bytes for it.  Bail out (uniformly,
  // before any barrier or TMEM use) if the dynamic window is aligned worse.
  if ((size_t)(smem - smem_raw) + 7 * TILE + SMALL_BYTES > (size_t)SMEM_BYTES) {
    if (threadIdx.x == 0) record_error(err, kErrBadArg);
    return;
  }
  uint8_t* sK = smem;
  uint8_t* sV = smem + TILE;
  uint8_t* sQ = smem + 2 * TILE;   // 2 stages
  uint8_t* sdO = smem + 4 * TILE;  // 2 stages
  uint8_t* sPdS = smem + 6 * TILE;
  float* s_lse = reinterpret_cast<float*>(smem + 7 * TILE);  // [2][128]
  float* s_delta = s_lse + 256;                               // [2][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_delta + 256);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;    // [2]
  uint64_t* q_empty = bars + 3;   // [2]
  uint64_t* do_full = bars + 5;   // [2]
  uint64_t* do_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;
  uint64_t* s_empty = bars + 10;
  uint64_t* dp_full = bars + 11;
  uint64_t* p_full = bars + 12;
  uint64_t* dv_done = bars + 13;
  uint64_t* ds_full = bars + 14;
  uint64_t* pds_free = bars + 15;
  uint64_t* dq_full = bars + 16;
  uint64_t* dq_empty = bars + 17;
  uint64_t* kv_done = bars + 18;
  uint64_t* drain = bars + 19;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_t = (S + BT - 1) / BT;
  const int G = nq / nkv;
  const int j = blockIdx.x / (B * nkv);  // smallest key tile (most work) first
  const int bk = blockIdx.x % (B * nkv);
  const int b = bk / nkv, kvh = bk % nkv;
  const int i0 = causal ? j : 0;
  const int n_iter = G * (n_t - i0);

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
      mbar_init(&do_full[s], 1);
      mbar_init(&do_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, 128);
    mbar_init(dp_full, 1);
    mbar_init(p_full, 128);
    mbar_init(dv_done, 1);
    mbar_init(ds_full, 128);
    mbar_init(pds_free, 1);
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

  if (warp == 0) {
    if (lane == 0) {
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
        const uint32_t ph = ((it >> 1) & 1) ^ 1;
        if (!tw(15, &q_empty[st], ph)) break;
        mbar_arrive_expect_tx(&q_full[st], TILE + 1024);
        for (int a = 0; a < 2; ++a)
          tma_load_3d(sQ + st * TILE + a * (TILE / 2), &tmQ, &q_full[st], h * HD + a * 64, i * BT, b);
        const int64_t row0 = ((int64_t)b * nq + h) * S + (int64_t)i * BT;  // 16B aligned: S % 8 == 0
        bulk_load(s_lse + st * 128, LSE + row0, 512, &q_full[st]);
        bulk_load(s_delta + st * 128, DELTA + row0, 512, &q_full[st]);
        if (!tw(15, &do_empty[st], ph)) break;
        mbar_arrive_expect_tx(&do_full[st], TILE);
        for (int a = 0; a < 2; ++a)
          tma_load_3d(sdO + st * TILE + a * (TILE / 2), &tmdO, &do_full[st], h * HD + a * 64, i * BT, b);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_kk = idesc_bf16(128, 128, false, false);  // both K-major
      constexpr uint32_t id_km = idesc_bf16(128, 128, false, true);   // A K-major, B MN-major
      constexpr uint32_t id_mm = idesc_bf16(128, 128, true, true);    // both MN-major
      const uint32_t k_base = smem_u32(sK), v_base = smem_u32(sV), pds_base = smem_u32(sPdS);
      bool ok = mbar_wait(kv_full, 0, err);
      const long long t_mma0 = clock64();
      for (int it = 0; it < n_iter && ok; ++it) {
        const int st = it & 1;
        const uint32_t ph = it & 1;
        const uint32_t q_base = smem_u32(sQ + st * TILE), do_base = smem_u32(sdO + st * TILE);
        if (!tw(0, &q_full[st], (it >> 1) & 1) || !tw(0, &do_full[st], (it >> 1) & 1) ||
            !tw(0, s_empty, ph ^ 1)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // S^T = K Q^T   (K = head dim)
          const uint32_t off = (kk >> 2) * (TILE / 2) + (kk & 3) * 32;
          mma_bf16_ss(tS, smem_desc_sw128(k_base + off, 16, 1024), smem_desc_sw128(q_base + off, 16, 1024),
                      id_kk, kk > 0);
        }
        mma_commit(s_full);
        if (!tw(1, dq_empty, ph ^ 1)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // dP^T = V dO^T
          const uint32_t off = (kk >> 2) * (TILE / 2) + (kk & 3) * 32;
          mma_bf16_ss(tdP, smem_desc_sw128(v_base + off, 16, 1024), smem_desc_sw128(do_base + off, 16, 1024),
                      id_kk, kk > 0);
        }
        mma_commit(dp_full);
        if (!tw(2, p_full, ph)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // dV += P^T dO   (K = queries)
          const uint32_t aoff = (kk >> 2) * (TILE / 2) + (kk & 3) * 32;
          mma_bf16_ss(tdV, smem_desc_sw128(pds_base + aoff, 16, 1024),
                      smem_desc_sw128(do_base + kk * 2048, TILE / 2, 1024), id_km, (it > 0 || kk > 0));
        }
        mma_commit(dv_done);
        if (!tw(3, ds_full, ph)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // dK += dS^T Q   (K = queries)
          const uint32_t aoff = (kk >> 2) * (TILE / 2) + (kk & 3) * 32;
          mma_bf16_ss(tdK, smem_desc_sw128(pds_base + aoff, 16, 1024),
                      smem_desc_sw128(q_base + kk * 2048, TILE / 2, 1024), id_km, (it > 0 || kk > 0));
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // dQ = dS K   (K = keys; dS read MN-major)
          mma_bf16_ss(tdP, smem_desc_sw128(pds_base + kk * 2048, TILE / 2, 1024),
                      smem_desc_sw128(k_base + kk * 2048, TILE / 2, 1024), id_mm, kk > 0);
        }
        mma_commit(&q_empty[st]);
        mma_commit(&do_empty[st]);
        mma_commit(pds_free);
        mma_commit(dq_full);
      }
      if (trace) tacc[4] = clock64() - t_mma0;
      if (ok) mma_commit(kv_done);
      else {
        mma_commit(drain);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(smem_u32(drain), 0) && globaltimer() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;        // key row within the tile (TMEM lane)
    const int kpos = j * BT + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float scale_log2 = scale * kLog2e;
    bool ok = true;
    const long long t_loop0 = clock64();
    long long tm = 0;
    for (int it = 0; it < n_iter; ++it) {
      const int h = kvh * G + it / (n_t - i0);
      const int i = i0 + it % (n_t - i0);
      const uint32_t ph = it & 1;
      const int st = it & 1;
      // lse / delta of query tile i arrive with Q_i (bulk copies on q_full)
      if (!tw(5, &q_full[st], (it >> 1) & 1)) { ok = false; break; }
      const float* lse_t = s_lse + st * 128;
      const float* delta_t = s_delta + st * 128;
      if (!tw(6, s_full, ph)) { ok = false; break; }
      tc_fence_after();
      if (trace) tm = clock64();
      float p[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + lane_off + c * 32, p + c * 32);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(s_empty);
      const bool diag = causal && (i == j);
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        float x = ex2(p[c] * scale_log2 - lse_t[c] * kLog2e);
        if ((diag && kpos > i * BT + c) || kpos >= S || i * BT + c >= S) x = 0.f;
        p[c] = x;
      }
      if (trace) tacc[7] += clock64() - tm;
      if (!tw(8, pds_free, ph ^ 1)) { ok = false; break; }
      if (trace) tm = clock64();
      // P^T -> smem (row = key, 128 queries in two 64-wide swizzled atoms)
#pragma unroll
      for (int a = 0; a < 2; ++a) {
        uint8_t* rowp = sPdS + a * (TILE / 2) + r * 128;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const float* pv = p + a * 64 + ch * 8;
          uint4 u;
          u.x = pack_bf16x2(pv[0], pv[1]);
          u.y = pack_bf16x2(pv[2], pv[3]);
          u.z = pack_bf16x2(pv[4], pv[5]);
          u.w = pack_bf16x2(pv[6], pv[7]);
          *reinterpret_cast<uint4*>(rowp + ((ch ^ (r & 7)) << 4)) = u;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
      if (trace) tacc[9] += clock64() - tm;
      if (!tw(10, dp_full, ph) || !tw(10, dv_done, ph)) { ok = false; break; }
      tc_fence_after();
      if (trace) tm = clock64();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float dp[32];
        tmem_ld32(tdP + lane_off + c * 32, dp);
        tmem_wait_ld();
        const int a = c >> 1;
        uint8_t* rowp = sPdS + a * (TILE / 2) + r * 128;
#pragma unroll
        for (int ch4 = 0; ch4 < 4; ++ch4) {
          const int ch = (c & 1) * 4 + ch4;  // 16-byte chunk within the 64-query atom
          float d[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int q = c * 32 + ch4 * 8 + e;
            const float dl = (i * BT + q < S) ? delta_t[q] : 0.f;
            d[e] = p[q] * (dp[ch4 * 8 + e] - dl) * scale;
          }
          uint4 u;
          u.x = pack_bf16x2(d[0], d[1]);
          u.y = pack_bf16x2(d[2], d[3]);
          u.z = pack_bf16x2(d[4], d[5]);
          u.w = pack_bf16x2(d[6], d[7]);
          *reinterpret_cast<uint4*>(rowp + ((ch ^ (r & 7)) << 4)) = u;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(ds_full);
      if (trace) tacc[11] += clock64() - tm;
      if (!tw(12, dq_full, ph)) { ok = false; break; }
      tc_fence_after();
      if (trace) tm = clock64();
      {
        const int q = i * BT + r;  // dQ lane = query row
        float* dst = dq_acc + ((int64_t)b * S + q) * ld_dqacc + (int64_t)h * HD;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld32(tdP + lane_off + c * 32, v);
          tmem_wait_ld();
          if (q < S) {
#pragma unroll
            for (int e = 0; e < 32; e += 4)
              atomicAdd(reinterpret_cast<float4*>(dst + c * 32 + e), make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(dq_empty);
      if (trace) tacc[13] += clock64() - tm;
    }
    if (trace) tacc[14] = clock64() - t_loop0;
    if (ok && mbar_wait(kv_done, 0, err)) {
      tc_fence_after();
      const bool valid = kpos < S;
      __nv_bfloat16* dvr = dV + ((int64_t)b * S + kpos) * lddv + (int64_t)kvh * HD;
      __nv_bfloat16* dkr = dK + ((int64_t)b * S + kpos) * lddk + (int64_t)kvh * HD;
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        float v[32];
        const uint32_t col = (c < 4 ? tdV : tdK) + (c & 3) * 32;
        tmem_ld32(col + lane_off, v);
        tmem_wait_ld();
        if (valid) {
          uint4* d4 = reinterpret_cast<uint4*>((c < 4 ? dvr : dkr) + (c & 3) * 32);
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
  }
  if (trace && (threadIdx.x == 0 || threadIdx.x == 32 || threadIdx.x == 64)) {
    long long* dst = trace + (int64_t)blockIdx.x * 16;
    for (int i = 0; i < 16; ++i)
      if (tacc[i]) atomicAdd(reinterpret_cast<unsigned long long*>(dst + i), (unsigned long long)tacc[i]);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// delta[b, h, s] = sum_d dO * O   (one warp per (token, head))
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ O, int64_t ldo,
                                  const __nv_bfloat16* __restrict__ dO, int64_t lddo, float* __restrict__ delta,
                                  int B, int S, int nq) {
  const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (item >= B * S * nq) return;
  const int t = item / nq, h = item % nq;
  const __nv_bfloat16* o = O + (int64_t)t * ldo + h * HD + lane * 4;
  const __nv_bfloat16* g = dO + (int64_t)t * lddo + h * HD + lane * 4;
  uint2 ov = *reinterpret_cast<const uint2*>(o);
  uint2 gv = *reinterpret_cast<const uint2*>(g);
  float2 o0 = unpack_bf16x2(ov.x), o1 = unpack_bf16x2(ov.y), g0 = unpack_bf16x2(gv.x), g1 = unpack_bf16x2(gv.y);
  float acc = o0.x * g0.x + o0.y * g0.y + o1.x * g1.x + o1.y * g1.y;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    const int b = t / S, s = t % S;
    delta[((int64_t)b * nq + h) * S + s] = acc;
  }
}

__global__ void cast_rows_kernel(const float* __restrict__ src, int64_t lds, __nv_bfloat16* __restrict__ dst,
                                 int64_t ldd, int rows, int cols) {
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
  static bool attr = false;
  if (!attr) {
    PB_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       SMEM_BYTES));
    attr = true;
  }
  const int T = p.B * p.S;
  const int items = T * p.nq;
  attn_delta_kernel<<<(items + 7) / 8, 256, 0, s>>>((const __nv_bfloat16*)p.o, p.ldo,
                                                    (const __nv_bfloat16*)p.dout, p.lddo, p.delta, p.B, p.S,
                                                    p.nq);
  PB_CUDA_CHECK(cudaGetLastError());
  const int64_t ld_acc = (int64_t)p.nq * HD;
  PB_CUDA_CHECK(cudaMemsetAsync(p.dq_acc, 0, (size_t)T * ld_acc * sizeof(float), s));
  const uint64_t S = p.S, B = p.B;
  CUtensorMap tq = make_tmap_3d_bf16(p.q, (uint64_t)p.nq * HD, S, B, p.ldq, S * p.ldq, 64, 128, 1);
  CUtensorMap tk = make_tmap_3d_bf16(p.k, (uint64_t)p.nkv * HD, S, B, p.ldk, S * p.ldk, 64, 128, 1);
  CUtensorMap tv = make_tmap_3d_bf16(p.v, (uint64_t)p.nkv * HD, S, B, p.ldv, S * p.ldv, 64, 128, 1);
  CUtensorMap tdo = make_tmap_3d_bf16(p.dout, (uint64_t)p.nq * HD, S, B, p.lddo, S * p.lddo, 64, 128, 1);
  const int n_t = (p.S + BT - 1) / BT;
  const int grid = p.B * p.nkv * n_t;
  attn_bwd_kernel<<<grid, kThreads, SMEM_BYTES, s>>>(tq, tk, tv, tdo, p.lse, p.delta, p.dq_acc, ld_acc,
                                                     (__nv_bfloat16*)p.dk, p.lddk, (__nv_bfloat16*)p.dv, p.lddv,
                                                     p.B, p.S, p.nq, p.nkv, p.scale, p.causal, error_word(),
                                                     p.trace);
  PB_CUDA_CHECK(cudaGetLastError());
  const int64_t cast_work = (int64_t)T * ld_acc / 4;
  int cgrid = (int)std::min<int64_t>((cast_work + 255) / 256, (int64_t)num_sms() * 16);
  cast_rows_kernel<<<cgrid, 256, 0, s>>>(p.dq_acc, ld_acc, (__nv_bfloat16*)p.dq, p.lddq, T, (int)ld_acc);
  PB_CUDA_CHECK(cudaGetLastError());
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
// (the per-row delta, a padded copy of lse, the fp32 dq accumulator and the
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
  // scratch layout: [err word 256 B][delta (rows+128) f32][lse copy (rows+128) f32][dq_acc T*ld_acc f32]
  const size_t off_delta = 256;
  const size_t off_lse = off_delta + round256((size_t)(rows + 128) * sizeof(float));
  const size_t off_acc = off_lse + round256((size_t)(rows + 128) * sizeof(float));
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
      if (cudaFuncSetAttribute(attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
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
  float* lse_pad = reinterpret_cast<float*>(base + off_lse);
  float* dq_acc = reinterpret_cast<float*>(base + off_acc);
  try {
    // zero what must start at zero: error word, delta / lse padding, dq accumulator
    PB_CUDA_CHECK(cudaMemsetAsync(err, 0, 256, stream));
    PB_CUDA_CHECK(cudaMemsetAsync(delta + rows, 0, 128 * sizeof(float), stream));
    PB_CUDA_CHECK(cudaMemcpyAsync(lse_pad, lse, (size_t)rows * sizeof(float), cudaMemcpyDeviceToDevice, stream));
    PB_CUDA_CHECK(cudaMemsetAsync(lse_pad + rows, 0, 128 * sizeof(float), stream));
    PB_CUDA_CHECK(cudaMemsetAsync(dq_acc, 0, (size_t)T * ld_acc * sizeof(float), stream));
    const int items = (int)(T * nq);
    attn_delta_kernel<<<(items + 7) / 8, 256, 0, stream>>>((const __nv_bfloat16*)o, ldo,
                                                           (const __nv_bfloat16*)dout, lddo, delta, B, S, nq);
    PB_CUDA_CHECK(cudaGetLastError());
    const uint64_t uS = S, uB = B;
    CUtensorMap tq = make_tmap_3d_bf16(q, (uint64_t)nq * HD, uS, uB, ldq, uS * ldq, 64, 128, 1);
    CUtensorMap tk = make_tmap_3d_bf16(k, (uint64_t)nkv * HD, uS, uB, ldk, uS * ldk, 64, 128, 1);
    CUtensorMap tv = make_tmap_3d_bf16(v, (uint64_t)nkv * HD, uS, uB, ldv, uS * ldv, 64, 128, 1);
    CUtensorMap tdo = make_tmap_3d_bf16(dout, (uint64_t)nq * HD, uS, uB, lddo, uS * lddo, 64, 128, 1);
    const int n_t = (S + BT - 1) / BT;
    attn_bwd_kernel<<<B * nkv * n_t, kThreads, SMEM_BYTES, stream>>>(
        tq, tk, tv, tdo, lse_pad, delta, dq_acc, ld_acc, (__nv_bfloat16*)dk, lddk, (__nv_bfloat16*)dv, lddv, B, S,
        nq, nkv, scale, causal != 0, err, nullptr);
    PB_CUDA_CHECK(cudaGetLastError());
    int sms = 0;
    PB_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int64_t cast_work = T * ld_acc / 4;
    const int cgrid = (int)std::min<int64_t>((cast_work + 255) / 256, (int64_t)sms * 16);
    cast_rows_kernel<<<cgrid, 256, 0, stream>>>(dq_acc, ld_acc, (__nv_bfloat16*)dq, lddq, (int)T, (int)ld_acc);
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
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= pb::kMaxDevices || !pb::g_noalloc_base[dev])
    return -1;
  int v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpy(&v, pb::g_noalloc_base[dev], sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  return v;
}
