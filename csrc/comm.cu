// In-kernel NVLink peer-to-peer collectives over symmetric memory.
//
// Buffers are allocated symmetrically (every rank maps every peer's buffer
// into its address space); these kernels read / write peers' memory with
// ordinary loads and stores over NVLink 5 / NVSwitch.  No TMA multicast and
// no library kernel ever touches a peer pointer.
//
//   signal_barrier   one warp: bump this buffer's device epoch counter, publish
//                    the new epoch into every peer's signal pad
//                    (release, system scope) and wait - bounded by limit_ns -
//                    until every peer has published it into ours.  A timeout
//                    records kErrPeerTimeout and returns (the host raises).
//   multi_copy       gather of up to kMaxSegs (src, dst, bytes) segments with
//                    16-byte vector loads; used for the FSDP all-gather, which
//                    writes each peer's shard straight into the parameter-major
//                    full buffer (no unpack pass).
//   reduce_segments  reduce-scatter / all-reduce: out[i] = scale * sum over
//                    peers of src_peer[i] (+ out[i] when accumulating), bf16 in
//                    and out, fp32 sums.
//   wait_flag        test hook: bounded wait on a flag that nobody sets.
//   multimem_all_reduce  NVLS all-reduce of a bf16 buffer bound to an NVLink
//                    multicast object: each rank reads its 1/world slice
//                    through the switch with multimem.ld_reduce (the switch
//                    sums every GPU's copy, fp32 accumulation) and stores the
//                    result back with multimem.st (the switch writes it to
//                    every GPU).  Each GPU receives the slice sums once and
//                    the broadcast once: half the NVLink traffic of a
//                    reduce-scatter followed by an all-gather over peer loads.
//
// Reference counterpart: the NCCL all_gather_into_tensor / reduce_scatter_
// tensor / all_reduce calls of parallel/parallel/engine/_dp_param_unit.py:
// 18-37,350,477 and engine.py:239.
#include <cuda_bf16.h>
#include <stdint.h>

#include <algorithm>

#include "comm.cuh"
#include "host_util.h"
#include "ptx.cuh"

namespace pb {
namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void signal_barrier_kernel(const uint64_t* __restrict__ peer_pads, int rank, int world, int slot_base,
                                      uint32_t* __restrict__ epoch_ctr, uint64_t limit_ns, int* err) {
  pdl_prologue();
  const int i = threadIdx.x;
  // the epoch lives on the device (one counter per buffer and channel, bumped
  // here), so a captured CUDA graph replays a fresh epoch every time
  const uint32_t epoch = *((volatile uint32_t*)epoch_ctr) + 1u;
  __syncwarp();
  if (i == 0) *epoch_ctr = epoch;
  if (i >= world) return;
  // make this rank's prior writes (earlier kernels on this stream) visible first
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  uint32_t* peer = reinterpret_cast<uint32_t*>(peer_pads[i]);
  st_release_sys(peer + slot_base + rank, epoch);
  const uint32_t* mine = reinterpret_cast<const uint32_t*>(peer_pads[rank]) + slot_base + i;
  const uint64_t t0 = globaltimer();
  uint32_t n = 0;
  while ((int32_t)(ld_acquire_sys(mine) - epoch) < 0) {
    if ((++n & 255u) == 0) {
      if (*((volatile int*)err) != 0) return;
      if (globaltimer() - t0 > limit_ns) {
        record_error(err, kErrPeerTimeout);
        return;
      }
    }
  }
}

// Segment of vector v: the last s with vec_start[s] <= v (binary search over
// the kernel-parameter table).
template <typename Segs>
__device__ __forceinline__ int find_seg(const Segs& segs, int64_t v) {
  int lo = 0, hi = segs.n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (segs.vec_start[mid] <= v) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

constexpr int kCopyChunkVecs = 4096;  // 64 KB of 16-byte vectors per chunk
constexpr int kCopyUnroll = 4;

// Chunked gather: one block per 64 KB chunk (short-lived blocks: a copy that
// overlaps compute never holds an SM for long, so the compute kernels' CTAs
// find room as soon as they need it), the chunk's first segment found once,
// and kCopyUnroll independent 16-byte loads in flight per thread (remote
// NVLink loads need many outstanding requests).
__global__ void __launch_bounds__(512) multi_copy_kernel(CopySegments segs) {
  pdl_prologue();
  const int64_t total = segs.vec_start[segs.n];
  {
    const int64_t c = blockIdx.x;
    const int64_t v0 = c * kCopyChunkVecs, v1 = min(total, v0 + kCopyChunkVecs);
    int seg = find_seg(segs, v0 + threadIdx.x < v1 ? v0 + threadIdx.x : v0);
    for (int64_t base = v0 + threadIdx.x; base < v1; base += kCopyUnroll * blockDim.x) {
      uint4 val[kCopyUnroll];
      uint8_t* dst[kCopyUnroll];
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t v = base + (int64_t)u * blockDim.x;
        dst[u] = nullptr;
        if (v < v1) {
          while (seg + 1 < segs.n && segs.vec_start[seg + 1] <= v) ++seg;
          const int64_t off = (v - segs.vec_start[seg]) * 16;
          val[u] = *reinterpret_cast<const uint4*>(segs.src[seg] + off);
          dst[u] = segs.dst[seg] + off;
        }
      }
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u)
        if (dst[u]) *reinterpret_cast<uint4*>(dst[u]) = val[u];
    }
  }
}

// out[i] = scale * sum_j src_j[i] (+ out[i]);  8 bf16 per vector, one block
// per chunk as multi_copy (one segment search per chunk, monotone advance).
__global__ void __launch_bounds__(512) reduce_segments_kernel(ReduceSegments segs, int world, float scale,
                                                              bool accumulate) {
  pdl_prologue();
  const int64_t total = segs.vec_start[segs.n];
  {
    const int64_t c = blockIdx.x;
    const int64_t v0 = c * kCopyChunkVecs, v1 = min(total, v0 + kCopyChunkVecs);
    int seg = find_seg(segs, v0 + threadIdx.x < v1 ? v0 + threadIdx.x : v0);
    for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
      while (seg + 1 < segs.n && segs.vec_start[seg + 1] <= v) ++seg;
      const int64_t off = (v - segs.vec_start[seg]) * 8;  // elements
      uint4 in[kMaxPeers];
#pragma unroll
      for (int j = 0; j < kMaxPeers; ++j)
        if (j < world) in[j] = *reinterpret_cast<const uint4*>(
                           reinterpret_cast<const __nv_bfloat16*>(segs.src[j][seg]) + off);
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
      for (int j = 0; j < kMaxPeers; ++j) {
        if (j >= world) break;
        const uint32_t* p = &in[j].x;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack_bf16x2(p[q]);
          acc[2 * q] += f.x;
          acc[2 * q + 1] += f.y;
        }
      }
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(segs.dst[seg]) + off;
      if (accumulate) {
        const uint4 u = *reinterpret_cast<const uint4*>(dst);
        const uint32_t* p = &u.x;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack_bf16x2(p[q]);
          acc[2 * q] = acc[2 * q] * scale + f.x;
          acc[2 * q + 1] = acc[2 * q + 1] * scale + f.y;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] *= scale;
      }
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      *reinterpret_cast<uint4*>(dst) = o;
    }
  }
}

// Vectors [lo, hi) of the multicast range: out = scale * sum over ranks;
// U independent 16-byte requests in flight per thread.
template <int U>
__global__ void __launch_bounds__(512) multimem_all_reduce_kernel(uint4* __restrict__ mc, int64_t lo, int64_t hi,
                                                                  float scale) {
  pdl_prologue();
  constexpr int kMmUnroll = U;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t base = lo + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < hi; base += kMmUnroll * stride) {
    uint4 v[kMmUnroll];
#pragma unroll
    for (int u = 0; u < kMmUnroll; ++u) {
      const int64_t i = base + u * stride;
      if (i < hi)
        asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v[u].x), "=r"(v[u].y), "=r"(v[u].z), "=r"(v[u].w)
                     : "l"(mc + i)
                     : "memory");
    }
#pragma unroll
    for (int u = 0; u < kMmUnroll; ++u) {
      const int64_t i = base + u * stride;
      if (i >= hi) continue;
      if (scale != 1.f) {
        uint32_t* w = &v[u].x;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack_bf16x2(w[q]);
          w[q] = pack_bf16x2(f.x * scale, f.y * scale);
        }
      }
      asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc + i), "r"(v[u].x),
                   "r"(v[u].y), "r"(v[u].z), "r"(v[u].w)
                   : "memory");
    }
  }
  // the closing barrier publishes these stores to the other ranks
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

__global__ void wait_flag_kernel(const uint32_t* flag, uint32_t target, uint64_t limit_ns, int* status) {
  pdl_prologue();
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const uint64_t t0 = globaltimer();
  uint32_t n = 0;
  while ((int32_t)(ld_acquire_sys(flag) - target) < 0) {
    if ((++n & 255u) == 0 && globaltimer() - t0 > limit_ns) {
      record_error(status, kErrPeerTimeout);
      return;
    }
  }
}


// One warp per row: copy row_bytes from the local source row to the peer row.
__global__ void row_scatter_kernel(const uint8_t* __restrict__ src, int64_t ld_src, const int64_t* __restrict__ src_row,
                                   const int32_t* __restrict__ dst_rank, const int64_t* __restrict__ dst_row,
                                   PeerBases peers, int64_t ld_dst, int64_t vecs, int64_t n) {
  pdl_prologue();
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  const int r = dst_rank[i];
  if (r < 0 || r >= kMaxPeers) return;
  const uint4* s4 = reinterpret_cast<const uint4*>(src + src_row[i] * ld_src);
  uint4* d4 = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(peers.p[r]) + dst_row[i] * ld_dst);
  for (int64_t v = lane; v < vecs; v += 32) d4[v] = s4[v];
}

// One warp per token: fp32 sum of its k_per routes' bf16 rows read from the owners.
__global__ void row_gather_sum_kernel(__nv_bfloat16* __restrict__ dst, int64_t ld_dst, int64_t n_tokens, int k_per,
                                      const int32_t* __restrict__ rank, const int64_t* __restrict__ row,
                                      PeerBases peers, int64_t ld_src, int64_t vecs) {
  pdl_prologue();
  const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= n_tokens) return;
  for (int64_t v = lane; v < vecs; v += 32) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < k_per; ++k) {
      const int r = rank[t * k_per + k];
      if (r < 0 || r >= kMaxPeers) continue;
      const uint4 u = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(peers.p[r]) +
                                                     row[t * k_per + k] * ld_src)[v];
      const uint32_t* w = &u.x;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(w[q]);
        acc[2 * q] += f.x;
        acc[2 * q + 1] += f.y;
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    reinterpret_cast<uint4*>(dst + t * ld_dst)[v] = o;
  }
}

// One warp per row: pull row_bytes from a peer row (zeros for rank < 0).
__global__ void row_gather_kernel(uint8_t* __restrict__ dst, int64_t ld_dst, const int32_t* __restrict__ rank,
                                  const int64_t* __restrict__ row, PeerBases peers, int64_t ld_src, int64_t vecs,
                                  int64_t n) {
  pdl_prologue();
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  const int r = rank[i];
  uint4* d4 = reinterpret_cast<uint4*>(dst + i * ld_dst);
  if (r < 0 || r >= kMaxPeers) {
    for (int64_t v = lane; v < vecs; v += 32) d4[v] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* s4 = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(peers.p[r]) + row[i] * ld_src);
  for (int64_t v = lane; v < vecs; v += 32) d4[v] = s4[v];
}

// Sliced small all-reduce: block b owns units [lo, hi).  It bumps its own
// epoch counter, stores its slice of `in` into slot `rank` of parity
// (epoch & 1) in every peer's region, publishes the epoch in each peer's flag
// [b][rank] (release, system scope), waits - bounded - for every peer's flag
// [b][j], then combines the `world` slots of its slice from its own region.
// The grid is the same for every call, so all blocks share the call's epoch.
// A peer raises its call-k flag only from its kernel k, which starts after its
// kernel k-1 - every read of the parity that call k+1 overwrites - has
// finished: two parities make the exchange safe without a closing barrier.
__global__ void small_ar_kernel(const float* __restrict__ in, float* __restrict__ out, int64_t units, int op,
                                PeerBases bases, int rank, int world, int64_t cap, uint32_t* __restrict__ epochs,
                                uint64_t limit_ns, int* err) {
  pdl_prologue();
  const int b = blockIdx.x;
  const int uf = op == kArLse3 ? 3 : 1;  // floats per unit
  const int64_t per = (units + gridDim.x - 1) / gridDim.x;
  const int64_t lo = (int64_t)b * per, hi = min(units, lo + per);
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) {
    s_epoch = epochs[b] + 1u;
    epochs[b] = s_epoch;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int par = epoch & 1;
  const int64_t slot_floats = cap * uf;
  const int64_t flags_off = 2 * (int64_t)world * slot_floats;  // in floats (uint32 flags follow the data)
  // push this rank's slice into every peer (planar layout: plane q of unit u at q * cap + u)
  for (int j = 0; j < world; ++j) {
    float* dst = reinterpret_cast<float*>(bases.p[j]) + ((int64_t)par * world + rank) * slot_floats;
    for (int q = 0; q < uf; ++q)
      for (int64_t u = lo + threadIdx.x; u < hi; u += blockDim.x) dst[q * cap + u] = in[q * units + u];
  }
  __syncthreads();
  if (threadIdx.x < world) {
    const int j = threadIdx.x;
    __threadfence_system();
    uint32_t* flag = reinterpret_cast<uint32_t*>(reinterpret_cast<float*>(bases.p[j]) + flags_off) +
                     b * world + rank;
    st_release_sys(flag, epoch);
    const uint32_t* mine =
        reinterpret_cast<const uint32_t*>(reinterpret_cast<const float*>(bases.p[rank]) + flags_off) + b * world + j;
    const uint64_t t0 = globaltimer();
    uint32_t n = 0;
    while ((int32_t)(ld_acquire_sys(mine) - epoch) < 0) {
      if ((++n & 255u) == 0) {
        if (*((volatile int*)err) != 0) break;
        if (globaltimer() - t0 > limit_ns) {
          record_error(err, kErrPeerTimeout);
          break;
        }
      }
    }
  }
  __syncthreads();
  const float* base = reinterpret_cast<const float*>(bases.p[rank]) + (int64_t)par * world * slot_floats;
  for (int64_t u = lo + threadIdx.x; u < hi; u += blockDim.x) {
    if (op == kArLse3) {
      float m = -INFINITY;
      for (int j = 0; j < world; ++j) m = fmaxf(m, base[j * slot_floats + u]);
      float se = 0.f, t = 0.f;
      for (int j = 0; j < world; ++j) {
        const float* sl = base + j * slot_floats;
        se += sl[cap + u] * __expf(sl[u] - m);
        t += sl[2 * cap + u];
      }
      out[u] = m + __logf(se);
      out[units + u] = t;
    } else {
      float acc = op == kArMax ? -INFINITY : 0.f;
      for (int j = 0; j < world; ++j) {
        const float v = base[j * slot_floats + u];
        acc = op == kArMax ? fmaxf(acc, v) : acc + v;
      }
      out[u] = acc;
    }
  }
}

}  // namespace

void signal_barrier(const uint64_t* peer_pads_dev, int rank, int world, int slot_base, uint32_t* epoch_ctr,
                    uint64_t limit_ns, cudaStream_t s) {
  PB_CHECK(world >= 1 && world <= kMaxPeers, "signal_barrier: world size");
  launch_k(signal_barrier_kernel, 1, 32, 0, s, peer_pads_dev, rank, world, slot_base, epoch_ctr, limit_ns, error_word());
  PB_CUDA_CHECK(cudaGetLastError());
}

unsigned chunk_grid(int64_t vecs) {
  const int64_t g = (vecs + kCopyChunkVecs - 1) / kCopyChunkVecs;
  PB_CHECK(g < (int64_t)1 << 31, "p2p copy: too many chunks");
  return (unsigned)std::max<int64_t>(1, g);
}

void multi_copy(const CopySegments& segs, cudaStream_t s) {
  if (segs.n == 0) return;
  launch_k(multi_copy_kernel, chunk_grid(segs.vec_start[segs.n]), 512, 0, s, segs);
  PB_CUDA_CHECK(cudaGetLastError());
}

void reduce_segments(const ReduceSegments& segs, int world, float scale, bool accumulate, cudaStream_t s) {
  if (segs.n == 0) return;
  launch_k(reduce_segments_kernel, chunk_grid(segs.vec_start[segs.n]), 512, 0, s, segs, world, scale, accumulate);
  PB_CUDA_CHECK(cudaGetLastError());
}

bool device_multicast_supported(int device) {
  using GetAttrFn = CUresult (*)(int*, CUdevice_attribute, CUdevice);
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuDeviceGetAttribute", &p, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || p == nullptr)
    return false;
  int v = 0;
  if (reinterpret_cast<GetAttrFn>(p)(&v, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, (CUdevice)device) != CUDA_SUCCESS)
    return false;
  return v != 0;
}

void multimem_all_reduce(void* mc, int64_t nelem, int rank, int world, float scale, cudaStream_t s, int blocks,
                         int unroll) {
  PB_CHECK(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world, "multimem_all_reduce: rank / world");
  PB_CHECK(nelem % 8 == 0 && reinterpret_cast<uintptr_t>(mc) % 16 == 0, "multimem_all_reduce: 16-byte vectors");
  PB_CHECK(unroll == 4 || unroll == 8, "multimem_all_reduce: unroll 4 or 8");
  const int64_t vecs = nelem / 8;
  const int64_t per = (vecs + world - 1) / world;
  const int64_t lo = std::min<int64_t>(vecs, per * rank), hi = std::min<int64_t>(vecs, lo + per);
  if (hi <= lo) return;
  // default 32 blocks: on 2 B200s the kernel alone took 28 / 174 / 662 us for
  // 8 / 64 / 256 MB with 32 blocks x 4 requests per thread, and 35 / 199 / 700
  // us with 592 blocks (more requests than the switch overlaps only queue)
  const int64_t need = (hi - lo + 512 * unroll - 1) / (512 * unroll);
  const int64_t g = std::max<int64_t>(1, std::min<int64_t>(need, blocks > 0 ? blocks : 32));
  if (unroll == 8)
    launch_k(multimem_all_reduce_kernel<8>, (unsigned)g, 512, 0, s, reinterpret_cast<uint4*>(mc), lo, hi, scale);
  else
    launch_k(multimem_all_reduce_kernel<4>, (unsigned)g, 512, 0, s, reinterpret_cast<uint4*>(mc), lo, hi, scale);
  PB_CUDA_CHECK(cudaGetLastError());
}

void wait_flag(const uint32_t* flag, uint32_t target, uint64_t limit_ns, int* status, cudaStream_t s) {
  launch_k(wait_flag_kernel, 1, 32, 0, s, flag, target, limit_ns, status);
  PB_CUDA_CHECK(cudaGetLastError());
}

void row_scatter(const void* src, int64_t ld_src_bytes, const int64_t* src_row, const int32_t* dst_rank,
                 const int64_t* dst_row, const PeerBases& peers, int64_t ld_dst_bytes, int64_t row_bytes, int64_t n,
                 cudaStream_t s) {
  PB_CHECK(row_bytes % 16 == 0 && ld_src_bytes % 16 == 0 && ld_dst_bytes % 16 == 0, "row_scatter: 16-byte rows");
  if (n == 0) return;
  const int64_t threads = n * 32;
  launch_k(row_scatter_kernel, (unsigned)((threads + 255) / 256), 256, 0, s,
      reinterpret_cast<const uint8_t*>(src), ld_src_bytes, src_row, dst_rank, dst_row, peers, ld_dst_bytes,
      row_bytes / 16, n);
  PB_CUDA_CHECK(cudaGetLastError());
}

void row_gather_sum(void* dst, int64_t ld_dst, int64_t n_tokens, int k_per, const int32_t* rank, const int64_t* row,
                    const PeerBases& peers, int64_t ld_src, int64_t cols, cudaStream_t s) {
  PB_CHECK(cols % 8 == 0 && ld_dst % 8 == 0 && ld_src % 8 == 0, "row_gather_sum: 16-byte rows");
  if (n_tokens == 0) return;
  const int64_t threads = n_tokens * 32;
  launch_k(row_gather_sum_kernel, (unsigned)((threads + 255) / 256), 256, 0, s,
      reinterpret_cast<__nv_bfloat16*>(dst), ld_dst, n_tokens, k_per, rank, row, peers, ld_src, cols / 8);
  PB_CUDA_CHECK(cudaGetLastError());
}

void row_gather(void* dst, int64_t ld_dst_bytes, const int32_t* rank, const int64_t* row, const PeerBases& peers,
                int64_t ld_src_bytes, int64_t row_bytes, int64_t n, cudaStream_t s) {
  PB_CHECK(row_bytes % 16 == 0 && ld_src_bytes % 16 == 0 && ld_dst_bytes % 16 == 0, "row_gather: 16-byte rows");
  if (n == 0) return;
  const int64_t threads = n * 32;
  launch_k(row_gather_kernel, (unsigned)((threads + 255) / 256), 256, 0, s, reinterpret_cast<uint8_t*>(dst), ld_dst_bytes, rank,
                                                                      row, peers, ld_src_bytes, row_bytes / 16, n);
  PB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace pb

namespace pb {

int64_t small_ar_region_floats(int world, int64_t cap_units, int op_unit_floats) {
  return 2 * (int64_t)world * cap_units * op_unit_floats + (int64_t)kSmallArMaxBlocks * world;
}

void small_all_reduce(const float* in, float* out, int64_t units, int op, const PeerBases& bases, int rank, int world,
                      int64_t cap_units, uint32_t* block_epochs, uint64_t limit_ns, cudaStream_t s) {
  PB_CHECK(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world, "small_all_reduce: rank / world");
  PB_CHECK(units <= cap_units, "small_all_reduce: more units than the buffer holds");
  PB_CHECK(op == kArSum || op == kArMax || op == kArLse3, "small_all_reduce: op");
  if (units == 0) return;
  // a fixed grid: every block takes part in every call, so all block epochs
  // (and the parity of the data slots) stay equal from call to call
  launch_k(small_ar_kernel, kSmallArBlocks, 256, 0, s, in, out, units, op, bases, rank, world, cap_units, block_epochs, limit_ns,
                                         error_word());
  PB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace pb
