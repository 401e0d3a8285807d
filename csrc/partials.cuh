// Block partials finished by the kernel that produced them.
//
// Weight gradients of the norms are column sums over all rows; each block of
// the producing kernel writes its partial row parts[b][0..len) (no atomics).
// Instead of a separate summing kernel, the blocks finish the sum themselves
// in a fixed order:
//   * blocks come in groups of kFinishGroup; the last block of a group to
//     arrive (per-group arrival counter) adds the group's rows in block order
//     and writes the group sum over the group's first row;
//   * the last group finisher to arrive adds the group sums in group order and
//     writes the result (bf16 or fp32; columns [0, len0) to out0, the rest to
//     out1).
// The order of every addition is fixed by the block and group indices, never
// by arrival order, so the result has the same bits on every run.  The
// finishers return their counters to zero, which keeps the counters valid for
// the next launch and for CUDA-graph replays.  Nobody waits: a block that is
// not last simply leaves.
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

namespace pb {

constexpr int kFinishGroup = 16;

struct PartialsOut {
  void* out0 = nullptr;         // columns [0, len0)
  void* out1 = nullptr;         // columns [len0, len)
  int len0 = 0;
  int out_bf16 = 1;
  unsigned* counters = nullptr;  // >= groups + 1 zeroed words; nullptr: leave the partials alone
};

#if defined(__CUDACC__)
// Call after this block's partial row is fully written (by any of its threads).
__device__ __forceinline__ void finish_partials_in_kernel(float* parts, int64_t stride, int len, int nblocks,
                                                          const PartialsOut& fin) {
  if (fin.counters == nullptr) return;
  __shared__ int s_last;
  const int b = blockIdx.x;
  const int g = b / kFinishGroup, ng = (nblocks + kFinishGroup - 1) / kFinishGroup;
  const int in_group = min(kFinishGroup, nblocks - g * kFinishGroup);
  __threadfence();  // this block's partial row before its arrival
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&fin.counters[g], 1u) == (unsigned)(in_group - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float* grow = parts + (int64_t)g * kFinishGroup * stride;
  for (int c = threadIdx.x; c < len; c += blockDim.x) {
    float t = 0.f;
    for (int i = 0; i < in_group; ++i) t += __ldcg(grow + (int64_t)i * stride + c);
    grow[c] = t;
  }
  if (threadIdx.x == 0) fin.counters[g] = 0u;
  __threadfence();  // the group sum before the group's arrival
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&fin.counters[ng], 1u) == (unsigned)(ng - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int c = threadIdx.x; c < len; c += blockDim.x) {
    float t = 0.f;
    for (int gg = 0; gg < ng; ++gg) t += __ldcg(parts + (int64_t)gg * kFinishGroup * stride + c);
    void* out = c < fin.len0 ? fin.out0 : fin.out1;
    const int oc = c < fin.len0 ? c : c - fin.len0;
    if (out == nullptr) continue;
    if (fin.out_bf16)
      reinterpret_cast<__nv_bfloat16*>(out)[oc] = __float2bfloat16(t);
    else
      reinterpret_cast<float*>(out)[oc] = t;
  }
  if (threadIdx.x == 0) fin.counters[ng] = 0u;
}
#endif  // __CUDACC__

}  // namespace pb
