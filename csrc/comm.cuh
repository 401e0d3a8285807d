// Peer-to-peer collective launchers (comm.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace pb {

constexpr int kMaxPeers = 8;
constexpr int kMaxCopySegs = 96;
constexpr int kMaxReduceSegs = 16;

struct CopySegments {
  const uint8_t* src[kMaxCopySegs];
  uint8_t* dst[kMaxCopySegs];
  int64_t vec_start[kMaxCopySegs + 1];  // prefix sums of 16-byte vectors
  int n;
};

struct ReduceSegments {
  const void* src[kMaxPeers][kMaxReduceSegs];
  void* dst[kMaxReduceSegs];
  int64_t vec_start[kMaxReduceSegs + 1];  // prefix sums of 8-element (bf16) vectors
  int n;
};

// peer_pads_dev: device array of `world` signal-pad pointers (uint32 words).
// Slot words used: [slot_base + r] for r in [0, world).
void signal_barrier(const uint64_t* peer_pads_dev, int rank, int world, int slot_base, uint32_t epoch,
                    uint64_t limit_ns, cudaStream_t s);
void multi_copy(const CopySegments& segs, cudaStream_t s);
void reduce_segments(const ReduceSegments& segs, int world, float scale, bool accumulate, cudaStream_t s);
void wait_flag(const uint32_t* flag, uint32_t target, uint64_t limit_ns, int* status, cudaStream_t s);

}  // namespace pb
