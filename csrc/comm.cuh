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
void signal_barrier(const uint64_t* peer_pads_dev, int rank, int world, int slot_base, uint32_t* epoch_ctr,
                    uint64_t limit_ns, cudaStream_t s);
// One short-lived 512-thread block per 64 KB chunk (they interleave with the
// CTAs of concurrent compute kernels).
void multi_copy(const CopySegments& segs, cudaStream_t s);
void reduce_segments(const ReduceSegments& segs, int world, float scale, bool accumulate, cudaStream_t s);
void wait_flag(const uint32_t* flag, uint32_t target, uint64_t limit_ns, int* status, cudaStream_t s);
// NVLS all-reduce over a multicast address (bf16, nelem % 8 == 0): this rank
// reduces and broadcasts vectors [rank, rank + 1) * ceil(vecs / world).  The
// caller brackets it with barriers (inputs staged; broadcasts landed).
// blocks: grid size (0 = default); unroll: requests in flight per thread (4 or 8).
void multimem_all_reduce(void* mc, int64_t nelem, int rank, int world, float scale, cudaStream_t s, int blocks = 0,
                         int unroll = 4);
// CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED of a device (switch multicast and
// in-switch reduction), read through the driver entry point.
bool device_multicast_supported(int device);

// Expert-parallel row exchange over peer memory (one warp per row, 16-byte
// vectors; row_bytes and all strides multiples of 16 bytes).
//   row_scatter:    peer[dst_rank[i]] + dst_row[i]*ld_dst  <-  src + src_row[i]*ld_src   (i < n)
//   row_gather_sum: dst[t] = sum_k peer[rank[t*k_per+k]] + row[t*k_per+k]*ld_src  (bf16 rows,
//                   fp32 sums; rank < 0 skips the route)
struct PeerBases {
  void* p[kMaxPeers];
};
void row_scatter(const void* src, int64_t ld_src_bytes, const int64_t* src_row, const int32_t* dst_rank,
                 const int64_t* dst_row, const PeerBases& peers, int64_t ld_dst_bytes, int64_t row_bytes, int64_t n,
                 cudaStream_t s);
void row_gather_sum(void* dst, int64_t ld_dst, int64_t n_tokens, int k_per, const int32_t* rank, const int64_t* row,
                    const PeerBases& peers, int64_t ld_src, int64_t cols, cudaStream_t s);
//   row_gather:     dst + i*ld_dst  <-  peer[rank[i]] + row[i]*ld_src   (row_bytes; rank < 0 writes zeros)
void row_gather(void* dst, int64_t ld_dst_bytes, const int32_t* rank, const int64_t* row, const PeerBases& peers,
                int64_t ld_src_bytes, int64_t row_bytes, int64_t n, cudaStream_t s);

// Small all-reduce of fp32 data over symmetric buffers (grad-norm partials,
// finite flags, loss statistics, the vocab-parallel log-sum-exp merge).
// Every rank's region (at bases.p[r]) holds two parities of `world` source
// slots of `cap` units, then the block flags: uint32 [kSmallArMaxBlocks][world].
// A unit is one float (SUM / MAX) or one row of three planes (LSE3: max,
// sum-exp, target -> out = [lse | target sum], rows planes each).
constexpr int kSmallArMaxBlocks = 64;
constexpr int kSmallArBlocks = 16;  // the grid of every call (<= kSmallArMaxBlocks)
enum SmallArOp { kArSum = 0, kArMax = 1, kArLse3 = 2 };
int64_t small_ar_region_floats(int world, int64_t cap_units, int op_unit_floats);
void small_all_reduce(const float* in, float* out, int64_t units, int op, const PeerBases& bases, int rank, int world,
                      int64_t cap_units, uint32_t* block_epochs, uint64_t limit_ns, cudaStream_t s);

}  // namespace pb
