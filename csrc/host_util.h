// Host-side helpers shared by every launcher: TMA descriptor encoding through
// the driver entry point, the per-device error word, SM counts and launch
// checks.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>
#include <utility>

namespace pb {

// Throws std::runtime_error with file/line context on a CUDA runtime error.
#define PB_CUDA_CHECK(expr)                                                               \
  do {                                                                                    \
    cudaError_t _e = (expr);                                                              \
    if (_e != cudaSuccess)                                                                \
      throw std::runtime_error(std::string("CUDA error ") + cudaGetErrorString(_e) +      \
                               " at " + __FILE__ + ":" + std::to_string(__LINE__));       \
  } while (0)

#define PB_CHECK(cond, msg)                                                        \
  do {                                                                             \
    if (!(cond)) throw std::runtime_error(std::string("parallel_b200: ") + (msg)); \
  } while (0)

// Device pointer to this device's 4-byte error word (allocated on first use,
// zero-initialised).  Kernels record timeouts there; the host reads it with
// read_error() and clears it with clear_error().
int* error_word(int device = -1);
// Counter slot (kSplitSlotInts zeroed ints) for one ordered split-K GEMM launch:
// the slots rotate, so launches that may run concurrently on different streams
// use different counters; each launch leaves its counters at zero.
constexpr int kSplitSlots = 16;
constexpr int kSplitSlotInts = 8192;
int* split_counters(int device = -1);
int read_error(int device = -1);
void clear_error(int device = -1);

int num_sms(int device = -1);

// Programmatic dependent launch (PB_PDL=1, read once; default off).  Every
// kernel of this library starts with pdl_prologue() (ptx.cuh), which waits
// for the previous kernel of the stream to complete and flush before anything
// else runs; with PB_PDL=1 launch_k also sets programmatic stream
// serialization, so the next kernel's launch and block set-up overlap this
// kernel's tail instead of following its completion.  The data order is the
// same either way (each kernel starts its work after its predecessor
// finished); without the attribute the prologue is a no-op.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  PB_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

// Encode a 2-D bf16 tiled tensor map with 128-byte swizzle.
//   inner/outer: extents in elements; row_stride_elems: stride of the outer
//   dimension in elements; box_inner/box_outer: tile extents in elements.
CUtensorMap make_tmap_2d_bf16(const void* base, uint64_t inner, uint64_t outer,
                              uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer,
                              bool swizzle128 = true);

// 2-D bf16 tensor map with a chosen swizzle span (0 = none, 32, 64 or 128 bytes);
// used for epilogue tile stores.
CUtensorMap make_tmap_2d_bf16_swz(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                                  uint32_t box_inner, uint32_t box_outer, int swizzle_bytes);

// Encode a 3-D bf16 tiled tensor map with 128-byte swizzle.
CUtensorMap make_tmap_3d_bf16(const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                              uint64_t stride1_elems, uint64_t stride2_elems, uint32_t b0,
                              uint32_t b1, uint32_t b2);

// Encode a 3-D fp32 tiled tensor map (used as the destination of bulk
// reduce-adds); swizzle128 needs b0 * 4 <= 128.
CUtensorMap make_tmap_3d_f32(void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1_elems,
                             uint64_t stride2_elems, uint32_t b0, uint32_t b1, uint32_t b2, bool swizzle128);

}  // namespace pb
