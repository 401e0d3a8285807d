// Bindings of the peer-to-peer collective kernels.  Pointers arrive as
// integers (peer addresses of symmetric buffers are not tensors of this
// process); every size and alignment is validated before a launch.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "comm.cuh"
#include "host_util.h"

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void p2p_barrier(int64_t peer_pads_dev, int64_t rank, int64_t world, int64_t slot_base, int64_t epoch,
                 double limit_s) {
  TORCH_CHECK(world >= 1 && world <= pb::kMaxPeers && rank >= 0 && rank < world, "p2p_barrier: bad rank/world");
  pb::signal_barrier(reinterpret_cast<const uint64_t*>(peer_pads_dev), (int)rank, (int)world, (int)slot_base,
                     (uint32_t)epoch, (uint64_t)(limit_s * 1e9), cur_stream());
}

// Copy segments (src_ptr -> dst_ptr, nbytes); all 16-byte aligned multiples.
void p2p_copy(const std::vector<int64_t>& src, const std::vector<int64_t>& dst, const std::vector<int64_t>& nbytes) {
  TORCH_CHECK(src.size() == dst.size() && src.size() == nbytes.size(), "p2p_copy: list sizes");
  size_t i = 0;
  while (i < src.size()) {
    pb::CopySegments segs{};
    int64_t acc = 0;
    int n = 0;
    for (; i < src.size() && n < pb::kMaxCopySegs; ++i) {
      TORCH_CHECK(src[i] % 16 == 0 && dst[i] % 16 == 0 && nbytes[i] % 16 == 0, "p2p_copy: 16-byte alignment");
      if (nbytes[i] == 0) continue;
      segs.src[n] = reinterpret_cast<const uint8_t*>(src[i]);
      segs.dst[n] = reinterpret_cast<uint8_t*>(dst[i]);
      segs.vec_start[n] = acc;
      acc += nbytes[i] / 16;
      ++n;
    }
    segs.vec_start[n] = acc;
    segs.n = n;
    pb::multi_copy(segs, cur_stream());
  }
}

// out_seg[k] = scale * sum_j src[j][k] (+ out_seg[k]); bf16, nelem[k] % 8 == 0.
void p2p_reduce(const std::vector<std::vector<int64_t>>& src, const std::vector<int64_t>& dst,
                const std::vector<int64_t>& nelem, double scale, bool accumulate) {
  const int world = (int)src.size();
  TORCH_CHECK(world >= 1 && world <= pb::kMaxPeers, "p2p_reduce: world");
  for (auto& v : src) TORCH_CHECK(v.size() == dst.size(), "p2p_reduce: segment lists");
  TORCH_CHECK(nelem.size() == dst.size(), "p2p_reduce: nelem");
  size_t i = 0;
  while (i < dst.size()) {
    pb::ReduceSegments segs{};
    int64_t acc = 0;
    int n = 0;
    for (; i < dst.size() && n < pb::kMaxReduceSegs; ++i) {
      TORCH_CHECK(nelem[i] % 8 == 0 && dst[i] % 16 == 0, "p2p_reduce: 16-byte alignment");
      if (nelem[i] == 0) continue;
      for (int j = 0; j < world; ++j) {
        TORCH_CHECK(src[j][i] % 16 == 0, "p2p_reduce: source alignment");
        segs.src[j][n] = reinterpret_cast<const void*>(src[j][i]);
      }
      segs.dst[n] = reinterpret_cast<void*>(dst[i]);
      segs.vec_start[n] = acc;
      acc += nelem[i] / 8;
      ++n;
    }
    segs.vec_start[n] = acc;
    segs.n = n;
    pb::reduce_segments(segs, world, (float)scale, accumulate, cur_stream());
  }
}

void wait_flag(const at::Tensor& flag, int64_t target, double limit_s, at::Tensor& status) {
  TORCH_CHECK(flag.is_cuda() && flag.scalar_type() == at::kInt && status.is_cuda() &&
              status.scalar_type() == at::kInt, "wait_flag: int32 CUDA tensors");
  const c10::cuda::CUDAGuard g(flag.device());
  pb::wait_flag(reinterpret_cast<const uint32_t*>(flag.data_ptr()), (uint32_t)target, (uint64_t)(limit_s * 1e9),
                status.data_ptr<int>(), cur_stream());
}

// Asynchronous copy of this device's error word into a pinned int32 tensor.
void error_word_copy_async(at::Tensor& pinned) {
  TORCH_CHECK(pinned.scalar_type() == at::kInt && pinned.is_pinned() && pinned.numel() >= 1, "pinned int32");
  PB_CUDA_CHECK(cudaMemcpyAsync(pinned.data_ptr(), pb::error_word(), sizeof(int), cudaMemcpyDeviceToHost,
                                cur_stream()));
}

}  // namespace

void register_comm(pybind11::module& m) {
  m.def("p2p_barrier", &p2p_barrier);
  m.def("p2p_copy", &p2p_copy);
  m.def("p2p_reduce", &p2p_reduce);
  m.def("wait_flag", &wait_flag);
  m.def("error_word_copy_async", &error_word_copy_async);
}
