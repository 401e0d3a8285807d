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

// epochs: int32 CUDA tensor of per-channel counters owned by this buffer; the
// kernel bumps epochs[channel] on the device (CUDA-graph replay safe).
void p2p_barrier(int64_t peer_pads_dev, int64_t rank, int64_t world, int64_t slot_base, at::Tensor& epochs,
                 int64_t channel, double limit_s) {
  TORCH_CHECK(world >= 1 && world <= pb::kMaxPeers && rank >= 0 && rank < world, "p2p_barrier: bad rank/world");
  TORCH_CHECK(epochs.is_cuda() && epochs.scalar_type() == at::kInt && channel >= 0 && channel < epochs.numel(),
              "p2p_barrier: epochs must be an int32 CUDA tensor with one counter per channel");
  pb::signal_barrier(reinterpret_cast<const uint64_t*>(peer_pads_dev), (int)rank, (int)world, (int)slot_base,
                     reinterpret_cast<uint32_t*>(epochs.data_ptr<int>()) + channel, (uint64_t)(limit_s * 1e9),
                     cur_stream());
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

// NVLS all-reduce of nelem bf16 values at the multicast address mc (see
// comm.cuh); the caller stages the inputs and brackets the call with barriers.
void multimem_all_reduce(int64_t mc, int64_t nelem, int64_t rank, int64_t world, double scale, int64_t blocks,
                         int64_t unroll) {
  pb::multimem_all_reduce(reinterpret_cast<void*>(mc), nelem, (int)rank, (int)world, (float)scale, cur_stream(),
                          (int)blocks, (int)unroll);
}

bool device_multicast_supported(int64_t device) { return pb::device_multicast_supported((int)device); }

int64_t small_ar_region_floats(int64_t world, int64_t cap_units) {
  return pb::small_ar_region_floats((int)world, cap_units, 3);
}

// op: 0 sum, 1 max (fp32 [units]); 2 lse3 (in [3, units]: max, sum-exp,
// target; out [2, units]: log-sum-exp, target sum).  bases: every rank's
// region (symmetric, small_ar_region_floats(world, cap) floats); epochs: int32
// [kSmallArMaxBlocks] device counters of this region.
void small_all_reduce(const at::Tensor& in, at::Tensor& out, int64_t units, int64_t op,
                      const std::vector<int64_t>& bases, int64_t rank, int64_t cap_units, at::Tensor& epochs,
                      double limit_s) {
  TORCH_CHECK(in.is_cuda() && in.scalar_type() == at::kFloat && in.is_contiguous() && out.is_cuda() &&
              out.scalar_type() == at::kFloat && out.is_contiguous(), "small_all_reduce: contiguous fp32 CUDA");
  const int64_t uf = op == pb::kArLse3 ? 3 : 1, of = op == pb::kArLse3 ? 2 : 1;
  TORCH_CHECK(in.numel() >= units * uf && out.numel() >= units * of, "small_all_reduce: tensor sizes");
  TORCH_CHECK(epochs.is_cuda() && epochs.scalar_type() == at::kInt && epochs.numel() >= pb::kSmallArMaxBlocks,
              "small_all_reduce: int32 epoch counters");
  TORCH_CHECK(bases.size() >= 1 && bases.size() <= (size_t)pb::kMaxPeers, "small_all_reduce: world");
  pb::PeerBases pb_{};
  for (size_t i = 0; i < bases.size(); ++i) pb_.p[i] = reinterpret_cast<void*>(bases[i]);
  const c10::cuda::CUDAGuard g(in.device());
  // slot capacity in units of this op: the region was sized for cap_units rows of 3 floats
  pb::small_all_reduce(in.data_ptr<float>(), out.data_ptr<float>(), units, (int)op, pb_, (int)rank,
                       (int)bases.size(), op == pb::kArLse3 ? cap_units : 3 * cap_units,
                       reinterpret_cast<uint32_t*>(epochs.data_ptr<int>()), (uint64_t)(limit_s * 1e9), cur_stream());
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

pb::PeerBases peer_bases(const std::vector<int64_t>& ptrs) {
  TORCH_CHECK(ptrs.size() >= 1 && ptrs.size() <= (size_t)pb::kMaxPeers, "1..8 peer pointers");
  pb::PeerBases b{};
  for (size_t i = 0; i < ptrs.size(); ++i) b.p[i] = reinterpret_cast<void*>(ptrs[i]);
  return b;
}

// row_scatter(src [rows, cols] any dtype, src_row int64 [n], dst_rank int32 [n], dst_row int64 [n],
//             peer_ptrs, ld_dst_bytes): src rows -> rows of the peers' buffers.
void row_scatter(const at::Tensor& src, const at::Tensor& src_row, const at::Tensor& dst_rank,
                 const at::Tensor& dst_row, const std::vector<int64_t>& peer_ptrs, int64_t ld_dst_bytes) {
  TORCH_CHECK(src.is_cuda() && src.dim() == 2 && src.stride(1) == 1, "row_scatter: src 2-D CUDA, unit inner stride");
  TORCH_CHECK(src_row.scalar_type() == at::kLong && dst_row.scalar_type() == at::kLong &&
                  dst_rank.scalar_type() == at::kInt && src_row.is_contiguous() && dst_row.is_contiguous() &&
                  dst_rank.is_contiguous(),
              "row_scatter: index dtypes");
  const int64_t n = src_row.numel();
  TORCH_CHECK(dst_rank.numel() == n && dst_row.numel() == n, "row_scatter: index lengths");
  const c10::cuda::CUDAGuard g(src.device());
  pb::row_scatter(src.data_ptr(), src.stride(0) * src.element_size(), src_row.data_ptr<int64_t>(),
                  dst_rank.data_ptr<int32_t>(), dst_row.data_ptr<int64_t>(), peer_bases(peer_ptrs), ld_dst_bytes,
                  src.size(1) * src.element_size(), n, at::cuda::getCurrentCUDAStream().stream());
}

// row_gather_sum(dst bf16 [tokens, cols], rank int32 [tokens*k], row int64 [tokens*k], peer_ptrs, ld_src):
// dst[t] = sum_k peer[rank][row] (rank < 0 skips).
void row_gather_sum(at::Tensor& dst, const at::Tensor& rank, const at::Tensor& row,
                    const std::vector<int64_t>& peer_ptrs, int64_t ld_src) {
  TORCH_CHECK(dst.is_cuda() && dst.scalar_type() == at::kBFloat16 && dst.dim() == 2 && dst.stride(1) == 1,
              "row_gather_sum: dst 2-D bf16");
  TORCH_CHECK(rank.scalar_type() == at::kInt && row.scalar_type() == at::kLong && rank.is_contiguous() &&
                  row.is_contiguous() && rank.numel() == row.numel(),
              "row_gather_sum: index tensors");
  const int64_t n_tokens = dst.size(0);
  TORCH_CHECK(n_tokens == 0 || rank.numel() % n_tokens == 0, "row_gather_sum: routes per token");
  const int k_per = n_tokens ? (int)(rank.numel() / n_tokens) : 0;
  const c10::cuda::CUDAGuard g(dst.device());
  pb::row_gather_sum(dst.data_ptr(), dst.stride(0), n_tokens, k_per, rank.data_ptr<int32_t>(), row.data_ptr<int64_t>(),
                     peer_bases(peer_ptrs), ld_src, dst.size(1), at::cuda::getCurrentCUDAStream().stream());
}

// row_gather(dst [n, cols] (16-byte rows), rank int32 [n], row int64 [n], peer_ptrs, ld_src_bytes)
void row_gather(at::Tensor& dst, const at::Tensor& rank, const at::Tensor& row, const std::vector<int64_t>& peer_ptrs,
                int64_t ld_src_bytes) {
  TORCH_CHECK(dst.is_cuda() && dst.dim() == 2 && dst.stride(1) == 1, "row_gather: dst 2-D CUDA");
  TORCH_CHECK(rank.scalar_type() == at::kInt && row.scalar_type() == at::kLong && rank.is_contiguous() &&
                  row.is_contiguous() && rank.numel() == dst.size(0) && row.numel() == dst.size(0),
              "row_gather: index tensors");
  const c10::cuda::CUDAGuard g(dst.device());
  pb::row_gather(dst.data_ptr(), dst.stride(0) * dst.element_size(), rank.data_ptr<int32_t>(), row.data_ptr<int64_t>(),
                 peer_bases(peer_ptrs), ld_src_bytes, dst.size(1) * dst.element_size(), dst.size(0),
                 at::cuda::getCurrentCUDAStream().stream());
}

void register_comm(pybind11::module& m) {
  m.def("p2p_barrier", &p2p_barrier);
  m.def("p2p_copy", &p2p_copy);
  m.def("p2p_reduce", &p2p_reduce);
  m.def("wait_flag", &wait_flag);
  m.def("multimem_all_reduce", &multimem_all_reduce, pybind11::arg("mc"), pybind11::arg("nelem"), pybind11::arg("rank"),
        pybind11::arg("world"), pybind11::arg("scale"), pybind11::arg("blocks") = 0, pybind11::arg("unroll") = 4);
  m.def("device_multicast_supported", &device_multicast_supported);
  m.def("small_ar_region_floats", &small_ar_region_floats);
  m.def("small_all_reduce", &small_all_reduce);
  m.def("row_scatter", &row_scatter);
  m.def("row_gather_sum", &row_gather_sum);
  m.def("row_gather", &row_gather);
  m.def("error_word_copy_async", &error_word_copy_async);
}
