// Bindings of the device-resident MoE routing kernels (moe.cu).  Peer
// addresses of symmetric buffers arrive as integers; shapes, dtypes and
// alignment are validated before every launch.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "comm.cuh"
#include "host_util.h"
#include "moe.cuh"

pb::PeerBases peer_bases(const std::vector<int64_t>& ptrs);

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_i32(const at::Tensor& t, int64_t n, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kInt && t.is_contiguous() && t.numel() >= n, what,
              ": int32 contiguous CUDA tensor of at least ", n, " elements");
}

void check_rows(const at::Tensor& t, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.stride(1) == 1 &&
                  t.stride(0) % 8 == 0 && t.size(1) % 8 == 0,
              what, ": 2-D bf16 CUDA rows, unit inner stride, 16-byte rows");
}

// moe_hist(topi int64 [T, K], mat fp32 [rows, E], row)
void moe_hist(const at::Tensor& topi, at::Tensor& mat, int64_t row) {
  TORCH_CHECK(topi.is_cuda() && topi.scalar_type() == at::kLong && topi.is_contiguous(), "moe_hist: topi int64");
  TORCH_CHECK(mat.is_cuda() && mat.scalar_type() == at::kFloat && mat.dim() == 2 && mat.is_contiguous(),
              "moe_hist: mat fp32 [rows, E]");
  const c10::cuda::CUDAGuard g(topi.device());
  pb::moe_hist(topi.data_ptr<int64_t>(), topi.numel(), (int)mat.size(1), mat.data_ptr<float>(), (int)mat.size(0),
               (int)row, cur_stream());
}

// moe_plan(topi, mat, my_row, E_loc, ep_rank, local_only, route_owner, route_row, own_cnt, own_off, krange,
//          tile_expert, n_tiles)
void moe_plan(const at::Tensor& topi, const at::Tensor& mat, int64_t my_row, int64_t E_loc, int64_t ep_rank,
              bool local_only, at::Tensor& route_owner, at::Tensor& route_row, at::Tensor& own_cnt,
              at::Tensor& own_off, at::Tensor& krange, at::Tensor& tile_expert, at::Tensor& n_tiles) {
  TORCH_CHECK(topi.is_cuda() && topi.scalar_type() == at::kLong && topi.is_contiguous(), "moe_plan: topi int64");
  TORCH_CHECK(mat.is_cuda() && mat.scalar_type() == at::kFloat && mat.dim() == 2 && mat.is_contiguous(),
              "moe_plan: mat fp32 [rows, E]");
  const int64_t n = topi.numel();
  check_i32(route_owner, n, "moe_plan: route_owner");
  check_i32(route_row, n, "moe_plan: route_row");
  check_i32(own_cnt, E_loc, "moe_plan: own_cnt");
  check_i32(own_off, E_loc, "moe_plan: own_off");
  check_i32(krange, 2 * E_loc, "moe_plan: krange");
  check_i32(tile_expert, 1, "moe_plan: tile_expert");
  check_i32(n_tiles, 1, "moe_plan: n_tiles");
  const c10::cuda::CUDAGuard g(topi.device());
  pb::MoePlanArgs a;
  a.topi = topi.data_ptr<int64_t>();
  a.n_routes = n;
  a.mat = mat.data_ptr<float>();
  a.mat_rows = (int)mat.size(0);
  a.my_row = (int)my_row;
  a.E = (int)mat.size(1);
  a.E_loc = (int)E_loc;
  a.ep_rank = (int)ep_rank;
  a.local_only = local_only ? 1 : 0;
  a.route_owner = route_owner.data_ptr<int32_t>();
  a.route_row = route_row.data_ptr<int32_t>();
  a.own_cnt = own_cnt.data_ptr<int32_t>();
  a.own_off = own_off.data_ptr<int32_t>();
  a.krange = krange.data_ptr<int32_t>();
  a.tile_expert = tile_expert.data_ptr<int32_t>();
  a.n_tiles = n_tiles.data_ptr<int32_t>();
  a.tiles_cap = (int)tile_expert.numel();
  pb::moe_plan(a, cur_stream());
}

// moe_dispatch(x bf16 [T, H], K, route_owner, route_row, dst_ptrs, ld_dst)
void moe_dispatch(const at::Tensor& x, int64_t K, const at::Tensor& owner, const at::Tensor& row,
                  const std::vector<int64_t>& dst, int64_t ldd) {
  check_rows(x, "moe_dispatch: x");
  check_i32(owner, x.size(0) * K, "moe_dispatch: route_owner");
  check_i32(row, x.size(0) * K, "moe_dispatch: route_row");
  TORCH_CHECK(ldd % 8 == 0 && ldd >= x.size(1), "moe_dispatch: destination row stride");
  const c10::cuda::CUDAGuard g(x.device());
  pb::moe_dispatch(x.data_ptr(), x.stride(0), (int)K, owner.data_ptr<int32_t>(), row.data_ptr<int32_t>(),
                   peer_bases(dst), ldd, x.size(1), x.size(0) * K, cur_stream());
}

// moe_copy_pad(src_ptr, ld_src, dst bf16 [rows_cap, H], tile_expert, n_tiles, own_cnt, own_off)
void moe_copy_pad(int64_t src_ptr, int64_t lds, at::Tensor& dst, const at::Tensor& tile_expert,
                  const at::Tensor& n_tiles, const at::Tensor& own_cnt, const at::Tensor& own_off) {
  check_rows(dst, "moe_copy_pad: dst");
  TORCH_CHECK(dst.size(0) == 128 * tile_expert.numel(), "moe_copy_pad: dst rows must be 128 x tiles_cap");
  TORCH_CHECK(lds % 8 == 0 && lds >= dst.size(1) && src_ptr % 16 == 0, "moe_copy_pad: source layout");
  check_i32(tile_expert, 1, "moe_copy_pad: tile_expert");
  check_i32(n_tiles, 1, "moe_copy_pad: n_tiles");
  check_i32(own_cnt, 1, "moe_copy_pad: own_cnt");
  check_i32(own_off, 1, "moe_copy_pad: own_off");
  const c10::cuda::CUDAGuard g(dst.device());
  pb::moe_copy_pad(reinterpret_cast<const void*>(src_ptr), lds, dst.data_ptr(), dst.stride(0), dst.size(1),
                   (int)tile_expert.numel(), tile_expert.data_ptr<int32_t>(), n_tiles.data_ptr<int32_t>(),
                   own_cnt.data_ptr<int32_t>(), own_off.data_ptr<int32_t>(), cur_stream());
}

// moe_combine(out bf16 [T, H], keep bf16 [T*K, H] or None, w fp32 [T, K] or None, route_owner, route_row,
//             src_ptrs, ld_src)
void moe_combine(at::Tensor& out, const c10::optional<at::Tensor>& keep, const c10::optional<at::Tensor>& w,
                 const at::Tensor& owner, const at::Tensor& row, const std::vector<int64_t>& src, int64_t lds) {
  check_rows(out, "moe_combine: out");
  const int64_t T = out.size(0);
  TORCH_CHECK(T == 0 || owner.numel() % T == 0, "moe_combine: routes per token");
  const int K = T ? (int)(owner.numel() / T) : 0;
  check_i32(owner, T * K, "moe_combine: route_owner");
  check_i32(row, T * K, "moe_combine: route_row");
  void* keep_ptr = nullptr;
  if (keep.has_value() && keep->defined()) {
    check_rows(*keep, "moe_combine: keep");
    TORCH_CHECK(keep->is_contiguous() && keep->size(0) == T * K && keep->size(1) == out.size(1), "moe_combine: keep");
    keep_ptr = keep->data_ptr();
  }
  const float* wp = nullptr;
  if (w.has_value() && w->defined()) {
    TORCH_CHECK(w->is_cuda() && w->scalar_type() == at::kFloat && w->is_contiguous() && w->numel() == T * K,
                "moe_combine: w fp32 [T, K]");
    wp = w->data_ptr<float>();
  }
  TORCH_CHECK(lds % 8 == 0 && lds >= out.size(1), "moe_combine: source row stride");
  const c10::cuda::CUDAGuard g(out.device());
  pb::moe_combine(out.data_ptr(), out.stride(0), keep_ptr, wp, owner.data_ptr<int32_t>(), row.data_ptr<int32_t>(),
                  peer_bases(src), lds, K, out.size(1), T, cur_stream());
}

// moe_combine_bwd(dout bf16 [T, H], kept bf16 [T*K, H], w fp32 [T, K], route_owner, route_row, dst_ptrs, ld_dst,
//                 dw fp32 [T, K])
void moe_combine_bwd(const at::Tensor& dout, const at::Tensor& kept, const at::Tensor& w, const at::Tensor& owner,
                     const at::Tensor& row, const std::vector<int64_t>& dst, int64_t ldd, at::Tensor& dw) {
  check_rows(dout, "moe_combine_bwd: dout");
  const int64_t T = dout.size(0);
  const int64_t n = owner.numel();
  TORCH_CHECK(T == 0 || n % T == 0, "moe_combine_bwd: routes per token");
  const int K = T ? (int)(n / T) : 0;
  check_rows(kept, "moe_combine_bwd: kept");
  TORCH_CHECK(kept.is_contiguous() && kept.size(0) == n && kept.size(1) == dout.size(1), "moe_combine_bwd: kept");
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == at::kFloat && w.is_contiguous() && w.numel() == n,
              "moe_combine_bwd: w fp32 [T, K]");
  TORCH_CHECK(dw.is_cuda() && dw.scalar_type() == at::kFloat && dw.is_contiguous() && dw.numel() == n,
              "moe_combine_bwd: dw fp32 [T, K]");
  check_i32(owner, n, "moe_combine_bwd: route_owner");
  check_i32(row, n, "moe_combine_bwd: route_row");
  TORCH_CHECK(ldd % 8 == 0 && ldd >= dout.size(1), "moe_combine_bwd: destination row stride");
  const c10::cuda::CUDAGuard g(dout.device());
  pb::moe_combine_bwd(dout.data_ptr(), dout.stride(0), kept.data_ptr(), w.data_ptr<float>(), owner.data_ptr<int32_t>(),
                      row.data_ptr<int32_t>(), peer_bases(dst), ldd, K, dout.size(1), n, dw.data_ptr<float>(),
                      cur_stream());
}

}  // namespace

void register_moe(pybind11::module& m) {
  m.def("moe_hist", &moe_hist);
  m.def("moe_plan", &moe_plan);
  m.def("moe_dispatch", &moe_dispatch);
  m.def("moe_copy_pad", &moe_copy_pad);
  m.def("moe_combine", &moe_combine);
  m.def("moe_combine_bwd", &moe_combine_bwd);
}
