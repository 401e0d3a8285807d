// Python bindings for the sm_100a kernels.  Each binding validates tensor
// shapes / dtypes / strides, derives leading dimensions and launches on the
// current PyTorch stream.  The kernels themselves live in the .cu files and
// see only raw pointers.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "gemm.cuh"
#include "host_util.h"
#include "ops.cuh"

namespace {

#define CHECK_CUDA_BF16(t) \
  TORCH_CHECK((t).is_cuda() && (t).scalar_type() == at::kBFloat16, #t " must be a CUDA bf16 tensor")

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// gemm(a, b, out, a_mn, b_mn, epi, alpha, r, b_up_offset)
//   a: [M, K] (a_mn=False) or [K, M] (a_mn=True), unit inner stride
//   b: [N, K] (b_mn=False) or [K, N] (b_mn=True), unit inner stride
//   out: [M, N] bf16 or fp32 depending on epi
void gemm(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, bool a_mn, bool b_mn, int64_t epi,
          double alpha, const c10::optional<at::Tensor>& r, int64_t b_up_offset, int64_t n_out, int64_t kernel,
          int64_t splits, const c10::optional<at::Tensor>& ws, bool accumulate) {
  CHECK_CUDA_BF16(a);
  CHECK_CUDA_BF16(b);
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 2, "gemm: 2-D operands expected");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && out.stride(1) == 1,
              "gemm: operands need a unit inner stride");
  const c10::cuda::CUDAGuard guard(a.device());
  pb::GemmParams p{};
  p.A = a.data_ptr();
  p.B = b.data_ptr();
  p.C = out.data_ptr();
  p.lda = a.stride(0);
  p.ldb = b.stride(0);
  p.ldc = out.stride(0);
  p.a_mn = a_mn;
  p.b_mn = b_mn;
  p.M = a_mn ? a.size(1) : a.size(0);
  p.K = a_mn ? a.size(0) : a.size(1);
  p.N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == p.K, "gemm: K mismatch");
  p.epi = (int)epi;
  p.alpha = (float)alpha;
  p.max_ctas = 0;
  TORCH_CHECK(kernel >= 0 && kernel <= 2, "gemm: kernel must be 0 (choose), 1 (one CTA) or 2 (CTA pair)");
  p.kernel = (int)kernel;
  TORCH_CHECK(splits >= 1 && splits <= 16, "gemm: splits in [1, 16]");
  p.splits = (int)splits;
  p.b_up_offset = b_up_offset;
  if (epi == pb::kEpiSwiGLU) {
    p.N = (int)n_out;
    TORCH_CHECK(b_up_offset + n_out <= b.size(0), "gemm: swiglu B too small");
  }
  // split-K into fp32 slabs: out is [splits * M, N], slab s = rows [s * M, (s + 1) * M)
  const int64_t out_rows = (epi == pb::kEpiStoreF32 && splits > 1) ? (int64_t)p.M * splits : p.M;
  TORCH_CHECK(out.size(0) == out_rows && out.size(1) == p.N, "gemm: output shape mismatch");
  TORCH_CHECK(out_rows == p.M || out.stride(0) == p.N, "gemm: fp32 slabs must be contiguous [splits * M, N]");
  if (epi == pb::kEpiSplitOrdered) {
    // ws: fp32 [M, >= N] running sums of the K slices (contents irrelevant);
    // out: bf16 or fp32, written (or added to, accumulate) by the last slice
    TORCH_CHECK(ws.has_value() && ws->defined() && ws->is_cuda() && ws->scalar_type() == at::kFloat &&
                    ws->dim() == 2 && ws->stride(1) == 1 && ws->size(0) >= p.M && ws->size(1) >= p.N,
                "gemm: the ordered split-K epilogue needs an fp32 workspace [M, N]");
    TORCH_CHECK(out.scalar_type() == at::kFloat || out.scalar_type() == at::kBFloat16, "gemm: output dtype");
    p.ws = ws->data_ptr<float>();
    p.ws_ld = ws->stride(0);
    p.out_f32 = out.scalar_type() == at::kFloat;
    p.accumulate = accumulate;
  } else {
    const bool f32 = epi == pb::kEpiStoreF32 || epi == pb::kEpiAccumF32 || epi == pb::kEpiAtomicF32;
    TORCH_CHECK(out.scalar_type() == (f32 ? at::kFloat : at::kBFloat16), "gemm: output dtype mismatch");
  }
  if (r.has_value() && r->defined()) {
    CHECK_CUDA_BF16(*r);
    TORCH_CHECK(r->stride(1) == 1, "gemm: r needs unit inner stride");
    p.R = r->data_ptr();
    p.ldr = r->stride(0);
  } else {
    TORCH_CHECK(epi != pb::kEpiResidualBf16, "gemm: residual epilogue needs r");
    p.R = nullptr;
    p.ldr = 0;
  }
  pb::gemm_bf16(p, cur_stream());
}

// gemm_ag: out = gather(A shards) @ B^T (or @ B when b_mn) with the
// sequence-parallel all-gather inside the GEMM kernel.  `dst` [T, K] receives
// the gathered A (kept for the weight gradient); src_ptrs[r] are the ranks'
// shards [batch*seq_local, K] (peer pointers of a symmetric buffer); flags is
// an int32 tensor with one counter per 256-row block of dst, bumped by
// 256/16 per block and call; `target` = that count after this call.
void gemm_ag(at::Tensor& dst, const std::vector<int64_t>& src_ptrs, int64_t src_ld, at::Tensor& flags,
             int64_t target, int64_t seq, int64_t seq_local, int64_t batch, const std::vector<int64_t>& m_order,
             const at::Tensor& b, at::Tensor& out, bool b_mn, int64_t epi, double alpha,
             const c10::optional<at::Tensor>& r, int64_t b_up_offset, int64_t n_out) {
  CHECK_CUDA_BF16(dst);
  CHECK_CUDA_BF16(b);
  TORCH_CHECK(dst.is_contiguous() && flags.is_cuda() && flags.scalar_type() == at::kInt, "gemm_ag: dst / flags");
  TORCH_CHECK(src_ptrs.size() >= 1 && src_ptrs.size() <= 8, "gemm_ag: 1..8 shards");
  TORCH_CHECK(m_order.size() == (size_t)((dst.size(0) + 255) / 256) && m_order.size() <= 64, "gemm_ag: m_order");
  TORCH_CHECK(flags.numel() >= (int64_t)m_order.size(), "gemm_ag: flags too small");
  const c10::cuda::CUDAGuard guard(dst.device());
  pb::GatherArgs g{};
  for (size_t i = 0; i < src_ptrs.size(); ++i) g.src[i] = reinterpret_cast<const void*>(src_ptrs[i]);
  g.dst = dst.data_ptr();
  g.flags = flags.data_ptr<int>();
  g.target = (int)target;
  g.nranks = (int)src_ptrs.size();
  g.seq = (int)seq;
  g.seq_local = (int)seq_local;
  g.batch = (int)batch;
  g.src_ld = src_ld;
  g.n_blocks = (int)m_order.size();
  for (size_t i = 0; i < m_order.size(); ++i) g.m_order[i] = (int)m_order[i];
  TORCH_CHECK(seq == seq_local * (int64_t)src_ptrs.size() && dst.size(0) == batch * seq, "gemm_ag: sizes");
  pb::GemmParams p{};
  p.A = dst.data_ptr();
  p.B = b.data_ptr();
  p.C = out.data_ptr();
  p.lda = dst.stride(0);
  p.ldb = b.stride(0);
  p.ldc = out.stride(0);
  p.a_mn = false;
  p.b_mn = b_mn;
  p.M = dst.size(0);
  p.K = dst.size(1);
  p.N = b_mn ? b.size(1) : b.size(0);
  p.epi = (int)epi;
  p.alpha = (float)alpha;
  p.b_up_offset = b_up_offset;
  if (epi == pb::kEpiSwiGLU) {
    p.N = (int)n_out;
    TORCH_CHECK(b_up_offset + n_out <= b.size(0), "gemm_ag: swiglu B too small");
  }
  TORCH_CHECK(out.size(0) == p.M && out.size(1) == p.N && out.scalar_type() == at::kBFloat16, "gemm_ag: out");
  if (r.has_value() && r->defined()) {
    CHECK_CUDA_BF16(*r);
    p.R = r->data_ptr();
    p.ldr = r->stride(0);
  }
  TORCH_CHECK(epi == pb::kEpiStoreBf16 || epi == pb::kEpiSwiGLU, "gemm_ag: store or SwiGLU epilogue");
  p.gather = &g;
  pb::gemm_bf16(p, cur_stream());
}

// gemm_rs: partial = A @ B^T (or A @ B when b_mn) over the full sequence, each
// output row stored as bf16 into its owner's receive buffer (peer_ptrs[owner])
// at slot `slot`: row (slot*slot_rows + b*seq_local + s % seq_local), stride ldc.
void gemm_rs(const at::Tensor& a, const at::Tensor& b, bool b_mn, double alpha, const std::vector<int64_t>& peer_ptrs,
             int64_t ldc, int64_t seq, int64_t seq_local, int64_t slot, int64_t slot_rows) {
  CHECK_CUDA_BF16(a);
  CHECK_CUDA_BF16(b);
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1, "gemm_rs: unit inner strides");
  TORCH_CHECK(peer_ptrs.size() >= 1 && peer_ptrs.size() <= 8 && seq == seq_local * (int64_t)peer_ptrs.size(),
              "gemm_rs: ranks / sequence");
  const c10::cuda::CUDAGuard guard(a.device());
  pb::ScatterArgs sc{};
  for (size_t i = 0; i < peer_ptrs.size(); ++i) sc.peer[i] = reinterpret_cast<void*>(peer_ptrs[i]);
  sc.nranks = (int)peer_ptrs.size();
  sc.seq = (int)seq;
  sc.seq_local = (int)seq_local;
  sc.slot = (int)slot;
  sc.slot_rows = slot_rows;
  pb::GemmParams p{};
  p.A = a.data_ptr();
  p.B = b.data_ptr();
  p.C = reinterpret_cast<void*>(peer_ptrs[0]);
  p.lda = a.stride(0);
  p.ldb = b.stride(0);
  p.ldc = ldc;
  p.a_mn = false;
  p.b_mn = b_mn;
  p.M = a.size(0);
  p.K = a.size(1);
  p.N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == p.K, "gemm_rs: K mismatch");
  TORCH_CHECK(p.M % seq == 0, "gemm_rs: rows must be whole sequences");
  p.epi = pb::kEpiStoreBf16;
  p.alpha = (float)alpha;
  p.scatter = &sc;
  pb::gemm_bf16(p, cur_stream());
}

// gemm_grouped(mode, a, b, out, work int32 [n, 4], krange int32 [E, 2] or None, E, b_mn, epi, alpha,
//              r=None, b_up_offset=0, n_out=0)
//   mode 1: a [M_pad, K], b [E, b_rows, K] (or [E, K, N] with b_mn), out [M_pad, N]
//   mode 2: a [rows, M_group], b [rows, N], out [E, M_group, N]
void gemm_grouped(int64_t mode, const at::Tensor& a, const at::Tensor& b, at::Tensor& out, const at::Tensor& work,
                  const c10::optional<at::Tensor>& krange, bool b_mn, int64_t epi, double alpha,
                  const c10::optional<at::Tensor>& r, int64_t b_up_offset, int64_t n_out,
                  const c10::optional<at::Tensor>& tile_expert, const c10::optional<at::Tensor>& n_tiles) {
  CHECK_CUDA_BF16(a);
  CHECK_CUDA_BF16(b);
  TORCH_CHECK(a.is_contiguous() && b.is_contiguous() && out.is_contiguous(), "gemm_grouped: contiguous operands");
  TORCH_CHECK(work.is_cuda() && work.scalar_type() == at::kInt && work.dim() == 2 && work.size(1) == 4 &&
                  work.is_contiguous(),
              "gemm_grouped: work must be int32 [n, 4]");
  const c10::cuda::CUDAGuard guard(a.device());
  pb::GroupedGemmParams p;
  p.mode = (int)mode;
  p.A = a.data_ptr();
  p.B = b.data_ptr();
  p.C = out.data_ptr();
  p.b_mn = b_mn;
  p.epi = (int)epi;
  p.alpha = (float)alpha;
  p.b_up_offset = b_up_offset;
  p.work = reinterpret_cast<const int4*>(work.data_ptr<int>());
  p.n_work = (int)work.size(0);
  if (mode == 1) {
    TORCH_CHECK(a.dim() == 2 && b.dim() == 3 && out.dim() == 2, "gemm_grouped rows: a 2-D, b 3-D, out 2-D");
    p.E = (int)b.size(0);
    p.M_total = (int)a.size(0);
    p.K = (int)a.size(1);
    p.lda = a.stride(0);
    p.ldb = b.stride(1);
    p.b_rows = b_mn ? b.size(1) : b.size(1);
    p.N = epi == pb::kEpiSwiGLU ? (int)n_out : (int)(b_mn ? b.size(2) : b.size(1));
    TORCH_CHECK((b_mn ? b.size(1) : b.size(2)) == p.K, "gemm_grouped rows: K mismatch");
    TORCH_CHECK(out.size(0) == p.M_total && out.size(1) == p.N, "gemm_grouped rows: out shape");
  } else {
    TORCH_CHECK(mode == 2 && krange.has_value() && krange->defined(), "gemm_grouped: mode 2 needs krange");
    TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 3 && a.size(0) == b.size(0), "gemm_grouped k: shapes");
    TORCH_CHECK(krange->is_cuda() && krange->scalar_type() == at::kInt && krange->is_contiguous() &&
                    krange->numel() == 2 * out.size(0),
                "gemm_grouped k: krange int32 [E, 2]");
    p.E = (int)out.size(0);
    p.M_group = (int)out.size(1);
    p.N = (int)out.size(2);
    p.rows = (int)a.size(0);
    p.K = (int)a.size(0);
    p.M_total = p.E * p.M_group;
    p.lda = a.stride(0);
    p.ldb = b.stride(0);
    TORCH_CHECK(a.size(1) == p.M_group && b.size(1) == p.N, "gemm_grouped k: operand widths");
    p.krange = reinterpret_cast<const int2*>(krange->data_ptr<int>());
  }
  const bool f32 = epi == pb::kEpiStoreF32 || epi == pb::kEpiAccumF32;
  TORCH_CHECK(out.scalar_type() == (f32 ? at::kFloat : at::kBFloat16), "gemm_grouped: output dtype");
  p.ldc = mode == 1 ? out.stride(0) : out.stride(1);
  if (r.has_value() && r->defined()) {
    CHECK_CUDA_BF16(*r);
    p.R = r->data_ptr();
    p.ldr = r->stride(0);
  }
  if (tile_expert.has_value() && tile_expert->defined()) {
    TORCH_CHECK(mode == 1 && n_tiles.has_value() && n_tiles->defined(), "gemm_grouped: device tiles need rows mode");
    TORCH_CHECK(tile_expert->is_cuda() && tile_expert->scalar_type() == at::kInt && tile_expert->is_contiguous() &&
                    tile_expert->numel() * 128 == p.M_total,
                "gemm_grouped: tile_expert int32 [M_pad / 128]");
    TORCH_CHECK(n_tiles->is_cuda() && n_tiles->scalar_type() == at::kInt && n_tiles->numel() >= 1,
                "gemm_grouped: n_tiles int32 [1]");
    p.tile_expert = tile_expert->data_ptr<int>();
    p.n_tiles = n_tiles->data_ptr<int>();
  }
  pb::gemm_grouped(p, cur_stream());
}

int64_t read_error(int64_t device) { return pb::read_error((int)device); }
void clear_error(int64_t device) { pb::clear_error((int)device); }
// Test hook: write an error code into the device's error word from the host
// (what a bounded device wait that gave up would leave there).
void set_error_for_test(int64_t device, int64_t code) {
  const int c = (int)code;
  PB_CUDA_CHECK(cudaMemcpy(pb::error_word((int)device), &c, sizeof(int), cudaMemcpyHostToDevice));
}

}  // namespace

void register_ops(pybind11::module& m);
void register_comm(pybind11::module& m);
void register_moe(pybind11::module& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "parallel_b200 sm_100a kernels";
  m.def("gemm", &gemm, "tcgen05 bf16 GEMM with fused epilogues", pybind11::arg("a"),
        pybind11::arg("b"), pybind11::arg("out"), pybind11::arg("a_mn"), pybind11::arg("b_mn"),
        pybind11::arg("epi"), pybind11::arg("alpha"), pybind11::arg("r") = pybind11::none(),
        pybind11::arg("b_up_offset") = 0, pybind11::arg("n_out") = 0, pybind11::arg("kernel") = 0,
        pybind11::arg("splits") = 1, pybind11::arg("ws") = pybind11::none(), pybind11::arg("accumulate") = false);
  m.def("gemm_ag", &gemm_ag, "GEMM with the sequence-parallel all-gather of A in the same kernel",
        pybind11::arg("dst"), pybind11::arg("src_ptrs"), pybind11::arg("src_ld"), pybind11::arg("flags"),
        pybind11::arg("target"), pybind11::arg("seq"), pybind11::arg("seq_local"), pybind11::arg("batch"),
        pybind11::arg("m_order"), pybind11::arg("b"), pybind11::arg("out"), pybind11::arg("b_mn"),
        pybind11::arg("epi"), pybind11::arg("alpha"), pybind11::arg("r") = pybind11::none(),
        pybind11::arg("b_up_offset") = 0, pybind11::arg("n_out") = 0);
  m.def("gemm_rs", &gemm_rs, "GEMM whose epilogue stores rows into their sequence-parallel owners' buffers",
        pybind11::arg("a"), pybind11::arg("b"), pybind11::arg("b_mn"), pybind11::arg("alpha"),
        pybind11::arg("peer_ptrs"), pybind11::arg("ldc"), pybind11::arg("seq"), pybind11::arg("seq_local"),
        pybind11::arg("slot"), pybind11::arg("slot_rows"));
  m.def("gemm_grouped", &gemm_grouped, "grouped (mixture-of-experts) GEMM driven by a device work table",
        pybind11::arg("mode"), pybind11::arg("a"), pybind11::arg("b"), pybind11::arg("out"), pybind11::arg("work"),
        pybind11::arg("krange"), pybind11::arg("b_mn"), pybind11::arg("epi"), pybind11::arg("alpha"),
        pybind11::arg("r") = pybind11::none(), pybind11::arg("b_up_offset") = 0, pybind11::arg("n_out") = 0,
        pybind11::arg("tile_expert") = pybind11::none(), pybind11::arg("n_tiles") = pybind11::none());
  m.def("grouped_tile_n", [](int64_t mode, int64_t n) { return (int64_t)pb::grouped_bn((int)mode, (int)n); },
        "column tile width of the grouped GEMM for a product with n output columns (mode 1 rows, 2 k)");
  m.def("read_error", &read_error);
  m.def("clear_error", &clear_error);
  m.def("set_error_for_test", &set_error_for_test);
  register_ops(m);
  register_comm(m);
  register_moe(m);
}
