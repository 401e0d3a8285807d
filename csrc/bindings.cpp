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
          double alpha, const c10::optional<at::Tensor>& r, int64_t b_up_offset, int64_t n_out, int64_t kernel) {
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
  p.b_up_offset = b_up_offset;
  if (epi == pb::kEpiSwiGLU) {
    p.N = (int)n_out;
    TORCH_CHECK(b_up_offset + n_out <= b.size(0), "gemm: swiglu B too small");
  }
  TORCH_CHECK(out.size(0) == p.M && out.size(1) == p.N, "gemm: output shape mismatch");
  const bool f32 = epi == pb::kEpiStoreF32 || epi == pb::kEpiAccumF32;
  TORCH_CHECK(out.scalar_type() == (f32 ? at::kFloat : at::kBFloat16), "gemm: output dtype mismatch");
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

int64_t read_error(int64_t device) { return pb::read_error((int)device); }
void clear_error(int64_t device) { pb::clear_error((int)device); }

}  // namespace

void register_ops(pybind11::module& m);
void register_comm(pybind11::module& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "parallel_b200 sm_100a kernels";
  m.def("gemm", &gemm, "tcgen05 bf16 GEMM with fused epilogues", pybind11::arg("a"),
        pybind11::arg("b"), pybind11::arg("out"), pybind11::arg("a_mn"), pybind11::arg("b_mn"),
        pybind11::arg("epi"), pybind11::arg("alpha"), pybind11::arg("r") = pybind11::none(),
        pybind11::arg("b_up_offset") = 0, pybind11::arg("n_out") = 0, pybind11::arg("kernel") = 0);
  m.def("read_error", &read_error);
  m.def("clear_error", &clear_error);
  register_ops(m);
  register_comm(m);
}
