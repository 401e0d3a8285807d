// Public interface of the persistent tcgen05 GEMM (gemm.cu).
//
//   C[m, n] = alpha * sum_k A(m, k) * B(n, k)   (+ epilogue)
//
// A is either K-major (row-major [M, K], element (m,k) at A[m*lda + k]) or
// MN-major (row-major [K, M], element (m,k) at A[k*lda + m]); B likewise with
// N in place of M.  With both operands K-major this is `x @ W.T` (the forward
// of nn.Linear); the MN-major forms give the data-gradient (dY @ W) and the
// weight-gradient (dY.T @ X) products without any transpose copies.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace pb {

enum GemmEpilogue : int {
  kEpiStoreBf16 = 0,      // C(bf16) = alpha*acc
  kEpiResidualBf16 = 1,   // C(bf16) = alpha*acc + R(bf16)
  kEpiStoreF32 = 2,       // C(f32)  = alpha*acc
  kEpiAccumBf16 = 3,      // C(bf16) += alpha*acc
  kEpiAccumF32 = 4,       // C(f32)  += alpha*acc
  kEpiSwiGLU = 5,         // B rows [0,N) are gate, [N,2N) are up (same ldb, "b_up_offset" rows
                          // apart): C(bf16) = silu(g)*u, and if R != null, R(bf16) receives the
                          // raw [g | u] pre-activations (ldr) for the backward.
};

struct GemmParams {
  const void* A;
  const void* B;
  void* C;
  const void* R;  // residual input (kEpiResidualBf16) or gate/up output (kEpiSwiGLU)
  int64_t lda, ldb, ldc, ldr;
  int M, N, K;
  bool a_mn, b_mn;
  int epi;
  float alpha;
  int64_t b_up_offset;  // kEpiSwiGLU: row offset (in N units) of the "up" half of B
  int max_ctas;         // 0 = one CTA per SM
  int kernel = 0;       // 0 = choose, 1 = one-CTA kernel, 2 = CTA-pair kernel
};

// Dispatches to the one-CTA (gemm.cu) or the CTA-pair (gemm_pair.cu) kernel.
void gemm_bf16(const GemmParams& p, cudaStream_t stream);
void gemm_bf16_pair(const GemmParams& p, cudaStream_t stream);

}  // namespace pb
