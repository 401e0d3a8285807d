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
  kEpiStoreF32 = 2,       // C(f32)  = alpha*acc; with splits > 1, K slice s writes slab s of
                          // C [splits, M, ldc] (fp32 partials, summed afterwards in slice order)
  kEpiAccumBf16 = 3,      // C(bf16) += alpha*acc
  kEpiAccumF32 = 4,       // C(f32)  += alpha*acc
  kEpiSwiGLU = 5,         // B rows [0,N) are gate, [N,2N) are up (same ldb, "b_up_offset" rows
                          // apart): C(bf16) = silu(g)*u, and if R != null, R(bf16) receives the
                          // raw [g | u] pre-activations (ldr) for the backward.
  kEpiAtomicF32 = 6,      // C(f32) += alpha*acc with atomic adds (split-K partial sums)
  kEpiSplitOrdered = 7,   // split-K without atomics: K slice s adds alpha*acc to the fp32 running
                          // sum of slices 0..s-1 (ws, ld ws_ld) once slice s-1 of the same tile
                          // published it, and the last slice writes C (bf16, or fp32 when
                          // out_f32; added to C's old value when accumulate).  The slices add in
                          // slice order, so the result has the same bits on every run.
};

// Sequence-parallel reduce-scatter epilogue: output row m = b*seq + s (a row
// of the full-sequence partial product) is stored, as bf16, into the receive
// buffer of its owner rank s / seq_local, in the sender's slot:
//   peer[owner] + (slot * slot_rows + b*seq_local + s % seq_local) * ldc.
// The owner later sums its nranks slots.
struct ScatterArgs {
  void* peer[8];
  int nranks = 0, seq = 0, seq_local = 0, slot = 0;
  int64_t slot_rows = 0;
};

// Sequence-parallel all-gather fused into the GEMM's A operand: rank r holds
// rows [b*seq_local, (b+1)*seq_local) of batch b in src[r]; the kernel's copy
// warps assemble dst (row b*seq + r*seq_local + sl) one 256-row block at a
// time, bump flags[block] per finished piece, and the TMA producer starts a
// tile only once its A block reached `target`.  M tiles run in m_order.
struct GatherArgs {
  const void* src[8];
  void* dst;
  int* flags;
  int target = 0;  // flag value of a complete block for this call
  int nranks = 0, seq = 0, seq_local = 0, batch = 0;
  int64_t src_ld = 0;  // row stride of the shards (elements)
  int n_blocks = 0;
  int m_order[64];
};
constexpr int kGatherRowsPerPiece = 16;

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
  int splits = 1;       // split-K slices (CTA-pair kernel, kEpiAtomicF32 / kEpiSplitOrdered)
  float* ws = nullptr;  // kEpiSplitOrdered: fp32 running sums [M, ws_ld] (no initial value needed)
  int64_t ws_ld = 0;
  bool out_f32 = false;     // kEpiSplitOrdered: C is fp32 (else bf16)
  bool accumulate = false;  // kEpiSplitOrdered: C += result
  const ScatterArgs* scatter = nullptr;  // kEpiStoreBf16 rows to their sequence-parallel owners
  const GatherArgs* gather = nullptr;    // A assembled from sequence-parallel shards in-kernel
};

// Grouped (mixture-of-experts) products, gemm_grouped.cu.  work: int4 per
// tile {expert, M tile, N tile, 0}; rows of one expert start at a 128-row
// aligned offset of A / C and are separated by zero rows.
//   mode 1 (rows): C[M_total, N] = A[M_total, K] x B_e, B stacked [E][b_rows][K]
//     (K-major) or [E][K][N] (b_mn); SwiGLU takes gate rows [0, N) and up rows
//     [b_up_offset, b_up_offset + N) of B_e.
//   mode 2 (k): C[E][M_group][N] = A_e^T B_e over rows krange[e] of
//     A [rows, M_group] and B [rows, N].
struct GroupedGemmParams {
  int mode = 1;
  const void* A = nullptr;
  const void* B = nullptr;
  void* C = nullptr;
  const void* R = nullptr;
  int64_t lda = 0, ldb = 0, ldc = 0, ldr = 0;
  int E = 0, M_total = 0, M_group = 0, rows = 0, N = 0, K = 0;
  int64_t b_rows = 0;
  bool b_mn = false;
  int epi = kEpiStoreBf16;
  float alpha = 1.f;
  int64_t b_up_offset = 0;
  const int4* work = nullptr;
  int n_work = 0;
  const int2* krange = nullptr;
  // rows mode over a device-described padded matrix: when tile_expert is set,
  // the work items are every (128-row tile, N tile) of the first *n_tiles
  // tiles, with the tile's expert from tile_expert; `work` / `n_work` are
  // unused and the grid is sized for M_total / 128 tiles
  const int* tile_expert = nullptr;
  const int* n_tiles = nullptr;
};
void gemm_grouped(const GroupedGemmParams& p, cudaStream_t stream);
// Column tile width (128 or 256) the grouped GEMM uses for a product with N
// output columns in `mode` (1 rows, 2 k); k-mode work tables tile N by it.
int grouped_bn(int mode, int N);

// Dispatches to the one-CTA (gemm.cu) or the CTA-pair (gemm_pair.cu) kernel.
void gemm_bf16(const GemmParams& p, cudaStream_t stream);
void gemm_bf16_pair(const GemmParams& p, cudaStream_t stream);

}  // namespace pb
