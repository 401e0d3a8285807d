// Launchers of the memory-bound sm_100a kernels (norms, RoPE, activations,
// embedding, cross-entropy, optimizer, gradient norm).  All take raw device
// pointers and run on the given stream; shapes are validated by the Python
// bindings.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace pb {

// ---- RMSNorm over the last dim (norm.cu)
// y = bf16(w * bf16(x * rstd)), rstd = rsqrt(mean(x^2) + eps)   (fp32 math)
void rmsnorm_fwd(const void* x, int64_t ldx, const void* w, void* y, int64_t ldy, float* rstd,
                 int rows, int cols, float eps, cudaStream_t s);
// dx = rstd * (w*dy - xhat * mean(w*dy*xhat)); dw_part (f32, optional) is a
// [rmsnorm_bwd_grid(rows), cols] matrix of block partials of
// sum_rows dy * bf16(xhat) (each block writes its row; sum_slices finishes the
// weight gradient in a fixed order, so it is deterministic).
// dres (optional, bf16 [rows, cols]) is added into dx: the residual-stream
// gradient of "x feeds both norm(x) and a residual add".
int rmsnorm_bwd_grid(int rows);
void rmsnorm_bwd(const void* dy, int64_t lddy, const void* x, int64_t ldx, const void* w,
                 const float* rstd, void* dx, int64_t lddx, float* dw_part, int rows, int cols,
                 cudaStream_t s, const void* dres = nullptr, int64_t lddres = 0);

// ---- per-head RMSNorm of q and k + rotate-half RoPE (norm.cu)
// qkv: [T, (nq + 2*nkv) * D] (row stride ldqkv); writes q_out [T, nq*D],
// k_out [T, nkv*D] (row strides ldq / ldk) and rstd [T, nq + nkv].
// cos/sin: bf16 tables [S, D] (HF layout: both halves equal); pos = t % S.
void qknorm_rope_fwd(const void* qkv, int64_t ldqkv, const void* qw, const void* kw,
                     const void* cos, const void* sin, void* q_out, int64_t ldq, void* k_out,
                     int64_t ldk, float* rstd, int T, int S, int nq, int nkv, int D, float eps,
                     cudaStream_t s);
// Backward: dq/dk: grads w.r.t. q_out/k_out.  Writes pre-norm grads into
// dqkv's q and k column blocks; dw_part (f32, optional) receives the block
// partials of the q / k norm weight grads, [qknorm_rope_bwd_grid(..), 2 * D]
// (q weights in the first D columns), finished by sum_slices.
int qknorm_rope_bwd_grid(int T, int nq, int nkv);
void qknorm_rope_bwd(const void* dq, int64_t lddq, const void* dk, int64_t lddk, const void* qkv,
                     int64_t ldqkv, const void* qw, const void* kw, const void* cos,
                     const void* sin, const float* rstd, void* dqkv, int64_t lddqkv,
                     float* dw_part, int T, int S, int nq, int nkv, int D, cudaStream_t s);

// ---- SwiGLU backward (act.cu): gu = [g | u] (row stride ldgu, u at column I)
// dgu[:, :I] = dh * u * silu'(g), dgu[:, I:] = dh * silu(g)
void swiglu_bwd(const void* dh, int64_t lddh, const void* gu, int64_t ldgu, void* dgu,
                int64_t lddgu, int T, int I, cudaStream_t s, const int* tiles128 = nullptr);
// h = silu(g) * u (used on the CPU-parity path and by the MoE experts)

// ---- embedding (act.cu)
void embedding_fwd(const int64_t* ids, const void* table, int64_t ldt, void* out, int64_t ldo,
                   int T, int H, int64_t vocab_start, int64_t vocab_rows, cudaStream_t s);
// grad_f32[ids[t]-vocab_start, :] += dy[t, :] (fp32 atomics, rows outside skipped)
void embedding_bwd(const int64_t* sorted_ids, const int64_t* perm, const void* dy, int64_t lddy, void* grad,
                   int64_t ldg, int T, int H, int64_t vocab_start, int64_t vocab_rows, bool accumulate,
                   cudaStream_t s);
// x (bf16, n elements) *= *s_dev unless *s_dev == 1
void scale_by_scalar(void* x, int64_t n, const float* s_dev, cudaStream_t s);

// ---- cross entropy over a [T, V] bf16 logits block (ce.cu)
// Row t's label is labels[t]; labels < 0 are ignored.  This rank holds vocab
// columns [v0, v0+V).  If lse_given, row_lse holds the (global) log-sum-exp,
// else it is computed from this block and written.  row_target receives the
// label's logit when the label falls inside this block (else 0).
// If write_grad, logits are overwritten with (softmax - onehot) * scale[0]
// (zeros for ignored rows).
void ce_fwd_bwd(void* logits, int64_t ld, const int64_t* labels, int T, int V, int64_t v0,
                const float* scale, float* row_lse, bool lse_given, float* row_target,
                bool write_grad, cudaStream_t s);
// inv[0] = 1 / max(1, #{t : labels[t] >= 0})   (one block)
void ce_valid_inv(const int64_t* labels, int T, float* inv, cudaStream_t s);
// out[0] = (accumulate ? out[0] : 0) + inv[0] * sum over valid rows of (lse - tgt),
// summed in a fixed order (one block, no atomics: the same bits on every run)
void ce_loss_reduce(const float* lse, const float* tgt, const int64_t* labels, int T, const float* inv, float* out,
                    bool accumulate, cudaStream_t s);
// Per-row max and sum(exp(x - max)) of this block (vocab-parallel merge).
void ce_row_stats(const void* logits, int64_t ld, int T, int V, float* row_max, float* row_sumexp,
                  cudaStream_t s);

// ---- casts / elementwise helpers (act.cu)
void cast_f32_to_bf16(const float* src, void* dst, int64_t n, cudaStream_t s);
// out[i] = (accumulate ? out[i] : 0) + sum_{k < slices} parts[k * stride + i] for i < len,
// summed in slice order (deterministic); out is bf16 (out_bf16) or f32.  Finishes
// block-partial weight gradients and split-K GEMM slices without atomics.
void sum_slices(const float* parts, int slices, int64_t len, int64_t stride, void* out, bool out_bf16,
                bool accumulate, cudaStream_t s);

// ---- optimizer (optim.cu)
// Multi-tensor AdamW over `n` segments.  Each segment: param (bf16),
// grad (bf16 or f32 when grad_f32), exp_avg / exp_avg_sq (bf16 or f32 when
// state_f32), numel.  grad_scale multiplies every gradient (clipping);
// `skip` (device int, may be null) makes the kernel a no-op when non-zero.
struct AdamSeg {
  void* p;
  const void* g;
  void* m;
  void* v;
  int64_t n;
};
void adamw_multi(const AdamSeg* segs_host, int nseg, float lr, float beta1, float beta2, float eps,
                 float wd, int step, const float* grad_scale_dev, const int* skip_dev, const float* hyper_dev,
                 bool grad_f32, bool state_f32, cudaStream_t s);
// Sum of squares of all segments into out[0] (f32, accumulated) and sets
// out_flag[0] = 1 if any element is non-finite.
struct NormSeg {
  const void* g;
  int64_t n;
  float weight;  // contribution multiplier (0 drops the segment)
};
// parts: device scratch of 2 * sumsq_chunks(..) floats (per-chunk sum, non-finite bit);
// out[0] = (accumulate ? out[0] : 0) + sum of squares (weighted), added in chunk order;
// out_flag[0] (optional) = (accumulate ? out_flag[0] : 0) | any non-finite element.
int64_t sumsq_chunks(const NormSeg* segs_host, int nseg);
void sumsq_multi(const NormSeg* segs_host, int nseg, bool f32, float* parts, float* out, int* out_flag,
                 bool accumulate, cudaStream_t s);
// scale = min(max_norm / (sqrt(total) + 1e-6), 1)  written to scale_out[0]
void clip_coef(const float* total_sumsq, float max_norm, float* scale_out, cudaStream_t s);

// Mixture-of-experts router (csrc/router.cu): softmax + top-k + renormalisation
// + route histogram of bf16 logits [T, E] (row stride ld); and its backward.
void router_fwd(const void* logits, int64_t ld, int T, int E, int K, bool renorm, float* probs, float* topv,
                int64_t* topi, int* counts, cudaStream_t s);
void router_bwd(const float* probs, const float* dprobs, const float* dtopv, const int64_t* topi, int T, int E, int K,
                bool renorm, void* dlogits, int64_t ld, cudaStream_t s);
// Load-balancing loss statistics over probabilities [R, E]: per-expert top-k
// counts and sums of the second softmax.
// parts: [aux_stats_grid(R), 2E] block partials (counts, then sums), finished
// by sum_slices in block order (deterministic)
int aux_stats_grid(int R);
void aux_stats(const float* probs, int R, int E, int K, float* parts, cudaStream_t s);
void aux_stats_bwd(const float* probs, const float* gsum, int R, int E, float* dprobs, cudaStream_t s);

}  // namespace pb
