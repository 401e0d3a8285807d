// Bindings of the memory-bound kernels (ops.cuh).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "attention.cuh"
#include "ops.cuh"

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

#define CHECK_BF16(t) \
  TORCH_CHECK((t).is_cuda() && (t).scalar_type() == at::kBFloat16 && (t).stride(-1) == 1, #t " must be CUDA bf16 with unit inner stride")
#define CHECK_F32(t) \
  TORCH_CHECK((t).is_cuda() && (t).scalar_type() == at::kFloat && (t).is_contiguous(), #t " must be contiguous CUDA fp32")

// Finish block partials [slices, len] (row stride `stride`) into `out` (bf16 or f32, contiguous, len elements).
void finish_partials(const at::Tensor& parts, int slices, int64_t len, int64_t stride, int64_t offset,
                     at::Tensor& out) {
  TORCH_CHECK(out.is_cuda() && out.is_contiguous() && out.numel() == len &&
                  (out.scalar_type() == at::kBFloat16 || out.scalar_type() == at::kFloat),
              "weight gradient: contiguous bf16 / fp32 CUDA tensor of ", len, " elements");
  pb::sum_slices(parts.data_ptr<float>() + offset, slices, len, stride, out.data_ptr(),
                 out.scalar_type() == at::kBFloat16, false, at::cuda::getCurrentCUDAStream().stream());
}

float* opt_f32(const c10::optional<at::Tensor>& t) {
  if (!t.has_value() || !t->defined()) return nullptr;
  CHECK_F32(*t);
  return t->data_ptr<float>();
}

void rmsnorm_fwd(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, const c10::optional<at::Tensor>& rstd,
                 double eps) {
  CHECK_BF16(x); CHECK_BF16(w); CHECK_BF16(y);
  TORCH_CHECK(x.dim() == 2 && y.dim() == 2, "rmsnorm: 2-D");
  const c10::cuda::CUDAGuard g(x.device());
  pb::rmsnorm_fwd(x.data_ptr(), x.stride(0), w.data_ptr(), y.data_ptr(), y.stride(0), opt_f32(rstd), x.size(0),
                  x.size(1), (float)eps, cur_stream());
}

void rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w, const at::Tensor& rstd,
                 at::Tensor& dx, const c10::optional<at::Tensor>& dw, const c10::optional<at::Tensor>& dres) {
  CHECK_BF16(dy); CHECK_BF16(x); CHECK_BF16(w); CHECK_BF16(dx); CHECK_F32(rstd);
  const c10::cuda::CUDAGuard g(x.device());
  const void* rp = nullptr;
  int64_t ldr = 0;
  if (dres.has_value() && dres->defined()) {
    CHECK_BF16(*dres);
    TORCH_CHECK(dres->size(0) == x.size(0) && dres->size(1) == x.size(1), "rmsnorm_bwd: dres shape");
    rp = dres->data_ptr();
    ldr = dres->stride(0);
  }
  // dw (optional, bf16 or fp32 [cols]) is overwritten: block partials, then a fixed-order sum
  at::Tensor parts;
  float* pp = nullptr;
  const int grid = pb::rmsnorm_bwd_grid((int)x.size(0));
  if (dw.has_value() && dw->defined()) {
    parts = at::empty({grid, x.size(1)}, x.options().dtype(at::kFloat));
    pp = parts.data_ptr<float>();
  }
  pb::rmsnorm_bwd(dy.data_ptr(), dy.stride(0), x.data_ptr(), x.stride(0), w.data_ptr(), rstd.data_ptr<float>(),
                  dx.data_ptr(), dx.stride(0), pp, x.size(0), x.size(1), cur_stream(), rp, ldr);
  if (pp) {
    at::Tensor out = *dw;
    finish_partials(parts, grid, x.size(1), x.size(1), 0, out);
  }
}

void qknorm_rope_fwd(const at::Tensor& qkv, const at::Tensor& qw, const at::Tensor& kw, const at::Tensor& cos,
                     const at::Tensor& sin, at::Tensor& q, at::Tensor& k, at::Tensor& rstd, int64_t S, int64_t nq,
                     int64_t nkv, double eps) {
  CHECK_BF16(qkv); CHECK_BF16(qw); CHECK_BF16(kw); CHECK_BF16(cos); CHECK_BF16(sin); CHECK_BF16(q); CHECK_BF16(k);
  CHECK_F32(rstd);
  const c10::cuda::CUDAGuard g(qkv.device());
  const int D = (int)qw.size(0);
  pb::qknorm_rope_fwd(qkv.data_ptr(), qkv.stride(0), qw.data_ptr(), kw.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                      q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), rstd.data_ptr<float>(), qkv.size(0),
                      (int)S, (int)nq, (int)nkv, D, (float)eps, cur_stream());
}

void qknorm_rope_bwd(const at::Tensor& dq, const at::Tensor& dk, const at::Tensor& qkv, const at::Tensor& qw,
                     const at::Tensor& kw, const at::Tensor& cos, const at::Tensor& sin, const at::Tensor& rstd,
                     at::Tensor& dqkv, const c10::optional<at::Tensor>& dqw, const c10::optional<at::Tensor>& dkw,
                     int64_t S, int64_t nq, int64_t nkv) {
  CHECK_BF16(dq); CHECK_BF16(dk); CHECK_BF16(qkv); CHECK_BF16(dqkv); CHECK_F32(rstd);
  const c10::cuda::CUDAGuard g(qkv.device());
  const int D = (int)qw.size(0);
  // dqw / dkw (optional, bf16 or fp32 [D]) are overwritten: block partials, then fixed-order sums
  const bool want = (dqw.has_value() && dqw->defined()) || (dkw.has_value() && dkw->defined());
  const int grid = pb::qknorm_rope_bwd_grid((int)qkv.size(0), (int)nq, (int)nkv);
  at::Tensor parts;
  if (want) parts = at::empty({grid, 2 * D}, qkv.options().dtype(at::kFloat));
  pb::qknorm_rope_bwd(dq.data_ptr(), dq.stride(0), dk.data_ptr(), dk.stride(0), qkv.data_ptr(), qkv.stride(0),
                      qw.data_ptr(), kw.data_ptr(), cos.data_ptr(), sin.data_ptr(), rstd.data_ptr<float>(),
                      dqkv.data_ptr(), dqkv.stride(0), want ? parts.data_ptr<float>() : nullptr, qkv.size(0), (int)S,
                      (int)nq, (int)nkv, D, cur_stream());
  if (dqw.has_value() && dqw->defined()) {
    at::Tensor out = *dqw;
    finish_partials(parts, grid, D, 2 * D, 0, out);
  }
  if (dkw.has_value() && dkw->defined()) {
    at::Tensor out = *dkw;
    finish_partials(parts, grid, D, 2 * D, D, out);
  }
}

// tiles128 (optional int32 CUDA [1]): only the first 128 * tiles128[0] rows are live
void swiglu_bwd(const at::Tensor& dh, const at::Tensor& gu, at::Tensor& dgu, const c10::optional<at::Tensor>& tiles128) {
  CHECK_BF16(dh); CHECK_BF16(gu); CHECK_BF16(dgu);
  const int* tiles = nullptr;
  if (tiles128.has_value() && tiles128->defined()) {
    TORCH_CHECK(tiles128->is_cuda() && tiles128->scalar_type() == at::kInt && tiles128->numel() >= 1,
                "swiglu_bwd: tiles128 int32 CUDA [1]");
    tiles = tiles128->data_ptr<int>();
  }
  const c10::cuda::CUDAGuard g(dh.device());
  pb::swiglu_bwd(dh.data_ptr(), dh.stride(0), gu.data_ptr(), gu.stride(0), dgu.data_ptr(), dgu.stride(0),
                 dh.size(0), dh.size(1), cur_stream(), tiles);
}

void embedding_fwd(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out, int64_t v0) {
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous(), "ids must be contiguous int64");
  CHECK_BF16(table); CHECK_BF16(out);
  const c10::cuda::CUDAGuard g(table.device());
  pb::embedding_fwd(ids.data_ptr<int64_t>(), table.data_ptr(), table.stride(0), out.data_ptr(), out.stride(0),
                    ids.numel(), table.size(1), v0, table.size(0), cur_stream());
}

// sorted_ids / perm: torch.sort(ids, stable=True); grad bf16 [vocab rows, H]
void embedding_bwd(const at::Tensor& sorted_ids, const at::Tensor& perm, const at::Tensor& dy, at::Tensor& grad,
                   int64_t v0, bool accumulate) {
  TORCH_CHECK(sorted_ids.scalar_type() == at::kLong && sorted_ids.is_contiguous() &&
              perm.scalar_type() == at::kLong && perm.is_contiguous() && perm.numel() == sorted_ids.numel(),
              "embedding_bwd: sorted ids and permutation must be contiguous int64 of one length");
  CHECK_BF16(dy); CHECK_BF16(grad);
  TORCH_CHECK(dy.size(0) == sorted_ids.numel() && dy.size(1) == grad.size(1), "embedding_bwd: shapes");
  const c10::cuda::CUDAGuard g(dy.device());
  pb::embedding_bwd(sorted_ids.data_ptr<int64_t>(), perm.data_ptr<int64_t>(), dy.data_ptr(), dy.stride(0),
                    grad.data_ptr(), grad.stride(0), sorted_ids.numel(), dy.size(1), v0, grad.size(0), accumulate,
                    cur_stream());
}

void scale_by_scalar(at::Tensor& x, const at::Tensor& s) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "scale_by_scalar: bf16 x");
  TORCH_CHECK(s.is_cuda() && s.scalar_type() == at::kFloat && s.numel() == 1, "scale_by_scalar: fp32 scalar");
  const c10::cuda::CUDAGuard g(x.device());
  pb::scale_by_scalar(x.data_ptr(), x.numel(), s.data_ptr<float>(), cur_stream());
}

// ---------------------------------------------------------------- MoE router
void router_fwd(const at::Tensor& logits, int64_t top_k, bool renorm, at::Tensor& probs, at::Tensor& topv,
                at::Tensor& topi, const c10::optional<at::Tensor>& counts) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kBFloat16 && logits.dim() == 2 &&
              logits.stride(1) == 1, "router_fwd: bf16 [T, E] logits with unit inner stride");
  const int64_t T = logits.size(0), E = logits.size(1);
  CHECK_F32(probs); CHECK_F32(topv);
  TORCH_CHECK(probs.numel() == T * E && topv.numel() == T * top_k, "router_fwd: output sizes");
  TORCH_CHECK(topi.scalar_type() == at::kLong && topi.is_contiguous() && topi.numel() == T * top_k,
              "router_fwd: int64 [T, k] indices");
  int* cnt = nullptr;
  if (counts.has_value() && counts->defined()) {
    TORCH_CHECK(counts->scalar_type() == at::kInt && counts->numel() == E, "router_fwd: int32 [E] counts");
    cnt = counts->data_ptr<int>();
  }
  const c10::cuda::CUDAGuard g(logits.device());
  pb::router_fwd(logits.data_ptr(), logits.stride(0), (int)T, (int)E, (int)top_k, renorm, probs.data_ptr<float>(),
                 topv.data_ptr<float>(), topi.data_ptr<int64_t>(), cnt, cur_stream());
}

void router_bwd(const at::Tensor& probs, const c10::optional<at::Tensor>& dprobs, const at::Tensor& dtopv,
                const at::Tensor& topi, bool renorm, at::Tensor& dlogits) {
  CHECK_F32(probs); CHECK_F32(dtopv); CHECK_BF16(dlogits);
  TORCH_CHECK(probs.dim() == 2 && topi.dim() == 2 && topi.scalar_type() == at::kLong && topi.is_contiguous(),
              "router_bwd: probs [T, E], topi int64 [T, k]");
  const int64_t T = probs.size(0), E = probs.size(1), K = topi.size(1);
  const float* dp = opt_f32(dprobs);
  if (dp) TORCH_CHECK(dprobs->numel() == T * E, "router_bwd: dprobs size");
  TORCH_CHECK(dtopv.numel() == T * K && dlogits.size(0) == T && dlogits.size(1) == E, "router_bwd: sizes");
  const c10::cuda::CUDAGuard g(probs.device());
  pb::router_bwd(probs.data_ptr<float>(), dp, dtopv.data_ptr<float>(), topi.data_ptr<int64_t>(), (int)T, (int)E,
                 (int)K, renorm, dlogits.data_ptr(), dlogits.stride(0), cur_stream());
}

void aux_stats(const at::Tensor& probs, int64_t top_k, at::Tensor& counts, at::Tensor& ssum) {
  CHECK_F32(probs); CHECK_F32(counts); CHECK_F32(ssum);
  TORCH_CHECK(probs.dim() == 2 && counts.numel() == probs.size(1) && ssum.numel() == probs.size(1),
              "aux_stats: probs [R, E], counts / sums [E]");
  const c10::cuda::CUDAGuard g(probs.device());
  // counts / ssum are overwritten: block partials, then sums in block order
  const int E = (int)probs.size(1);
  const int grid = pb::aux_stats_grid((int)probs.size(0));
  at::Tensor parts = at::empty({grid, 2 * E}, probs.options());
  if (probs.size(0) == 0) {
    parts.zero_();
  } else {
    pb::aux_stats(probs.data_ptr<float>(), (int)probs.size(0), E, (int)top_k, parts.data_ptr<float>(), cur_stream());
  }
  finish_partials(parts, grid, E, 2 * E, 0, counts);
  finish_partials(parts, grid, E, 2 * E, E, ssum);
}

void aux_stats_bwd(const at::Tensor& probs, const at::Tensor& gsum, at::Tensor& dprobs) {
  CHECK_F32(probs); CHECK_F32(gsum); CHECK_F32(dprobs);
  TORCH_CHECK(probs.dim() == 2 && gsum.numel() == probs.size(1) && dprobs.numel() == probs.numel(),
              "aux_stats_bwd: sizes");
  const c10::cuda::CUDAGuard g(probs.device());
  pb::aux_stats_bwd(probs.data_ptr<float>(), gsum.data_ptr<float>(), (int)probs.size(0), (int)probs.size(1),
                    dprobs.data_ptr<float>(), cur_stream());
}

void ce_fwd_bwd(at::Tensor& logits, const at::Tensor& labels, int64_t v0, const c10::optional<at::Tensor>& scale,
                const c10::optional<at::Tensor>& row_lse, bool lse_given, const c10::optional<at::Tensor>& row_target,
                bool write_grad) {
  CHECK_BF16(logits);
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous(), "labels must be contiguous int64");
  TORCH_CHECK(labels.numel() == logits.size(0), "ce: one label per row");
  const c10::cuda::CUDAGuard g(logits.device());
  pb::ce_fwd_bwd(logits.data_ptr(), logits.stride(0), labels.data_ptr<int64_t>(), logits.size(0), logits.size(1),
                 v0, opt_f32(scale), opt_f32(row_lse), lse_given, opt_f32(row_target), write_grad, cur_stream());
}

// ce_valid_inv(labels int64 [T], inv fp32 [1]): inv = 1 / max(1, #valid labels)
void ce_valid_inv(const at::Tensor& labels, at::Tensor& inv) {
  TORCH_CHECK(labels.is_cuda() && labels.scalar_type() == at::kLong && labels.is_contiguous(), "labels: int64 CUDA");
  CHECK_F32(inv);
  const c10::cuda::CUDAGuard g(labels.device());
  pb::ce_valid_inv(labels.data_ptr<int64_t>(), (int)labels.numel(), inv.data_ptr<float>(), cur_stream());
}

// ce_loss_reduce(lse, tgt fp32 [T], labels int64 [T], inv fp32 [1], out fp32 [1], accumulate)
void ce_loss_reduce(const at::Tensor& lse, const at::Tensor& tgt, const at::Tensor& labels, const at::Tensor& inv,
                    at::Tensor& out, bool accumulate) {
  CHECK_F32(lse); CHECK_F32(tgt); CHECK_F32(inv); CHECK_F32(out);
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous(), "labels: int64");
  TORCH_CHECK(lse.numel() == labels.numel() && tgt.numel() == labels.numel(), "ce_loss_reduce: one value per row");
  const c10::cuda::CUDAGuard g(lse.device());
  pb::ce_loss_reduce(lse.data_ptr<float>(), tgt.data_ptr<float>(), labels.data_ptr<int64_t>(), (int)labels.numel(),
                     inv.data_ptr<float>(), out.data_ptr<float>(), accumulate, cur_stream());
}

void ce_row_stats(const at::Tensor& logits, at::Tensor& row_max, at::Tensor& row_sumexp) {
  CHECK_BF16(logits); CHECK_F32(row_max); CHECK_F32(row_sumexp);
  const c10::cuda::CUDAGuard g(logits.device());
  pb::ce_row_stats(logits.data_ptr(), logits.stride(0), logits.size(0), logits.size(1), row_max.data_ptr<float>(),
                   row_sumexp.data_ptr<float>(), cur_stream());
}

// sum_slices(parts fp32 [slices, len] (contiguous), out bf16 / fp32 [len], accumulate):
// out = (accumulate ? out : 0) + sum over slices, in slice order
void sum_slices(const at::Tensor& parts, at::Tensor& out, bool accumulate) {
  CHECK_F32(parts);
  TORCH_CHECK(parts.is_contiguous() && parts.dim() >= 2, "sum_slices: parts [slices, ...] contiguous fp32");
  const int64_t len = parts.numel() / parts.size(0);
  TORCH_CHECK(out.is_cuda() && out.is_contiguous() && out.numel() == len &&
                  (out.scalar_type() == at::kBFloat16 || out.scalar_type() == at::kFloat),
              "sum_slices: out");
  const c10::cuda::CUDAGuard g(parts.device());
  pb::sum_slices(parts.data_ptr<float>(), (int)parts.size(0), len, len, out.data_ptr(),
                 out.scalar_type() == at::kBFloat16, accumulate, cur_stream());
}

void cast_f32_to_bf16(const at::Tensor& src, at::Tensor& dst) {
  CHECK_F32(src);
  TORCH_CHECK(dst.is_contiguous() && dst.scalar_type() == at::kBFloat16 && dst.numel() == src.numel(), "cast: dst");
  const c10::cuda::CUDAGuard g(src.device());
  pb::cast_f32_to_bf16(src.data_ptr<float>(), dst.data_ptr(), src.numel(), cur_stream());
}

// params/grads/exp_avgs/exp_avg_sqs: lists of equally sized tensors (1 segment each)
void adamw(const std::vector<at::Tensor>& params, const std::vector<at::Tensor>& grads,
           const std::vector<at::Tensor>& exp_avgs, const std::vector<at::Tensor>& exp_avg_sqs, double lr,
           double beta1, double beta2, double eps, double wd, int64_t step,
           const c10::optional<at::Tensor>& grad_scale, const c10::optional<at::Tensor>& skip,
           const c10::optional<at::Tensor>& hyper) {
  TORCH_CHECK(params.size() == grads.size() && params.size() == exp_avgs.size() &&
              params.size() == exp_avg_sqs.size(), "adamw: list sizes differ");
  if (params.empty()) return;
  const bool grad_f32 = grads[0].scalar_type() == at::kFloat;
  const bool state_f32 = exp_avgs[0].scalar_type() == at::kFloat;
  std::vector<pb::AdamSeg> segs;
  segs.reserve(params.size());
  for (size_t i = 0; i < params.size(); ++i) {
    TORCH_CHECK(params[i].is_contiguous() && grads[i].is_contiguous() && exp_avgs[i].is_contiguous() &&
                exp_avg_sqs[i].is_contiguous(), "adamw: tensors must be contiguous");
    TORCH_CHECK(params[i].scalar_type() == at::kBFloat16, "adamw: bf16 params");
    TORCH_CHECK((grads[i].scalar_type() == at::kFloat) == grad_f32, "adamw: mixed grad dtypes");
    TORCH_CHECK((exp_avgs[i].scalar_type() == at::kFloat) == state_f32, "adamw: mixed state dtypes");
    TORCH_CHECK(grads[i].numel() == params[i].numel() && exp_avgs[i].numel() == params[i].numel(),
                "adamw: numel mismatch");
    segs.push_back({params[i].data_ptr(), grads[i].data_ptr(), exp_avgs[i].data_ptr(), exp_avg_sqs[i].data_ptr(),
                    params[i].numel()});
  }
  const c10::cuda::CUDAGuard g(params[0].device());
  const int* skip_ptr = nullptr;
  if (skip.has_value() && skip->defined()) {
    TORCH_CHECK(skip->scalar_type() == at::kInt, "adamw: skip must be int32");
    skip_ptr = skip->data_ptr<int>();
  }
  pb::adamw_multi(segs.data(), (int)segs.size(), (float)lr, (float)beta1, (float)beta2, (float)eps, (float)wd,
                  (int)step, opt_f32(grad_scale), skip_ptr, opt_f32(hyper), grad_f32, state_f32, cur_stream());
}

// out / flag are overwritten (accumulate = false) or added to (accumulate = true)
void sumsq(const std::vector<at::Tensor>& grads, const std::vector<double>& weights, at::Tensor& out,
           const c10::optional<at::Tensor>& flag, bool accumulate) {
  CHECK_F32(out);
  if (grads.empty()) {
    if (!accumulate) {
      out.zero_();
      if (flag.has_value() && flag->defined()) flag->zero_();
    }
    return;
  }
  const bool f32 = grads[0].scalar_type() == at::kFloat;
  std::vector<pb::NormSeg> segs;
  for (size_t i = 0; i < grads.size(); ++i) {
    TORCH_CHECK(grads[i].is_contiguous(), "sumsq: contiguous grads");
    TORCH_CHECK((grads[i].scalar_type() == at::kFloat) == f32, "sumsq: mixed dtypes");
    segs.push_back({grads[i].data_ptr(), grads[i].numel(), (float)(weights.empty() ? 1.0 : weights[i])});
  }
  int* flag_ptr = nullptr;
  if (flag.has_value() && flag->defined()) flag_ptr = flag->data_ptr<int>();
  const c10::cuda::CUDAGuard g(out.device());
  at::Tensor parts = at::empty({2 * std::max<int64_t>(1, pb::sumsq_chunks(segs.data(), (int)segs.size()))},
                               out.options());
  pb::sumsq_multi(segs.data(), (int)segs.size(), f32, parts.data_ptr<float>(), out.data_ptr<float>(), flag_ptr,
                  accumulate, cur_stream());
}

void clip_coef(const at::Tensor& total, double max_norm, at::Tensor& out) {
  CHECK_F32(total); CHECK_F32(out);
  const c10::cuda::CUDAGuard g(total.device());
  pb::clip_coef(total.data_ptr<float>(), (float)max_norm, out.data_ptr<float>(), cur_stream());
}

void attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
              int64_t B, int64_t S, int64_t nq, int64_t nkv, double scale, bool causal,
              const c10::optional<at::Tensor>& trace) {
  CHECK_BF16(q); CHECK_BF16(k); CHECK_BF16(v); CHECK_BF16(o); CHECK_F32(lse);
  TORCH_CHECK(q.size(0) == B * S && k.size(0) == B * S && v.size(0) == B * S, "attn: token count");
  TORCH_CHECK(lse.numel() >= B * nq * S, "attn: lse too small");
  const c10::cuda::CUDAGuard g(q.device());
  pb::AttnParams p{q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr<float>(),
                   q.stride(0), k.stride(0), v.stride(0), o.stride(0), (int)B, (int)S, (int)nq, (int)nkv,
                   (int)(q.size(1) / nq), (float)scale, causal};
  if (trace.has_value() && trace->defined()) {
    TORCH_CHECK(trace->scalar_type() == at::kLong && trace->is_cuda(), "trace must be a CUDA int64 tensor");
    p.trace = reinterpret_cast<long long*>(trace->data_ptr<int64_t>());
  }
  pb::attention_fwd(p, cur_stream());
}

void attn_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
              const at::Tensor& dout, const at::Tensor& lse, at::Tensor& delta, at::Tensor& dq_acc, at::Tensor& dq,
              at::Tensor& dk, at::Tensor& dv, int64_t B, int64_t S, int64_t nq, int64_t nkv, double scale,
              bool causal, const c10::optional<at::Tensor>& trace, const c10::optional<at::Tensor>& ds_buf) {
  CHECK_BF16(q); CHECK_BF16(k); CHECK_BF16(v); CHECK_BF16(o); CHECK_BF16(dout); CHECK_BF16(dq); CHECK_BF16(dk);
  CHECK_BF16(dv); CHECK_F32(lse); CHECK_F32(delta); CHECK_F32(dq_acc);
  const int64_t D = q.size(1) / nq;
  // delta is the kernel's scratch: delta*scale and lse*log2(e), each padded by 128 entries
  TORCH_CHECK(lse.numel() >= B * nq * S, "attn bwd: lse too small");
  TORCH_CHECK(delta.numel() >= 2 * (B * nq * S + 128), "attn bwd: delta scratch needs 2 * (B*nq*S + 128) floats");
  TORCH_CHECK(delta.is_contiguous() && dq_acc.is_contiguous(), "attn bwd: scratch must be contiguous");
  const bool use_ds = ds_buf.has_value() && ds_buf->defined();
  TORCH_CHECK(use_ds || dq_acc.numel() >= B * S * nq * D, "attn bwd: dq_acc too small");
  const c10::cuda::CUDAGuard g(q.device());
  pb::AttnBwdParams p{};
  p.q = q.data_ptr(); p.k = k.data_ptr(); p.v = v.data_ptr(); p.o = o.data_ptr(); p.dout = dout.data_ptr();
  p.lse = lse.data_ptr<float>(); p.delta = delta.data_ptr<float>(); p.dq_acc = dq_acc.data_ptr<float>();
  p.dq = dq.data_ptr(); p.dk = dk.data_ptr(); p.dv = dv.data_ptr();
  p.ldq = q.stride(0); p.ldk = k.stride(0); p.ldv = v.stride(0); p.ldo = o.stride(0); p.lddo = dout.stride(0);
  p.lddq = dq.stride(0); p.lddk = dk.stride(0); p.lddv = dv.stride(0);
  p.B = (int)B; p.S = (int)S; p.nq = (int)nq; p.nkv = (int)nkv; p.D = (int)D; p.scale = (float)scale;
  p.causal = causal;
  if (trace.has_value() && trace->defined()) {
    TORCH_CHECK(trace->scalar_type() == at::kLong && trace->is_cuda(), "trace must be a CUDA int64 tensor");
    TORCH_CHECK(trace->numel() >= B * nkv * ((S + 127) / 128) * pb::kAttnBwdTraceSlots,
                "trace needs kAttnBwdTraceSlots int64 entries per CTA");
    p.trace = reinterpret_cast<long long*>(trace->data_ptr<int64_t>());
  }
  if (use_ds) {
    CHECK_BF16(*ds_buf);
    TORCH_CHECK(ds_buf->is_contiguous() && ds_buf->numel() >= pb::attention_bwd_ds_elems((int)B, (int)S, (int)nq, causal),
                "attn bwd: ds_buf too small (attn_bwd_ds_elems)");
    p.ds_buf = ds_buf->data_ptr();
  }
  pb::attention_bwd(p, cur_stream());
}

int64_t attn_bwd_ds_elems(int64_t B, int64_t S, int64_t nq, bool causal) {
  return pb::attention_bwd_ds_elems((int)B, (int)S, (int)nq, causal);
}

}  // namespace

void register_ops(pybind11::module& m) {
  namespace py = pybind11;
  m.def("rmsnorm_fwd", &rmsnorm_fwd, py::arg("x"), py::arg("w"), py::arg("y"), py::arg("rstd"), py::arg("eps"));
  m.def("rmsnorm_bwd", &rmsnorm_bwd, py::arg("dy"), py::arg("x"), py::arg("w"), py::arg("rstd"), py::arg("dx"),
        py::arg("dw"), py::arg("dres") = py::none());
  m.def("qknorm_rope_fwd", &qknorm_rope_fwd);
  m.def("qknorm_rope_bwd", &qknorm_rope_bwd);
  m.def("swiglu_bwd", &swiglu_bwd, pybind11::arg("dh"), pybind11::arg("gu"), pybind11::arg("dgu"),
        pybind11::arg("tiles128") = pybind11::none());
  m.def("embedding_fwd", &embedding_fwd);
  m.def("embedding_bwd", &embedding_bwd);
  m.def("scale_by_scalar", &scale_by_scalar);
  m.def("router_fwd", &router_fwd);
  m.def("router_bwd", &router_bwd);
  m.def("aux_stats", &aux_stats);
  m.def("aux_stats_bwd", &aux_stats_bwd);
  m.def("ce_fwd_bwd", &ce_fwd_bwd);
  m.def("ce_row_stats", &ce_row_stats);
  m.def("ce_valid_inv", &ce_valid_inv);
  m.def("ce_loss_reduce", &ce_loss_reduce);
  m.def("cast_f32_to_bf16", &cast_f32_to_bf16);
  m.def("sum_slices", &sum_slices);
  m.def("adamw", &adamw, py::arg("params"), py::arg("grads"), py::arg("exp_avgs"), py::arg("exp_avg_sqs"),
        py::arg("lr"), py::arg("beta1"), py::arg("beta2"), py::arg("eps"), py::arg("wd"), py::arg("step"),
        py::arg("grad_scale") = py::none(), py::arg("skip") = py::none(), py::arg("hyper") = py::none());
  m.def("sumsq", &sumsq, py::arg("grads"), py::arg("weights"), py::arg("out"), py::arg("flag") = py::none(),
        py::arg("accumulate") = true);
  m.def("clip_coef", &clip_coef);
  m.def("attn_fwd", &attn_fwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("lse"), py::arg("B"),
        py::arg("S"), py::arg("nq"), py::arg("nkv"), py::arg("scale"), py::arg("causal"),
        py::arg("trace") = py::none());
  m.def("attn_bwd", &attn_bwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("dout"),
        py::arg("lse"), py::arg("delta"), py::arg("dq_acc"), py::arg("dq"), py::arg("dk"), py::arg("dv"), py::arg("B"),
        py::arg("S"), py::arg("nq"), py::arg("nkv"), py::arg("scale"), py::arg("causal"),
        py::arg("trace") = py::none(), py::arg("ds_buf") = py::none());
  m.def("attn_bwd_ds_elems", &attn_bwd_ds_elems);
}
