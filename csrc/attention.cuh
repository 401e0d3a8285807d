// Causal GQA flash attention on the sm_100a tensor cores (attention_fwd.cu,
// attention_bwd.cu).
//
// Layouts (token-major, exactly what the QKV GEMM / QK-norm kernels write):
//   q  : [B*S, nq*D]   row stride ldq,  head h at column h*D
//   k  : [B*S, nkv*D]  row stride ldk
//   v  : [B*S, nkv*D]  row stride ldv   (may be a column view of the qkv buffer)
//   o  : [B*S, nq*D]   row stride ldo
//   lse: [B*nq, S]     fp32 natural-log sum-exp of the scaled scores
// Query head h reads kv head h / (nq / nkv).  D == 128.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace pb {

struct AttnParams {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse;
  int64_t ldq, ldk, ldv, ldo;
  int B, S, nq, nkv, D;
  float scale;  // softmax scale (1/sqrt(D))
  bool causal;
  long long* trace = nullptr;  // optional per-CTA phase timing [grid * 16]
};

void attention_fwd(const AttnParams& p, cudaStream_t s);

struct AttnBwdParams {
  const void* q;
  const void* k;
  const void* v;
  const void* o;
  const void* dout;
  const float* lse;
  float* delta;   // scratch of 2 * (B*nq*S + 128) floats: delta*scale, lse*log2(e)
  float* dq_acc;  // [B*S, nq*D] fp32 scratch (zeroed by the launcher), 16-byte aligned
  void* dq;
  void* dk;
  void* dv;
  int64_t ldq, ldk, ldv, ldo, lddo, lddq, lddk, lddv;
  int B, S, nq, nkv, D;
  float scale;
  bool causal;
  long long* trace = nullptr;  // optional per-CTA phase timing [grid * kAttnBwdTraceSlots]
  // dS tile buffer (attention_bwd_ds_elems bf16 elements): when set, dQ is
  // computed from stored dS tiles by a second kernel (no fp32 accumulator)
  void* ds_buf = nullptr;
};

constexpr int kAttnBwdTraceSlots = 24;

void attention_bwd(const AttnBwdParams& p, cudaStream_t s);
int64_t attention_bwd_ds_elems(int B, int S, int nq, bool causal);

}  // namespace pb

// Allocation-free attention backward (attention_bwd.cu).  These C entry points
// have no counterpart in the reference; they serve callers that cannot
// allocate device memory (see the comment above their definitions).  Return
// codes of pb_attention_bwd_noalloc: 0 ok, 1 problem larger than the fixed
// scratch array, 2 invalid arguments, 3 CUDA error (message from
// pb_attention_bwd_noalloc_last_error, per calling thread).
extern "C" {
int pb_attention_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const void* dout,
                             const float* lse, void* dq, void* dk, void* dv, int64_t ldq, int64_t ldk, int64_t ldv,
                             int64_t ldo, int64_t lddo, int64_t lddq, int64_t lddk, int64_t lddv, int B, int S,
                             int nq, int nkv, int D, float scale, int causal, cudaStream_t stream);
// bytes of the fixed per-device scratch array
size_t pb_attention_bwd_noalloc_scratch_bytes(void);
// message of the calling thread's last failed call ("" after a success)
const char* pb_attention_bwd_noalloc_last_error(void);
// bounded-wait status word of the last call on the current device (0 = no
// wait gave up; -1 = no call yet or a CUDA error); synchronises the device
int pb_attention_bwd_noalloc_device_status(void);
}
