// Host launchers of the non-GEMM kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace b200 {

int num_sms_cached();

void rmsnorm_fwd(const __nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* y, float* rstd, int rows, int d,
                 float eps, cudaStream_t s);
void rmsnorm_bwd(const __nv_bfloat16* dy, const __nv_bfloat16* x, const __nv_bfloat16* w, const float* rstd,
                 const __nv_bfloat16* dres, __nv_bfloat16* dx, float* dw, int rows, int d, cudaStream_t s);
void embedding_fwd(const int64_t* ids, const __nv_bfloat16* table, __nv_bfloat16* out, int rows, int d, int vocab,
                   cudaStream_t s);
void embedding_bwd(const int64_t* ids, const __nv_bfloat16* dy, float* dtable, int rows, int d, int vocab,
                   cudaStream_t s);
void rope_bwd(__nv_bfloat16* g, int rows, int ld, int rope_cols, int head_dim, int seq_len, const float* cosv,
              const float* sinv, cudaStream_t s);

// `dev_sc` (nullable): device scalars {lr / (1 - beta1^t), 1 / sqrt(1 - beta2^t)} written by adam_advance;
// when given they replace the host-computed bias corrections of `step` (replayable CUDA graphs).
void adamw_step(float* master, float* m, float* v, const float* g, void* param_out, bool param_bf16, size_t n,
                const float* scale_ptr, float scale_const, float lr, float beta1, float beta2, float eps, float wd,
                int step, cudaStream_t s, const float* dev_sc = nullptr);
// step_count[0] += 1 on the device, then dev_sc = {lr / (1 - beta1^t), 1 / sqrt(1 - beta2^t)} for the new t.
void adam_advance(int* step_count, float* dev_sc, float lr, float beta1, float beta2, cudaStream_t s);
void sum_squares(const void* x, bool is_bf16, size_t n, float* out, cudaStream_t s);
// Error record gets `code` if the device scalars *a and *b differ (no host synchronisation).
void record_if_different(const float* a, const float* b, int code, cudaStream_t s);
void cross_entropy_fwd(const __nv_bfloat16* logits, int ld, const int64_t* targets, int rows, int vocab, float* lse,
                       float* loss_sum, float* count, float* loss, cudaStream_t s);
void cross_entropy_bwd(__nv_bfloat16* logits, int ld, const int64_t* targets, int rows, int vocab, const float* lse,
                       const float* grad_loss, const float* count, cudaStream_t s);

// Flash attention (causal, GQA) on tcgen05.  q/k/v are column blocks of one [B*S, ld] matrix.
struct AttnParams {
  const __nv_bfloat16* qkv;  // [B*S, ld]; q at column 0, k at k_col, v at v_col
  int ld;
  int k_col, v_col;
  __nv_bfloat16* out;  // [B*S, H*hd]
  int ld_out;
  float* lse;          // [B, H, S] (natural-log units)
  int batch, seq, heads, kv_heads, head_dim;
  float scale;
  unsigned long long* trace = nullptr;  // debug: per-role phase clocks of CTA 0 (ZB_ATTN_TRACE=1), else null
};
void attention_fwd(const AttnParams& p, cudaStream_t s);
// Debug (ZB_ATTN_TRACE=1): phase clocks of CTA 0 of the last forward launch, kAttnTraceWords 64-bit words
// per role (role 0: MMA thread, 1: first softmax thread of tile A, 2: of tile B), as (event, clock64) pairs.
constexpr int kAttnTraceWords = 2048;
void attention_trace_read(unsigned long long* host_out);

struct AttnBwdParams {
  const __nv_bfloat16* qkv;
  int ld, k_col, v_col;
  const __nv_bfloat16* out;   // forward output O [B*S, H*hd]
  const __nv_bfloat16* dout;  // dO
  int ld_out;
  const float* lse;           // [B, H, S]
  float* delta;               // [B, H, S] scratch: rowsum(dO * O)
  float* dq_acc;              // [B*S, H*hd] fp32 scratch, all zero on entry
  bool rezero_dq_acc;         // leave dq_acc zeroed on exit (the caller keeps one zeroed buffer)
  __nv_bfloat16* dqkv;        // [B*S, ld] gradient of the fused qkv matrix (pre-RoPE q and k)
  const float* rope_cos;      // [seq, head_dim/2]: RoPE backward is applied to dq and dk
  const float* rope_sin;
  int batch, seq, heads, kv_heads, head_dim;
  float scale;
};
void attention_bwd(const AttnBwdParams& p, cudaStream_t s);

}  // namespace b200
