// Allocation-free entry point for the flash-attention backward pass.
//
// This entry point has no counterpart in the reference implementation; it is an addition of this
// library for callers that cannot allocate GPU memory themselves: code running inside a host
// process whose device memory is owned by another allocator (an inference server or framework
// that forbids stray cudaMalloc calls), code that runs where a cudaMalloc would synchronise the
// device at a bad moment, or plain C/C++ callers that hold only raw device pointers and have no
// allocator at all.  The regular path (the Python `attention_backward` wrapper) asks its caller to
// provide two scratch buffers (the per-row `delta` vector and an fp32 dQ accumulator); this entry
// point instead uses one scratch array compiled into the library:
//
//   * The scratch is a file-scope `static __device__` array of B200_ATTN_BWD_NOALLOC_SCRATCH_BYTES
//     (8 MiB).  Every GPU on which the library is loaded holds those 8 MiB until the process exits.
//   * A call needs  align256(16) + align256(4*B*H*S) + align256(4*B*S*H*hd)  bytes of it; larger
//     problems are rejected with B200_NOALLOC_ERR_TOO_LARGE (and a message on stderr) before any
//     work is queued.  Example: B*S = 4096 tokens with H*hd = 512 fits; the benchmark's 8192 x 768
//     does not (use the regular path there).
//   * The first call on each device looks up the array's device address (cudaGetSymbolAddress)
//     and sets the kernel's shared-memory attribute, with that device current.  Make that first
//     call before capturing a stream into a CUDA graph.  `stream` must belong to the current
//     device (the call checks, and rejects a stream of another device with ERR_INVALID).
//   * Errors inside the kernels (an expired bounded wait) do not change the return code, which
//     only covers argument checks and launches: read b200_attention_bwd_noalloc_last_error after
//     the call's work has finished to know whether `dqkv` is valid.
//   * The call allocates nothing: no cudaMalloc / cudaFree and no allocating library routine.  The
//     scratch is shared by every call on a device and keeps the previous call's contents; the
//     parts that must start at zero are cleared on the caller's stream at the start of each call.
//     Two calls whose work overlaps on the GPU (different streams without ordering) race on the
//     scratch and give wrong results; order them on one stream or with events.
//
// Arguments mirror the regular backward: `qkv` is the fused [B*S, ld] bf16 projection (q at column
// 0, k at k_col, v at v_col), `out` / `dout` the forward output and its gradient ([B*S, ld_out]),
// `lse` the forward's base-2 log-sum-exp [B, H, S], and `dqkv` ([B*S, ld], written) receives the
// gradient with respect to the pre-RoPE q|k|v columns; `rope_cos` / `rope_sin` are [S, hd/2] fp32.
// Column layout: heads*head_dim <= k_col, k_col + kv_heads*head_dim <= v_col,
// v_col + kv_heads*head_dim <= ld and heads*head_dim <= ld_out (checked).
// Returns 0 on success or one of the negative codes below.
#pragma once

#include <cuda_runtime.h>

#define B200_ATTN_BWD_NOALLOC_SCRATCH_BYTES (8u << 20)

#define B200_NOALLOC_OK 0
#define B200_NOALLOC_ERR_TOO_LARGE (-1)  // problem needs more scratch than the fixed array holds
#define B200_NOALLOC_ERR_INVALID (-2)    // unsupported shape or misaligned / null argument
#define B200_NOALLOC_ERR_CUDA (-3)       // a CUDA call failed (set-up or launch)

#ifdef __cplusplus
extern "C" {
#endif

int b200_attention_bwd_noalloc(const void* qkv, int ld, int k_col, int v_col, const void* out, const void* dout,
                               int ld_out, const float* lse, void* dqkv, const float* rope_cos,
                               const float* rope_sin, int batch, int seq, int heads, int kv_heads, int head_dim,
                               float scale, cudaStream_t stream);

// The kernels' error record of the last call on the current device, as four ints: code (0 = no
// error; 2 = a bounded wait inside the attention kernel expired, 7 = a range check of the
// debug-bounds build failed), where (the wait or check site), block (reporting block) and count.
// A non-zero code means that call's `dqkv` is not valid.  The record lives in the same fixed
// scratch array and is cleared by the next call, so read it after the call's work has finished
// (synchronise the call's stream first) and before the next call.  Copies 16 bytes with a
// synchronous cudaMemcpy (no allocation).  Returns 0 or B200_NOALLOC_ERR_INVALID / _CUDA.
int b200_attention_bwd_noalloc_last_error(int* record4);

#ifdef __cplusplus
}
#endif
