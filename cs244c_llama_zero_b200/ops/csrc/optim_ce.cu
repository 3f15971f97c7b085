// Optimizer and loss kernels.
//
// * adamw_step: one pass over flat fp32 state (reads g, m, v, master; writes m, v, master and the
//   model-dtype parameter).  The gradient scale (1/W times the clip coefficient) is read from
//   device memory so clipping never needs a host round trip.
// * sum_squares: fp32 sum of squares of a flat vector (grad-norm), block partials + atomics.
// * cross_entropy_fwd: per-row log-sum-exp over bf16 logits, loss summed over valid targets.
// * cross_entropy_bwd: dlogits = (softmax - onehot) * g / count, written in place over the logits.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>

#include "common.cuh"
#include "kernels.h"

namespace b200 {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

struct AdamArgs {
  float lr, beta1, beta2, eps, wd;
  float one_minus_b1, one_minus_b2;
  float step_size, inv_sqrt_bc2;  // lr / (1 - beta1^t) and 1 / sqrt(1 - beta2^t)
};

template <bool BF16_OUT>
__global__ void adamw_kernel(float* __restrict__ master, float* __restrict__ m, float* __restrict__ v,
                             const float* __restrict__ g, void* __restrict__ param_out, size_t n,
                             const float* __restrict__ scale_ptr, float scale_const, AdamArgs a,
                             const float* __restrict__ dev_sc) {
  pdl_wait_and_release();
  const float scale = (scale_ptr != nullptr ? *scale_ptr : 1.0f) * scale_const;
  const float decay = 1.0f - a.lr * a.wd;
  const float step = dev_sc != nullptr ? dev_sc[0] : a.step_size;
  if (dev_sc != nullptr) a.inv_sqrt_bc2 = dev_sc[1];
  const size_t n4 = n / 4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    float4 gp = reinterpret_cast<const float4*>(g)[i];
    float4 mp = reinterpret_cast<float4*>(m)[i];
    float4 vp = reinterpret_cast<float4*>(v)[i];
    float4 pp = reinterpret_cast<float4*>(master)[i];
    float gg[4] = {gp.x * scale, gp.y * scale, gp.z * scale, gp.w * scale};
    float mm[4] = {mp.x, mp.y, mp.z, mp.w};
    float vv[4] = {vp.x, vp.y, vp.z, vp.w};
    float pw[4] = {pp.x, pp.y, pp.z, pp.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      mm[e] = a.beta1 * mm[e] + a.one_minus_b1 * gg[e];
      vv[e] = a.beta2 * vv[e] + a.one_minus_b2 * gg[e] * gg[e];
      pw[e] *= decay;
      const float denom = sqrtf(vv[e]) * a.inv_sqrt_bc2 + a.eps;
      pw[e] -= step * mm[e] / denom;
    }
    reinterpret_cast<float4*>(m)[i] = make_float4(mm[0], mm[1], mm[2], mm[3]);
    reinterpret_cast<float4*>(v)[i] = make_float4(vv[0], vv[1], vv[2], vv[3]);
    reinterpret_cast<float4*>(master)[i] = make_float4(pw[0], pw[1], pw[2], pw[3]);
    if (param_out != nullptr) {
      if constexpr (BF16_OUT) {
        uint2 o;
        o.x = pack_bf16(pw[0], pw[1]);
        o.y = pack_bf16(pw[2], pw[3]);
        reinterpret_cast<uint2*>(param_out)[i] = o;
      } else {
        reinterpret_cast<float4*>(param_out)[i] = make_float4(pw[0], pw[1], pw[2], pw[3]);
      }
    }
  }
  // Tail (n not a multiple of 4).
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    const size_t i = n4 * 4 + threadIdx.x;
    const float gg = g[i] * scale;
    float mm = a.beta1 * m[i] + a.one_minus_b1 * gg;
    float vv = a.beta2 * v[i] + a.one_minus_b2 * gg * gg;
    float pw = master[i] * decay - step * mm / (sqrtf(vv) * a.inv_sqrt_bc2 + a.eps);
    m[i] = mm;
    v[i] = vv;
    master[i] = pw;
    if (param_out != nullptr) {
      if constexpr (BF16_OUT)
        reinterpret_cast<__nv_bfloat16*>(param_out)[i] = __float2bfloat16_rn(pw);
      else
        reinterpret_cast<float*>(param_out)[i] = pw;
    }
  }
}

__device__ __forceinline__ float to_float(float v) { return v; }
__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__global__ void sum_squares_kernel(const T* __restrict__ x, size_t n, float* __restrict__ out) {
  pdl_wait_and_release();
  float acc = 0.f;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float v = to_float(x[i]);
    acc += v * v;
  }
  acc = warp_sum(acc);
  __shared__ float part[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) part[warp] = acc;
  __syncthreads();
  if (warp == 0) {
    acc = lane < (int)(blockDim.x >> 5) ? part[lane] : 0.f;
    acc = warp_sum(acc);
    if (lane == 0) atomicAdd(out, acc);
  }
}

__global__ void sum_squares_f4_kernel(const float4* __restrict__ x, size_t n4, float* __restrict__ out) {
  pdl_wait_and_release();
  float acc = 0.f;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const float4 v = x[i];
    acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  acc = warp_sum(acc);
  __shared__ float part[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) part[warp] = acc;
  __syncthreads();
  if (warp == 0) {
    acc = lane < (int)(blockDim.x >> 5) ? part[lane] : 0.f;
    acc = warp_sum(acc);
    if (lane == 0) atomicAdd(out, acc);
  }
}

// One CTA (256 threads) per row.  Online max/sum per thread, then block reduction.
__global__ void ce_fwd_kernel(const __nv_bfloat16* __restrict__ logits, int ld, const int64_t* __restrict__ targets,
                              int rows, int vocab, float* __restrict__ lse_out, float* __restrict__ loss_sum,
                              float* __restrict__ count) {
  pdl_wait_and_release();
  const int row = blockIdx.x;
  if (row >= rows) return;
  const int64_t tgt = targets[row];
  const __nv_bfloat16* lr = logits + (size_t)row * ld;
  float mx = -INFINITY, sm = 0.f;
  const int n8 = vocab / 8;
  for (int i = threadIdx.x; i < n8; i += blockDim.x) {
    const uint4 q = reinterpret_cast<const uint4*>(lr)[i];
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    float f[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      f[2 * e] = bf16lo(w[e]);
      f[2 * e + 1] = bf16hi(w[e]);
    }
    float lm = f[0];
#pragma unroll
    for (int e = 1; e < 8; ++e) lm = fmaxf(lm, f[e]);
    if (lm > mx) {
      sm *= __expf(mx - lm);
      mx = lm;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) sm += __expf(f[e] - mx);
  }
  for (int i = n8 * 8 + threadIdx.x; i < vocab; i += blockDim.x) {
    const float f = __bfloat162float(lr[i]);
    if (f > mx) {
      sm *= __expf(mx - f);
      mx = f;
    }
    sm += __expf(f - mx);
  }
  __shared__ float smx[32], ssm[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float wm = warp_max(mx);
  float ws = sm * (mx == -INFINITY ? 0.f : __expf(mx - wm));
  ws = warp_sum(ws);
  if (lane == 0) {
    smx[warp] = wm;
    ssm[warp] = ws;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    float m2 = lane < nw ? smx[lane] : -INFINITY;
    float s2 = lane < nw ? ssm[lane] : 0.f;
    const float gm = warp_max(m2);
    s2 = s2 * (m2 == -INFINITY ? 0.f : __expf(m2 - gm));
    s2 = warp_sum(s2);
    if (lane == 0) {
      const float lse = gm + logf(s2);
      lse_out[row] = lse;
      if (tgt >= 0 && tgt < vocab) {
        atomicAdd(loss_sum, lse - __bfloat162float(lr[tgt]));
        atomicAdd(count, 1.0f);
      }
    }
  }
}

__global__ void ce_bwd_kernel(__nv_bfloat16* __restrict__ logits, int ld, const int64_t* __restrict__ targets,
                              int rows, int vocab, const float* __restrict__ lse, const float* __restrict__ grad_loss,
                              const float* __restrict__ count) {
  pdl_wait_and_release();
  const int row = blockIdx.x;
  if (row >= rows) return;
  const int64_t tgt = targets[row];
  __nv_bfloat16* lr = logits + (size_t)row * ld;
  const bool valid = tgt >= 0 && tgt < vocab;
  const float scale = valid ? (*grad_loss) / fmaxf(*count, 1.0f) : 0.f;
  const float l = lse[row];
  const int n8 = vocab / 8;
  for (int i = threadIdx.x; i < n8; i += blockDim.x) {
    uint4 q = reinterpret_cast<uint4*>(lr)[i];
    uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int c = i * 8 + 2 * e;
      float a = __expf(bf16lo(w[e]) - l) - (c == tgt ? 1.f : 0.f);
      float b = __expf(bf16hi(w[e]) - l) - (c + 1 == tgt ? 1.f : 0.f);
      w[e] = pack_bf16(a * scale, b * scale);
    }
    reinterpret_cast<uint4*>(lr)[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  for (int i = n8 * 8 + threadIdx.x; i < vocab; i += blockDim.x) {
    const float a = __expf(__bfloat162float(lr[i]) - l) - (i == tgt ? 1.f : 0.f);
    lr[i] = __float2bfloat16_rn(a * scale);
  }
}

__global__ void finalize_loss_kernel(const float* loss_sum, const float* count, float* loss) {
  pdl_wait_and_release();
  *loss = *loss_sum / fmaxf(*count, 1.0f);
}

// Advances the device step counter and writes the bias-corrected scalars for it (one thread).
// The scalars are computed in double and rounded once to float, exactly as the host computes them
// for a host-side step number (adam_step_size / adam_inv_sqrt_bc2), so a captured step replays with
// the bits of the eager step.
__global__ void adam_advance_kernel(int* step_count, float* dev_sc, float lr, float beta1, float beta2) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const int t = step_count[0] + 1;
  step_count[0] = t;
  dev_sc[0] = (float)((double)lr / (1.0 - pow((double)beta1, (double)t)));
  dev_sc[1] = (float)(1.0 / sqrt(1.0 - pow((double)beta2, (double)t)));
}

}  // namespace

void adam_advance(int* step_count, float* dev_sc, float lr, float beta1, float beta2, cudaStream_t s) {
  adam_advance_kernel<<<1, 32, 0, s>>>(step_count, dev_sc, lr, beta1, beta2);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void adamw_step(float* master, float* m, float* v, const float* g, void* param_out, bool param_bf16, size_t n,
                const float* scale_ptr, float scale_const, float lr, float beta1, float beta2, float eps, float wd,
                int step, cudaStream_t s, const float* dev_sc) {
  B200_CHECK((reinterpret_cast<uintptr_t>(master) & 15) == 0 && (reinterpret_cast<uintptr_t>(m) & 15) == 0 &&
                 (reinterpret_cast<uintptr_t>(v) & 15) == 0 && (reinterpret_cast<uintptr_t>(g) & 15) == 0,
             "adamw: fp32 buffers must be 16-byte aligned");
  B200_CHECK(param_out == nullptr || (reinterpret_cast<uintptr_t>(param_out) & 7) == 0,
             "adamw: parameter output must be 8-byte aligned");
  AdamArgs a;
  a.lr = lr;
  a.beta1 = beta1;
  a.beta2 = beta2;
  a.eps = eps;
  a.wd = wd;
  a.one_minus_b1 = 1.0f - beta1;
  a.one_minus_b2 = 1.0f - beta2;
  a.step_size = (float)((double)lr / (1.0 - std::pow((double)beta1, (double)step)));
  a.inv_sqrt_bc2 = (float)(1.0 / std::sqrt(1.0 - std::pow((double)beta2, (double)step)));
  const int threads = 256;
  const size_t work = std::max<size_t>(1, n / 4);
  const int blocks = (int)std::min<size_t>((work + threads - 1) / threads, (size_t)num_sms_cached() * 8);
  if (param_bf16)
    launch_k(adamw_kernel<true>, dim3(blocks), dim3(threads), 0, s, 1, master, m, v, g, param_out, n, scale_ptr, scale_const, a,
             dev_sc);
  else
    launch_k(adamw_kernel<false>, dim3(blocks), dim3(threads), 0, s, 1, master, m, v, g, param_out, n, scale_ptr, scale_const, a,
             dev_sc);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void sum_squares(const void* x, bool is_bf16, size_t n, float* out, cudaStream_t s) {
  B200_CUDA_CHECK(cudaMemsetAsync(out, 0, sizeof(float), s));
  const int threads = 512;
  const int blocks = (int)std::max<size_t>(1, std::min<size_t>((n + threads - 1) / threads, (size_t)num_sms_cached() * 4));
  if (is_bf16) {
    launch_k(sum_squares_kernel<__nv_bfloat16>, dim3(blocks), dim3(threads), 0, s, 1, reinterpret_cast<const __nv_bfloat16*>(x), n, out);
  } else if ((reinterpret_cast<uintptr_t>(x) & 15) == 0 && n % 4 == 0) {
    launch_k(sum_squares_f4_kernel, dim3(blocks), dim3(threads), 0, s, 1, reinterpret_cast<const float4*>(x), n / 4, out);
  } else {
    launch_k(sum_squares_kernel<float>, dim3(blocks), dim3(threads), 0, s, 1, reinterpret_cast<const float*>(x), n, out);
  }
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void cross_entropy_fwd(const __nv_bfloat16* logits, int ld, const int64_t* targets, int rows, int vocab, float* lse,
                       float* loss_sum, float* count, float* loss, cudaStream_t s) {
  B200_CHECK(ld % 8 == 0, "cross_entropy: logits row stride must be a multiple of 8");
  B200_CUDA_CHECK(cudaMemsetAsync(loss_sum, 0, sizeof(float), s));
  B200_CUDA_CHECK(cudaMemsetAsync(count, 0, sizeof(float), s));
  launch_k(ce_fwd_kernel, dim3(rows), dim3(256), 0, s, 1, logits, ld, targets, rows, vocab, lse, loss_sum, count);
  B200_CUDA_CHECK(cudaGetLastError());
  launch_k(finalize_loss_kernel, dim3(1), dim3(1), 0, s, 1, loss_sum, count, loss);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch(2);
}

void cross_entropy_bwd(__nv_bfloat16* logits, int ld, const int64_t* targets, int rows, int vocab, const float* lse,
                       const float* grad_loss, const float* count, cudaStream_t s) {
  launch_k(ce_bwd_kernel, dim3(rows), dim3(256), 0, s, 1, logits, ld, targets, rows, vocab, lse, grad_loss, count);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

}  // namespace b200
