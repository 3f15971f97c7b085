// Memory-bound kernels of the transformer block: RMSNorm forward/backward (with the residual
// gradient fused into the backward), token-embedding gather/scatter, RoPE backward.
//
// All of them move 16-byte vectors (8 bf16) per thread access and keep statistics in fp32.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace b200 {

namespace {

constexpr int kWarpsPerBlock = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void unpack8(const uint4& q, float (&f)[8]) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = bf16lo(w[i]);
    f[2 * i + 1] = bf16hi(w[i]);
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 q;
  q.x = pack_bf16(f[0], f[1]);
  q.y = pack_bf16(f[2], f[3]);
  q.z = pack_bf16(f[4], f[5]);
  q.w = pack_bf16(f[6], f[7]);
  return q;
}

// One warp per row; each lane owns VEC groups of 8 columns (d = 256 * VEC).
template <int VEC>
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                   __nv_bfloat16* __restrict__ y, float* __restrict__ rstd, int rows, int d,
                                   float eps) {
  pdl_wait_and_release();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  const __nv_bfloat16* xr = x + (size_t)row * d;
  float v[VEC][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d) {
      unpack8(*reinterpret_cast<const uint4*>(xr + c), v[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[i][e] * v[i][e];
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)d + eps);
  if (lane == 0 && rstd != nullptr) rstd[row] = r;
  __nv_bfloat16* yr = y + (size_t)row * d;
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d) {
      float wf[8], o[8];
      unpack8(*reinterpret_cast<const uint4*>(w + c), wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[i][e] * r * wf[e];
      *reinterpret_cast<uint4*>(yr + c) = pack8(o);
    }
  }
}

// dx = dres + rstd * (dy*w - xhat * mean(dy*w*xhat)); dw += sum_rows(dy * xhat) (fp32 atomics).
//
// Each warp owns ROWS rows and issues the x, dy and dres loads of all of them before any arithmetic,
// so a warp keeps several 16-byte loads per lane in flight (the kernel is bound by HBM latency x
// bytes in flight, not by arithmetic).  ROWS = 2 up to d = 1024 and 1 above (register budget).  The
// block's weight-gradient partials are summed in shared memory and added with one fp32 atomic per
// column per block.
template <int VEC, int ROWS>
__global__ void __launch_bounds__(32 * kWarpsPerBlock)
    rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                       const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
                       const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ dx,
                       float* __restrict__ dw, int rows, int d) {
  pdl_wait_and_release();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int row0 = (blockIdx.x * kWarpsPerBlock + warp) * ROWS;
  uint4 xq[ROWS][VEC], gq[ROWS][VEC], rq[ROWS][VEC];
  float r[ROWS];
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
  for (int k = 0; k < ROWS; ++k) {
    const int row = row0 + k;
    const bool ok = row < rows;
    r[k] = ok ? rstd[row] : 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int c = (i * 32 + lane) * 8;
      const bool in = ok && c < d;
      const size_t off = (size_t)row * d + c;
      xq[k][i] = in ? *reinterpret_cast<const uint4*>(x + off) : zero;
      gq[k][i] = in ? *reinterpret_cast<const uint4*>(dy + off) : zero;
      rq[k][i] = (in && dres != nullptr) ? *reinterpret_cast<const uint4*>(dres + off) : zero;
    }
  }
  float acc[VEC][8];
#pragma unroll
  for (int i = 0; i < VEC; ++i)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[i][e] = 0.f;
#pragma unroll
  for (int k = 0; k < ROWS; ++k) {
    const int row = row0 + k;
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < d) {
        float xv[8], dyv[8], wf[8];
        unpack8(xq[k][i], xv);
        unpack8(gq[k][i], dyv);
        unpack8(*reinterpret_cast<const uint4*>(w + c), wf);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float xh = xv[e] * r[k];
          dot += dyv[e] * wf[e] * xh;
          acc[i][e] += dyv[e] * xh;
        }
      }
    }
    dot = warp_sum(dot) / (float)d;
    if (row >= rows) continue;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < d) {
        float xv[8], dyv[8], wf[8], rv[8], o[8];
        unpack8(xq[k][i], xv);
        unpack8(gq[k][i], dyv);
        unpack8(rq[k][i], rv);
        unpack8(*reinterpret_cast<const uint4*>(w + c), wf);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = rv[e] + r[k] * (dyv[e] * wf[e] - xv[e] * r[k] * dot);
        *reinterpret_cast<uint4*>(dx + (size_t)row * d + c) = pack8(o);
      }
    }
  }
  // Reduce the weight gradient across the warps of the block, then one atomic per column.
  __shared__ float red[kWarpsPerBlock][32 * 8];
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
#pragma unroll
    for (int e = 0; e < 8; ++e) red[warp][lane * 8 + e] = acc[i][e];
    __syncthreads();
    for (int t = threadIdx.x; t < 256; t += blockDim.x) {
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < kWarpsPerBlock; ++k) s += red[k][t];
      const int c = i * 256 + t;
      if (c < d) atomicAdd(dw + c, s);
    }
    __syncthreads();
  }
}

// Wide rows (d > 2048, e.g. the 7B model's 4096): the per-lane register tiles of the kernel above
// would not fit, so each warp takes rows in turn and reads each row twice - pass 1 for the row's
// dot product sum(dy * w * x_hat), pass 2 (L1 / L2 hits) to write dx and to add dy * x_hat into
// its own fp32 weight-gradient row in shared memory (lane l owns columns 256k + 8l .. + 7, so the
// updates need no atomics).  The block sums its warps' rows and adds them with one fp32 atomic per
// column.
constexpr int kWideWarps = 4;
constexpr int kWideMaxD = 12288;  // kWideWarps fp32 rows of d columns in 192 KB of shared memory
__global__ void __launch_bounds__(32 * kWideWarps)
    rmsnorm_bwd_wide_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                            const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
                            const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ dx,
                            float* __restrict__ dw, int rows, int d) {
  pdl_wait_and_release();
  extern __shared__ float4 dw_rows4[];  // [kWideWarps][d / 4]
  float* dw_rows = reinterpret_cast<float*>(dw_rows4);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  for (int c = threadIdx.x; c < kWideWarps * d; c += blockDim.x) dw_rows[c] = 0.f;
  __syncthreads();
  float* mine = dw_rows + (size_t)warp * d;
  for (int row = blockIdx.x * kWideWarps + warp; row < rows; row += gridDim.x * kWideWarps) {
    const float r = rstd[row];
    const size_t base = (size_t)row * d;
    float dot = 0.f;
    for (int c = lane * 8; c < d; c += 256) {
      float xv[8], dyv[8], wf[8];
      unpack8(*reinterpret_cast<const uint4*>(x + base + c), xv);
      unpack8(*reinterpret_cast<const uint4*>(dy + base + c), dyv);
      unpack8(*reinterpret_cast<const uint4*>(w + c), wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) dot += dyv[e] * wf[e] * xv[e];
    }
    dot = warp_sum(dot) * r / (float)d;
    for (int c = lane * 8; c < d; c += 256) {
      float xv[8], dyv[8], wf[8], rv[8], o[8];
      unpack8(*reinterpret_cast<const uint4*>(x + base + c), xv);
      unpack8(*reinterpret_cast<const uint4*>(dy + base + c), dyv);
      unpack8(*reinterpret_cast<const uint4*>(w + c), wf);
      if (dres != nullptr) {
        unpack8(*reinterpret_cast<const uint4*>(dres + base + c), rv);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) rv[e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = rv[e] + r * (dyv[e] * wf[e] - xv[e] * r * dot);
      *reinterpret_cast<uint4*>(dx + base + c) = pack8(o);
      float4* acc = reinterpret_cast<float4*>(mine + c);
      float4 a0 = acc[0], a1 = acc[1];
      a0.x += dyv[0] * xv[0] * r; a0.y += dyv[1] * xv[1] * r; a0.z += dyv[2] * xv[2] * r; a0.w += dyv[3] * xv[3] * r;
      a1.x += dyv[4] * xv[4] * r; a1.y += dyv[5] * xv[5] * r; a1.z += dyv[6] * xv[6] * r; a1.w += dyv[7] * xv[7] * r;
      acc[0] = a0;
      acc[1] = a1;
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < kWideWarps; ++k) t += dw_rows[(size_t)k * d + c];
    atomicAdd(dw + c, t);
  }
}

__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                     __nv_bfloat16* __restrict__ out, int rows, int d, int vocab,
                                     DeviceErrors* errs) {
  pdl_wait_and_release();
  const int vec_per_row = d / 8;
  const size_t total = (size_t)rows * vec_per_row;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / vec_per_row);
    const int v = (int)(i % vec_per_row);
    int64_t id = ids[row];
    uint4 val = make_uint4(0, 0, 0, 0);
    if (id >= 0 && id < vocab)
      val = *reinterpret_cast<const uint4*>(table + (size_t)id * d + v * 8);
    else if (v == 0)
      report_error(errs, kErrBadIndex, row);  // the row reads as zeros; the host raises at its next check
    *reinterpret_cast<uint4*>(out + (size_t)row * d + v * 8) = val;
  }
}

__global__ void embedding_bwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ dy,
                                     float* __restrict__ dtable, int rows, int d, int vocab) {
  pdl_wait_and_release();
  const int vec_per_row = d / 8;
  const size_t total = (size_t)rows * vec_per_row;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / vec_per_row);
    const int v = (int)(i % vec_per_row);
    const int64_t id = ids[row];
    if (id < 0 || id >= vocab) continue;
    float g[8];
    unpack8(*reinterpret_cast<const uint4*>(dy + (size_t)row * d + v * 8), g);
    float* dst = dtable + (size_t)id * d + v * 8;
    atomicAdd(reinterpret_cast<float4*>(dst), make_float4(g[0], g[1], g[2], g[3]));
    atomicAdd(reinterpret_cast<float4*>(dst + 4), make_float4(g[4], g[5], g[6], g[7]));
  }
}

// In-place inverse rotation of the q and k columns of a [rows, ld] gradient.
__global__ void rope_bwd_kernel(__nv_bfloat16* __restrict__ g, int rows, int ld, int rope_cols, int head_dim,
                                int seq_len, const float* __restrict__ cosv, const float* __restrict__ sinv) {
  pdl_wait_and_release();
  const int half = head_dim / 2;
  const int groups_per_row = rope_cols / head_dim * (half / 8);
  const size_t total = (size_t)rows * groups_per_row;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / groups_per_row);
    const int gidx = (int)(i % groups_per_row);
    const int head = gidx / (half / 8);
    const int j = (gidx % (half / 8)) * 8;
    const int pos = row % seq_len;
    __nv_bfloat16* lo = g + (size_t)row * ld + head * head_dim + j;
    __nv_bfloat16* hi = lo + half;
    float a[8], b[8], oa[8], ob[8];
    unpack8(*reinterpret_cast<const uint4*>(lo), a);
    unpack8(*reinterpret_cast<const uint4*>(hi), b);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float c = cosv[(size_t)pos * half + j + e], s = sinv[(size_t)pos * half + j + e];
      oa[e] = a[e] * c + b[e] * s;
      ob[e] = b[e] * c - a[e] * s;
    }
    *reinterpret_cast<uint4*>(lo) = pack8(oa);
    *reinterpret_cast<uint4*>(hi) = pack8(ob);
  }
}

int grid_for(size_t work, int threads) {
  const size_t blocks = (work + threads - 1) / threads;
  const size_t cap = (size_t)num_sms_cached() * 16;
  return (int)std::max<size_t>(1, std::min(blocks, cap));
}

}  // namespace

int num_sms_cached() {
  static int n = 0;
  if (n == 0) {
    int dev;
    B200_CUDA_CHECK(cudaGetDevice(&dev));
    B200_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

void rmsnorm_fwd(const __nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* y, float* rstd, int rows, int d,
                 float eps, cudaStream_t s) {
  B200_CHECK(d % 8 == 0 && d <= 256 * 16, "rmsnorm: d must be a multiple of 8 and at most 4096");
  const int blocks = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  const int vec = (d + 255) / 256;
  if (vec <= 1)
    launch_k(rmsnorm_fwd_kernel<1>, dim3(blocks), dim3(32 * kWarpsPerBlock), 0, s, 1, x, w, y, rstd, rows, d, eps);
  else if (vec <= 2)
    launch_k(rmsnorm_fwd_kernel<2>, dim3(blocks), dim3(32 * kWarpsPerBlock), 0, s, 1, x, w, y, rstd, rows, d, eps);
  else if (vec <= 3)
    launch_k(rmsnorm_fwd_kernel<3>, dim3(blocks), dim3(32 * kWarpsPerBlock), 0, s, 1, x, w, y, rstd, rows, d, eps);
  else if (vec <= 4)
    launch_k(rmsnorm_fwd_kernel<4>, dim3(blocks), dim3(32 * kWarpsPerBlock), 0, s, 1, x, w, y, rstd, rows, d, eps);
  else if (vec <= 8)
    launch_k(rmsnorm_fwd_kernel<8>, dim3(blocks), dim3(32 * kWarpsPerBlock), 0, s, 1, x, w, y, rstd, rows, d, eps);
  else
    launch_k(rmsnorm_fwd_kernel<16>, dim3(blocks), dim3(32 * kWarpsPerBlock), 0, s, 1, x, w, y, rstd, rows, d, eps);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void rmsnorm_bwd(const __nv_bfloat16* dy, const __nv_bfloat16* x, const __nv_bfloat16* w, const float* rstd,
                 const __nv_bfloat16* dres, __nv_bfloat16* dx, float* dw, int rows, int d, cudaStream_t s) {
  B200_CHECK(d % 8 == 0 && d <= kWideMaxD, "rmsnorm_bwd: d must be a multiple of 8 and at most 12288");
  if (d > 256 * 8) {
    const size_t smem = (size_t)kWideWarps * d * sizeof(float);
    static std::atomic<unsigned long long> configured{0};
    once_per_device(configured, [&] {
      B200_CUDA_CHECK(cudaFuncSetAttribute(rmsnorm_bwd_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)((size_t)kWideWarps * kWideMaxD * sizeof(float))));
    });
    const int blocks = std::max(1, std::min((rows + kWideWarps - 1) / kWideWarps, 2 * num_sms_cached()));
    launch_k(rmsnorm_bwd_wide_kernel, dim3(blocks), dim3(32 * kWideWarps), smem, s, 1, dy, x, w, rstd, dres, dx, dw,
             rows, d);
    B200_CUDA_CHECK(cudaGetLastError());
    count_launch();
    return;
  }
  const int vec = (d + 255) / 256;
  const int per_block = kWarpsPerBlock * (vec <= 4 ? 2 : 1);
  const int blocks = std::max(1, (rows + per_block - 1) / per_block);
  const int threads = 32 * kWarpsPerBlock;
  if (vec <= 1)
    launch_k(rmsnorm_bwd_kernel<1, 2>, dim3(blocks), dim3(threads), 0, s, 1, dy, x, w, rstd, dres, dx, dw, rows, d);
  else if (vec <= 2)
    launch_k(rmsnorm_bwd_kernel<2, 2>, dim3(blocks), dim3(threads), 0, s, 1, dy, x, w, rstd, dres, dx, dw, rows, d);
  else if (vec <= 3)
    launch_k(rmsnorm_bwd_kernel<3, 2>, dim3(blocks), dim3(threads), 0, s, 1, dy, x, w, rstd, dres, dx, dw, rows, d);
  else if (vec <= 4)
    launch_k(rmsnorm_bwd_kernel<4, 2>, dim3(blocks), dim3(threads), 0, s, 1, dy, x, w, rstd, dres, dx, dw, rows, d);
  else
    launch_k(rmsnorm_bwd_kernel<8, 1>, dim3(blocks), dim3(threads), 0, s, 1, dy, x, w, rstd, dres, dx, dw, rows, d);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void embedding_fwd(const int64_t* ids, const __nv_bfloat16* table, __nv_bfloat16* out, int rows, int d, int vocab,
                   cudaStream_t s) {
  B200_CHECK(d % 8 == 0, "embedding: d must be a multiple of 8");
  launch_k(embedding_fwd_kernel, dim3(grid_for((size_t)rows * d / 8, 256)), dim3(256), 0, s, 1, ids, table, out, rows, d, vocab,
                                                                            device_errors_ptr());
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void embedding_bwd(const int64_t* ids, const __nv_bfloat16* dy, float* dtable, int rows, int d, int vocab,
                   cudaStream_t s) {
  launch_k(embedding_bwd_kernel, dim3(grid_for((size_t)rows * d / 8, 256)), dim3(256), 0, s, 1, ids, dy, dtable, rows, d, vocab);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void rope_bwd(__nv_bfloat16* g, int rows, int ld, int rope_cols, int head_dim, int seq_len, const float* cosv,
              const float* sinv, cudaStream_t s) {
  B200_CHECK(head_dim % 16 == 0 && rope_cols % head_dim == 0, "rope_bwd: bad head layout");
  const size_t work = (size_t)rows * (rope_cols / head_dim) * (head_dim / 16);
  launch_k(rope_bwd_kernel, dim3(grid_for(work, 256)), dim3(256), 0, s, 1, g, rows, ld, rope_cols, head_dim, seq_len, cosv, sinv);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

}  // namespace b200
