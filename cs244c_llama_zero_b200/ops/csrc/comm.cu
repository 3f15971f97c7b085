// NVLink 5 / NVSwitch collective kernels for the ZeRO engines.
//
// Data moves through symmetric memory: each rank's buffer is mapped on every GPU (peer pointers)
// and, when the NVSwitch supports it, bound to a multicast object.  With multicast the switch
// does the arithmetic: `multimem.ld_reduce` returns the sum over all ranks of one 16-byte vector
// and `multimem.st` writes one vector to every rank.  Without multicast the same kernels use
// plain peer loads and stores.
//
//   allreduce            each rank reduces its 1/W slice (ld_reduce) and broadcasts it (st), with
//                        the 1/W gradient averaging fused in
//   reduce_scatter_acc   each rank ld_reduces its own chunk and accumulates scale * sum into its
//                        local fp32 gradient shard (ZeRO-2/3 gradient reduce-scatter + averaging)
//   allgather            each rank multicasts its shard into every rank's buffer
//   adamw_allgather      AdamW on the local fp32 shard; the bf16 result is multicast straight into
//                        every rank's parameter buffer (ZeRO-1/2 update + parameter all-gather)
//   rs_adamw_allgather   the whole ZeRO-2 step without clipping in one kernel: each rank ld_reduces
//                        its chunk of the flat fp32 gradients, averages it, adds its squares to the
//                        norm, runs AdamW and multicasts the bf16 result (no gradient shard in HBM)
//   bucket_reduce        one gradient bucket (a transformer block's weights): each rank reduces its
//                        slice into its fp32 gradient segment, then the bucket buffer is cleared for
//                        reuse (ZeRO-2 gradient ring, interleaved shards)
//   adamw_allgather_seg  AdamW on the interleaved shard and the bf16 result multicast into every
//                        rank's parameter buffer, segment by segment
//   push_rs              reduce-scatter by peer stores into a landing area + a local sum (each byte
//                        crosses NVLink once; the better choice at 2 and 4 ranks)
//
// Ordering: every block of every rank runs the same grid, and block b synchronises with block b of
// every peer at kernel start (all inputs written) and at kernel end (all outputs delivered).  The
// barrier writes a per-block epoch into the peer's signal pad with st.release.sys and polls its own
// pad with ld.acquire.sys; the epochs live in device memory.  Every poll is bounded by a
// %globaltimer deadline; on expiry the block records an error in the device error record and returns.
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>

#include "comm.h"
#include "common.cuh"

namespace b200 {

namespace {

constexpr int kThreads = 512;
constexpr int kUnroll = 8;  // independent 16-byte vectors in flight per thread

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ float4 mc_ld_reduce_f32x4(uint64_t addr) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void mc_st_f32x4(uint64_t addr, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void mc_st_b128(uint64_t addr, uint4 v) {
  mc_st_f32x4(addr, make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w)));
}
// Sum over ranks of 8 bf16 values, accumulated in fp32 inside the switch, returned as bf16x2 words.
__device__ __forceinline__ uint4 mc_ld_reduce_bf16x8(uint64_t addr) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void bf16x8_to_f32(uint4 q, float (&f)[8]) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = bf16lo(w[i]);
    f[2 * i + 1] = bf16hi(w[i]);
  }
}
__device__ __forceinline__ uint4 f32_to_bf16x8(const float (&f)[8]) {
  return make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]), pack_bf16(f[4], f[5]), pack_bf16(f[6], f[7]));
}

// Returns this block's epoch for this call (same value on every rank: same call sequence, same grid).
__device__ __forceinline__ uint32_t next_epoch(const CommCtx& c) {
  __shared__ uint32_t e;
  if (threadIdx.x == 0) {
    e = c.epochs[blockIdx.x] + 1;
    c.epochs[blockIdx.x] = e;
  }
  __syncthreads();
  return e;
}

__device__ bool block_barrier(const CommCtx& c, uint32_t value) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  fence_sys();
  __syncthreads();
  if (threadIdx.x < c.world) {
    const int peer = threadIdx.x;
    uint32_t* remote = reinterpret_cast<uint32_t*>(c.pads[peer]) + blockIdx.x * kCommMaxWorld + c.rank;
    st_release_sys(remote, value);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(c.pads[c.rank]) + blockIdx.x * kCommMaxWorld + peer;
    const uint64_t t0 = globaltimer_ns();
    while ((int)(ld_acquire_sys(mine) - value) < 0) {
      if (globaltimer_ns() - t0 > c.timeout_ns) {
        report_error(c.errs, kErrCommBarrier, peer);
        ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

__device__ __forceinline__ size_t gtid() { return (size_t)blockIdx.x * blockDim.x + threadIdx.x; }
__device__ __forceinline__ size_t gstride() { return (size_t)gridDim.x * blockDim.x; }

template <bool MC>
__global__ void __launch_bounds__(kThreads) allreduce_f32_kernel(CommCtx c, size_t off, size_t n4, float scale) {
  const uint32_t e = next_epoch(c);
  if (!block_barrier(c, 2 * e)) return;
  const size_t per = (n4 + c.world - 1) / c.world;
  const size_t lo = (size_t)c.rank * per, hi = min(n4, lo + per);
  const size_t stride = gstride();
  for (size_t i0 = lo + gtid(); i0 < hi; i0 += stride * kUnroll) {
    float4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i >= hi) break;
      const size_t b = off + i * 16;
      if constexpr (MC) {
        v[u] = mc_ld_reduce_f32x4(c.mc + b);
      } else {
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int w = 0; w < c.world; ++w) {
          const float4 x = __ldcg(reinterpret_cast<const float4*>(c.peers[w] + b));
          v[u].x += x.x; v[u].y += x.y; v[u].z += x.z; v[u].w += x.w;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i >= hi) break;
      const size_t b = off + i * 16;
      float4 x = v[u];
      x.x *= scale; x.y *= scale; x.z *= scale; x.w *= scale;
      if constexpr (MC) {
        mc_st_f32x4(c.mc + b, x);
      } else {
        for (int w = 0; w < c.world; ++w) __stcg(reinterpret_cast<float4*>(c.peers[w] + b), x);
      }
    }
  }
  block_barrier(c, 2 * e + 1);
}

template <bool MC>
__global__ void __launch_bounds__(kThreads) reduce_scatter_acc_f32_kernel(CommCtx c, size_t off, size_t chunk4,
                                                                          float4* acc, float scale) {
  const uint32_t e = next_epoch(c);
  if (!block_barrier(c, 2 * e)) return;
  const size_t base = off + (size_t)c.rank * chunk4 * 16;
  const size_t stride = gstride();
  for (size_t i0 = gtid(); i0 < chunk4; i0 += stride * kUnroll) {
    float4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i >= chunk4) break;
      const size_t b = base + i * 16;
      if constexpr (MC) {
        v[u] = mc_ld_reduce_f32x4(c.mc + b);
      } else {
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int w = 0; w < c.world; ++w) {
          const float4 x = __ldcg(reinterpret_cast<const float4*>(c.peers[w] + b));
          v[u].x += x.x; v[u].y += x.y; v[u].z += x.z; v[u].w += x.w;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i >= chunk4) break;
      float4 a = acc[i];
      a.x += scale * v[u].x; a.y += scale * v[u].y; a.z += scale * v[u].z; a.w += scale * v[u].w;
      acc[i] = a;
    }
  }
  block_barrier(c, 2 * e + 1);
}

// Bucketed variant for reduce-scatter overlapped with backward: the region is one bucket of the
// flat buffer, and this rank reduces only the part of it that falls inside its own shard
// ([lo4, hi4) in 16-byte vectors from the region start; possibly empty), accumulating into acc[0..).
// Every rank still joins both barriers so the per-block epochs stay aligned.
template <bool MC>
__global__ void __launch_bounds__(kThreads) reduce_scatter_range_acc_f32_kernel(CommCtx c, size_t off, size_t lo4,
                                                                                size_t hi4, float4* acc, float scale) {
  const uint32_t e = next_epoch(c);
  if (!block_barrier(c, 2 * e)) return;
  const size_t n4 = hi4 > lo4 ? hi4 - lo4 : 0;
  const size_t base = off + lo4 * 16;
  const size_t stride = gstride();
  for (size_t i0 = gtid(); i0 < n4; i0 += stride * kUnroll) {
    float4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i >= n4) break;
      const size_t b = base + i * 16;
      if constexpr (MC) {
        v[u] = mc_ld_reduce_f32x4(c.mc + b);
      } else {
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int w = 0; w < c.world; ++w) {
          const float4 x = __ldcg(reinterpret_cast<const float4*>(c.peers[w] + b));
          v[u].x += x.x; v[u].y += x.y; v[u].z += x.z; v[u].w += x.w;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i >= n4) break;
      float4 a = acc[i];
      a.x += scale * v[u].x; a.y += scale * v[u].y; a.z += scale * v[u].z; a.w += scale * v[u].w;
      acc[i] = a;
    }
  }
  block_barrier(c, 2 * e + 1);
}

// bf16 variants: 16-byte vectors of 8 values; sums accumulate in fp32 (switch-side with multicast,
// in registers with peer loads) and are rounded once.
template <bool MC>
__global__ void __launch_bounds__(kThreads) allreduce_bf16_kernel(CommCtx c, size_t off, size_t n8, float scale) {
  const uint32_t e = next_epoch(c);
  if (!block_barrier(c, 2 * e)) return;
  const size_t per = (n8 + c.world - 1) / c.world;
  const size_t lo = (size_t)c.rank * per, hi = min(n8, lo + per);
  const size_t stride = gstride();
  for (size_t i0 = lo + gtid(); i0 < hi; i0 += stride * kUnroll) {
    float v[kUnroll][8];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i >= hi) break;
      const size_t b = off + i * 16;
      if constexpr (MC) {
        bf16x8_to_f32(mc_ld_reduce_bf16x8(c.mc + b), v[u]);
      } else {
#pragma unroll
        for (int t = 0; t < 8; ++t) v[u][t] = 0.f;
        for (int w = 0; w < c.world; ++w) {
          float x[8];
          bf16x8_to_f32(__ldcg(reinterpret_cast<const uint4*>(c.peers[w] + b)), x);
#pragma unroll
          for (int t = 0; t < 8; ++t) v[u][t] += x[t];
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i >= hi) break;
      const size_t b = off + i * 16;
#pragma unroll
      for (int t = 0; t < 8; ++t) v[u][t] *= scale;
      const uint4 o = f32_to_bf16x8(v[u]);
      if constexpr (MC) {
        mc_st_b128(c.mc + b, o);
      } else {
        for (int w = 0; w < c.world; ++w) __stcg(reinterpret_cast<uint4*>(c.peers[w] + b), o);
      }
    }
  }
  block_barrier(c, 2 * e + 1);
}

template <bool MC>
__global__ void __launch_bounds__(kThreads) reduce_scatter_acc_bf16_kernel(CommCtx c, size_t off, size_t chunk8,
                                                                           float* acc, float scale) {
  const uint32_t e = next_epoch(c);
  if (!block_barrier(c, 2 * e)) return;
  const size_t base = off + (size_t)c.rank * chunk8 * 16;
  const size_t stride = gstride();
  // kUnroll independent 16-byte loads in flight per thread (peer loads: W x kUnroll), as in the
  // fp32 kernels: the reduction is bound by NVLink latency x bytes in flight.
  for (size_t i0 = gtid(); i0 < chunk8; i0 += stride * kUnroll) {
    uint4 q[kUnroll];
    float v[kUnroll][8];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i >= chunk8) break;
      const size_t b = base + i * 16;
      if constexpr (MC) {
        q[u] = mc_ld_reduce_bf16x8(c.mc + b);
      } else {
#pragma unroll
        for (int t = 0; t < 8; ++t) v[u][t] = 0.f;
        for (int w = 0; w < c.world; ++w) {
          float x[8];
          bf16x8_to_f32(__ldcg(reinterpret_cast<const uint4*>(c.peers[w] + b)), x);
#pragma unroll
          for (int t = 0; t < 8; ++t) v[u][t] += x[t];
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i >= chunk8) break;
      if constexpr (MC) bf16x8_to_f32(q[u], v[u]);
      float4* a4 = reinterpret_cast<float4*>(acc + i * 8);
      float4 a0 = a4[0], a1 = a4[1];
      a0.x += scale * v[u][0]; a0.y += scale * v[u][1]; a0.z += scale * v[u][2]; a0.w += scale * v[u][3];
      a1.x += scale * v[u][4]; a1.y += scale * v[u][5]; a1.z += scale * v[u][6]; a1.w += scale * v[u][7];
      a4[0] = a0;
      a4[1] = a1;
    }
  }
  block_barrier(c, 2 * e + 1);
}

template <bool MC>
__global__ void __launch_bounds__(kThreads) allgather_kernel(CommCtx c, size_t off, size_t chunk16,
                                                             const uint4* shard) {
  const uint32_t e = next_epoch(c);
  if (!block_barrier(c, 2 * e)) return;
  const size_t base = off + (size_t)c.rank * chunk16 * 16;
  const size_t stride = gstride();
  for (size_t i0 = gtid(); i0 < chunk16; i0 += stride * kUnroll) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i < chunk16) v[u] = shard[i];
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i >= chunk16) break;
      const size_t b = base + i * 16;
      if constexpr (MC) {
        mc_st_b128(c.mc + b, v[u]);
      } else {
        for (int w = 0; w < c.world; ++w) __stcg(reinterpret_cast<uint4*>(c.peers[w] + b), v[u]);
      }
    }
  }
  block_barrier(c, 2 * e + 1);
}

struct AdamScalars {
  float lr, beta1, beta2, eps, decay, step, inv_sqrt_bc2, scale_const;
};

template <bool MC>
__global__ void __launch_bounds__(kThreads) adamw_allgather_kernel(CommCtx c, size_t param_off, size_t chunk8,
                                                                   float4* master, float4* m, float4* v,
                                                                   const float4* g, const float* scale_ptr,
                                                                   AdamScalars a, const float* dev_sc) {
  const uint32_t e = next_epoch(c);
  if (!block_barrier(c, 2 * e)) return;
  const float scale = (scale_ptr != nullptr ? *scale_ptr : 1.0f) * a.scale_const;
  if (dev_sc != nullptr) {  // bias corrections from the device step counter (replayable graphs)
    a.step = dev_sc[0];
    a.inv_sqrt_bc2 = dev_sc[1];
  }
  const size_t base = param_off + (size_t)c.rank * chunk8 * 16;  // chunk8 groups of 8 bf16 = 16 bytes
  for (size_t i = gtid(); i < chunk8; i += gstride()) {
    float out[8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const size_t k = 2 * i + h;
      float4 gp = g[k], mp = m[k], vp = v[k], pp = master[k];
      float gg[4] = {gp.x * scale, gp.y * scale, gp.z * scale, gp.w * scale};
      float mm[4] = {mp.x, mp.y, mp.z, mp.w}, vv[4] = {vp.x, vp.y, vp.z, vp.w}, pw[4] = {pp.x, pp.y, pp.z, pp.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        mm[t] = a.beta1 * mm[t] + (1.0f - a.beta1) * gg[t];
        vv[t] = a.beta2 * vv[t] + (1.0f - a.beta2) * gg[t] * gg[t];
        pw[t] = pw[t] * a.decay - a.step * mm[t] / (sqrtf(vv[t]) * a.inv_sqrt_bc2 + a.eps);
        out[4 * h + t] = pw[t];
      }
      m[k] = make_float4(mm[0], mm[1], mm[2], mm[3]);
      v[k] = make_float4(vv[0], vv[1], vv[2], vv[3]);
      master[k] = make_float4(pw[0], pw[1], pw[2], pw[3]);
    }
    const uint4 o = f32_to_bf16x8(out);
    const size_t b = base + i * 16;
    if constexpr (MC) {
      mc_st_b128(c.mc + b, o);
    } else {
      for (int w = 0; w < c.world; ++w) __stcg(reinterpret_cast<uint4*>(c.peers[w] + b), o);
    }
  }
  block_barrier(c, 2 * e + 1);
}

// Reduce-scatter of the gradients (context g) + sum of squares + AdamW + parameter all-gather
// (context c, whose barriers order the whole step).  Element k of this rank's chunk: gradient at
// g region [rank*chunk + k], optimizer state at master/m/v[k], parameter at c region [rank*chunk + k].
template <bool MC>
__global__ void __launch_bounds__(kThreads) rs_adamw_allgather_kernel(CommCtx c, CommCtx g, size_t g_off,
                                                                      size_t param_off, size_t chunk8,
                                                                      float4* master, float4* m, float4* v,
                                                                      float grad_scale, AdamScalars a,
                                                                      const float* dev_sc, float* sq_out) {
  const uint32_t e = next_epoch(c);
  if (!block_barrier(c, 2 * e)) return;
  if (dev_sc != nullptr) {
    a.step = dev_sc[0];
    a.inv_sqrt_bc2 = dev_sc[1];
  }
  const size_t gbase = g_off + (size_t)c.rank * chunk8 * 32;  // chunk8 groups of 8 fp32 = 32 bytes
  const size_t pbase = param_off + (size_t)c.rank * chunk8 * 16;
  float sq = 0.f;
  for (size_t i = gtid(); i < chunk8; i += gstride()) {
    float out[8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const size_t gb = gbase + i * 32 + h * 16;
      float4 gp;
      if constexpr (MC) {
        gp = mc_ld_reduce_f32x4(g.mc + gb);
      } else {
        gp = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int w = 0; w < g.world; ++w) {
          const float4 x = __ldcg(reinterpret_cast<const float4*>(g.peers[w] + gb));
          gp.x += x.x; gp.y += x.y; gp.z += x.z; gp.w += x.w;
        }
      }
      const size_t k = 2 * i + h;
      float4 mp = m[k], vp = v[k], pp = master[k];
      float gg[4] = {gp.x * grad_scale, gp.y * grad_scale, gp.z * grad_scale, gp.w * grad_scale};
      float mm[4] = {mp.x, mp.y, mp.z, mp.w}, vv[4] = {vp.x, vp.y, vp.z, vp.w}, pw[4] = {pp.x, pp.y, pp.z, pp.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        sq += gg[t] * gg[t];
        mm[t] = a.beta1 * mm[t] + (1.0f - a.beta1) * gg[t];
        vv[t] = a.beta2 * vv[t] + (1.0f - a.beta2) * gg[t] * gg[t];
        pw[t] = pw[t] * a.decay - a.step * mm[t] / (sqrtf(vv[t]) * a.inv_sqrt_bc2 + a.eps);
        out[4 * h + t] = pw[t];
      }
      m[k] = make_float4(mm[0], mm[1], mm[2], mm[3]);
      v[k] = make_float4(vv[0], vv[1], vv[2], vv[3]);
      master[k] = make_float4(pw[0], pw[1], pw[2], pw[3]);
    }
    const uint4 o = f32_to_bf16x8(out);
    const size_t b = pbase + i * 16;
    if constexpr (MC) {
      mc_st_b128(c.mc + b, o);
    } else {
      for (int w = 0; w < c.world; ++w) __stcg(reinterpret_cast<uint4*>(c.peers[w] + b), o);
    }
  }
  // this rank's share of the squared norm of the averaged gradient
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  __shared__ float part[kThreads / 32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < kThreads / 32 ? part[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0 && sq_out != nullptr) atomicAdd(sq_out, t);
  }
  block_barrier(c, 2 * e + 1);
}

__global__ void routed_add_kernel(const float4* __restrict__ src, size_t n, long long flat0, RouteTable t,
                                  DeviceErrors* errs) {
  const size_t n4 = n / 4;
  for (size_t i = gtid(); i < n4; i += gstride()) {
    const long long f = flat0 + 4 * (long long)i;
    const int owner = (int)(f / t.chunk);
    if (owner >= t.world) {
      report_error(errs, kErrBadIndex, 201);
      continue;
    }
    const float4 v = src[i];
    red_add_f32x4_sys(reinterpret_cast<float*>(t.base[owner]) + (f - (long long)owner * t.chunk),
                      __float_as_uint(v.x), __float_as_uint(v.y), __float_as_uint(v.z), __float_as_uint(v.w));
  }
  const float* tail = reinterpret_cast<const float*>(src);
  for (size_t k = n4 * 4 + gtid(); k < n; k += gstride()) {
    const long long f = flat0 + (long long)k;
    const int owner = (int)(f / t.chunk);
    if (owner >= t.world) {
      report_error(errs, kErrBadIndex, 202);
      continue;
    }
    red_add_f32_sys(reinterpret_cast<float*>(t.base[owner]) + (f - (long long)owner * t.chunk), tail[k]);
  }
}

__global__ void embedding_bwd_routed_kernel(const int64_t* __restrict__ ids, const uint4* __restrict__ dy, int rows,
                                            int d, int vocab, long long flat0, RouteTable t, DeviceErrors* errs) {
  const int vec = d / 8;
  const size_t total = (size_t)rows * vec;
  for (size_t i = gtid(); i < total; i += gstride()) {
    const int row = (int)(i / vec), v = (int)(i % vec);
    const int64_t id = ids[row];
    if (id < 0 || id >= vocab) continue;  // the forward pass recorded it already
    float g[8];
    bf16x8_to_f32(dy[i], g);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const long long f = flat0 + (long long)id * d + v * 8 + 4 * h;
      const int owner = (int)(f / t.chunk);
      if (owner >= t.world) {
        report_error(errs, kErrBadIndex, 203);
        continue;
      }
      red_add_f32x4_sys(reinterpret_cast<float*>(t.base[owner]) + (f - (long long)owner * t.chunk),
                        __float_as_uint(g[4 * h]), __float_as_uint(g[4 * h + 1]), __float_as_uint(g[4 * h + 2]),
                        __float_as_uint(g[4 * h + 3]));
    }
  }
}

// One gradient bucket of the ZeRO-2 gradient ring.  The bucket region [off, off + 16*W*part4) of
// every rank's bucket buffer holds that rank's gradient of one transformer block (zero past the
// block's end); rank r owns slice r (vectors [r*part4, (r+1)*part4)) of every bucket, so it reduces
// that slice over the ranks and adds scale * sum into its local fp32 gradient segment acc[0, part4)
// - no remote writes.  After the closing barrier every rank has read every slice, and block b
// zeroes the vectors that block b of every rank read from this rank's buffer: the buffer is ready
// for the next bucket.
template <bool MC>
__global__ void __launch_bounds__(kThreads) bucket_reduce_kernel(CommCtx c, size_t off, size_t part4, float4* acc,
                                                                  float scale) {
  const uint32_t e = next_epoch(c);
  if (!block_barrier(c, 2 * e)) return;
  const size_t base = off + (size_t)c.rank * part4 * 16;
  const size_t stride = gstride();
  for (size_t i0 = gtid(); i0 < part4; i0 += stride * kUnroll) {
    float4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i >= part4) break;
      const size_t b = base + i * 16;
      if constexpr (MC) {
        v[u] = mc_ld_reduce_f32x4(c.mc + b);
      } else {
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int w = 0; w < c.world; ++w) {
          const float4 x = __ldcg(reinterpret_cast<const float4*>(c.peers[w] + b));
          v[u].x += x.x; v[u].y += x.y; v[u].z += x.z; v[u].w += x.w;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const size_t i = i0 + u * stride;
      if (i >= part4) break;
      float4 a = acc[i];
      a.x += scale * v[u].x; a.y += scale * v[u].y; a.z += scale * v[u].z; a.w += scale * v[u].w;
      acc[i] = a;
    }
  }
  if (!block_barrier(c, 2 * e + 1)) return;
  // Block b of rank q read vectors q*part4 + j with j on the grid-stride walk from gtid(); the same
  // walk over every slice here clears exactly what block b of every rank has finished reading.
  float4* mine = reinterpret_cast<float4*>(c.peers[c.rank] + off);
  for (int q = 0; q < c.world; ++q) {
    float4* slice = mine + (size_t)q * part4;
    for (size_t j = gtid(); j < part4; j += stride) slice[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// AdamW on this rank's fp32 shard of the gradient ring's interleaved layout, with the bf16 result
// multicast into every rank's parameter buffer.  The shard is the concatenation of segments: segment
// s holds, at shard positions [seg[s].shard8 * 8, + part8 * 8), slice `rank` of one bucket, i.e. flat
// parameters starting at seg[s].param_off (bytes) + rank * part8 * 16; only its first seg[s].valid8
// groups of 8 lie inside the bucket (the rest pad the slice to a common length and are not written).
template <bool MC>
__global__ void __launch_bounds__(kThreads) adamw_allgather_seg_kernel(CommCtx c, const RingSeg* __restrict__ seg,
                                                                       int nseg, size_t total8, float4* master,
                                                                       float4* m, float4* v, const float4* g,
                                                                       const float* scale_ptr, AdamScalars a,
                                                                       const float* dev_sc) {
  const uint32_t e = next_epoch(c);
  if (!block_barrier(c, 2 * e)) return;
  const float scale = (scale_ptr != nullptr ? *scale_ptr : 1.0f) * a.scale_const;
  if (dev_sc != nullptr) {
    a.step = dev_sc[0];
    a.inv_sqrt_bc2 = dev_sc[1];
  }
  int s = 0;
  for (size_t i = gtid(); i < total8; i += gstride()) {
    while (s + 1 < nseg && (size_t)seg[s + 1].shard8 <= i) ++s;  // i only grows within a thread
    float out[8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const size_t k = 2 * i + h;
      float4 gp = g[k], mp = m[k], vp = v[k], pp = master[k];
      float gg[4] = {gp.x * scale, gp.y * scale, gp.z * scale, gp.w * scale};
      float mm[4] = {mp.x, mp.y, mp.z, mp.w}, vv[4] = {vp.x, vp.y, vp.z, vp.w}, pw[4] = {pp.x, pp.y, pp.z, pp.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        mm[t] = a.beta1 * mm[t] + (1.0f - a.beta1) * gg[t];
        vv[t] = a.beta2 * vv[t] + (1.0f - a.beta2) * gg[t] * gg[t];
        pw[t] = pw[t] * a.decay - a.step * mm[t] / (sqrtf(vv[t]) * a.inv_sqrt_bc2 + a.eps);
        out[4 * h + t] = pw[t];
      }
      m[k] = make_float4(mm[0], mm[1], mm[2], mm[3]);
      v[k] = make_float4(vv[0], vv[1], vv[2], vv[3]);
      master[k] = make_float4(pw[0], pw[1], pw[2], pw[3]);
    }
    const long long j = (long long)i - seg[s].shard8;
    if (j >= seg[s].valid8) continue;
    const uint4 o = f32_to_bf16x8(out);
    const size_t b = (size_t)seg[s].param_off + ((size_t)c.rank * seg[s].part8 + (size_t)j) * 16;
    if constexpr (MC) {
      mc_st_b128(c.mc + b, o);
    } else {
      for (int w = 0; w < c.world; ++w) __stcg(reinterpret_cast<uint4*>(c.peers[w] + b), o);
    }
  }
  block_barrier(c, 2 * e + 1);
}

// Push reduce-scatter (fp32): the data moves as posted peer stores instead of switch reductions or
// peer loads.  src (this rank's local data: W slices of part4 vectors, slice q starting at vector
// q * sstride4, so a call can cover one piece of every slice of a larger buffer) need not be
// symmetric; the
// context's buffer holds the landing area at land_off: W rows of part4 vectors, row q written by
// rank q.  Phase 1 stores slice q of src into rank q's row `rank`; after the middle barrier (block b
// of every rank has stored its vectors, which are the same j positions block b reads below) each
// rank adds its own slice and the W - 1 landed rows into acc.  A store crosses NVLink once, where a
// multicast reduction at two ranks reads every byte of both GPUs through the switch.  With clear_src
// the block zeroes the src vectors it has finished with (src is read by this rank only).
template <bool CLEAR>
__global__ void __launch_bounds__(kThreads) push_rs_f32_kernel(CommCtx c, float4* __restrict__ src, size_t sstride4,
                                                                size_t land_off, size_t part4, float4* acc,
                                                                float scale) {
  const uint32_t e = next_epoch(c);
  if (!block_barrier(c, 2 * e)) return;  // every rank's landing area is free again
  const size_t stride = gstride();
  for (int qi = 1; qi < c.world; ++qi) {
    const int q = (c.rank + qi) % c.world;  // each rank starts with a different destination
    float4* dst = reinterpret_cast<float4*>(c.peers[q] + land_off) + (size_t)c.rank * part4;
    const float4* s = src + (size_t)q * sstride4;
    for (size_t j0 = gtid(); j0 < part4; j0 += stride * kUnroll) {
      float4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const size_t j = j0 + u * stride;
        if (j < part4) v[u] = s[j];
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const size_t j = j0 + u * stride;
        if (j < part4) __stcg(dst + j, v[u]);
      }
    }
  }
  if (!block_barrier(c, 2 * e + 1)) return;
  const float4* land = reinterpret_cast<const float4*>(c.peers[c.rank] + land_off);
  float4* own = src + (size_t)c.rank * sstride4;
  for (size_t j = gtid(); j < part4; j += stride) {
    float4 t = own[j];
    for (int q = 0; q < c.world; ++q) {
      if (q == c.rank) continue;
      const float4 x = __ldcg(land + (size_t)q * part4 + j);  // written over NVLink: skip L1
      t.x += x.x; t.y += x.y; t.z += x.z; t.w += x.w;
    }
    float4 a = acc[j];
    a.x += scale * t.x; a.y += scale * t.y; a.z += scale * t.z; a.w += scale * t.w;
    acc[j] = a;
    if constexpr (CLEAR) {
      for (int q = 0; q < c.world; ++q) src[(size_t)q * sstride4 + j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}

__global__ void barrier_kernel(CommCtx c) {
  const uint32_t e = next_epoch(c);
  block_barrier(c, 2 * e);
  block_barrier(c, 2 * e + 1);
}

// Waits on a signal-pad slot that no peer writes; returns once the deadline passes.
__global__ void wait_unsignalled_kernel(CommCtx c, uint64_t timeout_ns) {
  if (threadIdx.x != 0) return;
  const uint32_t* slot =
      reinterpret_cast<const uint32_t*>(c.pads[c.rank]) + (kCommMaxBlocks - 1) * kCommMaxWorld + (kCommMaxWorld - 1);
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_sys(slot) != 0xFFFFFFFFu) {
    if (globaltimer_ns() - t0 > timeout_ns) {
      report_error(c.errs, kErrCommWait, -1);
      return;
    }
  }
}

__global__ void pace_begin_kernel(uint64_t* state, int slot) {
  if (threadIdx.x == 0) state[1 + slot] = globaltimer_ns();
}

// One thread books the link with a compare-and-swap on state[0], then sleeps until the booking ends.
__global__ void pace_end_kernel(uint64_t* state, int slot, uint64_t cost_ns, uint64_t timeout_ns,
                                DeviceErrors* errs) {
  if (threadIdx.x != 0) return;
  auto* link = reinterpret_cast<unsigned long long*>(state);
  const uint64_t stamp = *reinterpret_cast<volatile uint64_t*>(state + 1 + slot);
  unsigned long long seen = *reinterpret_cast<volatile unsigned long long*>(link);
  unsigned long long done;
  while (true) {
    done = (unsigned long long)max((uint64_t)seen, stamp) + cost_ns;
    const unsigned long long prev = atomicCAS(link, seen, done);
    if (prev == seen) break;
    seen = prev;
  }
  const uint64_t t0 = globaltimer_ns();
  if (done > t0 && done - t0 > timeout_ns) {  // a booking beyond the bound: report it instead of waiting
    report_error(errs, kErrPaceWait, slot);
    return;
  }
  for (uint64_t now = t0; now < done; now = globaltimer_ns()) {
    if (now - t0 > timeout_ns) {
      report_error(errs, kErrPaceWait, slot);
      return;
    }
    __nanosleep(done - now > 20000 ? 10000u : 500u);
  }
}

void check_ctx(const CommCtx& c) {
  B200_CHECK(c.world >= 1 && c.world <= kCommMaxWorld, "comm: world size out of range");
  B200_CHECK(c.blocks >= 1 && c.blocks < kCommMaxBlocks, "comm: block count out of range");
}

}  // namespace

// All collectives of one communicator use the same grid size (c.blocks) so that per-block epochs
// advance identically on every rank whatever the message size.
void comm_allreduce_f32(const CommCtx& c, size_t off, size_t n, float scale, cudaStream_t s) {
  check_ctx(c);
  B200_CHECK(n % 4 == 0 && off % 16 == 0, "comm_allreduce_f32: n must be a multiple of 4 and offset 16-aligned");
  if (c.mc)
    allreduce_f32_kernel<true><<<c.blocks, kThreads, 0, s>>>(c, off, n / 4, scale);
  else
    allreduce_f32_kernel<false><<<c.blocks, kThreads, 0, s>>>(c, off, n / 4, scale);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void comm_reduce_scatter_acc_f32(const CommCtx& c, size_t off, size_t chunk, float* acc, float scale, cudaStream_t s) {
  check_ctx(c);
  B200_CHECK(chunk % 4 == 0 && off % 16 == 0 && (reinterpret_cast<uintptr_t>(acc) & 15) == 0,
             "comm_reduce_scatter: chunk must be a multiple of 4, offset and acc 16-aligned");
  auto* a4 = reinterpret_cast<float4*>(acc);
  if (c.mc)
    reduce_scatter_acc_f32_kernel<true><<<c.blocks, kThreads, 0, s>>>(c, off, chunk / 4, a4, scale);
  else
    reduce_scatter_acc_f32_kernel<false><<<c.blocks, kThreads, 0, s>>>(c, off, chunk / 4, a4, scale);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void comm_reduce_scatter_range_acc_f32(const CommCtx& c, size_t off, size_t lo, size_t hi, float* acc, float scale,
                                       int blocks, cudaStream_t s) {
  check_ctx(c);
  // Fewer blocks than the communicator's grid are allowed (every rank must pass the same count):
  // the blocks left out simply skip this call's epochs on all ranks.
  const int grid = (blocks > 0 && blocks < c.blocks) ? blocks : c.blocks;
  B200_CHECK(lo % 4 == 0 && hi % 4 == 0 && off % 16 == 0 && (reinterpret_cast<uintptr_t>(acc) & 15) == 0,
             "comm_reduce_scatter_range: range ends must be multiples of 4, offset and acc 16-aligned");
  auto* a4 = reinterpret_cast<float4*>(acc);
  if (c.mc)
    reduce_scatter_range_acc_f32_kernel<true><<<grid, kThreads, 0, s>>>(c, off, lo / 4, hi / 4, a4, scale);
  else
    reduce_scatter_range_acc_f32_kernel<false><<<grid, kThreads, 0, s>>>(c, off, lo / 4, hi / 4, a4, scale);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void comm_allreduce_bf16(const CommCtx& c, size_t off, size_t n, float scale, cudaStream_t s) {
  check_ctx(c);
  B200_CHECK(n % 8 == 0 && off % 16 == 0, "comm_allreduce_bf16: n must be a multiple of 8 and offset 16-aligned");
  if (c.mc)
    allreduce_bf16_kernel<true><<<c.blocks, kThreads, 0, s>>>(c, off, n / 8, scale);
  else
    allreduce_bf16_kernel<false><<<c.blocks, kThreads, 0, s>>>(c, off, n / 8, scale);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void comm_reduce_scatter_acc_bf16(const CommCtx& c, size_t off, size_t chunk, float* acc, float scale,
                                  cudaStream_t s) {
  check_ctx(c);
  B200_CHECK(chunk % 8 == 0 && off % 16 == 0 && (reinterpret_cast<uintptr_t>(acc) & 15) == 0,
             "comm_reduce_scatter_bf16: chunk must be a multiple of 8, offset and acc 16-aligned");
  if (c.mc)
    reduce_scatter_acc_bf16_kernel<true><<<c.blocks, kThreads, 0, s>>>(c, off, chunk / 8, acc, scale);
  else
    reduce_scatter_acc_bf16_kernel<false><<<c.blocks, kThreads, 0, s>>>(c, off, chunk / 8, acc, scale);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void comm_allgather(const CommCtx& c, size_t off, size_t chunk_bytes, const void* shard, cudaStream_t s) {
  check_ctx(c);
  B200_CHECK(chunk_bytes % 16 == 0 && off % 16 == 0 && (reinterpret_cast<uintptr_t>(shard) & 15) == 0,
             "comm_allgather: 16-byte granularity required");
  const auto* src = reinterpret_cast<const uint4*>(shard);
  if (c.mc)
    allgather_kernel<true><<<c.blocks, kThreads, 0, s>>>(c, off, chunk_bytes / 16, src);
  else
    allgather_kernel<false><<<c.blocks, kThreads, 0, s>>>(c, off, chunk_bytes / 16, src);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void comm_gather_ce(const CommCtx& c, size_t off, size_t chunk_bytes, void* dst, cudaStream_t s) {
  check_ctx(c);
  // Start with the next rank so that at any moment the W ranks read from W different peers.
  for (int i = 0; i < c.world; ++i) {
    const int r = (c.rank + 1 + i) % c.world;
    const void* src = reinterpret_cast<const void*>(c.peers[r] + off);
    B200_CUDA_CHECK(cudaMemcpyAsync(static_cast<char*>(dst) + (size_t)r * chunk_bytes, src, chunk_bytes,
                                    cudaMemcpyDeviceToDevice, s));
  }
}

void comm_adamw_allgather(const CommCtx& c, size_t param_off, size_t chunk, float* master, float* m, float* v,
                          const float* grad, const float* scale_ptr, float scale_const, float lr, float beta1,
                          float beta2, float eps, float wd, int step, cudaStream_t s, const float* dev_sc) {
  check_ctx(c);
  B200_CHECK(chunk % 8 == 0 && param_off % 16 == 0, "comm_adamw_allgather: chunk must be a multiple of 8");
  AdamScalars a;
  a.lr = lr;
  a.beta1 = beta1;
  a.beta2 = beta2;
  a.eps = eps;
  a.decay = 1.0f - lr * wd;
  a.step = (float)(lr / (1.0 - std::pow((double)beta1, (double)step)));
  a.inv_sqrt_bc2 = (float)(1.0 / std::sqrt(1.0 - std::pow((double)beta2, (double)step)));
  a.scale_const = scale_const;
  auto* M = reinterpret_cast<float4*>(master);
  auto* Mm = reinterpret_cast<float4*>(m);
  auto* Vv = reinterpret_cast<float4*>(v);
  auto* G = reinterpret_cast<const float4*>(grad);
  if (c.mc)
    adamw_allgather_kernel<true><<<c.blocks, kThreads, 0, s>>>(c, param_off, chunk / 8, M, Mm, Vv, G, scale_ptr, a,
                                                                dev_sc);
  else
    adamw_allgather_kernel<false><<<c.blocks, kThreads, 0, s>>>(c, param_off, chunk / 8, M, Mm, Vv, G, scale_ptr, a,
                                                                 dev_sc);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void comm_rs_adamw_allgather(const CommCtx& c, const CommCtx& g, size_t g_off, size_t param_off, size_t chunk,
                             float* master, float* m, float* v, float grad_scale, float lr, float beta1, float beta2,
                             float eps, float wd, int step, const float* dev_sc, float* sq_out, cudaStream_t s) {
  check_ctx(c);
  check_ctx(g);
  B200_CHECK(c.world == g.world && c.rank == g.rank, "comm_rs_adamw_allgather: contexts of different groups");
  B200_CHECK((c.mc != 0) == (g.mc != 0), "comm_rs_adamw_allgather: both buffers multicast or neither");
  B200_CHECK(chunk % 8 == 0 && param_off % 16 == 0 && g_off % 16 == 0,
             "comm_rs_adamw_allgather: chunk must be a multiple of 8, offsets 16-aligned");
  B200_CHECK(((reinterpret_cast<uintptr_t>(master) | reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v)) &
              15) == 0,
             "comm_rs_adamw_allgather: optimizer state must be 16-byte aligned");
  AdamScalars a;
  a.lr = lr;
  a.beta1 = beta1;
  a.beta2 = beta2;
  a.eps = eps;
  a.decay = 1.0f - lr * wd;
  a.step = (float)(lr / (1.0 - std::pow((double)beta1, (double)step)));
  a.inv_sqrt_bc2 = (float)(1.0 / std::sqrt(1.0 - std::pow((double)beta2, (double)step)));
  a.scale_const = 1.0f;
  if (sq_out != nullptr) B200_CUDA_CHECK(cudaMemsetAsync(sq_out, 0, sizeof(float), s));
  auto* M = reinterpret_cast<float4*>(master);
  auto* Mm = reinterpret_cast<float4*>(m);
  auto* Vv = reinterpret_cast<float4*>(v);
  if (c.mc)
    rs_adamw_allgather_kernel<true><<<c.blocks, kThreads, 0, s>>>(c, g, g_off, param_off, chunk / 8, M, Mm, Vv,
                                                                  grad_scale, a, dev_sc, sq_out);
  else
    rs_adamw_allgather_kernel<false><<<c.blocks, kThreads, 0, s>>>(c, g, g_off, param_off, chunk / 8, M, Mm, Vv,
                                                                   grad_scale, a, dev_sc, sq_out);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void comm_routed_add(const float* src, size_t n, long long flat0, const RouteTable& t, DeviceErrors* errs,
                     cudaStream_t s) {
  B200_CHECK(t.world >= 1 && t.world <= kCommMaxWorld, "routed_add: 1..8 ranks");
  B200_CHECK(t.chunk > 0 && t.chunk % 4 == 0 && flat0 % 4 == 0 && flat0 >= 0,
             "routed_add: shard size and flat offset must be multiples of 4");
  B200_CHECK((reinterpret_cast<uintptr_t>(src) & 15) == 0, "routed_add: source must be 16-byte aligned");
  B200_CHECK(flat0 + (long long)n <= t.chunk * (long long)t.world, "routed_add: elements outside the sharded space");
  for (int r = 0; r < t.world; ++r)
    B200_CHECK(t.base[r] != 0 && t.base[r] % 16 == 0, "routed_add: shard bases must be 16-byte aligned");
  if (n == 0) return;
  const size_t work = std::max<size_t>(1, n / 4);
  const int blocks = (int)std::min<size_t>((work + kThreads - 1) / kThreads, 4 * 148);
  routed_add_kernel<<<blocks, kThreads, 0, s>>>(reinterpret_cast<const float4*>(src), n, flat0, t, errs);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void comm_embedding_bwd_routed(const int64_t* ids, const void* dy, int rows, int d, int vocab, long long flat0,
                               const RouteTable& t, DeviceErrors* errs, cudaStream_t s) {
  B200_CHECK(t.world >= 1 && t.world <= kCommMaxWorld, "embedding_bwd_routed: 1..8 ranks");
  B200_CHECK(d % 8 == 0 && flat0 % 4 == 0 && t.chunk > 0 && t.chunk % 4 == 0,
             "embedding_bwd_routed: d must be a multiple of 8, flat offset and shard size of 4");
  B200_CHECK(flat0 + (long long)vocab * d <= t.chunk * (long long)t.world,
             "embedding_bwd_routed: the table lies outside the sharded flat space");
  B200_CHECK((reinterpret_cast<uintptr_t>(dy) & 15) == 0, "embedding_bwd_routed: dy must be 16-byte aligned");
  for (int r = 0; r < t.world; ++r)
    B200_CHECK(t.base[r] != 0 && t.base[r] % 16 == 0, "embedding_bwd_routed: shard bases must be 16-byte aligned");
  const size_t total = (size_t)rows * (d / 8);
  if (total == 0) return;
  const int blocks = (int)std::min<size_t>((total + kThreads - 1) / kThreads, 4 * 148);
  embedding_bwd_routed_kernel<<<blocks, kThreads, 0, s>>>(ids, reinterpret_cast<const uint4*>(dy), rows, d, vocab,
                                                          flat0, t, errs);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void comm_bucket_reduce(const CommCtx& c, size_t off, size_t part, float* acc, float scale, int blocks,
                        cudaStream_t s) {
  check_ctx(c);
  B200_CHECK(part % 4 == 0 && off % 16 == 0 && (reinterpret_cast<uintptr_t>(acc) & 15) == 0,
             "bucket_reduce: slice length must be a multiple of 4, offset and acc 16-aligned");
  const int grid = (blocks > 0 && blocks < c.blocks) ? blocks : c.blocks;
  auto* a4 = reinterpret_cast<float4*>(acc);
  if (c.mc)
    bucket_reduce_kernel<true><<<grid, kThreads, 0, s>>>(c, off, part / 4, a4, scale);
  else
    bucket_reduce_kernel<false><<<grid, kThreads, 0, s>>>(c, off, part / 4, a4, scale);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void comm_adamw_allgather_seg(const CommCtx& c, const RingSeg* segs, int nseg, size_t total, float* master, float* m,
                              float* v, const float* grad, const float* scale_ptr, float scale_const, float lr,
                              float beta1, float beta2, float eps, float wd, int step, cudaStream_t s,
                              const float* dev_sc) {
  check_ctx(c);
  B200_CHECK(total % 8 == 0 && nseg >= 1, "adamw_allgather_seg: shard length must be a multiple of 8");
  B200_CHECK(((reinterpret_cast<uintptr_t>(master) | reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v) |
               reinterpret_cast<uintptr_t>(grad)) & 15) == 0,
             "adamw_allgather_seg: optimizer state and gradient must be 16-byte aligned");
  AdamScalars a;
  a.lr = lr;
  a.beta1 = beta1;
  a.beta2 = beta2;
  a.eps = eps;
  a.decay = 1.0f - lr * wd;
  a.step = (float)(lr / (1.0 - std::pow((double)beta1, (double)step)));
  a.inv_sqrt_bc2 = (float)(1.0 / std::sqrt(1.0 - std::pow((double)beta2, (double)step)));
  a.scale_const = scale_const;
  auto* M = reinterpret_cast<float4*>(master);
  auto* Mm = reinterpret_cast<float4*>(m);
  auto* Vv = reinterpret_cast<float4*>(v);
  auto* G = reinterpret_cast<const float4*>(grad);
  if (c.mc)
    adamw_allgather_seg_kernel<true><<<c.blocks, kThreads, 0, s>>>(c, segs, nseg, total / 8, M, Mm, Vv, G, scale_ptr,
                                                                    a, dev_sc);
  else
    adamw_allgather_seg_kernel<false><<<c.blocks, kThreads, 0, s>>>(c, segs, nseg, total / 8, M, Mm, Vv, G,
                                                                     scale_ptr, a, dev_sc);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void comm_push_reduce_scatter_f32(const CommCtx& c, float* src, size_t src_stride, size_t land_off, size_t part,
                                  float* acc, float scale, bool clear_src, cudaStream_t s) {
  check_ctx(c);
  B200_CHECK(part % 4 == 0 && src_stride % 4 == 0 && src_stride >= part && land_off % 16 == 0 &&
                 ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(acc)) & 15) == 0,
             "push_reduce_scatter: slice a multiple of 4 elements, landing offset, src and acc 16-aligned");
  auto* s4 = reinterpret_cast<float4*>(src);
  auto* a4 = reinterpret_cast<float4*>(acc);
  if (clear_src)
    push_rs_f32_kernel<true><<<c.blocks, kThreads, 0, s>>>(c, s4, src_stride / 4, land_off, part / 4, a4, scale);
  else
    push_rs_f32_kernel<false><<<c.blocks, kThreads, 0, s>>>(c, s4, src_stride / 4, land_off, part / 4, a4, scale);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void comm_barrier(const CommCtx& c, cudaStream_t s) {
  check_ctx(c);
  barrier_kernel<<<c.blocks, 32, 0, s>>>(c);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void comm_pace_begin(uint64_t* state, int slot, cudaStream_t s) {
  B200_CHECK(slot >= 0 && slot < kPaceSlots, "comm_pace_begin: slot out of range");
  pace_begin_kernel<<<1, 32, 0, s>>>(state, slot);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void comm_pace_end(uint64_t* state, int slot, uint64_t cost_ns, uint64_t timeout_ns, DeviceErrors* errs,
                   cudaStream_t s) {
  B200_CHECK(slot >= 0 && slot < kPaceSlots, "comm_pace_end: slot out of range");
  pace_end_kernel<<<1, 32, 0, s>>>(state, slot, cost_ns, timeout_ns, errs);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

void comm_wait_unsignalled(const CommCtx& c, uint64_t timeout_ns, cudaStream_t s) {
  wait_unsignalled_kernel<<<1, 32, 0, s>>>(c, timeout_ns);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

}  // namespace b200
