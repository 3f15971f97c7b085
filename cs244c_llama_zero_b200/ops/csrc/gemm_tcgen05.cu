// Persistent, warp-specialised bf16 GEMM on the 5th-generation tensor cores (sm_100a).
//
//   C[M, N] (op)= sum_k A(m, k) * B(n, k)         fp32 accumulation in tensor memory
//
// Structure (one CTA per SM, 320 threads):
//   warp 0      : TMA producer. Loads A (128 x 64) and B (BN x 64) bf16 tiles per k-block into a
//                 STAGES-deep shared-memory ring (128-byte swizzle, no multicast).
//   warp 1      : allocates 2*BN tensor-memory columns (double-buffered accumulator); lane 0 issues
//                 tcgen05.mma (M=128, N=BN, K=16) and tcgen05.commit to release smem stages and to
//                 hand a finished accumulator to the epilogue.
//   warps 2..9  : epilogue, two warpgroups splitting the tile columns. tcgen05.ld the accumulator
//                 (one row per thread), apply the fused operation, write to global memory,
//                 release the accumulator buffer.
// The epilogue of tile t overlaps the main loop of tile t+1.  Operands may be K-major or
// MN-major (the descriptor's major bit), so forward, data-gradient and weight-gradient GEMMs of a
// row-major nn.Linear weight all run without transposes.
//
// Fused epilogues:
//   EPI_STORE       C = acc (bf16)
//   EPI_RESIDUAL    C = R + acc (bf16)                          (o_proj / down_proj + residual)
//   EPI_ROPE        rotate-half RoPE on columns < rope_cols     (fused q|k|v projection)
//   EPI_SWIGLU      B tile = [gate rows | up rows]; C = silu(g)*u, aux = [g | u]
//   EPI_SWIGLU_BWD  acc = dA; reads [g | u]; C = [dG | dU]      (down_proj data gradient)
//   EPI_ACC_F32     C32 += acc (fp32 atomics; split-K)          (weight gradients into main_grad)
//
// Every mbarrier wait is bounded (see common.cuh); a CTA whose wait expires records an error
// and unwinds, releasing its tensor memory.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "gemm.h"

namespace b200 {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int A_STAGE_BYTES = BM * BK * 2;
constexpr int NUM_THREADS = 320;

template <int BN>
struct GemmCfg {
  static constexpr int B_STAGE_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + __expf(-g)); }

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr uint32_t IDESC = idesc_bf16_f32(BM, BN, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 8);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  const int total_units = p.tiles_m * p.tiles_n * p.splits;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        const int split = u % p.splits;
        const int tile = u / p.splits;
        const int tm = tile % p.tiles_m, tn = tile / p.tiles_m;
        const int m0 = tm * BM;
        const int kb0 = split * p.k_blocks_per_split;
        const int kb1 = min(p.total_k_blocks, kb0 + p.k_blocks_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, abort_flag, p.errs, kErrGemmWait, 0)) {
            ok = false;
            break;
          }
          uint8_t* sA = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sB = sA + A_STAGE_BYTES;
          mbar_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
          const int k0 = kb * BK;
          if constexpr (!A_MN) {
            tma_load_2d(sA, &tmA, &full_bar[stage], k0, m0);
          } else {
            tma_load_2d(sA, &tmA, &full_bar[stage], m0, k0);
            tma_load_2d(sA + 8192, &tmA, &full_bar[stage], m0 + 64, k0);
          }
          if constexpr (EPI == EPI_SWIGLU) {
            const int g0 = tn * (BN / 2);
            tma_load_2d(sB, &tmB, &full_bar[stage], k0, g0);
            tma_load_2d(sB + (BN / 2) * 128, &tmB, &full_bar[stage], k0, p.ffn + g0);
          } else if constexpr (!B_MN) {
            tma_load_2d(sB, &tmB, &full_bar[stage], k0, tn * BN);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(sB + j * 8192, &tmB, &full_bar[stage], tn * BN + 64 * j, k0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int t = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x, ++t) {
        const int split = u % p.splits;
        const int kb0 = split * p.k_blocks_per_split;
        const int kb1 = min(p.total_k_blocks, kb0 + p.k_blocks_per_split);
        const int acc = t & 1;
        const uint32_t acc_phase = (t >> 1) & 1;
        if (!mbar_wait_bounded(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, p.errs, kErrGemmWait, 1)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase, abort_flag, p.errs, kErrGemmWait, 2)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_STAGE_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = A_MN ? smem_desc_sw128(a_addr + k * 2048, 8192, 1024)
                                        : smem_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? smem_desc_sw128(b_addr + k * 2048, 8192, 1024)
                                        : smem_desc_sw128(b_addr + k * 32, 16, 1024);
            tc_mma_f16(d_tmem, adesc, bdesc, IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&tfull_bar[acc]);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue warps
    const int q = warp & 3;  // tensor-memory lane quarter this warp may access
    const int wg = (warp - 2) >> 2;  // epilogue warpgroup: columns [wg*BN/2, (wg+1)*BN/2)
    const int row = q * 32 + lane;
    int t = 0;
    for (int u = blockIdx.x; u < total_units; u += gridDim.x, ++t) {
      const int tile = u / p.splits;
      const int tm = tile % p.tiles_m, tn = tile / p.tiles_m;
      const int acc = t & 1;
      const uint32_t acc_phase = (t >> 1) & 1;
      if (!mbar_wait_bounded(&tfull_bar[acc], acc_phase, abort_flag, p.errs, kErrGemmWait, 3)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      const int m = tm * BM + row;
      const bool row_ok = m < p.M;

      if constexpr (EPI == EPI_STORE || EPI == EPI_RESIDUAL || EPI == EPI_ACC_F32) {
        const int n0 = tn * BN;
#pragma unroll 1
        for (int c = wg * (BN / 2); c < (wg + 1) * (BN / 2); c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c, r);
          tc_wait_ld();
          if (!row_ok) continue;
          const int nb = n0 + c;
          if constexpr (EPI == EPI_ACC_F32) {
            float* dst = p.C32 + (size_t)m * p.ldc32 + nb;
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              if (nb + j < p.N) {
                float4 v = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                                       __uint_as_float(r[j + 3]));
                atomicAdd(reinterpret_cast<float4*>(dst + j), v);
              }
            }
          } else {
            __nv_bfloat16* dst = p.C + (size_t)m * p.ldc + nb;
            const __nv_bfloat16* res = (EPI == EPI_RESIDUAL) ? p.R + (size_t)m * p.ldr + nb : nullptr;
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              if (nb + j >= p.N) break;
              float v[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(r[j + e]);
              if constexpr (EPI == EPI_RESIDUAL) {
                uint4 rv = *reinterpret_cast<const uint4*>(res + j);
                const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  v[2 * e] += bf16lo(rw[e]);
                  v[2 * e + 1] += bf16hi(rw[e]);
                }
              }
              uint4 o;
              o.x = pack_bf16(v[0], v[1]);
              o.y = pack_bf16(v[2], v[3]);
              o.z = pack_bf16(v[4], v[5]);
              o.w = pack_bf16(v[6], v[7]);
              *reinterpret_cast<uint4*>(dst + j) = o;
            }
          }
        }
      } else if constexpr (EPI == EPI_ROPE) {
        const int n0 = tn * BN;
        const int half = p.head_dim >> 1;
        const int pos = row_ok ? (m % p.seq_len) : 0;
#pragma unroll 1
        for (int h0 = wg * (BN / 2); h0 < (wg + 1) * (BN / 2); h0 += p.head_dim) {
          const int col = n0 + h0;
          const bool rotate = col < p.rope_cols;
#pragma unroll 1
          for (int j = 0; j < half; j += 32) {
            uint32_t lo[32], hi[32];
            tmem_ld_32x32b_x32(tbase + h0 + j, lo);
            tmem_ld_32x32b_x32(tbase + h0 + half + j, hi);
            tc_wait_ld();
            if (!row_ok || col >= p.N) continue;
            __nv_bfloat16* dlo = p.C + (size_t)m * p.ldc + col + j;
            __nv_bfloat16* dhi = dlo + half;
            const float* cs = p.rope_cos + (size_t)pos * half + j;
            const float* sn = p.rope_sin + (size_t)pos * half + j;
#pragma unroll
            for (int e = 0; e < 32; e += 8) {
              float a[8], b[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float x0 = __uint_as_float(lo[e + i]);
                const float x1 = __uint_as_float(hi[e + i]);
                if (rotate) {
                  const float c = cs[e + i], s = sn[e + i];
                  a[i] = x0 * c - x1 * s;
                  b[i] = x1 * c + x0 * s;
                } else {
                  a[i] = x0;
                  b[i] = x1;
                }
              }
              uint4 oa, ob;
              oa.x = pack_bf16(a[0], a[1]); oa.y = pack_bf16(a[2], a[3]);
              oa.z = pack_bf16(a[4], a[5]); oa.w = pack_bf16(a[6], a[7]);
              ob.x = pack_bf16(b[0], b[1]); ob.y = pack_bf16(b[2], b[3]);
              ob.z = pack_bf16(b[4], b[5]); ob.w = pack_bf16(b[6], b[7]);
              *reinterpret_cast<uint4*>(dlo + e) = oa;
              *reinterpret_cast<uint4*>(dhi + e) = ob;
            }
          }
        }
      } else if constexpr (EPI == EPI_SWIGLU) {
        const int n0 = tn * (BN / 2);
#pragma unroll 1
        for (int c = wg * (BN / 4); c < (wg + 1) * (BN / 4); c += 32) {
          uint32_t g[32], uu[32];
          tmem_ld_32x32b_x32(tbase + c, g);
          tmem_ld_32x32b_x32(tbase + BN / 2 + c, uu);
          tc_wait_ld();
          const int nb = n0 + c;
          if (!row_ok || nb >= p.N) continue;
          __nv_bfloat16* dh = p.C + (size_t)m * p.ldc + nb;
          __nv_bfloat16* dg = p.aux + (size_t)m * p.ld_aux + nb;
          __nv_bfloat16* du = dg + p.ffn;
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            float hv[8], gv[8], uv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              gv[i] = __uint_as_float(g[j + i]);
              uv[i] = __uint_as_float(uu[j + i]);
              hv[i] = silu_f(gv[i]) * uv[i];
            }
            uint4 oh, og, ou;
            oh.x = pack_bf16(hv[0], hv[1]); oh.y = pack_bf16(hv[2], hv[3]);
            oh.z = pack_bf16(hv[4], hv[5]); oh.w = pack_bf16(hv[6], hv[7]);
            og.x = pack_bf16(gv[0], gv[1]); og.y = pack_bf16(gv[2], gv[3]);
            og.z = pack_bf16(gv[4], gv[5]); og.w = pack_bf16(gv[6], gv[7]);
            ou.x = pack_bf16(uv[0], uv[1]); ou.y = pack_bf16(uv[2], uv[3]);
            ou.z = pack_bf16(uv[4], uv[5]); ou.w = pack_bf16(uv[6], uv[7]);
            *reinterpret_cast<uint4*>(dh + j) = oh;
            *reinterpret_cast<uint4*>(dg + j) = og;
            *reinterpret_cast<uint4*>(du + j) = ou;
          }
        }
      } else if constexpr (EPI == EPI_SWIGLU_BWD) {
        const int n0 = tn * BN;
#pragma unroll 1
        for (int c = wg * (BN / 2); c < (wg + 1) * (BN / 2); c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c, r);
          tc_wait_ld();
          const int nb = n0 + c;
          if (!row_ok || nb >= p.N) continue;
          const __nv_bfloat16* gsrc = p.aux_in + (size_t)m * p.ld_aux_in + nb;
          const __nv_bfloat16* usrc = gsrc + p.ffn;
          __nv_bfloat16* dg = p.C + (size_t)m * p.ldc + nb;
          __nv_bfloat16* du = dg + p.ffn;
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            const uint4 gq = *reinterpret_cast<const uint4*>(gsrc + j);
            const uint4 uq = *reinterpret_cast<const uint4*>(usrc + j);
            const uint32_t gw[4] = {gq.x, gq.y, gq.z, gq.w};
            const uint32_t uw[4] = {uq.x, uq.y, uq.z, uq.w};
            float dgv[8], duv[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const float gval = h ? bf16hi(gw[i]) : bf16lo(gw[i]);
                const float uval = h ? bf16hi(uw[i]) : bf16lo(uw[i]);
                const float da = __uint_as_float(r[j + 2 * i + h]);
                const float sig = 1.0f / (1.0f + __expf(-gval));
                const float s = gval * sig;
                duv[2 * i + h] = da * s;
                dgv[2 * i + h] = da * uval * sig * (1.0f + gval * (1.0f - sig));
              }
            }
            uint4 og, ou;
            og.x = pack_bf16(dgv[0], dgv[1]); og.y = pack_bf16(dgv[2], dgv[3]);
            og.z = pack_bf16(dgv[4], dgv[5]); og.w = pack_bf16(dgv[6], dgv[7]);
            ou.x = pack_bf16(duv[0], duv[1]); ou.y = pack_bf16(duv[2], duv[3]);
            ou.z = pack_bf16(duv[4], duv[5]); ou.w = pack_bf16(duv[6], duv[7]);
            *reinterpret_cast<uint4*>(dg + j) = og;
            *reinterpret_cast<uint4*>(du + j) = ou;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qres;
    B200_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qres));
    B200_CHECK(ptr != nullptr && qres == cudaDriverEntryPointSuccess, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

}  // namespace

CUtensorMap make_tmap_bf16_2d(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                              uint32_t box_inner, uint32_t box_outer) {
  B200_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base address must be 16-byte aligned");
  B200_CHECK((row_stride_elems * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                               box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  B200_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
  return map;
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    B200_CUDA_CHECK(cudaGetDevice(&dev));
    B200_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

template <int BN, bool A_MN, bool B_MN, int EPI>
static void launch_impl(const GemmOperands& op, GemmParams p, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  auto kernel = gemm_kernel<BN, A_MN, B_MN, EPI>;
  static bool configured = false;
  if (!configured) {
    B200_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES));
    configured = true;
  }
  // A operand: K-major -> global [M, K] (K contiguous); MN-major -> global [K, M] (M contiguous).
  CUtensorMap tmA = A_MN ? make_tmap_bf16_2d(op.A, (uint64_t)p.M, (uint64_t)p.K, op.lda, 64, 64)
                         : make_tmap_bf16_2d(op.A, (uint64_t)p.K, (uint64_t)p.M, op.lda, 64, BM);
  CUtensorMap tmB;
  if (EPI == EPI_SWIGLU) {
    tmB = make_tmap_bf16_2d(op.B, (uint64_t)p.K, (uint64_t)(2 * p.ffn), op.ldb, 64, BN / 2);
  } else if (B_MN) {
    tmB = make_tmap_bf16_2d(op.B, (uint64_t)p.N, (uint64_t)p.K, op.ldb, 64, 64);
  } else {
    tmB = make_tmap_bf16_2d(op.B, (uint64_t)p.K, (uint64_t)p.N, op.ldb, 64, BN);
  }
  const int out_cols_per_tile = (EPI == EPI_SWIGLU) ? BN / 2 : BN;
  p.tiles_m = (p.M + BM - 1) / BM;
  p.tiles_n = (p.N + out_cols_per_tile - 1) / out_cols_per_tile;
  p.total_k_blocks = (p.K + BK - 1) / BK;
  if (p.splits < 1) p.splits = 1;
  p.splits = std::min(p.splits, p.total_k_blocks);
  p.k_blocks_per_split = (p.total_k_blocks + p.splits - 1) / p.splits;
  p.splits = (p.total_k_blocks + p.k_blocks_per_split - 1) / p.k_blocks_per_split;
  p.errs = device_errors_ptr();
  const int units = p.tiles_m * p.tiles_n * p.splits;
  const int grid = std::max(1, std::min(units, num_sms()));
  kernel<<<grid, NUM_THREADS, Cfg::SMEM_BYTES, stream>>>(tmA, tmB, p);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

template <bool A_MN, bool B_MN, int EPI>
static void dispatch_bn(int bn, const GemmOperands& op, const GemmParams& p, cudaStream_t stream) {
  if (bn == 256)
    launch_impl<256, A_MN, B_MN, EPI>(op, p, stream);
  else
    launch_impl<128, A_MN, B_MN, EPI>(op, p, stream);
}

void gemm_launch(const GemmOperands& op, GemmParams p, int epi, bool a_mn, bool b_mn, int bn, cudaStream_t stream) {
  B200_CHECK(bn == 128 || bn == 256, "BN must be 128 or 256");
  B200_CHECK(p.N % 8 == 0, "GEMM output width N must be a multiple of 8");
  B200_CHECK((a_mn || p.K % 8 == 0) && (b_mn || p.K % 8 == 0), "GEMM K must be a multiple of 8 for K-major operands");
  B200_CHECK(!a_mn || p.M % 8 == 0, "GEMM M must be a multiple of 8 for an MN-major A operand");
  if (!a_mn && !b_mn) {
    switch (epi) {
      case EPI_STORE: return dispatch_bn<false, false, EPI_STORE>(bn, op, p, stream);
      case EPI_RESIDUAL: return dispatch_bn<false, false, EPI_RESIDUAL>(bn, op, p, stream);
      case EPI_ROPE: return dispatch_bn<false, false, EPI_ROPE>(bn, op, p, stream);
      case EPI_SWIGLU: return dispatch_bn<false, false, EPI_SWIGLU>(bn, op, p, stream);
      case EPI_ACC_F32: return dispatch_bn<false, false, EPI_ACC_F32>(bn, op, p, stream);
    }
  } else if (!a_mn && b_mn) {
    switch (epi) {
      case EPI_STORE: return dispatch_bn<false, true, EPI_STORE>(bn, op, p, stream);
      case EPI_SWIGLU_BWD: return dispatch_bn<false, true, EPI_SWIGLU_BWD>(bn, op, p, stream);
      case EPI_ACC_F32: return dispatch_bn<false, true, EPI_ACC_F32>(bn, op, p, stream);
    }
  } else if (a_mn && b_mn) {
    switch (epi) {
      case EPI_ACC_F32: return dispatch_bn<true, true, EPI_ACC_F32>(bn, op, p, stream);
      case EPI_STORE: return dispatch_bn<true, true, EPI_STORE>(bn, op, p, stream);
    }
  }
  B200_CHECK(false, "unsupported GEMM operand-major / epilogue combination");
}

}  // namespace b200
