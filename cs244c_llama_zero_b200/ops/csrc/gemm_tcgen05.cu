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
//   EPI_ACC_F32_ROUTED  owner's shard += acc over NVLink          (weight gradient + reduce-scatter)
//
// Every mbarrier wait is bounded (see common.cuh); a CTA whose wait expires records an error
// and unwinds, releasing its tensor memory.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <string>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "gemm.h"

namespace b200 {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int A_STAGE_BYTES = BM * BK * 2;
constexpr int NUM_THREADS = 320;

constexpr int kEpiWarps = 8;
constexpr int kChunkBytes = 2048;  // epilogue staging chunk: 32 rows x 64 B (32 bf16 or 16 fp32 columns)

// CG = 1: one CTA computes a 128 x BN tile.  CG = 2: a CTA pair (cluster of 2) computes a 256 x BN
// tile with cta_group::2 MMAs; each CTA stages its own 128 rows of A and half (BN / 2 rows) of B.
template <int BN, int CG = 1>
struct GemmCfg {
  static constexpr int B_STAGE_BYTES = (BN / CG) * BK * 2;
  static constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
  static constexpr int STAGES = (CG == 2 || BN == 128) ? 6 : 4;
  static constexpr int TMEM_COLS = (BN == 128) ? 256 : 512;  // power of two >= 2 * BN
  static constexpr int STAGING_BYTES = kEpiWarps * 2 * kChunkBytes;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + STAGING_BYTES + 1024 /*align*/ + 512 /*barriers*/;
  static_assert(SMEM_BYTES <= 232448, "GEMM shared memory exceeds the 227 KB per-block limit");
};

// Fast division (the `__fdividef` intrinsic): the denominator 1 + e^-g is >= 1, and where it
// overflows the result is the limit 0 either way.
__device__ __forceinline__ float sigmoid_f(float g) { return __fdividef(1.0f, 1.0f + __expf(-g)); }
__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// Byte offset of 16-byte column group j of row `row` inside a staging chunk.  The TMA maps of the
// outputs use the 64-byte swizzle (16-byte group index XOR bits 1..2 of the row); the chunk base is
// 2 KB aligned, so this is the layout TMA reads, and a warp writing one row per lane hits 32
// distinct banks per quarter-warp.
__device__ __forceinline__ uint32_t chunk_off(int row, int j) { return row * 64 + ((j ^ ((row >> 1) & 3)) << 4); }

__device__ __forceinline__ uint4 pack8f(const float (&v)[8]) {
  return make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
}

// This lane's 32 fp32 values (bit patterns) -> 32 bf16 of its row in the chunk.
__device__ __forceinline__ void write_chunk_bf16(uint8_t* buf, const uint32_t (&r)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(r[8 * j + e]);
    *reinterpret_cast<uint4*>(buf + chunk_off(lane, j)) = pack8f(v);
  }
}

// Next chunk of this warp's two-deep ring, once the TMA store issued from it two chunks ago has
// finished reading it.
__device__ __forceinline__ uint8_t* acquire_chunk(uint8_t* stg, int& bsel) {
  if ((threadIdx.x & 31) == 0) bulk_wait_group_read<1>();
  __syncwarp();
  uint8_t* buf = stg + bsel * kChunkBytes;
  bsel ^= 1;
  return buf;
}

// Hand a filled chunk to TMA: store (or fp32 add-reduce) it at (column c0, row c1) of `map`.
__device__ __forceinline__ void publish_chunk(const CUtensorMap* map, uint8_t* buf, int c0, int c1, bool reduce) {
  fence_proxy_async_smem();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) {
    if (reduce)
      tma_reduce_add_2d(map, buf, c0, c1);
    else
      tma_store_2d(map, buf, c0, c1);
    bulk_commit_group();
  }
}

// One work unit: a (tile, K-range) of problem `prob` (always 0 outside grouped launches).
struct Unit {
  int prob, tm, tn, kb0, kb1;
};

// The k-th unit of CTA group g out of G: strided for single problems; boustrophedon for grouped
// launches, whose unit list runs from the longest units to the shortest.
template <bool GROUPED>
__device__ __forceinline__ int unit_index(int k, int g, int G) {
  if constexpr (GROUPED)
    return k * G + ((k & 1) ? (G - 1 - g) : g);
  else
    return g + k * G;
}

template <bool GROUPED>
__device__ __forceinline__ Unit decode_unit(int u, const GemmParams& p, const GemmParams& p1) {
  int prob = 0, v = u;
  if constexpr (GROUPED) {
    if (u < p.grp_units_first) {
      prob = p.grp_first;
    } else {
      prob = 1 - p.grp_first;
      v = u - p.grp_units_first;
    }
  }
  const int splits = prob ? p1.splits : p.splits;
  const int tiles_m = prob ? p1.tiles_m : p.tiles_m;
  const int kbs = prob ? p1.k_blocks_per_split : p.k_blocks_per_split;
  const int total_kb = prob ? p1.total_k_blocks : p.total_k_blocks;
  const int split = v % splits, tile = v / splits;
  Unit d;
  d.prob = prob;
  d.tm = tile % tiles_m;
  d.tn = tile / tiles_m;
  d.kb0 = split * kbs;
  d.kb1 = min(total_kb, d.kb0 + kbs);
  return d;
}

// GROUPED: problem 0 is described by the template (A_MN, EPI = EPI_STORE, maps tmA/tmB/tmC, params
// p) and problem 1 is a weight gradient (MN-major A, EPI_ACC_F32, maps tmX/tmY/tmZ, params p1); with
// ROUTE1 problem 1's partial sums go to their owners' shards instead (EPI_ACC_F32_ROUTED, p1.route_*).
template <int BN, bool A_MN, bool B_MN, int EPI, int CG, bool GROUPED = false, bool ROUTE1 = false>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmX,
                const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmZ,
                const __grid_constant__ GemmParams p, const __grid_constant__ GemmParams p1) {
  using Cfg = GemmCfg<BN, CG>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr uint32_t IDESC = idesc_bf16_f32(BM * CG, BN, A_MN, B_MN);
  constexpr uint32_t IDESC_AMN = idesc_bf16_f32(BM * CG, BN, true, B_MN);  // grouped problem 1
  static_assert(!GROUPED || (EPI == EPI_STORE && !A_MN && B_MN), "grouped launches pair a dgrad with a wgrad");
  static_assert(!ROUTE1 || GROUPED, "ROUTE1 applies to the grouped launch's weight gradient");
  static_assert(CG == 1 || CG == 2, "CTA group of 1 or 2");
  static_assert(CG == 1 || !B_MN || (BN / 2) % 64 == 0, "pair tiles with an MN-major B need BN/2 % 64 == 0");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES + Cfg::STAGING_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* load_bar = tempty_bar + 2;  // two per epilogue warp (residual tiles)
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(load_bar + 2 * kEpiWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Pair bookkeeping: `rank` 0 is the leader that issues the MMAs; units are dealt per pair.
  const int rank = (CG == 2) ? (int)cluster_ctarank() : 0;
  const int group_id = blockIdx.x / CG, n_groups = gridDim.x / CG;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], kEpiWarps * CG);  // both CTAs' epilogue warps release the pair accumulator
    }
    for (int b = 0; b < 2 * kEpiWarps; ++b) mbar_init(&load_bar[b], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (CG == 2) {
      tmem_alloc_pair(tmem_base_slot, Cfg::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_base_slot, Cfg::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_sync();  // the peer's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;
  pdl_wait_and_release();  // operands / outputs are shared with the previous kernels of the stream

  const int total_units = GROUPED ? p.grp_units_total : p.tiles_m * p.tiles_n * p.splits;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int ku = 0; ok; ++ku) {
        const int u = unit_index<GROUPED>(ku, group_id, n_groups);
        if (u >= total_units) break;
        const Unit d = decode_unit<GROUPED>(u, p, p1);
        const int tn = d.tn;
        const int m0 = d.tm * BM * CG + rank * BM;
        const bool p1u = GROUPED && d.prob == 1;
        const bool a_mn = GROUPED ? p1u : A_MN;
        const CUtensorMap* mapA = p1u ? &tmX : &tmA;
        const CUtensorMap* mapB = p1u ? &tmY : &tmB;
        for (int kb = d.kb0; kb < d.kb1; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, abort_flag, p.errs, kErrGemmWait, 0)) {
            ok = false;
            break;
          }
          uint8_t* sA = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sB = sA + A_STAGE_BYTES;
          const int k0 = kb * BK;
          // All of a stage's bytes (both CTAs of a pair) count on the leader's full barrier.
          if (rank == 0) mbar_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES * CG);
          const uint32_t fb = (CG == 2) ? leader_bar_addr(&full_bar[stage]) : 0u;
          auto load = [&](void* dst, const CUtensorMap* map, int c0, int c1) {
            if constexpr (CG == 2)
              tma_load_2d_pair(dst, map, fb, c0, c1);
            else
              tma_load_2d(dst, map, &full_bar[stage], c0, c1);
          };
          if (!a_mn) {
            load(sA, mapA, k0, m0);
          } else {
            load(sA, mapA, m0, k0);
            load(sA + 8192, mapA, m0 + 64, k0);
          }
          if constexpr (EPI == EPI_SWIGLU) {
            const int g0 = tn * (BN / 2);
            if constexpr (CG == 2) {
              load(sB, &tmB, k0, rank == 0 ? g0 : p.ffn + g0);  // leader: gate rows, peer: up rows
            } else {
              load(sB, &tmB, k0, g0);
              load(sB + (BN / 2) * 128, &tmB, k0, p.ffn + g0);
            }
          } else if constexpr (!B_MN) {
            load(sB, mapB, k0, tn * BN + rank * (BN / CG));
          } else {
#pragma unroll
            for (int j = 0; j < BN / CG / 64; ++j) load(sB + j * 8192, mapB, tn * BN + rank * (BN / CG) + 64 * j, k0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int t = 0;
      bool ok = true;
      for (int ku = 0; ok; ++ku, ++t) {
        const int u = unit_index<GROUPED>(ku, group_id, n_groups);
        if (u >= total_units) break;
        const Unit d = decode_unit<GROUPED>(u, p, p1);
        const int kb0 = d.kb0, kb1 = d.kb1;
        const bool a_mn = GROUPED ? d.prob == 1 : A_MN;
        const uint32_t idesc = GROUPED ? (a_mn ? IDESC_AMN : IDESC) : IDESC;
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
            const uint64_t adesc = a_mn ? smem_desc_sw128(a_addr + k * 2048, 8192, 1024)
                                        : smem_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? smem_desc_sw128(b_addr + k * 2048, 8192, 1024)
                                        : smem_desc_sw128(b_addr + k * 32, 16, 1024);
            if constexpr (CG == 2)
              tc_mma_f16_pair(d_tmem, adesc, bdesc, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
            else
              tc_mma_f16(d_tmem, adesc, bdesc, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          if constexpr (CG == 2)
            tc_commit_pair(&empty_bar[stage], 0x3);  // frees the stage in both CTAs
          else
            tc_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (CG == 2)
          tc_commit_pair(&tfull_bar[acc], 0x3);
        else
          tc_commit(&tfull_bar[acc]);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue warps
    // Warp (q, wg) owns tile rows [32q, 32q+32) and columns [wg*BN/2, (wg+1)*BN/2).  Results go
    // through this warp's two 2 KB staging chunks (32 rows x 64 B, 64-byte swizzle) and leave with
    // TMA stores (fp32 weight gradients: TMA add-reductions), so global writes are full-line and
    // asynchronous; the ring of two chunks lets the next chunk fill while the previous one drains.
    const int q = warp & 3;
    const int wg = (warp - 2) >> 2;
    const int ew = warp - 2;
    uint8_t* stg = smem + STAGES * Cfg::STAGE_BYTES + ew * 2 * kChunkBytes;
    uint64_t* lbar = load_bar + ew * 2;
    uint32_t lphase[2] = {0u, 0u};
    int bsel = 0;
    int t = 0;
    bool ok = true;
    for (int ku = 0; ok; ++ku, ++t) {
      const int u = unit_index<GROUPED>(ku, group_id, n_groups);
      if (u >= total_units) break;
      const Unit d = decode_unit<GROUPED>(u, p, p1);
      const int tm = d.tm, tn = d.tn;
      const int acc = t & 1;
      const uint32_t acc_phase = (t >> 1) & 1;
      const int row0 = tm * BM * CG + rank * BM + q * 32;  // TMA row coordinate of this warp's chunk
      const int m = row0 + lane;
      const bool row_ok = m < ((GROUPED && d.prob == 1) ? p1.M : p.M);

      if constexpr (EPI == EPI_RESIDUAL) {
        // Prefetch the residual for the first two chunks while the main loop still runs.
        if (lane == 0) {
          bulk_wait_group_read<0>();
          for (int i = 0; i < 2 && i < BN / 64; ++i) {
            mbar_expect_tx(&lbar[i], kChunkBytes);
            tma_load_2d(stg + i * kChunkBytes, &tmX, &lbar[i], tn * BN + wg * (BN / 2) + 32 * i, row0);
          }
        }
        __syncwarp();
      }
      // SwiGLU backward: saved pre-activations of this row for chunk i (64 B of g and of u), loaded
      // one chunk ahead; the first chunk's loads are issued before the accumulator wait so that
      // their latency overlaps the main loop.
      uint4 gq[4], uq[4];
      auto load_gu = [&](int i) {
        const int n0 = tn * BN + wg * (BN / 2);
        const size_t gidx = (size_t)(row_ok ? m : 0) * p.ld_aux_in + n0 + 32 * i;
        const __nv_bfloat16* gsrc = p.aux_in + gidx;
        const long long aux_extent = (long long)p.M * p.ld_aux_in;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const bool in = n0 + 32 * i + 8 * j < p.N;
          const bool gin = in && B200_IN_BOUNDS(p.errs, gidx + 8 * j, 8, aux_extent, 100);
          const bool uin = in && B200_IN_BOUNDS(p.errs, gidx + p.ffn + 8 * j, 8, aux_extent, 101);
          gq[j] = gin ? *reinterpret_cast<const uint4*>(gsrc + 8 * j) : make_uint4(0u, 0u, 0u, 0u);
          uq[j] = uin ? *reinterpret_cast<const uint4*>(gsrc + p.ffn + 8 * j) : make_uint4(0u, 0u, 0u, 0u);
        }
      };
      if constexpr (EPI == EPI_SWIGLU_BWD) {
        // The saved pre-activations were written long ago (forward pass) and sit in DRAM; each lane
        // reads its own row, so eight warps cannot hide the latency.  Pull this row's g and u slices
        // of the current (first unit) and the next tile into L2 while the main loop runs.
        auto prefetch_row = [&](int unit_k) {
          const int uu = unit_index<GROUPED>(unit_k, group_id, n_groups);
          if (uu >= total_units) return;
          const Unit dn = decode_unit<GROUPED>(uu, p, p1);
          const int rown = dn.tm * BM * CG + rank * BM + q * 32 + lane;
          if (rown >= p.M) return;
          const int col = dn.tn * BN + wg * (BN / 2);
          const __nv_bfloat16* src = p.aux_in + (size_t)rown * p.ld_aux_in + col;
#pragma unroll
          for (int b = 0; b < BN / 2; b += 64) {  // BN / 2 columns = BN bytes = BN / 128 lines
            if (col + b < p.N) {
              prefetch_l2(src + b);
              prefetch_l2(src + p.ffn + b);
            }
          }
        };
        if (ku == 0) prefetch_row(0);
        prefetch_row(ku + 1);
        load_gu(0);
      }
      if (!mbar_wait_bounded(&tfull_bar[acc], acc_phase, abort_flag, p.errs, kErrGemmWait, 3)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;

      // fp32 add-reduction of the accumulator (weight gradients; grouped problem 1)
      auto acc_f32_epilogue = [&](const CUtensorMap* map) {
        const int n0 = tn * BN + wg * (BN / 2);
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 16) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(tbase + wg * (BN / 2) + c, r);
          tc_wait_ld();
          uint8_t* buf = acquire_chunk(stg, bsel);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            *reinterpret_cast<uint4*>(buf + chunk_off(lane, j)) =
                make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
          publish_chunk(map, buf, n0 + c, row0, true);
        }
      };
      // Each 16-byte group of this row's partial sums goes to the rank owning it: the reduction across
      // ranks happens in the owners' memory as the tiles finish, so no reduce-scatter runs after
      // backward.  Groups never straddle owners (flat0, ld, chunk and the column are multiples of 4).
      auto routed_f32_epilogue = [&](const GemmParams& q) {
        const int n0 = tn * BN + wg * (BN / 2);
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 16) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(tbase + wg * (BN / 2) + c, r);
          tc_wait_ld();
          if (m < q.M) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int col = n0 + c + 4 * j;
              if (col >= q.N) continue;
              const long long f = q.route_flat0 + (long long)m * q.route_ld + col;
              const int owner = (int)(f / q.route_chunk);
              if (owner < 0 || owner >= q.route_world) {
                report_error(q.errs, kErrBadIndex, 200);
                continue;
              }
              float* dst = reinterpret_cast<float*>(q.route_base[owner]) + (f - (long long)owner * q.route_chunk);
              red_add_f32x4_sys(dst, r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
            }
          }
        }
      };
      if (GROUPED && d.prob == 1) {
        if constexpr (GROUPED && ROUTE1)
          routed_f32_epilogue(p1);
        else if constexpr (GROUPED)
          acc_f32_epilogue(&tmZ);
      } else if constexpr (EPI == EPI_STORE || EPI == EPI_RESIDUAL) {
        const int n0 = tn * BN + wg * (BN / 2);
#pragma unroll 1
        for (int i = 0; i < BN / 64; ++i) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + wg * (BN / 2) + 32 * i, r);
          tc_wait_ld();
          uint8_t* buf;
          if constexpr (EPI == EPI_RESIDUAL) {
            const int b = i & 1;
            buf = stg + b * kChunkBytes;
            if (!mbar_wait_bounded(&lbar[b], lphase[b], abort_flag, p.errs, kErrGemmWait, 4)) { ok = false; break; }
            lphase[b] ^= 1u;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint4 rv = *reinterpret_cast<const uint4*>(buf + chunk_off(lane, j));
              const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
              float v[8];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                v[2 * e] = __uint_as_float(r[8 * j + 2 * e]) + bf16lo(rw[e]);
                v[2 * e + 1] = __uint_as_float(r[8 * j + 2 * e + 1]) + bf16hi(rw[e]);
              }
              *reinterpret_cast<uint4*>(buf + chunk_off(lane, j)) = pack8f(v);
            }
            publish_chunk(&tmC, buf, n0 + 32 * i, row0, false);
            if (i + 2 < BN / 64) {  // refill this buffer with the residual of chunk i + 2
              if (lane == 0) {
                bulk_wait_group_read<0>();
                mbar_expect_tx(&lbar[b], kChunkBytes);
                tma_load_2d(buf, &tmX, &lbar[b], n0 + 32 * (i + 2), row0);
              }
              __syncwarp();
            }
          } else {
            buf = acquire_chunk(stg, bsel);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float v[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(r[8 * j + e]);
              *reinterpret_cast<uint4*>(buf + chunk_off(lane, j)) = pack8f(v);
            }
            publish_chunk(&tmC, buf, n0 + 32 * i, row0, false);
          }
        }
      } else if constexpr (EPI == EPI_ACC_F32) {
        acc_f32_epilogue(&tmC);
      } else if constexpr (EPI == EPI_ACC_F32_ROUTED) {
        routed_f32_epilogue(p);
      } else if constexpr (EPI == EPI_ROPE) {
        const int n0 = tn * BN;
        const int half = p.head_dim >> 1;
        const int pos = row_ok ? (m % p.seq_len) : 0;
#pragma unroll 1
        for (int h0 = wg * (BN / 2); h0 < (wg + 1) * (BN / 2); h0 += p.head_dim) {
          const int col = n0 + h0;
          const bool rotate = col < p.rope_cols;
#pragma unroll 1
          for (int j0 = 0; j0 < half; j0 += 32) {
            uint32_t lo[32], hi[32];
            tmem_ld_32x32b_x32(tbase + h0 + j0, lo);
            tmem_ld_32x32b_x32(tbase + h0 + half + j0, hi);
            tc_wait_ld();
            // The tables are frequency-major ([head_dim/2, seq_len]): for one frequency the 32 lanes
            // of a warp (32 consecutive rows, so consecutive positions) read 32 consecutive floats,
            // one 128-byte line per load instead of 32 lines for position-major rows.
            if (rotate && B200_IN_BOUNDS(p.errs, (long long)(j0 + 31) * p.seq_len + pos, 1,
                                         (long long)p.seq_len * half, 102)) {
              const float* ct = p.rope_cos + (size_t)j0 * p.seq_len + pos;
              const float* st = p.rope_sin + (size_t)j0 * p.seq_len + pos;
#pragma unroll
              for (int e8 = 0; e8 < 32; e8 += 8) {
                float cs[8], sn[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                  cs[k] = __ldg(ct + (size_t)(e8 + k) * p.seq_len);
                  sn[k] = __ldg(st + (size_t)(e8 + k) * p.seq_len);
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                  const int e = e8 + k;
                  const float x0 = __uint_as_float(lo[e]), x1 = __uint_as_float(hi[e]);
                  lo[e] = __float_as_uint(x0 * cs[k] - x1 * sn[k]);
                  hi[e] = __float_as_uint(x1 * cs[k] + x0 * sn[k]);
                }
              }
            }
            uint8_t* ba = acquire_chunk(stg, bsel);
            write_chunk_bf16(ba, lo);
            publish_chunk(&tmC, ba, col + j0, row0, false);
            uint8_t* bb = acquire_chunk(stg, bsel);
            write_chunk_bf16(bb, hi);
            publish_chunk(&tmC, bb, col + half + j0, row0, false);
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
          uint8_t* bg = acquire_chunk(stg, bsel);
          write_chunk_bf16(bg, g);
          publish_chunk(&tmX, bg, nb, row0, false);
          uint8_t* bu = acquire_chunk(stg, bsel);
          write_chunk_bf16(bu, uu);
          publish_chunk(&tmY, bu, nb, row0, false);
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float gv = __uint_as_float(g[e]);
            g[e] = __float_as_uint(silu_f(gv) * __uint_as_float(uu[e]));
          }
          uint8_t* bh = acquire_chunk(stg, bsel);
          write_chunk_bf16(bh, g);
          publish_chunk(&tmC, bh, nb, row0, false);
        }
      } else if constexpr (EPI == EPI_SWIGLU_BWD) {
        const int n0 = tn * BN + wg * (BN / 2);
#pragma unroll 1
        for (int i = 0; i < BN / 64; ++i) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + wg * (BN / 2) + 32 * i, r);
          tc_wait_ld();
          uint32_t dg[32], du[32];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t gw[4] = {gq[j].x, gq[j].y, gq[j].z, gq[j].w};
            const uint32_t uw[4] = {uq[j].x, uq[j].y, uq[j].z, uq[j].w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float gval = (e & 1) ? bf16hi(gw[e >> 1]) : bf16lo(gw[e >> 1]);
              const float uval = (e & 1) ? bf16hi(uw[e >> 1]) : bf16lo(uw[e >> 1]);
              const float da = __uint_as_float(r[8 * j + e]);
              const float sig = sigmoid_f(gval);
              du[8 * j + e] = __float_as_uint(da * gval * sig);
              dg[8 * j + e] = __float_as_uint(da * uval * sig * (1.0f + gval * (1.0f - sig)));
            }
          }
          if (i + 1 < BN / 64) load_gu(i + 1);
          uint8_t* bg = acquire_chunk(stg, bsel);
          write_chunk_bf16(bg, dg);
          publish_chunk(&tmC, bg, n0 + 32 * i, row0, false);
          uint8_t* bu = acquire_chunk(stg, bsel);
          write_chunk_bf16(bu, du);
          publish_chunk(&tmY, bu, n0 + 32 * i, row0, false);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (CG == 2)
          mbar_arrive_cluster(&tempty_bar[acc], 0);  // the leader's MMA owns the pair accumulator
        else
          mbar_arrive(&tempty_bar[acc]);
      }
    }
    // Every staged chunk must have landed before the CTA's shared memory goes away.
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_sync();  // no remote arrive or pair MMA may target a departed peer
  if (warp == 1) {
    tc_fence_after();
    if constexpr (CG == 2)
      tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    else
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

CUtensorMap make_tmap_2d(CUtensorMapDataType dtype, int elem_bytes, const void* base, uint64_t inner, uint64_t outer,
                         uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle) {
  B200_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base address must be 16-byte aligned");
  B200_CHECK((row_stride_elems * elem_bytes) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(&map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  B200_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
  return map;
}

CUtensorMap make_tmap_bf16_2d(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                              uint32_t box_inner, uint32_t box_outer) {
  return make_tmap_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, inner, outer, row_stride_elems, box_inner, box_outer,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

// Epilogue output / residual maps: one staging chunk (32 rows x 64 B) per box, 64-byte swizzle.
static CUtensorMap epi_map_bf16(const void* base, int rows, int cols, int ld) {
  return make_tmap_2d(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, (uint64_t)cols, (uint64_t)rows, (uint64_t)ld, 32, 32,
                   CU_TENSOR_MAP_SWIZZLE_64B);
}
static CUtensorMap epi_map_f32(const void* base, int rows, int cols, int ld) {
  return make_tmap_2d(CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, (uint64_t)cols, (uint64_t)rows, (uint64_t)ld, 16, 32,
                   CU_TENSOR_MAP_SWIZZLE_64B);
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

template <int BN, bool A_MN, bool B_MN, int EPI, int CG>
static void launch_impl(const GemmOperands& op, GemmParams p, cudaStream_t stream) {
  using Cfg = GemmCfg<BN, CG>;
  auto kernel = gemm_kernel<BN, A_MN, B_MN, EPI, CG>;
  static std::atomic<unsigned long long> configured{0};
  once_per_device(configured, [&] {
    B200_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES));
  });
  // A operand: K-major -> global [M, K] (K contiguous); MN-major -> global [K, M] (M contiguous).
  CUtensorMap tmA = A_MN ? make_tmap_bf16_2d(op.A, (uint64_t)p.M, (uint64_t)p.K, op.lda, 64, 64)
                         : make_tmap_bf16_2d(op.A, (uint64_t)p.K, (uint64_t)p.M, op.lda, 64, BM);
  CUtensorMap tmB;
  if (EPI == EPI_SWIGLU) {
    tmB = make_tmap_bf16_2d(op.B, (uint64_t)p.K, (uint64_t)(2 * p.ffn), op.ldb, 64, BN / 2);
  } else if (B_MN) {
    tmB = make_tmap_bf16_2d(op.B, (uint64_t)p.N, (uint64_t)p.K, op.ldb, 64, 64);
  } else {
    tmB = make_tmap_bf16_2d(op.B, (uint64_t)p.K, (uint64_t)p.N, op.ldb, 64, BN / CG);
  }
  // Output side.  Maps that an epilogue does not use repeat tmA (never dereferenced).
  CUtensorMap tmC = tmA, tmX = tmA, tmY = tmA;
  if (EPI == EPI_ACC_F32) {
    tmC = epi_map_f32(p.C32, p.M, p.N, p.ldc32);
  } else if (EPI == EPI_ACC_F32_ROUTED) {
    // no output map: the epilogue adds into the owners' shards with vector reductions
  } else if (EPI == EPI_SWIGLU) {
    tmC = epi_map_bf16(p.C, p.M, p.ffn, p.ldc);
    tmX = epi_map_bf16(p.aux, p.M, p.ffn, p.ld_aux);
    tmY = epi_map_bf16(p.aux + p.ffn, p.M, p.ffn, p.ld_aux);
  } else if (EPI == EPI_SWIGLU_BWD) {
    tmC = epi_map_bf16(p.C, p.M, p.ffn, p.ldc);
    tmY = epi_map_bf16(p.C + p.ffn, p.M, p.ffn, p.ldc);
  } else {
    tmC = epi_map_bf16(p.C, p.M, p.N, p.ldc);
    if (EPI == EPI_RESIDUAL) tmX = epi_map_bf16(p.R, p.M, p.N, p.ldr);
  }
  const int out_cols_per_tile = (EPI == EPI_SWIGLU) ? BN / 2 : BN;
  p.tiles_m = (p.M + BM * CG - 1) / (BM * CG);
  p.tiles_n = (p.N + out_cols_per_tile - 1) / out_cols_per_tile;
  p.total_k_blocks = (p.K + BK - 1) / BK;
  if (p.splits < 1) p.splits = 1;
  p.splits = std::min(p.splits, p.total_k_blocks);
  p.k_blocks_per_split = (p.total_k_blocks + p.splits - 1) / p.splits;
  p.splits = (p.total_k_blocks + p.k_blocks_per_split - 1) / p.k_blocks_per_split;
  p.errs = device_errors_ptr();
  const int units = p.tiles_m * p.tiles_n * p.splits;
  const int groups = std::max(1, std::min(units, num_sms() / CG));
  launch_k(kernel, dim3(groups * CG), dim3(NUM_THREADS), Cfg::SMEM_BYTES, stream, CG, tmA, tmB, tmC, tmX, tmY, tmA, p,
           p);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

// Tile widths each epilogue supports: ROPE needs whole heads per epilogue warpgroup half and SWIGLU
// 32-column chunks of gate and up per half, so neither takes 192.
constexpr bool epi_supports_bn(int epi, int bn) {
  return bn == 128 || bn == 256 || (bn == 192 && epi != EPI_ROPE && epi != EPI_SWIGLU);
}

// CTA pairs with an MN-major B split B into halves of whole 64-column TMA boxes.
constexpr bool pair_supports(bool b_mn, int bn) { return !b_mn || (bn / 2) % 64 == 0; }

template <int CG, bool A_MN, bool B_MN, int EPI>
static void dispatch_bn_cg(int bn, const GemmOperands& op, const GemmParams& p, cudaStream_t stream) {
  if (bn == 256)
    launch_impl<256, A_MN, B_MN, EPI, CG>(op, p, stream);
  else if (bn == 192) {
    if constexpr (epi_supports_bn(EPI, 192) && (CG == 1 || pair_supports(B_MN, 192)))
      launch_impl<192, A_MN, B_MN, EPI, CG>(op, p, stream);
    else
      B200_CHECK(false, "BN = 192 is not available for this epilogue / operand layout / CTA group");
  } else
    launch_impl<128, A_MN, B_MN, EPI, CG>(op, p, stream);
}

template <bool A_MN, bool B_MN, int EPI>
static void dispatch_bn(int bn, int cg, const GemmOperands& op, const GemmParams& p, cudaStream_t stream) {
  if (cg == 2)
    dispatch_bn_cg<2, A_MN, B_MN, EPI>(bn, op, p, stream);
  else
    dispatch_bn_cg<1, A_MN, B_MN, EPI>(bn, op, p, stream);
}

// Tile width, CTA group and K-split for a persistent grid on `sms` SMs.  A work unit runs in rounds of
// sms / CG concurrent units; its time is (k-blocks + 3 for the pipeline fill) x the per-SM time of one
// 64-deep k-block, measured on B200 for each variant (microseconds; the bigger the per-SM tile, the
// better the time per FLOP, pairs better than single CTAs), plus the exposed last epilogue.
// Whether the residual / SwiGLU / SwiGLU-backward epilogues may run on CTA pairs (the cost model's
// own choice, the default) or stay on single CTAs (ZB_GEMM_PAIR_EPI=0).  Measured on B200 (isolated,
// L2 flushed, TFLOP/s single -> pair): SwiGLU 8192x4096x768 988 -> 1071, 8192x11008x2048 1449 -> 1618;
// residual 8192x768x2048 680 -> 720, 8192x2048x5504 1135 -> 1377; in the training step the 1.3B
// model's stage 0 went from 76.2 to 74.4 ms and `small` from 7.99 to 7.97 ms.
static bool pair_heavy_epilogues() {
  static const bool on = [] {
    const char* v = std::getenv("ZB_GEMM_PAIR_EPI");
    return v == nullptr || std::string(v) != "0";
  }();
  return on;
}

GemmTile choose_gemm_tile(int M, int N, int K, int epi, int head_dim, bool allow_split, bool b_mn, int sms,
                          int only_bn, int only_cg) {
  struct Variant {
    int cg, bn;
    double us_per_kblock;
  };
  static const Variant kVariants[] = {{2, 256, 0.418}, {2, 192, 0.400}, {1, 256, 0.465},
                                      {1, 192, 0.450}, {2, 128, 0.362}, {1, 128, 0.350}};
  const int kb = (K + BK - 1) / BK;
  const bool heavy = (epi == EPI_SWIGLU || epi == EPI_SWIGLU_BWD || epi == EPI_ROPE);
  GemmTile best{256, 1, 1};
  double best_cost = 1e30;
  for (const Variant& v : kVariants) {
    if (!epi_supports_bn(epi, v.bn) || (v.cg == 2 && !pair_supports(b_mn, v.bn))) continue;
    if ((only_bn > 0 && v.bn != only_bn) || (only_cg > 0 && v.cg != only_cg)) continue;
    // An earlier build measured the epilogues that read or write several tiles per output tile
    // (residual, SwiGLU forward / backward) slower as pairs; ZB_GEMM_PAIR_EPI=0 restores that choice.
    if (only_cg == 0 && v.cg == 2 && !pair_heavy_epilogues() &&
        (epi == EPI_RESIDUAL || epi == EPI_SWIGLU || epi == EPI_SWIGLU_BWD))
      continue;
    if (epi == EPI_ROPE && ((v.bn / 2) % head_dim) != 0) continue;
    const int out_cols = (epi == EPI_SWIGLU) ? v.bn / 2 : v.bn;
    const long tiles = (long)((M + BM * v.cg - 1) / (BM * v.cg)) * ((N + out_cols - 1) / out_cols);
    const int max_split = allow_split ? std::max(1, std::min(32, kb / 4)) : 1;
    const int slots = std::max(1, sms / v.cg);
    const double epi_us = (heavy ? 3.0 : 0.5) * v.bn / 256.0;
    // A residual tile on a CTA pair waits for both CTAs' epilogues before the shared accumulator is
    // released: ~1 us per round, which decides short-K shapes (8192x768x768: 450 TFLOP/s single vs
    // 410 as pairs) and not long ones (8192x768x2048: 681 vs 720).
    const double round_extra = (v.cg == 2 && epi == EPI_RESIDUAL) ? 1.0 : 0.0;
    for (int s = 1; s <= max_split; ++s) {
      const int kbs = (kb + s - 1) / s;
      const long units = tiles * ((kb + kbs - 1) / kbs);
      const long rounds = (units + slots - 1) / slots;
      const double cost = rounds * ((kbs + 3.0) * v.us_per_kblock + round_extra) + epi_us;
      if (cost < best_cost * 0.98) {
        best_cost = cost;
        best = {v.bn, s, v.cg};
      }
    }
  }
  return best;
}

// Host checks of a routed weight gradient's destination (see GemmParams::route_*).
static void check_route(const GemmParams& p) {
  B200_CHECK(p.route_world >= 1 && p.route_world <= kRouteMaxWorld, "routed wgrad: 1..8 ranks");
  B200_CHECK(p.route_chunk > 0 && p.route_chunk % 4 == 0 && p.route_flat0 % 4 == 0 && p.route_ld % 4 == 0 &&
                 p.route_ld >= p.N,
             "routed wgrad: shard size, flat offset and row stride must be multiples of 4 (ld >= N)");
  B200_CHECK(p.route_flat0 + (long long)(p.M - 1) * p.route_ld + p.N <= p.route_chunk * (long long)p.route_world,
             "routed wgrad: the weight lies outside the sharded flat space");
  for (int r = 0; r < p.route_world; ++r)
    B200_CHECK(p.route_base[r] != 0 && p.route_base[r] % 16 == 0, "routed wgrad: shard bases must be 16-byte aligned");
}

void gemm_launch(const GemmOperands& op, GemmParams p, int epi, bool a_mn, bool b_mn, int bn, cudaStream_t stream) {
  int cg = 1;
  const bool acc = epi == EPI_ACC_F32 || epi == EPI_ACC_F32_ROUTED;  // fp32-accumulating: K-split allowed
  const int model_epi = acc ? EPI_ACC_F32 : epi;                        // same cost model for both
  if (bn <= 0) {  // automatic tile width, CTA group (and K-split for the fp32-accumulating epilogue)
    const GemmTile t = choose_gemm_tile(p.M, p.N, p.K, model_epi, p.head_dim > 0 ? p.head_dim : 64,
                                        acc && p.splits <= 0, b_mn, num_sms(), 0, 0);
    bn = t.bn;
    cg = t.cg;
    if (acc && p.splits <= 0) p.splits = t.splits;
  } else {
    if (bn >= 1000) {  // explicit CTA-pair request (tests, benchmarks): 1000 + tile width
      bn -= 1000;
      cg = 2;
      B200_CHECK(pair_supports(b_mn, bn), "CTA pairs with an MN-major B need BN / 2 to be a multiple of 64");
    }
    if (acc && p.splits <= 0)  // explicit tile, automatic K-split
      p.splits = choose_gemm_tile(p.M, p.N, p.K, model_epi, 64, true, b_mn, num_sms(), bn, cg).splits;
  }
  if (epi == EPI_ACC_F32_ROUTED) check_route(p);
  if (p.splits <= 0) p.splits = 1;
  B200_CHECK(bn == 128 || bn == 192 || bn == 256, "BN must be 128, 192 or 256");
  B200_CHECK(epi_supports_bn(epi, bn), "this epilogue does not support BN = 192");
  B200_CHECK(epi != EPI_ROPE || (p.head_dim > 0 && (bn / 2) % p.head_dim == 0),
             "RoPE epilogue: half the tile width must be a multiple of head_dim");
  B200_CHECK(p.N % 8 == 0, "GEMM output width N must be a multiple of 8");
  B200_CHECK((a_mn || p.K % 8 == 0) && (b_mn || p.K % 8 == 0), "GEMM K must be a multiple of 8 for K-major operands");
  B200_CHECK(!a_mn || p.M % 8 == 0, "GEMM M must be a multiple of 8 for an MN-major A operand");
  if (!a_mn && !b_mn) {
    switch (epi) {
      case EPI_STORE: return dispatch_bn<false, false, EPI_STORE>(bn, cg, op, p, stream);
      case EPI_RESIDUAL: return dispatch_bn<false, false, EPI_RESIDUAL>(bn, cg, op, p, stream);
      case EPI_ROPE: return dispatch_bn<false, false, EPI_ROPE>(bn, cg, op, p, stream);
      case EPI_SWIGLU: return dispatch_bn<false, false, EPI_SWIGLU>(bn, cg, op, p, stream);
      case EPI_ACC_F32: return dispatch_bn<false, false, EPI_ACC_F32>(bn, cg, op, p, stream);
    }
  } else if (!a_mn && b_mn) {
    switch (epi) {
      case EPI_STORE: return dispatch_bn<false, true, EPI_STORE>(bn, cg, op, p, stream);
      case EPI_SWIGLU_BWD: return dispatch_bn<false, true, EPI_SWIGLU_BWD>(bn, cg, op, p, stream);
      case EPI_ACC_F32: return dispatch_bn<false, true, EPI_ACC_F32>(bn, cg, op, p, stream);
    }
  } else if (a_mn && b_mn) {
    switch (epi) {
      case EPI_ACC_F32: return dispatch_bn<true, true, EPI_ACC_F32>(bn, cg, op, p, stream);
      case EPI_ACC_F32_ROUTED: return dispatch_bn<true, true, EPI_ACC_F32_ROUTED>(bn, cg, op, p, stream);
      case EPI_STORE: return dispatch_bn<true, true, EPI_STORE>(bn, cg, op, p, stream);
    }
  }
  B200_CHECK(false, "unsupported GEMM operand-major / epilogue combination");
}

// Tile / split bookkeeping of one problem for a given tile shape (the launcher's fields).
static void fill_schedule(GemmParams& q, int bn, int cg, int splits) {
  q.tiles_m = (q.M + BM * cg - 1) / (BM * cg);
  q.tiles_n = (q.N + bn - 1) / bn;
  q.total_k_blocks = (q.K + BK - 1) / BK;
  q.splits = std::max(1, std::min(splits, q.total_k_blocks));
  q.k_blocks_per_split = (q.total_k_blocks + q.splits - 1) / q.splits;
  q.splits = (q.total_k_blocks + q.k_blocks_per_split - 1) / q.k_blocks_per_split;
}

// Makespan (in k-blocks, +3 per unit for the pipeline fill) of the grouped boustrophedon deal.
static long grouped_makespan(const GemmParams& p0, const GemmParams& p1, int G, int* first_out) {
  const long units0 = (long)p0.tiles_m * p0.tiles_n * p0.splits, units1 = (long)p1.tiles_m * p1.tiles_n * p1.splits;
  const int c0 = p0.k_blocks_per_split + 3, c1 = p1.k_blocks_per_split + 3;
  const int first = c1 > c0 ? 1 : 0;
  const long n_first = first ? units1 : units0;
  const int cost_first = first ? c1 : c0, cost_second = first ? c0 : c1;
  std::vector<long> load(G, 0);
  const long total = units0 + units1;
  for (long u = 0; u < total; ++u) {
    const long k = u / G, r = u % G;
    const long g = (k & 1) ? (G - 1 - r) : r;
    load[g] += (u < n_first) ? cost_first : cost_second;
  }
  *first_out = first;
  return *std::max_element(load.begin(), load.end());
}

constexpr int kGroupedBN = 256, kGroupedCG = 2;

long plan_dgrad_wgrad(GemmParams& p0, GemmParams& p1, int sms) {
  constexpr int BNG = kGroupedBN, CGG = kGroupedCG;
  const int G = std::max(1, sms / CGG);
  fill_schedule(p0, BNG, CGG, 1);
  int first = 0;
  if (p1.splits > 0) {
    fill_schedule(p1, BNG, CGG, p1.splits);
    grouped_makespan(p0, p1, G, &first);
  } else {
    long best = -1;
    int best_split = 1;
    const int kb1 = (p1.K + BK - 1) / BK;
    for (int s : {1, 2, 3, 4, 6, 8, 12, 16}) {
      if (s > 1 && kb1 / s < 4) break;
      GemmParams q = p1;
      fill_schedule(q, BNG, CGG, s);
      int f = 0;
      const long span = grouped_makespan(p0, q, G, &f);
      if (best < 0 || span < best) {
        best = span;
        best_split = s;
      }
    }
    fill_schedule(p1, BNG, CGG, best_split);
    grouped_makespan(p0, p1, G, &first);
  }
  const long units0 = (long)p0.tiles_m * p0.tiles_n * p0.splits, units1 = (long)p1.tiles_m * p1.tiles_n * p1.splits;
  p0.grp_first = first;
  p0.grp_units_first = (int)(first ? units1 : units0);
  p0.grp_units_total = (int)(units0 + units1);
  return grouped_makespan(p0, p1, G, &first);
}

void gemm_launch_dgrad_wgrad(const GemmOperands& op0, GemmParams p0, const GemmOperands& op1, GemmParams p1,
                             cudaStream_t stream) {
  constexpr int BNG = kGroupedBN, CGG = kGroupedCG;
  using Cfg = GemmCfg<BNG, CGG>;
  B200_CHECK(p0.N % 8 == 0 && p1.N % 8 == 0 && p0.K % 8 == 0 && p1.M % 8 == 0,
             "grouped dgrad/wgrad: N, K (dgrad) and M (wgrad) must be multiples of 8");
  const int G = std::max(1, num_sms() / CGG);
  const bool routed = p1.route_world > 0;  // problem 1 to the owners' shards instead of p1.C32
  if (routed) check_route(p1);
  plan_dgrad_wgrad(p0, p1, num_sms());
  p0.errs = p1.errs = device_errors_ptr();

  auto kernel = routed ? gemm_kernel<BNG, false, true, EPI_STORE, CGG, true, true>
                       : gemm_kernel<BNG, false, true, EPI_STORE, CGG, true, false>;
  static std::atomic<unsigned long long> configured[2];
  once_per_device(configured[routed], [&] {
    B200_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES));
  });
  // problem 0: A = dY [M0, K0] K-major, B = W [K0, N0] MN-major, C = dX (bf16)
  const CUtensorMap tmA = make_tmap_bf16_2d(op0.A, (uint64_t)p0.K, (uint64_t)p0.M, op0.lda, 64, BM);
  const CUtensorMap tmB = make_tmap_bf16_2d(op0.B, (uint64_t)p0.N, (uint64_t)p0.K, op0.ldb, 64, 64);
  const CUtensorMap tmC = epi_map_bf16(p0.C, p0.M, p0.N, p0.ldc);
  // problem 1: A = dY^T as [K1, M1] MN-major, B = X [K1, N1] MN-major, C = dW (fp32, accumulated)
  const CUtensorMap tmX = make_tmap_bf16_2d(op1.A, (uint64_t)p1.M, (uint64_t)p1.K, op1.lda, 64, 64);
  const CUtensorMap tmY = make_tmap_bf16_2d(op1.B, (uint64_t)p1.N, (uint64_t)p1.K, op1.ldb, 64, 64);
  const CUtensorMap tmZ = routed ? tmX : epi_map_f32(p1.C32, p1.M, p1.N, p1.ldc32);  // unused when routed
  const int groups = std::max(1, std::min(p0.grp_units_total, G));
  launch_k(kernel, dim3(groups * CGG), dim3(NUM_THREADS), Cfg::SMEM_BYTES, stream, CGG, tmA, tmB, tmC, tmX, tmY, tmZ,
           p0, p1);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

}  // namespace b200
