// Causal GQA flash-attention backward on the 5th-generation tensor cores (sm_100a).
//
// Work item: one (key/value block j of 128 rows, kv head, batch).  The item keeps K_j and V_j in
// shared memory and loops over every query head of its group and every query block i >= j:
//
//   S^T  = K_j Q_i^T           (M = kv, N = q,  K = hd)   tensor memory
//   dP^T = V_j dO_i^T          (M = kv, N = q,  K = hd)   tensor memory
//   P^T  = exp2(S^T * scale*log2e - lse2[q]),  dS^T = P^T * (dP^T - delta[q])
//   dV  += P^T dO_i            (M = kv, N = hd, K = q)    accumulated in tensor memory over the loop
//   dK  += dS^T Q_i            (M = kv, N = hd, K = q)    accumulated in tensor memory over the loop
//   dQ_i = dS K_j              (M = q,  N = hd, K = kv)   A operand = the same dS^T bytes read MN-major
//   dq_acc[q rows] += scale * dQ_i                        TMA add-reductions (hd 64) / fp32 vector atomics
//
// Scheduling: a persistent grid of min(items, SMs) CTAs.  Items are ordered by cost (block j costs
// group * (S/128 - j) iterations, so j = 0 first) and dealt to CTAs boustrophedon-style (CTA c takes
// items c, 2G-1-c, 2G+c, ...), which pairs long items with short ones.
//
// 320 threads: warp 0 TMA (K/V per item; Q, dO, lse and delta per iteration), warp 1 tensor-memory
// allocation + MMA issue, warps 2..9 two compute warpgroups.  Thread (wg, r) owns kv row r and the
// query columns [64*wg, 64*wg+64) of S^T / dP^T, then the output columns [wg*hd/2, (wg+1)*hd/2) of
// dQ / dV and its half of the RoPE pairs of dK.  lse / delta of the current query block arrive in
// shared memory with the Q / dO tiles and are read as broadcasts.  Epilogues: dK (times the softmax
// scale, RoPE backward applied) and dV are written as bf16 into the k / v columns of the fused
// q|k|v gradient; a small kernel converts dq_acc into the q columns with RoPE backward.
// delta = rowsum(dO * O) comes from a pre-pass.
#include <cuda.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "attention_bwd_noalloc.h"
#include "common.cuh"
#include "gemm.h"
#include "kernels.h"

namespace b200 {

namespace {

constexpr int BWD_THREADS = 320;
constexpr int kBwdChunk = 2048;  // dQ staging chunk: 32 rows x 16 fp32 (64 B rows, 64-byte swizzle)

template <int HD>
struct AttnBwdCfg {
  static constexpr int KB = HD / 64;
  static constexpr int TILE = 128 * HD * 2;     // bytes of one 128-row tile
  static constexpr int STAGES = (HD == 64) ? 2 : 1;
  static constexpr bool TMA_DQ = (HD == 64);    // dQ through TMA reductions (staging fits in smem)
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = TILE;
  static constexpr int QD_OFF = 2 * TILE;       // stages of (Q_i, dO_i)
  static constexpr int PT_OFF = QD_OFF + STAGES * 2 * TILE;
  static constexpr int DST_OFF = PT_OFF + 128 * 128 * 2;
  static constexpr int LD_OFF = DST_OFF + 128 * 128 * 2;  // per stage: lse2[128] | delta[128]
  static constexpr int STG_OFF = LD_OFF + STAGES * 1024;
  static constexpr int STG_BYTES = TMA_DQ ? 8 * 2 * kBwdChunk : 0;
  static constexpr int BAR_OFF = STG_OFF + STG_BYTES;
  static constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;
  static_assert(SMEM_BYTES <= 232448, "attention backward shared memory exceeds 227 KB");
  // tensor-memory columns
  static constexpr int T_ST = 0, T_DPT = 128, T_DV = 256, T_DK = 256 + HD;
  static constexpr int T_DQ = (HD == 64) ? 384 : 0;
  static constexpr int TMEM_COLS = 512;
  static constexpr int HALF = HD / 2;
};

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Untiled bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void store_swizzled_row(uint8_t* base, int r, int c, const uint32_t (&pk)[16]) {
  // 32 bf16 values (columns c .. c+31) of row r of a [128 x 128] K-major SW128 tile.
  const int kblk = c >> 6;
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) {
    const int chunk = ((c & 63) >> 3) + ch;
    const int sw = chunk ^ (r & 7);
    *reinterpret_cast<uint4*>(base + kblk * 16384 + r * 128 + sw * 16) =
        make_uint4(pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
  }
}

template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[N]) {
  if constexpr (N == 32) {
    tmem_ld_32x32b_x32(taddr, r);
  } else {
    static_assert(N == 16, "16 or 32 columns");
    tmem_ld_32x32b_x16(taddr, r);
  }
}

// Work item u of the cost-ordered list -> (kv block j, kv head, batch).
struct BwdItem {
  int j, kvh, b;
};
__device__ __forceinline__ BwdItem bwd_item(int u, int batch, int kv_heads) {
  const int per_j = batch * kv_heads;
  const int r = u % per_j;
  return {u / per_j, r % kv_heads, r / kv_heads};
}
// k-th item of CTA c in a grid of G CTAs (boustrophedon deal), or -1 past the end.
__device__ __forceinline__ int bwd_item_index(int k, int c, int G, int n_items) {
  const int u = k * G + ((k & 1) ? (G - 1 - c) : c);
  return u < n_items ? u : -1;
}

template <int HD>
__global__ void __launch_bounds__(BWD_THREADS, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_dq, AttnBwdParams p, DeviceErrors* errs) {
  using C = AttnBwdCfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + 1;
  uint64_t* q_full = bars + 2;
  uint64_t* q_empty = q_full + C::STAGES;
  uint64_t* st_full = q_empty + C::STAGES;
  uint64_t* p_ready = st_full + 1;
  uint64_t* dq_full = p_ready + 1;
  uint64_t* dq_free = dq_full + 1;
  uint64_t* epi_done = dq_free + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(epi_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qb = p.seq / 128;
  const int group = p.heads / p.kv_heads;
  const int n_items = p.batch * p.kv_heads * n_qb;
  const int G = gridDim.x, cta = blockIdx.x;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    mbar_init(st_full, 1);
    mbar_init(p_ready, 8);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 8);
    mbar_init(epi_done, 8);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait_and_release();  // q|k|v, O, dO, lse, delta come from earlier kernels of the stream

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_qkv);
      tma_prefetch_desc(&tm_do);
      int g = 0;  // global iteration counter (stage ring position)
      bool ok = true;
      for (int k = 0, u; ok && (u = bwd_item_index(k, cta, G, n_items)) >= 0; ++k) {
        const BwdItem w = bwd_item(u, p.batch, p.kv_heads);
        const int row0 = w.b * p.seq;
        const int n_q = n_qb - w.j;
        if (!mbar_wait_bounded(kv_empty, (k & 1) ^ 1u, abort_flag, errs, kErrAttnWait, 9)) break;
        mbar_expect_tx(kv_full, 2 * C::TILE);
#pragma unroll
        for (int kb = 0; kb < C::KB; ++kb) {
          tma_load_2d(smem + C::K_OFF + kb * 16384, &tm_qkv, kv_full, p.k_col + w.kvh * HD + 64 * kb,
                      row0 + w.j * 128);
          tma_load_2d(smem + C::V_OFF + kb * 16384, &tm_qkv, kv_full, p.v_col + w.kvh * HD + 64 * kb,
                      row0 + w.j * 128);
        }
        for (int it = 0; it < group * n_q; ++it, ++g) {
          const int h = w.kvh * group + it / n_q;
          const int i = w.j + it % n_q;
          const int st = g % C::STAGES;
          if (!mbar_wait_bounded(&q_empty[st], ((g / C::STAGES) & 1) ^ 1u, abort_flag, errs, kErrAttnWait, 10)) {
            ok = false;
            break;
          }
          uint8_t* qs = smem + C::QD_OFF + st * 2 * C::TILE;
          uint8_t* ds = qs + C::TILE;
          uint8_t* ls = smem + C::LD_OFF + st * 1024;
          const size_t vec = ((size_t)w.b * p.heads + h) * p.seq + (size_t)i * 128;
          mbar_expect_tx(&q_full[st], 2 * C::TILE + 1024);
#pragma unroll
          for (int kb = 0; kb < C::KB; ++kb) {
            tma_load_2d(qs + kb * 16384, &tm_qkv, &q_full[st], h * HD + 64 * kb, row0 + i * 128);
            tma_load_2d(ds + kb * 16384, &tm_do, &q_full[st], h * HD + 64 * kb, row0 + i * 128);
          }
          if (B200_IN_BOUNDS(errs, vec, 128, (long long)p.batch * p.heads * p.seq, 110)) {
            bulk_load(ls, p.lse + vec, 512, &q_full[st]);
            bulk_load(ls + 512, p.delta + vec, 512, &q_full[st]);
          } else {  // the 1024 skipped bytes were announced above: mark them complete without an arrival
            asm volatile("mbarrier.complete_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&q_full[st])), "r"(1024)
                         : "memory");
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t ID_KV = idesc_bf16_f32(128, HD, false, true);
      constexpr uint32_t ID_Q = idesc_bf16_f32(128, HD, true, true);
      const uint32_t k_addr = smem_u32(smem + C::K_OFF);
      const uint32_t v_addr = smem_u32(smem + C::V_OFF);
      const uint32_t pt_addr = smem_u32(smem + C::PT_OFF);
      const uint32_t dst_addr = smem_u32(smem + C::DST_OFF);
      int g = 0;
      bool ok = true;
      for (int k = 0, u; ok && (u = bwd_item_index(k, cta, G, n_items)) >= 0; ++k) {
        const BwdItem w = bwd_item(u, p.batch, p.kv_heads);
        const int n_it = group * (n_qb - w.j);
        if (!mbar_wait_bounded(kv_full, k & 1, abort_flag, errs, kErrAttnWait, 11)) break;
        for (int it = 0; it < n_it; ++it, ++g) {
          const int st = g % C::STAGES;
          if (!mbar_wait_bounded(&q_full[st], (g / C::STAGES) & 1, abort_flag, errs, kErrAttnWait, 12)) {
            ok = false;
            break;
          }
          if (HD == 128 && g > 0 && !mbar_wait_bounded(dq_free, (g - 1) & 1, abort_flag, errs, kErrAttnWait, 13)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t q_addr = smem_u32(smem + C::QD_OFF + st * 2 * C::TILE);
          const uint32_t do_addr = q_addr + C::TILE;
#pragma unroll
          for (int ks = 0; ks < HD / 16; ++ks) {
            const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
            tc_mma_f16(tmem + C::T_ST, smem_desc_sw128(k_addr + off, 16, 1024),
                       smem_desc_sw128(q_addr + off, 16, 1024), ID_S, ks > 0 ? 1u : 0u);
          }
#pragma unroll
          for (int ks = 0; ks < HD / 16; ++ks) {
            const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
            tc_mma_f16(tmem + C::T_DPT, smem_desc_sw128(v_addr + off, 16, 1024),
                       smem_desc_sw128(do_addr + off, 16, 1024), ID_S, ks > 0 ? 1u : 0u);
          }
          tc_commit(st_full);
          if (!mbar_wait_bounded(p_ready, g & 1, abort_flag, errs, kErrAttnWait, 14)) {
            ok = false;
            break;
          }
          if (HD == 64 && g > 0 && !mbar_wait_bounded(dq_free, (g - 1) & 1, abort_flag, errs, kErrAttnWait, 15)) {
            ok = false;
            break;
          }
          // The previous item's dK / dV must be read out before this item's first MMA overwrites them.
          if (it == 0 && k > 0 && !mbar_wait_bounded(epi_done, (k - 1) & 1, abort_flag, errs, kErrAttnWait, 18)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {  // K = 128 query rows
            const uint32_t aoff = (ks >> 2) * 16384 + (ks & 3) * 32;
            const uint32_t boff = ks * 2048;
            const uint32_t acc = (it > 0 || ks > 0) ? 1u : 0u;
            tc_mma_f16(tmem + C::T_DV, smem_desc_sw128(pt_addr + aoff, 16, 1024),
                       smem_desc_sw128(do_addr + boff, 16384, 1024), ID_KV, acc);
            tc_mma_f16(tmem + C::T_DK, smem_desc_sw128(dst_addr + aoff, 16, 1024),
                       smem_desc_sw128(q_addr + boff, 16384, 1024), ID_KV, acc);
          }
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {  // K = 128 kv rows
            tc_mma_f16(tmem + C::T_DQ, smem_desc_sw128(dst_addr + ks * 2048, 16384, 1024),
                       smem_desc_sw128(k_addr + ks * 2048, 16384, 1024), ID_Q, ks > 0 ? 1u : 0u);
          }
          tc_commit(dq_full);
          tc_commit(&q_empty[st]);
        }
        if (!ok) break;
        tc_commit(kv_empty);  // K_j / V_j no longer read once this item's MMAs complete
      }
    }
  } else {
    const int wg = (warp - 2) >> 2;  // columns [64*wg, 64*wg + 64) of S^T / dP^T
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;    // kv row for S^T / dK / dV; query row for dQ
    const int col0 = wg * 64;
    const uint32_t lane_base = tmem + ((uint32_t)(q4 * 32) << 16);
    const float scale2 = p.scale * 1.4426950408889634f;
    uint8_t* pt = smem + C::PT_OFF;
    uint8_t* dst = smem + C::DST_OFF;
    uint8_t* stg = smem + C::STG_OFF + (warp - 2) * 2 * kBwdChunk;
    int g = 0;
    bool ok = true;
    for (int k = 0, u; ok && (u = bwd_item_index(k, cta, G, n_items)) >= 0; ++k) {
      const BwdItem w = bwd_item(u, p.batch, p.kv_heads);
      const int n_q = n_qb - w.j;
      const int n_it = group * n_q;
      const int row0 = w.b * p.seq;
      for (int it = 0; it < n_it; ++it, ++g) {
        const int h = w.kvh * group + it / n_q;
        const int i = w.j + it % n_q;
        if (!mbar_wait_bounded(st_full, g & 1, abort_flag, errs, kErrAttnWait, 16)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const bool diag = (i == w.j);
        const float* lds = reinterpret_cast<const float*>(smem + C::LD_OFF + (g % C::STAGES) * 1024);
#pragma unroll
        for (int c = 0; c < 64; c += 32) {
          uint32_t sv[32], dpv[32];
          tmem_ld_32x32b_x32(lane_base + C::T_ST + col0 + c, sv);
          tmem_ld_32x32b_x32(lane_base + C::T_DPT + col0 + c, dpv);
          float lse_v[32], del_v[32];
          const float4* l4 = reinterpret_cast<const float4*>(lds + col0 + c);
          const float4* d4 = reinterpret_cast<const float4*>(lds + 128 + col0 + c);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float4 a = l4[e], dd = d4[e];
            lse_v[4 * e] = a.x; lse_v[4 * e + 1] = a.y; lse_v[4 * e + 2] = a.z; lse_v[4 * e + 3] = a.w;
            del_v[4 * e] = dd.x; del_v[4 * e + 1] = dd.y; del_v[4 * e + 2] = dd.z; del_v[4 * e + 3] = dd.w;
          }
          tc_wait_ld();
          uint32_t pk[16], dk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            float pv[2], dv[2];
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              float pr = ex2_approx(fmaf(__uint_as_float(sv[e + t]), scale2, -lse_v[e + t]));
              if (diag && (col0 + c + e + t < r)) pr = 0.f;
              pv[t] = pr;
              dv[t] = pr * (__uint_as_float(dpv[e + t]) - del_v[e + t]);
            }
            pk[e >> 1] = pack_bf16(pv[0], pv[1]);
            dk[e >> 1] = pack_bf16(dv[0], dv[1]);
          }
          store_swizzled_row(pt, r, col0 + c, pk);
          store_swizzled_row(dst, r, col0 + c, dk);
        }
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_ready);
        // dQ_i rows (thread = query row r of block i), this warpgroup's half of the columns
        if (!mbar_wait_bounded(dq_full, g & 1, abort_flag, errs, kErrAttnWait, 17)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if constexpr (C::TMA_DQ) {
          // 32 columns = two 16-column fp32 chunks; both staging chunks of this warp are free once
          // the previous iteration's reductions have read them.
          if (lane == 0) bulk_wait_group_read<0>();
          __syncwarp();
#pragma unroll
          for (int hc = 0; hc < 2; ++hc) {
            uint32_t qv[16];
            tmem_ld_32x32b_x16(lane_base + C::T_DQ + wg * C::HALF + 16 * hc, qv);
            tc_wait_ld();
            uint8_t* buf = stg + hc * kBwdChunk;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              const int off = lane * 64 + ((jj ^ ((lane >> 1) & 3)) << 4);
              *reinterpret_cast<float4*>(buf + off) =
                  make_float4(__uint_as_float(qv[4 * jj]) * p.scale, __uint_as_float(qv[4 * jj + 1]) * p.scale,
                              __uint_as_float(qv[4 * jj + 2]) * p.scale, __uint_as_float(qv[4 * jj + 3]) * p.scale);
            }
          }
          fence_async_smem();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(dq_free);
#pragma unroll
            for (int hc = 0; hc < 2; ++hc)
              tma_reduce_add_2d(&tm_dq, stg + hc * kBwdChunk, h * HD + wg * C::HALF + 16 * hc,
                                row0 + i * 128 + q4 * 32);
            bulk_commit_group();
          }
        } else {
          const size_t dq_idx = (size_t)(row0 + i * 128 + r) * (p.heads * HD) + h * HD + wg * C::HALF;
          float* dq_row = p.dq_acc + dq_idx;
          const bool dq_in = B200_IN_BOUNDS(errs, dq_idx, C::HALF, (long long)p.batch * p.seq * p.heads * HD, 111);
#pragma unroll
          for (int c = 0; c < C::HALF; c += 32) {
            uint32_t qv[32];
            tmem_ld_32x32b_x32(lane_base + C::T_DQ + wg * C::HALF + c, qv);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
              if (dq_in)
                atomicAdd(reinterpret_cast<float4*>(dq_row + c + e),
                        make_float4(__uint_as_float(qv[e]) * p.scale, __uint_as_float(qv[e + 1]) * p.scale,
                                    __uint_as_float(qv[e + 2]) * p.scale, __uint_as_float(qv[e + 3]) * p.scale));
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(dq_free);
        }
      }
      if (!ok) break;
      // The item's last dq_full also covers its final dV / dK accumulation.
      tc_fence_after();
      const int kv_row = row0 + w.j * 128 + r;
      const int pos = w.j * 128 + r;
      constexpr int HALF = C::HALF;
      constexpr int QTR = HALF / 2;  // RoPE pairs per warpgroup
      __nv_bfloat16* dk_out = p.dqkv + (size_t)kv_row * p.ld + p.k_col + w.kvh * HD;
      __nv_bfloat16* dv_out = p.dqkv + (size_t)kv_row * p.ld + p.v_col + w.kvh * HD + wg * HALF;
#pragma unroll
      for (int c = 0; c < HALF; c += 32) {
        uint32_t vv[32];
        tmem_ld_32x32b_x32(lane_base + C::T_DV + wg * HALF + c, vv);
        tc_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint4 o;
          o.x = pack_bf16(__uint_as_float(vv[e]), __uint_as_float(vv[e + 1]));
          o.y = pack_bf16(__uint_as_float(vv[e + 2]), __uint_as_float(vv[e + 3]));
          o.z = pack_bf16(__uint_as_float(vv[e + 4]), __uint_as_float(vv[e + 5]));
          o.w = pack_bf16(__uint_as_float(vv[e + 6]), __uint_as_float(vv[e + 7]));
          *reinterpret_cast<uint4*>(dv_out + c + e) = o;
        }
      }
      {
        const int c0 = wg * QTR;  // this warpgroup's RoPE pair range [c0, c0 + QTR)
        uint32_t lo[QTR], hi[QTR];
        tmem_ld_cols<QTR>(lane_base + C::T_DK + c0, lo);
        tmem_ld_cols<QTR>(lane_base + C::T_DK + HALF + c0, hi);
        tc_wait_ld();
        const float* cs = p.rope_cos + (size_t)pos * HALF + c0;
        const float* sn = p.rope_sin + (size_t)pos * HALF + c0;
#pragma unroll
        for (int e = 0; e < QTR; e += 8) {
          float a[8], bb[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const float x0 = __uint_as_float(lo[e + t]) * p.scale;
            const float x1 = __uint_as_float(hi[e + t]) * p.scale;
            const float cv = cs[e + t], sv = sn[e + t];
            a[t] = x0 * cv + x1 * sv;
            bb[t] = x1 * cv - x0 * sv;
          }
          uint4 wa, wb;
          wa.x = pack_bf16(a[0], a[1]); wa.y = pack_bf16(a[2], a[3]);
          wa.z = pack_bf16(a[4], a[5]); wa.w = pack_bf16(a[6], a[7]);
          wb.x = pack_bf16(bb[0], bb[1]); wb.y = pack_bf16(bb[2], bb[3]);
          wb.z = pack_bf16(bb[4], bb[5]); wb.w = pack_bf16(bb[6], bb[7]);
          *reinterpret_cast<uint4*>(dk_out + c0 + e) = wa;
          *reinterpret_cast<uint4*>(dk_out + HALF + c0 + e) = wb;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(epi_done);
    }
    if (C::TMA_DQ && lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------
// head_dim 64: software-pipelined variant.
//
// Same work items and math as attn_bwd_kernel, with the tensor cores and the softmax warps
// overlapped.  Per iteration g (one query block of one head) the MMA warp issues
//     S^T(g+1) dP^T(g+1) | dV(g) | dK(g) dQ(g)
// as soon as the softmax warps hand over block g, so the softmax of block g+1 starts after two MMAs
// and runs while the tensor cores compute dV(g), dK(g) and dQ(g).  What makes that legal:
//   * P^T(g) goes to TENSOR memory (bf16, in columns of its own) and dV(g) takes it from there (A
//     operand in tensor memory); the softmax of g+1 writes P^T(g+1) there only after the commit
//     behind dV(g) (pt_free);
//   * dS^T goes to shared memory (dK reads it K-major, dQ reads it MN-major as dS), double-buffered:
//     the softmax of g+1 writes the buffer dK(g-1) / dQ(g-1) read, and the commit that releases
//     S^T(g+1) to it comes after those MMAs;
//   * dQ is read out by the softmax warps one iteration late (after handing over P^T / dS^T of the
//     next block); dQ(g+1) waits for that readout (dq_free), which is due long before.
// Tensor memory: S^T [0,128) | dP^T [128,256) | dV [256,320) | dK [320,384) | dQ [384,448) | P^T.
// 384 threads: warp 0 TMA, warp 1 MMA (+ tensor-memory allocation), warps 2-3 idle, warpgroups
// 1 and 2 compute (thread = kv row for S^T / dP^T / dK / dV, query row for dQ; warpgroup w owns
// query columns [64w, 64w + 64) and output columns [32w, 32w + 32)).
// ---------------------------------------------------------------------------------------------
struct AttnBwd64Cfg {
  static constexpr int HD = 64;
  static constexpr int TILE = 128 * HD * 2;    // 16 KB
  static constexpr int STAGES = 2;             // (Q_i, dO_i, lse, delta) ring
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = TILE;
  static constexpr int QD_OFF = 2 * TILE;
  static constexpr int DST_OFF = QD_OFF + STAGES * 2 * TILE;  // two dS^T buffers of 128 x 128 bf16
  static constexpr int LD_OFF = DST_OFF + 2 * 128 * 128 * 2;  // per stage: lse2[128] | delta[128]
  static constexpr int STG_OFF = LD_OFF + STAGES * 1024;      // dQ staging: 8 warps x 2 chunks
  static constexpr int BAR_OFF = STG_OFF + 8 * 2 * kBwdChunk;
  static constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;
  static_assert(SMEM_BYTES <= 232448, "attention backward (hd 64) shared memory exceeds 227 KB");
  // tensor memory: S^T | dP^T | dV | dK | dQ | P^T (bf16, packed two per column)
  static constexpr int T_ST = 0, T_DPT = 128, T_DV = 256, T_DK = 320, T_DQ = 384, T_PT = 448;
  static constexpr int TMEM_COLS = 512;
  static constexpr int THREADS = 384;
  static constexpr int REGS_LOW = 72, REGS_HIGH = 216;  // 128 * 72 + 256 * 216 = 384 * 168
  static constexpr int EMU = 0;  // exponentials on the FMA pipe: columns with (c & 7) >= 8 - EMU (0 measured fastest)
};

template <int EMU>
__global__ void __launch_bounds__(AttnBwd64Cfg::THREADS, 1)
    attn_bwd_hd64_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                         const __grid_constant__ CUtensorMap tm_dq, AttnBwdParams p, DeviceErrors* errs) {
  using C = AttnBwd64Cfg;
  constexpr int HD = C::HD;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + 1;
  uint64_t* q_full = bars + 2;              // [STAGES]
  uint64_t* q_empty = q_full + C::STAGES;   // [STAGES]
  uint64_t* st_full = q_empty + C::STAGES;  // S^T and dP^T of the next block complete
  uint64_t* p_ready = st_full + 1;          // 8 warps: P^T in tensor memory, dS^T in shared memory
  uint64_t* dq_full = p_ready + 1;          // dQ of the block complete
  uint64_t* dq_free = dq_full + 1;          // 8 warps: dQ read out
  uint64_t* pt_free = dq_free + 1;          // dV has read P^T: the next block's P^T may be written
  uint64_t* epi_done = pt_free + 1;         // 8 warps: the item's dK / dV have been read out
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(epi_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qb = p.seq / 128;
  const int group = p.heads / p.kv_heads;
  const int n_items = p.batch * p.kv_heads * n_qb;
  const int G = gridDim.x, cta = blockIdx.x;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    mbar_init(st_full, 1);
    mbar_init(p_ready, 8);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 8);
    mbar_init(pt_free, 1);
    mbar_init(epi_done, 8);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait_and_release();  // q|k|v, O, dO, lse, delta come from earlier kernels of the stream

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::REGS_LOW));
    if (warp == 0 && lane == 0) {
      tma_prefetch_desc(&tm_qkv);
      tma_prefetch_desc(&tm_do);
      int g = 0;  // global iteration counter (stage ring position)
      bool ok = true;
      for (int k = 0, u; ok && (u = bwd_item_index(k, cta, G, n_items)) >= 0; ++k) {
        const BwdItem w = bwd_item(u, p.batch, p.kv_heads);
        const int row0 = w.b * p.seq;
        const int n_q = n_qb - w.j;
        if (!mbar_wait_bounded(kv_empty, (k & 1) ^ 1u, abort_flag, errs, kErrAttnWait, 9)) break;
        mbar_expect_tx(kv_full, 2 * C::TILE);
        tma_load_2d(smem + C::K_OFF, &tm_qkv, kv_full, p.k_col + w.kvh * HD, row0 + w.j * 128);
        tma_load_2d(smem + C::V_OFF, &tm_qkv, kv_full, p.v_col + w.kvh * HD, row0 + w.j * 128);
        for (int it = 0; it < group * n_q; ++it, ++g) {
          const int h = w.kvh * group + it / n_q;
          const int i = w.j + it % n_q;
          const int st = g % C::STAGES;
          if (!mbar_wait_bounded(&q_empty[st], ((g / C::STAGES) & 1) ^ 1u, abort_flag, errs, kErrAttnWait, 10)) {
            ok = false;
            break;
          }
          uint8_t* qs = smem + C::QD_OFF + st * 2 * C::TILE;
          uint8_t* ds = qs + C::TILE;
          uint8_t* ls = smem + C::LD_OFF + st * 1024;
          const size_t vec = ((size_t)w.b * p.heads + h) * p.seq + (size_t)i * 128;
          mbar_expect_tx(&q_full[st], 2 * C::TILE + 1024);
          tma_load_2d(qs, &tm_qkv, &q_full[st], h * HD, row0 + i * 128);
          tma_load_2d(ds, &tm_do, &q_full[st], h * HD, row0 + i * 128);
          if (B200_IN_BOUNDS(errs, vec, 128, (long long)p.batch * p.heads * p.seq, 110)) {
            bulk_load(ls, p.lse + vec, 512, &q_full[st]);
            bulk_load(ls + 512, p.delta + vec, 512, &q_full[st]);
          } else {  // the 1024 skipped bytes were announced above: mark them complete without an arrival
            asm volatile("mbarrier.complete_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&q_full[st])), "r"(1024)
                         : "memory");
          }
        }
      }
    } else if (warp == 1 && lane == 0) {
      constexpr uint32_t ID_S = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t ID_KV = idesc_bf16_f32(128, HD, false, true);
      constexpr uint32_t ID_Q = idesc_bf16_f32(128, HD, true, true);
      const uint32_t k_addr = smem_u32(smem + C::K_OFF);
      const uint32_t v_addr = smem_u32(smem + C::V_OFF);
      int g = 0;
      bool ok = true;
      // S^T = K Q^T and dP^T = V dO^T of global iteration gg (stage gg % STAGES)
      auto issue_scores = [&](int gg) -> bool {
        const int st = gg % C::STAGES;
        if (!mbar_wait_bounded(&q_full[st], (gg / C::STAGES) & 1, abort_flag, errs, kErrAttnWait, 12)) return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(smem + C::QD_OFF + st * 2 * C::TILE);
        const uint32_t do_addr = q_addr + C::TILE;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
          const uint32_t off = ks * 32;
          tc_mma_f16(tmem + C::T_ST, smem_desc_sw128(k_addr + off, 16, 1024), smem_desc_sw128(q_addr + off, 16, 1024),
                     ID_S, ks > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
          const uint32_t off = ks * 32;
          tc_mma_f16(tmem + C::T_DPT, smem_desc_sw128(v_addr + off, 16, 1024),
                     smem_desc_sw128(do_addr + off, 16, 1024), ID_S, ks > 0 ? 1u : 0u);
        }
        tc_commit(st_full);
        return true;
      };
      for (int k = 0, u; ok && (u = bwd_item_index(k, cta, G, n_items)) >= 0; ++k) {
        const BwdItem w = bwd_item(u, p.batch, p.kv_heads);
        const int n_it = group * (n_qb - w.j);
        if (!mbar_wait_bounded(kv_full, k & 1, abort_flag, errs, kErrAttnWait, 11)) break;
        tc_fence_after();
        if (!issue_scores(g)) break;
        for (int it = 0; it < n_it; ++it, ++g) {
          const int st = g % C::STAGES;
          const int b = g & 1;
          if (!mbar_wait_bounded(p_ready, g & 1, abort_flag, errs, kErrAttnWait, 14)) {
            ok = false;
            break;
          }
          // The previous item's dK / dV must be read out before this item's first MMAs overwrite them.
          if (it == 0 && k > 0 && !mbar_wait_bounded(epi_done, (k - 1) & 1, abort_flag, errs, kErrAttnWait, 18)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t q_addr = smem_u32(smem + C::QD_OFF + st * 2 * C::TILE);
          const uint32_t do_addr = q_addr + C::TILE;
          const uint32_t dst_addr = smem_u32(smem + C::DST_OFF + b * 128 * 128 * 2);
          // the next block's scores first: its softmax then overlaps this block's dV / dK / dQ
          if (it + 1 < n_it && !issue_scores(g + 1)) {
            ok = false;
            break;
          }
          // dV += P^T dO: P^T from its own tensor-memory columns (query columns packed two per
          // column), dO MN-major
          const uint64_t d_do = smem_desc_sw128(do_addr, 16384, 1024);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            tc_mma_f16_ts(tmem + C::T_DV, tmem + C::T_PT + ks * 8, d_do + ks * (2048 >> 4), ID_KV,
                          (it > 0 || ks > 0) ? 1u : 0u);
          tc_commit(pt_free);
          // dK += dS^T Q (A = dS^T K-major, B = Q MN-major)
          const uint64_t d_ds = smem_desc_sw128(dst_addr, 16, 1024);
          const uint64_t d_q = smem_desc_sw128(q_addr, 16384, 1024);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint32_t aoff = (ks >> 2) * 16384 + (ks & 3) * 32;
            tc_mma_f16(tmem + C::T_DK, d_ds + (aoff >> 4), d_q + ks * (2048 >> 4), ID_KV,
                       (it > 0 || ks > 0) ? 1u : 0u);
          }
          // dQ = dS K, once the previous block's dQ has been read out
          if (g >= 1 && !mbar_wait_bounded(dq_free, (g - 1) & 1, abort_flag, errs, kErrAttnWait, 15)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t d_dsq = smem_desc_sw128(dst_addr, 16384, 1024);
          const uint64_t d_k = smem_desc_sw128(k_addr, 16384, 1024);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            tc_mma_f16(tmem + C::T_DQ, d_dsq + ks * (2048 >> 4), d_k + ks * (2048 >> 4), ID_Q, ks > 0 ? 1u : 0u);
          tc_commit(dq_full);
          tc_commit(&q_empty[st]);
        }
        if (!ok) break;
        tc_commit(kv_empty);  // K_j / V_j no longer read once this item's MMAs complete
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(C::REGS_HIGH));
    const int wg = (warp - 4) >> 2;  // query columns [64*wg, 64*wg + 64) of S^T / dP^T
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;    // kv row for S^T / dK / dV; query row for dQ
    const int col0 = wg * 64;
    const uint32_t lane_base = tmem + ((uint32_t)(q4 * 32) << 16);
    const float scale2 = p.scale * 1.4426950408889634f;
    uint8_t* stg = smem + C::STG_OFF + (warp - 4) * 2 * kBwdChunk;
    int g = 0;
    bool ok = true;
    // dQ of iteration gq (query block i, head h) -> scaled fp32 TMA add-reductions into dq_acc
    auto dq_readout = [&](int gq, int h, int i, int row0) -> bool {
      if (!mbar_wait_bounded(dq_full, gq & 1, abort_flag, errs, kErrAttnWait, 17)) return false;
      tc_fence_after();
      if (lane == 0) bulk_wait_group_read<0>();  // both staging chunks of this warp are free
      __syncwarp();
#pragma unroll
      for (int hc = 0; hc < 2; ++hc) {
        uint32_t qv[16];
        tmem_ld_32x32b_x16(lane_base + C::T_DQ + wg * 32 + 16 * hc, qv);
        tc_wait_ld();
        uint8_t* buf = stg + hc * kBwdChunk;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int off = lane * 64 + ((jj ^ ((lane >> 1) & 3)) << 4);
          *reinterpret_cast<float4*>(buf + off) =
              make_float4(__uint_as_float(qv[4 * jj]) * p.scale, __uint_as_float(qv[4 * jj + 1]) * p.scale,
                          __uint_as_float(qv[4 * jj + 2]) * p.scale, __uint_as_float(qv[4 * jj + 3]) * p.scale);
        }
      }
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(dq_free);
#pragma unroll
        for (int hc = 0; hc < 2; ++hc)
          tma_reduce_add_2d(&tm_dq, stg + hc * kBwdChunk, h * HD + wg * 32 + 16 * hc, row0 + i * 128 + q4 * 32);
        bulk_commit_group();
      }
      return true;
    };
    for (int k = 0, u; ok && (u = bwd_item_index(k, cta, G, n_items)) >= 0; ++k) {
      const BwdItem w = bwd_item(u, p.batch, p.kv_heads);
      const int n_q = n_qb - w.j;
      const int n_it = group * n_q;
      const int row0 = w.b * p.seq;
      for (int it = 0; it < n_it; ++it, ++g) {
        const int i = w.j + it % n_q;
        if (!mbar_wait_bounded(st_full, g & 1, abort_flag, errs, kErrAttnWait, 16)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const bool diag = (i == w.j);
        const float* lds = reinterpret_cast<const float*>(smem + C::LD_OFF + (g % C::STAGES) * 1024);
        uint8_t* dst = smem + C::DST_OFF + (g & 1) * 128 * 128 * 2;
        uint32_t ppk[32];  // this thread's 64 bf16 probabilities, packed in pairs
#pragma unroll
        for (int c = 0; c < 64; c += 32) {
          uint32_t sv[32], dpv[32];
          tmem_ld_32x32b_x32(lane_base + C::T_ST + col0 + c, sv);
          tmem_ld_32x32b_x32(lane_base + C::T_DPT + col0 + c, dpv);
          float lse_v[32], del_v[32];  // this chunk's query columns: shared-memory broadcasts, 16 B each
          const float4* l4 = reinterpret_cast<const float4*>(lds + col0 + c);
          const float4* d4 = reinterpret_cast<const float4*>(lds + 128 + col0 + c);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float4 a = l4[e], dd = d4[e];
            lse_v[4 * e] = a.x; lse_v[4 * e + 1] = a.y; lse_v[4 * e + 2] = a.z; lse_v[4 * e + 3] = a.w;
            del_v[4 * e] = dd.x; del_v[4 * e + 1] = dd.y; del_v[4 * e + 2] = dd.z; del_v[4 * e + 3] = dd.w;
          }
          tc_wait_ld();
          if (diag) {  // key row r sees query columns >= r only: masked scores exponentiate to 0
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (col0 + c + e < r) sv[e] = __float_as_uint(-INFINITY);
          }
          uint32_t dk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            float pv[2], dv[2];
            if constexpr (EMU == 4) {  // one MUFU operation for the pair (fp16 inputs)
              ex2_pair_f16(fmaf(__uint_as_float(sv[e]), scale2, -lse_v[e]),
                           fmaf(__uint_as_float(sv[e + 1]), scale2, -lse_v[e + 1]), pv[0], pv[1]);
            } else {
#pragma unroll
              for (int t = 0; t < 2; ++t) {
                const float x = fmaf(__uint_as_float(sv[e + t]), scale2, -lse_v[e + t]);
                // (the FMA-pipe exp2 gives 2^-125 for a masked score: nothing at bf16 precision)
                pv[t] = (((e + t) & 7) >= 8 - EMU) ? exp2_fma(x) : ex2_approx(x);
              }
            }
#pragma unroll
            for (int t = 0; t < 2; ++t) dv[t] = pv[t] * (__uint_as_float(dpv[e + t]) - del_v[e + t]);
            ppk[(c + e) >> 1] = pack_bf16(pv[0], pv[1]);
            dk[e >> 1] = pack_bf16(dv[0], dv[1]);
          }
          store_swizzled_row(dst, r, col0 + c, dk);
        }
        // P^T into its own columns (this warpgroup's 64 query columns packed into 32), once dV of the
        // previous block has read them
        if (g >= 1 && !mbar_wait_bounded(pt_free, (g - 1) & 1, abort_flag, errs, kErrAttnWait, 19)) {
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_st_32x32b_x32(lane_base + C::T_PT + wg * 32, ppk);
        tc_wait_st();
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_ready);
        if (it > 0) {  // dQ of the previous block, read out one iteration late
          const int ip = w.j + (it - 1) % n_q;
          const int hp = w.kvh * group + (it - 1) / n_q;
          if (!dq_readout(g - 1, hp, ip, row0)) {
            ok = false;
            break;
          }
        }
      }
      if (!ok) break;
      // the item's last dQ, then dK / dV (its last dq_full also covers the final dV / dK MMAs)
      if (!dq_readout(g - 1, w.kvh * group + (n_it - 1) / n_q, w.j + (n_it - 1) % n_q, row0)) break;
      const int kv_row = row0 + w.j * 128 + r;
      const int pos = w.j * 128 + r;
      constexpr int HALF = HD / 2;
      constexpr int QTR = HALF / 2;  // RoPE pairs per warpgroup
      __nv_bfloat16* dk_out = p.dqkv + (size_t)kv_row * p.ld + p.k_col + w.kvh * HD;
      __nv_bfloat16* dv_out = p.dqkv + (size_t)kv_row * p.ld + p.v_col + w.kvh * HD + wg * HALF;
      {
        uint32_t vv[32];
        tmem_ld_32x32b_x32(lane_base + C::T_DV + wg * HALF, vv);
        tc_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint4 o;
          o.x = pack_bf16(__uint_as_float(vv[e]), __uint_as_float(vv[e + 1]));
          o.y = pack_bf16(__uint_as_float(vv[e + 2]), __uint_as_float(vv[e + 3]));
          o.z = pack_bf16(__uint_as_float(vv[e + 4]), __uint_as_float(vv[e + 5]));
          o.w = pack_bf16(__uint_as_float(vv[e + 6]), __uint_as_float(vv[e + 7]));
          *reinterpret_cast<uint4*>(dv_out + e) = o;
        }
      }
      {
        const int c0 = wg * QTR;  // this warpgroup's RoPE pair range [c0, c0 + QTR)
        uint32_t lo[QTR], hi[QTR];
        tmem_ld_32x32b_x16(lane_base + C::T_DK + c0, lo);
        tmem_ld_32x32b_x16(lane_base + C::T_DK + HALF + c0, hi);
        tc_wait_ld();
        const float* cs = p.rope_cos + (size_t)pos * HALF + c0;
        const float* sn = p.rope_sin + (size_t)pos * HALF + c0;
#pragma unroll
        for (int e = 0; e < QTR; e += 8) {
          float a[8], bb[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const float x0 = __uint_as_float(lo[e + t]) * p.scale;
            const float x1 = __uint_as_float(hi[e + t]) * p.scale;
            const float cv = cs[e + t], sv = sn[e + t];
            a[t] = x0 * cv + x1 * sv;
            bb[t] = x1 * cv - x0 * sv;
          }
          uint4 wa, wb;
          wa.x = pack_bf16(a[0], a[1]); wa.y = pack_bf16(a[2], a[3]);
          wa.z = pack_bf16(a[4], a[5]); wa.w = pack_bf16(a[6], a[7]);
          wb.x = pack_bf16(bb[0], bb[1]); wb.y = pack_bf16(bb[2], bb[3]);
          wb.z = pack_bf16(bb[4], bb[5]); wb.w = pack_bf16(bb[6], bb[7]);
          *reinterpret_cast<uint4*>(dk_out + c0 + e) = wa;
          *reinterpret_cast<uint4*>(dk_out + HALF + c0 + e) = wb;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(epi_done);
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// delta[b, h, s] = sum_c dO[row, h*hd + c] * O[row, h*hd + c].  One warp per row: lane l takes the
// 16-byte column groups l, l+32, ...; a head spans hd/8 consecutive groups (8 or 16 lanes), reduced
// with butterfly shuffles inside that lane group, so every lane loads on every round.
template <int HD>
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout, int ld,
                                  float* __restrict__ delta, int rows, int seq, int heads) {
  pdl_wait_and_release();
  constexpr int G = HD / 8;  // lanes per head
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int groups = heads * G;
  const int b = row / seq, s = row % seq;
  for (int c0 = 0; c0 < groups; c0 += 32) {
    const int c = c0 + lane;
    float acc = 0.f;
    if (c < groups) {
      const uint4 qa = *reinterpret_cast<const uint4*>(o + (size_t)row * ld + c * 8);
      const uint4 qg = *reinterpret_cast<const uint4*>(dout + (size_t)row * ld + c * 8);
      const uint32_t wa[4] = {qa.x, qa.y, qa.z, qa.w}, wg[4] = {qg.x, qg.y, qg.z, qg.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) acc += bf16lo(wa[e]) * bf16lo(wg[e]) + bf16hi(wa[e]) * bf16hi(wg[e]);
    }
#pragma unroll
    for (int off = G / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (c < groups && (lane % G) == 0) delta[((size_t)b * heads + c / G) * seq + s] = acc;
  }
}

// q columns of dqkv = RoPE^T(dq_acc) in bf16; 8 consecutive pairs per thread.
__global__ void attn_dq_convert_kernel(const float* dq_acc, __nv_bfloat16* __restrict__ dqkv, int ld, int rows,
                                       int seq, int heads, int hd, const float* __restrict__ cosv,
                                       const float* __restrict__ sinv, bool rezero) {
  pdl_wait_and_release();
  const int half = hd / 2;
  const int groups = half / 8;
  const size_t total = (size_t)rows * heads * groups;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total; idx += (size_t)gridDim.x * blockDim.x) {
    const int row = (int)(idx / (heads * groups));
    const int rem = (int)(idx % (heads * groups));
    const int h = rem / groups, c = (rem % groups) * 8;
    const int pos = row % seq;
    const float* src = dq_acc + (size_t)row * heads * hd + h * hd;
    const float4 a0 = *reinterpret_cast<const float4*>(src + c), a1 = *reinterpret_cast<const float4*>(src + c + 4);
    const float4 b0 = *reinterpret_cast<const float4*>(src + half + c);
    const float4 b1 = *reinterpret_cast<const float4*>(src + half + c + 4);
    const float x0[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const float x1[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    if (rezero) {  // leave the accumulator zeroed for the next backward that reuses it
      float* w = const_cast<float*>(src);
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(w + c) = z;
      *reinterpret_cast<float4*>(w + c + 4) = z;
      *reinterpret_cast<float4*>(w + half + c) = z;
      *reinterpret_cast<float4*>(w + half + c + 4) = z;
    }
    float lo[8], hi[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const float cv = cosv[(size_t)pos * half + c + t], sv = sinv[(size_t)pos * half + c + t];
      lo[t] = x0[t] * cv + x1[t] * sv;
      hi[t] = x1[t] * cv - x0[t] * sv;
    }
    __nv_bfloat16* out = dqkv + (size_t)row * ld + h * hd;
    uint4 wl, wh;
    wl.x = pack_bf16(lo[0], lo[1]); wl.y = pack_bf16(lo[2], lo[3]);
    wl.z = pack_bf16(lo[4], lo[5]); wl.w = pack_bf16(lo[6], lo[7]);
    wh.x = pack_bf16(hi[0], hi[1]); wh.y = pack_bf16(hi[2], hi[3]);
    wh.z = pack_bf16(hi[4], hi[5]); wh.w = pack_bf16(hi[6], hi[7]);
    *reinterpret_cast<uint4*>(out + c) = wl;
    *reinterpret_cast<uint4*>(out + half + c) = wh;
  }
}

void launch_delta(const __nv_bfloat16* o, const __nv_bfloat16* dout, int ld, float* delta, int rows, int seq, int heads,
                  int hd, cudaStream_t s) {
  const int blocks = (rows * 32 + 255) / 256;
  if (hd == 64)
    launch_k(attn_delta_kernel<64>, dim3(blocks), dim3(256), 0, s, 1, o, dout, ld, delta, rows, seq, heads);
  else
    launch_k(attn_delta_kernel<128>, dim3(blocks), dim3(256), 0, s, 1, o, dout, ld, delta, rows, seq, heads);
  B200_CUDA_CHECK(cudaGetLastError());
}

// dq_acc as a TMA target: fp32 [rows, heads*hd], one 32-row x 16-column chunk per box.
CUtensorMap make_dq_map(const AttnBwdParams& p) {
  const int rows = p.batch * p.seq, cols = p.heads * p.head_dim;
  return make_tmap_2d(CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.dq_acc, (uint64_t)cols, (uint64_t)rows, (uint64_t)cols, 16,
                      32, CU_TENSOR_MAP_SWIZZLE_64B);
}

int bwd_grid(const AttnBwdParams& p) {
  const int items = p.batch * p.kv_heads * (p.seq / 128);
  return std::max(1, std::min(items, num_sms_cached()));
}

// ZB_ATTN_BWD_EMU=0..3 overrides the share of FMA-pipe exponentials (eighths of the columns), 4 selects
// half-precision pairs (one MUFU operation per two exponentials); for tuning.
int bwd_emu_override() {
  static const int v = [] {
    const char* e = std::getenv("ZB_ATTN_BWD_EMU");
    return (e != nullptr && *e >= '0' && *e <= '4' && e[1] == 0) ? (*e - '0') : -1;
  }();
  return v;
}

// Raise the dynamic shared-memory limit of every hd-64 variant (a per-device attribute).
cudaError_t set_bwd64_smem_limits() {
  cudaError_t e = cudaSuccess;
  void (*variants[5])(CUtensorMap, CUtensorMap, CUtensorMap, AttnBwdParams, DeviceErrors*) = {
      attn_bwd_hd64_kernel<0>, attn_bwd_hd64_kernel<1>, attn_bwd_hd64_kernel<2>, attn_bwd_hd64_kernel<3>,
      attn_bwd_hd64_kernel<4>};
  for (auto k : variants)
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnBwd64Cfg::SMEM_BYTES);
  return e;
}

// head_dim 64 runs the software-pipelined kernel, 128 the original one.
template <int HD>
void launch_bwd(const AttnBwdParams& p, const CUtensorMap& tq, const CUtensorMap& tdo, const CUtensorMap& tdq,
                DeviceErrors* errs, cudaStream_t s) {
  if constexpr (HD == 64) {
    auto kernel = attn_bwd_hd64_kernel<AttnBwd64Cfg::EMU>;
    switch (bwd_emu_override()) {
      case 0: kernel = attn_bwd_hd64_kernel<0>; break;
      case 1: kernel = attn_bwd_hd64_kernel<1>; break;
      case 2: kernel = attn_bwd_hd64_kernel<2>; break;
      case 3: kernel = attn_bwd_hd64_kernel<3>; break;
      case 4: kernel = attn_bwd_hd64_kernel<4>; break;
      default: break;
    }
    launch_k(kernel, dim3(bwd_grid(p)), dim3(AttnBwd64Cfg::THREADS), AttnBwd64Cfg::SMEM_BYTES, s, 1, tq, tdo, tdq, p,
             errs);
  } else {
    using C = AttnBwdCfg<HD>;
    launch_k(attn_bwd_kernel<HD>, dim3(bwd_grid(p)), dim3(BWD_THREADS), C::SMEM_BYTES, s, 1, tq, tdo, tdq, p, errs);
  }
}

}  // namespace

void attention_bwd(const AttnBwdParams& p, cudaStream_t s) {
  B200_CHECK(p.head_dim == 64 || p.head_dim == 128, "attention_bwd: head_dim must be 64 or 128");
  B200_CHECK(p.seq % 128 == 0, "attention_bwd: seq_len must be a multiple of 128");
  B200_CHECK(p.rope_cos != nullptr && p.rope_sin != nullptr, "attention_bwd: RoPE tables required");
  const int rows = p.batch * p.seq;
  launch_delta(p.out, p.dout, p.ld_out, p.delta, rows, p.seq, p.heads, p.head_dim, s);
  CUtensorMap tq = make_tmap_bf16_2d(p.qkv, (uint64_t)p.ld, (uint64_t)rows, (uint64_t)p.ld, 64, 128);
  CUtensorMap tdo = make_tmap_bf16_2d(p.dout, (uint64_t)p.ld_out, (uint64_t)rows, (uint64_t)p.ld_out, 64, 128);
  CUtensorMap tdq = make_dq_map(p);
  static std::atomic<unsigned long long> configured{0};
  once_per_device(configured, [] {
    B200_CUDA_CHECK(set_bwd64_smem_limits());
    B200_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         AttnBwdCfg<128>::SMEM_BYTES));
  });
  if (p.head_dim == 64)
    launch_bwd<64>(p, tq, tdo, tdq, device_errors_ptr(), s);
  else
    launch_bwd<128>(p, tq, tdo, tdq, device_errors_ptr(), s);
  B200_CUDA_CHECK(cudaGetLastError());
  const size_t work = (size_t)rows * p.heads * (p.head_dim / 16);
  const int blocks = (int)std::min<size_t>((work + 255) / 256, (size_t)num_sms_cached() * 16);
  launch_k(attn_dq_convert_kernel, dim3(blocks), dim3(256), 0, s, 1, (const float*)p.dq_acc, p.dqkv, p.ld, rows, p.seq,
           p.heads, p.head_dim, p.rope_cos, p.rope_sin, p.rezero_dq_acc);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch(3);
}

// ---------------------------------------------------------------------------------------------
// Allocation-free variant (declared in attention_bwd_noalloc.h, which documents the contract).
// The scratch that the regular path takes from its caller (error record, delta, dQ accumulator)
// lives in one fixed device array; host code reaches it only through the address returned by
// cudaGetSymbolAddress, because the array's name in host code is a host-side stand-in.
// ---------------------------------------------------------------------------------------------
namespace {

static __device__ __align__(256) unsigned char g_attn_bwd_scratch[B200_ATTN_BWD_NOALLOC_SCRATCH_BYTES];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
unsigned char* g_noalloc_scratch_addr[kNoAllocMaxDevices] = {};  // device address of the array, per device

constexpr size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Once per device, with that device current: resolve the array's device address and raise the
// bwd kernels' dynamic shared-memory limit.  Returns nullptr (after printing why) on failure.
unsigned char* noalloc_scratch_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_scratch_addr[dev] != nullptr) return g_noalloc_scratch_addr[dev];
  void* addr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&addr, g_attn_bwd_scratch);
  if (e != cudaSuccess || addr == nullptr) {
    std::fprintf(stderr, "b200_attention_bwd_noalloc: cudaGetSymbolAddress failed on device %d: %s\n", dev,
                 cudaGetErrorString(e));
    return nullptr;
  }
  e = set_bwd64_smem_limits();
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_bwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             AttnBwdCfg<128>::SMEM_BYTES);
  if (e != cudaSuccess) {
    std::fprintf(stderr, "b200_attention_bwd_noalloc: cudaFuncSetAttribute failed: %s\n", cudaGetErrorString(e));
    return nullptr;
  }
  g_noalloc_scratch_addr[dev] = static_cast<unsigned char*>(addr);
  return g_noalloc_scratch_addr[dev];
}

}  // namespace

}  // namespace b200

extern "C" int b200_attention_bwd_noalloc(const void* qkv, int ld, int k_col, int v_col, const void* out,
                                          const void* dout, int ld_out, const float* lse, void* dqkv,
                                          const float* rope_cos, const float* rope_sin, int batch, int seq, int heads,
                                          int kv_heads, int head_dim, float scale, cudaStream_t stream) {
  using namespace b200;
  const auto aligned16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (qkv == nullptr || out == nullptr || dout == nullptr || lse == nullptr || dqkv == nullptr ||
      rope_cos == nullptr || rope_sin == nullptr || !aligned16(qkv) || !aligned16(out) || !aligned16(dout) ||
      !aligned16(dqkv) || !aligned16(lse) || (head_dim != 64 && head_dim != 128) || batch <= 0 || seq <= 0 ||
      seq % 128 != 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 || ld % 8 != 0 || ld_out % 8 != 0 ||
      k_col % 64 != 0 || v_col % 64 != 0) {
    std::fprintf(stderr, "b200_attention_bwd_noalloc: invalid arguments (head_dim must be 64 or 128, seq a multiple "
                         "of 128, heads a multiple of kv_heads, pointers 16-byte aligned)\n");
    return B200_NOALLOC_ERR_INVALID;
  }
  // Column extents: q, k and v must each fit before the next block and inside the row; the output
  // rows must hold every query head.
  const long long q_w = (long long)heads * head_dim, kv_w = (long long)kv_heads * head_dim;
  if (q_w > k_col || k_col + kv_w > v_col || v_col + kv_w > ld || q_w > ld_out) {
    std::fprintf(stderr,
                 "b200_attention_bwd_noalloc: column layout does not fit (need heads*head_dim <= k_col, "
                 "k_col + kv_heads*head_dim <= v_col, v_col + kv_heads*head_dim <= ld, heads*head_dim <= ld_out)\n");
    return B200_NOALLOC_ERR_INVALID;
  }
  // The scratch address is per device: the stream must belong to the current device.
  {
    int cur = 0, sdev = 0;
    if (cudaGetDevice(&cur) != cudaSuccess) return B200_NOALLOC_ERR_CUDA;
    if (stream != nullptr) {
      if (cudaStreamGetDevice(stream, &sdev) != cudaSuccess) return B200_NOALLOC_ERR_CUDA;
      if (sdev != cur) {
        std::fprintf(stderr, "b200_attention_bwd_noalloc: stream belongs to device %d but device %d is current\n",
                     sdev, cur);
        return B200_NOALLOC_ERR_INVALID;
      }
    }
  }
  const size_t rows = (size_t)batch * seq;
  const size_t err_bytes = align256(sizeof(DeviceErrors));
  const size_t delta_bytes = align256((size_t)batch * heads * seq * sizeof(float));
  const size_t dq_bytes = align256(rows * heads * head_dim * sizeof(float));
  const size_t need = err_bytes + delta_bytes + dq_bytes;
  if (need > B200_ATTN_BWD_NOALLOC_SCRATCH_BYTES) {
    std::fprintf(stderr,
                 "b200_attention_bwd_noalloc: problem needs %zu bytes of scratch but the fixed array holds %u "
                 "(batch=%d seq=%d heads=%d head_dim=%d); use the regular attention backward instead\n",
                 need, (unsigned)B200_ATTN_BWD_NOALLOC_SCRATCH_BYTES, batch, seq, heads, head_dim);
    return B200_NOALLOC_ERR_TOO_LARGE;
  }
  unsigned char* scratch = noalloc_scratch_for_current_device();
  if (scratch == nullptr) return B200_NOALLOC_ERR_CUDA;
  auto* errs = reinterpret_cast<DeviceErrors*>(scratch);
  float* delta = reinterpret_cast<float*>(scratch + err_bytes);
  float* dq_acc = reinterpret_cast<float*>(scratch + err_bytes + delta_bytes);
  try {
    // The error record and the dQ accumulator must start at zero; delta is fully overwritten.
    if (cudaMemsetAsync(errs, 0, sizeof(DeviceErrors), stream) != cudaSuccess ||
        cudaMemsetAsync(dq_acc, 0, rows * heads * head_dim * sizeof(float), stream) != cudaSuccess)
      return B200_NOALLOC_ERR_CUDA;
    AttnBwdParams p{};
    p.qkv = static_cast<const __nv_bfloat16*>(qkv);
    p.ld = ld;
    p.k_col = k_col;
    p.v_col = v_col;
    p.out = static_cast<const __nv_bfloat16*>(out);
    p.dout = static_cast<const __nv_bfloat16*>(dout);
    p.ld_out = ld_out;
    p.lse = lse;
    p.delta = delta;
    p.dq_acc = dq_acc;
    p.dqkv = static_cast<__nv_bfloat16*>(dqkv);
    p.rope_cos = rope_cos;
    p.rope_sin = rope_sin;
    p.batch = batch;
    p.seq = seq;
    p.heads = heads;
    p.kv_heads = kv_heads;
    p.head_dim = head_dim;
    p.scale = scale;
    launch_delta(p.out, p.dout, p.ld_out, p.delta, (int)rows, seq, heads, head_dim, stream);
    const CUtensorMap tq = make_tmap_bf16_2d(p.qkv, (uint64_t)ld, (uint64_t)rows, (uint64_t)ld, 64, 128);
    const CUtensorMap tdo = make_tmap_bf16_2d(p.dout, (uint64_t)ld_out, (uint64_t)rows, (uint64_t)ld_out, 64, 128);
    const CUtensorMap tdq = make_dq_map(p);
    if (head_dim == 64)
      launch_bwd<64>(p, tq, tdo, tdq, errs, stream);
    else
      launch_bwd<128>(p, tq, tdo, tdq, errs, stream);
    const size_t work = rows * heads * (head_dim / 16);
    const int blocks = (int)std::min<size_t>((work + 255) / 256, (size_t)num_sms_cached() * 16);
    launch_k(attn_dq_convert_kernel, dim3(blocks), dim3(256), 0, stream, 1, (const float*)dq_acc, p.dqkv, ld, (int)rows,
             seq, heads, head_dim, rope_cos, rope_sin, false);
    count_launch(3);
  } catch (const std::exception& ex) {
    std::fprintf(stderr, "b200_attention_bwd_noalloc: %s\n", ex.what());
    return B200_NOALLOC_ERR_INVALID;
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    std::fprintf(stderr, "b200_attention_bwd_noalloc: launch failed: %s\n", cudaGetErrorString(e));
    return B200_NOALLOC_ERR_CUDA;
  }
  return B200_NOALLOC_OK;
}

extern "C" int b200_attention_bwd_noalloc_last_error(int* record4) {
  using namespace b200;
  if (record4 == nullptr) return B200_NOALLOC_ERR_INVALID;
  unsigned char* scratch = noalloc_scratch_for_current_device();
  if (scratch == nullptr) return B200_NOALLOC_ERR_CUDA;
  DeviceErrors rec{};
  const cudaError_t e = cudaMemcpy(&rec, scratch, sizeof(DeviceErrors), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    std::fprintf(stderr, "b200_attention_bwd_noalloc_last_error: %s\n", cudaGetErrorString(e));
    return B200_NOALLOC_ERR_CUDA;
  }
  record4[0] = rec.code;
  record4[1] = rec.where;
  record4[2] = rec.block;
  record4[3] = rec.count;
  return B200_NOALLOC_OK;
}
