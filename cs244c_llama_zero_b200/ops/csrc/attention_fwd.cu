// Causal GQA flash-attention forward on the 5th-generation tensor cores (sm_100a).
//
// Persistent: one CTA per SM walks a longest-first list of work items.  An item is a PAIR of
// query tiles (rows [256p, 256p + 128) = tile A and [256p + 128, 256p + 256) = tile B) of one query
// head and batch; the two tiles share every key/value tile both need and are processed ping-pong,
// so the tensor cores work on one tile while the softmax warps work on the other.
//
// 384 threads (three warpgroups; the first hands registers to the other two with setmaxnreg):
//   warp 0      TMA producer: the item's two Q tiles, then K_j / V_j tiles into a STAGES-deep ring.
//               Q, K and V are column blocks of the fused [B*S, ld] q|k|v projection output, so one
//               tensor map serves all three and K/V are never repeated for grouped heads: query head
//               h reads kv head h / (H / KV).
//   warp 1      allocates the 512 tensor-memory columns; lane 0 issues the MMAs:
//                 S_t = Q_t K_j^T   (M = 128, N = 128, K = hd; A and B from shared memory)
//                 O_t += P_t V_j    (M = 128, N = hd, K = 128; A = P_t from TENSOR memory, B = V_j)
//               in the order S_A(0) S_B(0) | PV_A(j) S_A(j+1) PV_B(j) S_B(j+1) | ..., so while the
//               softmax warps of tile A work on S_A(j+1), the tensor cores run PV_B(j) and S_B(j+1).
//   warps 2, 3  idle after set-up.
//   warps 4..7  softmax of tile A, warps 8..11 softmax of tile B: ONE THREAD PER QUERY ROW.  The thread
//               reads its row's 128 scores from tensor memory into registers (no cross-thread max
//               exchange), exponentiates in the base-2 domain (a share of the columns on the FMA pipe
//               through exp2_fma, the rest on MUFU), writes the bf16 probabilities back into the
//               same tensor-memory columns (P aliases S: the PV MMA reads them from there), and keeps
//               the row sum.  The running maximum is raised lazily: O is rescaled (read, scaled and
//               written back in tensor memory by the same thread) only when a new score exceeds the
//               maximum in use by more than 2^8, so most blocks skip the correction.
// At the end of its tile the thread reads O, divides by the row sum and stores bf16; the row's
// log-sum-exp is stored in base-2 units scaled by log2(e)/sqrt(hd), from which the backward pass
// rebuilds P with one exp2.
//
// Tensor memory: S_A [0,128) | S_B [128,256) | O_A [256, 256+hd) | O_B [256+hd, 256+2hd).
// Ordering facts used: tcgen05.mma of one thread execute in issue order, so S_t(j+1) (which writes
// the columns P_t(j) occupies) runs after PV_t(j) has read them, and the commit after S_t(j+1)
// also covers PV_t(j): a softmax thread that sees S_t(j+1) may read and rescale O_t.
#include <cuda.h>

#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "gemm.h"
#include "kernels.h"

namespace b200 {

namespace {

constexpr int ATT_THREADS = 384;
// Register split (setmaxnreg): the launch gives 168 per thread (384 x 168 = 64512); the producer /
// MMA warpgroup drops to REGS_LOW and the two softmax warpgroups rise to REGS_HIGH, with
// 128 * REGS_LOW + 256 * REGS_HIGH <= 64512 (checked in AttnFwdCfg).
constexpr int kLaunchRegs = 168;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when the max grows by > 2^8
// EMU value selecting the half-precision-pair exponential (two results per MUFU operation) instead of
// an fp32 MUFU / FMA-polynomial split.
constexpr int kEmuHalfPairs = 4;

template <int HD>
struct AttnFwdCfg {
  static constexpr int KB = HD / 64;                 // 64-column swizzle blocks per row
  static constexpr int TILE_BYTES = 128 * HD * 2;    // one 128-row tile of Q, K or V
  static constexpr int STAGES = (HD == 64) ? 3 : 2;  // K/V ring
  static constexpr int Q_BUFS = (HD == 64) ? 2 : 1;  // Q pairs: the next item's Q loads during this one
  // Default share of the exponentials done on the FMA pipe (columns c with (c & 7) >= 8 - EMU; the
  // kernel is instantiated for 0..3).  Measured on B200 at the benchmark shape: 0 (all on MUFU) is
  // fastest for hd 64 (43.0 us vs 45.1 / 45.1 / 47.1 us for 1 / 2 / 3): the softmax is bound by
  // issue and latency, not by the MUFU rate, so the 9-instruction polynomial only adds work.
  static constexpr int EMU = (HD == 64) ? 0 : 1;
  static constexpr int REGS_LOW = (HD == 64) ? 64 : 88;
  static constexpr int REGS_HIGH = (HD == 64) ? 216 : 208;
  static_assert(128 * REGS_LOW + 256 * REGS_HIGH <= ATT_THREADS * kLaunchRegs, "register split over budget");
  // hd 64: the row sums come from the tensor cores.  Each ring stage holds K, V and a 16 KB block of
  // bf16 ones right after V, so the PV MMA runs with N = hd + 16 over [V | 1] and column hd of O
  // accumulates sum_k P[r, k] (the same bf16 P that O sums, rescaled with O) - no per-element adds.
  // hd 128 has no tensor-memory room for the extra columns and adds the sums in registers.
  static constexpr bool ONES = (HD == 64);
  static constexpr int O_COLS = ONES ? HD + 16 : HD;  // O columns per tile in tensor memory
  static constexpr int STAGE_BYTES = (ONES ? 3 : 2) * TILE_BYTES;
  static constexpr int Q_OFF = 0;
  static constexpr int KV_OFF = Q_BUFS * 2 * TILE_BYTES;
  static constexpr int BAR_OFF = KV_OFF + STAGES * STAGE_BYTES;
  static constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;
  static_assert(SMEM_BYTES <= 232448, "attention forward shared memory exceeds 227 KB");
  static constexpr int TMEM_COLS = 512;
  static constexpr int T_S = 0;      // + 128 * tile
  static constexpr int T_O = 256;    // + O_COLS * tile
  static_assert(T_O + 2 * O_COLS <= TMEM_COLS, "attention forward tensor memory");
};

// Work items are (query-tile pair, head, batch), numbered longest first (pair index n_pairs - 1
// first).  CTA c of G takes items c, 2G - 1 - c, 2G + c, ... (boustrophedon deal), so every CTA's
// list runs from long to short and the totals even out.
struct FwdItem {
  int pair, h, b;
};
__device__ __forceinline__ int fwd_item_index(int k, int c, int G, int n_items) {
  const int u = k * G + ((k & 1) ? (G - 1 - c) : c);
  return u < n_items ? u : -1;
}
__device__ __forceinline__ FwdItem fwd_item(int u, int n_pairs, int heads, int batch) {
  const int per = heads * batch;
  const int r = u % per;
  return {n_pairs - 1 - u / per, r % heads, r / heads};
}
// Number of key/value blocks tile t (0 = A, 1 = B) of pair `pair` attends to; 0 if the tile lies
// past the sequence end (odd number of 128-row blocks).
__device__ __forceinline__ int tile_kv_blocks(int pair, int t, int n_qb) {
  const int qb = 2 * pair + t;
  return qb < n_qb ? qb + 1 : 0;
}

// Debug phase clocks (ZB_ATTN_TRACE=1): role r of CTA 0 appends (event, clock64) pairs.
__device__ __forceinline__ void trace_ev(const AttnParams& p, int role, int& n, int ev) {
  if (p.trace != nullptr && blockIdx.x == 0 && n < kAttnTraceWords / 2) {
    p.trace[role * kAttnTraceWords + 2 * n] = (unsigned long long)ev;
    p.trace[role * kAttnTraceWords + 2 * n + 1] = clock64();
    ++n;
  }
}

template <int HD, int EMU>
__global__ void __launch_bounds__(ATT_THREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm, AttnParams p, DeviceErrors* errs) {
  using C = AttnFwdCfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars;                 // [Q_BUFS]
  uint64_t* q_empty = q_full + C::Q_BUFS;  // [Q_BUFS]
  uint64_t* kv_full = q_empty + C::Q_BUFS;
  uint64_t* kv_empty = kv_full + C::STAGES;
  uint64_t* s_full = kv_empty + C::STAGES;  // [2 tiles]
  uint64_t* p_full = s_full + 2;            // [2 tiles], 4 warps each
  uint64_t* o_done = p_full + 2;            // [2 tiles]: the tile's last PV of the item completed
  uint64_t* o_free = o_done + 2;            // [2 tiles], 4 warps: the epilogue has read O
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_free + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qb = p.seq / 128;
  const int n_pairs = (n_qb + 1) / 2;
  const int n_items = n_pairs * p.heads * p.batch;
  const int G = gridDim.x, c = blockIdx.x;
  const int group = p.heads / p.kv_heads;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::Q_BUFS; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_done[t], 1);
      mbar_init(&o_free[t], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  if constexpr (C::ONES) {  // the ones block after every V tile (never written by TMA)
    for (int st = 0; st < C::STAGES; ++st) {
      uint4* ones = reinterpret_cast<uint4*>(smem + C::KV_OFF + st * C::STAGE_BYTES + 2 * C::TILE_BYTES);
      for (int i = threadIdx.x; i < C::TILE_BYTES / 16; i += ATT_THREADS)
        ones[i] = make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);
    }
    fence_proxy_async_smem();  // generic-proxy writes read by the tensor cores
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait_and_release();  // q|k|v come from the previous kernel of the stream

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::REGS_LOW));
    if (warp == 0 && lane == 0) {
      tma_prefetch_desc(&tm);
      int g = 0;  // global key/value block counter (ring position)
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int u = fwd_item_index(k, c, G, n_items);
        if (u < 0) break;
        const FwdItem it = fwd_item(u, n_pairs, p.heads, p.batch);
        const int row0 = it.b * p.seq;
        const int kvh = it.h / group;
        const int nA = tile_kv_blocks(it.pair, 0, n_qb), nB = tile_kv_blocks(it.pair, 1, n_qb);
        const int qs = k % C::Q_BUFS;
        // The slot's previous Q pair is free once every score MMA of that item has completed.
        if (k >= C::Q_BUFS &&
            !mbar_wait_bounded(&q_empty[qs], ((k / C::Q_BUFS) - 1) & 1, abort_flag, errs, kErrAttnWait, 10))
          break;
        uint8_t* qbase = smem + C::Q_OFF + qs * 2 * C::TILE_BYTES;
        const int n_tiles = nB > 0 ? 2 : 1;
        mbar_expect_tx(&q_full[qs], n_tiles * C::TILE_BYTES);
        for (int t = 0; t < n_tiles; ++t)
#pragma unroll
          for (int kb = 0; kb < C::KB; ++kb)
            tma_load_2d(qbase + t * C::TILE_BYTES + kb * 16384, &tm, &q_full[qs], it.h * HD + 64 * kb,
                        row0 + (2 * it.pair + t) * 128);
        const int nkv = max(nA, nB);
        for (int j = 0; j < nkv; ++j, ++g) {
          const int st = g % C::STAGES;
          if (!mbar_wait_bounded(&kv_empty[st], ((g / C::STAGES) & 1) ^ 1u, abort_flag, errs, kErrAttnWait, 0)) {
            ok = false;
            break;
          }
          uint8_t* ks = smem + C::KV_OFF + st * C::STAGE_BYTES;
          uint8_t* vs = ks + C::TILE_BYTES;
          mbar_expect_tx(&kv_full[st], 2 * C::TILE_BYTES);
#pragma unroll
          for (int kb = 0; kb < C::KB; ++kb) {
            tma_load_2d(ks + kb * 16384, &tm, &kv_full[st], p.k_col + kvh * HD + 64 * kb, row0 + j * 128);
            tma_load_2d(vs + kb * 16384, &tm, &kv_full[st], p.v_col + kvh * HD + 64 * kb, row0 + j * 128);
          }
        }
      }
    } else if (warp == 1 && lane == 0) {
      constexpr uint32_t IDESC_S = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t IDESC_O = idesc_bf16_f32(128, C::O_COLS, false, true);
      int g = 0;             // global key/value block counter
      int tn = 0;            // trace entries
      int pn[2] = {0, 0};    // P handed over per tile (p_full phases)
      int on[2] = {0, 0};    // items finished per tile (o_done / o_free phases)
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int u = fwd_item_index(k, c, G, n_items);
        if (u < 0) break;
        const FwdItem it = fwd_item(u, n_pairs, p.heads, p.batch);
        const int n[2] = {tile_kv_blocks(it.pair, 0, n_qb), tile_kv_blocks(it.pair, 1, n_qb)};
        const int nkv = max(n[0], n[1]);
        const int qs = k % C::Q_BUFS;
        const uint32_t q_addr = smem_u32(smem + C::Q_OFF + qs * 2 * C::TILE_BYTES);
        if (!mbar_wait_bounded(&q_full[qs], (k / C::Q_BUFS) & 1, abort_flag, errs, kErrAttnWait, 2)) break;
        // S_t = Q_t K^T for the K tile in ring stage st
        auto issue_s = [&](int t, int st) {
          // descriptors built once; a k-step moves the start-address field (bytes >> 4, no carry:
          // shared addresses stay below 2^18)
          const uint64_t dq = smem_desc_sw128(q_addr + t * C::TILE_BYTES, 16, 1024);
          const uint64_t dk = smem_desc_sw128(smem_u32(smem + C::KV_OFF + st * C::STAGE_BYTES), 16, 1024);
#pragma unroll
          for (int ks = 0; ks < HD / 16; ++ks) {
            const uint64_t off = ((ks >> 2) * 16384 + (ks & 3) * 32) >> 4;
            tc_mma_f16(tmem + C::T_S + t * 128, dq + off, dk + off, IDESC_S, ks > 0 ? 1u : 0u);
          }
          tc_commit(&s_full[t]);
        };
        int st = g % C::STAGES;
        if (!mbar_wait_bounded(&kv_full[st], (g / C::STAGES) & 1, abort_flag, errs, kErrAttnWait, 1)) break;
        tc_fence_after();
#pragma unroll
        for (int t = 0; t < 2; ++t)
          if (n[t] > 0) issue_s(t, st);
        for (int j = 0; ok && j < nkv; ++j) {
          st = (g + j) % C::STAGES;
          const int st1 = (g + j + 1) % C::STAGES;
          bool next_loaded = false;
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (!ok) break;
            if (j >= n[t]) continue;
            trace_ev(p, 0, tn, 10 + t);
            if (!mbar_wait_bounded(&p_full[t], pn[t] & 1, abort_flag, errs, kErrAttnWait, 3 + t)) {
              ok = false;
              break;
            }
            ++pn[t];
            // the tile's first PV of this item overwrites O_t: the previous item's epilogue must have read it
            if (j == 0 && on[t] > 0 &&
                !mbar_wait_bounded(&o_free[t], (on[t] - 1) & 1, abort_flag, errs, kErrAttnWait, 5 + t)) {
              ok = false;
              break;
            }
            tc_fence_after();
            // O_t (+)= P_t V_j; P_t is read from tile t's S columns
            const uint64_t dv =
                smem_desc_sw128(smem_u32(smem + C::KV_OFF + st * C::STAGE_BYTES + C::TILE_BYTES), 16384, 1024);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
              tc_mma_f16_ts(tmem + C::T_O + t * C::O_COLS, tmem + C::T_S + t * 128 + ks * 8, dv + ks * (2048 >> 4),
                            IDESC_O, (j == 0 && ks == 0) ? 0u : 1u);
            trace_ev(p, 0, tn, 20 + t);
            if (j + 1 == n[t]) {
              tc_commit(&o_done[t]);
              ++on[t];
            } else {
              if (!next_loaded) {
                if (!mbar_wait_bounded(&kv_full[st1], ((g + j + 1) / C::STAGES) & 1, abort_flag, errs,
                                       kErrAttnWait, 1)) {
                  ok = false;
                  break;
                }
                next_loaded = true;
                tc_fence_after();
              }
              issue_s(t, st1);
            }
          }
          if (!ok) break;
          tc_commit(&kv_empty[st]);  // K_j / V_j free once this block's MMAs have completed
        }
        g += nkv;
        tc_commit(&q_empty[qs]);  // every score MMA of the item has been issued
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(C::REGS_HIGH));
    // softmax: tile t, query row r of the tile
    const int t = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_cols = tmem + lane_off + C::T_S + t * 128;
    const uint32_t o_cols = tmem + lane_off + C::T_O + t * C::O_COLS;
    const float scale2 = p.scale * kLog2e;
    int sn = 0, on = 0;
    int tn = 0;
    const int trole = (lane == 0 && quarter == 0) ? 1 + t : -1;  // the first row of each tile traces
    auto tev = [&](int ev) {
      if (trole > 0) trace_ev(p, trole, tn, ev);
    };
    for (int k = 0;; ++k) {
      const int u = fwd_item_index(k, c, G, n_items);
      if (u < 0) break;
      const FwdItem it = fwd_item(u, n_pairs, p.heads, p.batch);
      const int n = tile_kv_blocks(it.pair, t, n_qb);
      if (n == 0) continue;  // tile past the end of the sequence
      float m_used = 0.f, l = 0.f;
      bool ok = true;
      for (int j = 0; j < n; ++j) {
        tev(1);
        if (!mbar_wait_bounded(&s_full[t], sn & 1, abort_flag, errs, kErrAttnWait, 11 + t)) {
          ok = false;
          break;
        }
        ++sn;
        tc_fence_after();
        uint32_t s[4][32];  // the row's 128 scores (fp32 bits), later its 64 bf16 pairs of P
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) tmem_ld_32x32b_x32(s_cols + 32 * q4, s[q4]);
        tc_wait_ld();
        tev(2);
        const bool diag = (j == n - 1);  // key block == query block: mask columns past the row
        if (diag) {  // masked scores become -inf: they drop out of the max and exponentiate to 0
#pragma unroll
          for (int e = 0; e < 128; ++e)
            if (e > r) s[e >> 5][e & 31] = __float_as_uint(-INFINITY);
        }
        // row max: 8 independent chains of three-input maxes (one chain would serialise 128 ops)
        float mx8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mx8[e] = __uint_as_float(s[0][e]);
#pragma unroll
        for (int e = 8; e < 128; e += 2)
          mx8[(e >> 1) & 7] = fmax3f(mx8[(e >> 1) & 7], __uint_as_float(s[e >> 5][e & 31]),
                                     __uint_as_float(s[e >> 5][(e + 1) & 31]));
        const float mx = fmax3f(fmax3f(mx8[0], mx8[1], mx8[2]), fmax3f(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
        const float m_row = mx * scale2;
        tev(3);
        if (j == 0) {
          m_used = m_row;
        } else if (__any_sync(0xffffffffu, m_row > m_used + kRescaleThreshold)) {
          // The decision is taken for the whole warp: tcgen05.ld / tcgen05.st are warp-collective
          // (.sync.aligned) and must not run in divergent code.  Lanes whose maximum did not grow
          // past the threshold keep theirs (alpha = 1); the others raise it to the block maximum.
          // O_t holds the sum up to block j-1 (complete: the commit of S_t(j) covers PV_t(j-1)).
          const float m_new = (m_row > m_used + kRescaleThreshold) ? m_row : m_used;
          const float alpha = ex2_approx(m_used - m_new);
          l *= alpha;
#pragma unroll
          for (int cc = 0; cc < HD; cc += 32) {
            uint32_t ov[32];
            tmem_ld_32x32b_x32(o_cols + cc, ov);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
            tmem_st_32x32b_x32(o_cols + cc, ov);
          }
          if constexpr (C::ONES) {  // the row-sum columns scale with O
            uint32_t lv[16];
            tmem_ld_32x32b_x16(o_cols + HD, lv);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) lv[e] = __float_as_uint(__uint_as_float(lv[e]) * alpha);
            tmem_st_32x32b_x16(o_cols + HD, lv);
          }
          m_used = m_new;
        }
        // probabilities, row sum (8 chains), bf16 P into the same tensor-memory columns.  A masked
        // score is -inf: ex2 gives 0 and the FMA-pipe exp2 gives 2^-125 (its input is clamped), which
        // is no contribution at fp32 / bf16 precision next to the row maximum's 1.
        float rs8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int e = 0; e < 128; e += 2) {
          const float x0 = fmaf(__uint_as_float(s[e >> 5][e & 31]), scale2, -m_used);
          const float x1 = fmaf(__uint_as_float(s[e >> 5][(e + 1) & 31]), scale2, -m_used);
          float p0, p1;
          if constexpr (EMU == kEmuHalfPairs) {
            ex2_pair_f16(x0, x1, p0, p1);
          } else {
            p0 = ((e & 7) >= 8 - EMU) ? exp2_fma(x0) : ex2_approx(x0);
            p1 = (((e + 1) & 7) >= 8 - EMU) ? exp2_fma(x1) : ex2_approx(x1);
          }
          if constexpr (!C::ONES) {
            rs8[e & 7] += p0;
            rs8[(e + 1) & 7] += p1;
          }
          s[e >> 6][(e >> 1) & 31] = pack_bf16(p0, p1);  // pair e/2 lands below column e: already read
        }
        if constexpr (!C::ONES) l += ((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) + ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7]));
        tev(4);
        tmem_st_32x32b_x32(s_cols + 0, s[0]);
        tmem_st_32x32b_x32(s_cols + 32, s[1]);
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
        tev(5);
      }
      if (!ok) break;
      // epilogue: O / l -> bf16 rows, base-2 log-sum-exp
      tev(6);
      if (!mbar_wait_bounded(&o_done[t], on & 1, abort_flag, errs, kErrAttnWait, 13 + t)) break;
      tev(7);
      ++on;
      tc_fence_after();
      const int q_row = (2 * it.pair + t) * 128 + r;
      if constexpr (C::ONES) {  // the row sum accumulated by the tensor cores
        uint32_t lv[16];
        tmem_ld_32x32b_x16(o_cols + HD, lv);
        tc_wait_ld();
        l = __uint_as_float(lv[0]);
      }
      const float inv_l = 1.0f / l;
      const size_t out_idx = (size_t)(it.b * p.seq + q_row) * p.ld_out + it.h * HD;
      __nv_bfloat16* dst = p.out + out_idx;
      const bool out_in = B200_IN_BOUNDS(errs, out_idx, HD, (long long)p.batch * p.seq * p.ld_out, 120);
#pragma unroll
      for (int cc = 0; cc < HD; cc += 32) {
        uint32_t ov[32];
        tmem_ld_32x32b_x32(o_cols + cc, ov);
        tc_wait_ld();
        if (cc + 32 >= HD) {  // every column read: O_t may be overwritten by the next item
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&o_free[t]);
        }
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint4 w;
          w.x = pack_bf16(__uint_as_float(ov[e]) * inv_l, __uint_as_float(ov[e + 1]) * inv_l);
          w.y = pack_bf16(__uint_as_float(ov[e + 2]) * inv_l, __uint_as_float(ov[e + 3]) * inv_l);
          w.z = pack_bf16(__uint_as_float(ov[e + 4]) * inv_l, __uint_as_float(ov[e + 5]) * inv_l);
          w.w = pack_bf16(__uint_as_float(ov[e + 6]) * inv_l, __uint_as_float(ov[e + 7]) * inv_l);
          if (out_in) *reinterpret_cast<uint4*>(dst + cc + e) = w;
        }
      }
      const size_t lse_idx = ((size_t)it.b * p.heads + it.h) * p.seq + q_row;
      if (B200_IN_BOUNDS(errs, lse_idx, 1, (long long)p.batch * p.heads * p.seq, 121))
        p.lse[lse_idx] = m_used + log2f(l);
      tev(8);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int HD, int EMU>
void launch_fwd_emu(const AttnParams& p, const CUtensorMap& tm, cudaStream_t s) {
  using C = AttnFwdCfg<HD>;
  static std::atomic<unsigned long long> configured{0};
  once_per_device(configured, [] {
    B200_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel<HD, EMU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::SMEM_BYTES));
  });
  const int n_qb = p.seq / 128;
  const int items = ((n_qb + 1) / 2) * p.heads * p.batch;
  const int grid = std::max(1, std::min(items, num_sms_cached()));
  launch_k(attn_fwd_kernel<HD, EMU>, dim3(grid), dim3(ATT_THREADS), C::SMEM_BYTES, s, 1, tm, p, device_errors_ptr());
}

// ZB_ATTN_FWD_EMU=0..3 overrides the share of FMA-pipe exponentials (eighths of the columns), 4 selects
// the half-precision pairs; for tuning.
int fwd_emu_override() {
  static const int v = [] {
    const char* e = std::getenv("ZB_ATTN_FWD_EMU");
    return (e != nullptr && *e >= '0' && *e <= '4' && e[1] == 0) ? (*e - '0') : -1;
  }();
  return v;
}

template <int HD>
void launch_fwd(const AttnParams& p, const CUtensorMap& tm, cudaStream_t s) {
  const int emu = fwd_emu_override() >= 0 ? fwd_emu_override() : AttnFwdCfg<HD>::EMU;
  switch (emu) {
    case 1: launch_fwd_emu<HD, 1>(p, tm, s); break;
    case 2: launch_fwd_emu<HD, 2>(p, tm, s); break;
    case 3: launch_fwd_emu<HD, 3>(p, tm, s); break;
    case kEmuHalfPairs: launch_fwd_emu<HD, kEmuHalfPairs>(p, tm, s); break;
    default: launch_fwd_emu<HD, 0>(p, tm, s); break;
  }
}

}  // namespace

namespace {
unsigned long long* g_trace = nullptr;  // debug tracing buffer (ZB_ATTN_TRACE=1), one per process
bool trace_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("ZB_ATTN_TRACE");
    return e != nullptr && e[0] == '1';
  }();
  return on;
}
}  // namespace

void attention_trace_read(unsigned long long* host_out) {
  B200_CHECK(g_trace != nullptr, "attention trace: run a forward with ZB_ATTN_TRACE=1 first");
  B200_CUDA_CHECK(cudaMemcpy(host_out, g_trace, 3 * kAttnTraceWords * 8, cudaMemcpyDeviceToHost));
}

void attention_fwd(const AttnParams& p_in, cudaStream_t s) {
  AttnParams p = p_in;
  if (trace_enabled()) {  // debug only: one buffer, cleared before each traced launch
    if (g_trace == nullptr) B200_CUDA_CHECK(cudaMalloc(&g_trace, 3 * kAttnTraceWords * 8));
    B200_CUDA_CHECK(cudaMemsetAsync(g_trace, 0, 3 * kAttnTraceWords * 8, s));
    p.trace = g_trace;
  }
  B200_CHECK(p.head_dim == 64 || p.head_dim == 128, "attention: head_dim must be 64 or 128");
  B200_CHECK(p.seq % 128 == 0, "attention: seq_len must be a multiple of 128");
  B200_CHECK(p.heads % p.kv_heads == 0, "attention: heads must be a multiple of kv_heads");
  CUtensorMap tm = make_tmap_bf16_2d(p.qkv, (uint64_t)p.ld, (uint64_t)p.batch * p.seq, (uint64_t)p.ld, 64, 128);
  if (p.head_dim == 64)
    launch_fwd<64>(p, tm, s);
  else
    launch_fwd<128>(p, tm, s);
  B200_CUDA_CHECK(cudaGetLastError());
  count_launch();
}

}  // namespace b200
