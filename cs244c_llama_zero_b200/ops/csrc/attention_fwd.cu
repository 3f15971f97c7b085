// Causal GQA flash-attention forward on the 5th-generation tensor cores (sm_100a).
//
// Persistent: one CTA per SM walks a longest-first list of (query block of 128 rows, query head,
// batch) items, 320 threads:
//   warp 0      TMA producer: Q once, then K_j / V_j tiles into a STAGES-deep ring.  Q, K and V
//               are column blocks of the fused [B*S, ld] q|k|v projection output, so one tensor
//               map serves all three and K/V are never repeated for grouped heads: query head h
//               reads kv head h / (H / KV).
//   warp 1      allocates tensor memory; lane 0 issues S_j = Q K_j^T (M=128, N=128, K=hd) into a
//               double-buffered S accumulator, and O_j = P_j V_j (M=128, N=hd, K=128) into a
//               double-buffered O accumulator once the softmax warps have written P_j.
//   warps 2..9  softmax, two warpgroups.  Thread (wg, r) owns query row r and the 64 score columns
//               [64*wg, 64*wg+64) and the output columns [wg*hd/2, (wg+1)*hd/2).  Row maxima are
//               combined through shared memory once per block (one named barrier); row sums stay
//               per warpgroup until the end.  Scores are read from tensor memory, masked only on
//               the diagonal block, exponentiated with one FFMA + ex2.approx in the base-2 domain,
//               written as bf16 P in the 128-byte-swizzled K-major layout the MMA reads, and
//               O_{j-1} is folded into registers with the running rescale factor.
// The log-sum-exp of every row is stored in base-2 units scaled by log2(e)/sqrt(hd) so the
// backward pass can rebuild P with one exp2.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "gemm.h"
#include "kernels.h"

namespace b200 {

namespace {

constexpr int ATT_THREADS = 320;
constexpr float kLog2e = 1.4426950408889634f;

template <int HD>
struct AttnFwdCfg {
  static constexpr int KB = HD / 64;                 // 64-column swizzle blocks per row
  static constexpr int TILE_BYTES = 128 * HD * 2;    // one 128-row tile of Q, K or V
  static constexpr int STAGES = (HD == 64) ? 3 : 2;
  static constexpr int Q_BUFS = (HD == 64) ? 2 : 1;  // the next item's Q loads during this item
  static constexpr int P_BYTES = 128 * 128 * 2;
  static constexpr int P_BUFS = (HD == 64) ? 2 : 1;
  static constexpr int Q_OFF = 0;
  static constexpr int KV_OFF = Q_BUFS * TILE_BYTES;
  static constexpr int P_OFF = KV_OFF + STAGES * 2 * TILE_BYTES;
  static constexpr int RED_OFF = P_OFF + P_BUFS * P_BYTES;  // row-max exchange [2 parity][2 wg][128]
  static constexpr int BAR_OFF = RED_OFF + 3 * 2 * 128 * 4;
  static constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;
  static constexpr int TMEM_COLS = 512;
  static constexpr int O_TMEM = 256;  // O accumulators start after the two S buffers
  static constexpr int HALF_O = HD / 2;
};

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Work items are (query block, head, batch), numbered longest causal row first: item u has query
// block n_qb - 1 - u / (H * B).  CTA c of G takes items c, 2G - 1 - c, 2G + c, ... (boustrophedon
// deal), so every CTA's list runs from long to short and the totals even out.
struct FwdItem {
  int qb, h, b;
};
__device__ __forceinline__ int fwd_item_index(int k, int c, int G, int n_items) {
  const int u = k * G + ((k & 1) ? (G - 1 - c) : c);
  return u < n_items ? u : -1;
}
__device__ __forceinline__ FwdItem fwd_item(int u, int n_qb, int heads, int batch) {
  const int per = heads * batch;
  const int r = u % per;
  return {n_qb - 1 - u / per, r % heads, r / heads};
}

// Persistent: one CTA per SM walks its item list.  Every barrier phase comes from counters that run
// across items (g: key/value block, score, probability and PV index; k: item index), so the
// producer loads the next item's Q and K/V and the MMA warp issues its first score block while the
// softmax warps still finish the current item.
template <int HD>
__global__ void __launch_bounds__(ATT_THREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm, AttnParams p, DeviceErrors* errs) {
  using C = AttnFwdCfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars;                    // [Q_BUFS]
  uint64_t* q_empty = q_full + C::Q_BUFS;     // [Q_BUFS]
  uint64_t* kv_full = q_empty + C::Q_BUFS;
  uint64_t* kv_empty = kv_full + C::STAGES;
  uint64_t* s_full = kv_empty + C::STAGES;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_full = p_full + 2;
  uint64_t* o_free = o_full + 2;
  uint64_t* red_bar = o_free + 2;  // [0..1]: row-max exchange per parity, [2]: final row-sum exchange
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_bar + 3);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(smem + C::RED_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qb = p.seq / 128;
  const int n_items = n_qb * p.heads * p.batch;
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
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 8);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 8);
    }
    for (int i = 0; i < 3; ++i) mbar_init(&red_bar[i], 8);
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
  pdl_wait_and_release();  // q|k|v come from the previous kernel of the stream

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm);
      int g = 0;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int u = fwd_item_index(k, c, G, n_items);
        if (u < 0) break;
        const FwdItem it = fwd_item(u, n_qb, p.heads, p.batch);
        const int row0 = it.b * p.seq;
        const int kvh = it.h / group;
        const int qs = k % C::Q_BUFS;
        // The slot's previous Q is free once every score MMA of that item has completed.
        if (k >= C::Q_BUFS &&
            !mbar_wait_bounded(&q_empty[qs], ((k / C::Q_BUFS) - 1) & 1, abort_flag, errs, kErrAttnWait, 10))
          break;
        mbar_expect_tx(&q_full[qs], C::TILE_BYTES);
#pragma unroll
        for (int kb = 0; kb < C::KB; ++kb)
          tma_load_2d(smem + C::Q_OFF + qs * C::TILE_BYTES + kb * 16384, &tm, &q_full[qs], it.h * HD + 64 * kb,
                      row0 + it.qb * 128);
        for (int j = 0; j <= it.qb; ++j, ++g) {
          const int st = g % C::STAGES;
          const uint32_t ph = (g / C::STAGES) & 1;
          if (!mbar_wait_bounded(&kv_empty[st], ph ^ 1u, abort_flag, errs, kErrAttnWait, 0)) {
            ok = false;
            break;
          }
          uint8_t* ks = smem + C::KV_OFF + st * 2 * C::TILE_BYTES;
          uint8_t* vs = ks + C::TILE_BYTES;
          mbar_expect_tx(&kv_full[st], 2 * C::TILE_BYTES);
#pragma unroll
          for (int kb = 0; kb < C::KB; ++kb) {
            tma_load_2d(ks + kb * 16384, &tm, &kv_full[st], p.k_col + kvh * HD + 64 * kb, row0 + j * 128);
            tma_load_2d(vs + kb * 16384, &tm, &kv_full[st], p.v_col + kvh * HD + 64 * kb, row0 + j * 128);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC_S = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t IDESC_O = idesc_bf16_f32(128, HD, false, true);
      // Score MMAs run one block ahead of the PV MMAs, across item boundaries: `sk`/`sj` is the
      // item / block of the next score block to issue, `sg` its global index.
      int sk = 0, sj = 0, sg = 0;
      int s_u = fwd_item_index(0, c, G, n_items);
      int s_nkv = s_u >= 0 ? fwd_item(s_u, n_qb, p.heads, p.batch).qb + 1 : 0;
      auto issue_s = [&]() -> bool {
        const int qs = sk % C::Q_BUFS;
        if (sj == 0 && !mbar_wait_bounded(&q_full[qs], (sk / C::Q_BUFS) & 1, abort_flag, errs, kErrAttnWait, 2))
          return false;
        const int st = sg % C::STAGES;
        if (!mbar_wait_bounded(&kv_full[st], (sg / C::STAGES) & 1, abort_flag, errs, kErrAttnWait, 1)) return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(smem + C::Q_OFF + qs * C::TILE_BYTES);
        const uint32_t k_addr = smem_u32(smem + C::KV_OFF + st * 2 * C::TILE_BYTES);
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
          const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
          tc_mma_f16(tmem + (sg & 1) * 128, smem_desc_sw128(q_addr + off, 16, 1024),
                     smem_desc_sw128(k_addr + off, 16, 1024), IDESC_S, ks > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[sg & 1]);
        ++sg;
        if (++sj == s_nkv) {  // last score block of this item: its Q slot frees when these MMAs finish
          tc_commit(&q_empty[qs]);
          ++sk;
          sj = 0;
          s_u = fwd_item_index(sk, c, G, n_items);
          s_nkv = s_u >= 0 ? fwd_item(s_u, n_qb, p.heads, p.batch).qb + 1 : 0;
        }
        return true;
      };
      bool ok = s_u < 0 || issue_s();
      // PV of global block g, after the score block g + 1 has been issued (if there is one).
      for (int g = 0; ok && g < sg; ++g) {
        if (s_u >= 0 && !issue_s()) break;
        if (!mbar_wait_bounded(&p_full[g & 1], (g >> 1) & 1, abort_flag, errs, kErrAttnWait, 3)) break;
        if (g >= 2 && !mbar_wait_bounded(&o_free[g & 1], ((g - 2) >> 1) & 1, abort_flag, errs, kErrAttnWait, 4)) break;
        tc_fence_after();
        const int st = g % C::STAGES;
        const uint32_t v_addr = smem_u32(smem + C::KV_OFF + st * 2 * C::TILE_BYTES + C::TILE_BYTES);
        const uint32_t p_addr = smem_u32(smem + C::P_OFF + (g % C::P_BUFS) * C::P_BYTES);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t poff = (ks >> 2) * 16384 + (ks & 3) * 32;
          tc_mma_f16(tmem + C::O_TMEM + (g & 1) * HD, smem_desc_sw128(p_addr + poff, 16, 1024),
                     smem_desc_sw128(v_addr + ks * 2048, 16384, 1024), IDESC_O, ks > 0 ? 1u : 0u);
        }
        tc_commit(&o_full[g & 1]);
        tc_commit(&kv_empty[st]);
      }
    }
  } else {
    const int wg = (warp - 2) >> 2;   // warpgroup: score columns [64*wg, 64*wg+64)
    const int q = warp & 3;            // tensor-memory lane quarter
    const int r = q * 32 + lane;       // query row within the block
    const int col0 = wg * 64;
    const int ocol0 = wg * C::HALF_O;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const float scale2 = p.scale * kLog2e;
    int g = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int u = fwd_item_index(k, c, G, n_items);
      if (u < 0) break;
      const FwdItem it = fwd_item(u, n_qb, p.heads, p.batch);
      const int n_kv = it.qb + 1;
      const int row0 = it.b * p.seq;
      float m = -INFINITY, l = 0.f;
      float o[C::HALF_O];
#pragma unroll
      for (int i = 0; i < C::HALF_O; ++i) o[i] = 0.f;
      for (int j = 0; j < n_kv; ++j, ++g) {
        if (!mbar_wait_bounded(&s_full[g & 1], (g >> 1) & 1, abort_flag, errs, kErrAttnWait, 5)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sbase = lane_base + (g & 1) * 128 + col0;
        const bool diag = (j == it.qb);
        // pass 1: partial row max of the raw scores over this warpgroup's 64 columns
        float pmx = -INFINITY;
#pragma unroll
        for (int cc = 0; cc < 64; cc += 32) {
          uint32_t sv[32];
          tmem_ld_32x32b_x32(sbase + cc, sv);
          tc_wait_ld();
          if (diag) {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (col0 + cc + e <= r) pmx = fmaxf(pmx, __uint_as_float(sv[e]));
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) pmx = fmaxf(pmx, __uint_as_float(sv[e]));
          }
        }
        float* red_slot = red + (g & 1) * 256;
        red_slot[wg * 128 + r] = pmx;
        __syncwarp();
        if (lane == 0) mbar_arrive(&red_bar[g & 1]);
        if (!mbar_wait_bounded(&red_bar[g & 1], (g >> 1) & 1, abort_flag, errs, kErrAttnWait, 8)) {
          ok = false;
          break;
        }
        const float other = red_slot[(wg ^ 1) * 128 + r];
        const float mx = fmaxf(m, fmaxf(pmx, other) * scale2);  // scaled, base-2 domain
        const float alpha = ex2_approx(m - mx);
        // P buffer reuse: PV_{g-1} must have finished reading it (and PV_{g-2}, folded at g - 1).
        if (j >= 1 &&
            !mbar_wait_bounded(&o_full[(g - 1) & 1], ((g - 1) >> 1) & 1, abort_flag, errs, kErrAttnWait, 6)) {
          ok = false;
          break;
        }
        // pass 2: probabilities, partial row sum, bf16 P into swizzled shared memory
        uint8_t* pbuf = smem + C::P_OFF + (g % C::P_BUFS) * C::P_BYTES;
        float rs = 0.f;
#pragma unroll
        for (int cc = 0; cc < 64; cc += 32) {
          uint32_t sv[32];
          tmem_ld_32x32b_x32(sbase + cc, sv);
          tc_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            float p0 = ex2_approx(fmaf(__uint_as_float(sv[e]), scale2, -mx));
            float p1 = ex2_approx(fmaf(__uint_as_float(sv[e + 1]), scale2, -mx));
            if (diag) {
              if (col0 + cc + e > r) p0 = 0.f;
              if (col0 + cc + e + 1 > r) p1 = 0.f;
            }
            rs += p0 + p1;
            pk[e >> 1] = pack_bf16(p0, p1);
          }
          const int col = col0 + cc;
          const int kblk = col >> 6;
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            const int chunk = ((col & 63) >> 3) + ch;  // 16-byte chunk within the 128-byte row
            const int sw = chunk ^ (r & 7);
            *reinterpret_cast<uint4*>(pbuf + kblk * 16384 + r * 128 + sw * 16) =
                make_uint4(pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
          }
        }
        l = l * alpha + rs;
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[g & 1]);
        if (j >= 1) {
          tc_fence_after();
          const uint32_t obase = lane_base + C::O_TMEM + ((g - 1) & 1) * HD + ocol0;
#pragma unroll
          for (int cc = 0; cc < C::HALF_O; cc += 32) {
            uint32_t ov[32];
            tmem_ld_32x32b_x32(obase + cc, ov);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[cc + e] = (o[cc + e] + __uint_as_float(ov[e])) * alpha;
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&o_free[(g - 1) & 1]);
        } else {
#pragma unroll
          for (int i = 0; i < C::HALF_O; ++i) o[i] *= alpha;
        }
        m = mx;
      }
      if (!ok) break;
      // Combine the two warpgroups' partial row sums (the slot is reused per item: both
      // warpgroups pass the next item's first row-max exchange before either writes it again).
      float* lred = red + 512;
      lred[wg * 128 + r] = l;
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_bar[2]);
      if (!mbar_wait_bounded(&red_bar[2], k & 1, abort_flag, errs, kErrAttnWait, 9)) break;
      const float l_total = l + lred[(wg ^ 1) * 128 + r];
      const int gl = g - 1;  // global index of this item's last block
      if (!mbar_wait_bounded(&o_full[gl & 1], (gl >> 1) & 1, abort_flag, errs, kErrAttnWait, 7)) break;
      tc_fence_after();
      const uint32_t obase = lane_base + C::O_TMEM + (gl & 1) * HD + ocol0;
      const float inv_l = 1.0f / l_total;
      const size_t out_idx = (size_t)(row0 + it.qb * 128 + r) * p.ld_out + it.h * HD + ocol0;
      __nv_bfloat16* dst = p.out + out_idx;
      const bool out_in =
          B200_IN_BOUNDS(errs, out_idx, C::HALF_O, (long long)p.batch * p.seq * p.ld_out, 120);
#pragma unroll
      for (int cc = 0; cc < C::HALF_O; cc += 32) {
        uint32_t ov[32];
        tmem_ld_32x32b_x32(obase + cc, ov);
        tc_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint4 w;
          w.x = pack_bf16((o[cc + e] + __uint_as_float(ov[e])) * inv_l, (o[cc + e + 1] + __uint_as_float(ov[e + 1])) * inv_l);
          w.y = pack_bf16((o[cc + e + 2] + __uint_as_float(ov[e + 2])) * inv_l, (o[cc + e + 3] + __uint_as_float(ov[e + 3])) * inv_l);
          w.z = pack_bf16((o[cc + e + 4] + __uint_as_float(ov[e + 4])) * inv_l, (o[cc + e + 5] + __uint_as_float(ov[e + 5])) * inv_l);
          w.w = pack_bf16((o[cc + e + 6] + __uint_as_float(ov[e + 6])) * inv_l, (o[cc + e + 7] + __uint_as_float(ov[e + 7])) * inv_l);
          if (out_in) *reinterpret_cast<uint4*>(dst + cc + e) = w;
        }
      }
      // The last O buffer of the item is free for the PV two blocks later.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[gl & 1]);
      const size_t lse_idx = ((size_t)it.b * p.heads + it.h) * p.seq + it.qb * 128 + r;
      if (wg == 0 && B200_IN_BOUNDS(errs, lse_idx, 1, (long long)p.batch * p.heads * p.seq, 121))
        p.lse[lse_idx] = m + log2f(l_total);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int HD>
void launch_fwd(const AttnParams& p, const CUtensorMap& tm, cudaStream_t s) {
  using C = AttnFwdCfg<HD>;
  static std::atomic<unsigned long long> configured{0};
  once_per_device(configured, [] {
    B200_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
  });
  const int items = (p.seq / 128) * p.heads * p.batch;
  const int grid = std::max(1, std::min(items, num_sms_cached()));
  launch_k(attn_fwd_kernel<HD>, dim3(grid), dim3(ATT_THREADS), C::SMEM_BYTES, s, 1, tm, p, device_errors_ptr());
}

}  // namespace

void attention_fwd(const AttnParams& p, cudaStream_t s) {
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
