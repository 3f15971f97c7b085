// Host-visible interface of the tcgen05 GEMM (see gemm_tcgen05.cu).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace b200 {

enum GemmEpilogue : int {
  EPI_STORE = 0,
  EPI_RESIDUAL = 1,
  EPI_ROPE = 2,
  EPI_SWIGLU = 3,
  EPI_SWIGLU_BWD = 4,
  EPI_ACC_F32 = 5,
  // Weight gradient with its reduce-scatter fused in: each fp32 partial sum is added straight into
  // the gradient shard of the rank that owns that element (flat index / shard size), over NVLink
  // peer mappings, with red.global.add.v4.f32 at system scope.  No local gradient buffer is written.
  EPI_ACC_F32_ROUTED = 6,
};

constexpr int kRouteMaxWorld = 8;

struct GemmOperands {
  const void* A;  // bf16; K-major: [M, K] with row stride lda; MN-major: [K, M] with row stride lda
  const void* B;  // bf16; K-major: [N, K] with row stride ldb; MN-major: [K, N] with row stride ldb
  uint64_t lda;
  uint64_t ldb;
};

struct GemmParams {
  int M, N, K;
  int tiles_m, tiles_n, splits, k_blocks_per_split, total_k_blocks;  // filled by the launcher
  __nv_bfloat16* C;
  int ldc;
  const __nv_bfloat16* R;
  int ldr;
  float* C32;
  int ldc32;
  const float* rope_cos;  // [head_dim/2, seq_len] (frequency-major, see rope_tables_t)
  const float* rope_sin;
  int seq_len;
  int head_dim;
  int rope_cols;  // columns [0, rope_cols) are rotated (q and k)
  __nv_bfloat16* aux;  // SwiGLU forward: [M, 2*ffn] pre-activations (g | u)
  int ld_aux;
  const __nv_bfloat16* aux_in;  // SwiGLU backward: [M, 2*ffn] saved (g | u)
  int ld_aux_in;
  int ffn;
  DeviceErrors* errs;
  // Grouped launches (gemm_launch_dgrad_wgrad): units [0, grp_units_first) belong to problem
  // grp_first, the rest (up to grp_units_total) to the other one.
  int grp_first, grp_units_first, grp_units_total;
  // EPI_ACC_F32_ROUTED: output element (m, n) has flat index route_flat0 + m * route_ld + n; rank
  // r = flat / route_chunk owns it and it lands at route_base[r][flat - r * route_chunk] (fp32 shard
  // of rank r, mapped on this GPU).
  uint64_t route_base[kRouteMaxWorld];
  int route_world;
  int route_ld;
  long long route_chunk;
  long long route_flat0;
};

struct GemmTile {
  int bn, splits, cg;
};
// Tile width (128 / 192 / 256), CTA group (1 or a pair) and K-split minimising the modelled time.
// only_bn / only_cg > 0 restrict the search to that tile width / CTA group.
GemmTile choose_gemm_tile(int M, int N, int K, int epi, int head_dim, bool allow_split, bool b_mn, int sms,
                          int only_bn = 0, int only_cg = 0);

int num_sms();
// Generic 2D tiled tensor map (dims {inner, outer}, row stride in elements); throws on misaligned
// base or stride.
CUtensorMap make_tmap_2d(CUtensorMapDataType dtype, int elem_bytes, const void* base, uint64_t inner, uint64_t outer,
                         uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle);
CUtensorMap make_tmap_bf16_2d(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                              uint32_t box_inner, uint32_t box_outer);
void gemm_launch(const GemmOperands& op, GemmParams p, int epi, bool a_mn, bool b_mn, int bn, cudaStream_t stream);
// One persistent launch computing two independent GEMMs of a linear layer's backward pass:
//   problem 0: dX[M0, N0] = dY[M0, K0] @ W[K0, N0]          (A K-major, B MN-major, bf16 store)
//   problem 1: dW[M1, N1] += dY^T[M1, K1] @ X[K1, N1]       (A MN-major, B MN-major, fp32 add-reduce)
// Their tiles are dealt together, longest first, so neither one's partial last wave idles SMs.
// splits1 <= 0 chooses problem 1's K-split for the combined schedule.
void gemm_launch_dgrad_wgrad(const GemmOperands& op0, GemmParams p0, const GemmOperands& op1, GemmParams p1,
                             cudaStream_t stream);
// The grouped launch's schedule (host only): fills both problems' tile / split fields and the
// grouping fields of p0 for `sms` SMs and returns the modelled makespan in k-blocks per CTA pair.
long plan_dgrad_wgrad(GemmParams& p0, GemmParams& p1, int sms);

}  // namespace b200
