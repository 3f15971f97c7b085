// Python bindings of the sm_100a kernels.  Every entry point validates shapes, dtypes, devices
// and alignment, then launches on the current PyTorch CUDA stream.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cmath>
#include <memory>
#include <optional>

#include "comm.h"
#include "gemm.h"
#include "kernels.h"

namespace {

using at::Tensor;

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_cuda(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}
void check_bf16_2d(const Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bfloat16");
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, name, " must be 2-D with unit column stride");
  TORCH_CHECK(t.stride(0) % 8 == 0, name, " row stride must be a multiple of 8 elements");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, " must be 16-byte aligned");
}
void check_f32(const Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == at::kFloat, name, " must be float32");
}

b200::GemmParams base_params(int M, int N, int K) {
  b200::GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.splits = 1;
  return p;
}

// y[M,N] = x[M,K] @ w[N,K]^T (+ residual)
void linear_fwd(Tensor x, Tensor w, Tensor out, std::optional<Tensor> residual, int64_t bn) {
  check_bf16_2d(x, "x");
  check_bf16_2d(w, "w");
  check_bf16_2d(out, "out");
  const int M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && out.size(0) == M && out.size(1) == N, "linear_fwd: shape mismatch");
  c10::cuda::CUDAGuard g(x.device());
  auto p = base_params(M, N, K);
  p.C = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldc = out.stride(0);
  int epi = b200::EPI_STORE;
  if (residual.has_value()) {
    check_bf16_2d(*residual, "residual");
    TORCH_CHECK(residual->size(0) == M && residual->size(1) == N, "residual shape mismatch");
    p.R = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    p.ldr = residual->stride(0);
    epi = b200::EPI_RESIDUAL;
  }
  b200::GemmOperands op{x.data_ptr(), w.data_ptr(), (uint64_t)x.stride(0), (uint64_t)w.stride(0)};
  b200::gemm_launch(op, p, epi, false, false, (int)bn, cur_stream());
}

void qkv_rope_fwd(Tensor x, Tensor w, Tensor out, Tensor cos, Tensor sin, int64_t seq_len, int64_t head_dim,
                  int64_t rope_cols, int64_t bn) {
  check_bf16_2d(x, "x");
  check_bf16_2d(w, "w");
  check_bf16_2d(out, "out");
  check_f32(cos, "cos");
  check_f32(sin, "sin");
  const int M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && out.size(0) == M && out.size(1) == N, "qkv_rope_fwd: shape mismatch");
  TORCH_CHECK(N % head_dim == 0 && 256 % head_dim == 0, "qkv_rope_fwd: head_dim must divide 256 and N");
  TORCH_CHECK(cos.numel() >= seq_len * head_dim / 2 && sin.numel() >= seq_len * head_dim / 2 &&
                  cos.is_contiguous() && sin.is_contiguous(),
              "rope tables too small (frequency-major [head_dim/2, seq_len], contiguous)");
  c10::cuda::CUDAGuard g(x.device());
  auto p = base_params(M, N, K);
  p.C = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldc = out.stride(0);
  p.rope_cos = cos.data_ptr<float>();
  p.rope_sin = sin.data_ptr<float>();
  p.seq_len = seq_len;
  p.head_dim = head_dim;
  p.rope_cols = rope_cols;
  b200::GemmOperands op{x.data_ptr(), w.data_ptr(), (uint64_t)x.stride(0), (uint64_t)w.stride(0)};
  b200::gemm_launch(op, p, b200::EPI_ROPE, false, false, (int)bn, cur_stream());
}

// h = silu(x @ Wg^T) * (x @ Wu^T); gu = [x @ Wg^T | x @ Wu^T].  w_gu = [Wg; Wu] of shape [2*ffn, K].
void swiglu_fwd(Tensor x, Tensor w_gu, Tensor h, Tensor gu, int64_t bn) {
  check_bf16_2d(x, "x");
  check_bf16_2d(w_gu, "w_gu");
  check_bf16_2d(h, "h");
  check_bf16_2d(gu, "gu");
  const int M = x.size(0), K = x.size(1), ffn = w_gu.size(0) / 2;
  TORCH_CHECK(w_gu.size(0) == 2 * ffn && w_gu.size(1) == K, "swiglu_fwd: weight shape");
  TORCH_CHECK(h.size(0) == M && h.size(1) == ffn && gu.size(0) == M && gu.size(1) == 2 * ffn, "swiglu_fwd: outputs");
  TORCH_CHECK(ffn % 8 == 0, "ffn must be a multiple of 8");
  c10::cuda::CUDAGuard g(x.device());
  auto p = base_params(M, ffn, K);
  p.C = reinterpret_cast<__nv_bfloat16*>(h.data_ptr());
  p.ldc = h.stride(0);
  p.aux = reinterpret_cast<__nv_bfloat16*>(gu.data_ptr());
  p.ld_aux = gu.stride(0);
  p.ffn = ffn;
  b200::GemmOperands op{x.data_ptr(), w_gu.data_ptr(), (uint64_t)x.stride(0), (uint64_t)w_gu.stride(0)};
  b200::gemm_launch(op, p, b200::EPI_SWIGLU, false, false, (int)bn, cur_stream());
}

// dx[M,K] = dy[M,N] @ w[N,K]
void linear_dgrad(Tensor dy, Tensor w, Tensor dx, int64_t bn) {
  check_bf16_2d(dy, "dy");
  check_bf16_2d(w, "w");
  check_bf16_2d(dx, "dx");
  const int M = dy.size(0), N = dy.size(1), K = w.size(1);
  TORCH_CHECK(w.size(0) == N && dx.size(0) == M && dx.size(1) == K, "linear_dgrad: shape mismatch");
  c10::cuda::CUDAGuard g(dy.device());
  auto p = base_params(M, K, N);
  p.C = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  p.ldc = dx.stride(0);
  b200::GemmOperands op{dy.data_ptr(), w.data_ptr(), (uint64_t)dy.stride(0), (uint64_t)w.stride(0)};
  b200::gemm_launch(op, p, b200::EPI_STORE, false, true, (int)bn, cur_stream());
}

// dgu = swiglu'(gu) * (dy @ w_down), with w_down [d, ffn] and gu/dgu [M, 2*ffn].
void swiglu_dgrad(Tensor dy, Tensor w_down, Tensor gu, Tensor dgu) {
  check_bf16_2d(dy, "dy");
  check_bf16_2d(w_down, "w_down");
  check_bf16_2d(gu, "gu");
  check_bf16_2d(dgu, "dgu");
  const int M = dy.size(0), d = dy.size(1), ffn = w_down.size(1);
  TORCH_CHECK(w_down.size(0) == d && gu.size(1) == 2 * ffn && dgu.size(1) == 2 * ffn && gu.size(0) == M &&
                  dgu.size(0) == M,
              "swiglu_dgrad: shape mismatch");
  c10::cuda::CUDAGuard g(dy.device());
  auto p = base_params(M, ffn, d);
  p.C = reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr());
  p.ldc = dgu.stride(0);
  p.aux_in = reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr());
  p.ld_aux_in = gu.stride(0);
  p.ffn = ffn;
  b200::GemmOperands op{dy.data_ptr(), w_down.data_ptr(), (uint64_t)dy.stride(0), (uint64_t)w_down.stride(0)};
  b200::gemm_launch(op, p, b200::EPI_SWIGLU_BWD, false, true, 0, cur_stream());
}

// dw[N,K] (fp32) += dy[M,N]^T @ x[M,K]
void linear_wgrad(Tensor dy, Tensor x, Tensor dw, int64_t splits, int64_t bn) {
  check_bf16_2d(dy, "dy");
  check_bf16_2d(x, "x");
  check_f32(dw, "dw");
  const int M = dy.size(0), N = dy.size(1), K = x.size(1);
  TORCH_CHECK(x.size(0) == M, "linear_wgrad: token counts differ");
  TORCH_CHECK(dw.dim() == 2 && dw.size(0) == N && dw.size(1) == K && dw.stride(1) == 1, "linear_wgrad: dw shape");
  TORCH_CHECK(dw.stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(dw.data_ptr()) % 16 == 0, "dw alignment");
  c10::cuda::CUDAGuard g(dy.device());
  auto p = base_params(N, K, M);
  p.C32 = dw.data_ptr<float>();
  p.ldc32 = dw.stride(0);
  p.splits = splits > 0 ? (int)splits : 0;  // 0: chosen with the tile width
  b200::GemmOperands op{dy.data_ptr(), x.data_ptr(), (uint64_t)dy.stride(0), (uint64_t)x.stride(0)};
  b200::gemm_launch(op, p, b200::EPI_ACC_F32, true, true, (int)bn, cur_stream());
}

// dw = dy^T @ x with the reduce-scatter fused into the epilogue: element (n, k) of dw has flat index
// flat0 + n * ld + k in a flat space split into `bases.size()` shards of `chunk` fp32 elements, and its
// partial sum is added straight into the owning shard (`bases[r]`: rank r's shard as mapped on this
// GPU; on one GPU they may all be local buffers).  Every rank calls this with its own dy / x; the
// shards hold the sum over ranks once every rank's call has finished (order them with a barrier).
void linear_wgrad_routed(Tensor dy, Tensor x, int64_t flat0, int64_t ld, int64_t chunk, std::vector<int64_t> bases,
                         int64_t splits, int64_t bn) {
  check_bf16_2d(dy, "dy");
  check_bf16_2d(x, "x");
  const int M = dy.size(0), N = dy.size(1), K = x.size(1);
  TORCH_CHECK(x.size(0) == M, "linear_wgrad_routed: token counts differ");
  TORCH_CHECK(!bases.empty() && (int)bases.size() <= b200::kRouteMaxWorld, "linear_wgrad_routed: 1..8 shards");
  c10::cuda::CUDAGuard g(dy.device());
  auto p = base_params(N, K, M);
  p.splits = splits > 0 ? (int)splits : 0;
  p.route_world = (int)bases.size();
  for (size_t r = 0; r < bases.size(); ++r) p.route_base[r] = (uint64_t)bases[r];
  p.route_ld = (int)ld;
  p.route_chunk = chunk;
  p.route_flat0 = flat0;
  b200::GemmOperands op{dy.data_ptr(), x.data_ptr(), (uint64_t)dy.stride(0), (uint64_t)x.stride(0)};
  b200::gemm_launch(op, p, b200::EPI_ACC_F32_ROUTED, true, true, (int)bn, cur_stream());
}

// Adds src (fp32, contiguous) into the owners' gradient shards: element k has flat index flat0 + k,
// owned by rank (flat / chunk); bases[r] is rank r's shard as mapped on this GPU (see comm.h).
void routed_add(Tensor src, int64_t flat0, int64_t chunk, std::vector<int64_t> bases) {
  check_f32(src, "src");
  TORCH_CHECK(src.is_contiguous(), "routed_add: contiguous source required");
  TORCH_CHECK(!bases.empty() && (int)bases.size() <= b200::kCommMaxWorld, "routed_add: 1..8 shards");
  b200::RouteTable t{};
  t.world = (int)bases.size();
  t.chunk = chunk;
  for (size_t r = 0; r < bases.size(); ++r) t.base[r] = (uint64_t)bases[r];
  c10::cuda::CUDAGuard g(src.device());
  b200::comm_routed_add(src.data_ptr<float>(), (size_t)src.numel(), flat0, t, b200::device_errors_ptr(), cur_stream());
}

// Embedding backward straight into the owners' shards (routed ZeRO-2): see comm.h.
void embedding_bwd_routed(Tensor ids, Tensor dy, int64_t vocab, int64_t flat0, int64_t chunk,
                          std::vector<int64_t> bases) {
  check_cuda(ids, "ids");
  check_bf16_2d(dy, "dy");
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous() && ids.numel() == dy.size(0),
              "embedding_bwd_routed: one int64 id per dy row");
  TORCH_CHECK(dy.is_contiguous(), "embedding_bwd_routed: contiguous dy required");
  TORCH_CHECK(!bases.empty() && (int)bases.size() <= b200::kCommMaxWorld, "embedding_bwd_routed: 1..8 shards");
  b200::RouteTable t{};
  t.world = (int)bases.size();
  t.chunk = chunk;
  for (size_t r = 0; r < bases.size(); ++r) t.base[r] = (uint64_t)bases[r];
  c10::cuda::CUDAGuard g(dy.device());
  b200::comm_embedding_bwd_routed(ids.data_ptr<int64_t>(), dy.data_ptr(), (int)dy.size(0), (int)dy.size(1), (int)vocab,
                                  flat0, t, b200::device_errors_ptr(), cur_stream());
}

// dx = dy @ w and dw += dy^T @ x in one persistent launch (the two GEMMs of a linear layer's
// backward pass share dy and are independent of each other).
void linear_dgrad_wgrad(Tensor dy, Tensor w, Tensor x, Tensor dx, Tensor dw, int64_t splits) {
  check_bf16_2d(dy, "dy");
  check_bf16_2d(w, "w");
  check_bf16_2d(x, "x");
  check_bf16_2d(dx, "dx");
  check_f32(dw, "dw");
  const int T = dy.size(0), out = dy.size(1), in = w.size(1);
  TORCH_CHECK(w.size(0) == out && dx.size(0) == T && dx.size(1) == in, "linear_dgrad_wgrad: dgrad shape mismatch");
  TORCH_CHECK(x.size(0) == T && x.size(1) == in, "linear_dgrad_wgrad: x shape mismatch");
  TORCH_CHECK(dw.dim() == 2 && dw.size(0) == out && dw.size(1) == in && dw.stride(1) == 1, "linear_dgrad_wgrad: dw shape");
  TORCH_CHECK(dw.stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(dw.data_ptr()) % 16 == 0, "dw alignment");
  c10::cuda::CUDAGuard g(dy.device());
  auto p0 = base_params(T, in, out);
  p0.C = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  p0.ldc = dx.stride(0);
  b200::GemmOperands op0{dy.data_ptr(), w.data_ptr(), (uint64_t)dy.stride(0), (uint64_t)w.stride(0)};
  auto p1 = base_params(out, in, T);
  p1.C32 = dw.data_ptr<float>();
  p1.ldc32 = dw.stride(0);
  p1.splits = splits > 0 ? (int)splits : 0;
  b200::GemmOperands op1{dy.data_ptr(), x.data_ptr(), (uint64_t)dy.stride(0), (uint64_t)x.stride(0)};
  b200::gemm_launch_dgrad_wgrad(op0, p0, op1, p1, cur_stream());
}

// The grouped launch with its weight gradient routed to the owners' shards (see linear_wgrad_routed):
// dx = dy @ w, and dw = dy^T @ x added into the shards, element (o, i) at flat index flat0 + o * ld + i.
void linear_dgrad_wgrad_routed(Tensor dy, Tensor w, Tensor x, Tensor dx, int64_t flat0, int64_t ld, int64_t chunk,
                               std::vector<int64_t> bases, int64_t splits) {
  check_bf16_2d(dy, "dy");
  check_bf16_2d(w, "w");
  check_bf16_2d(x, "x");
  check_bf16_2d(dx, "dx");
  const int T = dy.size(0), out = dy.size(1), in = w.size(1);
  TORCH_CHECK(w.size(0) == out && dx.size(0) == T && dx.size(1) == in, "linear_dgrad_wgrad_routed: dgrad shapes");
  TORCH_CHECK(x.size(0) == T && x.size(1) == in, "linear_dgrad_wgrad_routed: x shape");
  TORCH_CHECK(!bases.empty() && (int)bases.size() <= b200::kRouteMaxWorld, "linear_dgrad_wgrad_routed: 1..8 shards");
  c10::cuda::CUDAGuard g(dy.device());
  auto p0 = base_params(T, in, out);
  p0.C = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  p0.ldc = dx.stride(0);
  b200::GemmOperands op0{dy.data_ptr(), w.data_ptr(), (uint64_t)dy.stride(0), (uint64_t)w.stride(0)};
  auto p1 = base_params(out, in, T);
  p1.splits = splits > 0 ? (int)splits : 0;
  p1.route_world = (int)bases.size();
  for (size_t r = 0; r < bases.size(); ++r) p1.route_base[r] = (uint64_t)bases[r];
  p1.route_ld = (int)ld;
  p1.route_chunk = chunk;
  p1.route_flat0 = flat0;
  b200::GemmOperands op1{dy.data_ptr(), x.data_ptr(), (uint64_t)dy.stride(0), (uint64_t)x.stride(0)};
  b200::gemm_launch_dgrad_wgrad(op0, p0, op1, p1, cur_stream());
}

// Host-only views of the GEMM schedulers (no GPU needed), for tests and tooling.
// (bn, splits, cg) that the automatic tile choice picks for one GEMM on `sms` SMs.
std::vector<int64_t> gemm_tile_choice(int64_t M, int64_t N, int64_t K, int64_t epi, int64_t head_dim, bool allow_split,
                                      bool b_mn, int64_t sms) {
  const b200::GemmTile t = b200::choose_gemm_tile((int)M, (int)N, (int)K, (int)epi, (int)head_dim, allow_split, b_mn,
                                                  (int)sms);
  return {t.bn, t.splits, t.cg};
}

// The grouped dgrad + wgrad schedule of a linear layer [T tokens, out x in weight] on `sms` SMs:
// (wgrad splits, wgrad k-blocks per split, problem dealt first, units of that problem, all units,
//  modelled makespan in k-blocks, dgrad tiles, wgrad tiles).
std::vector<int64_t> grouped_dgrad_wgrad_plan(int64_t T, int64_t out, int64_t in, int64_t sms, int64_t splits) {
  auto p0 = base_params((int)T, (int)in, (int)out);
  auto p1 = base_params((int)out, (int)in, (int)T);
  p1.splits = splits > 0 ? (int)splits : 0;
  const long span = b200::plan_dgrad_wgrad(p0, p1, (int)sms);
  return {p1.splits, p1.k_blocks_per_split, p0.grp_first, p0.grp_units_first, p0.grp_units_total, span,
          (int64_t)p0.tiles_m * p0.tiles_n, (int64_t)p1.tiles_m * p1.tiles_n};
}

// Generic entry for tests: C = A op B with explicit majors.
void gemm_raw(Tensor A, Tensor B, Tensor C, int64_t M, int64_t N, int64_t K, bool a_mn, bool b_mn, int64_t bn,
              int64_t splits) {
  check_bf16_2d(A, "A");
  check_bf16_2d(B, "B");
  c10::cuda::CUDAGuard g(A.device());
  auto p = base_params(M, N, K);
  int epi = b200::EPI_STORE;
  if (C.scalar_type() == at::kFloat) {
    p.C32 = C.data_ptr<float>();
    p.ldc32 = C.stride(0);
    p.splits = splits > 0 ? (int)splits : 1;
    epi = b200::EPI_ACC_F32;
  } else {
    check_bf16_2d(C, "C");
    p.C = reinterpret_cast<__nv_bfloat16*>(C.data_ptr());
    p.ldc = C.stride(0);
  }
  b200::GemmOperands op{A.data_ptr(), B.data_ptr(), (uint64_t)A.stride(0), (uint64_t)B.stride(0)};
  b200::gemm_launch(op, p, epi, a_mn, b_mn, (int)bn, cur_stream());
}

void rmsnorm_fwd(Tensor x, Tensor w, Tensor y, std::optional<Tensor> rstd, double eps) {
  check_bf16_2d(x, "x");
  check_bf16_2d(y, "y");
  check_cuda(w, "w");
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous(), "w must be contiguous bf16");
  TORCH_CHECK(x.stride(0) == x.size(1) && y.stride(0) == y.size(1), "rmsnorm: rows must be contiguous");
  c10::cuda::CUDAGuard g(x.device());
  float* r = nullptr;
  if (rstd.has_value()) {
    check_f32(*rstd, "rstd");
    r = rstd->data_ptr<float>();
  }
  b200::rmsnorm_fwd(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                    reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()),
                    r, x.size(0), x.size(1), (float)eps, cur_stream());
}

void rmsnorm_bwd(Tensor dy, Tensor x, Tensor w, Tensor rstd, std::optional<Tensor> dres, Tensor dx, Tensor dw) {
  check_bf16_2d(dy, "dy");
  check_bf16_2d(x, "x");
  check_bf16_2d(dx, "dx");
  check_f32(rstd, "rstd");
  check_f32(dw, "dw");
  TORCH_CHECK(dw.is_contiguous() && dw.numel() == x.size(1), "dw must be contiguous [d] fp32");
  c10::cuda::CUDAGuard g(x.device());
  const __nv_bfloat16* r = nullptr;
  if (dres.has_value()) {
    check_bf16_2d(*dres, "dres");
    r = reinterpret_cast<const __nv_bfloat16*>(dres->data_ptr());
  }
  b200::rmsnorm_bwd(reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()),
                    reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                    reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), rstd.data_ptr<float>(), r,
                    reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), dw.data_ptr<float>(), x.size(0), x.size(1),
                    cur_stream());
}

void embedding_fwd(Tensor ids, Tensor table, Tensor out) {
  check_cuda(ids, "ids");
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous(), "ids must be contiguous int64");
  check_bf16_2d(table, "table");
  check_bf16_2d(out, "out");
  c10::cuda::CUDAGuard g(table.device());
  b200::embedding_fwd(ids.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()),
                      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), ids.numel(), table.size(1), table.size(0),
                      cur_stream());
}

void embedding_bwd(Tensor ids, Tensor dy, Tensor dtable) {
  check_cuda(ids, "ids");
  check_bf16_2d(dy, "dy");
  check_f32(dtable, "dtable");
  TORCH_CHECK(dtable.is_contiguous() && reinterpret_cast<uintptr_t>(dtable.data_ptr()) % 16 == 0, "dtable layout");
  c10::cuda::CUDAGuard g(dy.device());
  b200::embedding_bwd(ids.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()),
                      dtable.data_ptr<float>(), ids.numel(), dy.size(1), dtable.size(0), cur_stream());
}

void rope_bwd(Tensor g, int64_t rope_cols, int64_t head_dim, int64_t seq_len, Tensor cos, Tensor sin) {
  check_bf16_2d(g, "g");
  check_f32(cos, "cos");
  check_f32(sin, "sin");
  c10::cuda::CUDAGuard gd(g.device());
  b200::rope_bwd(reinterpret_cast<__nv_bfloat16*>(g.data_ptr()), g.size(0), g.stride(0), rope_cols, head_dim,
                 seq_len, cos.data_ptr<float>(), sin.data_ptr<float>(), cur_stream());
}

// Device scalars of adam_advance: float32 [2] on the device of the optimizer state.
const float* dev_scalars_ptr(const std::optional<Tensor>& sc) {
  if (!sc.has_value()) return nullptr;
  check_f32(*sc, "dev_scalars");
  TORCH_CHECK(sc->numel() >= 2, "dev_scalars: 2 elements required");
  return sc->data_ptr<float>();
}

void adamw(Tensor master, Tensor m, Tensor v, Tensor grad, std::optional<Tensor> param_out,
           std::optional<Tensor> scale, double scale_const, double lr, double beta1, double beta2, double eps,
           double wd, int64_t step, std::optional<Tensor> dev_scalars) {
  check_f32(master, "master");
  check_f32(m, "exp_avg");
  check_f32(v, "exp_avg_sq");
  check_f32(grad, "grad");
  const size_t n = master.numel();
  TORCH_CHECK(m.numel() == (int64_t)n && v.numel() == (int64_t)n && grad.numel() == (int64_t)n, "adamw: sizes");
  TORCH_CHECK(master.is_contiguous() && m.is_contiguous() && v.is_contiguous() && grad.is_contiguous(),
              "adamw: contiguous state required");
  c10::cuda::CUDAGuard g(master.device());
  void* out = nullptr;
  bool out_bf16 = false;
  if (param_out.has_value()) {
    check_cuda(*param_out, "param_out");
    TORCH_CHECK(param_out->numel() == (int64_t)n && param_out->is_contiguous(), "adamw: param_out");
    out_bf16 = param_out->scalar_type() == at::kBFloat16;
    TORCH_CHECK(out_bf16 || param_out->scalar_type() == at::kFloat, "adamw: param_out dtype");
    out = param_out->data_ptr();
  }
  const float* sp = nullptr;
  if (scale.has_value()) {
    check_f32(*scale, "scale");
    sp = scale->data_ptr<float>();
  }
  b200::adamw_step(master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), grad.data_ptr<float>(), out,
                   out_bf16, n, sp, (float)scale_const, (float)lr, (float)beta1, (float)beta2, (float)eps, (float)wd,
                   (int)step, cur_stream(), dev_scalars_ptr(dev_scalars));
}

// step_count (int32 [1]) += 1 and dev_scalars (float32 [2]) = the bias corrections of the new step, on
// the current stream: the optimizer's step number lives on the device, so a captured step replays.
void adam_advance(Tensor step_count, Tensor dev_scalars, double lr, double beta1, double beta2) {
  check_cuda(step_count, "step_count");
  TORCH_CHECK(step_count.scalar_type() == at::kInt && step_count.numel() >= 1, "adam_advance: int32 step counter");
  const float* sc = dev_scalars_ptr(dev_scalars);
  c10::cuda::CUDAGuard g(step_count.device());
  b200::adam_advance(step_count.data_ptr<int32_t>(), const_cast<float*>(sc), (float)lr, (float)beta1, (float)beta2,
                     cur_stream());
}

void sum_squares(Tensor x, Tensor out) {
  check_cuda(x, "x");
  check_f32(out, "out");
  TORCH_CHECK(x.is_contiguous(), "sum_squares: contiguous input required");
  TORCH_CHECK(x.scalar_type() == at::kFloat || x.scalar_type() == at::kBFloat16, "sum_squares dtype");
  c10::cuda::CUDAGuard g(x.device());
  b200::sum_squares(x.data_ptr(), x.scalar_type() == at::kBFloat16, x.numel(), out.data_ptr<float>(), cur_stream());
}

void cross_entropy_fwd(Tensor logits, Tensor targets, Tensor lse, Tensor loss_sum, Tensor count, Tensor loss) {
  check_bf16_2d(logits, "logits");
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.numel() == logits.size(0), "targets");
  c10::cuda::CUDAGuard g(logits.device());
  b200::cross_entropy_fwd(reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0),
                          targets.data_ptr<int64_t>(), logits.size(0), logits.size(1), lse.data_ptr<float>(),
                          loss_sum.data_ptr<float>(), count.data_ptr<float>(), loss.data_ptr<float>(), cur_stream());
}

void cross_entropy_bwd(Tensor logits, Tensor targets, Tensor lse, Tensor grad_loss, Tensor count) {
  check_bf16_2d(logits, "logits");
  c10::cuda::CUDAGuard g(logits.device());
  b200::cross_entropy_bwd(reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), logits.stride(0),
                          targets.data_ptr<int64_t>(), logits.size(0), logits.size(1), lse.data_ptr<float>(),
                          grad_loss.data_ptr<float>(), count.data_ptr<float>(), cur_stream());
}

// Column layout of the fused q|k|v rows and of the attention output rows: q at 0, k at k_col, v at
// v_col, each block inside the row and before the next one; every query head inside an output row.
void check_attn_columns(int64_t qkv_ld, int64_t k_col, int64_t v_col, int64_t out_ld, int64_t heads, int64_t kv_heads,
                        int64_t head_dim) {
  const int64_t q_w = heads * head_dim, kv_w = kv_heads * head_dim;
  TORCH_CHECK(q_w <= k_col, "attention: q columns (heads*head_dim = ", q_w, ") overlap k_col = ", k_col);
  TORCH_CHECK(k_col + kv_w <= v_col, "attention: k columns end at ", k_col + kv_w, " past v_col = ", v_col);
  TORCH_CHECK(v_col + kv_w <= qkv_ld, "attention: v columns end at ", v_col + kv_w, " past the row stride ", qkv_ld);
  TORCH_CHECK(q_w <= out_ld, "attention: output rows (stride ", out_ld, ") hold fewer than heads*head_dim = ", q_w);
}

void attention_fwd(Tensor qkv, int64_t k_col, int64_t v_col, Tensor out, Tensor lse, int64_t batch, int64_t seq,
                   int64_t heads, int64_t kv_heads, int64_t head_dim, double scale) {
  check_bf16_2d(qkv, "qkv");
  check_bf16_2d(out, "out");
  check_f32(lse, "lse");
  TORCH_CHECK(qkv.size(0) == batch * seq && out.size(0) == batch * seq, "attention: row count");
  TORCH_CHECK(lse.numel() == batch * heads * seq, "attention: lse size");
  TORCH_CHECK(out.size(1) >= heads * head_dim, "attention: out has fewer columns than heads*head_dim");
  check_attn_columns(qkv.stride(0), k_col, v_col, out.stride(0), heads, kv_heads, head_dim);
  TORCH_CHECK(qkv.size(1) >= v_col + kv_heads * head_dim, "attention: qkv has fewer columns than its v block needs");
  c10::cuda::CUDAGuard g(qkv.device());
  b200::AttnParams p{};
  p.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  p.ld = qkv.stride(0);
  p.k_col = k_col;
  p.v_col = v_col;
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ld_out = out.stride(0);
  p.lse = lse.data_ptr<float>();
  p.batch = batch;
  p.seq = seq;
  p.heads = heads;
  p.kv_heads = kv_heads;
  p.head_dim = head_dim;
  p.scale = (float)scale;
  b200::attention_fwd(p, cur_stream());
}

void attention_bwd(Tensor qkv, int64_t k_col, int64_t v_col, Tensor out, Tensor dout, Tensor lse, Tensor delta,
                   Tensor dq_acc, Tensor dqkv, Tensor cos, Tensor sin, int64_t batch, int64_t seq, int64_t heads,
                   int64_t kv_heads, int64_t head_dim, double scale, bool rezero_dq_acc) {
  check_f32(cos, "cos");
  check_f32(sin, "sin");
  TORCH_CHECK(cos.numel() >= seq * head_dim / 2 && sin.numel() >= seq * head_dim / 2, "rope table too small");
  check_bf16_2d(qkv, "qkv");
  check_bf16_2d(out, "out");
  check_bf16_2d(dout, "dout");
  check_bf16_2d(dqkv, "dqkv");
  check_f32(lse, "lse");
  check_f32(delta, "delta");
  check_f32(dq_acc, "dq_acc");
  TORCH_CHECK(dq_acc.numel() >= batch * seq * heads * head_dim, "dq_acc too small");
  TORCH_CHECK(dqkv.stride(0) == qkv.stride(0), "dqkv must share the qkv row stride");
  TORCH_CHECK(qkv.size(0) == batch * seq && out.size(0) == batch * seq && dout.size(0) == batch * seq &&
                  dqkv.size(0) == batch * seq, "attention_bwd: row count");
  check_attn_columns(qkv.stride(0), k_col, v_col, out.stride(0), heads, kv_heads, head_dim);
  TORCH_CHECK(qkv.size(1) >= v_col + kv_heads * head_dim && dqkv.size(1) >= v_col + kv_heads * head_dim,
              "attention_bwd: qkv / dqkv have fewer columns than the v block needs");
  TORCH_CHECK(out.size(1) >= heads * head_dim && dout.size(1) >= heads * head_dim,
              "attention_bwd: out / dout have fewer columns than heads*head_dim");
  c10::cuda::CUDAGuard g(qkv.device());
  b200::AttnBwdParams p{};
  p.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  p.ld = qkv.stride(0);
  p.k_col = k_col;
  p.v_col = v_col;
  p.out = reinterpret_cast<const __nv_bfloat16*>(out.data_ptr());
  p.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  p.ld_out = out.stride(0);
  TORCH_CHECK(dout.stride(0) == out.stride(0), "dout must share the output row stride");
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.dq_acc = dq_acc.data_ptr<float>();
  p.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  p.rope_cos = cos.data_ptr<float>();
  p.rope_sin = sin.data_ptr<float>();
  p.batch = batch;
  p.seq = seq;
  p.heads = heads;
  p.kv_heads = kv_heads;
  p.head_dim = head_dim;
  p.scale = (float)scale;
  p.rezero_dq_acc = rezero_dq_acc;
  b200::attention_bwd(p, cur_stream());
}

// ----------------------------------------------------------------------------------- comm
// Python-side handle for one symmetric buffer: peer / multicast / signal-pad addresses come from
// the symmetric-memory rendezvous; the per-block epoch counters are a small local int32 tensor.
class CommContext {
 public:
  CommContext(int64_t rank, int64_t world, std::vector<int64_t> peers, int64_t mc, std::vector<int64_t> pads,
              Tensor epochs, int64_t blocks, int64_t timeout_ns)
      : epochs_(epochs), device_(epochs.device()) {
    TORCH_CHECK(world >= 1 && world <= b200::kCommMaxWorld, "comm: world size 1..8");
    TORCH_CHECK((int64_t)peers.size() == world && (int64_t)pads.size() == world, "comm: one peer/pad per rank");
    TORCH_CHECK(epochs.is_cuda() && epochs.scalar_type() == at::kInt && epochs.numel() >= b200::kCommMaxBlocks,
                "comm: epochs must be a CUDA int32 tensor of at least 64 elements");
    TORCH_CHECK(blocks >= 1 && blocks < b200::kCommMaxBlocks, "comm: blocks 1..63");
    c_ = b200::CommCtx{};
    c_.rank = rank;
    c_.world = world;
    for (int i = 0; i < world; ++i) {
      c_.peers[i] = (uint64_t)peers[i];
      c_.pads[i] = (uint64_t)pads[i];
    }
    c_.mc = (uint64_t)mc;
    c_.epochs = reinterpret_cast<uint32_t*>(epochs.data_ptr<int32_t>());
    c_.timeout_ns = (uint64_t)timeout_ns;
    c_.blocks = blocks;
  }
  void allreduce_f32(int64_t off, int64_t n, double scale) {
    c10::cuda::CUDAGuard g(device_);
    prepare();
    b200::comm_allreduce_f32(c_, off, n, (float)scale, cur_stream());
  }
  void allreduce_bf16(int64_t off, int64_t n, double scale) {
    c10::cuda::CUDAGuard g(device_);
    prepare();
    b200::comm_allreduce_bf16(c_, off, n, (float)scale, cur_stream());
  }
  void reduce_scatter_acc_f32(int64_t off, int64_t chunk, Tensor acc, double scale) {
    check_acc(acc, chunk);
    c10::cuda::CUDAGuard g(device_);
    prepare();
    b200::comm_reduce_scatter_acc_f32(c_, off, chunk, acc.data_ptr<float>(), (float)scale, cur_stream());
  }
  void reduce_scatter_range_acc_f32(int64_t off, int64_t lo, int64_t hi, Tensor acc, double scale, int64_t blocks) {
    TORCH_CHECK(hi >= lo, "reduce_scatter_range: hi < lo");
    check_acc(acc, hi - lo);
    c10::cuda::CUDAGuard g(device_);
    prepare();
    b200::comm_reduce_scatter_range_acc_f32(c_, off, lo, hi, acc.data_ptr<float>(), (float)scale, (int)blocks,
                                            cur_stream());
  }
  // Gradient ring: acc[0, part) += scale * sum_ranks(slice `rank` of the bucket at off); the bucket is
  // zero on every rank afterwards (see comm.h).
  void bucket_reduce(int64_t off, int64_t part, Tensor acc, double scale, int64_t blocks) {
    check_acc(acc, part);
    c10::cuda::CUDAGuard g(device_);
    prepare();
    b200::comm_bucket_reduce(c_, off, part, acc.data_ptr<float>(), (float)scale, (int)blocks, cur_stream());
  }
  // AdamW on an interleaved ring shard + bf16 all-gather into this (parameter) buffer.  segs: int64
  // CUDA tensor [nseg, 4] of (shard8, part8, valid8, param_off) rows.
  void adamw_allgather_seg(Tensor segs, int64_t total, Tensor master, Tensor m, Tensor v, Tensor grad,
                           std::optional<Tensor> scale, double scale_const, double lr, double beta1, double beta2,
                           double eps, double wd, int64_t step, std::optional<Tensor> dev_scalars) {
    TORCH_CHECK(segs.is_cuda() && segs.scalar_type() == at::kLong && segs.dim() == 2 && segs.size(1) == 4 &&
                    segs.is_contiguous() && segs.size(0) >= 1,
                "adamw_allgather_seg: segments must be a contiguous CUDA int64 [n, 4] tensor");
    for (auto* t : {&master, &m, &v, &grad}) {
      check_f32(*t, "adam state");
      TORCH_CHECK(t->is_contiguous() && t->numel() >= total, "adam state too small");
    }
    const float* sp = nullptr;
    if (scale.has_value()) {
      check_f32(*scale, "scale");
      sp = scale->data_ptr<float>();
    }
    c10::cuda::CUDAGuard g(device_);
    prepare();
    static_assert(sizeof(b200::RingSeg) == 4 * sizeof(int64_t), "RingSeg layout");
    b200::comm_adamw_allgather_seg(c_, reinterpret_cast<const b200::RingSeg*>(segs.data_ptr<int64_t>()),
                                   (int)segs.size(0), (size_t)total, master.data_ptr<float>(), m.data_ptr<float>(),
                                   v.data_ptr<float>(), grad.data_ptr<float>(), sp, (float)scale_const, (float)lr,
                                   (float)beta1, (float)beta2, (float)eps, (float)wd, (int)step, cur_stream(),
                                   dev_scalars_ptr(dev_scalars));
  }
  // Push reduce-scatter with this buffer as the landing area (see comm.h).
  void push_reduce_scatter_f32(Tensor src, int64_t src_stride, int64_t land_off, int64_t part, Tensor acc,
                               double scale, bool clear_src) {
    check_f32(src, "src");
    TORCH_CHECK(src.is_contiguous() && src_stride >= part && src.numel() >= src_stride * (c_.world - 1) + part,
                "push_reduce_scatter: src too small for W slices");
    check_acc(acc, part);
    c10::cuda::CUDAGuard g(device_);
    prepare();
    b200::comm_push_reduce_scatter_f32(c_, src.data_ptr<float>(), src_stride, land_off, part, acc.data_ptr<float>(),
                                       (float)scale, clear_src, cur_stream());
  }
  void reduce_scatter_acc_bf16(int64_t off, int64_t chunk, Tensor acc, double scale) {
    check_acc(acc, chunk);
    c10::cuda::CUDAGuard g(device_);
    prepare();
    b200::comm_reduce_scatter_acc_bf16(c_, off, chunk, acc.data_ptr<float>(), (float)scale, cur_stream());
  }
  void allgather(int64_t off, int64_t chunk_bytes, Tensor shard) {
    check_cuda(shard, "shard");
    TORCH_CHECK(shard.is_contiguous() && shard.numel() * shard.element_size() >= chunk_bytes, "shard too small");
    c10::cuda::CUDAGuard g(device_);
    prepare();
    b200::comm_allgather(c_, off, chunk_bytes, shard.data_ptr(), cur_stream());
  }
  void gather_ce(int64_t off, int64_t chunk_bytes, Tensor dst) {
    TORCH_CHECK(dst.is_cuda() && dst.is_contiguous(), "gather_ce: contiguous CUDA destination required");
    TORCH_CHECK(dst.numel() * dst.element_size() >= chunk_bytes * c_.world, "gather_ce: destination too small");
    c10::cuda::CUDAGuard g(device_);
    b200::comm_gather_ce(c_, off, chunk_bytes, dst.data_ptr(), cur_stream());
  }
  void adamw_allgather(int64_t param_off, int64_t chunk, Tensor master, Tensor m, Tensor v, Tensor grad,
                       std::optional<Tensor> scale, double scale_const, double lr, double beta1, double beta2,
                       double eps, double wd, int64_t step, std::optional<Tensor> dev_scalars) {
    for (auto* t : {&master, &m, &v, &grad}) {
      check_f32(*t, "adam state");
      TORCH_CHECK(t->is_contiguous() && t->numel() >= chunk, "adam state too small");
    }
    const float* sp = nullptr;
    if (scale.has_value()) {
      check_f32(*scale, "scale");
      sp = scale->data_ptr<float>();
    }
    c10::cuda::CUDAGuard g(device_);
    prepare();
    b200::comm_adamw_allgather(c_, param_off, chunk, master.data_ptr<float>(), m.data_ptr<float>(),
                               v.data_ptr<float>(), grad.data_ptr<float>(), sp, (float)scale_const, (float)lr,
                               (float)beta1, (float)beta2, (float)eps, (float)wd, (int)step, cur_stream(),
                               dev_scalars_ptr(dev_scalars));
  }
  // The ZeRO-2 step without clipping in one kernel (see comm.h): `grads` is the context of the flat
  // fp32 gradient buffer, this context the bf16 parameter buffer.
  void rs_adamw_allgather(CommContext& grads, int64_t g_off, int64_t param_off, int64_t chunk, Tensor master,
                          Tensor m, Tensor v, double grad_scale, double lr, double beta1, double beta2, double eps,
                          double wd, int64_t step, std::optional<Tensor> dev_scalars, std::optional<Tensor> sq_out) {
    for (auto* t : {&master, &m, &v}) {
      check_f32(*t, "adam state");
      TORCH_CHECK(t->is_contiguous() && t->numel() >= chunk, "adam state too small");
    }
    TORCH_CHECK(grads.device() == device_, "rs_adamw_allgather: buffers on different devices");
    float* sq = nullptr;
    if (sq_out.has_value()) {
      check_f32(*sq_out, "sq_out");
      sq = sq_out->data_ptr<float>();
    }
    c10::cuda::CUDAGuard g(device_);
    prepare();
    grads.prepare();
    b200::comm_rs_adamw_allgather(c_, grads.c_, g_off, param_off, chunk, master.data_ptr<float>(),
                                  m.data_ptr<float>(), v.data_ptr<float>(), (float)grad_scale, (float)lr, (float)beta1,
                                  (float)beta2, (float)eps, (float)wd, (int)step, dev_scalars_ptr(dev_scalars), sq,
                                  cur_stream());
  }
  void barrier() {
    c10::cuda::CUDAGuard g(device_);
    prepare();
    b200::comm_barrier(c_, cur_stream());
  }
  void wait_unsignalled(int64_t timeout_ns) {
    c10::cuda::CUDAGuard g(device_);
    prepare();
    b200::comm_wait_unsignalled(c_, (uint64_t)timeout_ns, cur_stream());
  }
  bool multicast() const { return c_.mc != 0; }
  int64_t blocks() const { return c_.blocks; }
  // Copy-engine pull of every rank's region[off, off + chunk_bytes) into dst on stream s.
  void gather_ce_on(int64_t off, int64_t chunk_bytes, void* dst, cudaStream_t s) const {
    b200::comm_gather_ce(c_, off, chunk_bytes, dst, s);
  }
  int64_t world() const { return c_.world; }
  const c10::Device& device() const { return device_; }

 private:
  void prepare() { c_.errs = b200::device_errors_ptr(); }
  static void check_acc(const Tensor& acc, int64_t chunk) {
    check_f32(acc, "acc");
    TORCH_CHECK(acc.numel() >= chunk && acc.is_contiguous(), "acc too small or not contiguous");
  }
  b200::CommCtx c_;
  Tensor epochs_;
  c10::Device device_;
};

// Cost in ns of `link_bytes` bytes on an emulated link of `gbps` Gbit/s plus a fixed latency
// (bits / (Gbit/s) = ns).  gbps <= 0 means no bandwidth term.
int64_t pace_cost_ns(int64_t link_bytes, double gbps, double latency_ms) {
  double ns = latency_ms > 0 ? latency_ms * 1e6 : 0.0;
  if (gbps > 0) ns += 8.0 * (double)link_bytes / gbps;
  return (int64_t)std::llround(ns);
}

// One GPU's emulated link for the `nvlink` bandwidth mode: owns the device state of the paced
// transfers (link free time + start stamps) and hands out stamp slots round-robin.  Shared by the
// collectives on the compute stream and the ZeRO-3 gathers on their side stream, so both queue on
// the same link.
class LinkPacer {
 public:
  LinkPacer(int64_t device_index, double gbps, double latency_ms, int64_t timeout_ns)
      : device_(c10::Device(c10::DeviceType::CUDA, (c10::DeviceIndex)device_index)),
        gbps_(gbps), latency_ms_(latency_ms), timeout_ns_(timeout_ns) {
    c10::cuda::CUDAGuard g(device_);
    state_ = at::zeros({1 + b200::kPaceSlots}, at::TensorOptions().dtype(at::kLong).device(device_));
  }
  int64_t cost_ns(int64_t link_bytes) const { return pace_cost_ns(link_bytes, gbps_, latency_ms_); }
  int64_t begin_on(cudaStream_t s) {
    c10::cuda::CUDAGuard g(device_);
    const int slot = (int)(next_++ % b200::kPaceSlots);
    b200::comm_pace_begin(state(), slot, s);
    return slot;
  }
  void end_on(int64_t slot, int64_t link_bytes, cudaStream_t s) {
    c10::cuda::CUDAGuard g(device_);
    b200::comm_pace_end(state(), (int)slot, (uint64_t)cost_ns(link_bytes), (uint64_t)timeout_ns_,
                        b200::device_errors_ptr(), s);
  }
  int64_t begin() {
    c10::cuda::CUDAGuard g(device_);
    return begin_on(cur_stream());
  }
  void end(int64_t slot, int64_t link_bytes) {
    c10::cuda::CUDAGuard g(device_);
    end_on(slot, link_bytes, cur_stream());
  }
  double gbps() const { return gbps_; }
  double latency_ms() const { return latency_ms_; }
  Tensor state_tensor() const { return state_; }

 private:
  uint64_t* state() { return reinterpret_cast<uint64_t*>(state_.data_ptr<int64_t>()); }
  c10::Device device_;
  double gbps_, latency_ms_;
  int64_t timeout_ns_;
  Tensor state_;
  uint64_t next_ = 0;
};

// Stream/event plumbing of the ZeRO-3 prefetching parameter gather, kept native so that one module's
// prefetch costs one call from Python.  Slots are staging buffers; for each slot the object keeps
// the event that the last gather into it finished (`written`) and the event that its last reader
// on the compute stream finished (`used`).  Gathers are copy-engine pulls (no kernel).  Each gather
// can be timed with a pair of events into one of a few categories.
class PullGather {
 public:
  PullGather(int64_t slots, int64_t categories, int64_t device_index)
      : device_(c10::Device(c10::DeviceType::CUDA, (c10::DeviceIndex)device_index)),
        side_(at::cuda::getStreamFromPool(false, (c10::DeviceIndex)device_index)) {
    TORCH_CHECK(slots >= 1 && slots <= 16 && categories >= 1, "PullGather: 1..16 slots");
    c10::cuda::CUDAGuard g(device_);
    written_.resize(slots);
    used_.resize(slots);
    has_written_.assign(slots, false);
    has_used_.assign(slots, false);
    for (int64_t i = 0; i < slots; ++i) {
      B200_CUDA_CHECK(cudaEventCreateWithFlags(&written_[i], cudaEventDisableTiming));
      B200_CUDA_CHECK(cudaEventCreateWithFlags(&used_[i], cudaEventDisableTiming));
    }
    B200_CUDA_CHECK(cudaEventCreateWithFlags(&ready_, cudaEventDisableTiming));
    B200_CUDA_CHECK(cudaEventCreateWithFlags(&join_, cudaEventDisableTiming));
    ms_.assign(categories, 0.0);
    calls_.assign(categories, 0);
  }
  ~PullGather() {
    for (auto e : written_) cudaEventDestroy(e);
    for (auto e : used_) cudaEventDestroy(e);
    for (auto& t : timed_) {
      cudaEventDestroy(t.start);
      cudaEventDestroy(t.end);
    }
    for (auto e : free_timing_) cudaEventDestroy(e);
    cudaEventDestroy(ready_);
    cudaEventDestroy(join_);
  }

  // Gather into `slot` on the side stream, after the slot's last reader and after the last
  // mark_ready(); the compute stream picks it up with acquire(slot).
  void prefetch(const CommContext& ctx, int64_t slot, int64_t off, int64_t chunk_bytes, int64_t dst,
                int64_t category, bool timed) {
    c10::cuda::CUDAGuard g(device_);
    cudaStream_t s = side_.stream();
    if (has_used_.at(slot)) B200_CUDA_CHECK(cudaStreamWaitEvent(s, used_[slot], 0));
    if (has_ready_) B200_CUDA_CHECK(cudaStreamWaitEvent(s, ready_, 0));
    copy(ctx, off, chunk_bytes, dst, category, timed, s);
    B200_CUDA_CHECK(cudaEventRecord(written_[slot], s));
    has_written_[slot] = true;
  }
  // Gather into `slot` on the current stream (after any side-stream gather still writing it).
  void gather_now(const CommContext& ctx, int64_t slot, int64_t off, int64_t chunk_bytes, int64_t dst,
                  int64_t category, bool timed) {
    c10::cuda::CUDAGuard g(device_);
    cudaStream_t s = cur_stream();
    if (has_written_.at(slot)) B200_CUDA_CHECK(cudaStreamWaitEvent(s, written_[slot], 0));
    copy(ctx, off, chunk_bytes, dst, category, timed, s);
  }
  // The current stream waits for the side-stream gather into `slot`.
  void acquire(int64_t slot) {
    c10::cuda::CUDAGuard g(device_);
    if (has_written_.at(slot)) B200_CUDA_CHECK(cudaStreamWaitEvent(cur_stream(), written_[slot], 0));
  }
  // The slot's reader (queued on the current stream so far) is done with it once this point is reached.
  void release(int64_t slot) {
    c10::cuda::CUDAGuard g(device_);
    B200_CUDA_CHECK(cudaEventRecord(used_.at(slot), cur_stream()));
    has_used_[slot] = true;
  }
  // Later gathers start after the work queued on the current stream so far (the barrier that
  // follows the stores' rewrite).
  void mark_ready() {
    c10::cuda::CUDAGuard g(device_);
    B200_CUDA_CHECK(cudaEventRecord(ready_, cur_stream()));
    has_ready_ = true;
  }
  // The current stream waits for every gather issued so far.
  void join() {
    c10::cuda::CUDAGuard g(device_);
    B200_CUDA_CHECK(cudaEventRecord(join_, side_.stream()));
    B200_CUDA_CHECK(cudaStreamWaitEvent(cur_stream(), join_, 0));
  }
  // Per-category totals (ms) and call counts of the timed gathers since the last call; waits for them.
  std::pair<std::vector<double>, std::vector<int64_t>> take_times() {
    c10::cuda::CUDAGuard g(device_);
    for (auto& t : timed_) {
      B200_CUDA_CHECK(cudaEventSynchronize(t.end));
      float ms = 0.f;
      B200_CUDA_CHECK(cudaEventElapsedTime(&ms, t.start, t.end));
      ms_[t.category] += ms;
      calls_[t.category] += 1;
      free_timing_.push_back(t.start);
      free_timing_.push_back(t.end);
    }
    timed_.clear();
    auto out = std::make_pair(ms_, calls_);
    std::fill(ms_.begin(), ms_.end(), 0.0);
    std::fill(calls_.begin(), calls_.end(), 0);
    return out;
  }
  void reset_times() { take_times(); }
  int64_t side_stream() const { return (int64_t)side_.stream(); }
  // Pace every later gather on `pacer`'s emulated link (None: stop pacing).  A gather moves
  // (world - 1) shards across this GPU's link.
  void set_pacer(std::shared_ptr<LinkPacer> pacer) { pacer_ = std::move(pacer); }

 private:
  struct Timed {
    cudaEvent_t start, end;
    int64_t category;
  };
  cudaEvent_t timing_event() {
    if (!free_timing_.empty()) {
      cudaEvent_t e = free_timing_.back();
      free_timing_.pop_back();
      return e;
    }
    cudaEvent_t e;
    B200_CUDA_CHECK(cudaEventCreate(&e));
    return e;
  }
  void copy(const CommContext& ctx, int64_t off, int64_t chunk_bytes, int64_t dst, int64_t category, bool timed,
            cudaStream_t s) {
    TORCH_CHECK(ctx.device() == device_, "PullGather: communicator on another device");
    TORCH_CHECK(category >= 0 && category < (int64_t)ms_.size(), "PullGather: bad category");
    Timed t{nullptr, nullptr, category};
    if (timed) {
      t.start = timing_event();
      t.end = timing_event();
      B200_CUDA_CHECK(cudaEventRecord(t.start, s));
    }
    const int64_t slot = pacer_ ? pacer_->begin_on(s) : -1;
    ctx.gather_ce_on(off, chunk_bytes, reinterpret_cast<void*>(dst), s);
    if (pacer_) pacer_->end_on(slot, (ctx.world() - 1) * chunk_bytes, s);
    if (timed) {
      B200_CUDA_CHECK(cudaEventRecord(t.end, s));
      timed_.push_back(t);
    }
  }
  c10::Device device_;
  at::cuda::CUDAStream side_;
  std::vector<cudaEvent_t> written_, used_, free_timing_;
  std::vector<bool> has_written_, has_used_;
  bool has_ready_ = false;
  cudaEvent_t ready_, join_;
  std::vector<Timed> timed_;
  std::vector<double> ms_;
  std::vector<int64_t> calls_;
  std::shared_ptr<LinkPacer> pacer_;
};

int64_t launch_count() { return b200::launch_counter().load(); }
// A CUDA-graph replay launches the kernels it captured as graph nodes: count them as launches.
void add_launch_count(int64_t n) { b200::count_launch((int)n); }

std::vector<int64_t> read_device_errors() {
  b200::DeviceErrors e{};
  B200_CUDA_CHECK(cudaMemcpy(&e, b200::device_errors_ptr(), sizeof(e), cudaMemcpyDeviceToHost));
  return {e.code, e.where, e.block, e.count};
}

void reset_device_errors() { B200_CUDA_CHECK(cudaMemset(b200::device_errors_ptr(), 0, sizeof(b200::DeviceErrors))); }

// Copies this device's error record into `host` (pinned int32[4]: code, where, block, count) on the
// current stream, without synchronising: read it once an event recorded after this call completes.
void device_errors_to_host(Tensor host) {
  TORCH_CHECK(!host.is_cuda() && host.is_pinned() && host.scalar_type() == at::kInt && host.numel() >= 4 &&
                  host.is_contiguous(),
              "device_errors_to_host: pinned contiguous int32 host tensor of >= 4 elements required");
  B200_CUDA_CHECK(cudaMemcpyAsync(host.data_ptr<int32_t>(), b200::device_errors_ptr(), sizeof(b200::DeviceErrors),
                                  cudaMemcpyDeviceToHost, cur_stream()));
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels: tcgen05 GEMMs with fused epilogues, flash attention, norms, optimizer, collectives";
  m.def("linear_fwd", &linear_fwd, py::arg("x"), py::arg("w"), py::arg("out"), py::arg("residual") = py::none(),
        py::arg("bn") = 0);
  m.def("qkv_rope_fwd", &qkv_rope_fwd, py::arg("x"), py::arg("w"), py::arg("out"), py::arg("cos"), py::arg("sin"),
        py::arg("seq_len"), py::arg("head_dim"), py::arg("rope_cols"), py::arg("bn") = 0);
  m.def("swiglu_fwd", &swiglu_fwd, py::arg("x"), py::arg("w_gu"), py::arg("h"), py::arg("gu"), py::arg("bn") = 0);
  m.def("linear_dgrad", &linear_dgrad, py::arg("dy"), py::arg("w"), py::arg("dx"), py::arg("bn") = 0);
  m.def("gemm_tile_choice", &gemm_tile_choice, py::arg("M"), py::arg("N"), py::arg("K"), py::arg("epi"),
        py::arg("head_dim"), py::arg("allow_split"), py::arg("b_mn"), py::arg("sms"));
  m.def("grouped_dgrad_wgrad_plan", &grouped_dgrad_wgrad_plan, py::arg("T"), py::arg("out"), py::arg("inp"),
        py::arg("sms"), py::arg("splits") = 0);
  m.def("linear_dgrad_wgrad", &linear_dgrad_wgrad, py::arg("dy"), py::arg("w"), py::arg("x"), py::arg("dx"),
        py::arg("dw"), py::arg("splits") = 0);
  m.def("swiglu_dgrad", &swiglu_dgrad);
  m.def("linear_dgrad_wgrad_routed", &linear_dgrad_wgrad_routed, py::arg("dy"), py::arg("w"), py::arg("x"),
        py::arg("dx"), py::arg("flat0"), py::arg("ld"), py::arg("chunk"), py::arg("bases"), py::arg("splits") = 0);
  m.def("embedding_bwd_routed", &embedding_bwd_routed, py::arg("ids"), py::arg("dy"), py::arg("vocab"),
        py::arg("flat0"), py::arg("chunk"), py::arg("bases"));
  m.def("routed_add", &routed_add, py::arg("src"), py::arg("flat0"), py::arg("chunk"), py::arg("bases"));
  m.def("linear_wgrad_routed", &linear_wgrad_routed, py::arg("dy"), py::arg("x"), py::arg("flat0"), py::arg("ld"),
        py::arg("chunk"), py::arg("bases"), py::arg("splits") = 0, py::arg("bn") = 0);
  m.def("linear_wgrad", &linear_wgrad, py::arg("dy"), py::arg("x"), py::arg("dw"), py::arg("splits") = 0,
        py::arg("bn") = 0);
  m.def("gemm_raw", &gemm_raw);
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("embedding_fwd", &embedding_fwd);
  m.def("embedding_bwd", &embedding_bwd);
  m.def("rope_bwd", &rope_bwd);
  m.def("adamw", &adamw, py::arg("master"), py::arg("m"), py::arg("v"), py::arg("grad"), py::arg("param_out"),
        py::arg("scale"), py::arg("scale_const"), py::arg("lr"), py::arg("beta1"), py::arg("beta2"), py::arg("eps"),
        py::arg("wd"), py::arg("step"), py::arg("dev_scalars") = py::none());
  m.def("adam_advance", &adam_advance);
  m.def("sum_squares", &sum_squares);
  m.def("record_if_different", [](Tensor a, Tensor b, int64_t code) {
    check_f32(a, "a");
    check_f32(b, "b");
    c10::cuda::CUDAGuard g(a.device());
    b200::record_if_different(a.data_ptr<float>(), b.data_ptr<float>(), (int)code, cur_stream());
  }, "error record gets `code` when the two device scalars differ");
  m.def("cross_entropy_fwd", &cross_entropy_fwd);
  m.def("cross_entropy_bwd", &cross_entropy_bwd);
  m.def("attention_fwd", &attention_fwd);
  m.def("attention_trace", []() {
    auto out = torch::empty({3, b200::kAttnTraceWords}, torch::dtype(torch::kInt64));
    b200::attention_trace_read(reinterpret_cast<unsigned long long*>(out.data_ptr<int64_t>()));
    return out;
  }, "debug: phase clocks of CTA 0 of the last attention forward run with ZB_ATTN_TRACE=1");
  m.def("attention_bwd", &attention_bwd, py::arg("qkv"), py::arg("k_col"), py::arg("v_col"), py::arg("out"),
        py::arg("dout"), py::arg("lse"), py::arg("delta"), py::arg("dq_acc"), py::arg("dqkv"), py::arg("cos"),
        py::arg("sin"), py::arg("batch"), py::arg("seq"), py::arg("heads"), py::arg("kv_heads"), py::arg("head_dim"),
        py::arg("scale"), py::arg("rezero_dq_acc") = false);
  m.def("launch_count", &launch_count);
  m.def("add_launch_count", &add_launch_count);
  m.def("read_device_errors", &read_device_errors);
  m.def("reset_device_errors", &reset_device_errors);
  m.def("device_errors_to_host", &device_errors_to_host);
  py::class_<CommContext>(m, "CommContext")
      .def(py::init<int64_t, int64_t, std::vector<int64_t>, int64_t, std::vector<int64_t>, Tensor, int64_t, int64_t>())
      .def("allreduce_f32", &CommContext::allreduce_f32)
      .def("allreduce_bf16", &CommContext::allreduce_bf16)
      .def("reduce_scatter_acc_f32", &CommContext::reduce_scatter_acc_f32)
      .def("reduce_scatter_acc_bf16", &CommContext::reduce_scatter_acc_bf16)
      .def("reduce_scatter_range_acc_f32", &CommContext::reduce_scatter_range_acc_f32)
      .def("push_reduce_scatter_f32", &CommContext::push_reduce_scatter_f32, py::arg("src"), py::arg("src_stride"),
           py::arg("land_off"), py::arg("part"), py::arg("acc"), py::arg("scale"), py::arg("clear_src") = false)
      .def("bucket_reduce", &CommContext::bucket_reduce, py::arg("off"), py::arg("part"), py::arg("acc"),
           py::arg("scale"), py::arg("blocks") = 0)
      .def("adamw_allgather_seg", &CommContext::adamw_allgather_seg, py::arg("segs"), py::arg("total"),
           py::arg("master"), py::arg("m"), py::arg("v"), py::arg("grad"), py::arg("scale"), py::arg("scale_const"),
           py::arg("lr"), py::arg("beta1"), py::arg("beta2"), py::arg("eps"), py::arg("wd"), py::arg("step"),
           py::arg("dev_scalars") = py::none())
      .def("allgather", &CommContext::allgather)
      .def("gather_ce", &CommContext::gather_ce)
      .def("adamw_allgather", &CommContext::adamw_allgather, py::arg("param_off"), py::arg("chunk"),
           py::arg("master"), py::arg("m"), py::arg("v"), py::arg("grad"), py::arg("scale"), py::arg("scale_const"),
           py::arg("lr"), py::arg("beta1"), py::arg("beta2"), py::arg("eps"), py::arg("wd"), py::arg("step"),
           py::arg("dev_scalars") = py::none())
      .def("rs_adamw_allgather", &CommContext::rs_adamw_allgather, py::arg("grads"), py::arg("g_off"),
           py::arg("param_off"), py::arg("chunk"), py::arg("master"), py::arg("m"), py::arg("v"),
           py::arg("grad_scale"), py::arg("lr"), py::arg("beta1"), py::arg("beta2"), py::arg("eps"), py::arg("wd"),
           py::arg("step"), py::arg("dev_scalars") = py::none(), py::arg("sq_out") = py::none())
      .def("barrier", &CommContext::barrier)
      .def("wait_unsignalled", &CommContext::wait_unsignalled)
      .def_property_readonly("multicast", &CommContext::multicast)
      .def_property_readonly("blocks", &CommContext::blocks);
  m.def("pace_cost_ns", &pace_cost_ns, py::arg("link_bytes"), py::arg("gbps"), py::arg("latency_ms"));
  py::class_<LinkPacer, std::shared_ptr<LinkPacer>>(m, "LinkPacer")
      .def(py::init<int64_t, double, double, int64_t>(), py::arg("device_index"), py::arg("gbps"),
           py::arg("latency_ms"), py::arg("timeout_ns"))
      .def("cost_ns", &LinkPacer::cost_ns)
      .def("begin", &LinkPacer::begin)
      .def("end", &LinkPacer::end)
      .def_property_readonly("gbps", &LinkPacer::gbps)
      .def_property_readonly("latency_ms", &LinkPacer::latency_ms)
      .def_property_readonly("state", &LinkPacer::state_tensor);
  py::class_<PullGather>(m, "PullGather")
      .def(py::init<int64_t, int64_t, int64_t>(), py::arg("slots"), py::arg("categories"), py::arg("device_index"))
      .def("prefetch", &PullGather::prefetch)
      .def("gather_now", &PullGather::gather_now)
      .def("acquire", &PullGather::acquire)
      .def("release", &PullGather::release)
      .def("mark_ready", &PullGather::mark_ready)
      .def("join", &PullGather::join)
      .def("take_times", &PullGather::take_times)
      .def("reset_times", &PullGather::reset_times)
      .def("set_pacer", &PullGather::set_pacer, py::arg("pacer").none(true))
      .def_property_readonly("side_stream", &PullGather::side_stream);

}
