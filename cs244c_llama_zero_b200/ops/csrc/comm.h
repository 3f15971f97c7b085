// NVLink / NVSwitch collective kernels over symmetric memory (see comm.cu).
//
// Every rank owns one buffer of a symmetric allocation; `peers[r]` is rank r's buffer as a
// pointer valid on this GPU (NVLink peer mapping), `mc` the NVSwitch multicast address of the
// same allocation (0 when the switch cannot multicast).  Offsets are in bytes from the buffer
// base and identical on every rank.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "common.cuh"

namespace b200 {

constexpr int kCommMaxWorld = 8;
constexpr int kCommMaxBlocks = 64;

struct CommCtx {
  int rank;
  int world;
  uint64_t peers[kCommMaxWorld];  // rank r's buffer base, mapped on this GPU
  uint64_t mc;                     // multicast base (0 = none)
  uint64_t pads[kCommMaxWorld];   // rank r's signal pad base, mapped on this GPU
  uint32_t* epochs;                // [kCommMaxBlocks] per-block barrier epochs (local memory)
  DeviceErrors* errs;
  uint64_t timeout_ns;
  int blocks;                      // grid size used by every collective of this communicator
};

// In place: region[0, n) = scale * sum_ranks(region); fp32.
void comm_allreduce_f32(const CommCtx& c, size_t off_bytes, size_t n, float scale, cudaStream_t s);
// acc[0, chunk) += scale * sum_ranks(region[rank*chunk, (rank+1)*chunk)); fp32 region and acc.
void comm_reduce_scatter_acc_f32(const CommCtx& c, size_t off_bytes, size_t chunk, float* acc, float scale,
                                 cudaStream_t s);
// acc[0, hi - lo) += scale * sum_ranks(region[lo, hi)), fp32 (elements, multiples of 4; lo == hi is
// allowed): one bucket's share of this rank's shard, for reduce-scatter overlapped with backward.
// `blocks` > 0 runs it on that many blocks (fewer SMs taken from concurrent compute); same on all ranks.
void comm_reduce_scatter_range_acc_f32(const CommCtx& c, size_t off_bytes, size_t lo, size_t hi, float* acc,
                                       float scale, int blocks, cudaStream_t s);
// bf16 variants (fp32 accumulation of the sum; the reduce-scatter accumulates into an fp32 shard).
void comm_allreduce_bf16(const CommCtx& c, size_t off_bytes, size_t n, float scale, cudaStream_t s);
void comm_reduce_scatter_acc_bf16(const CommCtx& c, size_t off_bytes, size_t chunk, float* acc, float scale,
                                  cudaStream_t s);
// Every rank's `shard` (chunk_bytes, 16-byte multiple) lands at region[rank*chunk_bytes] on all ranks.
void comm_allgather(const CommCtx& c, size_t off_bytes, size_t chunk_bytes, const void* shard, cudaStream_t s);
// Pull-mode all-gather on the copy engines: dst[r*chunk_bytes, (r+1)*chunk_bytes) = rank r's
// region[0, chunk_bytes) for every r, as one peer-to-device copy per rank on stream s (no kernel, no
// SMs, no barrier).  The caller guarantees every rank's source region is stable while it is read.
void comm_gather_ce(const CommCtx& c, size_t off_bytes, size_t chunk_bytes, void* dst, cudaStream_t s);
// AdamW on this rank's fp32 shard, then the bf16 result is written into every rank's parameter
// region at [rank*chunk] (fused update + all-gather).  `dev_sc` as in adamw_step (kernels.h).
void comm_adamw_allgather(const CommCtx& c, size_t param_off_bytes, size_t chunk, float* master, float* m, float* v,
                          const float* grad, const float* scale_ptr, float scale_const, float lr, float beta1,
                          float beta2, float eps, float wd, int step, cudaStream_t s, const float* dev_sc = nullptr);
// The ZeRO-2 step without clipping as one kernel: g's region [g_off + rank*chunk*4, +chunk*4) summed
// over ranks (fp32) and scaled by grad_scale is this rank's averaged gradient shard; its squared norm
// is added to *sq_out (zeroed first; nullable); AdamW updates master/m/v [chunk]; the bf16 result
// lands in every rank's parameter region of c at [param_off + rank*chunk*2].  Barriers use c.
void comm_rs_adamw_allgather(const CommCtx& c, const CommCtx& g, size_t g_off, size_t param_off, size_t chunk,
                             float* master, float* m, float* v, float grad_scale, float lr, float beta1, float beta2,
                             float eps, float wd, int step, const float* dev_sc, float* sq_out, cudaStream_t s);
// Routed gradient push (ZeRO-2 without a full gradient buffer): element k of src (fp32, n elements,
// 16-byte aligned) has flat index flat0 + k; rank r = flat / chunk owns it and it is added at
// bases[r] + (flat - r * chunk) with system-scope reductions (bases: every rank's fp32 gradient shard
// as mapped on this GPU).  flat0 and chunk must be multiples of 4.
struct RouteTable {
  uint64_t base[kCommMaxWorld];
  int world;
  long long chunk;
};
void comm_routed_add(const float* src, size_t n, long long flat0, const RouteTable& t, DeviceErrors* errs,
                     cudaStream_t s);
// ZeRO-2 gradient ring (interleaved shards): region [off, off + 4*W*part) of every rank's bucket
// buffer holds its fp32 gradient of one bucket; rank r owns slice r = [r*part, (r+1)*part) and gets
// acc[0, part) += scale * sum_ranks(slice r).  When the kernel ends the whole region is zero on every
// rank.  part a multiple of 4; `blocks` as for the range reduce-scatter.
void comm_bucket_reduce(const CommCtx& c, size_t off_bytes, size_t part, float* acc, float scale, int blocks,
                        cudaStream_t s);
// One segment of an interleaved shard (all fields in units of 8 elements except param_off): shard
// groups [shard8, shard8 + part8) are slice `rank` of a bucket whose parameters start at byte
// param_off of the parameter buffer; the first valid8 groups of the slice lie inside the bucket.
struct RingSeg {
  long long shard8;
  long long part8;
  long long valid8;
  long long param_off;
};
// AdamW over the whole interleaved shard (total elements, multiple of 8; master / m / v / grad in
// shard order) and the bf16 results of the valid groups written into every rank's parameter buffer
// at param_off + (rank * part8 + j) * 16.  `segs` is a device array of nseg entries sorted by shard8.
void comm_adamw_allgather_seg(const CommCtx& c, const RingSeg* segs, int nseg, size_t total, float* master, float* m,
                              float* v, const float* grad, const float* scale_ptr, float scale_const, float lr,
                              float beta1, float beta2, float eps, float wd, int step, cudaStream_t s,
                              const float* dev_sc = nullptr);
// Push reduce-scatter: src (local fp32, not necessarily symmetric) holds W slices of `part` elements,
// slice q at src + q * src_stride; this context's buffer holds a landing area of W x part fp32 at
// land_off.  acc[0, part) += scale * (src slice rank + the other ranks' slice `rank`).  With
// clear_src the W slices of src are zero afterwards.
void comm_push_reduce_scatter_f32(const CommCtx& c, float* src, size_t src_stride, size_t land_off, size_t part,
                                  float* acc, float scale, bool clear_src, cudaStream_t s);
// Embedding backward into the owners' shards: row r of dy (bf16 [rows, d], contiguous) is added at
// table row ids[r] of the weight whose element (i, k) has flat index flat0 + i * d + k (ids outside
// [0, vocab) are skipped).  d must be a multiple of 8, flat0 of 4.
void comm_embedding_bwd_routed(const int64_t* ids, const void* dy, int rows, int d, int vocab, long long flat0,
                               const RouteTable& t, DeviceErrors* errs, cudaStream_t s);
// Standalone barrier among the ranks (every block of the communicator's grid).
void comm_barrier(const CommCtx& c, cudaStream_t s);
// A wait that nobody satisfies: used by tests to exercise the bounded-wait error path.
void comm_wait_unsignalled(const CommCtx& c, uint64_t timeout_ns, cudaStream_t s);

// Device-paced link emulation (the `nvlink` bandwidth mode of the experiment harness): every paced
// transfer of one GPU books one emulated link.  `state` is a device array of 1 + kPaceSlots words:
// state[0] is the %globaltimer time at which the link is next free, state[1 + slot] the start stamp
// of the transfer using `slot`.  pace_begin stamps the clock on stream s before the transfer;
// pace_end, after it, books the link for cost_ns starting at max(stamp, link free time) and holds
// the stream until that booking ends, so the transfer takes max(its own time, its share of the
// link).  Transfers on several streams queue on the same link.  The hold is bounded by timeout_ns
// (the error record gets kErrPaceWait when it runs out).
constexpr int kPaceSlots = 1024;
void comm_pace_begin(uint64_t* state, int slot, cudaStream_t s);
void comm_pace_end(uint64_t* state, int slot, uint64_t cost_ns, uint64_t timeout_ns, DeviceErrors* errs,
                   cudaStream_t s);

}  // namespace b200
