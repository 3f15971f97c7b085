"""NVLink / NVSwitch collectives over symmetric memory (``--collective-impl nvls`` / ``p2p``).

Buffers that the ZeRO engines reduce or gather (the flat fp32 gradient buffer, the flat model-dtype
parameter buffer, ZeRO-3 staging buffers) are allocated as symmetric memory: torch's symmetric-memory
rendezvous maps every rank's buffer on every GPU and, when the NVSwitch supports it, binds the
allocation to a multicast object.  The collectives on those buffers are this package's own sm_100a
kernels (``ops/csrc/comm.cu``):

* ``allreduce_scaled_``          NVLS ``multimem.ld_reduce`` + ``multimem.st`` with the 1/W scale fused
* ``reduce_scatter_accumulate_`` ``multimem.ld_reduce`` of this rank's chunk, scaled and accumulated into
                                 the fp32 gradient shard in the same kernel
* ``allgather_into``             ``multimem.st`` of the shard into every rank's buffer
* ``adamw_allgather``            AdamW on the shard fused with the multicast all-gather of the bf16 result
* ``pull_allgather_into``        copy-engine pulls of every rank's shard (no kernel, no barrier): the ZeRO-3
                                 per-module parameter gather, prefetched on a side stream

``impl="p2p"`` runs the same kernels with plain peer loads/stores instead of multicast.  Calls on
tensors that are not part of a registered symmetric buffer (and the reference-compatible
``allreduce`` / ``reduce_scatter`` / ``allgather`` API) fall back to NCCL, like ``TorchCollectives``.

Every device-side wait is bounded (``ZB_COMM_TIMEOUT_S``, default 30 s); an expired wait is recorded in
the device error record, which :meth:`NvlinkCollectives.check_errors` turns into a ``CommTimeoutError``.

With ``ZERO_NVLINK_BW_GBPS`` / ``ZERO_NVLINK_LATENCY_MS`` set, every transfer above is paced on the
device to an emulated link of that bandwidth (:mod:`.pacing`; the harness's ``nvlink`` bandwidth mode).
"""

from __future__ import annotations

import os
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from ...ops import CommTimeoutError  # re-exported: raised for expired collective waits
from ..collectives import TorchCollectives, _maybe_simulate_collective_delay, _world
from .pacing import link_bytes, make_pacer


def _timeout_ns() -> int:
    return int(float(os.environ.get("ZB_COMM_TIMEOUT_S", "30")) * 1e9)


def _pace_timeout_ns() -> int:
    """Bound on one paced hold (it also waits out the transfers queued before it on the link)."""
    return int(float(os.environ.get("ZB_PACE_TIMEOUT_S", "120")) * 1e9)


class SymmetricBuffer:
    """One symmetric allocation + the kernel context that addresses it on every rank."""

    def __init__(self, numel: int, dtype: torch.dtype, device: torch.device, use_multicast: bool,
                 group=None, blocks: int = 48) -> None:
        import torch.distributed._symmetric_memory as symm_mem

        from ... import ops

        group = group or dist.group.WORLD
        self.tensor = symm_mem.empty(numel, dtype=dtype, device=device)
        self.tensor.zero_()
        self.handle = symm_mem.rendezvous(self.tensor, group)
        self.rank = self.handle.rank
        self.world = self.handle.world_size
        mc = int(self.handle.multicast_ptr) if use_multicast else 0
        pad_bytes = int(self.handle.signal_pad_size)
        # barrier slots: 8 uint32 per block; the last block's slots are reserved for tests
        blocks = max(1, min(blocks, pad_bytes // (4 * 8) - 1, 63))
        self.epochs = torch.zeros(64, dtype=torch.int32, device=device)
        self.ctx = ops.load_extension().CommContext(
            self.rank, self.world, [int(p) for p in self.handle.buffer_ptrs], mc,
            [int(p) for p in self.handle.signal_pad_ptrs], self.epochs, blocks, _timeout_ns())
        self.multicast = mc != 0
        self.base = self.tensor.data_ptr()
        self.nbytes = self.tensor.numel() * self.tensor.element_size()

    def offset_of(self, t: torch.Tensor) -> Optional[int]:
        ptr = t.data_ptr()
        if self.base <= ptr and ptr + t.numel() * t.element_size() <= self.base + self.nbytes:
            return ptr - self.base
        return None


class NvlinkCollectives(TorchCollectives):
    """ZeRO collectives as NVLink/NVSwitch kernels on symmetric buffers; NCCL for everything else."""

    supports_fused = True

    def __init__(self, device: Optional[torch.device] = None, use_multicast: bool = True) -> None:
        self.name = "nvls" if use_multicast else "p2p"
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.use_multicast = use_multicast
        self.buffers: List[SymmetricBuffer] = []
        self.pacer = make_pacer(self.device, _pace_timeout_ns())  # None unless the nvlink bandwidth mode is on
        self._skip = 0  # fault injection: barrier-synchronised collectives left out on purpose
        self._landing: Optional[SymmetricBuffer] = None  # push reduce-scatter landing area (lazy)
        self._old_landings: List[SymmetricBuffer] = []  # outgrown areas stay mapped (kernels may be in flight)

    def skip_next_collective(self, count: int = 1) -> None:
        """Fault injection: leave out (do not launch) the next ``count`` barrier-synchronised collective
        kernels of this rank, so the peers' bounded barrier waits expire (``ZB_FAULT=skip_signal``)."""
        self._skip += int(count)

    def _skipped(self, op: str) -> bool:
        if self._skip <= 0:
            return False
        self._skip -= 1
        import sys

        print(f"[fault] {op}: kernel left out, no barrier signal posted", file=sys.stderr, flush=True)
        return True

    def _pace_begin(self) -> int:
        return self.pacer.begin() if self.pacer is not None else -1

    def _pace_end(self, slot: int, op: str, full_bytes: int) -> None:
        if self.pacer is not None:
            self.pacer.end(slot, link_bytes(op, full_bytes, self._w()))

    # -- push reduce-scatter -----------------------------------------------------------------
    # Largest landing area (W rows of one piece); bigger reduce-scatters run piece by piece.
    LANDING_MAX_BYTES = 256 << 20

    def rs_push(self) -> bool:
        """Whether fp32 reduce-scatters run as peer stores into a landing area plus a local sum
        (``ZB_RS_MODE=push``) or as multicast reductions / peer loads (``switch``, the default).
        ``auto``: push at 2 and 4 ranks and whenever multicast is off.  Measured at 2 B200 (fp32,
        1 GiB): multicast 323 GB/s bus, push 220 GB/s, peer loads 127 GB/s; `small` stage 2 / 3 steps
        8.87 / 10.09 ms with multicast vs 9.25 / 10.31 ms with push.  So multicast stays the default;
        push is kept for switches without multicast."""
        mode = os.environ.get("ZB_RS_MODE", "switch")
        if mode in ("push", "switch"):
            return mode == "push"
        return (not self.use_multicast) or self._w() <= 4

    def _landing_area(self, numel: int) -> SymmetricBuffer:
        """A symmetric fp32 landing area of at least ``numel`` elements (a collective when it grows:
        every rank asks for the same sizes in the same order)."""
        if self._landing is None or self._landing.tensor.numel() < numel:
            if self._landing is not None:
                self._old_landings.append(self._landing)
            self._landing = SymmetricBuffer(int(numel), torch.float32, self.device, self.use_multicast)
        return self._landing

    def _push_rs(self, src: torch.Tensor, part: int, acc: torch.Tensor, scale: float, clear: bool) -> None:
        """acc[:part] += scale * (src slice rank + peers' slice rank) where src holds W slices of ``part``
        fp32 elements back to back; pieces of at most LANDING_MAX_BYTES of landing area per kernel."""
        world = self._w()
        piece = max(4, (self.LANDING_MAX_BYTES // (4 * world)) // 4 * 4)
        piece = min(piece, part)
        land = self._landing_area(world * piece)
        for a in range(0, part, piece):
            n = min(piece, part - a)
            land.ctx.push_reduce_scatter_f32(src[a:], part, 0, n, acc[a:], float(scale), bool(clear))

    # -- allocation --------------------------------------------------------------------------
    def alloc(self, numel: int, dtype: torch.dtype) -> torch.Tensor:
        """A zero-filled symmetric buffer (collective call: every rank must allocate the same sizes)."""
        buf = SymmetricBuffer(int(numel), dtype, self.device, self.use_multicast)
        self.buffers.append(buf)
        return buf.tensor

    def _locate(self, t: torch.Tensor) -> Optional[Tuple[SymmetricBuffer, int]]:
        if not t.is_cuda or not t.is_contiguous():
            return None
        for buf in self.buffers:
            off = buf.offset_of(t)
            if off is not None and buf.tensor.dtype == t.dtype:
                return buf, off
        return None

    def locate_symmetric(self, t: torch.Tensor) -> Optional[Tuple[object, int]]:
        """(kernel context, byte offset) of a tensor inside one of this object's symmetric buffers."""
        hit = self._locate(t)
        return None if hit is None else (hit[0].ctx, hit[1])

    def check_errors(self) -> None:
        """Raise ``CommTimeoutError`` (or ``DeviceWaitError``) if any kernel's bounded wait expired."""
        from ... import ops

        ops.raise_for_device_errors(ops.load_extension().read_device_errors())

    # -- fused entry points ------------------------------------------------------------------------
    def allreduce_scaled_(self, flat: torch.Tensor, scale: float) -> torch.Tensor:
        hit = self._locate(flat)
        if hit is None or flat.dtype not in (torch.float32, torch.bfloat16) or flat.numel() % 8:
            return super().allreduce_scaled_(flat, scale)
        buf, off = hit
        if self._skipped("allreduce"):
            return flat
        slot = self._pace_begin()
        if flat.dtype == torch.float32:
            buf.ctx.allreduce_f32(off, flat.numel(), scale)
        else:
            buf.ctx.allreduce_bf16(off, flat.numel(), scale)
        self._pace_end(slot, "allreduce", flat.numel() * flat.element_size())
        _maybe_simulate_collective_delay(flat.numel() * flat.element_size(), self._w())
        return flat

    def reduce_scatter_accumulate_(self, acc: torch.Tensor, flat: torch.Tensor, scale: float) -> torch.Tensor:
        hit = self._locate(flat)
        world = self._w()
        push = (flat.dtype == torch.float32 and flat.is_cuda and flat.is_contiguous() and self.rs_push()
                and world > 1)
        if ((hit is None and not push) or flat.dtype not in (torch.float32, torch.bfloat16)
                or flat.numel() % (8 * world) or acc.dtype != torch.float32):
            return super().reduce_scatter_accumulate_(acc, flat, scale)
        if self._skipped("reduce_scatter"):
            return acc
        slot = self._pace_begin()
        if push:  # the source need not be symmetric: peers never read it
            self._push_rs(flat, flat.numel() // world, acc, scale, False)
            self._pace_end(slot, "reduce_scatter", flat.numel() * flat.element_size())
            _maybe_simulate_collective_delay(acc.numel() * flat.element_size(), world)
            return acc
        buf, off = hit
        if flat.dtype == torch.float32:
            buf.ctx.reduce_scatter_acc_f32(off, flat.numel() // world, acc, scale)
        else:
            buf.ctx.reduce_scatter_acc_bf16(off, flat.numel() // world, acc, scale)
        self._pace_end(slot, "reduce_scatter", flat.numel() * flat.element_size())
        _maybe_simulate_collective_delay(acc.numel() * flat.element_size(), world)
        return acc

    supports_range_reduce_scatter = True

    def reduce_scatter_range_accumulate_(self, shard_acc: torch.Tensor, flat: torch.Tensor, lo: int, hi: int,
                                         shard_lo: int, scale: float, blocks: int = 0) -> bool:
        """shard_acc += scale * sum_ranks(flat[lo:hi]) restricted to this rank's shard.

        ``flat`` is the whole symmetric fp32 buffer, ``shard_acc`` this rank's shard of it
        (``flat[shard_lo : shard_lo + shard_acc.numel()]`` in the flat layout).  Every rank must call
        this for the same buckets in the same order (each call is a collective).  Returns False, doing
        nothing, when ``flat`` is not a symmetric fp32 buffer of this object or the bounds are not
        4-element aligned.  ``blocks`` > 0 limits the kernel to that many thread blocks (every rank must
        pass the same value), leaving the other SMs to compute that runs concurrently.
        """
        hit = self._locate(flat)
        if hit is None or flat.dtype != torch.float32 or lo % 4 or hi % 4 or shard_lo % 4:
            return False
        buf, off = hit
        shard_hi = shard_lo + shard_acc.numel()
        a, b = max(lo, shard_lo), min(hi, shard_hi)
        if b <= a:
            a = b = lo  # empty share: still join the collective's barriers
            acc = shard_acc
        else:
            acc = shard_acc[a - shard_lo:]
        if self._skipped("reduce_scatter_range"):
            return True
        slot = self._pace_begin()
        buf.ctx.reduce_scatter_range_acc_f32(off + lo * 4, a - lo, b - lo, acc, scale, int(blocks))
        self._pace_end(slot, "reduce_scatter", (hi - lo) * 4)
        return True

    supports_bucket_reduce = True

    def bucket_reduce_(self, bucket: torch.Tensor, acc: torch.Tensor, scale: float, blocks: int = 0) -> bool:
        """Gradient ring: ``acc += scale * sum_ranks(slice rank of bucket)`` and ``bucket`` cleared.

        ``bucket`` (fp32, inside one of this object's symmetric buffers, ``W * part`` elements) holds
        this rank's gradient of one bucket; rank r owns slice ``[r*part, (r+1)*part)`` and ``acc``
        (``part`` elements, local fp32) is its gradient segment.  When the kernel ends the bucket is
        zero on every rank.  A collective: every rank calls it for the same buckets in the same order.
        Returns False, doing nothing, when the bucket does not qualify."""
        hit = self._locate(bucket)
        world = self._w()
        n = bucket.numel()
        if hit is None or bucket.dtype != torch.float32 or n % (4 * world) or acc.numel() != n // world:
            return False
        buf, off = hit
        if self._skipped("bucket_reduce"):
            return True
        slot = self._pace_begin()
        if self.rs_push():
            self._push_rs(bucket, n // world, acc, scale, True)
        else:
            buf.ctx.bucket_reduce(off, n // world, acc, float(scale), int(blocks))
        self._pace_end(slot, "reduce_scatter", n * 4)
        return True

    def adamw_allgather_segments(self, params_flat: torch.Tensor, segs: torch.Tensor, master: torch.Tensor,
                                 exp_avg: torch.Tensor, exp_avg_sq: torch.Tensor, grad: torch.Tensor, scale, cfg,
                                 step: int, dev_scalars: Optional[torch.Tensor] = None) -> bool:
        """AdamW on an interleaved ring shard + the bf16 all-gather of every segment into
        ``params_flat`` (the symmetric parameter buffer; ``segs`` as for the native kernel, with byte
        offsets relative to ``params_flat``).  False, doing nothing, when the buffers do not qualify."""
        hit = self._locate(params_flat)
        total = master.numel()
        if hit is None or params_flat.dtype != torch.bfloat16 or total % 8 or grad.dtype != torch.float32:
            return False
        buf, off = hit
        if off:
            segs = segs.clone()
            segs[:, 3] += off
        scale_t = scale.reshape(1).float() if isinstance(scale, torch.Tensor) else None
        scale_c = 1.0 if isinstance(scale, torch.Tensor) else float(scale if scale is not None else 1.0)
        if self._skipped("adamw_allgather"):
            return True
        slot = self._pace_begin()
        buf.ctx.adamw_allgather_seg(segs, total, master, exp_avg, exp_avg_sq, grad.contiguous(), scale_t, scale_c,
                                    cfg.lr, cfg.betas[0], cfg.betas[1], cfg.eps, cfg.weight_decay, step, dev_scalars)
        self._pace_end(slot, "allgather", total * 2 * self._w())
        return True

    def reduce_scatter_into(self, out: torch.Tensor, flat: torch.Tensor) -> torch.Tensor:
        if out.dtype == torch.float32 and self._locate(flat) is not None:
            out.zero_()
            return self.reduce_scatter_accumulate_(out, flat, 1.0)
        return super().reduce_scatter_into(out, flat)

    def allgather_into(self, out: torch.Tensor, shard: torch.Tensor) -> torch.Tensor:
        hit = self._locate(out)
        world = self._w()
        chunk_bytes = shard.numel() * shard.element_size()
        if (hit is None or out.numel() != shard.numel() * world or chunk_bytes % 16 or not shard.is_contiguous()
                or shard.dtype != out.dtype):
            return super().allgather_into(out, shard)
        buf, off = hit
        if self._skipped("allgather"):
            return out
        slot = self._pace_begin()
        buf.ctx.allgather(off, chunk_bytes, shard)
        self._pace_end(slot, "allgather", chunk_bytes * world)
        _maybe_simulate_collective_delay(chunk_bytes, world)
        return out

    supports_pull_gather = True

    def pull_allgather_into(self, out: torch.Tensor, shard: torch.Tensor) -> bool:
        """out[r*n : (r+1)*n] = rank r's ``shard`` (n elements) for every r, read by the copy engines.

        ``shard`` must lie in a symmetric buffer of this object (same offset on every rank).  No kernel
        and no barrier: one peer-to-device copy per rank on the current stream, so the caller must
        guarantee that no rank rewrites its shard while another may be reading it.  Returns False,
        doing nothing, when the tensors do not qualify.
        """
        hit = self._locate(shard)
        world = self._w()
        nbytes = shard.numel() * shard.element_size()
        if (hit is None or out.dtype != shard.dtype or out.numel() < shard.numel() * world or nbytes % 16
                or not out.is_contiguous() or not out.is_cuda):
            return False
        buf, off = hit
        slot = self._pace_begin()
        buf.ctx.gather_ce(off, nbytes, out)
        self._pace_end(slot, "allgather", nbytes * world)
        _maybe_simulate_collective_delay(nbytes, world)
        return True

    def adamw_allgather(self, params_flat: torch.Tensor, master: torch.Tensor, exp_avg: torch.Tensor,
                        exp_avg_sq: torch.Tensor, grad: torch.Tensor, scale, cfg, step: int,
                        dev_scalars: Optional[torch.Tensor] = None) -> bool:
        """AdamW on the shard + multicast all-gather of the bf16 result; False if not applicable."""
        hit = self._locate(params_flat)
        world = self._w()
        chunk = master.numel()
        if (hit is None or params_flat.dtype != torch.bfloat16 or params_flat.numel() != chunk * world
                or chunk % 8 or grad.dtype != torch.float32):
            return False
        buf, off = hit
        scale_t = scale.reshape(1).float() if isinstance(scale, torch.Tensor) else None
        scale_c = 1.0 if isinstance(scale, torch.Tensor) else float(scale if scale is not None else 1.0)
        if self._skipped("adamw_allgather"):
            return True
        slot = self._pace_begin()
        buf.ctx.adamw_allgather(off, chunk, master, exp_avg, exp_avg_sq, grad.contiguous(), scale_t, scale_c, cfg.lr,
                                cfg.betas[0], cfg.betas[1], cfg.eps, cfg.weight_decay, step, dev_scalars)
        self._pace_end(slot, "allgather", chunk * 2 * world)
        return True

    def allreduce_sum_small_(self, t: torch.Tensor) -> bool:
        """``t`` (at most 8 fp32 values on this GPU) = its sum over ranks, with this package's all-reduce
        kernel on a small symmetric buffer instead of an NCCL call (the gradient-norm scalar).  The
        buffer is allocated at the first call, which is therefore a collective: every rank must make
        the same calls in the same order, as with every collective.  False if ``t`` does not qualify."""
        if t.dtype != torch.float32 or t.numel() > 8 or not t.is_cuda or self._w() == 1:
            return False
        if getattr(self, "_scalars", None) is None:
            self._scalars = self.alloc(8, torch.float32)
        buf = self._scalars
        buf.zero_()
        buf[: t.numel()].copy_(t.reshape(-1))
        if self._skipped("allreduce_small"):
            return True
        self._locate(buf)[0].ctx.allreduce_f32(0, 8, 1.0)
        t.reshape(-1).copy_(buf[: t.numel()])
        return True

    supports_routed_grads = True

    def shard_bases(self, t: torch.Tensor) -> Optional[List[int]]:
        """Every rank's address of symmetric tensor ``t`` (same offset in each rank's buffer), as mapped
        on this GPU, or None when ``t`` is not in one of this object's symmetric buffers."""
        hit = self._locate(t)
        if hit is None:
            return None
        buf, off = hit
        return [int(ptr) + off for ptr in buf.handle.buffer_ptrs]

    def routed_push(self, src: torch.Tensor, flat0: int, chunk: int, bases: List[int]) -> None:
        """Add fp32 ``src`` (flat indices ``flat0 ..``) into the owning ranks' shards (``bases``) over
        NVLink; the owners see the sums after the next barrier."""
        from ... import ops

        if self._skipped("routed_push"):
            return
        ops.load_extension().routed_add(src, int(flat0), int(chunk), bases)

    supports_fused_step = True

    def reduce_scatter_adamw_allgather(self, params_flat: torch.Tensor, grads_flat: torch.Tensor, master: torch.Tensor,
                                       exp_avg: torch.Tensor, exp_avg_sq: torch.Tensor, grad_scale: float, cfg,
                                       step: int, dev_scalars: Optional[torch.Tensor] = None,
                                       sq_out: Optional[torch.Tensor] = None) -> bool:
        """The whole unclipped ZeRO-2 update in one kernel: reduce-scatter of ``grads_flat`` (fp32,
        symmetric) times ``grad_scale``, its squared norm added to ``sq_out``, AdamW on this rank's
        shard state and the bf16 all-gather into ``params_flat`` (symmetric).  No fp32 gradient shard
        is written.  Returns False, doing nothing, when the buffers do not qualify."""
        hp, hg = self._locate(params_flat), self._locate(grads_flat)
        world = self._w()
        chunk = master.numel()
        if (hp is None or hg is None or params_flat.dtype != torch.bfloat16 or grads_flat.dtype != torch.float32
                or params_flat.numel() != chunk * world or grads_flat.numel() != chunk * world or chunk % 8
                or hp[0].multicast != hg[0].multicast):
            return False
        if self._skipped("rs_adamw_allgather"):
            return True
        (pbuf, poff), (gbuf, goff) = hp, hg
        slot = self._pace_begin()
        pbuf.ctx.rs_adamw_allgather(gbuf.ctx, goff, poff, chunk, master, exp_avg, exp_avg_sq, float(grad_scale), cfg.lr,
                                    cfg.betas[0], cfg.betas[1], cfg.eps, cfg.weight_decay, step, dev_scalars, sq_out)
        # reduce-scatter of the fp32 gradients, then all-gather of the bf16 shards
        self._pace_end(slot, "reduce_scatter", grads_flat.numel() * 4)
        slot = self._pace_begin()
        self._pace_end(slot, "allgather", params_flat.numel() * 2)
        return True

    def barrier(self) -> None:
        if self.buffers:
            if not self._skipped("barrier"):
                self.buffers[0].ctx.barrier()
        else:
            dist.barrier()

    @staticmethod
    def _w() -> int:
        return _world()
