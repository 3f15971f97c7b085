"""ZeRO stages 0, 1 and 2 over one flat parameter space.

Behaviour per stage matches the reference:

* stage 0 (``zero/stage0_ddp.py:27-169``): fp32 master + Adam moments for every
  parameter; gradient all-reduce, average, optional global-norm clipping, AdamW on the
  full vector, write back the model-dtype parameters.
* stage 1 (``zero/stage1_optimizer.py:29-189``): optimizer state only for this rank's
  shard; full all-reduce, clip on the full vector, AdamW on the shard, all-gather of the
  updated model-dtype shards.
* stage 2 (``zero/stage2_optimizer.py:29-311``): gradients are reduce-scattered after every
  ``backward`` (once per micro-batch) and accumulated, averaged, into an fp32 shard; the
  global norm is the all-reduced sum of squares of the shards; AdamW on the shard; all-gather.

B200-first differences: parameters are views of one flat buffer and weight gradients
accumulate in one flat fp32 buffer (``main_grad``) so no ``torch.cat`` flattening or
per-parameter hooks are needed; the collectives work in place on those buffers, and an
implementation with device kernels (``--collective-impl nvls``) fuses the averaging and
accumulation into the reduction; the AdamW update is one fused kernel that also writes the
model-dtype copy; clipping never synchronises with the host.
"""

from __future__ import annotations

import os
import time
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn as nn

from .base import ZeROEngineBase
from .common import (
    FlatParamSpace,
    build_flat_param_metadata,
    bytes_to_mb,
    tensor_num_bytes,
    tensors_num_bytes,
)
from .optim import adamw_update_, clip_coefficient, global_norm_from_local_sq, sum_of_squares


class _ShardRoute:
    """Where a weight gradient goes in routed stage 2: the fp32 shard of the rank owning each element
    (flat index // chunk), addressed through the collectives' NVLink mappings."""

    def __init__(self, collectives, chunk: int, bases: List[int]) -> None:
        self.collectives = collectives
        self.chunk = int(chunk)
        self.bases = list(bases)

    def push(self, src: torch.Tensor, flat0: int) -> None:
        src = src.contiguous()
        if src.data_ptr() % 16:
            src = src.clone()
        self.collectives.routed_push(src, flat0, self.chunk, self.bases)


class _FlatEngine(ZeROEngineBase):
    """Common structure for the stages whose parameters are replicated between steps."""

    shard_optimizer = False

    def __init__(self, model: nn.Module, **kwargs) -> None:
        super().__init__(model, **kwargs)
        self.meta = build_flat_param_metadata(model)
        allocator = getattr(self.collectives, "alloc", None) if self.world_size > 1 and self.device.type == "cuda" else None
        self.space = FlatParamSpace(self.meta, self.world_size, self.rank, with_grads=self._full_grad_buffer(),
                                    allocator=allocator)
        if self.shard_optimizer:
            master_src = self.space.shard(self.space.params)
        else:
            master_src = self.space.params
        self._master = master_src.float().clone()
        self._exp_avg = torch.zeros_like(self._master)
        self._exp_avg_sq = torch.zeros_like(self._master)

    def _full_grad_buffer(self) -> bool:
        """Whether this engine keeps a full-size flat fp32 gradient buffer (``param.main_grad``)."""
        return True

    # Names kept from the reference engines.
    @property
    def master_params(self) -> torch.Tensor:
        return self._master

    @property
    def local_master_param_shard(self) -> torch.Tensor:
        return self._master

    @property
    def exp_avg(self) -> torch.Tensor:
        return self._exp_avg

    @property
    def exp_avg_sq(self) -> torch.Tensor:
        return self._exp_avg_sq

    def zero_grad(self) -> None:
        self.clock.reset()
        self.space.grads.zero_()
        for p in self.meta.params:
            p.grad = None

    # -- device-side step counter (replayable CUDA graphs of the whole step) ----------------------
    def use_device_step(self, on: bool = True) -> None:
        """Keep the optimizer's step number on the device: each update first advances a device
        counter (one tiny kernel) and the AdamW kernels take their bias corrections from it, so a
        captured step replays correctly.  The host ``step_count`` is still kept by the caller."""
        if not on or self.device.type != "cuda":
            self._dev_step = None
            return
        self._dev_step = (torch.full((1,), int(self.step_count), dtype=torch.int32, device=self.device),
                          torch.zeros(2, dtype=torch.float32, device=self.device))

    def _device_scalars(self) -> Optional[torch.Tensor]:
        dev = getattr(self, "_dev_step", None)
        if dev is None:
            return None
        from ...ops import functional as B

        B.adam_advance(dev[0], dev[1], self.adam.lr, self.adam.betas[0], self.adam.betas[1])
        return dev[1]

    def _adamw(self, grads: torch.Tensor, scale: torch.Tensor, dev_scalars: Optional[torch.Tensor] = None) -> None:
        if dev_scalars is None:
            dev_scalars = self._device_scalars()
        with self.clock.measure("optimizer"):
            adamw_update_(self._master, self._exp_avg, self._exp_avg_sq, grads, self.adam, self.step_count,
                          grad_scale=scale, param_out=self._param_out(), dev_scalars=dev_scalars)

    def _adamw_and_gather(self, grads: torch.Tensor, scale: torch.Tensor) -> None:
        """Sharded update followed by the parameter all-gather; one fused kernel when available."""
        dev_scalars = self._device_scalars()
        fused = getattr(self.collectives, "adamw_allgather", None) if self.world_size > 1 else None
        if fused is not None and self.device.type == "cuda":
            with self.clock.measure("post_allgather", tensor_num_bytes(self.space.shard(self.space.params))):
                done = fused(self.space.params, self._master, self._exp_avg, self._exp_avg_sq, grads, scale, self.adam,
                             self.step_count, dev_scalars)
            if done:
                return
        self._adamw(grads, scale, dev_scalars)
        self._allgather_params()

    # -- the unclipped step as one kernel (stages 1 and 2) -------------------------------------------
    def _setup_fused_step(self) -> None:
        """``ZB_FUSED_STEP=1``: with the NVLink collectives and no clipping, the step is ONE kernel
        (reduce-scatter of the flat fp32 gradients -> averaged shard -> squared norm -> AdamW ->
        bf16 all-gather, ``rs_adamw_allgather``): no fp32 gradient shard is written and read back,
        and the separate norm kernel and one launch + barrier pair go away.  Stage 2's
        reduce-scatter then happens once per step instead of after every backward (the sum is the
        same); stage 1's full all-reduce becomes that reduce-scatter (without clipping only this
        rank's shard of the averaged gradient is needed; the norm over the shards equals the norm of
        the full vector).  Steps with clipping take the unfused path."""
        coll = self.collectives
        self._fused_step = bool(
            os.environ.get("ZB_FUSED_STEP", "0") == "1" and self.space.grads is not None
            and self.world_size > 1 and self.device.type == "cuda"
            and not getattr(self, "_overlap", False) and getattr(coll, "supports_fused_step", False)
            and coll.locate_symmetric(self.space.params) is not None
            and coll.locate_symmetric(self.space.grads) is not None
            and self.space.params.numel() == self.space.chunk * self.world_size)
        self._fused_sq = torch.zeros(1, dtype=torch.float32, device=self.device) if self._fused_step else None

    def _fused_update(self, labels: Tuple[str, ...]) -> Optional[torch.Tensor]:
        """The unclipped step in one kernel; None (nothing done) if the collectives decline.
        ``labels[0]`` is recorded before the kernel, the rest after it (memory trace)."""
        self.space.fold_autograd_grads()
        step = self.step_count + 1
        dev_scalars = self._device_scalars()
        nbytes = tensor_num_bytes(self.space.grads)
        self._record_memory_event(labels[0])
        category = "backward_reduce_scatter" if self.stage == 2 else "allreduce"
        with self.clock.measure(category, nbytes):
            with self.collectives.label_scope(f"stage{self.stage}.step.reduce_scatter_adamw_allgather"):
                ok = self.collectives.reduce_scatter_adamw_allgather(
                    self.space.params, self.space.grads, self._master, self._exp_avg, self._exp_avg_sq,
                    1.0 / self.world_size, self.adam, step, dev_scalars, self._fused_sq)
        if not ok:
            if dev_scalars is not None:  # give back the device step taken for the declined kernel
                self._dev_step[0].sub_(1)
            return None
        self.step_count = step
        self.clock.count("post_allgather", tensor_num_bytes(self.space.shard(self.space.params)))
        for label in labels[1:]:
            self._record_memory_event(label)
        return global_norm_from_local_sq(self._fused_sq, sharded=True, collectives=self.collectives)

    def _param_out(self) -> torch.Tensor:
        return self.space.shard(self.space.params) if self.shard_optimizer else self.space.params

    def _allgather_params(self) -> None:
        if self.world_size == 1:
            return
        with self.clock.measure("post_allgather", tensor_num_bytes(self.space.shard(self.space.params))):
            self.collectives.allgather_into(self.space.params, self.space.shard(self.space.params))

    # -- gradient wire format ------------------------------------------------------------
    def _wire_bf16(self) -> Optional[torch.Tensor]:
        """``ZB_GRAD_COMM=bf16``: the gradient all-reduce / reduce-scatter moves bf16 (the reference's
        gradient dtype, half the link bytes of the fp32 ``main_grad`` buffer): the fp32 gradients are
        cast into a bf16 staging buffer (symmetric when the collectives allocate, so the NVLink
        kernels reduce it with fp32 accumulation in the switch) and reduced there.  Returns that
        buffer, or None for the default fp32 wire format."""
        if os.environ.get("ZB_GRAD_COMM", "fp32") != "bf16" or self.world_size == 1 or self.space.grads is None:
            return None
        stage = getattr(self, "_bf16_wire", None)
        if stage is None:
            alloc = getattr(self.collectives, "alloc", None) if self.device.type == "cuda" else None
            n = self.space.grads.numel()
            stage = alloc(n, torch.bfloat16) if alloc is not None else torch.zeros(n, dtype=torch.bfloat16,
                                                                                   device=self.device)
            self._bf16_wire = stage
        return stage

    def _allreduce_grads(self, grads: torch.Tensor, scale: float) -> None:
        """``grads = scale * sum_ranks(grads)`` in the configured wire format."""
        wire = self._wire_bf16()
        if wire is None:
            self.collectives.allreduce_scaled_(grads, scale)
            return
        wire.copy_(grads)
        self.collectives.allreduce_scaled_(wire, scale)
        grads.copy_(wire)

    def _reduce_scatter_grads(self, acc: torch.Tensor, grads: torch.Tensor, scale: float) -> None:
        """``acc += scale * chunk_rank(sum_ranks(grads))`` in the configured wire format."""
        wire = self._wire_bf16()
        if wire is None:
            self.collectives.reduce_scatter_accumulate_(acc, grads, scale)
            return
        wire.copy_(grads)
        self.collectives.reduce_scatter_accumulate_(acc, wire, scale)

    # -- state dict ---------------------------------------------------------------------
    def _hparams(self) -> Dict[str, object]:
        return {"lr": self.lr, "betas": self.betas, "eps": self.eps, "weight_decay": self.weight_decay}

    def memory_state_breakdown_mb(self) -> Dict[str, float]:
        params_mb = bytes_to_mb(sum(p.numel() for p in self.meta.params) * self.space.params.element_size())
        grads_mb = bytes_to_mb(self._logical_grad_bytes())
        optimizer_mb = bytes_to_mb(tensors_num_bytes([self._master, self._exp_avg, self._exp_avg_sq]))
        return {"params_mb": params_mb, "grads_mb": grads_mb, "optimizer_mb": optimizer_mb,
                "total_mb": params_mb + grads_mb + optimizer_mb}

    def _logical_grad_bytes(self) -> int:
        return self.meta.total_numel * self.space.params.element_size()


class ZeROStage0DDP(_FlatEngine):
    """Full replication + gradient all-reduce + local AdamW."""

    stage = 0

    def _update(self, max_grad_norm: float) -> torch.Tensor:
        self.space.fold_autograd_grads()
        grads = self.space.grads
        inv_w = 1.0 / self.world_size
        if self.world_size > 1:
            self._record_memory_event("measured_step_stage0_pre_allreduce")
            with self.clock.measure("allreduce", tensor_num_bytes(grads)):
                self._allreduce_grads(grads, inv_w)
            self._record_memory_event("measured_step_stage0_post_allreduce")
        norm = sum_of_squares(grads).sqrt()
        self.step_count += 1
        self._adamw(grads, clip_coefficient(norm, max_grad_norm))
        self._record_memory_event("measured_step_stage0_post_optimizer")
        return norm

    def step_async(self, max_grad_norm: float = 0.0) -> torch.Tensor:
        return self._update(max_grad_norm)

    def step_with_stats(self, max_grad_norm: float = 0.0) -> Dict[str, float]:
        t0 = time.perf_counter()
        norm = self._update(max_grad_norm)
        return self._stats(norm, t0, {"allreduce": "allreduce"})

    def state_dict(self) -> Dict[str, object]:
        return {
            "rank": self.rank,
            "world_size": self.world_size,
            "step_count": self.step_count,
            "master_params": self.space.padded_to_logical(self._master).cpu(),
            "exp_avg": self.space.padded_to_logical(self._exp_avg).cpu(),
            "exp_avg_sq": self.space.padded_to_logical(self._exp_avg_sq).cpu(),
            "hparams": self._hparams(),
        }

    def load_state_dict(self, state: Dict[str, object]) -> None:
        self.step_count = int(state["step_count"])
        dev = self.device
        self._master.copy_(self.space.logical_to_padded(state["master_params"].to(dev, torch.float32)))
        self._exp_avg.copy_(self.space.logical_to_padded(state["exp_avg"].to(dev, torch.float32)))
        self._exp_avg_sq.copy_(self.space.logical_to_padded(state["exp_avg_sq"].to(dev, torch.float32)))
        self.space.params.copy_(self._master)


class _ShardedStateMixin:
    """state_dict/load_state_dict for the shard-holding stages (1 and 2)."""

    def state_dict(self) -> Dict[str, object]:
        state = {
            "step_count": self.step_count,
            "rank": self.rank,
            "world_size": self.world_size,
            "shard_start": self.space.shard_start,
            "shard_end": self.space.shard_start + self.space.chunk,
            "layout": "padded_flat_v1",
            "local_master_param_shard": self._master.detach().cpu(),
            "exp_avg": self._exp_avg.detach().cpu(),
            "exp_avg_sq": self._exp_avg_sq.detach().cpu(),
            "hparams": self._hparams(),
        }
        extra = getattr(self, "_extra_state", None)
        if callable(extra):
            state.update(extra())
        return state

    def load_state_dict(self, state: Dict[str, object]) -> None:
        self.step_count = int(state["step_count"])
        self._master.copy_(state["local_master_param_shard"].to(self.device, torch.float32))
        self._exp_avg.copy_(state["exp_avg"].to(self.device, torch.float32))
        self._exp_avg_sq.copy_(state["exp_avg_sq"].to(self.device, torch.float32))
        self._param_out().copy_(self._master)
        self._allgather_params()


class ZeROStage1Optimizer(_ShardedStateMixin, _FlatEngine):
    """Sharded optimizer state; full gradient all-reduce; all-gather of updated shards."""

    stage = 1
    shard_optimizer = True

    def __init__(self, model: nn.Module, **kwargs) -> None:
        super().__init__(model, **kwargs)
        self._setup_fused_step()

    def _update(self, max_grad_norm: float) -> torch.Tensor:
        if self._fused_step and max_grad_norm <= 0:
            norm = self._fused_update(tuple(f"measured_step_stage1_{x}" for x in (
                "pre_allreduce", "post_allreduce", "pre_allgather", "post_allgather")))
            if norm is not None:
                return norm
        self.space.fold_autograd_grads()
        grads = self.space.grads
        if self.world_size > 1:
            self._record_memory_event("measured_step_stage1_pre_allreduce")
            with self.clock.measure("allreduce", tensor_num_bytes(grads)):
                self._allreduce_grads(grads, 1.0 / self.world_size)
            self._record_memory_event("measured_step_stage1_post_allreduce")
        norm = sum_of_squares(grads).sqrt()
        self.step_count += 1
        self._record_memory_event("measured_step_stage1_pre_allgather")
        self._adamw_and_gather(self.space.shard(grads), clip_coefficient(norm, max_grad_norm))
        self._record_memory_event("measured_step_stage1_post_allgather")
        return norm

    def step_async(self, max_grad_norm: float = 0.0) -> torch.Tensor:
        return self._update(max_grad_norm)

    def step_with_stats(self, max_grad_norm: float = 0.0) -> Dict[str, float]:
        t0 = time.perf_counter()
        norm = self._update(max_grad_norm)
        return self._stats(norm, t0, {"allreduce": "allreduce", "post_allgather": "post_allgather"})


class ZeROStage2Optimizer(_ShardedStateMixin, _FlatEngine):
    """Sharded optimizer state and gradients; replicated parameters."""

    stage = 2
    shard_optimizer = True

    def __init__(self, model: nn.Module, grad_bucket_numel: int = 16 * 1024 * 1024, **kwargs) -> None:
        self._ring = False
        super().__init__(model, **kwargs)
        # Accepted for CLI compatibility: buckets are transformer blocks (see _setup_ring).
        self.grad_bucket_numel = grad_bucket_numel
        self._routed = self.space.grads is None and self._routed_requested()
        if self._routed:
            self._setup_routed()
            return
        if self.space.grads is None:  # the gradient ring was requested
            if self._setup_ring():
                return
            self.space.grads = self.collectives.alloc(self.space.padded_numel, torch.float32)
            self.space.bind_grads()
        # On one rank the reduce-scatter is the identity, so the gradient shard IS the flat gradient
        # buffer: no copy of the gradients after backward, nothing extra to zero per step (stage 0's
        # memory traffic).  Several micro-batches accumulate in place, which gives the same sum.
        self._shard_is_buffer = self.world_size == 1
        if self._shard_is_buffer:
            self.grad_shard = self.space.shard(self.space.grads)
        else:
            self.grad_shard = torch.zeros(self.space.chunk, dtype=torch.float32, device=self.device)
        self._pending_flush = False
        self._setup_overlap()
        self._setup_fused_step()

    # -- gradients routed to their owners (no full gradient buffer) --------------------------------
    def _full_grad_buffer(self) -> bool:
        return not (self._routed_requested() or self._ring_requested())

    # -- gradient ring: per-block buckets reduced into the owners' shards during backward ----------
    # ``ZB_STAGE2_GRADS=auto`` takes the gradient ring when the full fp32 gradient buffer would be
    # at least this large.  The ring adds one bucket kernel (two cross-rank barriers, a clear) per
    # transformer block to the backward's critical path: ~0.6 ms per step for the 110 M-parameter
    # `small` model at 2 GPUs (9.49 vs 8.87 ms), a fixed cost per block that a 7B model's blocks
    # (tens of ms each) hide in the noise, where the 28 GB the ring saves per GPU decide how large a
    # batch fits.
    RING_AUTO_MIN_BYTES = 16 << 30

    def _ring_requested(self) -> bool:
        """Stage 2 with the NVLink collectives on several GPUs: the gradient ring when
        ``ZB_STAGE2_GRADS=ring``, or under ``auto`` (the default) when the full gradient buffer would
        reach ``RING_AUTO_MIN_BYTES``; never with the fused one-kernel step or the overlapped
        flat-buffer reduce-scatter (both work on the full buffer)."""
        mode = os.environ.get("ZB_STAGE2_GRADS", "auto")
        if mode not in ("auto", "ring") or self.world_size == 1 or self.device.type != "cuda":
            return False
        if os.environ.get("ZB_FUSED_STEP", "0") == "1" or os.environ.get("ZB_OVERLAP_REDUCE_SCATTER", "0") == "1":
            return False
        if not getattr(self.collectives, "supports_bucket_reduce", False):
            return False
        if mode == "auto":
            from .common import aligned_layout

            _, numel, _ = aligned_layout(self.meta, self.world_size)
            return numel * 4 >= self.RING_AUTO_MIN_BYTES
        return True

    @property
    def gradient_mode(self) -> str:
        """How this engine holds gradients: ``full`` (flat fp32 buffer), ``ring`` or ``routed``."""
        return "ring" if self._ring else "routed" if getattr(self, "_routed", False) else "full"

    def _block_ranges(self) -> List[Tuple[int, int, List[nn.Parameter]]]:
        """(lo, hi, params) of every transformer block's contiguous flat range, in flat order; hi is
        rounded up to a multiple of 8 (parameters start 64-element aligned, so ranges stay disjoint)."""
        offset = {id(p): off for p, off in zip(self.meta.params, self.space.offsets)}
        out = []
        for module in self.model.modules():
            if type(module).__name__ != "TransformerBlock":
                continue
            ps = [p for p in module.parameters() if id(p) in offset]
            if not ps:
                continue
            lo = min(offset[id(p)] for p in ps)
            hi = max(offset[id(p)] + p.numel() for p in ps)
            out.append((lo, (hi + 7) // 8 * 8, ps))
        out.sort(key=lambda r: r[0])
        for (_, hi0, _), (lo1, _, _) in zip(out, out[1:]):
            if lo1 < hi0:
                return []
        if any(lo % 8 for lo, _, _ in out):
            return []
        return out

    def _setup_ring(self) -> bool:
        """Gradient memory without a full fp32 buffer, with the reduce-scatter spread over backward.

        Buckets: every transformer block's flat range, and the ranges between them (embedding, final
        norm, LM head: the edge buckets).  Each bucket of n elements is cut into W slices of ``part``
        elements (n rounded up to 8W); rank r owns slice r of EVERY bucket, so its shard - gradient,
        fp32 master, Adam moments - is the concatenation of its slices (the interleaved layout), and a
        bucket's reduce-scatter is balanced and writes nothing remote.  Each block's weight gradients
        accumulate into one of ``ZB_STAGE2_RING_SLOTS`` (default 2) symmetric bucket buffers (block j
        uses slot j mod slots), the edge buckets into their own.  As soon as a block's backward has
        issued its weight gradients (the block kernels' grad-ready hook), one kernel on the same
        stream reduces this rank's slice of the bucket into its gradient segment, averaged, and
        clears the bucket; the slot is free for block j - slots, which the stream runs afterwards.
        The edge buckets are reduced when backward ends.  The update is one kernel: AdamW over the
        shard and the bf16 all-gather of every slice.  Gradient memory: the shard (4 B/param / W)
        plus the slots and edge buffers, instead of 4 B/param."""
        ranges = self._block_ranges()
        if not ranges:
            return False
        W, r = self.world_size, self.rank
        used = (self.space.numel + 7) // 8 * 8
        buckets, cursor = [], 0  # (lo, hi, block index or -1)
        for j, (lo, hi, _) in enumerate(ranges):
            if lo > cursor:
                buckets.append((cursor, lo, -1))
            buckets.append((lo, hi, j))
            cursor = hi
        if cursor < used:
            buckets.append((cursor, used, -1))
        coll = self.collectives
        n_slots = max(1, int(os.environ.get("ZB_STAGE2_RING_SLOTS", "2")))
        seg_rows, shard_off = [], 0
        self._ring_buckets = []  # (lo, hi, part, shard offset, block index or -1)
        for lo, hi, j in buckets:
            part = -(-(hi - lo) // (8 * W)) * 8
            valid = max(0, min(part, (hi - lo) - r * part))
            seg_rows.append((shard_off // 8, part // 8, valid // 8, lo * self.space.params.element_size()))
            self._ring_buckets.append((lo, hi, part, shard_off, j))
            shard_off += part
        total = shard_off
        slot_numel = max(W * part for lo, hi, part, off, j in self._ring_buckets if j >= 0)
        self._ring_slots = [coll.alloc(slot_numel, torch.float32) for _ in range(n_slots)]
        self._ring_edge_bufs = {i: coll.alloc(W * part, torch.float32)
                                for i, (lo, hi, part, off, j) in enumerate(self._ring_buckets) if j < 0}
        self._ring_segs = torch.tensor(seg_rows, dtype=torch.int64, device=self.device)
        self._ring_seg_rows = seg_rows
        self._ring_block_bucket = {j: i for i, (_, _, _, _, j) in enumerate(self._ring_buckets) if j >= 0}
        self._ring_block_of = {}
        for j, (_, _, ps) in enumerate(ranges):
            for p in ps:
                self._ring_block_of[id(p)] = j
        self._ring_params: List[List[nn.Parameter]] = [[] for _ in self._ring_buckets]
        for p, off in zip(self.meta.params, self.space.offsets):
            i = next(i for i, (lo, hi, _, _, _) in enumerate(self._ring_buckets) if lo <= off < hi)
            lo, _, _, _, j = self._ring_buckets[i]
            buf = self._ring_slots[j % n_slots] if j >= 0 else self._ring_edge_bufs[i]
            p.main_grad = buf[off - lo : off - lo + p.numel()].view(p.shape)
            self._ring_params[i].append(p)
        # the shard in interleaved order: gradient, fp32 master and Adam moments
        self.grad_shard = torch.zeros(total, dtype=torch.float32, device=self.device)
        master = torch.zeros(total, dtype=torch.float32, device=self.device)
        for (lo, hi, part, off, _), row in zip(self._ring_buckets, seg_rows):
            valid = row[2] * 8
            if valid:
                master[off : off + valid].copy_(self.space.params[lo + r * part : lo + r * part + valid])
        self._master = master
        self._exp_avg = torch.zeros_like(master)
        self._exp_avg_sq = torch.zeros_like(master)
        from ...ops import functional as F

        self._ring = True
        self._ring_hook = F.register_grad_ready_hook(self._on_ring_block_ready)
        self._shard_is_buffer = False
        self._pending_flush = False
        self._overlap = False
        self._fused_step = False
        self._fused_sq = None
        return True

    def _ring_reduce(self, i: int) -> None:
        lo, hi, part, off, j = self._ring_buckets[i]
        W = self.world_size
        bucket = (self._ring_slots[j % len(self._ring_slots)] if j >= 0 else self._ring_edge_bufs[i])[: W * part]
        with self.clock.measure("backward_reduce_scatter", W * part * 4):
            with self.collectives.label_scope("stage2.backward.reduce_scatter.bucket"):
                ok = self.collectives.bucket_reduce_(bucket, self.grad_shard[off : off + part], 1.0 / W)
        if not ok:
            raise RuntimeError("gradient ring: bucket reduce unavailable")

    def _on_ring_block_ready(self, params) -> None:
        """Every backward of a block writes its slot once and reduces it once, whoever runs it."""
        j = self._ring_block_of.get(id(params[0])) if params else None
        if j is not None:
            self._ring_reduce(self._ring_block_bucket[j])

    def _ring_flush(self) -> None:
        """After backward: blocks whose gradients autograd left in ``param.grad`` (modules that do not
        run as one block kernel, so no hook fired), then the edge buckets."""
        self._record_memory_event("measured_step_stage2_pre_reduce_scatter")
        for i in reversed(range(len(self._ring_buckets))):
            j = self._ring_buckets[i][4]
            pending = [p for p in self._ring_params[i] if p.grad is not None]
            for p in pending:
                p.main_grad.add_(p.grad.detach().to(torch.float32))
                p.grad = None
            if j < 0 or pending:
                self._ring_reduce(i)
        self._record_memory_event("measured_step_stage2_post_reduce_scatter")

    def _ring_update(self, scale: torch.Tensor) -> None:
        """AdamW on the interleaved shard and the bf16 all-gather of every slice (one kernel with the
        NVLink collectives; otherwise AdamW on the master and per-bucket all-gathers)."""
        dev_scalars = self._device_scalars()
        fused = getattr(self.collectives, "adamw_allgather_segments", None)
        if fused is not None and self.device.type == "cuda":
            with self.clock.measure("post_allgather", self._master.numel() * 2):
                if fused(self.space.params, self._ring_segs, self._master, self._exp_avg, self._exp_avg_sq,
                         self.grad_shard, scale, self.adam, self.step_count, dev_scalars):
                    return
        with self.clock.measure("optimizer"):
            adamw_update_(self._master, self._exp_avg, self._exp_avg_sq, self.grad_shard, self.adam, self.step_count,
                          grad_scale=scale, param_out=None, dev_scalars=dev_scalars)
        self._ring_write_params()

    def _ring_write_params(self) -> None:
        """Every rank's parameters from every rank's master slices (per bucket: an all-gather of the
        model-dtype slices, then the valid part copied into the flat parameter buffer)."""
        import torch.distributed as dist

        W = self.world_size
        with self.clock.measure("post_allgather", self._master.numel() * 2):
            for lo, hi, part, off, _ in self._ring_buckets:
                mine = self._master[off : off + part].to(self.space.params.dtype)
                parts = [torch.empty_like(mine) for _ in range(W)]
                dist.all_gather(parts, mine)
                self.space.params[lo:hi].copy_(torch.cat(parts)[: hi - lo])

    def _ring_bytes(self) -> int:
        if not self._ring:
            return 0
        return tensors_num_bytes(list(self._ring_slots) + list(self._ring_edge_bufs.values()))

    def _routed_requested(self) -> bool:
        return bool(os.environ.get("ZB_ROUTED_GRADS", "0") == "1" and self.world_size > 1
                    and self.device.type == "cuda" and getattr(self.collectives, "supports_routed_grads", False))

    def _setup_routed(self) -> None:
        """``ZB_ROUTED_GRADS=1`` (NVLink collectives): no rank keeps a full gradient buffer.  The
        gradient shard of every rank is a symmetric fp32 buffer of ``chunk`` elements; every weight
        gradient, as its kernel finishes it, is added straight into the owning ranks' shards over
        NVLink (``param.grad_route``: the B200 kernels write a temporary buffer that the sink pushes
        with system-scope vector reductions), so no reduce-scatter runs after backward and gradient
        memory is the shard only (4 B/param / W instead of 4 B/param).  A barrier at ``zero_grad``
        (every shard cleared before anyone adds) and one before the update (every addition landed)
        order the pushes."""
        coll = self.collectives
        self.grad_shard = coll.alloc(self.space.chunk, torch.float32)  # rank r's buffer is shard r
        bases = coll.shard_bases(self.grad_shard)
        if bases is None:
            raise RuntimeError("routed gradients need the shard in a symmetric buffer of the collectives")
        route = _ShardRoute(coll, self.space.chunk, bases)
        for p, off in zip(self.meta.params, self.space.offsets):
            p.grad_route = (route, int(off))
        self._route = route
        self._shard_is_buffer = False
        self._pending_flush = False
        self._overlap = False
        self._fused_step = False
        self._fused_sq = None

    def _push_autograd_grads(self) -> None:
        """Gradients that reached ``param.grad`` through autograd (modules outside the B200 kernels)."""
        for p, off in zip(self.meta.params, self.space.offsets):
            if p.grad is not None:
                self._route.push(p.grad.detach().to(torch.float32).reshape(-1), int(off))
                p.grad = None

    def _routed_update(self, max_grad_norm: float) -> torch.Tensor:
        self._push_autograd_grads()
        self._record_memory_event("measured_step_stage2_pre_reduce_scatter")
        with self.clock.measure("backward_reduce_scatter", 0):
            self.collectives.barrier()  # every rank's additions have landed in the owners' shards
        self._record_memory_event("measured_step_stage2_post_reduce_scatter")
        inv_w = 1.0 / self.world_size
        # the shard holds the sum over ranks: the averaged gradient's norm is 1/W of its norm
        norm = global_norm_from_local_sq(sum_of_squares(self.grad_shard), sharded=True,
                                         collectives=self.collectives) * inv_w
        self.step_count += 1
        self._record_memory_event("measured_step_stage2_pre_allgather")
        with self.collectives.label_scope("stage2.step.allgather.updated_param_shard"):
            self._adamw_and_gather(self.grad_shard, clip_coefficient(norm, max_grad_norm) * inv_w)
        self._record_memory_event("measured_step_stage2_post_allgather")
        self._record_memory_event("measured_step_stage2_post_step_free_grad_shard")
        return norm

    # -- reduce-scatter overlapped with backward -------------------------------------------
    def _setup_overlap(self) -> None:
        """Per-block gradient buckets reduced on a high-priority stream while backward continues.

        Enabled with ``ZB_OVERLAP_REDUCE_SCATTER=1`` when the collectives offer a bucketed
        reduce-scatter on the flat gradient buffer (the NVLink kernels).  Each transformer block's parameters occupy one contiguous range of the
        flat space; when the block's backward has issued its weight gradients, that range is
        reduce-scattered (each rank reduces the part inside its shard) on the side stream.  The
        ranges no block covers (embedding / head / final norm) are reduced when backward ends.
        """
        self._overlap = False
        self._buckets: List[Tuple[int, int]] = []
        self._bucket_of: Dict[int, int] = {}
        if not (self.world_size > 1 and self.device.type == "cuda"
                and getattr(self.collectives, "supports_range_reduce_scatter", False)):
            return
        # Opt-in.  Measured on 2 B200 (small model, stage 2): 10.32 ms/step without, 13.07 ms with (8-block
        # buckets) and 11.13 ms (full-grid buckets): a bucket kernel that waits at its cross-rank barrier
        # holds SMs that the statically scheduled persistent GEMM CTAs need, so its wait lands on the
        # critical path.  Worth revisiting with dynamically scheduled (work-counter) compute kernels.
        if os.environ.get("ZB_OVERLAP_REDUCE_SCATTER", "0") != "1":
            return
        offset = {id(p): off for p, off in zip(self.meta.params, self.space.offsets)}
        for module in self.model.modules():
            if type(module).__name__ != "TransformerBlock":
                continue
            ps = [p for p in module.parameters() if id(p) in offset]
            if not ps:
                continue
            lo = min(offset[id(p)] for p in ps)
            hi = max(offset[id(p)] + p.numel() for p in ps)
            hi = (hi + 3) // 4 * 4
            if lo % 4:
                return  # layout not bucketable; keep the single reduce-scatter
            for p in ps:
                self._bucket_of[id(p)] = len(self._buckets)
            self._buckets.append((lo, hi))
        if not self._buckets:
            return
        from ...ops import functional as F

        self._comm_stream = torch.cuda.Stream(device=self.device, priority=-1)
        self._launched: List[int] = []
        self._overlap_active = False
        self._hook = F.register_grad_ready_hook(self._on_block_grads_ready)
        self._overlap = True

    # Thread blocks for buckets reduced while backward runs: few, so that the persistent compute
    # kernels keep almost every SM; the final flush runs alone and uses the full grid.
    OVERLAP_BLOCKS = 8

    def _reduce_range(self, lo: int, hi: int, blocks: int = 0) -> None:
        grads = self.space.grads
        with self.clock.measure("backward_reduce_scatter", (hi - lo) * grads.element_size()):
            ok = self.collectives.reduce_scatter_range_accumulate_(self.grad_shard, grads, lo, hi,
                                                                   self.space.shard_start, 1.0 / self.world_size,
                                                                   blocks)
        if not ok:
            raise RuntimeError("bucketed reduce-scatter unavailable for the flat gradient buffer")

    def _on_block_grads_ready(self, params) -> None:
        if not self._overlap_active or not params:
            return
        b = self._bucket_of.get(id(params[0]))
        if b is None or b in self._launched:
            return
        ready = torch.cuda.Event()
        ready.record()
        with torch.cuda.stream(self._comm_stream):
            self._comm_stream.wait_event(ready)
            self._reduce_range(*self._buckets[b], blocks=self.OVERLAP_BLOCKS)
        self._launched.append(b)

    @property
    def flat_grad_buffer(self) -> torch.Tensor:
        return self.space.grads

    def zero_grad(self) -> None:
        if self._ring:  # the buckets are cleared by the kernels that reduce them
            self.clock.reset()
            for p in self.meta.params:
                p.grad = None
            self.grad_shard.zero_()
            self._pending_flush = True
            return
        if self._routed:
            self.clock.reset()
            for p in self.meta.params:
                p.grad = None
            self.grad_shard.zero_()
            self.collectives.barrier()  # no rank adds into a shard before its owner has cleared it
            self._pending_flush = True
            return
        super().zero_grad()
        if not self._shard_is_buffer:
            self.grad_shard.zero_()
        self._pending_flush = True

    def backward(self, loss: torch.Tensor) -> None:
        if self._ring:
            loss.backward()
            self._ring_flush()
            self._pending_flush = False
            return
        if self._overlap:
            self._launched = []
            self._overlap_active = True
        try:
            loss.backward()
        finally:
            if self._overlap:
                self._overlap_active = False
        self._pending_flush = True
        if not (self._fused_step or self._routed):  # those reduce inside the step / while backward runs
            self._flush_flat_grad_buffer()

    def _flush_overlapped(self) -> None:
        """Reduce what the per-block buckets did not cover, then join the side stream."""
        grads = self.space.grads
        covered = sorted(self._buckets[b] for b in self._launched)
        rest, cursor = [], 0
        for lo, hi in covered:
            if lo > cursor:
                rest.append((cursor, lo))
            cursor = max(cursor, hi)
        if cursor < grads.numel():
            rest.append((cursor, grads.numel()))
        ready = torch.cuda.Event()
        ready.record()
        with torch.cuda.stream(self._comm_stream):
            self._comm_stream.wait_event(ready)
            for lo, hi in rest:
                self._reduce_range(lo, hi)
        torch.cuda.current_stream().wait_stream(self._comm_stream)
        grads.zero_()
        self._pending_flush = False

    def _flush_flat_grad_buffer(self) -> None:
        if not self._pending_flush:
            return
        self.space.fold_autograd_grads()
        grads = self.space.grads
        if self._overlap and self._launched:
            self._record_memory_event("measured_step_stage2_pre_reduce_scatter")
            with self.collectives.label_scope("stage2.backward.reduce_scatter.flat_grad_buffer"):
                self._flush_overlapped()
            self._record_memory_event("measured_step_stage2_post_reduce_scatter")
            return
        self._record_memory_event("measured_step_stage2_pre_reduce_scatter")
        with self.clock.measure("backward_reduce_scatter", tensor_num_bytes(grads)):
            with self.collectives.label_scope("stage2.backward.reduce_scatter.flat_grad_buffer"):
                if self.world_size > 1:
                    self._reduce_scatter_grads(self.grad_shard, grads, 1.0 / self.world_size)
                elif not self._shard_is_buffer:
                    self.grad_shard.add_(grads)
        self._record_memory_event("measured_step_stage2_post_reduce_scatter")
        if not self._shard_is_buffer:
            grads.zero_()
        self._pending_flush = False

    def _update(self, max_grad_norm: float) -> torch.Tensor:
        if self._routed:
            return self._routed_update(max_grad_norm)
        if self._ring:
            return self._ring_step(max_grad_norm)
        if any(p.grad is not None for p in self.meta.params) and not hasattr(self.meta.params[0], "main_grad"):
            raise RuntimeError("Stage 2 expects gradients in the flat buffer")
        if self._fused_step and max_grad_norm <= 0 and self._pending_flush:
            norm = self._fused_update(tuple(f"measured_step_stage2_{x}" for x in (
                "pre_reduce_scatter", "post_reduce_scatter", "pre_allgather", "post_allgather",
                "post_step_free_grad_shard")))
            if norm is not None:
                self._pending_flush = False
                return norm
        if not self._ring:
            self._flush_flat_grad_buffer()
        norm = global_norm_from_local_sq(sum_of_squares(self.grad_shard), sharded=self.world_size > 1,
                                         collectives=self.collectives)
        self.step_count += 1
        self._record_memory_event("measured_step_stage2_pre_allgather")
        with self.collectives.label_scope("stage2.step.allgather.updated_param_shard"):
            self._adamw_and_gather(self.grad_shard, clip_coefficient(norm, max_grad_norm))
        self._record_memory_event("measured_step_stage2_post_allgather")
        self._record_memory_event("measured_step_stage2_post_step_free_grad_shard")
        return norm

    def _ring_step(self, max_grad_norm: float) -> torch.Tensor:
        if self._pending_flush:  # backward ran outside engine.backward()
            self._ring_flush()
            self._pending_flush = False
        norm = global_norm_from_local_sq(sum_of_squares(self.grad_shard), sharded=True,
                                         collectives=self.collectives)
        self.step_count += 1
        self._record_memory_event("measured_step_stage2_pre_allgather")
        with self.collectives.label_scope("stage2.step.allgather.updated_param_shard"):
            self._ring_update(clip_coefficient(norm, max_grad_norm))
        self._record_memory_event("measured_step_stage2_post_allgather")
        self._record_memory_event("measured_step_stage2_post_step_free_grad_shard")
        return norm

    def step_async(self, max_grad_norm: float = 0.0) -> torch.Tensor:
        return self._update(max_grad_norm)

    def step_with_stats(self, max_grad_norm: float = 0.0) -> Dict[str, float]:
        t0 = time.perf_counter()
        norm = self._update(max_grad_norm)
        return self._stats(norm, t0, {"backward_reduce_scatter": "backward_reduce_scatter",
                                      "post_allgather": "post_allgather"})

    def state_dict(self) -> Dict[str, object]:
        state = super().state_dict()
        if self._ring:  # the shard holds slice `rank` of every bucket, in bucket order
            state["layout"] = "ring_interleaved_v1"
            state["ring_segments"] = [(lo, hi, part, off) for lo, hi, part, off, _ in self._ring_buckets]
            state.pop("shard_start", None)
            state.pop("shard_end", None)
        return state

    def load_state_dict(self, state: Dict[str, object]) -> None:
        if not self._ring:
            super().load_state_dict(state)
            return
        if state.get("layout") != "ring_interleaved_v1" or [tuple(x) for x in state["ring_segments"]] != [
                (lo, hi, part, off) for lo, hi, part, off, _ in self._ring_buckets]:
            raise ValueError("checkpoint shard layout differs from this engine's gradient-ring layout")
        self.step_count = int(state["step_count"])
        self._master.copy_(state["local_master_param_shard"].to(self.device, torch.float32))
        self._exp_avg.copy_(state["exp_avg"].to(self.device, torch.float32))
        self._exp_avg_sq.copy_(state["exp_avg_sq"].to(self.device, torch.float32))
        if "grad_shard" in state:
            self.grad_shard.copy_(state["grad_shard"].to(self.device, torch.float32))
        self._ring_write_params()

    def _logical_grad_bytes(self) -> int:
        return self.space.chunk * self.space.params.element_size()

    def _debug_memory_components_mb(self) -> Dict[str, float]:
        return {
            "logical_params_mb": bytes_to_mb(sum(p.numel() for p in self.meta.params) * self.space.params.element_size()),
            "logical_grads_mb": bytes_to_mb(self._logical_grad_bytes()),
            "logical_optimizer_mb": bytes_to_mb(tensors_num_bytes([self._master, self._exp_avg, self._exp_avg_sq])),
            "live_full_grads_mb": 0.0,
            "live_flat_grad_buffer_mb": bytes_to_mb(tensor_num_bytes(self.space.grads)) if self.space.grads is not None
            else bytes_to_mb(self._ring_bytes()),
            "live_grad_shard_mb": bytes_to_mb(tensor_num_bytes(self.grad_shard)),
            "comm_temp_mb": 0.0,
        }

    def debug_memory_components_mb(self) -> Dict[str, float]:
        return self._debug_memory_components_mb()

    def live_model_state_breakdown_mb(self) -> Dict[str, float]:
        base = self.memory_state_breakdown_mb()
        shard_bytes = 0 if self._shard_is_buffer else tensor_num_bytes(self.grad_shard)  # a view of the buffer
        flat_bytes = tensor_num_bytes(self.space.grads) if self.space.grads is not None else self._ring_bytes()
        grads_mb = bytes_to_mb(flat_bytes + shard_bytes)
        base["total_mb"] += grads_mb - base["grads_mb"]
        base["grads_mb"] = grads_mb
        return base

    def _extra_state(self) -> Dict[str, object]:
        return {"grad_shard": self.grad_shard.detach().cpu()}
