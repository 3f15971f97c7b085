"""Training-session API: one object that owns the process group, model, collectives and
ZeRO engine, and runs one optimizer step per call.

This is the public entry point a user (and the benchmark) calls::

    from cs244c_llama_zero_b200.train import TrainSession, SessionConfig
    sess = TrainSession(SessionConfig(model_size="baseline-small", zero_stage=2, batch_size=8, seq_len=1024))
    loss = sess.train_step(input_ids)          # input_ids: int64 [B, S] on the host or the device
    print(float(loss))

Semantics follow the reference's ``train_zero.py`` step (``train_zero.py:416-589``):
zero_grad -> prepare_forward -> for each micro-batch: forward under bf16 autocast with labels ==
inputs (the model shifts them), backward(loss / grad_accum) -> optimizer step.  Inputs given on
the host are copied with a non-blocking H2D transfer from pinned memory.

``SessionConfig(cuda_graph=True)`` (ZeRO stages 0-2 on CUDA) runs the first ``graph_warmup_steps``
steps eagerly on a side stream, then captures one whole step (H2D-staged input buffer -> zero_grad ->
forward -> backward -> collectives -> optimizer) into a CUDA graph and replays it for every later
step: the host issues one launch per step instead of several hundred.  The optimizer's step number
lives on the device then (``use_device_step``), so the captured AdamW bias corrections advance on
each replay.  Per-collective timing is off in graph mode.  Call ``reset_graph()`` after anything
that replaces the engine's buffers (``load_state_dict``); the next step captures again.
"""

from __future__ import annotations

import contextlib
import os
from dataclasses import dataclass, field
from datetime import timedelta
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from ..models import BASELINE_VOCAB_SIZE, LlamaForCausalLM, ModelConfig, build_config
from ..parallel.collectives import TracingCollectives, pick_collectives
from ..parallel.zero import ENGINES
from ..profiler.nvtx import nvtx_range


@dataclass
class SessionConfig:
    model_size: str = "baseline-small"
    vocab_size: int = BASELINE_VOCAB_SIZE
    seq_len: int = 1024
    batch_size: int = 8
    grad_accum_steps: int = 1
    zero_stage: int = 0
    collective_impl: str = "torch"
    dtype: str = "bfloat16"
    backend: str = "auto"  # "b200" on CUDA, "torch" on CPU
    learning_rate: float = 3e-4
    weight_decay: float = 0.1
    betas: Tuple[float, float] = (0.9, 0.95)
    eps: float = 1e-8
    max_grad_norm: float = 0.0
    seed: int = 1337
    loss_chunk_size: int = 128
    activation_checkpointing: bool = False
    profile_collectives: bool = False
    model_overrides: dict = field(default_factory=dict)
    pg_timeout_s: float = 600.0
    cuda_graph: bool = False  # capture the whole step once and replay it (stages 0-2, CUDA)
    graph_warmup_steps: int = 3


def init_distributed(timeout_s: float = 600.0) -> Tuple[int, int, torch.device]:
    """torchrun environment -> (rank, world, device); NCCL on CUDA, Gloo on CPU."""
    if "RANK" not in os.environ or "WORLD_SIZE" not in os.environ:
        if torch.cuda.is_available():
            return 0, 1, torch.device("cuda", torch.cuda.current_device())
        return 0, 1, torch.device("cpu")
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local_rank = int(os.environ.get("LOCAL_RANK", rank))
    if torch.cuda.is_available():
        torch.cuda.set_device(local_rank)
        device = torch.device("cuda", local_rank)
        if not dist.is_initialized():
            dist.init_process_group(backend="nccl", timeout=timedelta(seconds=timeout_s), device_id=device)
    else:
        device = torch.device("cpu")
        if not dist.is_initialized():
            dist.init_process_group(backend="gloo", timeout=timedelta(seconds=timeout_s))
    return rank, world, device


def model_param_dtype(device: torch.device, dtype_name: str) -> torch.dtype:
    if device.type != "cuda" or dtype_name == "float32":
        return torch.float32
    return torch.bfloat16


DEVICE_INIT_MIN_PARAMS = 1_000_000_000


def build_model(cfg: ModelConfig, device: torch.device, dtype: torch.dtype) -> LlamaForCausalLM:
    """The model in ``dtype`` on ``device``.  Models of a billion parameters or more are created and
    initialised on the GPU itself (normal(0, 0.02) from the CUDA generator; same initialisation order):
    building a 7B model on the host first would take minutes and ~28 GB of host memory per rank.
    Smaller models are initialised on the host, which reproduces the reference's weights for a seed."""
    from ..models.config import estimate_num_parameters

    if device.type == "cuda" and estimate_num_parameters(cfg) >= DEVICE_INIT_MIN_PARAMS:
        with torch.device(device):
            model = LlamaForCausalLM(cfg)
        return model.to(dtype=dtype)
    return LlamaForCausalLM(cfg).to(device=device, dtype=dtype)


def broadcast_model(model: torch.nn.Module) -> None:
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        for p in model.parameters():
            dist.broadcast(p.data, src=0)


class AsyncLoss:
    """A step's loss on its way to the host (see ``TrainSession.train_step_async``).

    The session reuses its pinned slots round-robin (4 of them), so read a handle within three
    further steps.
    """

    def __init__(self, host: torch.Tensor, event: Optional["torch.cuda.Event"],
                 errors: Optional[torch.Tensor] = None) -> None:
        self._host = host
        self._event = event
        self._errors = errors  # pinned copy of the device error record taken with the loss

    def item(self) -> float:
        """The loss; raises ``DeviceWaitError`` if a kernel's bounded wait expired up to this step."""
        if self._event is not None:
            self._event.synchronize()
        if self._errors is not None:
            from ..ops import raise_for_device_errors

            raise_for_device_errors(self._errors.tolist())
        return float(self._host[0])

    @property
    def nbytes(self) -> int:
        """Bytes this handle brings back to the host (loss + error record)."""
        extra = 0 if self._errors is None else self._errors.numel() * self._errors.element_size()
        return self._host.numel() * self._host.element_size() + extra


class TrainSession:
    def __init__(self, cfg: SessionConfig, model_cfg: Optional[ModelConfig] = None) -> None:
        self.cfg = cfg
        self.rank, self.world_size, self.device = init_distributed(cfg.pg_timeout_s)
        torch.manual_seed(cfg.seed)
        if self.device.type == "cuda":
            torch.cuda.manual_seed_all(cfg.seed)
            torch.backends.cuda.matmul.allow_tf32 = True
            torch.backends.cudnn.allow_tf32 = True
        self.model_cfg = model_cfg or build_config(cfg.model_size, vocab_size=cfg.vocab_size, max_seq_len=cfg.seq_len,
                                                   **cfg.model_overrides)
        backend = cfg.backend
        if backend == "auto":
            backend = "b200" if self.device.type == "cuda" else "torch"
        self.backend = backend
        dtype = model_param_dtype(self.device, cfg.dtype)
        self.model = build_model(self.model_cfg, self.device, dtype)
        self.model.set_loss_chunk_size(cfg.loss_chunk_size)
        self.model.set_activation_checkpointing(cfg.activation_checkpointing)
        self.model.set_backend(backend)
        broadcast_model(self.model)
        collectives = pick_collectives(self.world_size, cfg.collective_impl, self.device)
        if cfg.profile_collectives:
            collectives = TracingCollectives(collectives)
        self.collectives = collectives
        self.engine = ENGINES[cfg.zero_stage](
            model=self.model, lr=cfg.learning_rate, betas=cfg.betas, eps=cfg.eps, weight_decay=cfg.weight_decay,
            collectives=collectives,
        )
        self._staging: Optional[torch.Tensor] = None
        self._loss_ring: Optional[List[torch.Tensor]] = None  # pinned host slots of train_step_async
        self._loss_slot = 0
        self.autocast = dtype == torch.bfloat16
        self._autocast_cache = True
        # CUDA-graph mode state
        self._graph: Optional["torch.cuda.CUDAGraph"] = None
        self._graph_ids: Optional[torch.Tensor] = None
        self._graph_loss: Optional[torch.Tensor] = None
        self._graph_warm = 0
        self._warm_stream: Optional["torch.cuda.Stream"] = None
        self.graph_kernels_per_step = 0
        if cfg.cuda_graph:
            reason = self.graph_unsupported_reason()
            if reason:
                raise ValueError(f"cuda_graph: {reason}")

    # ----------------------------------------------------------------------------- steps
    def _to_device(self, input_ids: torch.Tensor) -> torch.Tensor:
        if input_ids.device == self.device:
            return input_ids
        if self._staging is None or self._staging.shape != input_ids.shape:
            self._staging = torch.empty(input_ids.shape, dtype=torch.long, device=self.device)
        self._staging.copy_(input_ids, non_blocking=True)
        return self._staging

    def _loss_scale_context(self, n: int):
        """On the B200 backend: announce that each micro-batch loss is back-propagated as ``loss / n``,
        which lets the LM head compute its gradients during the forward pass (no logits tensor)."""
        if self.backend != "b200" or self.device.type != "cuda":
            return contextlib.nullcontext()
        from ..ops import functional as B

        if not hasattr(self, "_loss_scales"):
            self._loss_scales = {}
        if n not in self._loss_scales:
            self._loss_scales[n] = torch.full((), 1.0 / n, dtype=torch.float32, device=self.device)
        return B.loss_gradient_scale(self._loss_scales[n])

    def forward_backward(self, micro_batches: Sequence[torch.Tensor]) -> torch.Tensor:
        """Run every micro-batch; returns the mean loss as a device scalar (no host sync)."""
        total = torch.zeros((), dtype=torch.float32, device=self.device)
        n = len(micro_batches)
        for ids in micro_batches:
            ids = self._to_device(ids)
            with nvtx_range("forward"), torch.autocast(device_type=self.device.type, dtype=torch.bfloat16,
                                                       enabled=self.autocast, cache_enabled=self._autocast_cache), \
                    self._loss_scale_context(n):
                loss = self.model(input_ids=ids, labels=ids, return_logits=False).loss
            with nvtx_range("backward"):
                self.engine.backward(loss / n)
            total = total + loss.detach().float()
        return total / n

    def train_step(self, input_ids: torch.Tensor) -> torch.Tensor:
        """One optimizer step on ``input_ids`` ([grad_accum * B, S] or [B, S]); returns the loss (device).

        In graph mode the returned tensor is the graph's static output: read (or copy) it before the
        next step overwrites it.
        """
        if self.cfg.cuda_graph and self.device.type == "cuda":
            return self._train_step_graphed(input_ids)
        return self._train_step_eager(input_ids)

    # ----------------------------------------------------------------------------- CUDA graph
    def graph_unsupported_reason(self) -> Optional[str]:
        """Why this session cannot run its step as a CUDA graph (None when it can)."""
        if self.device.type != "cuda":
            return None  # graph mode is a no-op on CPU
        if self.cfg.zero_stage == 3:
            return "ZeRO-3 gathers parameters on a side stream with host-managed events; use stages 0-2"
        if self.cfg.activation_checkpointing:
            return "activation checkpointing replays the forward with host RNG bookkeeping"
        if self.cfg.profile_collectives:
            return "the collective trace times calls on the host"
        if os.environ.get("ZERO_SIM_BW_GBPS") or os.environ.get("ZERO_SIM_LATENCY_MS"):
            return "the simulated bandwidth mode sleeps on the host (use the nvlink mode, which paces on the device)"
        return None

    def reset_graph(self) -> None:
        """Drop the captured step (the next step captures again, after no further warm-up)."""
        self._graph = None
        self._graph_loss = None
        self.engine.use_device_step(False)
        self.engine.clock.timing = True

    def _train_step_graphed(self, input_ids: torch.Tensor) -> torch.Tensor:
        if self._graph is None:
            if self._graph_warm < self.cfg.graph_warmup_steps:
                # Eager warm-up on a side stream: lazy initialisation (extension buffers, tensor maps,
                # NCCL communicators, allocator pools) happens before capture, off the capture stream.
                self._graph_warm += 1
                if self._warm_stream is None:
                    self._warm_stream = torch.cuda.Stream(device=self.device)
                cur = torch.cuda.current_stream(self.device)
                self._warm_stream.wait_stream(cur)
                with torch.cuda.stream(self._warm_stream):
                    loss = self._train_step_eager(input_ids)
                cur.wait_stream(self._warm_stream)
                return loss
            return self._capture(input_ids)
        self._graph_ids.copy_(input_ids, non_blocking=True)
        self._graph.replay()
        self.engine.step_count += 1
        from .. import ops

        ops.count_graph_kernels(self.graph_kernels_per_step)
        return self._graph_loss

    def _capture(self, input_ids: torch.Tensor) -> torch.Tensor:
        from .. import ops

        self._graph_ids = torch.empty(input_ids.shape, dtype=torch.long, device=self.device)
        self._graph_ids.copy_(input_ids, non_blocking=True)
        self.engine.use_device_step(True)  # device counter = host step_count; the replay advances it
        self.engine.clock.timing = False
        self._autocast_cache = False
        torch.cuda.synchronize(self.device)
        before = ops.launch_count()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            loss = self._train_step_eager(self._graph_ids)  # host step_count advances once, for this call
        self.graph_kernels_per_step = ops.launch_count() - before
        self._graph, self._graph_loss = graph, loss
        graph.replay()  # capture only records: this runs the call's step
        return loss

    def _train_step_eager(self, input_ids: torch.Tensor) -> torch.Tensor:
        micro = list(input_ids.chunk(self.cfg.grad_accum_steps, dim=0)) if self.cfg.grad_accum_steps > 1 else [input_ids]
        self.model.train()
        self.engine.zero_grad()
        self.engine.prepare_forward()
        loss = self.forward_backward(micro)
        with nvtx_range("optimizer"):
            self.engine.step_async(max_grad_norm=self.cfg.max_grad_norm)
        return loss

    def train_step_async(self, input_ids: torch.Tensor) -> "AsyncLoss":
        """``train_step`` whose loss comes back to the host without stalling the launch queue.

        The loss is copied into pinned host memory on the compute stream (non-blocking); read it with
        ``.item()`` one step later, by which time the copy has normally landed, so the host keeps
        queuing the next step while the GPU finishes this one.
        """
        loss = self.train_step(input_ids)
        if self.device.type != "cuda":
            return AsyncLoss(loss.detach().float().reshape(1), None)
        if self._loss_ring is None:
            self._loss_ring = [torch.empty(1, dtype=torch.float32).pin_memory() for _ in range(4)]
            self._error_ring = [torch.zeros(4, dtype=torch.int32).pin_memory() for _ in range(4)]
        slot = self._loss_slot
        buf = self._loss_ring[slot]
        self._loss_slot = (slot + 1) % len(self._loss_ring)
        buf.copy_(loss.detach().float().reshape(1), non_blocking=True)
        errors = None
        if self.backend == "b200":  # the kernels' error record rides along with the loss (16 bytes)
            from .. import ops

            errors = self._error_ring[slot]
            ops.load_extension().device_errors_to_host(errors)
        ev = torch.cuda.Event()
        ev.record()
        return AsyncLoss(buf, ev, errors)

    def check_device_errors(self) -> None:
        """Synchronously read the kernels' error record; raises ``DeviceWaitError`` if a wait expired."""
        if self.device.type == "cuda" and self.backend == "b200":
            from .. import ops

            ops.check_device_errors()

    def close(self) -> None:
        self._graph = None  # a graph holding NCCL calls must go before the process group does
        if dist.is_available() and dist.is_initialized():
            dist.barrier()
            dist.destroy_process_group()
