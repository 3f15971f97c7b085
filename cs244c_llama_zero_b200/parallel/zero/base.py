"""Shared engine machinery: construction, comm timing, memory events, stats.

The engine duck type follows the reference (``zero/stage0_ddp.py:27-169``):
``zero_grad()``, ``prepare_forward() -> {"prepare_comm_ms"}``, ``backward(loss)``,
``step_with_stats(max_grad_norm) -> dict``, ``step(max_grad_norm) -> float``,
``memory_state_breakdown_mb()``, ``live_model_state_breakdown_mb()``,
``state_dict()`` / ``load_state_dict()`` and the attributes ``memory_tracker``,
``memory_trace_active``, ``memory_state_timeline``.

Additions: ``step_async(max_grad_norm)`` performs the same update without any host
synchronisation or statistics (used by the benchmark and CUDA-graph capture), and
communication time is measured with CUDA events on the stream that issued the
collective (device time), falling back to ``perf_counter`` on CPU.
"""

from __future__ import annotations

import time
from contextlib import contextmanager
from typing import Dict, Iterator, List, Optional, Tuple

import torch
import torch.nn as nn

from ..collectives import CollectiveOps, LocalCollectives, SendRecvCollectives, TorchCollectives
from .common import get_rank_world_size
from .optim import AdamWConfig


class CommClock:
    """Accumulates communication intervals per category on the device timeline."""

    def __init__(self, device: torch.device) -> None:
        self.cuda = device.type == "cuda" and torch.cuda.is_available()
        # False while a step is captured into a CUDA graph: events recorded during capture are graph
        # dependencies, not timestamps, so intervals are neither recorded nor read then.
        self.timing = True
        self._pending: Dict[str, List[Tuple[object, object]]] = {}
        self._host_ms: Dict[str, float] = {}
        self.calls: Dict[str, int] = {}
        self.bytes: Dict[str, int] = {}
        # callables returning {category: ms} for intervals timed elsewhere (native code) since their last call
        self._sources: List[object] = []

    def add_source(self, fn) -> None:
        self._sources.append(fn)

    def count(self, category: str, num_bytes: int = 0) -> None:
        """Count one call whose interval a registered source times."""
        self.calls[category] = self.calls.get(category, 0) + 1
        self.bytes[category] = self.bytes.get(category, 0) + int(num_bytes)

    def _drain(self) -> None:
        for fn in self._sources:
            for category, ms in fn().items():
                self._host_ms[category] = self._host_ms.get(category, 0.0) + ms

    def reset(self) -> None:
        self._drain()
        self._pending.clear()
        self._host_ms.clear()
        self.calls.clear()
        self.bytes.clear()

    @contextmanager
    def measure(self, category: str, num_bytes: int = 0) -> Iterator[None]:
        self.calls[category] = self.calls.get(category, 0) + 1
        self.bytes[category] = self.bytes.get(category, 0) + int(num_bytes)
        if not self.timing:
            yield
        elif self.cuda:
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record()
            yield
            end.record()
            self._pending.setdefault(category, []).append((start, end))
        else:
            t0 = time.perf_counter()
            yield
            self._host_ms[category] = self._host_ms.get(category, 0.0) + (time.perf_counter() - t0) * 1000.0

    def ms(self, category: str) -> float:
        self._drain()
        total = self._host_ms.get(category, 0.0)
        for start, end in self._pending.get(category, []):
            end.synchronize()
            total += float(start.elapsed_time(end))
        return total

    def total_ms(self, categories: Optional[List[str]] = None) -> float:
        self._drain()
        cats = categories if categories is not None else sorted(set(self._pending) | set(self._host_ms))
        return sum(self.ms(c) for c in cats)


class ZeROEngineBase:
    stage: int = -1

    def __init__(
        self,
        model: nn.Module,
        lr: float = 3e-4,
        betas: Tuple[float, float] = (0.9, 0.95),
        eps: float = 1e-8,
        weight_decay: float = 0.1,
        collectives: Optional[CollectiveOps] = None,
        memory_tracker=None,
        memory_trace_active: bool = False,
        memory_state_timeline: Optional[List[Dict[str, object]]] = None,
    ) -> None:
        self.model = model
        self.lr = lr
        self.betas = tuple(betas)
        self.eps = eps
        self.weight_decay = weight_decay
        self.rank, self.world_size = get_rank_world_size()
        if collectives is None:
            collectives = SendRecvCollectives() if self.world_size > 1 else LocalCollectives()
        self.collectives = collectives
        self.memory_tracker = memory_tracker
        self.memory_trace_active = memory_trace_active
        self.memory_state_timeline = memory_state_timeline
        self.step_count = 0
        first = next(p for p in model.parameters() if p.requires_grad)
        self.device = first.device
        self.param_dtype = first.dtype
        self.clock = CommClock(self.device)

    # ---------------------------------------------------------------- helpers
    @property
    def adam(self) -> AdamWConfig:
        return AdamWConfig(lr=self.lr, betas=self.betas, eps=self.eps, weight_decay=self.weight_decay)

    @property
    def uses_fused_comm(self) -> bool:
        return bool(getattr(self.collectives, "supports_fused", False)) and self.device.type == "cuda"

    def _record_memory_event(self, label: str) -> None:
        if self.memory_tracker is None or not self.memory_trace_active:
            return
        self.memory_tracker.record(label)
        if self.memory_state_timeline is not None:
            entry = {"label": label, **self.live_model_state_breakdown_mb()}
            extra = getattr(self, "_debug_memory_components_mb", None)
            if callable(extra):
                entry.update(extra())
            self.memory_state_timeline.append(entry)

    def prepare_forward(self) -> Dict[str, float]:
        return {"prepare_comm_ms": 0.0}

    def backward(self, loss: torch.Tensor) -> None:
        loss.backward()

    def step(self, max_grad_norm: float = 0.0) -> float:
        return float(self.step_with_stats(max_grad_norm=max_grad_norm)["grad_norm"])

    def _stats(self, grad_norm: torch.Tensor, t0: float, extra_categories: Dict[str, str]) -> Dict[str, float]:
        stats: Dict[str, float] = {"grad_norm": float(grad_norm)}
        comm = 0.0
        for key, category in extra_categories.items():
            ms = self.clock.ms(category)
            comm += ms
            stats[f"communication_{key}_ms"] = ms
            stats[f"communication_{key}_calls"] = float(self.clock.calls.get(category, 0))
            stats[f"communication_{key}_bytes"] = float(self.clock.bytes.get(category, 0))
        stats["comm_ms"] = comm
        stats["optim_ms"] = self.clock.ms("optimizer")
        stats["total_ms"] = (time.perf_counter() - t0) * 1000.0
        return stats

    def live_model_state_breakdown_mb(self) -> Dict[str, float]:
        return self.memory_state_breakdown_mb()

    def memory_state_breakdown_mb(self) -> Dict[str, float]:  # pragma: no cover - overridden
        raise NotImplementedError


def is_torch_or_local(collectives: CollectiveOps) -> bool:
    inner = getattr(collectives, "inner", collectives)
    return isinstance(inner, (TorchCollectives, LocalCollectives))
