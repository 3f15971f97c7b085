"""FLOP accounting (reference ``profiler/flops.py:15-100``).

``estimate_transformer_train_flops`` keeps the reference's formula, including its
3x training multiplier (4x for ZeRO-3, which recomputes the forward), so reported
TFLOP/s values stay comparable.  ``executed_train_flops`` gives the FLOPs the
B200 path really executes (causal attention counted once per pair, no 4x for
recompute unless asked) for roofline fractions.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass
from typing import TYPE_CHECKING, Callable, Dict, Generic, List, Optional, Tuple, TypeVar

import torch

if TYPE_CHECKING:
    from ..models.config import ModelConfig

T = TypeVar("T")


@dataclass
class FlopSnapshot:
    label: str
    total_flops: float

    def to_dict(self) -> Dict[str, float | str]:
        return {"label": self.label, "total_flops": self.total_flops}


def flops_to_tflops_per_second(total_flops: float, step_time_s: float) -> float:
    """FLOPs done in ``step_time_s`` seconds, as TFLOP/s."""
    if not (total_flops >= 0.0 and step_time_s > 0.0):
        raise ValueError("total_flops must be >= 0 and step_time_s must be > 0")
    return total_flops / (step_time_s * 1e12)


def _forward_terms(cfg: "ModelConfig", batch_size: int, seq_len: int) -> Dict[str, float]:
    tokens = float(batch_size * seq_len)
    d, ffn, vocab = float(cfg.dim), float(cfg.ffn_dim), float(cfg.vocab_size)
    kv = float(cfg.kv_dim)
    return {
        "attn_proj": 2.0 * tokens * (2.0 * d * d + 2.0 * d * kv),
        "attn_score": 2.0 * batch_size * cfg.n_heads * float(seq_len) ** 2 * cfg.head_dim,
        "mlp": 2.0 * tokens * d * ffn * 3.0,
        "pointwise": tokens * (8.0 * d + 4.0 * ffn),
        "lm_head": 2.0 * tokens * d * vocab,
    }


def estimate_transformer_train_flops(
    cfg: "ModelConfig",
    batch_size: int,
    seq_len: int,
    grad_accum_steps: int = 1,
    world_size: int = 1,
    stage: int = 0,
) -> float:
    if batch_size <= 0 or seq_len <= 0 or grad_accum_steps <= 0 or world_size <= 0:
        raise ValueError("batch_size, seq_len, grad_accum_steps, and world_size must be positive")
    t = _forward_terms(cfg, batch_size, seq_len)
    per_layer = t["attn_proj"] + 2.0 * t["attn_score"] + t["mlp"] + t["pointwise"]
    forward = cfg.n_layers * per_layer + t["lm_head"]
    multiplier = 4.0 if stage == 3 else 3.0
    return forward * multiplier * float(grad_accum_steps * world_size)


def executed_train_flops(cfg: "ModelConfig", batch_size: int, seq_len: int, recompute_forward: bool = False) -> float:
    """Tensor-core FLOPs of one training micro-step on one GPU (causal attention halved)."""
    t = _forward_terms(cfg, batch_size, seq_len)
    matmul = cfg.n_layers * (t["attn_proj"] + t["mlp"]) + t["lm_head"]
    attention = cfg.n_layers * 2.0 * t["attn_score"] * 0.5
    total = 3.0 * matmul + 3.5 * attention  # backward of attention recomputes P: 2.5x forward
    if recompute_forward:
        total += matmul + attention
    return total


FALLBACK_PEAK_BF16_TFLOPS = 1400.0  # sustained dense bf16 GEMM of a B200 under its 1 kW power cap


def peak_bf16_tflops(root: Optional[str] = None) -> Tuple[float, str]:
    """(dense bf16 TFLOP/s per GPU, where it came from) for roofline fractions.

    Order: ``ZB_PEAK_TFLOPS``; ``bf16_tflops_sustained`` of a ``MEASURED_PEAKS.json`` (a cuBLAS bf16
    GEMM timed on the same pool) in ``root`` or the repository root; else the fallback constant.
    A training step runs for seconds under the power cap, so the sustained figure is the fair one.
    """
    env = os.environ.get("ZB_PEAK_TFLOPS", "").strip()
    if env:
        return float(env), "ZB_PEAK_TFLOPS"
    base = root or os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    path = os.path.join(base, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            data = json.load(fh)
        value = float(data.get("bf16_tflops_sustained") or data["bf16_tflops"])
        if value > 0:
            return value, "measured"
    except (OSError, ValueError, KeyError, TypeError):
        pass
    return FALLBACK_PEAK_BF16_TFLOPS, "fallback"


def roofline_fraction(executed_flops: float, seconds: float, peak_tflops: float) -> Optional[float]:
    """Achieved tensor-core FLOP/s over the peak (None without a positive time or peak)."""
    if seconds <= 0 or peak_tflops <= 0:
        return None
    return executed_flops / seconds / (peak_tflops * 1e12)


class FlopTracker(Generic[T]):
    """Counts the FLOPs of one call by intercepting the ATen operators it dispatches.

    Same surface as the reference's tracker (``profiler/flops.py:68-100``): ``measure(label, fn)``
    returns ``(fn(), total FLOPs or None)`` and ``as_dicts()`` lists ``{label, total_flops}`` records.
    Here the count comes from ``torch.utils.flop_counter.FlopCounterMode`` (a dispatch-mode
    interpreter of matmul / convolution / attention FLOP formulas) instead of the profiler, so it
    needs no trace and works the same on CPU and CUDA.  The package's own fused kernels are not ATen
    operators; for the B200 backend use ``estimate_transformer_train_flops`` / ``executed_train_flops``.
    """

    def __init__(self, device: Optional[torch.device] = None) -> None:
        self.device = device
        self.snapshots: List[FlopSnapshot] = []

    def measure(self, label: str, fn: Callable[[], T]) -> Tuple[T, Optional[float]]:
        from torch.utils.flop_counter import FlopCounterMode

        counter = FlopCounterMode(display=False)
        with counter:
            result = fn()
        if self.device is not None and self.device.type == "cuda" and torch.cuda.is_available():
            torch.cuda.synchronize(self.device)
        total = float(counter.get_total_flops())
        if total <= 0.0:
            return result, None
        self.snapshots.append(FlopSnapshot(label=label, total_flops=total))
        return result, total

    def as_dicts(self) -> List[Dict[str, float | str]]:
        return [snap.to_dict() for snap in self.snapshots]
