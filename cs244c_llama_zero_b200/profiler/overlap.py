"""Overlap efficiency (reference ``profiler/overlap.py:4-22``)."""

from __future__ import annotations


def overlap_efficiency(step_ms: float, compute_ms: float, communication_ms: float) -> float:
    """Fraction of the hideable communication time that was hidden.

    0 means ``step == compute + comm``; 1 means ``step == max(compute, comm)``.
    """
    if step_ms <= 0 or compute_ms < 0 or communication_ms < 0:
        raise ValueError("step_ms must be > 0 and component times must be >= 0")
    serial = compute_ms + communication_ms
    ideal = max(compute_ms, communication_ms)
    if serial <= ideal:
        return 1.0
    return max(0.0, min(1.0, (serial - step_ms) / (serial - ideal)))
