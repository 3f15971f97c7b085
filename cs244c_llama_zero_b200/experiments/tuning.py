"""Micro-batch tuning: find the largest per-GPU micro-batch that fits, and predict good first guesses.

Two pieces are shared by the fit-to-memory bandwidth sweep and the stage-3 GPU-count sweep:

* :func:`search_max_batch_size` - a boundary search over the micro-batch size.  It probes an initial
  guess, walks geometrically (up while the probe fits, down while it does not) until the boundary is
  bracketed, then bisects on the ``multiple`` grid.  Every size is evaluated at most once.  The probe
  order is part of the observable behaviour (each probe is a multi-minute training launch), and it
  matches the reference's ``experiments/run_fit_memory_bandwidth.py:_select_max_batch_size``
  (reference tests ``tests/test_fit_memory_bandwidth.py``).
* :func:`predict_initial_batch_size` - seeds the search for the next GPU count from what earlier GPU
  counts measured: a linear peak-memory model ``peak(b, n) = slope * b + c(n)`` with
  ``c(n) = c_inf + c_shard / n`` (ZeRO-3 shards the model state over ``n`` ranks), falling back to
  scaling the previous selection by the GPU-count ratio.  Same predictor kinds and payload keys as
  the reference's ``experiments/run_stage3_scaling_sweep.py:_predict_initial_batch_size``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from pathlib import Path
from statistics import median
from typing import Callable, Dict, List, Optional, Sequence, Tuple

MEMORY_METRICS = (
    "peak_cuda_allocated_mb",
    "peak_cuda_reserved_mb",
    "peak_cuda_max_allocated_mb",
    "peak_cuda_max_reserved_mb",
)


@dataclass
class TuningTrial:
    """One probe of the search: a short training launch at ``batch_size`` and whether it fit."""

    batch_size: int
    fits: bool
    peak_memory_mb: Optional[float]
    return_code: int
    reason: str
    case_id: str
    log_path: str
    profile_path: str
    mean_tokens_per_s: Optional[float]


# ------------------------------------------------------------------------------ grid helpers
def round_up(value: int, multiple: int) -> int:
    """Smallest multiple of ``multiple`` >= ``value`` (never below one step)."""
    if multiple <= 1:
        return max(1, value)
    return max(multiple, -(-value // multiple) * multiple)


def round_down(value: int, multiple: int) -> int:
    """Largest multiple of ``multiple`` <= ``value`` (never below one step)."""
    if multiple <= 1:
        return max(1, value)
    return max(multiple, (value // multiple) * multiple)


def initial_guess(min_batch_size: int, max_batch_size: int, multiple: int, initial_batch_size: int) -> int:
    """The first probe: the configured guess (or the interval midpoint), clamped and snapped to the grid."""
    multiple = max(1, multiple)
    guess = initial_batch_size if initial_batch_size > 0 else (min_batch_size + max_batch_size) // 2
    guess = round_down(min(max_batch_size, max(min_batch_size, guess)), multiple)
    return guess if guess >= min_batch_size else round_up(min_batch_size, multiple)


def _grow(current: int, multiple: int, factor: float, ceiling: int) -> int:
    step = max(current + multiple, math.ceil(current * max(factor, 1.1)))
    return min(ceiling, round_up(step, multiple))


def _shrink(current: int, multiple: int, factor: float, floor_size: int) -> int:
    smaller = round_down(max(floor_size, math.floor(current / max(factor, 1.1))), multiple)
    if smaller >= current:
        smaller = current - multiple
    return max(round_up(floor_size, multiple), smaller)


# ------------------------------------------------------------------------------ boundary search
def search_max_batch_size(min_batch_size: int, max_batch_size: int, batch_size_multiple: int,
                          growth_factor: float, initial_batch_size: int,
                          evaluator: Callable[[int], TuningTrial]) -> Tuple[TuningTrial, List[TuningTrial]]:
    """Largest fitting micro-batch on the ``batch_size_multiple`` grid in ``[min, max]``.

    Returns ``(best_trial, all_trials_sorted_by_batch)``; raises ``RuntimeError`` when even the
    smallest size fails.
    """
    if min_batch_size < 1:
        raise ValueError("min_batch_size must be >= 1")
    if max_batch_size < min_batch_size:
        raise ValueError("max_batch_size must be >= min_batch_size")
    step = max(1, batch_size_multiple)
    ceiling = round_down(max_batch_size, step)
    seen: Dict[int, TuningTrial] = {}

    def probe(size: int) -> TuningTrial:
        if size not in seen:
            seen[size] = evaluator(size)
        return seen[size]

    def ordered() -> List[TuningTrial]:
        return sorted(seen.values(), key=lambda t: t.batch_size)

    size = initial_guess(min_batch_size, max_batch_size, step, initial_batch_size)
    trial = probe(size)
    best: Optional[TuningTrial] = None
    fail_at: Optional[int] = None
    if trial.fits:
        # bracket from below: grow until a probe fails or the ceiling is reached
        best = trial
        while fail_at is None:
            nxt = _grow(size, step, growth_factor, ceiling) if size < ceiling else size
            if nxt == size:
                return best, ordered()
            size = nxt
            trial = probe(size)
            if trial.fits:
                best = trial
            else:
                fail_at = size
    else:
        # bracket from above: shrink until a probe fits
        fail_at = size
        while best is None:
            if size <= min_batch_size:
                raise RuntimeError(f"no fitting batch size found: minimum tried microbatch {size} failed "
                                   f"({trial.reason})")
            size = _shrink(size, step, growth_factor, min_batch_size)
            trial = probe(size)
            if trial.fits:
                best = trial
            else:
                fail_at = size

    lo, hi = best.batch_size, fail_at
    while hi - lo > step:
        mid = round_down((lo + hi) // 2, step)
        mid = lo + step if mid <= lo else mid
        if mid >= hi:
            break
        trial = probe(mid)
        if trial.fits:
            best, lo = trial, mid
        else:
            hi = mid
    return best, ordered()


# ------------------------------------------------------------------------------ trial classification
def classify_result(result, *, fit_mode: str, memory_metric: str,
                    memory_budget_mb: Optional[float]) -> Tuple[bool, Optional[float], str]:
    """(fits, peak_mb, reason) of one harness ``CaseResult``.

    ``oom_boundary``: any clean exit fits.  ``memory_budget``: a clean exit fits only when its
    ``memory_metric`` stays within ``memory_budget_mb``.  A failed launch whose log mentions
    "out of memory" is reported as ``oom``.
    """
    if result.return_code != 0:
        log = Path(result.log_path)
        if log.exists() and "out of memory" in log.read_text(errors="replace").lower():
            return False, None, "oom"
        return False, None, f"return_code_{result.return_code}"
    raw = getattr(result, memory_metric)
    peak = None if raw is None else float(raw)
    if fit_mode == "oom_boundary":
        return True, peak, "ok"
    if peak is None:
        return False, None, "missing_memory_metric"
    if memory_budget_mb is None:
        raise ValueError("memory_budget_mb is required when fit_mode=memory_budget")
    return (False, peak, "over_budget") if peak > memory_budget_mb else (True, peak, "ok")


def trial_from_result(result, *, fit_mode: str, memory_metric: str,
                      memory_budget_mb: Optional[float]) -> TuningTrial:
    fits, peak, reason = classify_result(result, fit_mode=fit_mode, memory_metric=memory_metric,
                                         memory_budget_mb=memory_budget_mb)
    return TuningTrial(batch_size=int(result.config["batch_size"]), fits=fits, peak_memory_mb=peak,
                       return_code=int(result.return_code), reason=reason, case_id=result.case_id,
                       log_path=result.log_path, profile_path=result.profile_path,
                       mean_tokens_per_s=result.mean_tokens_per_s)


def memory_probe_extra_args(base: str, warmup_steps: int) -> str:
    """train_zero flags that make a probe measure the peak of one post-warm-up step."""
    extra = f"--measure-memory-step --memory-warmup-steps {warmup_steps}"
    return f"{base.strip()} {extra}" if base.strip() else extra


def detect_gpu_total_memory_mb(nproc_per_node: int) -> float:
    """Smallest total memory (MiB) over the first ``nproc_per_node`` visible GPUs."""
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("fit-to-memory tuning requires CUDA")
    visible = torch.cuda.device_count()
    if visible < nproc_per_node:
        raise RuntimeError(f"requested nproc_per_node={nproc_per_node}, but only {visible} CUDA device(s) are visible")
    return min(torch.cuda.get_device_properties(i).total_memory / 2**20 for i in range(nproc_per_node))


# ------------------------------------------------------------------------------ memory model
def least_squares_line(points: Sequence[Tuple[float, float]]) -> Optional[Tuple[float, float]]:
    """(slope, intercept) of the ordinary least-squares line, or None when under-determined."""
    if len(points) < 2:
        return None
    n = float(len(points))
    mx = sum(x for x, _ in points) / n
    my = sum(y for _, y in points) / n
    sxx = sum((x - mx) ** 2 for x, _ in points)
    if sxx <= 0.0:
        return None
    slope = sum((x - mx) * (y - my) for x, y in points) / sxx
    return slope, my - slope * mx


def _measured(trials: Sequence[TuningTrial]) -> List[TuningTrial]:
    return [t for t in trials if t.fits and t.peak_memory_mb is not None]


def activation_mb_per_sample(history: Dict[int, List[TuningTrial]]) -> Optional[float]:
    """Median over GPU counts of the fitted d(peak MB)/d(batch); only positive slopes count."""
    slopes = []
    for trials in history.values():
        by_batch = {int(t.batch_size): float(t.peak_memory_mb) for t in _measured(trials)}
        line = least_squares_line([(float(b), m) for b, m in sorted(by_batch.items())])
        if line is not None and line[0] > 0.0:
            slopes.append(line[0])
    return float(median(slopes)) if slopes else None


def constant_memory_mb(history: Dict[int, List[TuningTrial]], slope: float) -> Dict[int, float]:
    """Per GPU count: mean of (peak - slope * batch) over measured probes (the batch-independent part)."""
    out = {}
    for gpus, trials in history.items():
        rest = [float(t.peak_memory_mb) - slope * float(t.batch_size) for t in _measured(trials)]
        if rest:
            out[int(gpus)] = sum(rest) / len(rest)
    return out


def predict_from_memory_model(*, gpu_count: int, batch_size_multiple: int, min_batch_size: int,
                              max_batch_size: int, previous_selected_batch_size: Optional[int],
                              previous_gpu_count: Optional[int], selected_trials_by_gpu_count: Dict[int, TuningTrial],
                              trial_history_by_gpu_count: Dict[int, List[TuningTrial]]
                              ) -> Tuple[Optional[int], Dict[str, object]]:
    slope = activation_mb_per_sample(trial_history_by_gpu_count)
    if slope is None or slope <= 0.0:
        return None, {"kind": "insufficient_memory_slope"}
    consts = constant_memory_mb(trial_history_by_gpu_count, slope)
    if not consts:
        return None, {"kind": "insufficient_constant_terms", "activation_slope_mb_per_sample": slope}
    chosen = [t for t in selected_trials_by_gpu_count.values()
              if t.fits and t.peak_memory_mb is not None and int(t.batch_size) > 0]
    if not chosen:
        return None, {"kind": "insufficient_budget", "activation_slope_mb_per_sample": slope}
    budget = max(float(t.peak_memory_mb) for t in chosen)
    if len(consts) >= 2:
        fit = least_squares_line([(1.0 / n, c) for n, c in sorted(consts.items())])
        if fit is None:
            return None, {"kind": "degenerate_constant_fit", "activation_slope_mb_per_sample": slope}
        shard_mb, fixed_mb = fit
        const_pred = fixed_mb + shard_mb / float(gpu_count)
        kind = "memory_model"
    else:
        n0, c0 = sorted(consts.items())[0]
        const_pred = c0 * float(n0) / float(gpu_count)
        kind = "single_point_shard_scale"
    room = budget - const_pred
    if room <= 0.0:
        return None, {"kind": "non_positive_available_memory", "activation_slope_mb_per_sample": slope,
                      "budget_mb": budget, "constant_prediction_mb": const_pred}
    raw = int(math.floor(room / slope))
    pred = max(min_batch_size, round_down(raw, batch_size_multiple))
    if previous_selected_batch_size is not None:
        pred = max(int(previous_selected_batch_size), pred)
    pred = max(min_batch_size, min(max_batch_size, pred))
    return pred, {"kind": kind, "activation_slope_mb_per_sample": slope,
                  "constant_by_gpu_count_mb": {str(k): v for k, v in sorted(consts.items())},
                  "budget_mb": budget, "constant_prediction_mb": const_pred, "raw_prediction": raw,
                  "previous_selected_batch_size": previous_selected_batch_size,
                  "previous_gpu_count": previous_gpu_count}


def predict_initial_batch_size(args, *, gpu_count: int, previous_selected_batch_size: Optional[int],
                               previous_gpu_count: Optional[int],
                               selected_trials_by_gpu_count: Dict[int, TuningTrial],
                               trial_history_by_gpu_count: Dict[int, List[TuningTrial]]
                               ) -> Tuple[int, Dict[str, object]]:
    """First probe for ``gpu_count``: memory model (needs two GPU counts), else shard ratio, else config.

    ``args`` supplies ``min_batch_size``, ``max_batch_size``, ``batch_size_multiple``,
    ``initial_batch_size`` and ``tuning_strategy`` (``predictive`` or ``exponential``).
    """
    lo, hi, step = int(args.min_batch_size), int(args.max_batch_size), int(args.batch_size_multiple)
    if str(args.tuning_strategy) == "predictive":
        info: Dict[str, object] = {"kind": "insufficient_history_for_memory_model"}
        if len(selected_trials_by_gpu_count) >= 2 and len(trial_history_by_gpu_count) >= 2:
            pred, info = predict_from_memory_model(
                gpu_count=gpu_count, batch_size_multiple=step, min_batch_size=lo, max_batch_size=hi,
                previous_selected_batch_size=previous_selected_batch_size, previous_gpu_count=previous_gpu_count,
                selected_trials_by_gpu_count=selected_trials_by_gpu_count,
                trial_history_by_gpu_count=trial_history_by_gpu_count)
            if pred is not None:
                return pred, info
        if previous_selected_batch_size is not None and previous_gpu_count:
            scaled = int(math.floor(previous_selected_batch_size * gpu_count / float(previous_gpu_count)))
            scaled = round_down(max(previous_selected_batch_size, scaled), step)
            scaled = max(lo, min(hi, scaled))
            info = dict(info)
            info.update(kind="shard_ratio", raw_prediction=scaled,
                        previous_selected_batch_size=previous_selected_batch_size,
                        previous_gpu_count=previous_gpu_count)
            return scaled, info
    guess = int(args.initial_batch_size)
    if previous_selected_batch_size is not None:
        guess = max(guess, int(previous_selected_batch_size))
    return guess, {"kind": "configured_initial_guess", "raw_prediction": guess}
