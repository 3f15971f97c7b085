"""AdamW update and gradient-norm helpers used by every ZeRO stage.

Semantics are the reference's hand-written AdamW (``zero/stage0_ddp.py:73-88``):
decoupled weight decay applied to the fp32 master *before* the Adam step,
bias corrections from the step count, ``denom = sqrt(v)/sqrt(bc2) + eps`` and
``step = lr/bc1``; clipping multiplies the averaged gradient by
``max_norm/(norm+1e-6)`` when ``norm > max_norm`` (``zero/stage0_ddp.py:66-71``).

On CUDA tensors one fused sm_100a kernel does the whole update (read g, m, v, master;
write m, v, master and the bf16 model parameter), with the gradient scale (1/W and
the clip coefficient) read from device memory so no host synchronisation is needed.
CPU tensors (gloo test runs) use the equivalent eager formulation.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple, Union

import torch
import torch.distributed as dist

Scale = Union[float, torch.Tensor]


@dataclass
class AdamWConfig:
    lr: float = 3e-4
    betas: Tuple[float, float] = (0.9, 0.95)
    eps: float = 1e-8
    weight_decay: float = 0.1


def adamw_update_(
    master: torch.Tensor,
    exp_avg: torch.Tensor,
    exp_avg_sq: torch.Tensor,
    grad: torch.Tensor,
    cfg: AdamWConfig,
    step: int,
    grad_scale: Optional[Scale] = None,
    param_out: Optional[torch.Tensor] = None,
    dev_scalars: Optional[torch.Tensor] = None,
) -> None:
    """One AdamW step over flat fp32 state; ``grad`` is multiplied by ``grad_scale`` first.

    ``param_out`` (model dtype, same length) receives the updated master cast to its dtype.
    ``dev_scalars`` (CUDA only): the step's bias corrections on the device, from ``adam_advance``.
    """
    if master.numel() == 0:
        return
    if master.is_cuda:
        from ...ops import functional as B

        B.adamw_step(master, exp_avg, exp_avg_sq, grad, param_out, cfg.lr, cfg.betas[0], cfg.betas[1], cfg.eps,
                     cfg.weight_decay, step, grad_scale, dev_scalars)
        return
    beta1, beta2 = cfg.betas
    g = grad if grad.dtype == torch.float32 else grad.float()
    if grad_scale is not None:
        g = g * grad_scale
    exp_avg.mul_(beta1).add_(g, alpha=1.0 - beta1)
    exp_avg_sq.mul_(beta2).addcmul_(g, g, value=1.0 - beta2)
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    if cfg.weight_decay != 0.0:
        master.mul_(1.0 - cfg.lr * cfg.weight_decay)
    denom = exp_avg_sq.sqrt().div_(math.sqrt(bc2)).add_(cfg.eps)
    master.addcdiv_(exp_avg, denom, value=-cfg.lr / bc1)
    if param_out is not None:
        param_out.copy_(master)


def sum_of_squares(t: torch.Tensor) -> torch.Tensor:
    """fp32 device scalar ``sum(t^2)``."""
    if t.numel() == 0:
        return torch.zeros((), dtype=torch.float32, device=t.device)
    if t.is_cuda:
        from ...ops import functional as B

        return B.sum_squares(t)
    t32 = t.float()
    return torch.dot(t32, t32)


def clip_coefficient(norm: torch.Tensor, max_grad_norm: float) -> torch.Tensor:
    """``max/(norm+1e-6)`` where ``norm > max`` else 1, as a device scalar."""
    if max_grad_norm <= 0:
        return torch.ones((), dtype=torch.float32, device=norm.device)
    return torch.where(norm > max_grad_norm, max_grad_norm / (norm + 1e-6), torch.ones_like(norm))


def global_norm_from_local_sq(local_sq: torch.Tensor, sharded: bool, collectives=None) -> torch.Tensor:
    """sqrt of the (all-reduced when sharded) sum of squares; stays on device.  Collectives with a
    small-vector all-reduce kernel (the NVLink ones) reduce the scalar themselves; otherwise NCCL/gloo."""
    total = local_sq.reshape(1).clone()
    if sharded and dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        small = getattr(collectives, "allreduce_sum_small_", None)
        if small is None or not small(total):
            dist.all_reduce(total)
    return total.sqrt().reshape(())
