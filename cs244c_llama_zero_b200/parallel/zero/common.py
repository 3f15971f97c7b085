"""Flat-parameter bookkeeping shared by the ZeRO engines.

Public helpers keep the reference's names and semantics (``zero/common.py:1-228``):
``FlatParamMetadata``, ``ShardSpec`` / ``compute_shard_spec`` (ceil-sized chunks),
``unique_trainable_params`` (tied weights counted once), ``flatten_*`` and
``assign_flat_params`` (in-place copy when shapes match).

The engines themselves do not flatten with ``torch.cat`` on the hot path.  Instead
:class:`FlatParamSpace` re-homes every parameter as a view of one contiguous
buffer (padded to a multiple of the world size so sharded collectives work in
place), and gives each parameter a ``main_grad`` view of one contiguous fp32
gradient buffer.  The B200 kernels accumulate weight gradients straight into
``main_grad``; gradients that autograd leaves in ``p.grad`` (eager backend) are
folded in by :meth:`FlatParamSpace.fold_autograd_grads`.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Iterable, List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn

_MB = 1024.0 * 1024.0


@dataclass
class FlatParamMetadata:
    params: List[nn.Parameter]
    offsets: List[int]
    shapes: List[torch.Size]
    total_numel: int
    device: torch.device


@dataclass
class ShardSpec:
    rank: int
    world_size: int
    shard_start: int
    shard_end: int
    shard_numel: int
    chunk_size: int


def tensor_num_bytes(tensor: Optional[torch.Tensor]) -> int:
    return 0 if tensor is None else int(tensor.numel() * tensor.element_size())


def bytes_to_mb(num_bytes: int) -> float:
    return float(num_bytes) / _MB


def unique_trainable_params(params: List[nn.Parameter]) -> List[nn.Parameter]:
    seen, out = set(), []
    for p in params:
        if p.requires_grad and id(p) not in seen:
            seen.add(id(p))
            out.append(p)
    return out


def params_num_bytes(params: Iterable[nn.Parameter]) -> int:
    return sum(tensor_num_bytes(p.data) for p in unique_trainable_params(list(params)))


def grads_num_bytes(params: Iterable[nn.Parameter]) -> int:
    return sum(tensor_num_bytes(p.grad) for p in unique_trainable_params(list(params)))


def tensors_num_bytes(tensors: Iterable[Optional[torch.Tensor]]) -> int:
    return sum(tensor_num_bytes(t) for t in tensors)


def get_rank_world_size() -> Tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def build_flat_param_metadata_from_params(params: List[nn.Parameter]) -> FlatParamMetadata:
    params = unique_trainable_params(params)
    if not params:
        raise ValueError("Model has no trainable parameters")
    offsets, shapes, cursor = [], [], 0
    for p in params:
        offsets.append(cursor)
        shapes.append(torch.Size(p.shape))
        cursor += p.numel()
    return FlatParamMetadata(params=params, offsets=offsets, shapes=shapes, total_numel=cursor, device=params[0].device)


def build_flat_param_metadata(model: nn.Module) -> FlatParamMetadata:
    return build_flat_param_metadata_from_params(list(model.parameters()))


def compute_shard_spec(total_numel: int, rank: int, world_size: int) -> ShardSpec:
    chunk = max(1, math.ceil(total_numel / world_size))
    start = rank * chunk
    end = min(start + chunk, total_numel)
    return ShardSpec(rank, world_size, start, end, max(0, end - start), chunk)


def model_param_dtype(meta: FlatParamMetadata) -> torch.dtype:
    return meta.params[0].dtype


def _copy_range_into(meta: FlatParamMetadata, dst: torch.Tensor, start: int, end: int, grads: bool = False) -> None:
    """Copy elements ``[start, end)`` of the logical flat vector into ``dst``."""
    for p, off in zip(meta.params, meta.offsets):
        lo, hi = max(off, start), min(off + p.numel(), end)
        if hi <= lo:
            continue
        src = p.grad if grads else p.data
        if src is None:
            dst[lo - start : hi - start].zero_()
            continue
        dst[lo - start : hi - start].copy_(src.detach().reshape(-1)[lo - off : hi - off])


def flatten_params_fp32(meta: FlatParamMetadata) -> torch.Tensor:
    return flatten_params_dtype(meta, torch.float32)


def flatten_params_dtype(meta: FlatParamMetadata, dtype: torch.dtype) -> torch.Tensor:
    out = torch.empty(meta.total_numel, dtype=dtype, device=meta.device)
    _copy_range_into(meta, out, 0, meta.total_numel)
    return out


def flatten_param_shard_fp32(meta: FlatParamMetadata, shard_start: int, shard_end: int) -> torch.Tensor:
    return flatten_param_shard_dtype(meta, shard_start, shard_end, torch.float32)


def flatten_param_shard_dtype(meta: FlatParamMetadata, shard_start: int, shard_end: int, dtype: torch.dtype) -> torch.Tensor:
    out = torch.empty(max(0, shard_end - shard_start), dtype=dtype, device=meta.device)
    if out.numel():
        _copy_range_into(meta, out, shard_start, shard_end)
    return out


def flatten_grads_fp32(meta: FlatParamMetadata) -> torch.Tensor:
    return flatten_grads_dtype(meta, torch.float32)


def flatten_grads_dtype(meta: FlatParamMetadata, dtype: torch.dtype) -> torch.Tensor:
    out = torch.empty(meta.total_numel, dtype=dtype, device=meta.device)
    _copy_range_into(meta, out, 0, meta.total_numel, grads=True)
    return out


def assign_flat_params(meta: FlatParamMetadata, flat_params: torch.Tensor) -> None:
    """Write a flat vector back into the parameters, reusing storage when shapes match."""
    if flat_params.numel() < meta.total_numel:
        raise ValueError(f"flat_params too small: {flat_params.numel()} < {meta.total_numel}")
    for p, off, shape in zip(meta.params, meta.offsets, meta.shapes):
        chunk = flat_params[off : off + math.prod(shape)].view(shape)
        if p.data.shape == shape and p.data.dtype == chunk.dtype and p.data.device == chunk.device:
            p.data.copy_(chunk)
        elif p.data.shape == shape:
            p.data.copy_(chunk.to(dtype=p.dtype, device=p.device))
        else:
            p.data = chunk.to(dtype=p.dtype, device=p.device).clone()


def assign_flat_grads(meta: FlatParamMetadata, flat_grads: torch.Tensor) -> None:
    if flat_grads.numel() < meta.total_numel:
        raise ValueError(f"flat_grads too small: {flat_grads.numel()} < {meta.total_numel}")
    for p, off, shape in zip(meta.params, meta.offsets, meta.shapes):
        chunk = flat_grads[off : off + math.prod(shape)].view(shape).to(dtype=p.dtype, device=p.device)
        if p.grad is None or p.grad.shape != shape:
            p.grad = chunk.clone()
        else:
            p.grad.copy_(chunk)


class FlatParamSpace:
    """One contiguous parameter buffer + one contiguous fp32 gradient buffer.

    ``params``   : ``[padded_numel]`` in the model dtype; each parameter's ``.data`` is a view.
    ``grads``    : ``[padded_numel]`` fp32; each parameter's ``.main_grad`` is a view
                   (allocated only when ``with_grads``).
    ``padded_numel`` is ``chunk * world`` so rank ``r``'s shard is ``[r*chunk, (r+1)*chunk)``
    and sharded all-gathers / reduce-scatters can run in place.

    Parameters are laid out in ``model.parameters()`` order, which keeps q|k|v and
    gate|up adjacent: the B200 block kernels treat them as single fused weights.
    """

    def __init__(self, meta: FlatParamMetadata, world_size: int, rank: int, with_grads: bool = True,
                 param_dtype: Optional[torch.dtype] = None, device: Optional[torch.device] = None,
                 alignment: int = 64, allocator=None) -> None:
        self.meta = meta
        self.world_size = world_size
        self.rank = rank
        self.device = device or meta.device
        self.param_dtype = param_dtype or model_param_dtype(meta)
        self.offsets, self.numel, self.chunk = aligned_layout(meta, world_size, alignment)
        self.padded_numel = self.chunk * world_size
        # ``allocator(numel, dtype)`` lets a collectives implementation place the buffers in memory
        # its kernels can address on every rank (symmetric memory); default: ordinary device memory.
        alloc = allocator or (lambda n, dt: torch.zeros(n, dtype=dt, device=self.device))
        self.params = alloc(self.padded_numel, self.param_dtype)
        self.params.zero_()
        for p, off in zip(meta.params, self.offsets):
            self.params[off : off + p.numel()].copy_(p.data.reshape(-1))
        self.grads: Optional[torch.Tensor] = None
        self.bind_params()
        if with_grads:
            self.grads = alloc(self.padded_numel, torch.float32)
            self.grads.zero_()
            self.bind_grads()

    # -- views ------------------------------------------------------------------------
    def param_view(self, idx: int) -> torch.Tensor:
        shape = self.meta.shapes[idx]
        return self.params[self.offsets[idx] : self.offsets[idx] + shape.numel()].view(shape)

    def bind_params(self) -> None:
        for idx, p in enumerate(self.meta.params):
            p.data = self.param_view(idx)

    def bind_grads(self) -> None:
        assert self.grads is not None
        for idx, p in enumerate(self.meta.params):
            shape = self.meta.shapes[idx]
            p.main_grad = self.grads[self.offsets[idx] : self.offsets[idx] + shape.numel()].view(shape)

    def unbind_grads(self) -> None:
        for p in self.meta.params:
            if hasattr(p, "main_grad"):
                del p.main_grad

    @property
    def shard_start(self) -> int:
        return self.rank * self.chunk

    def shard(self, flat: torch.Tensor) -> torch.Tensor:
        return flat[self.shard_start : self.shard_start + self.chunk]

    def fold_autograd_grads(self) -> bool:
        """Accumulate any ``p.grad`` left by autograd into ``grads``; returns True if any."""
        assert self.grads is not None
        found = False
        for p in self.meta.params:
            if p.grad is not None:
                p.main_grad.add_(p.grad.to(torch.float32))
                p.grad = None
                found = True
        return found

    def logical_to_padded(self, flat: torch.Tensor) -> torch.Tensor:
        """Map a reference-layout flat vector (no alignment gaps) into this space's layout."""
        out = torch.zeros(self.padded_numel, dtype=flat.dtype, device=flat.device)
        for p, src_off, dst_off in zip(self.meta.params, self.meta.offsets, self.offsets):
            out[dst_off : dst_off + p.numel()].copy_(flat[src_off : src_off + p.numel()])
        return out

    def padded_to_logical(self, flat: torch.Tensor) -> torch.Tensor:
        out = torch.empty(self.meta.total_numel, dtype=flat.dtype, device=flat.device)
        for p, dst_off, src_off in zip(self.meta.params, self.meta.offsets, self.offsets):
            out[dst_off : dst_off + p.numel()].copy_(flat[src_off : src_off + p.numel()])
        return out


def _round_up(x: int, m: int) -> int:
    return ((x + m - 1) // m) * m


def aligned_layout(meta: FlatParamMetadata, world_size: int, alignment: int = 64) -> Tuple[List[int], int, int]:
    """Offsets rounded up to ``alignment`` elements, the used length, and the per-rank chunk.

    The chunk is a multiple of ``alignment`` so every rank's shard starts 128-byte aligned.
    """
    offsets: List[int] = []
    cursor = 0
    for p in meta.params:
        cursor = _round_up(cursor, alignment)
        offsets.append(cursor)
        cursor += p.numel()
    chunk = max(alignment, _round_up(math.ceil(cursor / world_size), alignment))
    return offsets, cursor, chunk
