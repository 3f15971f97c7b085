"""ZeRO stage 3: parameters, gradients and optimizer state all sharded.

Behaviour follows the reference (``zero/stage3_optimizer.py:1-576``): one handle per
parametrised module (``tok_embeddings``, ``layers.i``, ``norm``, ``lm_head``; a tied head
reuses the embedding handle); between module calls the parameters are empty
(``numel() == 0``); the model's ``_call_parametrized_module`` hook routes each call through
an autograd function that all-gathers the module's parameters, runs the module without
building a graph, and releases the parameters; its backward all-gathers again, restores the
saved RNG and autocast state, recomputes the module with gradients, and reduce-scatters the
module's gradients into an fp32 shard (averaged over ranks).  The optimizer step computes the
global norm from all shards, clips, and runs AdamW per handle.  ``summon_full_params()`` is a
re-entrant context that materialises every handle.

B200-first structure: each handle keeps a model-dtype copy of its shard (the all-gather source),
the all-gather writes straight into one aligned full-size buffer whose slices become the
parameters, and the recomputed backward accumulates weight gradients in a full-size fp32
``main_grad`` buffer that is reduce-scattered (with the 1/W scale fused in implementations
that support it) and released.
"""

from __future__ import annotations

import os
import time
from contextlib import contextmanager
from typing import Dict, Iterator, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn

from .base import ZeROEngineBase
from .common import (
    FlatParamMetadata,
    aligned_layout,
    build_flat_param_metadata_from_params,
    bytes_to_mb,
    grads_num_bytes,
    params_num_bytes,
    tensors_num_bytes,
    unique_trainable_params,
)
from ..collectives import _maybe_simulate_collective_delay
from ...profiler import nvtx
from .optim import adamw_update_, clip_coefficient, global_norm_from_local_sq, sum_of_squares


class Stage3ParamHandle:
    def __init__(self, name: str, meta: FlatParamMetadata, engine: "ZeROStage3Optimizer") -> None:
        self.name = name
        self.meta = meta
        self.engine = engine
        self.module_names: List[str] = [name]
        self.world_size = engine.world_size
        self.rank = engine.rank
        self.device = meta.device
        self.param_dtype = meta.params[0].dtype
        self.offsets, self.numel, self.chunk = aligned_layout(meta, self.world_size)
        self.padded_numel = self.chunk * self.world_size
        full = torch.zeros(self.padded_numel, dtype=torch.float32, device=self.device)
        for p, off, shape in zip(meta.params, self.offsets, meta.shapes):
            full[off : off + shape.numel()].copy_(p.data.reshape(-1))
        start = self.rank * self.chunk
        self.local_master_param_shard = full[start : start + self.chunk].clone()
        self.param_shard = self.local_master_param_shard.to(self.param_dtype)
        self.exp_avg = torch.zeros_like(self.local_master_param_shard)
        self.exp_avg_sq = torch.zeros_like(self.local_master_param_shard)
        self.grad_shard = torch.zeros_like(self.local_master_param_shard)
        self.full_params: Optional[torch.Tensor] = None
        self.materialized = True
        self._view_cache: Dict[Tuple[int, torch.dtype], List[torch.Tensor]] = {}
        self._empty = torch.empty(0, dtype=self.param_dtype, device=self.device)  # released parameters' data
        self._bind(full.to(self.param_dtype))

    # Reference-compatible shard bookkeeping.
    @property
    def shard_start(self) -> int:
        return self.rank * self.chunk

    @property
    def shard_end(self) -> int:
        return self.shard_start + self.chunk

    @property
    def full_param_bytes(self) -> int:
        return self.meta.total_numel * torch.tensor([], dtype=self.param_dtype).element_size()

    def _views(self, full: torch.Tensor, cache: bool) -> List[torch.Tensor]:
        """Per-parameter views of a full-size buffer; cached for the engine's persistent buffers."""
        key = (full.data_ptr(), full.dtype)
        views = self._view_cache.get(key) if cache else None
        if views is None:
            views = [full[off : off + shape.numel()].view(shape) for off, shape in zip(self.offsets, self.meta.shapes)]
            if cache:
                self._view_cache[key] = views
        return views

    def _bind(self, full: torch.Tensor, cache: bool = False) -> None:
        self.full_params = full
        for p, v in zip(self.meta.params, self._views(full, cache)):
            p.data = v
        self.materialized = True

    def materialize(self, phase: str) -> None:
        if self.materialized:
            return
        eng = self.engine
        if self.world_size == 1:  # one rank holds everything: the shard is the full parameter vector
            self._bind(self.param_shard, cache=True)
            return
        if eng._pull is not None and phase in ("forward", "backward"):
            full = eng._pull.materialize(self, phase)
            if full is not None:
                self._bind(full, cache=True)
                return
        staging = eng._staging_params(self.padded_numel, self.param_dtype) if phase in ("forward", "backward") else None
        full = staging if staging is not None else torch.empty(self.padded_numel, dtype=self.param_dtype,
                                                              device=self.device)
        category = {"forward": "forward_allgather", "backward": "backward_allgather"}.get(phase, "summon_allgather")
        with eng.clock.measure(category, self.full_param_bytes):
            with eng.collectives.label_scope(f"stage3.{phase}.allgather.{self.name}"):
                if self.world_size > 1:
                    eng.collectives.allgather_into(full, self.param_shard)
                else:
                    full.copy_(self.param_shard)
        self._bind(full, cache=staging is not None)

    def reshard(self) -> None:
        if not self.materialized:
            return
        if self.engine._pull is not None:
            self.engine._pull.release(self)
        empty = self._empty
        for p in self.meta.params:
            if p.grad is not None:
                p.grad = None
            p.data = empty
        self.full_params = None
        self.materialized = False

    def reset_grad(self) -> None:
        self.grad_shard.zero_()

    def begin_grad(self) -> Optional[torch.Tensor]:
        """Full-size fp32 gradient buffer bound to every parameter's ``main_grad``.  On one rank the
        gradient shard is that buffer (the reduce-scatter would be the identity): the weight-gradient
        kernels accumulate into it directly and None is returned."""
        if self.world_size == 1:
            for p, v in zip(self.meta.params, self._views(self.grad_shard, True)):
                p.main_grad = v
            return None
        buf = self.engine._staging_grads(self.padded_numel)
        persistent = buf is not None
        if buf is None:
            buf = torch.zeros(self.padded_numel, dtype=torch.float32, device=self.device)
        else:
            buf.zero_()
        for p, v in zip(self.meta.params, self._views(buf, persistent)):
            p.main_grad = v
        return buf

    def end_grad(self, buf: torch.Tensor, param_grads: Sequence[Optional[torch.Tensor]]) -> None:
        if self.device.type == "cuda":
            from ...ops import functional as B

            B.join_weight_grads(self.device)  # weight-gradient GEMMs may still run on their side stream
        for p, g in zip(self.meta.params, param_grads):
            if g is not None:
                p.main_grad.add_(g.to(torch.float32))
        for p in self.meta.params:
            if hasattr(p, "main_grad"):
                del p.main_grad
        if buf is None:  # one rank: accumulated into the gradient shard in place
            return
        eng = self.engine
        with eng.clock.measure("backward_reduce_scatter", self.full_param_bytes):
            with eng.collectives.label_scope(f"stage3.backward.reduce_scatter.{self.name}"):
                if self.world_size > 1:
                    eng.collectives.reduce_scatter_accumulate_(self.grad_shard, buf, 1.0 / self.world_size)
                else:
                    self.grad_shard.add_(buf)


class _ShardedModuleFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, runner: "_ModuleRunner", token: torch.Tensor, *args):
        del token
        ctx.runner = runner
        ctx.is_tensor = [torch.is_tensor(a) for a in args]
        ctx.wants_grad = [
            torch.is_tensor(a) and a.requires_grad and (a.is_floating_point() or a.is_complex()) for a in args
        ]
        ctx.constants = [None if torch.is_tensor(a) else a for a in args]
        ctx.save_for_backward(*[a.detach() for a in args if torch.is_tensor(a)])
        ctx.cpu_rng = torch.get_rng_state()
        dev = runner.device
        ctx.cuda_rng = torch.cuda.get_rng_state(dev) if dev.type == "cuda" else None
        if dev.type == "cuda":
            ctx.autocast = (torch.is_autocast_enabled("cuda"), torch.get_autocast_dtype("cuda"))
        elif dev.type == "cpu":
            ctx.autocast = (torch.is_autocast_enabled("cpu"), torch.get_autocast_dtype("cpu"))
        else:
            ctx.autocast = (False, torch.float32)
        eng = runner.engine
        eng._record_memory_event(f"measured_step_stage3_{runner.name}_pre_allgather_forward")
        runner.handle.materialize("forward")
        eng._record_memory_event(f"measured_step_stage3_{runner.name}_post_allgather_forward")
        with torch.no_grad():
            out = runner.module(*args)
        eng._record_memory_event(f"measured_step_stage3_{runner.name}_after_forward")
        runner.handle.reshard()
        eng._record_memory_event(f"measured_step_stage3_{runner.name}_after_forward_discard")
        return out

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        runner = ctx.runner
        eng = runner.engine
        dev = runner.device
        devices = [dev.index if dev.index is not None else torch.cuda.current_device()] if dev.type == "cuda" else []
        saved = iter(ctx.saved_tensors)
        with torch.random.fork_rng(devices=devices, enabled=True):
            torch.set_rng_state(ctx.cpu_rng)
            if ctx.cuda_rng is not None:
                torch.cuda.set_rng_state(ctx.cuda_rng, device=devices[0])
            eng._record_memory_event(f"measured_step_stage3_{runner.name}_pre_allgather_backward")
            runner.handle.materialize("backward")
            eng._record_memory_event(f"measured_step_stage3_{runner.name}_post_allgather_backward")
            grad_buf = runner.handle.begin_grad()
            rebuilt, inputs = [], []
            with torch.enable_grad():
                for is_t, wants, const in zip(ctx.is_tensor, ctx.wants_grad, ctx.constants):
                    if not is_t:
                        rebuilt.append(const)
                        continue
                    t = next(saved).detach()
                    if wants:
                        t.requires_grad_(True)
                        inputs.append(t)
                    rebuilt.append(t)
                enabled, dtype = ctx.autocast
                with torch.autocast(device_type=dev.type, dtype=dtype, enabled=enabled and dev.type in ("cpu", "cuda")):
                    out = runner.module(*rebuilt)
                params = list(runner.handle.meta.params)
                grads = torch.autograd.grad(out, inputs + params, grad_outputs=grad_output, allow_unused=True)
            input_grads, param_grads = grads[: len(inputs)], grads[len(inputs) :]
            eng._record_memory_event(f"measured_step_stage3_{runner.name}_after_layer_backward")
            runner.handle.end_grad(grad_buf, param_grads)
            del grad_buf
            runner.handle.reshard()
            eng._record_memory_event(f"measured_step_stage3_{runner.name}_after_reduce_scatter_discard")
        it = iter(input_grads)
        out_grads = [next(it) if (is_t and wants) else None for is_t, wants in zip(ctx.is_tensor, ctx.wants_grad)]
        return (None, None, *out_grads)


class _ModuleRunner:
    def __init__(self, name: str, module: nn.Module, handle: Stage3ParamHandle, engine: "ZeROStage3Optimizer") -> None:
        self.name = name
        self.module = module
        self.handle = handle
        self.engine = engine
        self.device = handle.device
        # A grad-requiring dummy input guarantees the autograd node exists even when the
        # module's real input (token ids) does not require grad.
        self.autograd_token = torch.zeros(1, dtype=torch.float32, device=self.device, requires_grad=True)

    def keeps_graph(self, args) -> bool:
        """True when this call can keep its graph instead of being recomputed in backward.

        Only the B200 kernels' autograd functions qualify: they save activations and read the
        parameters at backward time (so re-gathered parameters are seen), while eager PyTorch ops save
        the parameter tensors themselves, which are released between calls.
        """
        if self.engine.recompute or not torch.is_grad_enabled():
            return False
        m = self.module
        kind = type(m).__name__
        if kind == "TransformerBlock":
            return (getattr(m, "use_b200", False) and (len(args) < 2 or args[1] is None)
                    and not (m.training and m.cfg.dropout > 0))
        if kind == "LMHead":  # labels given: the fused LM-head + cross-entropy function
            return getattr(m, "use_b200", False) and len(args) > 1 and args[1] is not None
        return False

    def call(self, *args):
        if self.keeps_graph(args):
            return self._call_keeping_graph(args)
        return _ShardedModuleFunction.apply(self, self.autograd_token, *args)

    # backward nodes of the B200 functions that take the whole module (activations saved, parameters
    # read through the Parameter objects when the node runs)
    _KEPT_NODES = ("_BlockFnBackward", "_LMHeadCEFnBackward")

    def _call_keeping_graph(self, args):
        """Run the module in the caller's graph; hooks on its single backward node re-gather the
        parameters and bind the gradient buffer before the node runs, and reduce-scatter and release
        them after it."""
        handle, eng, name = self.handle, self.engine, self.name
        eng._record_memory_event(f"measured_step_stage3_{name}_pre_allgather_forward")
        handle.materialize("forward")
        out = self.module(*args)
        eng._record_memory_event(f"measured_step_stage3_{name}_after_forward")
        handle.reshard()
        node = out.grad_fn
        if node is None or type(node).__name__ not in self._KEPT_NODES:
            raise RuntimeError(f"stage 3: {name} was expected to end in one of {self._KEPT_NODES}, got {node}")
        state = {}

        def before(grad_outputs):
            handle.materialize("backward")
            state["buf"] = handle.begin_grad()

        def after(grad_inputs, grad_outputs):
            eng._record_memory_event(f"measured_step_stage3_{name}_after_layer_backward")
            handle.end_grad(state.pop("buf"), ())
            handle.reshard()

        node.register_prehook(before)
        node.register_hook(after)
        return out


class _PullGather:
    """Per-module parameter all-gathers as copy-engine pulls, prefetched one module ahead.

    Every rank keeps its model-dtype parameter shards in one symmetric buffer (the store, identical
    layout on every rank).  Gathering a module is one peer-to-device copy per rank into a staging
    slot: no kernel (the GEMMs keep every SM) and no barrier (ranks do not wait for one another
    module by module).  While module ``i`` computes, module ``i+1``'s copies run on a side stream; the
    order is predicted from the previous step's sequence of (module, forward/backward) gathers, and
    prefetching stops for the step at the first gather that does not match.  The streams, events
    and copies live in the native ``PullGather`` object, so a module's gather costs one call.

    Safety of the barrier-free reads: a rank rewrites its store only in the optimizer step, which
    comes after the global-norm all-reduce, and every rank joins that all-reduce only after all of
    its copies of the step have finished (the compute stream waits for the side stream first);
    the next step's reads start only after a device barrier that follows every rank's update.
    """

    CATEGORIES = ("forward_allgather", "backward_allgather")

    def __init__(self, engine: "ZeROStage3Optimizer", store: torch.Tensor, slots: List[torch.Tensor],
                 native=None) -> None:
        from ..collectives import simulated_collective_delay_s

        self.engine = engine
        self.store = store
        self.slots = slots
        self.slot_ptrs = [t.data_ptr() for t in slots]
        if native is None:  # the streams / events / copies object (a stand-in can be passed in tests)
            from ... import ops

            dev = engine.device.index if engine.device.index is not None else torch.cuda.current_device()
            native = ops.load_extension().PullGather(len(slots), len(self.CATEGORIES), dev)
        self.native = native
        coll = engine.collectives
        pacer = getattr(coll, "pacer", None)  # nvlink bandwidth mode: gathers queue on the emulated link
        if pacer is not None:
            native.set_pacer(pacer)
        elsize = store.element_size()
        self.where: Dict[int, Tuple[object, int, int]] = {}  # id(handle) -> (comm context, byte offset, chunk bytes)
        for h in engine._handle_order:
            ctx, off = coll.locate_symmetric(h.param_shard)
            self.where[id(h)] = (ctx, off, h.chunk * elsize)
        self.simulate = simulated_collective_delay_s(1 << 20, engine.world_size) > 0
        self.record_gather = getattr(coll, "record_external", None)
        self.elsize = elsize
        self.bound: List[Optional[Stage3ParamHandle]] = [None] * len(slots)
        self.pending: Dict[int, int] = {}  # id(handle) -> slot holding its prefetched parameters
        self.ring = 0
        self.plan: Optional[List[Tuple[Stage3ParamHandle, str]]] = None
        self.pos = 0
        self.trace: List[Tuple[Stage3ParamHandle, str]] = []
        self.trace_cap = 64 * (len(engine._handle_order) + 1)
        self.prefetches = 0
        engine.clock.add_source(self._times)

    def _times(self) -> Dict[str, float]:
        ms, _ = self.native.take_times()
        return {c: m for c, m in zip(self.CATEGORIES, ms) if m}

    # -- slots ---------------------------------------------------------------------------------
    def _take_slot(self) -> Optional[int]:
        s = self.ring
        if self.bound[s] is not None:
            return None
        self.ring = (s + 1) % len(self.slots)
        for key, slot in list(self.pending.items()):
            if slot == s:
                del self.pending[key]
        return s

    def _issue(self, handle: Stage3ParamHandle, slot: int, phase: str, prefetch: bool) -> None:
        cat = 0 if phase == "forward" else 1
        self.engine.clock.count(self.CATEGORIES[cat], handle.full_param_bytes)
        ctx, off, nbytes = self.where[id(handle)]
        issue = self.native.prefetch if prefetch else self.native.gather_now
        if nvtx.enabled():
            nvtx.mark(f"stage3.{phase}.{'prefetch' if prefetch else 'gather'}.{handle.name}")
        t0 = time.perf_counter()
        issue(ctx, slot, off, nbytes, self.slot_ptrs[slot], cat, True)
        if self.simulate:
            _maybe_simulate_collective_delay(nbytes, self.engine.world_size)
        if self.record_gather is not None:  # the collective-trace wrapper: one "allgather" record per gather
            self.record_gather("allgather", f"stage3.{phase}.allgather.{handle.name}", nbytes,
                       handle.padded_numel * self.elsize, (time.perf_counter() - t0) * 1000.0, str(self.store.device),
                       str(self.store.dtype).replace("torch.", ""))

    def _prefetch(self, handle: Stage3ParamHandle, phase: str) -> None:
        # A handle that is bound right now (the last forward module is the first backward one) is
        # gathered again into the other slot, which it takes over when it is next materialised.
        if id(handle) in self.pending:
            return
        s = self._take_slot()
        if s is None:
            return
        self._issue(handle, s, phase, prefetch=True)
        self.pending[id(handle)] = s
        self.prefetches += 1

    # -- module calls --------------------------------------------------------------------------
    def materialize(self, handle: Stage3ParamHandle, phase: str) -> Optional[torch.Tensor]:
        s = self.pending.pop(id(handle), None)
        if s is not None:
            self.native.acquire(s)
        else:
            s = self._take_slot()
            if s is None:
                return None
            self._issue(handle, s, phase, prefetch=False)
        self.bound[s] = handle
        self._advance(handle, phase)
        return self.slots[s][: handle.padded_numel]

    def release(self, handle: Stage3ParamHandle) -> None:
        for s, h in enumerate(self.bound):
            if h is handle:
                self.native.release(s)
                self.bound[s] = None

    def _advance(self, handle: Stage3ParamHandle, phase: str) -> None:
        if len(self.trace) < self.trace_cap:
            self.trace.append((handle, phase))
        plan = self.plan
        if plan is None:
            return
        if self.pos < len(plan) and plan[self.pos][0] is handle and plan[self.pos][1] == phase:
            self.pos += 1
            if self.pos < len(plan):
                self._prefetch(*plan[self.pos])
        else:
            self.plan = None

    # -- step boundaries -----------------------------------------------------------------------
    def begin_forward(self) -> None:
        self.trace = []
        self.pos = 0

    def before_store_write(self) -> None:
        """Every copy issued so far has finished before the compute stream goes on."""
        self.native.join()
        self.pending.clear()

    def after_store_write(self, next_plan: bool) -> None:
        """Barrier so that no rank reads a shard before its owner has rewritten it; then prefetch the
        first module of the next step."""
        self.engine.collectives.barrier()
        self.native.mark_ready()
        if next_plan:
            self.plan = list(self.trace) if 0 < len(self.trace) < self.trace_cap else None
        self.trace = []
        self.pos = 0
        if self.plan:
            self._prefetch(*self.plan[0])


class ZeROStage3Optimizer(ZeROEngineBase):
    stage = 3

    def __init__(self, model: nn.Module, recompute: bool = False, **kwargs) -> None:
        super().__init__(model, **kwargs)
        # recompute=True: every module is re-run in backward (the reference's behaviour).  False:
        # modules running on the B200 kernels keep their activations; the others still recompute.
        self.recompute = bool(recompute)
        self._pull: Optional[_PullGather] = None
        self._summon_depth = 0
        self.handles: Dict[str, Stage3ParamHandle] = {}
        self._handle_order: List[Stage3ParamHandle] = []
        self._module_runners: Dict[str, _ModuleRunner] = {}
        self._build_module_runners()
        self.model._zero3_executor = self
        self._reshard_all_params()
        # Symmetric staging for the per-module all-gather (two slots, so one module can be gathered
        # while the previous one is still in use) and for the backward reduce-scatter input.
        self._stage_params: List[torch.Tensor] = []
        self._stage_slot = 0
        self._stage_grads: Optional[torch.Tensor] = None
        alloc = getattr(self.collectives, "alloc", None)
        use_pull = False
        if alloc is not None and self.world_size > 1 and self.device.type == "cuda":
            largest = max(h.padded_numel for h in self._handle_order)
            self._stage_params = [alloc(largest, self.param_dtype) for _ in range(2)]
            self._stage_grads = alloc(largest, torch.float32)
            use_pull = (getattr(self.collectives, "supports_pull_gather", False)
                        and os.environ.get("ZB_STAGE3_PULL", "1") != "0")
        self._flat: Optional[Dict[str, torch.Tensor]] = None
        if all(h.param_dtype == self.param_dtype for h in self._handle_order):
            self._flatten_shards(alloc if use_pull else None)
            if use_pull:
                self._pull = _PullGather(self, self._flat["param_shard"], self._stage_params)
                self._pull.after_store_write(next_plan=False)

    def _flatten_shards(self, alloc) -> None:
        """Put every handle's shards (fp32 master, moments, gradient; model-dtype parameters) at the
        same offsets of one flat buffer each, so that the norm, AdamW and zeroing run once per step
        over all handles.  With ``alloc`` the parameter buffer is symmetric memory: the store that the
        peers' copy engines read in the per-module gathers."""
        total = sum(h.chunk for h in self._handle_order)
        dev = self.device
        flat = {name: torch.zeros(total, dtype=torch.float32, device=dev)
                for name in ("local_master_param_shard", "exp_avg", "exp_avg_sq", "grad_shard")}
        flat["param_shard"] = (alloc(total, self.param_dtype) if alloc is not None
                               else torch.empty(total, dtype=self.param_dtype, device=dev))
        off = 0
        for h in self._handle_order:
            for name, buf in flat.items():
                view = buf[off : off + h.chunk]
                view.copy_(getattr(h, name))
                setattr(h, name, view)
            off += h.chunk
        self._flat = flat

    def _staging_params(self, numel: int, dtype: torch.dtype) -> Optional[torch.Tensor]:
        if not self._stage_params or dtype != self._stage_params[0].dtype or self._pull is not None:
            return None
        buf = self._stage_params[self._stage_slot]
        self._stage_slot ^= 1
        return buf[:numel]

    def _staging_grads(self, numel: int) -> Optional[torch.Tensor]:
        return None if self._stage_grads is None else self._stage_grads[:numel]

    def _module_specs(self) -> List[Tuple[str, nn.Module]]:
        specs = [("tok_embeddings", self.model.tok_embeddings)]
        specs += [(f"layers.{i}", layer) for i, layer in enumerate(self.model.layers)]
        specs += [("norm", self.model.norm), ("lm_head", self.model.lm_head)]
        return specs

    def _build_module_runners(self) -> None:
        by_params: Dict[Tuple[int, ...], Stage3ParamHandle] = {}
        for name, module in self._module_specs():
            params = unique_trainable_params(list(module.parameters(recurse=True)))
            if not params:
                continue
            key = tuple(sorted(id(p) for p in params))
            handle = by_params.get(key)
            if handle is None:
                handle = Stage3ParamHandle(name, build_flat_param_metadata_from_params(params), self)
                by_params[key] = handle
                self.handles[name] = handle
                self._handle_order.append(handle)
            elif name not in handle.module_names:
                handle.module_names.append(name)
            self._module_runners[name] = _ModuleRunner(name, module, handle, self)

    def call_module(self, module_name: str, module: nn.Module, *args):
        runner = self._module_runners.get(module_name)
        if runner is None or runner.module is not module:
            return module(*args)
        return runner.call(*args)

    def _reshard_all_params(self) -> None:
        if self._summon_depth > 0:
            return
        for h in self._handle_order:
            h.reshard()

    @contextmanager
    def summon_full_params(self) -> Iterator[nn.Module]:
        self._summon_depth += 1
        if self._summon_depth == 1:
            for h in self._handle_order:
                h.materialize("summon")
        try:
            yield self.model
        finally:
            self._summon_depth -= 1
            if self._summon_depth == 0:
                self._reshard_all_params()

    def prepare_forward(self) -> Dict[str, float]:
        self._reshard_all_params()
        if self._pull is not None:
            self._pull.begin_forward()
        return {"prepare_comm_ms": 0.0}

    def zero_grad(self) -> None:
        self.clock.reset()
        if self._flat is not None:
            self._flat["grad_shard"].zero_()
        else:
            for h in self._handle_order:
                h.reset_grad()
        for p in self.model.parameters():
            p.grad = None
        self._reshard_all_params()

    def _global_norm(self) -> torch.Tensor:
        if self._flat is not None:
            total = sum_of_squares(self._flat["grad_shard"]).reshape(1)
        else:
            total = torch.zeros(1, dtype=torch.float32, device=self.device)
            for h in self._handle_order:
                total += sum_of_squares(h.grad_shard)
        # the NVLink collectives sum the scalar with their own kernel (whose device barrier orders the
        # ranks like the NCCL call it replaces); other implementations use torch.distributed
        return global_norm_from_local_sq(total, sharded=self.world_size > 1, collectives=self.collectives)

    def _update(self, max_grad_norm: float) -> torch.Tensor:
        if self._pull is not None:
            # before the global-norm all-reduce: a peer rewrites its store only after that all-reduce
            self._pull.before_store_write()
        norm = self._global_norm()
        scale = clip_coefficient(norm, max_grad_norm)
        self.step_count += 1
        with self.clock.measure("optimizer"):
            if self._flat is not None:
                f = self._flat
                adamw_update_(f["local_master_param_shard"], f["exp_avg"], f["exp_avg_sq"], f["grad_shard"], self.adam,
                              self.step_count, grad_scale=scale, param_out=f["param_shard"])
            else:
                for h in self._handle_order:
                    adamw_update_(h.local_master_param_shard, h.exp_avg, h.exp_avg_sq, h.grad_shard, self.adam,
                                  self.step_count, grad_scale=scale, param_out=h.param_shard)
        self._reshard_all_params()
        if self._pull is not None:
            self._pull.after_store_write(next_plan=True)
        return norm

    def step_async(self, max_grad_norm: float = 0.0) -> torch.Tensor:
        return self._update(max_grad_norm)

    def step_with_stats(self, max_grad_norm: float = 0.0) -> Dict[str, float]:
        t0 = time.perf_counter()
        norm = self._update(max_grad_norm)
        return self._stats(norm, t0, {
            "forward_allgather": "forward_allgather",
            "backward_allgather": "backward_allgather",
            "backward_reduce_scatter": "backward_reduce_scatter",
        })

    # -- accounting -----------------------------------------------------------------------
    def _logical_shard_bytes(self) -> int:
        return sum(h.chunk * torch.tensor([], dtype=h.param_dtype).element_size() for h in self._handle_order)

    def _optimizer_tensors(self) -> List[torch.Tensor]:
        out: List[torch.Tensor] = []
        for h in self._handle_order:
            out += [h.local_master_param_shard, h.exp_avg, h.exp_avg_sq]
        return out

    def memory_state_breakdown_mb(self) -> Dict[str, float]:
        shard = bytes_to_mb(self._logical_shard_bytes())
        opt = bytes_to_mb(tensors_num_bytes(self._optimizer_tensors()))
        return {"params_mb": shard, "grads_mb": shard, "optimizer_mb": opt, "total_mb": 2 * shard + opt}

    def live_model_state_breakdown_mb(self) -> Dict[str, float]:
        shard = self._logical_shard_bytes()
        params_mb = bytes_to_mb(shard + params_num_bytes(self.model.parameters()))
        grads_mb = bytes_to_mb(shard + grads_num_bytes(self.model.parameters()))
        opt = bytes_to_mb(tensors_num_bytes(self._optimizer_tensors()))
        return {"params_mb": params_mb, "grads_mb": grads_mb, "optimizer_mb": opt, "total_mb": params_mb + grads_mb + opt}

    def state_dict(self) -> Dict[str, object]:
        return {
            "step_count": self.step_count,
            "rank": self.rank,
            "world_size": self.world_size,
            "handles": {
                h.name: {
                    "module_names": list(h.module_names),
                    "shard_start": h.shard_start,
                    "shard_end": h.shard_end,
                    "local_master_param_shard": h.local_master_param_shard.detach().cpu(),
                    "exp_avg": h.exp_avg.detach().cpu(),
                    "exp_avg_sq": h.exp_avg_sq.detach().cpu(),
                }
                for h in self._handle_order
            },
            "hparams": {"lr": self.lr, "betas": self.betas, "eps": self.eps, "weight_decay": self.weight_decay},
        }

    def load_state_dict(self, state: Dict[str, object]) -> None:
        if self._pull is not None:
            self._pull.before_store_write()
        self.step_count = int(state["step_count"])
        saved_handles = state["handles"]
        for h in self._handle_order:
            if h.name not in saved_handles:
                raise KeyError(f"missing stage3 handle state for '{h.name}'")
            saved = saved_handles[h.name]
            h.local_master_param_shard.copy_(saved["local_master_param_shard"].to(h.device, torch.float32))
            h.exp_avg.copy_(saved["exp_avg"].to(h.device, torch.float32))
            h.exp_avg_sq.copy_(saved["exp_avg_sq"].to(h.device, torch.float32))
            h.param_shard.copy_(h.local_master_param_shard)
            h.grad_shard.zero_()
        self._reshard_all_params()
        if self._pull is not None:
            self._pull.after_store_write(next_plan=False)
