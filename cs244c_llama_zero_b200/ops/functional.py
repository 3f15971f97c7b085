"""Autograd functions of the B200 backend, built on the sm_100a kernels in ``_C``.

Weight gradients are accumulated in fp32 directly into ``param.main_grad`` when the ZeRO
engine has bound one (the flat gradient buffer); the function then returns ``None`` for that
parameter so autograd never materialises a separate ``.grad`` tensor.  Without a bound
``main_grad`` (plain model use) the gradient is returned to autograd as usual.

Every function here requires CUDA tensors and the compiled extension; there is no eager
fallback on this path.
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import load_extension

_C = None


def _ext():
    global _C
    if _C is None:
        _C = load_extension()
    return _C


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError("the b200 backend runs on CUDA tensors only; use backend='torch' on CPU")


# ------------------------------------------------------------------------------ helpers
def fused_view(params: Sequence[torch.Tensor]) -> Optional[torch.Tensor]:
    """A single [sum(rows), cols] view over row-concatenated 2-D tensors that are adjacent in memory."""
    first = params[0]
    cols = first.shape[1]
    expected = first.data_ptr()
    storage = first.untyped_storage().data_ptr()
    for p in params:
        if p.dim() != 2 or p.shape[1] != cols or not p.is_contiguous() or p.data_ptr() != expected:
            return None
        if p.untyped_storage().data_ptr() != storage:
            return None
        expected += p.numel() * p.element_size()
    rows = sum(p.shape[0] for p in params)
    return torch.as_strided(first, (rows, cols), (cols, 1))


def fused_weight(params: Sequence[torch.Tensor]) -> torch.Tensor:
    view = fused_view([p.detach() for p in params])
    if view is not None:
        return view
    return torch.cat([p.detach() for p in params], dim=0)


class _GradSink:
    """fp32 accumulation target for the gradient of one (possibly fused) weight.

    Three modes: the engine's flat gradient buffer (``param.main_grad``, written in place); a ZeRO-2
    gradient route (``param.grad_route = (route, flat offset)``: the kernels write a temporary fp32
    buffer that ``finish`` adds straight into the owning ranks' gradient shards over NVLink); or a
    temporary buffer handed back to autograd (plain model use)."""

    def __init__(self, params: Sequence[torch.nn.Parameter]) -> None:
        self.params = list(params)
        self._buffer: Optional[torch.Tensor] = None
        self.routes = [getattr(p, "grad_route", None) for p in self.params]
        if not all(r is not None for r in self.routes):
            self.routes = None
        mains = [getattr(p, "main_grad", None) for p in self.params]
        if self.routes is not None:
            self.direct = False
        elif all(m is not None for m in mains):
            self._buffer = fused_view(mains) if len(mains) > 1 else mains[0].view(self.params[0].shape)
            self.direct = self._buffer is not None
        else:
            self.direct = False

    @property
    def buffer(self) -> torch.Tensor:
        """The fp32 target the kernels accumulate into (a zeroed temporary unless written in place)."""
        if self._buffer is None:
            rows = sum(p.shape[0] for p in self.params)
            shape = (rows,) + tuple(self.params[0].shape[1:])
            self._buffer = torch.zeros(shape, dtype=torch.float32, device=self.params[0].device)
        return self._buffer

    def route_of_fused(self):
        """(route, flat offset, row length) when the sink's weights are routed and lie back to back in the
        flat space (a fused q|k|v or gate|up weight reads as one matrix there), else None."""
        if self.routes is None or self._buffer is not None or any(p.dim() != 2 for p in self.params):
            return None
        route, first = self.routes[0]
        cols = self.params[0].shape[1]
        expected = first
        for p, (r, off) in zip(self.params, self.routes):
            if r is not route or off != expected or p.shape[1] != cols:
                return None
            expected += p.numel()
        return route, first, cols

    def wgrad_routed(self, dy: torch.Tensor, x: torch.Tensor) -> bool:
        """Routed mode, one 2-D weight: ``dw = dy^T x`` straight into the owners' shards by the
        weight-gradient GEMM's own epilogue (no temporary, no push).  False if not applicable."""
        if self.routes is None or len(self.params) != 1 or self.params[0].dim() != 2 or self._buffer is not None:
            return False
        route, offset = self.routes[0]
        _ext().linear_wgrad_routed(dy, x, offset, self.params[0].shape[1], route.chunk, route.bases)
        return True

    def finish(self) -> List[Optional[torch.Tensor]]:
        """Per-parameter gradients to hand back to autograd (None when accumulated in place)."""
        if self.direct:
            return [None] * len(self.params)
        if self.routes is not None:  # into the owners' shards; nothing goes back to autograd
            if self._buffer is None:  # written by a routed kernel already
                return [None] * len(self.params)
            flat = self._buffer.reshape(-1)
            start = 0
            for p, (route, offset) in zip(self.params, self.routes):
                route.push(flat[start : start + p.numel()], offset)
                start += p.numel()
            return [None] * len(self.params)
        out: List[Optional[torch.Tensor]] = []
        row = 0
        for p in self.params:
            part = self.buffer[row : row + p.shape[0]] if self.buffer.dim() > 1 else self.buffer
            row += p.shape[0] if self.buffer.dim() > 1 else 0
            main = getattr(p, "main_grad", None)
            if main is not None:
                main.add_(part.view(p.shape))
                out.append(None)
            else:
                out.append(part.view(p.shape).to(p.dtype))
        return out


_ROPE_CACHE: Dict[Tuple, Tuple[torch.Tensor, torch.Tensor]] = {}


def rope_tables(seq_len: int, head_dim: int, theta: float, device: torch.device) -> Tuple[torch.Tensor, torch.Tensor]:
    """fp32 ``cos``/``sin`` of ``pos * theta^(-2i/hd)`` with shape ``[seq_len, head_dim/2]``."""
    key = (seq_len, head_dim, float(theta), str(device))
    if key not in _ROPE_CACHE:
        inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
        angles = torch.outer(torch.arange(seq_len, dtype=torch.float32), inv_freq)
        _ROPE_CACHE[key] = (angles.cos().to(device).contiguous(), angles.sin().to(device).contiguous())
    return _ROPE_CACHE[key]


def rope_tables_t(seq_len: int, head_dim: int, theta: float, device: torch.device) -> Tuple[torch.Tensor, torch.Tensor]:
    """The same tables frequency-major, ``[head_dim/2, seq_len]``: the layout the q|k|v GEMM's RoPE
    epilogue reads (a warp's 32 consecutive positions of one frequency are one 128-byte line)."""
    key = ("t", seq_len, head_dim, float(theta), str(device))
    if key not in _ROPE_CACHE:
        cos, sin = rope_tables(seq_len, head_dim, theta, device)
        _ROPE_CACHE[key] = (cos.t().contiguous(), sin.t().contiguous())
    return _ROPE_CACHE[key]


# ------------------------------------------------------------------------------ RMSNorm
class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: torch.Tensor, weight: torch.nn.Parameter, eps: float):
        _require_cuda(x)
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
        _ext().rmsnorm_fwd(x2, weight.detach().contiguous(), y, rstd, eps)
        ctx.save_for_backward(x2, rstd)
        ctx.weight = weight
        ctx.shape = shape
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy: torch.Tensor):
        x2, rstd = ctx.saved_tensors
        w = ctx.weight
        dy2 = dy.reshape(x2.shape).contiguous()
        dx = torch.empty_like(x2)
        sink = _GradSink([w])
        _ext().rmsnorm_bwd(dy2, x2, w.detach().contiguous(), rstd, None, dx, sink.buffer.view(-1))
        return dx.view(ctx.shape), sink.finish()[0], None


def rms_norm(x: torch.Tensor, weight: torch.nn.Parameter, eps: float) -> torch.Tensor:
    return _RMSNormFn.apply(x, weight, eps)


# ------------------------------------------------------------------------------ embedding
class _EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids: torch.Tensor, weight: torch.nn.Parameter):
        _require_cuda(ids, weight)
        flat = ids.reshape(-1).contiguous()
        out = torch.empty(flat.numel(), weight.shape[1], dtype=weight.dtype, device=weight.device)
        _ext().embedding_fwd(flat, weight.detach(), out)
        ctx.save_for_backward(flat)
        ctx.weight = weight
        return out.view(*ids.shape, weight.shape[1])

    @staticmethod
    def backward(ctx, dy: torch.Tensor):
        (flat,) = ctx.saved_tensors
        sink = _GradSink([ctx.weight])
        dy2 = dy.reshape(flat.numel(), -1).contiguous()
        fused = sink.route_of_fused()
        if fused is not None:  # routed ZeRO-2: rows added straight into the owners' shards
            route, flat0, cols = fused
            _ext().embedding_bwd_routed(flat, dy2, ctx.weight.shape[0], flat0, route.chunk, route.bases)
        else:
            _ext().embedding_bwd(flat, dy2, sink.buffer)
        return None, sink.finish()[0]


def embedding(ids: torch.Tensor, weight: torch.nn.Parameter) -> torch.Tensor:
    return _EmbeddingFn.apply(ids, weight)


# ------------------------------------------------------------------------------ attention
def attention_forward(qkv: torch.Tensor, batch: int, seq: int, heads: int, kv_heads: int, head_dim: int,
                      out: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Causal GQA attention over the fused projection ``qkv = [q | k | v]`` -> (o [T, H*hd], lse2)."""
    T = batch * seq
    if out is None:
        out = torch.empty(T, heads * head_dim, dtype=qkv.dtype, device=qkv.device)
    lse = torch.empty(batch * heads * seq, dtype=torch.float32, device=qkv.device)
    _ext().attention_fwd(qkv, heads * head_dim, (heads + kv_heads) * head_dim, out, lse, batch, seq, heads,
                         kv_heads, head_dim, 1.0 / math.sqrt(head_dim))
    return out, lse


_DQ_ACC: Dict[Tuple[int, int], torch.Tensor] = {}


def _zeroed_dq_accumulator(numel: int, device: torch.device) -> torch.Tensor:
    """One fp32 dQ accumulator per (device, size), zeroed once: the backward's dQ conversion kernel
    writes it back to zero after reading it, so no per-call fill is needed.  Backwards run one at a
    time on a device's stream, which is what makes the sharing safe."""
    key = (device.index if device.index is not None else torch.cuda.current_device(), numel)
    buf = _DQ_ACC.get(key)
    if buf is None:
        buf = torch.zeros(numel, dtype=torch.float32, device=device)
        _DQ_ACC[key] = buf
    return buf


def attention_backward(qkv: torch.Tensor, out: torch.Tensor, dout: torch.Tensor, lse: torch.Tensor, batch: int,
                       seq: int, heads: int, kv_heads: int, head_dim: int, dqkv: torch.Tensor,
                       cos: torch.Tensor, sin: torch.Tensor) -> None:
    """dqkv = gradient w.r.t. the *pre-RoPE* q|k|v projection (RoPE backward is fused)."""
    T = batch * seq
    delta = torch.empty(batch * heads * seq, dtype=torch.float32, device=qkv.device)
    dq_acc = _zeroed_dq_accumulator(T * heads * head_dim, qkv.device)
    _ext().attention_bwd(qkv, heads * head_dim, (heads + kv_heads) * head_dim, out, dout.contiguous(), lse, delta,
                         dq_acc, dqkv, cos, sin, batch, seq, heads, kv_heads, head_dim, 1.0 / math.sqrt(head_dim),
                         True)


# ------------------------------------------------------------------------------ transformer block
# Called at the end of each block's backward with the block's parameters, once all of their weight
# gradients have been issued on the current stream (a ZeRO engine starts that block's gradient
# reduction from here, overlapping it with the rest of the backward).
# ------------------------------------------------------------------------------ weight-gradient stream
# The weight-gradient GEMMs of a block's backward do not feed anything later in the backward pass,
# so they run on a side stream: their CTAs take the SMs that the input-gradient GEMMs and the
# attention kernels leave idle in their last, partial waves.  The compute stream waits for them at
# the end of the backward pass (an autograd-engine callback) or earlier through
# ``join_weight_grads()`` (the ZeRO-3 per-module reduce-scatter, grad-ready hooks).
# Opt-in (ZB_WGRAD_STREAM=1): on one B200 it measured 9.11-9.40 ms vs 9.46 ms per stage-0 step but
# 10.9-17.6 ms vs 9.91 ms per stage-2 step.  The GEMMs are persistent with a static tile schedule, so
# a CTA that starts late on an SM held by the other stream delays its kernel's last tiles.
_WGRAD_STREAMS: Dict[int, torch.cuda.Stream] = {}
_WGRAD_PENDING: Dict[int, Optional[torch.cuda.Stream]] = {}  # device -> compute stream that must join
_WGRAD_CALLBACK_QUEUED = [False]


def _wgrad_enabled() -> bool:
    import os

    return os.environ.get("ZB_WGRAD_STREAM", "0") == "1"


def join_weight_grads(device: Optional[torch.device] = None) -> None:
    """Make the current stream wait for every weight-gradient GEMM issued so far on ``device``."""
    idx = torch.cuda.current_device() if device is None or device.index is None else device.index
    main = _WGRAD_PENDING.get(idx)
    if main is not None:
        main.wait_stream(_WGRAD_STREAMS[idx])
        cur = torch.cuda.current_stream(idx)
        if cur != main:
            cur.wait_stream(_WGRAD_STREAMS[idx])
        _WGRAD_PENDING[idx] = None


def _join_all_weight_grads() -> None:
    _WGRAD_CALLBACK_QUEUED[0] = False
    for idx, main in list(_WGRAD_PENDING.items()):
        if main is not None:
            main.wait_stream(_WGRAD_STREAMS[idx])
            _WGRAD_PENDING[idx] = None


class _WgradLauncher:
    """Issues ``C.linear_wgrad`` calls of one backward node, on the side stream when enabled."""

    def __init__(self, device: torch.device) -> None:
        self.side = None
        if _wgrad_enabled():
            idx = device.index if device.index is not None else torch.cuda.current_device()
            self.idx = idx
            self.side = _WGRAD_STREAMS.get(idx)
            if self.side is None:
                self.side = _WGRAD_STREAMS[idx] = torch.cuda.Stream(device=idx)
            self.main = torch.cuda.current_stream(idx)

    def __call__(self, dy: torch.Tensor, x: torch.Tensor, out: torch.Tensor) -> None:
        C = _ext()
        if self.side is None:
            C.linear_wgrad(dy, x, out)
            return
        self.side.wait_stream(self.main)
        with torch.cuda.stream(self.side):
            C.linear_wgrad(dy, x, out)
        for t in (dy, x, out):
            t.record_stream(self.side)
        _WGRAD_PENDING[self.idx] = self.main
        if not _WGRAD_CALLBACK_QUEUED[0]:
            torch.autograd.Variable._execution_engine.queue_callback(_join_all_weight_grads)
            _WGRAD_CALLBACK_QUEUED[0] = True


def _grouped_backward_enabled() -> bool:
    import os

    return os.environ.get("ZB_GROUPED_BWD", "1") != "0"


def _dgrad_and_wgrad_sink(dy: torch.Tensor, w: torch.Tensor, x: torch.Tensor, dx: torch.Tensor, sink: "_GradSink",
                          wgrad: "_WgradLauncher") -> None:
    """``_dgrad_and_wgrad`` into a gradient sink; a routed sink gets the weight gradient straight into
    its owners' shards from the grouped launch's epilogue (no temporary buffer, no push)."""
    fused = sink.route_of_fused() if wgrad.side is None and _grouped_backward_enabled() else None
    if fused is not None:
        route, flat0, cols = fused
        _ext().linear_dgrad_wgrad_routed(dy, w, x, dx, flat0, cols, route.chunk, route.bases)
        return
    _dgrad_and_wgrad(dy, w, x, dx, sink.buffer, wgrad)


def _dgrad_and_wgrad(dy: torch.Tensor, w: torch.Tensor, x: torch.Tensor, dx: torch.Tensor, dw: torch.Tensor,
                     wgrad: "_WgradLauncher") -> None:
    """dx = dy @ w and dw += dy^T @ x: one grouped persistent GEMM launch (both problems' tiles dealt
    together), or two launches when the weight gradient runs on its own stream."""
    C = _ext()
    if wgrad.side is None and _grouped_backward_enabled():
        C.linear_dgrad_wgrad(dy, w, x, dx, dw)
        return
    C.linear_dgrad(dy, w, dx)
    wgrad(dy, x, dw)


_GRAD_READY_HOOKS: List = []


def register_grad_ready_hook(fn) -> "_HookHandle":
    _GRAD_READY_HOOKS.append(fn)
    return _HookHandle(fn)


class _HookHandle:
    def __init__(self, fn) -> None:
        self.fn = fn

    def remove(self) -> None:
        if self.fn in _GRAD_READY_HOOKS:
            _GRAD_READY_HOOKS.remove(self.fn)


class _BlockFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w_in, wq, wk, wv, wo, w_post, wg, wu, wd, meta):
        _require_cuda(x)
        cfg, params = meta
        B, S, d = x.shape
        T = B * S
        H, KV, hd, ffn = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim
        eps = cfg.rms_norm_eps
        C = _ext()
        xf = x.reshape(T, d).contiguous()
        w_qkv = fused_weight([wq, wk, wv])
        w_gu = fused_weight([wg, wu])
        cos, sin = rope_tables(S, hd, cfg.rope_theta, x.device)

        h1 = torch.empty_like(xf)
        rstd1 = torch.empty(T, dtype=torch.float32, device=x.device)
        C.rmsnorm_fwd(xf, w_in.detach(), h1, rstd1, eps)
        qkv = torch.empty(T, (H + 2 * KV) * hd, dtype=x.dtype, device=x.device)
        cos_t, sin_t = rope_tables_t(S, hd, cfg.rope_theta, x.device)
        C.qkv_rope_fwd(h1, w_qkv, qkv, cos_t, sin_t, S, hd, (H + KV) * hd)
        attn, lse = attention_forward(qkv, B, S, H, KV, hd)
        x2 = torch.empty_like(xf)
        C.linear_fwd(attn, wo.detach(), x2, xf)
        h2 = torch.empty_like(xf)
        rstd2 = torch.empty(T, dtype=torch.float32, device=x.device)
        C.rmsnorm_fwd(x2, w_post.detach(), h2, rstd2, eps)
        act = torch.empty(T, ffn, dtype=x.dtype, device=x.device)
        gu = torch.empty(T, 2 * ffn, dtype=x.dtype, device=x.device)
        C.swiglu_fwd(h2, w_gu, act, gu)
        x3 = torch.empty_like(xf)
        C.linear_fwd(act, wd.detach(), x3, x2)

        ctx.save_for_backward(xf, h1, rstd1, qkv, attn, lse, x2, h2, rstd2, gu, act)
        ctx.cfg = cfg
        ctx.params = params
        ctx.shape = (B, S, d)
        return x3.view(B, S, d)

    @staticmethod
    def backward(ctx, dy):
        xf, h1, rstd1, qkv, attn, lse, x2, h2, rstd2, gu, act = ctx.saved_tensors
        cfg = ctx.cfg
        w_in, wq, wk, wv, wo, w_post, wg, wu, wd = ctx.params
        B, S, d = ctx.shape
        T = B * S
        H, KV, hd, ffn = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim
        C = _ext()
        dy3 = dy.reshape(T, d).contiguous()
        w_qkv = fused_weight([wq, wk, wv])
        w_gu = fused_weight([wg, wu])
        cos, sin = rope_tables(S, hd, cfg.rope_theta, dy.device)

        wgrad = _WgradLauncher(dy.device)
        # MLP: down projection (SwiGLU backward fused into its data-gradient epilogue)
        dgu = torch.empty_like(gu)
        C.swiglu_dgrad(dy3, wd.detach(), gu, dgu)
        sink_d = _GradSink([wd])
        if wgrad.side is None and sink_d.wgrad_routed(dy3, act):
            pass  # the GEMM epilogue added it into the owners' shards (routed ZeRO-2)
        else:
            wgrad(dy3, act, sink_d.buffer)
        dh2 = torch.empty_like(xf)
        sink_gu = _GradSink([wg, wu])
        _dgrad_and_wgrad_sink(dgu, w_gu, h2, dh2, sink_gu, wgrad)
        del dgu
        dx2 = torch.empty_like(xf)
        sink_post = _GradSink([w_post])
        C.rmsnorm_bwd(dh2, x2, w_post.detach(), rstd2, dy3, dx2, sink_post.buffer.view(-1))
        # attention
        dattn = torch.empty_like(attn)
        sink_o = _GradSink([wo])
        _dgrad_and_wgrad_sink(dx2, wo.detach(), attn, dattn, sink_o, wgrad)
        dqkv = torch.empty_like(qkv)
        attention_backward(qkv, attn, dattn, lse, B, S, H, KV, hd, dqkv, cos, sin)
        dh1 = torch.empty_like(xf)
        sink_qkv = _GradSink([wq, wk, wv])
        _dgrad_and_wgrad_sink(dqkv, w_qkv, h1, dh1, sink_qkv, wgrad)
        dx = torch.empty_like(xf)
        sink_in = _GradSink([w_in])
        C.rmsnorm_bwd(dh1, xf, w_in.detach(), rstd1, dx2, dx, sink_in.buffer.view(-1))

        if not (sink_qkv.direct and sink_gu.direct and sink_o.direct and sink_d.direct) or _GRAD_READY_HOOKS:
            join_weight_grads(dy.device)  # the sinks' buffers / the hooks read the gradients now
        g_qkv = sink_qkv.finish()
        g_gu = sink_gu.finish()
        for hook in list(_GRAD_READY_HOOKS):  # every weight gradient of this block has been issued
            hook(ctx.params)
        return (dx.view(B, S, d), sink_in.finish()[0], g_qkv[0], g_qkv[1], g_qkv[2], sink_o.finish()[0],
                sink_post.finish()[0], g_gu[0], g_gu[1], sink_d.finish()[0], None)


def transformer_block(x: torch.Tensor, block) -> torch.Tensor:
    a, m = block.attn, block.mlp
    params = (block.input_norm.weight, a.q_proj.weight, a.k_proj.weight, a.v_proj.weight, a.o_proj.weight,
              block.post_attn_norm.weight, m.gate_proj.weight, m.up_proj.weight, m.down_proj.weight)
    return _BlockFn.apply(x, *params, (block.cfg, params))


# ------------------------------------------------------------------------------ LM head + CE
def shifted_targets(labels: torch.Tensor) -> torch.Tensor:
    """``targets[b, s] = labels[b, s+1]`` and ``-100`` at the last position of every row."""
    tgt = torch.full_like(labels, -100)
    tgt[:, :-1] = labels[:, 1:]
    return tgt.reshape(-1).contiguous()


# The training loops of this package scale every micro-batch's loss by a known factor (1 / gradient
# accumulation steps) before backward.  Inside ``loss_gradient_scale(scale)`` the LM head + cross-
# entropy computes its gradients during the forward pass already, a block of rows at a time, with that
# scale: no [tokens, vocab] logits tensor is ever allocated (one block of rows is), the weight
# gradient goes straight into the flat fp32 gradient buffer, and backward only hands back the input
# gradient.  Backward checks on the device that the scale it receives is the announced one and
# records an error (``kErrGradScale``) otherwise.
_LOSS_GRAD_SCALE: List[Optional[torch.Tensor]] = [None]
LM_HEAD_BLOCK_BYTES = 256 << 20  # logits block of the gradient-in-forward path (rows rounded to 128)


class loss_gradient_scale:
    """Context manager: losses computed inside will be back-propagated with gradient ``scale``
    (a float32 device scalar, e.g. ``1 / grad_accum_steps``).  Enables the LM head's gradient-in-
    forward path; without it the head keeps the whole logits tensor for its backward."""

    def __init__(self, scale: Optional[torch.Tensor]) -> None:
        self.scale = scale

    def __enter__(self):
        self._prev = _LOSS_GRAD_SCALE[0]
        _LOSS_GRAD_SCALE[0] = self.scale
        return self

    def __exit__(self, *exc):
        _LOSS_GRAD_SCALE[0] = self._prev
        return False


def _lm_block_rows(vocab: int, total: int) -> int:
    import os

    budget = int(os.environ.get("ZB_LM_BLOCK_MB", "0") or 0) << 20 or LM_HEAD_BLOCK_BYTES
    rows = max(128, (budget // (2 * vocab)) // 128 * 128)
    return min(rows, total)


class _LMHeadCEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: torch.Tensor, weight: torch.nn.Parameter, labels: torch.Tensor,
                scale: Optional[torch.Tensor] = None):
        _require_cuda(x, weight)
        B, S, d = x.shape
        T = B * S
        V = weight.shape[0]
        C = _ext()
        xf = x.reshape(T, d).contiguous()
        targets = shifted_targets(labels)
        ctx.weight = weight
        ctx.shape = (B, S, d)
        sink = _GradSink([weight]) if scale is not None else None
        if sink is not None and sink.direct:
            return _LMHeadCEFn._forward_with_gradients(ctx, C, xf, weight, targets, scale, sink, T, V)
        logits = torch.empty(T, V, dtype=x.dtype, device=x.device)
        C.linear_fwd(xf, weight.detach(), logits, None)
        lse = torch.empty(T, dtype=torch.float32, device=x.device)
        scratch = torch.empty(3, dtype=torch.float32, device=x.device)
        loss_sum, count, loss = scratch[0:1], scratch[1:2], scratch[2:3]
        C.cross_entropy_fwd(logits, targets, lse, loss_sum, count, loss)
        ctx.eager_grads = False
        ctx.save_for_backward(xf, logits, targets, lse, scratch)
        return loss.view(())

    @staticmethod
    def _forward_with_gradients(ctx, C, xf, weight, targets, scale, sink, T, V):
        """Blocks of rows: logits -> loss terms -> dlogits (in place, times scale / count) -> the input
        gradient rows and the weight gradient (into the flat buffer).  Only one block of logits lives."""
        dev = xf.device
        count = ((targets >= 0) & (targets < V)).sum().to(torch.float32).reshape(1)
        rows = _lm_block_rows(V, T)
        block = torch.empty(rows, V, dtype=xf.dtype, device=dev)
        lse = torch.empty(T, dtype=torch.float32, device=dev)
        dx = torch.empty_like(xf)
        n_blocks = (T + rows - 1) // rows
        scratch = torch.empty(n_blocks, 3, dtype=torch.float32, device=dev)  # per block: loss sum, count, mean
        w = weight.detach()
        launcher = _WgradLauncher(dev)
        for bi, r0 in enumerate(range(0, T, rows)):
            r1 = min(T, r0 + rows)
            logits = block[: r1 - r0]
            C.linear_fwd(xf[r0:r1], w, logits, None)
            C.cross_entropy_fwd(logits, targets[r0:r1], lse[r0:r1], scratch[bi, 0:1], scratch[bi, 1:2],
                                scratch[bi, 2:3])
            C.cross_entropy_bwd(logits, targets[r0:r1], lse[r0:r1], scale.reshape(1), count)
            _dgrad_and_wgrad_sink(logits, w, xf[r0:r1], dx[r0:r1], sink, launcher)
        loss = scratch[:, 0].sum() / count.clamp_min(1.0)[0]
        ctx.eager_grads = True
        ctx.save_for_backward(dx, scale.reshape(1))
        return loss

    @staticmethod
    def backward(ctx, grad_loss: torch.Tensor):
        C = _ext()
        if ctx.eager_grads:
            dx, scale = ctx.saved_tensors
            g = grad_loss.reshape(1).to(torch.float32).contiguous()
            C.record_if_different(g, scale, 8)
            # exact for any incoming scale (a ratio of 1 keeps the bits); the weight gradient was added
            # with the announced scale
            return (dx * (g / scale).reshape(())).view(ctx.shape), None, None, None
        xf, logits, targets, lse, scratch = ctx.saved_tensors
        g = grad_loss.reshape(1).to(torch.float32).contiguous()
        C.cross_entropy_bwd(logits, targets, lse, g, scratch[1:2])
        w = ctx.weight
        dx = torch.empty_like(xf)
        sink = _GradSink([w])
        _dgrad_and_wgrad_sink(logits, w.detach(), xf, dx, sink, _WgradLauncher(xf.device))
        if not sink.direct:
            join_weight_grads(xf.device)
        return dx.view(ctx.shape), sink.finish()[0], None, None


def lm_head_cross_entropy(x: torch.Tensor, weight: torch.nn.Parameter, labels: torch.Tensor) -> torch.Tensor:
    """Mean next-token cross-entropy of ``x @ weight^T`` against ``labels`` shifted by one."""
    scale = _LOSS_GRAD_SCALE[0]
    eager = scale is not None and torch.is_grad_enabled() and (x.requires_grad or weight.requires_grad)
    return _LMHeadCEFn.apply(x, weight, labels, scale if eager else None)


# ------------------------------------------------------------------------------ optimizer
def adamw_step(master, exp_avg, exp_avg_sq, grad, param_out, lr, beta1, beta2, eps, weight_decay, step,
               grad_scale=None, dev_scalars=None) -> None:
    """Fused AdamW; ``dev_scalars`` (from :func:`adam_advance`) replaces the host step's bias corrections."""
    scale_t, scale_c = None, 1.0
    if isinstance(grad_scale, torch.Tensor):
        scale_t = grad_scale.reshape(1).to(torch.float32)
    elif grad_scale is not None:
        scale_c = float(grad_scale)
    out = param_out.reshape(-1) if param_out is not None else None
    _ext().adamw(master.reshape(-1), exp_avg.reshape(-1), exp_avg_sq.reshape(-1), grad.reshape(-1).float()
                 if grad.dtype != torch.float32 else grad.reshape(-1), out, scale_t, scale_c, lr, beta1, beta2,
                 eps, weight_decay, step, dev_scalars)


def adam_advance(step_count: torch.Tensor, dev_scalars: torch.Tensor, lr: float, beta1: float, beta2: float) -> None:
    """Device step counter += 1 and the bias-corrected scalars of the new step (one tiny kernel)."""
    _ext().adam_advance(step_count, dev_scalars, lr, beta1, beta2)


def sum_squares(t: torch.Tensor) -> torch.Tensor:
    out = torch.empty(1, dtype=torch.float32, device=t.device)
    _ext().sum_squares(t.reshape(-1).contiguous(), out)
    return out.reshape(())


def device_errors() -> List[int]:
    """[code, where, block, count] recorded by kernels whose bounded waits expired."""
    return list(_ext().read_device_errors())


def reset_device_errors() -> None:
    _ext().reset_device_errors()
