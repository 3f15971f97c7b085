"""LLaMA-style causal LM with two execution backends.

``backend="torch"`` is the eager PyTorch formulation with the reference's exact
semantics (``model/llama.py:14-335``): RMSNorm computed in the input dtype,
half-rotation RoPE, GQA with the key/value heads expanded for SDPA, SwiGLU,
pre-norm blocks, tied LM head, chunked LM-head cross-entropy, per-block
activation checkpointing and the ``_call_parametrized_module`` hook through which
a ZeRO-3 executor intercepts every parametrised module.  It runs anywhere and is
the numerical oracle for the B200 path.

``backend="b200"`` routes the same modules through the hand-written sm_100a
kernels in :mod:`cs244c_llama_zero_b200.ops`: one fused autograd function per
transformer block (fused QKV GEMM with RoPE epilogue, GQA flash attention without
K/V repetition, O-projection GEMM with residual epilogue, gate|up GEMM with SwiGLU
epilogue, down GEMM with residual epilogue, RMSNorm kernels) and a fused
LM-head + cross-entropy.  Module names, parameter names and initialisation
order are the reference's, so state dicts are interchangeable.
"""

from __future__ import annotations

from dataclasses import dataclass
from functools import partial
from typing import Any, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint as activation_checkpoint

from .config import ModelConfig

BACKENDS = ("torch", "b200")


class _BackendMixin:
    """Every module carries the backend name so ZeRO-3 runners can call it directly."""

    backend: str = "torch"

    @property
    def use_b200(self) -> bool:
        return self.backend == "b200"


def _rms_normalize(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """Eager RMSNorm in the input's dtype: each row divided by its root mean square, then scaled."""
    inv_rms = (x * x).mean(dim=-1, keepdim=True).add(eps).rsqrt()
    return x * inv_rms * weight


class RMSNorm(nn.Module, _BackendMixin):
    """Root-mean-square normalisation with a learned per-channel gain (reference ``model/llama.py:14-22``)."""

    def __init__(self, hidden_size: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self.use_b200:
            return _rms_normalize(x, self.weight, self.eps)
        from ..ops import functional as B

        return B.rms_norm(x, self.weight, self.eps)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """(x1, x2) -> (-x2, x1) over the two halves of the last dimension."""
    lo, hi = x.chunk(2, dim=-1)
    return torch.cat((hi.neg(), lo), dim=-1)


def _rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    return x * cos + rotate_half(x) * sin


def apply_rotary_pos_emb(
    q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Half-rotation RoPE of queries and keys with full-width ``cos``/``sin`` tables."""
    return _rotate(q, cos, sin), _rotate(k, cos, sin)


def rope_inv_freq(head_dim: int, base: float) -> torch.Tensor:
    """Rotation frequency of each channel pair: base^(-2i/head_dim)."""
    exponents = torch.arange(0, head_dim, 2).float() / head_dim
    return 1.0 / (base ** exponents)


class RotaryEmbedding(nn.Module):
    """cos/sin tables ``[1, 1, S, head_dim]`` for positions ``0..S-1`` (reference ``model/llama.py:42-69``).

    The tables are kept for the longest length seen so far (and rebuilt on a new device or dtype);
    shorter requests are prefix views.
    """

    def __init__(self, dim: int, base: float = 500_000.0) -> None:
        super().__init__()
        self.register_buffer("inv_freq", rope_inv_freq(dim, base), persistent=False)
        self.max_seq_len_cached = 0
        self.register_buffer("cos_cached", torch.empty(0), persistent=False)
        self.register_buffer("sin_cached", torch.empty(0), persistent=False)

    def _tables_valid(self, seq_len: int, device: torch.device, dtype: torch.dtype) -> bool:
        return seq_len <= self.max_seq_len_cached and self.cos_cached.device == device and self.cos_cached.dtype == dtype

    def _build_cache(self, seq_len: int, device: torch.device, dtype: torch.dtype) -> None:
        freq = self.inv_freq.to(device)
        pos = torch.arange(seq_len, device=device, dtype=freq.dtype)
        angle = (pos[:, None] * freq[None, :]).repeat(1, 2)  # both halves of a pair share an angle
        self.cos_cached = angle.cos().to(dtype).view(1, 1, seq_len, -1)
        self.sin_cached = angle.sin().to(dtype).view(1, 1, seq_len, -1)
        self.max_seq_len_cached = seq_len

    def forward(self, seq_len: int, device: torch.device, dtype: torch.dtype) -> Tuple[torch.Tensor, torch.Tensor]:
        if not self._tables_valid(seq_len, device, dtype):
            self._build_cache(seq_len, device, dtype)
        return self.cos_cached[..., :seq_len, :], self.sin_cached[..., :seq_len, :]


class GroupedQueryAttention(nn.Module, _BackendMixin):
    """Causal grouped-query attention: ``n_heads`` query heads share ``n_kv_heads`` key/value heads.

    Eager path: SDPA on [B, heads, S, hd] with the key/value heads expanded to the query heads
    (reference ``model/llama.py:72-133``); an explicit mask replaces the causal one when given.
    """

    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.n_heads = cfg.n_heads
        self.n_kv_heads = cfg.n_kv_heads
        self.head_dim = cfg.head_dim
        self.dropout = cfg.dropout
        self.scale = self.head_dim ** -0.5
        self.q_proj = nn.Linear(cfg.dim, cfg.n_heads * self.head_dim, bias=False)
        self.k_proj = nn.Linear(cfg.dim, cfg.n_kv_heads * self.head_dim, bias=False)
        self.v_proj = nn.Linear(cfg.dim, cfg.n_kv_heads * self.head_dim, bias=False)
        self.o_proj = nn.Linear(cfg.n_heads * self.head_dim, cfg.dim, bias=False)
        self.rotary = RotaryEmbedding(dim=self.head_dim, base=cfg.rope_theta)

    def _split_heads(self, t: torch.Tensor, heads: int) -> torch.Tensor:
        b, s, _ = t.shape
        return t.reshape(b, s, heads, self.head_dim).permute(0, 2, 1, 3)

    def _expand_kv(self, t: torch.Tensor) -> torch.Tensor:
        group = self.n_heads // self.n_kv_heads
        return t if group == 1 else torch.repeat_interleave(t, group, dim=1)

    def _attend(self, q, k, v, mask: Optional[torch.Tensor]) -> torch.Tensor:
        p_drop = self.dropout if self.training else 0.0
        return F.scaled_dot_product_attention(q, k, v, attn_mask=mask, dropout_p=p_drop, is_causal=mask is None)

    def forward(self, x: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        b, s, _ = x.shape
        q = self._split_heads(self.q_proj(x), self.n_heads)
        k = self._split_heads(self.k_proj(x), self.n_kv_heads)
        v = self._split_heads(self.v_proj(x), self.n_kv_heads)
        cos, sin = self.rotary(seq_len=s, device=q.device, dtype=q.dtype)
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
        y = self._attend(q, self._expand_kv(k), self._expand_kv(v), attention_mask)
        return self.o_proj(y.permute(0, 2, 1, 3).reshape(b, s, self.n_heads * self.head_dim))


class SwiGLU(nn.Module):
    """``down(dropout(silu(gate(x)) * up(x)))``."""

    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.gate_proj = nn.Linear(cfg.dim, cfg.ffn_dim, bias=False)
        self.up_proj = nn.Linear(cfg.dim, cfg.ffn_dim, bias=False)
        self.down_proj = nn.Linear(cfg.ffn_dim, cfg.dim, bias=False)
        self.dropout = nn.Dropout(cfg.dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        hidden = F.silu(self.gate_proj(x)) * self.up_proj(x)
        return self.down_proj(self.dropout(hidden))


class TransformerBlock(nn.Module, _BackendMixin):
    """Pre-norm block: ``x += attn(norm1(x)); x += mlp(norm2(x))``."""

    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.input_norm = RMSNorm(cfg.dim, eps=cfg.rms_norm_eps)
        self.attn = GroupedQueryAttention(cfg)
        self.post_attn_norm = RMSNorm(cfg.dim, eps=cfg.rms_norm_eps)
        self.mlp = SwiGLU(cfg)

    def forward(self, x: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.use_b200 and attention_mask is None and not (self.training and self.cfg.dropout > 0):
            from ..ops import functional as B

            return B.transformer_block(x, self)
        x = x + self.attn(self.input_norm(x), attention_mask=attention_mask)
        return x + self.mlp(self.post_attn_norm(x))


class TokenEmbedding(nn.Embedding, _BackendMixin):
    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        if self.use_b200:
            from ..ops import functional as B

            return B.embedding(input_ids, self.weight)
        return super().forward(input_ids)


class LMHead(nn.Linear, _BackendMixin):
    """Vocabulary projection.  With labels on the B200 backend it returns the fused
    LM-head + shifted cross-entropy loss (mean over non-ignored targets) instead of logits."""

    def forward(self, x: torch.Tensor, labels: Optional[torch.Tensor] = None) -> torch.Tensor:
        if labels is not None:
            from ..ops import functional as B

            return B.lm_head_cross_entropy(x, self.weight, labels)
        return super().forward(x)


@dataclass
class CausalLMOutput:
    logits: Optional[torch.Tensor]
    loss: Optional[torch.Tensor] = None


class LlamaForCausalLM(nn.Module):
    def __init__(self, cfg: ModelConfig, backend: str = "torch") -> None:
        super().__init__()
        self.cfg = cfg
        self.tok_embeddings = TokenEmbedding(cfg.vocab_size, cfg.dim)
        self.dropout = nn.Dropout(cfg.dropout)
        self.layers = nn.ModuleList([TransformerBlock(cfg) for _ in range(cfg.n_layers)])
        self.norm = RMSNorm(cfg.dim, eps=cfg.rms_norm_eps)
        self.lm_head = LMHead(cfg.dim, cfg.vocab_size, bias=False)
        if cfg.tie_word_embeddings:
            self.lm_head.weight = self.tok_embeddings.weight
        self.apply(self._init_weights)
        self._zero3_executor = None
        self.loss_chunk_size = 0
        self.activation_checkpointing = False
        self.backend = "torch"
        self.set_backend(backend)

    # ------------------------------------------------------------------ setup
    def _init_weights(self, module: nn.Module) -> None:
        if isinstance(module, (nn.Linear, nn.Embedding)):
            nn.init.normal_(module.weight, mean=0.0, std=self.cfg.initializer_range)
            if isinstance(module, nn.Linear) and module.bias is not None:
                nn.init.zeros_(module.bias)

    def set_backend(self, backend: str) -> None:
        if backend not in BACKENDS:
            raise ValueError(f"unknown backend {backend!r}; expected one of {BACKENDS}")
        if backend == "b200":
            from .. import ops

            ops.require_extension()
        self.backend = backend
        for module in self.modules():
            if isinstance(module, _BackendMixin):
                module.backend = backend

    def set_loss_chunk_size(self, chunk_size: int) -> None:
        if chunk_size < 0:
            raise ValueError(f"loss chunk size must be non-negative, got {chunk_size}")
        self.loss_chunk_size = int(chunk_size)

    def set_activation_checkpointing(self, enabled: bool) -> None:
        self.activation_checkpointing = bool(enabled)

    # ---------------------------------------------------------------- forward
    def forward(
        self,
        input_ids: torch.Tensor,
        labels: Optional[torch.Tensor] = None,
        attention_mask: Optional[torch.Tensor] = None,
        return_logits: bool = True,
    ) -> CausalLMOutput:
        """Logits and/or the next-token loss of ``input_ids`` [B, S].

        ``labels`` has the inputs' shape; position t is scored against ``labels[:, t + 1]`` (the
        shift happens here) and ``-100`` targets are ignored.  With ``return_logits=False`` the
        training loss avoids materialising logits: the B200 backend runs its fused LM-head +
        cross-entropy, the eager backend scores ``loss_chunk_size`` positions at a time.
        """
        self._check_shapes(input_ids, labels)
        hidden = self._trunk(input_ids, attention_mask)
        if labels is None:
            return CausalLMOutput(logits=self._head(hidden))
        fused = self.backend == "b200" and not return_logits and input_ids.size(1) > 1
        if fused:
            return CausalLMOutput(logits=None, loss=self._head(hidden, labels))
        if not return_logits and self._should_chunk_training_loss(input_ids):
            return CausalLMOutput(logits=None, loss=self._chunked_cross_entropy(hidden, labels))
        logits = self._head(hidden)
        loss = self._full_cross_entropy(logits, labels)
        return CausalLMOutput(logits=logits if return_logits else None, loss=loss)

    @staticmethod
    def _check_shapes(input_ids: torch.Tensor, labels: Optional[torch.Tensor]) -> None:
        if input_ids.ndim != 2:
            raise ValueError(f"input_ids should have shape [batch, seq], got {tuple(input_ids.shape)}")
        if labels is not None and labels.shape != input_ids.shape:
            raise ValueError(
                f"labels should have same shape as input_ids; got {tuple(labels.shape)} vs {tuple(input_ids.shape)}"
            )

    def _trunk(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor]) -> torch.Tensor:
        """Embedding -> blocks (optionally checkpointed) -> final norm."""
        h = self.dropout(self._call_parametrized_module("tok_embeddings", self.tok_embeddings, input_ids))
        for i in range(len(self.layers)):
            if self._should_checkpoint_activations(h):
                run = partial(self._call_layer, i, attention_mask=attention_mask)
                h = activation_checkpoint(run, h, use_reentrant=False)
            else:
                h = self._call_layer(i, h, attention_mask)
        return self._call_parametrized_module("norm", self.norm, h)

    def _head(self, hidden: torch.Tensor, labels: Optional[torch.Tensor] = None) -> torch.Tensor:
        if labels is None:
            return self._call_parametrized_module("lm_head", self.lm_head, hidden)
        return self._call_parametrized_module("lm_head", self.lm_head, hidden, labels)

    def _call_layer(self, layer_idx: int, hidden: torch.Tensor, attention_mask: Optional[torch.Tensor]) -> torch.Tensor:
        return self._call_parametrized_module(f"layers.{layer_idx}", self.layers[layer_idx], hidden, attention_mask)

    def _should_checkpoint_activations(self, hidden: torch.Tensor) -> bool:
        return bool(self.activation_checkpointing and self.training and hidden.requires_grad
                    and self._zero3_executor is None)

    def _should_chunk_training_loss(self, input_ids: torch.Tensor) -> bool:
        return self.loss_chunk_size > 0 and input_ids.size(1) > 1 and self._zero3_executor is None

    def _full_cross_entropy(self, logits: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        if logits.size(1) < 2:
            return logits.sum() * 0.0  # nothing to predict; keeps the graph connected
        pred = logits[:, :-1].reshape(-1, logits.size(-1))
        return F.cross_entropy(pred, labels[:, 1:].reshape(-1), ignore_index=-100)

    def _chunked_cross_entropy(self, hidden: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        """Mean next-token loss computed ``loss_chunk_size`` positions at a time: the LM head runs
        on one slice of positions, its summed loss is added, and the slice's logits are freed."""
        if hidden.size(1) < 2:
            return hidden.sum() * 0.0
        inputs = hidden[:, :-1].split(self.loss_chunk_size, dim=1)
        targets = labels[:, 1:].split(self.loss_chunk_size, dim=1)
        loss_sum = torch.zeros((), device=hidden.device, dtype=torch.float32)
        for h, t in zip(inputs, targets):
            logits = self._head(h)
            loss_sum = loss_sum + F.cross_entropy(logits.reshape(-1, logits.size(-1)), t.reshape(-1),
                                                  ignore_index=-100, reduction="sum")
        n_scored = labels[:, 1:].ne(-100).sum().clamp_min(1)
        return loss_sum / n_scored.to(loss_sum.dtype)

    def _call_parametrized_module(self, module_name: str, module: nn.Module, *args: Any) -> torch.Tensor:
        """Every parametrised call goes through here so a ZeRO-3 executor can gather around it."""
        if self._zero3_executor is not None:
            return self._zero3_executor.call_module(module_name, module, *args)
        return module(*args)

    @torch.no_grad()
    def generate(
        self, input_ids: torch.Tensor, max_new_tokens: int, temperature: float = 1.0, top_k: Optional[int] = None
    ) -> torch.Tensor:
        """Autoregressive sampling over a sliding ``max_seq_len`` window; ``temperature <= 0`` is greedy."""
        self.eval()
        out = input_ids
        for _ in range(max_new_tokens):
            last = self(out[:, -self.cfg.max_seq_len:]).logits[:, -1]
            out = torch.cat([out, self._pick_next(last, temperature, top_k)], dim=1)
        return out

    @staticmethod
    def _pick_next(logits: torch.Tensor, temperature: float, top_k: Optional[int]) -> torch.Tensor:
        if temperature <= 0:
            return logits.argmax(dim=-1, keepdim=True)
        scaled = logits / temperature
        if top_k is not None:
            k = min(top_k, scaled.size(-1))
            floor = scaled.topk(k, dim=-1).values[..., -1:]
            scaled = scaled.masked_fill(scaled < floor, float("-inf"))
        return torch.multinomial(scaled.softmax(dim=-1), num_samples=1)
