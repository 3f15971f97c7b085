"""LLaMA-style causal LM with two execution backends.

``backend="torch"`` is the eager PyTorch formulation with the reference's exact
semantics (``model/llama.py:14-335``): RMSNorm computed in the input dtype,
half-rotation RoPE, GQA with materialised K/V repetition and SDPA, SwiGLU,
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


class RMSNorm(nn.Module, _BackendMixin):
    """``x * rsqrt(mean(x^2) + eps) * w`` (reference ``model/llama.py:14-22``)."""

    def __init__(self, hidden_size: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.use_b200:
            from ..ops import functional as B

            return B.rms_norm(x, self.weight, self.eps)
        scale = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps)
        return x * scale * self.weight


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def apply_rotary_pos_emb(
    q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor
) -> Tuple[torch.Tensor, torch.Tensor]:
    return q * cos + rotate_half(q) * sin, k * cos + rotate_half(k) * sin


def rope_inv_freq(head_dim: int, base: float) -> torch.Tensor:
    return 1.0 / (base ** (torch.arange(0, head_dim, 2).float() / head_dim))


class RotaryEmbedding(nn.Module):
    """cos/sin tables of shape ``[1, 1, S, head_dim]`` (reference ``model/llama.py:42-69``)."""

    def __init__(self, dim: int, base: float = 500_000.0) -> None:
        super().__init__()
        self.register_buffer("inv_freq", rope_inv_freq(dim, base), persistent=False)
        self.max_seq_len_cached = 0
        self.register_buffer("cos_cached", torch.empty(0), persistent=False)
        self.register_buffer("sin_cached", torch.empty(0), persistent=False)

    def _build_cache(self, seq_len: int, device: torch.device, dtype: torch.dtype) -> None:
        positions = torch.arange(seq_len, device=device, dtype=self.inv_freq.dtype)
        angles = torch.outer(positions, self.inv_freq.to(device))
        table = torch.cat((angles, angles), dim=-1)
        self.cos_cached = table.cos()[None, None].to(dtype)
        self.sin_cached = table.sin()[None, None].to(dtype)
        self.max_seq_len_cached = seq_len

    def forward(self, seq_len: int, device: torch.device, dtype: torch.dtype) -> Tuple[torch.Tensor, torch.Tensor]:
        if seq_len > self.max_seq_len_cached or self.cos_cached.device != device or self.cos_cached.dtype != dtype:
            self._build_cache(seq_len, device, dtype)
        return self.cos_cached[:, :, :seq_len], self.sin_cached[:, :, :seq_len]


class GroupedQueryAttention(nn.Module, _BackendMixin):
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

    def _repeat_kv(self, t: torch.Tensor) -> torch.Tensor:
        if self.n_kv_heads == self.n_heads:
            return t
        return t.repeat_interleave(self.n_heads // self.n_kv_heads, dim=1)

    def forward(self, x: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        bsz, seq_len, _ = x.shape
        q = self.q_proj(x).view(bsz, seq_len, self.n_heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(x).view(bsz, seq_len, self.n_kv_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(x).view(bsz, seq_len, self.n_kv_heads, self.head_dim).transpose(1, 2)
        cos, sin = self.rotary(seq_len=seq_len, device=q.device, dtype=q.dtype)
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
        k, v = self._repeat_kv(k), self._repeat_kv(v)
        p_drop = self.dropout if self.training else 0.0
        if hasattr(F, "scaled_dot_product_attention"):
            y = F.scaled_dot_product_attention(
                q, k, v, attn_mask=attention_mask, dropout_p=p_drop, is_causal=attention_mask is None
            )
        else:  # pragma: no cover - every supported torch has SDPA
            scores = torch.matmul(q, k.transpose(-2, -1)) * self.scale
            if attention_mask is None:
                future = torch.ones(seq_len, seq_len, device=x.device, dtype=torch.bool).triu(1)
                scores = scores.masked_fill(future, float("-inf"))
            else:
                scores = scores + attention_mask
            probs = F.dropout(F.softmax(scores, dim=-1), p=p_drop, training=self.training)
            y = torch.matmul(probs, v)
        y = y.transpose(1, 2).contiguous().view(bsz, seq_len, self.n_heads * self.head_dim)
        return self.o_proj(y)


class SwiGLU(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.gate_proj = nn.Linear(cfg.dim, cfg.ffn_dim, bias=False)
        self.up_proj = nn.Linear(cfg.dim, cfg.ffn_dim, bias=False)
        self.down_proj = nn.Linear(cfg.ffn_dim, cfg.dim, bias=False)
        self.dropout = nn.Dropout(cfg.dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(self.dropout(F.silu(self.gate_proj(x)) * self.up_proj(x)))


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
        if input_ids.ndim != 2:
            raise ValueError(f"input_ids should have shape [batch, seq], got {tuple(input_ids.shape)}")
        if labels is not None and labels.shape != input_ids.shape:
            raise ValueError(
                f"labels should have same shape as input_ids; got {tuple(labels.shape)} vs {tuple(input_ids.shape)}"
            )

        x = self._call_parametrized_module("tok_embeddings", self.tok_embeddings, input_ids)
        x = self.dropout(x)
        for layer_idx in range(len(self.layers)):
            if self._should_checkpoint_activations(x):
                x = activation_checkpoint(
                    lambda h, _i=layer_idx, _m=attention_mask: self._call_layer(_i, h, _m), x, use_reentrant=False
                )
            else:
                x = self._call_layer(layer_idx, x, attention_mask)
        x = self._call_parametrized_module("norm", self.norm, x)

        if self.backend == "b200" and labels is not None and not return_logits and input_ids.size(1) > 1:
            loss = self._call_parametrized_module("lm_head", self.lm_head, x, labels)
            return CausalLMOutput(logits=None, loss=loss)

        logits = None
        if labels is None or return_logits or not self._should_chunk_training_loss(input_ids):
            logits = self._call_parametrized_module("lm_head", self.lm_head, x)
        loss = None
        if labels is not None:
            if logits is not None:
                loss = self._full_cross_entropy(logits, labels)
            else:
                loss = self._chunked_cross_entropy(x, labels)
            if not return_logits:
                logits = None
        return CausalLMOutput(logits=logits, loss=loss)

    def _call_layer(self, layer_idx: int, hidden: torch.Tensor, attention_mask: Optional[torch.Tensor]) -> torch.Tensor:
        return self._call_parametrized_module(f"layers.{layer_idx}", self.layers[layer_idx], hidden, attention_mask)

    def _should_checkpoint_activations(self, hidden: torch.Tensor) -> bool:
        return (
            self.activation_checkpointing
            and self.training
            and self._zero3_executor is None
            and hidden.requires_grad
        )

    def _should_chunk_training_loss(self, input_ids: torch.Tensor) -> bool:
        return self.loss_chunk_size > 0 and input_ids.size(1) > 1 and self._zero3_executor is None

    def _full_cross_entropy(self, logits: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        if logits.size(1) <= 1:
            return logits.sum() * 0.0
        return F.cross_entropy(logits[:, :-1, :].transpose(1, 2), labels[:, 1:], ignore_index=-100)

    def _chunked_cross_entropy(self, hidden: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        seq_len = hidden.size(1)
        if seq_len <= 1:
            return hidden.sum() * 0.0
        total_loss = torch.zeros((), device=hidden.device, dtype=torch.float32)
        total_tokens = torch.zeros((), device=labels.device, dtype=torch.long)
        for start in range(0, seq_len - 1, self.loss_chunk_size):
            end = min(start + self.loss_chunk_size, seq_len - 1)
            target = labels[:, start + 1 : end + 1]
            logits = self._call_parametrized_module("lm_head", self.lm_head, hidden[:, start:end, :])
            total_loss = total_loss + F.cross_entropy(
                logits.transpose(1, 2), target, ignore_index=-100, reduction="sum"
            )
            total_tokens = total_tokens + target.ne(-100).sum()
        return total_loss / total_tokens.clamp_min(1).to(dtype=total_loss.dtype)

    def _call_parametrized_module(self, module_name: str, module: nn.Module, *args: Any) -> torch.Tensor:
        executor = self._zero3_executor
        if executor is None:
            return module(*args)
        return executor.call_module(module_name, module, *args)

    @torch.no_grad()
    def generate(
        self, input_ids: torch.Tensor, max_new_tokens: int, temperature: float = 1.0, top_k: Optional[int] = None
    ) -> torch.Tensor:
        self.eval()
        for _ in range(max_new_tokens):
            window = input_ids[:, -self.cfg.max_seq_len :]
            next_logits = self(window).logits[:, -1, :]
            if temperature <= 0:
                next_token = next_logits.argmax(dim=-1, keepdim=True)
            else:
                next_logits = next_logits / temperature
                if top_k is not None:
                    kth = torch.topk(next_logits, min(top_k, next_logits.size(-1))).values[:, [-1]]
                    next_logits[next_logits < kth] = float("-inf")
                next_token = torch.multinomial(F.softmax(next_logits, dim=-1), num_samples=1)
            input_ids = torch.cat([input_ids, next_token], dim=1)
        return input_ids
