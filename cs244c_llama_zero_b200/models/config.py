"""Model configuration and presets.

Behavioural parity with the reference's ``model/config.py:18-161``:

* ``ModelConfig`` fields, defaults and validation rules (``model/config.py:18-51``),
* ``ffn_dim`` defaulting to ``round_up(int(8*d/3), 256)`` (``model/config.py:7-15``),
* the ``tiny``/``small``/``medium`` presets (``model/config.py:78-114``),
* the analytic parameter count (``model/config.py:129-161``).

On top of those, the B200 benchmark shapes are registered as extra presets
(``baseline-tiny``, ``baseline-small``, ``baseline-1.3b``, ``baseline-7b``), and
``build_config`` accepts explicit per-field overrides.
"""

from __future__ import annotations

from dataclasses import dataclass, fields
from typing import Callable, Dict, Optional


def round_up_to_multiple(value: int, multiple_of: int) -> int:
    remainder = value % multiple_of
    return value if remainder == 0 else value + (multiple_of - remainder)


def default_ffn_dim(dim: int) -> int:
    """SwiGLU width used by LLaMA: 8/3 of the model width rounded up to 256."""
    return round_up_to_multiple(int((8 * dim) / 3), 256)


@dataclass
class ModelConfig:
    name: str
    vocab_size: int
    max_seq_len: int
    dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    ffn_dim: Optional[int] = None
    rope_theta: float = 500_000.0
    rms_norm_eps: float = 1e-5
    dropout: float = 0.0
    tie_word_embeddings: bool = True
    initializer_range: float = 0.02

    def __post_init__(self) -> None:
        if self.ffn_dim is None:
            self.ffn_dim = default_ffn_dim(self.dim)
        checks = [
            (self.dim > 0 and self.n_layers > 0, "dim and n_layers must be positive"),
            (self.n_heads > 0 and self.n_kv_heads > 0, "n_heads and n_kv_heads must be positive"),
            (self.dim % self.n_heads == 0, "dim must be divisible by n_heads"),
            (self.n_heads % self.n_kv_heads == 0, "n_heads must be divisible by n_kv_heads"),
            ((self.dim // self.n_heads) % 2 == 0, "head_dim must be even for rotary embeddings"),
            (self.vocab_size > 0 and self.max_seq_len > 0, "vocab_size and max_seq_len must be positive"),
            (self.ffn_dim > 0, "ffn_dim must be positive"),
        ]
        for ok, message in checks:
            if not ok:
                raise ValueError(message)

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return (self.n_heads + 2 * self.n_kv_heads) * self.head_dim

    def with_vocab_size(self, vocab_size: int) -> "ModelConfig":
        return ModelConfig(**{**self.to_dict(), "vocab_size": vocab_size})

    def replace(self, **overrides) -> "ModelConfig":
        return ModelConfig(**{**self.to_dict(), **overrides})

    def to_dict(self) -> Dict[str, object]:
        return {f.name: getattr(self, f.name) for f in fields(self)}


def _preset(name: str, dim: int, n_layers: int, n_heads: int, n_kv_heads: int, **extra) -> Callable[..., ModelConfig]:
    def build(vocab_size: int = 128_256, max_seq_len: int = 2048) -> ModelConfig:
        return ModelConfig(
            name=name,
            vocab_size=vocab_size,
            max_seq_len=max_seq_len,
            dim=dim,
            n_layers=n_layers,
            n_heads=n_heads,
            n_kv_heads=n_kv_heads,
            **extra,
        )

    build.__name__ = f"build_{name.replace('-', '_').replace('.', '_')}_config"
    return build


# Reference presets (model/config.py:78-114), unchanged.
build_tiny_config = _preset("tiny", dim=320, n_layers=4, n_heads=10, n_kv_heads=2)
build_small_config = _preset("small", dim=1152, n_layers=12, n_heads=18, n_kv_heads=6)
build_medium_config = _preset("medium", dim=2048, n_layers=24, n_heads=32, n_kv_heads=8)

# B200 benchmark shapes. Vocabulary 32000 is passed by the callers that use them.
build_baseline_tiny_config = _preset(
    "baseline-tiny", dim=256, n_layers=4, n_heads=4, n_kv_heads=2, ffn_dim=688, rope_theta=10_000.0,
    tie_word_embeddings=False,
)
build_baseline_small_config = _preset("baseline-small", dim=768, n_layers=12, n_heads=12, n_kv_heads=4, ffn_dim=2048)
build_baseline_1_3b_config = _preset("baseline-1.3b", dim=2048, n_layers=24, n_heads=16, n_kv_heads=8, ffn_dim=5504)
build_baseline_7b_config = _preset("baseline-7b", dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, ffn_dim=11008)

PRESETS: Dict[str, Callable[..., ModelConfig]] = {
    "tiny": build_tiny_config,
    "small": build_small_config,
    "medium": build_medium_config,
    "baseline-tiny": build_baseline_tiny_config,
    "baseline-small": build_baseline_small_config,
    "baseline-1.3b": build_baseline_1_3b_config,
    "baseline-7b": build_baseline_7b_config,
}

# Vocabulary used by the benchmark configs.
BASELINE_VOCAB_SIZE = 32_000


def build_config(size: str, vocab_size: int = 128_256, max_seq_len: int = 2048, **overrides) -> ModelConfig:
    key = size.lower().strip()
    if key not in PRESETS:
        raise ValueError(f"Unknown model size '{size}'. Expected one of {sorted(PRESETS)}")
    cfg = PRESETS[key](vocab_size=vocab_size, max_seq_len=max_seq_len)
    overrides = {k: v for k, v in overrides.items() if v is not None}
    if overrides:
        if "dim" in overrides and "ffn_dim" not in overrides:
            overrides["ffn_dim"] = None
        cfg = cfg.replace(**overrides)
    return cfg


def estimate_num_parameters(cfg: ModelConfig) -> int:
    """Analytic parameter count: embedding + blocks + final norm (+ untied head)."""
    per_block = (
        2 * cfg.dim * cfg.dim  # q and o projections
        + 2 * cfg.dim * cfg.kv_dim  # k and v projections
        + 3 * cfg.dim * cfg.ffn_dim  # gate, up, down
        + 2 * cfg.dim  # two RMSNorm weights
    )
    total = cfg.vocab_size * cfg.dim + cfg.n_layers * per_block + cfg.dim
    if not cfg.tie_word_embeddings:
        total += cfg.vocab_size * cfg.dim
    return total


def human_readable_count(num_params: int) -> str:
    for threshold, suffix in ((1_000_000_000, "B"), (1_000_000, "M"), (1_000, "K")):
        if num_params >= threshold:
            return f"{num_params / threshold:.2f}{suffix}"
    return str(num_params)
