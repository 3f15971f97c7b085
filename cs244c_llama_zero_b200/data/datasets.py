"""Token streams for training.

Parity with the reference's ``data/fineweb.py``:

* ``SyntheticPatternDataset`` - deterministic ``arange(cursor, cursor+S+1) % V`` chunks
  (``data/fineweb.py:100-122``),
* ``PackedFineWebDataset`` - tokenised text packed into ``S+1`` chunks with EOS between
  documents (``data/fineweb.py:52-97``),
* ``RankShardIterableDataset`` - strided ``idx % world == rank`` sharding
  (``data/fineweb.py:125-139``),
* ``load_llama_tokenizer`` / ``load_fineweb_stream`` (``data/fineweb.py:17-49``).

Added for the benchmark configs: ``UniformRandomTokenDataset`` (uniform int64 tokens in
``[0, V)`` from a seeded generator, one independent stream per rank).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable, Iterator, Optional

import torch
from torch.utils.data import IterableDataset


@dataclass
class TokenizerBundle:
    tokenizer: object
    vocab_size: int
    eos_token_id: int


def load_llama_tokenizer(tokenizer_name: str) -> TokenizerBundle:
    try:
        from transformers import AutoTokenizer
    except ImportError as exc:  # pragma: no cover - transformers is in the image
        raise RuntimeError("transformers is required for real-data training") from exc
    tokenizer = AutoTokenizer.from_pretrained(tokenizer_name, use_fast=True)
    if tokenizer.eos_token_id is None:
        raise ValueError(f"Tokenizer '{tokenizer_name}' has no eos_token_id")
    if tokenizer.pad_token_id is None:
        tokenizer.pad_token = tokenizer.eos_token
    return TokenizerBundle(tokenizer=tokenizer, vocab_size=tokenizer.vocab_size, eos_token_id=tokenizer.eos_token_id)


def load_fineweb_stream(subset: str, split: str = "train", shuffle_buffer: int = 10_000, seed: int = 42):
    try:
        from datasets import load_dataset
    except ImportError as exc:
        raise RuntimeError("the `datasets` package is required for FineWeb-Edu streaming") from exc
    stream = load_dataset("HuggingFaceFW/fineweb-edu", subset, split=split, streaming=True)
    return stream.shuffle(buffer_size=shuffle_buffer, seed=seed)


class PackedFineWebDataset(IterableDataset):
    """Packs a text stream into fixed ``seq_len + 1`` token chunks."""

    def __init__(
        self,
        text_iterable: Iterable,
        tokenizer,
        seq_len: int,
        eos_token_id: int,
        text_key: str = "text",
        add_eos_between_samples: bool = True,
    ) -> None:
        super().__init__()
        self.text_iterable = text_iterable
        self.tokenizer = tokenizer
        self.seq_len = seq_len
        self.eos_token_id = eos_token_id
        self.text_key = text_key
        self.add_eos_between_samples = add_eos_between_samples

    def __iter__(self) -> Iterator[torch.Tensor]:
        pending: list[int] = []
        chunk_len = self.seq_len + 1
        for row in self.text_iterable:
            text = row.get(self.text_key, "") if isinstance(row, dict) else str(row)
            if not text:
                continue
            ids = self.tokenizer.encode(text, add_special_tokens=False)
            if not ids:
                continue
            pending.extend(ids)
            if self.add_eos_between_samples:
                pending.append(self.eos_token_id)
            while len(pending) >= chunk_len:
                yield torch.tensor(pending[:chunk_len], dtype=torch.long)
                del pending[:chunk_len]


class SyntheticPatternDataset(IterableDataset):
    """Deterministic offline stream of consecutive token ids modulo the vocabulary."""

    def __init__(self, seq_len: int, vocab_size: int, num_sequences: Optional[int] = None) -> None:
        super().__init__()
        self.seq_len = seq_len
        self.vocab_size = vocab_size
        self.num_sequences = num_sequences

    def __iter__(self) -> Iterator[torch.Tensor]:
        cursor = 0
        produced = 0
        length = self.seq_len + 1
        while self.num_sequences is None or produced < self.num_sequences:
            yield torch.arange(cursor, cursor + length, dtype=torch.long) % self.vocab_size
            cursor = (cursor + length) % self.vocab_size
            produced += 1


class UniformRandomTokenDataset(IterableDataset):
    """Uniform random token ids in ``[0, vocab_size)``; reproducible from ``seed``.

    Each chunk has ``seq_len + 1`` tokens, so ``batch_from_chunk`` yields ``seq_len``
    inputs with labels equal to the inputs (the model shifts them by one).
    """

    def __init__(self, seq_len: int, vocab_size: int, seed: int = 0, num_sequences: Optional[int] = None) -> None:
        super().__init__()
        self.seq_len = seq_len
        self.vocab_size = vocab_size
        self.seed = seed
        self.num_sequences = num_sequences

    def __iter__(self) -> Iterator[torch.Tensor]:
        gen = torch.Generator().manual_seed(self.seed)
        produced = 0
        while self.num_sequences is None or produced < self.num_sequences:
            yield torch.randint(0, self.vocab_size, (self.seq_len + 1,), generator=gen, dtype=torch.long)
            produced += 1


class RankShardIterableDataset(IterableDataset):
    """Keeps every ``world_size``-th sample starting at ``rank``."""

    def __init__(self, dataset: IterableDataset, rank: int, world_size: int) -> None:
        super().__init__()
        if rank < 0 or world_size <= 0 or rank >= world_size:
            raise ValueError(f"invalid rank/world_size: rank={rank}, world_size={world_size}")
        self.dataset = dataset
        self.rank = rank
        self.world_size = world_size

    def __iter__(self):
        for idx, sample in enumerate(self.dataset):
            if idx % self.world_size == self.rank:
                yield sample
