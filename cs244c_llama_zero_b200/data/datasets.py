"""Token streams for training: synthetic, uniform-random and packed real text, plus rank sharding.

Every stream yields 1-D int64 chunks of ``seq_len + 1`` tokens (inputs and shifted labels come from
the same chunk).  Same behaviour and names as the reference's ``data/fineweb.py``:

* ``SyntheticPatternDataset``: chunk ``i`` holds ``(i*(S+1) + t) % V`` for ``t < S+1``
  (``data/fineweb.py:100-122``);
* ``PackedFineWebDataset``: documents tokenised without special tokens, optionally separated by
  EOS, cut into consecutive chunks; a trailing partial chunk is never yielded
  (``data/fineweb.py:52-97``);
* ``RankShardIterableDataset``: rank ``r`` of ``W`` keeps samples ``r, r+W, r+2W, ...``
  (``data/fineweb.py:125-139``);
* ``load_llama_tokenizer`` / ``load_fineweb_stream`` (``data/fineweb.py:17-49``).

Added here: ``UniformRandomTokenDataset`` (uniform int64 tokens in ``[0, V)`` from a seeded
generator; the benchmark configs' data).
"""

from __future__ import annotations

import itertools
from dataclasses import dataclass
from typing import Iterable, Iterator, List, Optional

import torch
from torch.utils.data import IterableDataset


@dataclass
class TokenizerBundle:
    tokenizer: object
    vocab_size: int
    eos_token_id: int


def load_llama_tokenizer(tokenizer_name: str) -> TokenizerBundle:
    """A fast Hugging Face tokenizer with an EOS id (its pad token defaults to EOS)."""
    try:
        from transformers import AutoTokenizer
    except ImportError as exc:  # pragma: no cover - transformers is in the image
        raise RuntimeError("real-text training needs the `transformers` package") from exc
    tok = AutoTokenizer.from_pretrained(tokenizer_name, use_fast=True)
    eos = tok.eos_token_id
    if eos is None:
        raise ValueError(f"Tokenizer '{tokenizer_name}' has no eos_token_id")
    if tok.pad_token_id is None:
        tok.pad_token = tok.eos_token
    return TokenizerBundle(tokenizer=tok, vocab_size=tok.vocab_size, eos_token_id=eos)


def load_fineweb_stream(subset: str, split: str = "train", shuffle_buffer: int = 10_000, seed: int = 42):
    """FineWeb-Edu ``subset`` as a streaming dataset, shuffled through a ``shuffle_buffer`` window."""
    try:
        from datasets import load_dataset
    except ImportError as exc:
        raise RuntimeError("FineWeb-Edu streaming needs the `datasets` package") from exc
    return load_dataset("HuggingFaceFW/fineweb-edu", subset, split=split, streaming=True).shuffle(
        buffer_size=shuffle_buffer, seed=seed)


def _document_text(row, key: str) -> str:
    return row.get(key, "") if isinstance(row, dict) else str(row)


class PackedFineWebDataset(IterableDataset):
    """Packs a stream of documents into ``seq_len + 1`` token chunks.

    Tokens accumulate in a flat list with a read cursor; the consumed prefix is dropped only when it
    outgrows the unread part, so packing costs O(1) amortised per token.
    """

    def __init__(self, text_iterable: Iterable, tokenizer, seq_len: int, eos_token_id: int, text_key: str = "text",
                 add_eos_between_samples: bool = True) -> None:
        super().__init__()
        self.text_iterable = text_iterable
        self.tokenizer = tokenizer
        self.seq_len = seq_len
        self.eos_token_id = eos_token_id
        self.text_key = text_key
        self.add_eos_between_samples = add_eos_between_samples

    def _token_runs(self) -> Iterator[List[int]]:
        sep = [self.eos_token_id] if self.add_eos_between_samples else []
        for row in self.text_iterable:
            text = _document_text(row, self.text_key)
            ids = self.tokenizer.encode(text, add_special_tokens=False) if text else None
            if ids:
                yield list(ids) + sep

    def __iter__(self) -> Iterator[torch.Tensor]:
        width = self.seq_len + 1
        buf: List[int] = []
        head = 0
        for run in self._token_runs():
            buf.extend(run)
            while len(buf) - head >= width:
                yield torch.tensor(buf[head:head + width], dtype=torch.long)
                head += width
            if head > len(buf) - head:
                buf, head = buf[head:], 0


class SyntheticPatternDataset(IterableDataset):
    """Deterministic offline stream: consecutive token ids modulo the vocabulary, chunk after chunk."""

    def __init__(self, seq_len: int, vocab_size: int, num_sequences: Optional[int] = None) -> None:
        super().__init__()
        self.seq_len = seq_len
        self.vocab_size = vocab_size
        self.num_sequences = num_sequences

    def __iter__(self) -> Iterator[torch.Tensor]:
        width = self.seq_len + 1
        offsets = torch.arange(width, dtype=torch.long)
        indices = itertools.count() if self.num_sequences is None else range(self.num_sequences)
        for i in indices:
            start = (i * width) % self.vocab_size
            yield (offsets + start) % self.vocab_size


class UniformRandomTokenDataset(IterableDataset):
    """Uniform random token ids in ``[0, vocab_size)``; reproducible from ``seed``.

    Each chunk has ``seq_len + 1`` tokens, so a batch built from it has ``seq_len`` inputs with the
    labels equal to the inputs (the model shifts them by one).
    """

    def __init__(self, seq_len: int, vocab_size: int, seed: int = 0, num_sequences: Optional[int] = None) -> None:
        super().__init__()
        self.seq_len = seq_len
        self.vocab_size = vocab_size
        self.seed = seed
        self.num_sequences = num_sequences

    def __iter__(self) -> Iterator[torch.Tensor]:
        gen = torch.Generator().manual_seed(self.seed)
        count = itertools.count() if self.num_sequences is None else range(self.num_sequences)
        for _ in count:
            yield torch.randint(0, self.vocab_size, (self.seq_len + 1,), generator=gen, dtype=torch.long)


class RankShardIterableDataset(IterableDataset):
    """Rank ``rank`` of ``world_size`` sees every ``world_size``-th sample, starting at its own index."""

    def __init__(self, dataset: IterableDataset, rank: int, world_size: int) -> None:
        super().__init__()
        if not (world_size > 0 and 0 <= rank < world_size):
            raise ValueError(f"invalid rank/world_size: rank={rank}, world_size={world_size}")
        self.dataset = dataset
        self.rank = rank
        self.world_size = world_size

    def __iter__(self):
        return itertools.islice(iter(self.dataset), self.rank, None, self.world_size)
