from .datasets import (
    PackedFineWebDataset,
    RankShardIterableDataset,
    SyntheticPatternDataset,
    TokenizerBundle,
    UniformRandomTokenDataset,
    load_fineweb_stream,
    load_llama_tokenizer,
)

__all__ = [
    "PackedFineWebDataset",
    "RankShardIterableDataset",
    "SyntheticPatternDataset",
    "TokenizerBundle",
    "UniformRandomTokenDataset",
    "load_fineweb_stream",
    "load_llama_tokenizer",
]
