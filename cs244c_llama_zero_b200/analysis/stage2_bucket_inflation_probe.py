"""How much a bucketed stage-2 reduce-scatter would inflate the bytes on the wire.

Stage 2 reduce-scatters the flat gradient buffer, and rank r keeps [r*c, (r+1)*c) with
c = ceil(N / W).  If the buffer were instead reduce-scattered in parameter-aligned buckets of about
``--grad-bucket-mb``, each bucket would have to be padded so that every rank receives its own slice
of it: the packed input is W * (largest per-rank piece), which for buckets lying inside one rank's
shard is W times the bucket.  This probe walks the model's flat parameter order, forms the buckets,
and reports logical vs packed bytes (and the buckets that touch a single shard).  It is why this
repository's stage 2 issues one reduce-scatter of the whole buffer (and the reference removed its
bucketing).  Same quantities as the reference's ``analysis/stage2_bucket_inflation_probe.py``.
"""

from __future__ import annotations

import argparse
from dataclasses import dataclass
from typing import List, Sequence, Tuple

from cs244c_llama_zero_b200.models import LlamaForCausalLM, build_config

MB = 1024.0 * 1024.0


@dataclass
class BucketRow:
    index: int
    bucket_mb: float
    packed_mb: float
    inflation: float
    shard_piece_mbs: List[float]


def bucket_ranges(numels: Sequence[int], bucket_numel: int) -> List[Tuple[int, int]]:
    """Consecutive parameter-aligned [start, end) ranges of the flat buffer, each <= bucket_numel
    unless a single parameter is larger."""
    out, start, size, off = [], 0, 0, 0
    for n in numels:
        if size and size + n > bucket_numel:
            out.append((start, off))
            start, size = off, 0
        size += n
        off += n
    if size:
        out.append((start, off))
    return out


def inflation_rows(numels: Sequence[int], world: int, bucket_numel: int, elem_bytes: int = 4) -> List[BucketRow]:
    total = sum(numels)
    chunk = -(-total // world)
    rows = []
    for i, (s, e) in enumerate(bucket_ranges(numels, bucket_numel)):
        pieces = [max(0, min(e, (r + 1) * chunk, total) - max(s, r * chunk)) for r in range(world)]
        packed = world * max(1, max(pieces))
        rows.append(BucketRow(i, (e - s) * elem_bytes / MB, packed * elem_bytes / MB, packed / (e - s),
                              [p * elem_bytes / MB for p in pieces]))
    return rows


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Quantify stage-2 reduce-scatter bucket padding inflation")
    p.add_argument("--model-size", default="small")
    p.add_argument("--vocab-size", type=int, default=8192)
    p.add_argument("--seq-len", type=int, default=128)
    p.add_argument("--world-size", type=int, default=4)
    p.add_argument("--grad-bucket-mb", type=float, default=64.0)
    p.add_argument("--print-buckets", action="store_true")
    a = p.parse_args(argv)
    import torch

    with torch.device("meta"):
        model = LlamaForCausalLM(build_config(a.model_size, vocab_size=a.vocab_size, max_seq_len=a.seq_len))
    seen, numels = set(), []
    for prm in model.parameters():
        if id(prm) not in seen:
            seen.add(id(prm))
            numels.append(prm.numel())
    rows = inflation_rows(numels, a.world_size, max(1, int(a.grad_bucket_mb * MB / 4)))
    total = sum(numels)
    logical = sum(r.bucket_mb for r in rows)
    packed = sum(r.packed_mb for r in rows)
    print(f"model={a.model_size} vocab_size={a.vocab_size} world_size={a.world_size}")
    print(f"model_mb={total * 4 / MB:.2f} rank_shard_mb={-(-total // a.world_size) * 4 / MB:.2f}")
    print(f"target_bucket_mb={a.grad_bucket_mb:.2f} bucket_count={len(rows)} "
          f"single_shard_buckets={sum(1 for r in rows if sum(x > 0 for x in r.shard_piece_mbs) == 1)}/{len(rows)}")
    print(f"logical_bucketed_mb={logical:.2f} packed_reduce_scatter_input_mb={packed:.2f} "
          f"inflation={packed / logical:.3f}x")
    if a.print_buckets:
        for r in rows:
            print(f"  bucket {r.index:3d}: {r.bucket_mb:8.2f} MB -> {r.packed_mb:8.2f} MB ({r.inflation:.2f}x) "
                  f"pieces={[round(x, 2) for x in r.shard_piece_mbs]}")


if __name__ == "__main__":
    main()
