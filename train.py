"""Single-process LLaMA training (reference ``train.py``: same flags, step line and checkpoints).

Uses ``torch.optim.AdamW`` (and a GradScaler for fp16) like the reference.  On CUDA with bf16 the
model runs on the sm_100a kernel backend (``--backend auto``); fp32/fp16 and CPU runs use the eager
backend.  ``make_data_loader`` / ``batch_from_chunk`` are shared with ``train_zero.py``.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import random
import time
from contextlib import nullcontext
from dataclasses import dataclass
from typing import Dict, Iterator, Tuple

import torch
from torch.utils.data import DataLoader

from cs244c_llama_zero_b200.data import (
    PackedFineWebDataset,
    RankShardIterableDataset,
    SyntheticPatternDataset,
    UniformRandomTokenDataset,
    load_fineweb_stream,
    load_llama_tokenizer,
)
from cs244c_llama_zero_b200.models import PRESETS, LlamaForCausalLM, build_config, estimate_num_parameters, human_readable_count


@dataclass
class TrainBatch:
    input_ids: torch.Tensor
    labels: torch.Tensor


def add_model_args(parser: argparse.ArgumentParser, default_size: str = "tiny") -> None:
    parser.add_argument("--model-size", type=str, default=default_size, choices=sorted(PRESETS))
    parser.add_argument("--dim", type=int, default=None)
    parser.add_argument("--n-layers", type=int, default=None)
    parser.add_argument("--n-heads", type=int, default=None)
    parser.add_argument("--n-kv-heads", type=int, default=None)
    parser.add_argument("--ffn-dim", type=int, default=None)
    parser.add_argument("--rope-theta", type=float, default=None)
    parser.add_argument("--untie-embeddings", action="store_true")
    parser.add_argument("--backend", choices=["auto", "b200", "torch"], default="auto",
                        help="b200: sm_100a kernels (CUDA, bf16); torch: eager PyTorch; auto: b200 when possible")


def add_data_args(parser: argparse.ArgumentParser, default_mode: str) -> None:
    parser.add_argument("--data-mode", type=str, default=default_mode, choices=["fineweb", "synthetic", "random"])
    parser.add_argument("--tokenizer-name", type=str, default="meta-llama/Llama-3.1-8B")
    parser.add_argument("--fineweb-subset", type=str, default="sample-10BT")
    parser.add_argument("--fineweb-split", type=str, default="train")
    parser.add_argument("--shuffle-buffer", type=int, default=10_000)
    parser.add_argument("--synthetic-vocab-size", type=int, default=8_192)
    parser.add_argument("--allow-synthetic-fallback", action="store_true")


def parse_args(argv=None) -> argparse.Namespace:
    parser = argparse.ArgumentParser(description="Single-process LLaMA training baseline")
    add_model_args(parser)
    parser.add_argument("--seq-len", type=int, default=512)
    parser.add_argument("--batch-size", type=int, default=2)
    parser.add_argument("--grad-accum-steps", type=int, default=8)
    parser.add_argument("--max-steps", type=int, default=200)
    parser.add_argument("--learning-rate", type=float, default=3e-4)
    parser.add_argument("--weight-decay", type=float, default=0.1)
    parser.add_argument("--beta1", type=float, default=0.9)
    parser.add_argument("--beta2", type=float, default=0.95)
    parser.add_argument("--max-grad-norm", type=float, default=1.0)
    parser.add_argument("--dtype", type=str, default="bfloat16", choices=["float32", "float16", "bfloat16"])
    parser.add_argument("--device", type=str, default="cuda")
    parser.add_argument("--seed", type=int, default=1337)
    parser.add_argument("--loss-chunk-size", type=int, default=128)
    parser.add_argument("--activation-checkpointing", action="store_true")
    add_data_args(parser, default_mode="fineweb")
    parser.add_argument("--log-interval", type=int, default=10)
    parser.add_argument("--checkpoint-interval", type=int, default=100)
    parser.add_argument("--save-dir", type=str, default="checkpoints")
    return parser.parse_args(argv)


def set_seed(seed: int) -> None:
    random.seed(seed)
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)


def choose_device(device_arg: str) -> torch.device:
    if device_arg == "cuda" and not torch.cuda.is_available():
        print("[warn] CUDA requested but unavailable; falling back to CPU")
        return torch.device("cpu")
    return torch.device(device_arg)


def model_config_from_args(args: argparse.Namespace, vocab_size: int):
    return build_config(
        args.model_size, vocab_size=vocab_size, max_seq_len=args.seq_len, dim=args.dim, n_layers=args.n_layers,
        n_heads=args.n_heads, n_kv_heads=args.n_kv_heads, ffn_dim=args.ffn_dim, rope_theta=args.rope_theta,
        tie_word_embeddings=(False if getattr(args, "untie_embeddings", False) else None),
    )


def resolve_backend(args: argparse.Namespace, device: torch.device, param_dtype: torch.dtype) -> str:
    if args.backend != "auto":
        return args.backend
    if device.type == "cuda" and param_dtype == torch.bfloat16:
        from cs244c_llama_zero_b200 import ops

        if ops.extension_available():
            return "b200"
    return "torch"


def make_data_loader(args: argparse.Namespace, vocab_size_for_model: int, rank: int = 0,
                     world_size: int = 1) -> Tuple[DataLoader, int, Dict[str, str]]:
    """Token stream of ``seq_len + 1`` chunks, strided over ranks (reference ``train.py:95-136``)."""
    metadata: Dict[str, str] = {}
    if args.data_mode == "fineweb":
        bundle = load_llama_tokenizer(args.tokenizer_name)
        stream = load_fineweb_stream(args.fineweb_subset, args.fineweb_split, args.shuffle_buffer, args.seed)
        dataset = PackedFineWebDataset(stream, bundle.tokenizer, args.seq_len, bundle.eos_token_id)
        vocab_size = bundle.vocab_size
        metadata["tokenizer"] = args.tokenizer_name
        metadata["dataset"] = f"HuggingFaceFW/fineweb-edu:{args.fineweb_subset}/{args.fineweb_split}"
    elif args.data_mode == "random":
        vocab_size = vocab_size_for_model
        dataset = UniformRandomTokenDataset(args.seq_len, vocab_size, seed=args.seed + 7919 * rank)
        metadata["tokenizer"] = "synthetic"
        metadata["dataset"] = "uniform_random"
    else:
        vocab_size = vocab_size_for_model
        dataset = SyntheticPatternDataset(seq_len=args.seq_len, vocab_size=vocab_size)
        metadata["tokenizer"] = "synthetic"
        metadata["dataset"] = "synthetic_pattern"
    if world_size > 1 and args.data_mode != "random":
        dataset = RankShardIterableDataset(dataset, rank=rank, world_size=world_size)
        metadata["data_sharding"] = f"rank_stride:{rank}/{world_size}"
    loader = DataLoader(dataset, batch_size=args.batch_size, num_workers=0, pin_memory=torch.cuda.is_available())
    return loader, vocab_size, metadata


def batch_from_chunk(chunk: torch.Tensor) -> TrainBatch:
    """``[B, S+1]`` chunk -> inputs ``[B, S]`` with labels == inputs (the model shifts them)."""
    input_ids = chunk[:, :-1].contiguous()
    return TrainBatch(input_ids=input_ids, labels=input_ids.clone())


def autocast_context(device: torch.device, dtype_name: str):
    if device.type != "cuda" or dtype_name == "float32":
        return nullcontext()
    return torch.autocast(device_type="cuda", dtype=torch.float16 if dtype_name == "float16" else torch.bfloat16)


def model_param_dtype(device: torch.device, dtype_name: str) -> torch.dtype:
    if device.type != "cuda" or dtype_name == "float32":
        return torch.float32
    return torch.float16 if dtype_name == "float16" else torch.bfloat16


def save_checkpoint(save_dir: str, step: int, model, optimizer, args, extra: Dict[str, object]) -> str:
    os.makedirs(save_dir, exist_ok=True)
    path = os.path.join(save_dir, f"step_{step:06d}.pt")
    torch.save({"step": step, "model_state_dict": model.state_dict(), "optimizer_state_dict": optimizer.state_dict(),
                "train_args": vars(args), "extra": extra}, path)
    return path


def train(args: argparse.Namespace) -> None:
    set_seed(args.seed)
    device = choose_device(args.device)
    base_vocab = args.synthetic_vocab_size
    try:
        loader, vocab, metadata = make_data_loader(args, vocab_size_for_model=base_vocab)
    except Exception as exc:
        if not args.allow_synthetic_fallback:
            raise
        print(f"[warn] failed to initialize fineweb pipeline ({exc}); falling back to synthetic data")
        args.data_mode = "synthetic"
        loader, vocab, metadata = make_data_loader(args, vocab_size_for_model=base_vocab)
    cfg = model_config_from_args(args, vocab)
    dtype = model_param_dtype(device, args.dtype)
    model = LlamaForCausalLM(cfg).to(device=device, dtype=dtype)
    model.set_loss_chunk_size(args.loss_chunk_size)
    model.set_activation_checkpointing(args.activation_checkpointing)
    backend = resolve_backend(args, device, dtype)
    model.set_backend(backend)
    optimizer = torch.optim.AdamW(model.parameters(), lr=args.learning_rate, betas=(args.beta1, args.beta2),
                                  weight_decay=args.weight_decay)
    scaler = torch.amp.GradScaler("cuda", enabled=device.type == "cuda" and args.dtype == "float16")
    n_params = estimate_num_parameters(cfg)
    print(f"[init] model={cfg.name} params={human_readable_count(n_params)} ({n_params:,}) vocab={cfg.vocab_size:,} "
          f"seq_len={cfg.max_seq_len} device={device.type} dtype={args.dtype} backend={backend}")
    print(f"[init] data_mode={args.data_mode} metadata={json.dumps(metadata)}")
    tokens_per_step = args.batch_size * args.grad_accum_steps * args.seq_len
    data_iter: Iterator[torch.Tensor] = iter(loader)
    recent = []
    t_start = time.perf_counter()
    for step in range(1, args.max_steps + 1):
        model.train()
        optimizer.zero_grad(set_to_none=True)
        t0 = time.perf_counter()
        micro_losses = []
        for _ in range(args.grad_accum_steps):
            try:
                chunk = next(data_iter)
            except StopIteration:
                data_iter = iter(loader)
                chunk = next(data_iter)
            batch = batch_from_chunk(chunk)
            ids = batch.input_ids.to(device, non_blocking=True)
            labels = batch.labels.to(device, non_blocking=True)
            with autocast_context(device, args.dtype):
                loss = model(input_ids=ids, labels=labels, return_logits=False).loss
            micro_losses.append(float(loss.detach().float()))
            scaler.scale(loss / args.grad_accum_steps).backward()
        if args.max_grad_norm > 0:
            scaler.unscale_(optimizer)
            grad_norm = float(torch.nn.utils.clip_grad_norm_(model.parameters(), max_norm=args.max_grad_norm))
        else:
            grad_norm = math.nan
        scaler.step(optimizer)
        scaler.update()
        step_loss = sum(micro_losses) / len(micro_losses)
        recent = (recent + [step_loss])[-100:]
        tokens_per_second = tokens_per_step / max(time.perf_counter() - t0, 1e-8)
        if step % args.log_interval == 0 or step == 1 or step == args.max_steps:
            print(f"[step {step:05d}] loss={step_loss:.4f} avg100={sum(recent) / len(recent):.4f} "
                  f"tokens/s={tokens_per_second:,.0f} grad_norm={grad_norm:.3f}", flush=True)
        if args.checkpoint_interval > 0 and (step % args.checkpoint_interval == 0 or step == args.max_steps):
            path = save_checkpoint(args.save_dir, step, model, optimizer, args,
                                   {"model_config": cfg.to_dict(), "step_loss": step_loss})
            print(f"[checkpoint] wrote {path}")
    print(f"[done] trained {args.max_steps} steps in {time.perf_counter() - t_start:.1f}s")


def main(argv=None) -> None:
    train(parse_args(argv))


if __name__ == "__main__":
    main()
