"""The PR1 reference configuration on the CPU: 'tiny' LLaMA, ZeRO-3, gloo, world size 2, fp32.

Shape d256 / 4 layers / 4 query heads / 2 KV heads / SwiGLU 688 / RMSNorm eps 1e-5 / RoPE theta 1e4 /
vocab 32000, untied embeddings; sequence 128, micro-batch 4 per rank, gradient accumulation 2,
20 steps, AdamW lr 3e-4 (betas 0.9 / 0.95, eps 1e-8, weight decay 0.1), weights normal(0, 0.02),
tokens uniform in [0, 32000) from seed 0 (labels = inputs; the models shift them).

Runs the same steps through this package's ZeRO-3 engine and through the reference's own ZeRO-3
engine (installed in ``baseline/_ref``), each with both of its collective implementations (the
ring over send/recv and torch.distributed), starting from identical weights (same seed, same
initialisation order) and on identical micro-batches, and prints one JSON line per run with the
tokens/s (wall clock, max over ranks) and the per-step losses, then the largest loss difference
between the two implementations.

    python baseline/pr1_tiny_cpu.py [--steps 20] [--impls mine,reference] [--collectives ring,torch]
"""

from __future__ import annotations

import argparse
import json
import os
import socket
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF = os.path.join(HERE, "_ref")

SHAPE = dict(dim=256, n_layers=4, n_heads=4, n_kv_heads=2, ffn_dim=688, rope_theta=10_000.0, rms_norm_eps=1e-5,
             vocab_size=32_000, tie_word_embeddings=False)
SEQ, MICRO, ACCUM, WORLD = 128, 4, 2, 2
HP = dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _batches(steps: int, rank: int):
    """[step][micro] int64 [MICRO, SEQ] for this rank, drawn in one fixed order for every run."""
    import torch

    g = torch.Generator().manual_seed(0)
    out = []
    for _ in range(steps):
        per_rank = [[torch.randint(0, SHAPE["vocab_size"], (MICRO, SEQ), generator=g) for _ in range(ACCUM)]
                    for _ in range(WORLD)]
        out.append(per_rank[rank])
    return out


def _build(impl: str, coll_name: str):
    import torch

    torch.manual_seed(1234)
    if impl == "mine":
        sys.path.insert(0, ROOT)
        from cs244c_llama_zero_b200.models import LlamaForCausalLM, ModelConfig
        from cs244c_llama_zero_b200.parallel.collectives import pick_collectives
        from cs244c_llama_zero_b200.parallel.zero import ZeROStage3Optimizer

        model = LlamaForCausalLM(ModelConfig(name="pr1-tiny", max_seq_len=SEQ, **SHAPE))
        coll = pick_collectives(WORLD, coll_name, torch.device("cpu"))
    else:
        sys.path.insert(0, REF)
        from collectives import SendRecvCollectives, TorchCollectives
        from model.config import ModelConfig
        from model.llama import LlamaForCausalLM
        from zero import ZeROStage3Optimizer

        model = LlamaForCausalLM(ModelConfig(name="pr1-tiny", max_seq_len=SEQ, **SHAPE))
        coll = SendRecvCollectives() if coll_name == "ring" else TorchCollectives()
    return model, ZeROStage3Optimizer(model=model, collectives=coll, **HP)


def _worker(rank: int, port: int, impl: str, coll_name: str, steps: int, queue) -> None:
    import torch
    import torch.distributed as dist

    torch.set_num_threads(max(1, (os.cpu_count() or 2) // WORLD))
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD)
    try:
        model, engine = _build(impl, coll_name)
        data = _batches(steps, rank)
        losses = []
        dist.barrier()
        t0 = time.perf_counter()
        for micro in data:
            model.train()
            engine.zero_grad()
            engine.prepare_forward()
            total = 0.0
            for ids in micro:
                loss = model(input_ids=ids, labels=ids, return_logits=False).loss
                engine.backward(loss / ACCUM)
                total += float(loss.detach()) / ACCUM
            engine.step_with_stats(max_grad_norm=0.0)
            t = torch.tensor([total])
            dist.all_reduce(t)
            losses.append(float(t) / WORLD)
        elapsed = torch.tensor([time.perf_counter() - t0])
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
        if rank == 0:
            tokens = steps * WORLD * ACCUM * MICRO * SEQ
            queue.put({"impl": impl, "collectives": coll_name, "tokens_per_s": tokens / float(elapsed),
                       "seconds": float(elapsed), "losses": losses})
    finally:
        dist.barrier()
        dist.destroy_process_group()


def run(impl: str, coll_name: str, steps: int) -> dict:
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.SimpleQueue()
    mp.start_processes(_worker, args=(_free_port(), impl, coll_name, steps, queue), nprocs=WORLD, join=True,
                       start_method="spawn")
    return queue.get()


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--impls", default="mine,reference")
    p.add_argument("--collectives", default="ring,torch")
    a = p.parse_args(argv)
    impls = [x for x in a.impls.split(",") if x]
    if "reference" in impls and not os.path.isdir(os.path.join(REF, "zero")):
        print(json.dumps({"impl": "reference", "unavailable": "reference not installed in baseline/_ref"}))
        impls.remove("reference")
    results = []
    for coll in [x for x in a.collectives.split(",") if x]:
        for impl in impls:
            rec = run(impl, coll, a.steps)
            rec.update({"config": "PR1 tiny d256/L4/H4/KV2/ffn688/V32000 untied, ZeRO-3, CPU gloo, W=2, fp32, "
                                  f"S{SEQ} B{MICRO} GA{ACCUM}, {a.steps} steps"})
            print(json.dumps(rec), flush=True)
            results.append(rec)
    by = {(r["impl"], r["collectives"]): r["losses"] for r in results}
    for coll in {r["collectives"] for r in results}:
        if ("mine", coll) in by and ("reference", coll) in by:
            diff = max(abs(x - y) for x, y in zip(by[("mine", coll)], by[("reference", coll)]))
            print(json.dumps({"collectives": coll, "max_abs_loss_diff_mine_vs_reference": diff}), flush=True)


if __name__ == "__main__":
    main()
