"""Reference arm of ``bench.py``: the unmodified reference implementation on the same workload.

It imports the reference's own ``model``, ``zero`` and ``collectives`` packages from
``baseline/_ref`` (installed there with pip from the read-only reference tree) and drives them
the way the reference's ``train_zero.py`` does (``train_zero.py:303-321, 416-581``):
bf16 parameters, bf16 autocast, ``--loss-chunk-size 128``, ``LocalCollectives`` on one GPU and
``TorchCollectives`` (NCCL) otherwise, ``engine.zero_grad / prepare_forward / backward /
step_with_stats``.  Only the model shape (the benchmark's 'small' config, which the reference CLI
cannot express) and the token source (uniform random ids) differ from its CLI defaults.
Nothing from this repository's package is imported here.
"""

from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")


def _unavailable(reason: str) -> None:
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)


def main(args, ClockSampler, base_record, emit, time_device, time_wall, random_batches, max_over_ranks, metric,
         model_desc) -> None:
    if not os.path.isdir(os.path.join(REF, "zero")):
        _unavailable("reference not installed in baseline/_ref (install: python -m pip install --no-index --no-build-isolation --find-links /opt/wheelhouse --no-deps --target baseline/_ref <copy of the reference tree with a pyproject.toml>)")
        return
    sys.path.insert(0, REF)
    from datetime import timedelta

    import torch
    import torch.distributed as dist
    from collectives import LocalCollectives, TorchCollectives
    from model.config import ModelConfig
    from model.llama import LlamaForCausalLM
    from zero import ZeROStage0DDP, ZeROStage1Optimizer, ZeROStage2Optimizer, ZeROStage3Optimizer

    engines = {0: ZeROStage0DDP, 1: ZeROStage1Optimizer, 2: ZeROStage2Optimizer, 3: ZeROStage3Optimizer}
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1 and not dist.is_initialized():
        dist.init_process_group(backend="nccl", timeout=timedelta(seconds=600), device_id=device)
    torch.backends.cuda.matmul.allow_tf32 = True
    torch.backends.cudnn.allow_tf32 = True
    torch.backends.cudnn.benchmark = True
    vocab = 32000
    tokens_per_step = args.batch_size * args.seq_len * world
    per_stage, e2e, clocks, headline_ms = {}, None, None, None
    for stage in args.stage_list:
        torch.manual_seed(1337)
        cfg = ModelConfig(name="small", vocab_size=vocab, max_seq_len=args.seq_len, dim=768, n_layers=12, n_heads=12,
                          n_kv_heads=4, ffn_dim=2048)
        model = LlamaForCausalLM(cfg).to(device=device, dtype=torch.bfloat16)
        model.set_loss_chunk_size(128)
        if world > 1:
            for p in model.parameters():
                dist.broadcast(p.data, src=0)
        coll = LocalCollectives() if world == 1 else TorchCollectives()
        engine = engines[stage](model=model, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, collectives=coll)
        host = random_batches(4, args.batch_size, args.seq_len, vocab, seed=1234 + rank * 100 + stage)
        dev = [h.to(device) for h in host]
        it = {"i": 0}
        last = {}

        def step(batch):
            model.train()
            engine.zero_grad()
            engine.prepare_forward()
            with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
                loss = model(input_ids=batch, labels=batch, return_logits=False).loss
            engine.backward(loss)
            last["stats"] = engine.step_with_stats(max_grad_norm=0.0)
            return loss

        def device_step():
            step(dev[it["i"] % len(dev)])
            it["i"] += 1

        sampler = ClockSampler([local], getattr(args, "clocks_csv", None)) if stage == args.headline_stage and rank == 0 else None
        if sampler:
            sampler.__enter__()
        for _ in range(args.warmup):
            device_step()
        ms = time_device(device_step, args.steps)
        if sampler:
            sampler.__exit__(None, None, None)
            clocks = sampler.summary()
        entry = {"tokens_per_s": tokens_per_step / (ms / 1000.0), "ms_per_step": ms,
                 "comm_ms": max_over_ranks(float(last["stats"].get("comm_ms", 0.0)))}
        if stage == args.headline_stage:
            headline_ms = ms
            if not args.no_e2e:
                def e2e_step():
                    batch = host[it["i"] % len(host)].to(device, non_blocking=True)
                    it["i"] += 1
                    float(step(batch))

                e2e_ms = time_wall(e2e_step, args.steps)
                e2e = {"value": tokens_per_step / (e2e_ms / 1000.0), "unit": "tokens/s", "ms_per_step": e2e_ms,
                       "h2d_bytes_per_step": host[0].numel() * 8, "d2h_bytes_per_step": 4,
                       "api": "reference LlamaForCausalLM + ZeROStage*.step_with_stats"}
        per_stage[str(stage)] = entry
        if hasattr(engine, "summon_full_params"):
            model._zero3_executor = None
        del engine, model
        torch.cuda.empty_cache()
    rec = base_record(args, world, "reference")
    rec.update({
        "value": per_stage[str(args.headline_stage)]["tokens_per_s"],
        "ms_per_step": headline_ms,
        "config": {"model": model_desc, "global_batch": args.batch_size * world, "micro_batch_per_gpu": args.batch_size,
                   "seq_len": args.seq_len, "grad_accum": 1, "parallelism": f"dp{world}",
                   "zero_stage": args.headline_stage, "collective_impl": "torch" if world > 1 else "local",
                   "loss_chunk_size": 128},
        "per_stage": per_stage,
        "e2e": e2e,
        "gpu_launches": 0,
        "clocks": clocks,
    })
    emit(rec, rank)
    if dist.is_available() and dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
