"""Reference arm of ``bench.py``: the unmodified reference implementation on the same workload.

It imports the reference's own ``model``, ``zero`` and ``collectives`` packages from
``baseline/_ref`` (installed there with pip from the read-only reference tree) and drives them
the way the reference's ``train_zero.py`` does (``train_zero.py:303-321, 416-581``):
bf16 parameters, bf16 autocast, ``--loss-chunk-size 128``, ``LocalCollectives`` on one GPU and
``TorchCollectives`` (NCCL) otherwise, ``engine.zero_grad / prepare_forward / backward /
step_with_stats``.  Only the model shapes (the benchmark's 'small' config and, under ``per_config``,
the 1.3B config, which the reference CLI cannot express) and the token source (uniform random ids)
differ from its CLI defaults.
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
         model_desc, config_shapes=None) -> None:
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
    shapes = config_shapes or {}
    small = shapes.get("baseline-small", dict(dim=768, n_layers=12, n_heads=12, n_kv_heads=4, ffn_dim=2048))

    def measure(shape, batch, seq, headline):
        tokens_per_step = batch * seq * world
        out = {"per_stage": {}, "e2e": None, "clocks": None, "headline_ms": None}
        for stage in args.stage_list:
            torch.manual_seed(1337)
            cfg = ModelConfig(name="bench", vocab_size=vocab, max_seq_len=seq, dim=shape["dim"],
                              n_layers=shape["n_layers"], n_heads=shape["n_heads"], n_kv_heads=shape["n_kv_heads"],
                              ffn_dim=shape["ffn_dim"])
            model = LlamaForCausalLM(cfg).to(device=device, dtype=torch.bfloat16)
            model.set_loss_chunk_size(128)
            if world > 1:
                for p in model.parameters():
                    dist.broadcast(p.data, src=0)
            coll = LocalCollectives() if world == 1 else TorchCollectives()
            engine = engines[stage](model=model, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                                    collectives=coll)
            host = random_batches(4, batch, seq, vocab, seed=1234 + rank * 100 + stage)
            dev = [h.to(device) for h in host]
            it = {"i": 0}
            last = {}

            def step(b):
                model.train()
                engine.zero_grad()
                engine.prepare_forward()
                with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
                    loss = model(input_ids=b, labels=b, return_logits=False).loss
                engine.backward(loss)
                last["stats"] = engine.step_with_stats(max_grad_norm=0.0)
                return loss

            def device_step():
                step(dev[it["i"] % len(dev)])
                it["i"] += 1

            is_head = headline and stage == args.headline_stage
            sampler = ClockSampler([local], getattr(args, "clocks_csv", None)) if is_head and rank == 0 else None
            if sampler:
                sampler.__enter__()
            for _ in range(args.warmup):
                device_step()
            ms = time_device(device_step, args.steps)
            if sampler:
                sampler.__exit__(None, None, None)
                out["clocks"] = sampler.summary()
            entry = {"tokens_per_s": tokens_per_step / (ms / 1000.0), "ms_per_step": ms,
                     "comm_ms": max_over_ranks(float(last["stats"].get("comm_ms", 0.0)))}
            if is_head:
                out["headline_ms"] = ms
                if not args.no_e2e:
                    def e2e_step():
                        b = host[it["i"] % len(host)].to(device, non_blocking=True)
                        it["i"] += 1
                        float(step(b))

                    e2e_ms = time_wall(e2e_step, args.steps)
                    out["e2e"] = {"value": tokens_per_step / (e2e_ms / 1000.0), "unit": "tokens/s",
                                  "ms_per_step": e2e_ms, "h2d_bytes_per_step": host[0].numel() * 8,
                                  "d2h_bytes_per_step": 4,
                                  "api": "reference LlamaForCausalLM + ZeROStage*.step_with_stats"}
            out["per_stage"][str(stage)] = entry
            if hasattr(engine, "summon_full_params"):
                model._zero3_executor = None
            del engine, model
            torch.cuda.empty_cache()
        return out

    head = measure(small, args.batch_size, args.seq_len, True)
    per_config = {}
    for size in getattr(args, "extra_list", []):
        shape = shapes.get(size)
        if shape is None:
            continue
        extra = measure(shape, shape["batch"], shape["seq"], False)
        per_config[size] = {"model": f"{size} LLaMA d{shape['dim']}/L{shape['n_layers']}/H{shape['n_heads']}/"
                                     f"KV{shape['n_kv_heads']}/ffn{shape['ffn_dim']}/V{vocab} (tied embeddings)",
                            "global_batch": shape["batch"] * world, "micro_batch_per_gpu": shape["batch"],
                            "seq_len": shape["seq"], "per_stage": extra["per_stage"]}
    rec = base_record(args, world, "reference")
    rec.update({
        "value": head["per_stage"][str(args.headline_stage)]["tokens_per_s"],
        "ms_per_step": head["headline_ms"],
        "config": {"model": model_desc, "global_batch": args.batch_size * world, "micro_batch_per_gpu": args.batch_size,
                   "seq_len": args.seq_len, "grad_accum": 1, "parallelism": f"dp{world}",
                   "zero_stage": args.headline_stage, "collective_impl": "torch" if world > 1 else "local",
                   "loss_chunk_size": 128},
        "per_stage": head["per_stage"],
        "per_config": per_config,
        "e2e": head["e2e"],
        "gpu_launches": 0,
        "clocks": head["clocks"],
    })
    emit(rec, rank)
    if dist.is_available() and dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
