"""Training CLI: ``python -m uno_b200.train --model DIR|preset:NAME --output-dir OUT ...``.

Single process, or one process per GPU under ``torchrun`` (data parallel: the
frozen base is replicated, LoRA gradients are averaged across ranks).
Data is synthetic Zipf token ids (``--data synthetic``) or a JSONL file of
pre-tokenised ``{"input_ids", "labels"}`` rows.  The curriculum comes from a
YAML file (``--curriculum``) or from ``--block-sizes`` / ``--steps-per-stage``.

The option names of the reference trainer (``training/train.py``) are
accepted as well: ``--learning-rate``, ``--per-device-batch-size``,
``--gradient-accumulation-steps``, ``--dataset-path``,
``--resume-from-checkpoint``, ``--tv-gamma`` / ``--kl-beta`` / ``--ce-alpha``
(the loss weights), and ``--deepspeed CONFIG``, whose ZeRO stage, gradient
clipping, micro-batch and accumulation settings map onto this trainer
(stage 3 shards the frozen base like ``--fsdp``; stage 2 is the default
sharded optimizer).  Metrics go to stdout and ``OUTPUT_DIR/metrics.jsonl``,
and to a Weights & Biases run with ``--wandb-mode online|offline``
(``train/metrics_sink.py``).
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

from uno_b200.train.metrics_sink import MetricsSink, check_wandb


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--model", required=True)
    p.add_argument("--output-dir", required=True)
    p.add_argument("--curriculum", help="curriculum YAML, or 'released' for the released run's schedule")
    p.add_argument("--block-sizes", default="4,8,16")
    p.add_argument("--steps-per-stage", type=int, default=1)
    p.add_argument("--seq-len", type=int, default=128)
    p.add_argument("--global-batch", type=int, default=2)
    p.add_argument("--micro-batch", "--per-device-batch-size", dest="micro_batch", type=int, default=None)
    p.add_argument("--gradient-accumulation-steps", type=int,
                   help="with --block-sizes: sets the global batch to world * micro-batch * steps")
    p.add_argument("--data", "--dataset-path", dest="data", default="synthetic")
    p.add_argument("--prompt-len", type=int, default=0)
    p.add_argument("--pack-rows", action="store_true",
                   help="pack several prepared rows per sequence instead of one padded row per sequence")
    p.add_argument("--lr", "--learning-rate", dest="lr", type=float, default=1e-4)
    p.add_argument("--warmup-steps", type=int, default=0)
    p.add_argument("--lr-schedule", choices=("constant", "cosine"), default="constant",
                   help="after the warmup: constant (the released recipe) or cosine decay to 0")
    p.add_argument("--weight-decay", type=float, default=0.0)
    p.add_argument("--max-grad-norm", type=float, default=None, help="gradient-norm clip (default 1.0)")
    p.add_argument("--lora-rank", type=int, default=64)
    p.add_argument("--lora-alpha", type=int, default=None)
    p.add_argument("--lora-target", default="all")
    p.add_argument("--lora-dropout", type=float, default=0.0, help="only 0 (the recipe's value) is supported")
    p.add_argument("--tv-weight", "--tv-gamma", dest="tv_weight", type=float, default=1.0)
    p.add_argument("--kl-weight", "--kl-beta", dest="kl_weight", type=float, default=0.0)
    p.add_argument("--ce-weight", "--ce-alpha", dest="ce_weight", type=float, default=0.0)
    p.add_argument("--ce-target", choices=("teacher", "ground_truth"), default="teacher")
    p.add_argument("--mask-token-id", type=int)
    p.add_argument("--device", choices=("cuda", "cpu"), default="cuda")
    p.add_argument("--checkpoint-layers", action="store_true")
    p.add_argument("--resume", "--resume-from-checkpoint", dest="resume")
    p.add_argument("--run-name", help="recorded in the run manifest")
    p.add_argument("--logging-steps", type=int, default=1, help="print metrics every N optimizer steps")
    p.add_argument("--deepspeed", help="DeepSpeed JSON config: its ZeRO stage, clipping and batch settings apply")
    p.add_argument("--model-cache-dir", help="Hugging Face cache for a hub model id")
    p.add_argument("--local-files-only", action="store_true")
    p.add_argument("--local-rank", "--local_rank", dest="local_rank", type=int, default=-1,
                   help="launcher compatibility; LOCAL_RANK in the environment takes precedence")
    p.add_argument("--dataloader-num-workers", type=int, default=0, help="accepted; rows are packed in-process")
    p.add_argument("--wandb-project", default=os.environ.get("WANDB_PROJECT", "uno-training"),
                   help="W&B project of the run (metrics also go to OUTPUT_DIR/metrics.jsonl)")
    p.add_argument("--wandb-mode", choices=("online", "offline", "disabled"),
                   default=os.environ.get("WANDB_MODE", "disabled"),
                   help="W&B reporting; online needs credentials (default: $WANDB_MODE, else disabled)")
    p.add_argument("--max-steps", type=int, help="stop after this many optimizer steps (default: curriculum end)")
    p.add_argument("--fsdp", action="store_true",
                   help="CUDA: shard the frozen projection weights over the ranks (GEMMs read peers' rows)")
    p.add_argument("--seed", type=int, default=0)
    return p


def apply_deepspeed_config(args, path: str) -> dict:
    """Map a DeepSpeed JSON config onto this trainer's options (explicit flags win).

    ``zero_optimization.stage`` 3 shards the frozen base (``--fsdp``), 0-2
    keep it replicated with the sharded optimizer; ``gradient_clipping`` sets
    the clip norm; numeric ``train_micro_batch_size_per_gpu`` and
    ``gradient_accumulation_steps`` set the micro-batch and accumulation
    (``"auto"`` leaves them to the other flags).  Returns what was applied.
    """
    with open(path, encoding="utf-8") as fh:
        cfg = json.load(fh)
    applied = {}
    stage = int((cfg.get("zero_optimization") or {}).get("stage", 2))
    if stage >= 3 and not args.fsdp:
        args.fsdp = True
        applied["fsdp"] = True
    clip = cfg.get("gradient_clipping")
    if isinstance(clip, (int, float)) and args.max_grad_norm is None:
        args.max_grad_norm = float(clip)
        applied["max_grad_norm"] = float(clip)
    micro = cfg.get("train_micro_batch_size_per_gpu")
    if isinstance(micro, int) and args.micro_batch is None:
        args.micro_batch = micro
        applied["micro_batch"] = micro
    accum = cfg.get("gradient_accumulation_steps")
    if isinstance(accum, int) and args.gradient_accumulation_steps is None:
        args.gradient_accumulation_steps = accum
        applied["gradient_accumulation_steps"] = accum
    applied["zero_stage"] = stage
    return applied


def main(argv: list[str] | None = None) -> list[dict]:
    args = build_parser().parse_args(argv)
    check_wandb(args.wandb_mode)
    deepspeed = apply_deepspeed_config(args, args.deepspeed) if args.deepspeed else None
    if args.micro_batch is None:
        args.micro_batch = 1
    if args.max_grad_norm is None:
        args.max_grad_norm = 1.0
    if args.lora_dropout:
        raise SystemExit("LoRA dropout is not implemented; the released recipe trains with --lora-dropout 0")
    from uno_b200.models.decoder import build_model
    from uno_b200.models.presets import resolve_preset
    from uno_b200.train import BlockCurriculumPlan, LoraSettings, TrainableLoRA, UnoObjectiveConfig, UnoTrainer
    from uno_b200.train.config import manifest_digest, validate_resume_manifest, write_run_manifest
    from uno_b200.train.data import batches_from_rows, data_manifest, load_jsonl, pack_rows, pad_rows, \
        synthetic_batches
    from uno_b200.utils.hf_compat import load_model_config
    from uno_b200.utils.loader import dummy_init, load_model

    world, rank, group = 1, 0, None
    if "WORLD_SIZE" in os.environ and int(os.environ["WORLD_SIZE"]) > 1:
        backend = "nccl" if args.device == "cuda" else "gloo"
        dist.init_process_group(backend)
        world, rank, group = dist.get_world_size(), dist.get_rank(), dist.group.WORLD
    local = int(os.environ.get("LOCAL_RANK", max(args.local_rank, 0)))
    device = torch.device("cuda", local) if args.device == "cuda" else torch.device("cpu")
    if device.type == "cuda":
        torch.cuda.set_device(device)

    if args.model.startswith("preset:"):
        cfg, model_dir = resolve_preset(args.model[len("preset:"):]), None
    else:
        from uno_b200.utils.hub import resolve_hf_snapshot

        model_dir = resolve_hf_snapshot(args.model, cache_dir=args.model_cache_dir,
                                        local_files_only=args.local_files_only, artifact_name="model")
        cfg = load_model_config(model_dir)
    dtype = torch.float32 if device.type == "cpu" else torch.bfloat16
    torch.set_default_dtype(dtype)
    with torch.device(device):
        model = build_model(cfg)
    torch.set_default_dtype(torch.float32)
    if model_dir is None:
        dummy_init(model, seed=args.seed)
    else:
        load_model(model, model_dir)
    mask_id = args.mask_token_id if args.mask_token_id is not None else cfg.mask_token_id
    if mask_id is None:
        raise SystemExit("the model config has no mask_token_id; pass --mask-token-id")

    if args.curriculum == "released":  # the released run's six-stage schedule
        from uno_b200.train.curriculum import released_curriculum

        plan = BlockCurriculumPlan.from_mapping(released_curriculum())
    elif args.curriculum:
        plan = BlockCurriculumPlan.from_yaml(args.curriculum)
    else:
        global_batch = args.global_batch
        if args.gradient_accumulation_steps:
            global_batch = world * args.micro_batch * args.gradient_accumulation_steps
        plan = BlockCurriculumPlan.fixed([int(b) for b in args.block_sizes.split(",")], args.steps_per_stage,
                                         args.seq_len, global_batch, args.seed)
    accumulation = plan.global_batch_size // (world * args.micro_batch)
    if args.gradient_accumulation_steps and args.gradient_accumulation_steps != accumulation:
        raise SystemExit(f"--gradient-accumulation-steps {args.gradient_accumulation_steps} does not give the "
                         f"curriculum's global batch {plan.global_batch_size} with {world} ranks x micro-batch "
                         f"{args.micro_batch} (that needs {accumulation})")
    plan.validate_runtime(world_size=world, per_device_batch=args.micro_batch, accumulation=accumulation)
    settings = LoraSettings(target=args.lora_target, rank=args.lora_rank, alpha=args.lora_alpha)
    objective = UnoObjectiveConfig(ce_target=args.ce_target, ce_weight=args.ce_weight, kl_weight=args.kl_weight,
                                   tv_weight=args.tv_weight)
    lora = TrainableLoRA(cfg, settings, device=device, seed=args.seed)
    if args.data == "synthetic":
        batches = synthetic_batches(args.micro_batch, plan.sequence_length, cfg.vocab_size, prompt_len=args.prompt_len,
                                    seed=args.seed * 7919 + rank)
        data_info = {"kind": "synthetic-zipf-1.1", "seed": args.seed}
    else:
        collate = pack_rows if args.pack_rows else pad_rows
        batches = batches_from_rows(collate(load_jsonl(args.data), plan.sequence_length), args.micro_batch,
                                    seed=args.seed * 7919 + rank)
        data_info = data_manifest([args.data]) | {"collation": "pack" if args.pack_rows else "pad"}
    compat = {"model": args.model, "curriculum_sha256": plan.sha256(), "lora": vars(settings) | {"alpha": settings.resolved_alpha},
              "objective": vars(objective), "mask_token_id": int(mask_id), "data": data_info,
              "micro_batch": args.micro_batch, "world_size": world, "lr_schedule": args.lr_schedule}
    out = args.output_dir
    os.makedirs(out, exist_ok=True)
    trainer = UnoTrainer(model, lora, objective=objective, curriculum=plan, mask_token_id=mask_id, lr=args.lr,
                         warmup_steps=args.warmup_steps, weight_decay=args.weight_decay,
                         max_grad_norm=args.max_grad_norm, output_dir=out, checkpoint_layers=args.checkpoint_layers,
                         seed=args.seed, process_group=group, base_model_name=args.model, fsdp=args.fsdp,
                         lr_schedule=args.lr_schedule)
    if args.resume:
        validate_resume_manifest(out, compat)
        trainer.resume(args.resume)
    elif rank == 0:
        extra = {"compatibility_sha256_short": manifest_digest(compat)[:12], "run_name": args.run_name,
                 "wandb": {"project": args.wandb_project, "mode": args.wandb_mode}}
        if deepspeed is not None:
            extra["deepspeed_config"] = {"path": args.deepspeed, "applied": deepspeed}
        write_run_manifest(out, compat, extra)
    last = min(plan.max_steps, args.max_steps or plan.max_steps)
    history = []
    sink = MetricsSink(out, rank=rank, wandb_mode=args.wandb_mode, wandb_project=args.wandb_project,
                       run_name=args.run_name, config=compat, resume=bool(args.resume))
    try:
        while trainer.step < last:
            metrics = trainer.train_step([next(batches) for _ in range(accumulation)])
            history.append(metrics)
            sink.log(metrics)
            if rank == 0 and (trainer.step % max(1, args.logging_steps) == 0 or trainer.step == last):
                print(json.dumps(metrics), flush=True)
    finally:
        sink.close()
    if rank == 0:
        lora.save(os.path.join(out, "final_adapter"), args.model)
    if group is not None:
        dist.destroy_process_group()
    return history


if __name__ == "__main__":
    main()
