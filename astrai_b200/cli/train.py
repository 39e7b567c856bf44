"""Training entry point with the reference CLI's flags.

    python -m astrai_b200.cli.train --train_type seq --param_path MODEL_DIR --data_root_path DATA ...

Parity: scripts/tools/train.py:97-616 of the reference (same flag names,
defaults and choices; MuonMix on hidden matrices + AdamW on the rest; total
steps and warmup from the dataset length; scheduler kwargs per schedule
type; DecoderBlock checkpointing with --gradient_checkpointing). Added
flags: ``--comm_backend fused`` (NVLink peer-memory gradient all-reduce for
ddp), ``--expert_parallel`` (shard MoE experts over the ranks),
``--profile_dir``, ``--shard_muon`` (owner-sharded Muon: each rank runs
Newton-Schulz on 1/world of the matrices and writes the updated weights into
every replica over NVLink).
"""

from __future__ import annotations

import argparse
import os
from functools import partial
from typing import List, Optional

import torch


def parse_args(argv: Optional[List[str]] = None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="Train a model with astrai_b200.")
    a = p.add_argument
    a("--train_type", type=str, required=True, choices=["seq", "sft", "dpo", "grpo", "online_grpo", "online_dpo"])
    a("--data_root_path", type=str, required=True, help="Dataset root (bin / h5 / jsonl).")
    a("--param_path", type=str, required=True, help="Model directory: config.json, tokenizer, weights.")
    a("--resume", action="store_true", help="Resume from the checkpoint in --param_path.")
    a("--n_epoch", type=int, default=1)
    a("--batch_per_device", type=int, default=1)
    a("--grad_accum_steps", type=int, default=1)
    a("--warmup_ratio", type=float, default=0.05)
    a("--max_lr", type=float, default=3e-4)
    a("--max_grad_norm", type=float, default=1.0)
    a("--weight_decay", type=float, default=0.1)
    a("--muon_momentum", type=float, default=0.95)
    a("--muon_nesterov", type=lambda s: str(s).lower() in ("1", "true", "yes"), default=True)
    a("--muon_ns_steps", type=int, default=5)
    a("--muon_adjust_lr", type=str, default="match_rms_adamw", choices=["original", "match_rms_adamw"])
    a("--random_seed", type=int, default=3407)
    a("--num_workers", type=int, default=4)
    a("--no_pin_memory", dest="pin_memory", action="store_false")
    a("--window_size", type=int, default=None)
    a("--stride", type=int, default=None)
    a("--dpo_beta", type=float, default=0.1, help="DPO beta value.")
    a("--group_size", type=int, default=4, help="GRPO group size.")
    a("--grpo_clip_eps", type=float, default=0.2)
    a("--grpo_kl_coef", type=float, default=0.01)
    a("--label_smoothing", type=float, default=0.0)
    a("--rollout_interval", type=int, default=512)
    a("--rollout_temperature", type=float, default=0.7)
    a("--rollout_top_k", type=int, default=0)
    a("--rollout_top_p", type=float, default=0.9)
    a("--rollout_max_tokens", type=int, default=1024)
    a("--gradient_checkpointing", action="store_true", default=False)
    a("--ckpt_interval", type=int, default=5000)
    a("--ckpt_dir", type=str, default="checkpoint")
    a("--val_split", type=float, default=None)
    a("--val_step", type=int, default=1000)
    a("--metrics", type=str, nargs="+", default=["loss"])
    a("--log_dir", type=str, default="checkpoint/logs")
    a("--start_epoch", type=int, default=0)
    a("--start_samples", type=int, default=0)
    a("--master_addr", type=str, default="localhost")
    a("--master_port", type=str, default="29500")
    a("--backend", type=str, default="nccl")
    a("--nprocs", type=int, default=1, help="Number of GPUs to use.")
    a("--parallel_mode", type=str, default="none", choices=["none", "ddp", "fsdp", "fsdp2"])
    a("--device_type", type=str, default="cuda")
    a("--start_method", type=str, default="spawn", choices=["spawn", "fork", "forkserver"])
    a("--neftune_alpha", type=float, default=0.0)
    a("--schedule_type", type=str, default="cosine", choices=["cosine", "sgdr", "wsd"])
    a("--min_rate", type=float, default=None)
    a("--cycle_length", type=int, default=None)
    a("--t_mult", type=int, default=2)
    a("--stable_steps", type=int, default=None)
    a("--decay_steps", type=int, default=None)
    # additions
    a("--comm_backend", type=str, default="nccl", choices=["nccl", "fused"],
      help="ddp gradient exchange: NCCL, or the NVLink peer-memory all-reduce fused with the grad norm.")
    a("--expert_parallel", action="store_true", help="Split MoE experts over the ranks (ddp).")
    a("--shard_muon", action="store_true",
      help="ddp: each rank orthogonalises 1/world of the Muon matrices and writes the update into every replica.")
    a("--profile_dir", type=str, default=None)
    return p.parse_args(argv)


def compute_total_steps(dataset_len: int, n_epoch: int, batch_per_device: int, nprocs: int,
                        grad_accum_steps: int) -> int:
    per_replica = -(-dataset_len // nprocs)
    batches = -(-per_replica // batch_per_device)
    return (batches // grad_accum_steps) * n_epoch


def scheduler_kwargs(schedule_type: str, total_steps: int, warmup_ratio: float, min_rate=None, cycle_length=None,
                     t_mult: int = 2, stable_steps=None, decay_steps=None) -> dict:
    warm = min(int(warmup_ratio * total_steps), total_steps)
    kw = {"warmup_steps": warm}
    rest = total_steps - warm
    if schedule_type == "cosine":
        kw["lr_decay_steps"] = rest
    elif schedule_type == "sgdr":
        kw["cycle_length"] = cycle_length or rest
        kw["t_mult"] = t_mult
    elif schedule_type == "wsd":
        st = stable_steps or max(1, int(rest * 0.8))
        kw["stable_steps"] = st
        kw["decay_steps"] = max(1, decay_steps or (rest - st))
    if min_rate is not None:
        kw["min_rate"] = min_rate
    return kw


def build_config(args: argparse.Namespace):
    from astrai_b200.config import AutoRegressiveLMConfig, TrainConfig
    from astrai_b200.dataset import DatasetFactory, dpo_collate_fn, grpo_collate_fn
    from astrai_b200.models import AutoRegressiveLM, DecoderBlock
    from astrai_b200.optim import MuonMix
    from astrai_b200.trainer import SchedulerFactory

    if not os.path.exists(args.param_path):
        raise FileNotFoundError(args.param_path)
    if args.nprocs > 1 and args.parallel_mode == "none":
        raise ValueError("--nprocs > 1 requires --parallel_mode to be 'ddp', 'fsdp', or 'fsdp2'")
    config = AutoRegressiveLMConfig.from_file(os.path.join(args.param_path, "config.json"))
    config.neftune_alpha = args.neftune_alpha
    window = args.window_size or config.max_position_embeddings
    dataset = DatasetFactory.load(train_type=args.train_type, load_path=args.data_root_path, window_size=window,
                                  stride=args.stride, tokenizer_path=args.param_path)
    total = compute_total_steps(len(dataset), args.n_epoch, args.batch_per_device, args.nprocs,
                                args.grad_accum_steps)
    skw = scheduler_kwargs(args.schedule_type, total, args.warmup_ratio, args.min_rate, args.cycle_length,
                           args.t_mult, args.stable_steps, args.decay_steps)
    collate = {"dpo": dpo_collate_fn, "grpo": grpo_collate_fn}.get(args.train_type)
    executor_kwargs = {}
    if args.parallel_mode == "ddp":
        executor_kwargs.update(comm_backend=args.comm_backend, expert_parallel=args.expert_parallel)
    return TrainConfig(
        model_fn=lambda: AutoRegressiveLM(config).to(dtype=torch.bfloat16),
        strategy=args.train_type, dataset=dataset,
        optimizer_fn=partial(MuonMix, lr=args.max_lr, weight_decay=args.weight_decay, momentum=args.muon_momentum,
                             nesterov=args.muon_nesterov, ns_steps=args.muon_ns_steps,
                             adjust_lr_fn=args.muon_adjust_lr, shard_muon=args.shard_muon),
        scheduler_fn=lambda o: SchedulerFactory.create(args.schedule_type, o, **skw),
        ckpt_dir=args.ckpt_dir, n_epoch=args.n_epoch, batch_per_device=args.batch_per_device,
        start_epoch=args.start_epoch, start_samples=args.start_samples, ckpt_interval=args.ckpt_interval,
        grad_accum_steps=args.grad_accum_steps, max_grad_norm=args.max_grad_norm, random_seed=args.random_seed,
        num_workers=args.num_workers, pin_memory=args.pin_memory, nprocs=args.nprocs, backend=args.backend,
        master_addr=args.master_addr, master_port=args.master_port, parallel_mode=args.parallel_mode,
        device_type=args.device_type, start_method=args.start_method, val_split=args.val_split,
        val_step=args.val_step, metrics=args.metrics, log_dir=args.log_dir,
        gradient_checkpointing_modules=[DecoderBlock] if args.gradient_checkpointing else [],
        executor_kwargs=executor_kwargs,
        extra_kwargs={"beta": args.dpo_beta, "label_smoothing": args.label_smoothing, "clip_eps": args.grpo_clip_eps,
                      "kl_coef": args.grpo_kl_coef, "group_size": args.group_size},
        neftune_alpha=args.neftune_alpha, collate_fn=collate, rollout_interval=args.rollout_interval,
        rollout_temperature=args.rollout_temperature, rollout_top_k=args.rollout_top_k,
        rollout_top_p=args.rollout_top_p, rollout_max_tokens=args.rollout_max_tokens,
        comm_backend=args.comm_backend, profile_dir=args.profile_dir,
    )


def main(argv: Optional[List[str]] = None) -> None:
    from astrai_b200.trainer import Trainer

    args = parse_args(argv)
    Trainer(build_config(args)).train(param_path=args.param_path, resume=args.resume)


if __name__ == "__main__":
    main()
