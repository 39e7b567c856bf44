"""Training configuration.

Field names, defaults and the required-field validation follow the reference
``TrainConfig`` (astrai/config/train_config.py:17-181), because the CLI, the
checkpoint ``meta.json`` (which embeds ``to_dict()``) and user scripts depend
on them. Fields added here: ``comm_backend`` (``"nccl"`` or ``"fused"``: who
moves gradients between GPUs), ``cuda_graph`` (replay each micro-step's forward
and backward from a CUDA graph, for fixed-shape batches on the seq / sft
strategies) and ``profile_dir`` (torch.profiler trace output).
"""

from __future__ import annotations

from dataclasses import dataclass, field, fields
from typing import Any, Callable, Dict, List, Optional

from astrai_b200.config.base import BaseConfig
from astrai_b200.models.components.lora import LoRAConfig


def _req(**kw):
    return {"required": True, **kw}


@dataclass
class TrainConfig(BaseConfig):
    model_fn: Callable = field(default=None, metadata=_req(help="Builds the model."))
    strategy: str = field(default=None, metadata=_req(help="Training strategy name."))
    dataset: Any = field(default=None, metadata=_req(help="Training dataset."))
    optimizer_fn: Callable = field(default=None, metadata=_req(help="Builds the optimizer."))
    scheduler_fn: Callable = field(default=None, metadata=_req(help="Builds the LR scheduler."))
    n_epoch: int = 1
    batch_per_device: int = 4
    grad_accum_steps: int = 1
    max_grad_norm: Optional[float] = 1.0
    gradient_checkpointing_modules: List[Any] = field(default_factory=list)
    start_epoch: int = 0
    start_samples: int = 0
    ckpt_dir: str = "./checkpoint"
    ckpt_interval: int = 5000
    lora: Optional[LoRAConfig] = None
    log_dir: str = "./checkpoint/logs"
    metrics: List[str] = field(default_factory=lambda: ["loss", "lr", "grad_norm"])
    random_seed: int = 3407
    num_workers: int = 0
    prefetch_factor: Optional[int] = None
    pin_memory: bool = False
    collate_fn: Optional[Callable] = None
    nprocs: int = 1
    backend: str = "nccl"
    master_addr: str = "localhost"
    master_port: str = "29500"
    parallel_mode: str = "none"
    start_method: str = "spawn"
    device_type: str = "cuda"
    val_dataset: Any = None
    val_split: Optional[float] = None
    val_step: int = 1000
    neftune_alpha: float = 0.0
    rollout_interval: int = 512
    rollout_temperature: float = 0.7
    rollout_top_k: int = 0
    rollout_top_p: float = 0.9
    rollout_max_tokens: int = 1024
    reward_model_fn: Optional[Callable] = None
    executor_kwargs: Dict[str, Any] = field(default_factory=dict)
    extra_kwargs: Dict[str, Any] = field(default_factory=dict)
    # additions
    comm_backend: str = "nccl"
    cuda_graph: bool = False
    profile_dir: Optional[str] = None

    def __post_init__(self):
        self.validate()

    def validate(self) -> None:
        for f in fields(self):
            if f.metadata.get("required") and getattr(self, f.name) is None:
                raise ValueError(f"TrainConfig.{f.name} is required but got None.")
