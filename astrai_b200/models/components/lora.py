"""Low-rank adapters (parity: astrai/model/components/lora.py:24-198).

``LoRALinear`` wraps a frozen ``Linear``: ``y = W x + (B (A x)) * alpha / r``
with ``A ~ N(0,1)/r`` and ``B = 0``; ``inject_lora`` replaces children whose
attribute name is in ``target_modules``; ``merge_lora`` folds the update into
W; adapters are saved as ``adapter_model.safetensors`` (keys ending in
``.lora_A`` / ``.lora_B``) plus ``adapter_config.json`` (``r``, ``alpha``,
``target_modules``) - the reference's adapter format.
"""

from __future__ import annotations

import logging
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Optional, Set

import torch
import torch.nn as nn

from astrai_b200.models.components.basic import Linear
from astrai_b200.ops.gemm import linear as _linear
from astrai_b200.serialization import load_json, load_safetensors, save_json, save_safetensors

logger = logging.getLogger(__name__)

TARGET_MODULES_ATTN = {"q_proj", "k_proj", "v_proj", "o_proj"}
TARGET_MODULES_FFN = {"up", "gate", "down"}


@dataclass
class LoRAConfig:
    r: int = 16
    alpha: int = 32
    target_modules: tuple = ("q_proj", "v_proj")


class LoRALinear(nn.Module):
    def __init__(self, base: Linear, r: int = 16, alpha: int = 32):
        super().__init__()
        self.register_parameter("weight", base.weight)
        self.weight.requires_grad_(False)
        self.bias = base.bias
        if self.bias is not None:
            self.bias.requires_grad_(False)
        self.r = r
        self.scaling = alpha / r
        dev, dt = self.weight.device, self.weight.dtype
        self.lora_A = nn.Parameter(torch.randn(r, self.weight.shape[1], device=dev, dtype=dt) / r)
        self.lora_B = nn.Parameter(torch.zeros(self.weight.shape[0], r, device=dev, dtype=dt))
        self._merged = False

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        out = _linear(x, self.weight, residual=residual, bias=self.bias)
        if not self._merged:
            out = out + _linear(_linear(x, self.lora_A), self.lora_B) * self.scaling
        return out

    @torch.no_grad()
    def merge(self) -> None:
        if self._merged:
            return
        self.weight.data += (self.lora_B.float() @ self.lora_A.float() * self.scaling).to(self.weight.dtype)
        self._merged = True
        del self.lora_A
        del self.lora_B


def _linear_children(model: nn.Module) -> dict:
    names: dict = {}
    for n, m in model.named_modules():
        if isinstance(m, Linear):
            names.setdefault(n.rpartition(".")[2], []).append(n)
    return names


def lora_count(model: nn.Module) -> int:
    return sum(1 for m in model.modules() if isinstance(m, LoRALinear))


def inject_lora(model: nn.Module, r: int = 16, alpha: int = 32, target_modules: Optional[Set[str]] = None) -> LoRAConfig:
    targets = set(target_modules) if target_modules is not None else set(TARGET_MODULES_ATTN)
    injected = 0
    for name, module in list(model.named_modules()):
        if not isinstance(module, Linear):
            continue
        parent_name, _, child = name.rpartition(".")
        if child not in targets:
            continue
        parent = model.get_submodule(parent_name) if parent_name else model
        setattr(parent, child, LoRALinear(module, r=r, alpha=alpha))
        injected += 1
    if injected == 0:
        logger.warning("No LoRA layers injected. Available Linear names: %s; targets: %s",
                       sorted(_linear_children(model)), sorted(targets))
    return LoRAConfig(r=r, alpha=alpha, target_modules=tuple(sorted(targets)))


def merge_lora(model: nn.Module) -> None:
    n = 0
    for m in model.modules():
        if isinstance(m, LoRALinear):
            m.merge()
            n += 1
    if n == 0:
        logger.warning("No LoRA layers to merge.")


def save_lora(model: nn.Module, save_dir: str, config: LoRAConfig) -> None:
    sd = {k: v for k, v in model.state_dict().items() if k.endswith((".lora_A", ".lora_B"))}
    if not sd:
        raise RuntimeError("No LoRA parameters found in model (not injected, or already merged).")
    p = Path(save_dir)
    p.mkdir(parents=True, exist_ok=True)
    save_safetensors(sd, p / "adapter_model.safetensors")
    cfg = asdict(config)
    cfg["target_modules"] = list(cfg["target_modules"])
    save_json(cfg, p / "adapter_config.json")


def load_lora(model: nn.Module, load_dir: str) -> LoRAConfig:
    p = Path(load_dir)
    raw = load_json(p / "adapter_config.json")
    config = LoRAConfig(r=raw["r"], alpha=raw["alpha"], target_modules=tuple(raw["target_modules"]))
    if lora_count(model) == 0:
        inject_lora(model, r=config.r, alpha=config.alpha, target_modules=set(config.target_modules))
    weights = load_safetensors(p / "adapter_model.safetensors")
    try:
        missing, _ = model.load_state_dict(weights, strict=False)
    except RuntimeError as e:
        if "size mismatch" in str(e):
            raise RuntimeError(f"LoRA weight shapes do not match the model (r={config.r}): {e}") from e
        raise
    if lora_count(model) == 0:
        raise RuntimeError("No LoRA layers found after loading.")
    lora_missing = [k for k in missing if "lora" in k]
    if lora_missing:
        raise RuntimeError(f"LoRA weight keys not found in model: {lora_missing}")
    return config
