"""Low-rank adapters on the model's projections.

Interface kept from the reference (astrai/model/components/lora.py:24-198), because adapter
files move between the two frameworks: ``LoRAConfig(r, alpha, target_modules)``, the
``LoRALinear`` parameter names (``weight``, ``bias``, ``lora_A`` [r, in], ``lora_B`` [out, r]),
the initialisation (A ~ N(0, 1) / r, B = 0, so an adapter starts as the identity), the update
``y = x W^T + (x A^T) B^T * alpha / r``, and the adapter files ``adapter_model.safetensors``
(only the ``*.lora_A`` / ``*.lora_B`` tensors) + ``adapter_config.json``.

Design here: adapters are attached by :func:`_swap_children`, one walk over the module tree
that replaces every :class:`Linear` whose attribute name is targeted. An adapter's merged state
is simply "its low-rank parameters are gone": :meth:`LoRALinear.merge` folds ``B A * scale`` into
the frozen weight in fp32 and deletes them, so a merged model saves like a plain one. All
products run on the framework's GEMM (`ops.gemm.linear`), the residual add of the
o/down projections included.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass
from pathlib import Path
from typing import Callable, Dict, Iterable, List, Optional, Set, Tuple

import torch
import torch.nn as nn

from astrai_b200.models.components.basic import Linear
from astrai_b200.ops.gemm import linear as _linear
from astrai_b200.serialization import load_json, load_safetensors, save_json, save_safetensors

logger = logging.getLogger(__name__)

TARGET_MODULES_ATTN = {"q_proj", "k_proj", "v_proj", "o_proj"}
TARGET_MODULES_FFN = {"up", "gate", "down"}

ADAPTER_WEIGHTS = "adapter_model.safetensors"
ADAPTER_CONFIG = "adapter_config.json"
_ADAPTER_SUFFIXES = (".lora_A", ".lora_B")


@dataclass
class LoRAConfig:
    r: int = 16
    alpha: int = 32
    target_modules: tuple = ("q_proj", "v_proj")

    def to_json(self) -> Dict:
        return {"r": int(self.r), "alpha": self.alpha, "target_modules": list(self.target_modules)}

    @classmethod
    def from_json(cls, d: Dict) -> "LoRAConfig":
        return cls(r=int(d["r"]), alpha=d["alpha"], target_modules=tuple(d["target_modules"]))


class LoRALinear(nn.Module):
    """A frozen projection plus a trainable rank-``r`` update scaled by ``alpha / r``."""

    def __init__(self, base: Linear, r: int = 16, alpha: int = 32):
        super().__init__()
        self.weight = base.weight
        self.bias = base.bias
        for p in (self.weight, self.bias):
            if p is not None:
                p.requires_grad_(False)
        self.r = r
        self.scaling = alpha / r
        n_out, n_in = self.weight.shape
        like = {"device": self.weight.device, "dtype": self.weight.dtype}
        self.lora_A = nn.Parameter(torch.randn(r, n_in, **like) / r)
        self.lora_B = nn.Parameter(torch.zeros(n_out, r, **like))

    @property
    def merged(self) -> bool:
        return "lora_A" not in self._parameters

    # the reference exposes the flag as a private attribute; keep it readable
    _merged = merged

    def delta_weight(self) -> torch.Tensor:
        """The adapter's contribution to the weight, ``B @ A * alpha / r`` in fp32."""
        return (self.lora_B.float() @ self.lora_A.float()) * self.scaling

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        y = _linear(x, self.weight, residual=residual, bias=self.bias)
        if self.merged:
            return y
        return y + _linear(_linear(x, self.lora_A), self.lora_B) * self.scaling

    @torch.no_grad()
    def merge(self) -> None:
        """Fold the update into ``weight`` (in fp32, then cast back) and drop the adapter."""
        if self.merged:
            return
        self.weight.copy_((self.weight.float() + self.delta_weight()).to(self.weight.dtype))
        del self.lora_A, self.lora_B


def _swap_children(model: nn.Module, wanted: Callable[[str, nn.Module], bool],
                   make: Callable[[nn.Module], nn.Module]) -> List[str]:
    """Replace every child module for which ``wanted(attribute name, module)`` holds by
    ``make(module)``; returns the dotted paths that were replaced."""
    hits: List[Tuple[nn.Module, str, str]] = []
    for path, mod in model.named_modules():
        parent, _, attr = path.rpartition(".")
        if path and wanted(attr, mod):
            hits.append((model.get_submodule(parent) if parent else model, attr, path))
    for owner, attr, _ in hits:
        setattr(owner, attr, make(getattr(owner, attr)))
    return [p for _, _, p in hits]


def _adapters(model: nn.Module) -> Iterable[LoRALinear]:
    return (m for m in model.modules() if isinstance(m, LoRALinear))


def lora_count(model: nn.Module) -> int:
    """Number of adapted projections that are not merged yet."""
    return sum(not m.merged for m in _adapters(model))


def inject_lora(model: nn.Module, r: int = 16, alpha: int = 32,
                target_modules: Optional[Set[str]] = None) -> LoRAConfig:
    """Wrap every :class:`Linear` child named in ``target_modules`` (default: the attention
    projections) with a :class:`LoRALinear`; returns the config to save with the adapter."""
    targets = set(TARGET_MODULES_ATTN if target_modules is None else target_modules)
    done = _swap_children(model, lambda attr, m: attr in targets and isinstance(m, Linear),
                          lambda m: LoRALinear(m, r=r, alpha=alpha))
    if not done:
        present = sorted({p.rpartition(".")[2] for p, m in model.named_modules() if isinstance(m, Linear)})
        logger.warning("inject_lora: none of %s names a Linear of this model (its Linear names: %s)",
                       sorted(targets), present)
    return LoRAConfig(r=r, alpha=alpha, target_modules=tuple(sorted(targets)))


def merge_lora(model: nn.Module) -> None:
    """Fold every live adapter into its base weight."""
    live = [m for m in _adapters(model) if not m.merged]
    for m in live:
        m.merge()
    if not live:
        logger.warning("merge_lora: the model has no unmerged adapter")


def save_lora(model: nn.Module, save_dir: str, config: LoRAConfig) -> None:
    """Write the adapter tensors and their config into ``save_dir``."""
    tensors = {k: v for k, v in model.state_dict().items() if k.endswith(_ADAPTER_SUFFIXES)}
    if not tensors:
        raise RuntimeError("save_lora: nothing to save; inject adapters first (merged adapters are part of "
                           "the base weights and are saved with the model)")
    out = Path(save_dir)
    out.mkdir(parents=True, exist_ok=True)
    save_safetensors(tensors, out / ADAPTER_WEIGHTS)
    save_json(config.to_json(), out / ADAPTER_CONFIG)


def load_lora(model: nn.Module, load_dir: str) -> LoRAConfig:
    """Attach (if needed) and load the adapter saved in ``load_dir``; returns its config."""
    src = Path(load_dir)
    config = LoRAConfig.from_json(load_json(src / ADAPTER_CONFIG))
    if lora_count(model) == 0:
        inject_lora(model, r=config.r, alpha=config.alpha, target_modules=set(config.target_modules))
    if lora_count(model) == 0:
        raise RuntimeError(f"load_lora: the adapter targets {list(config.target_modules)}, which match no "
                           "projection of this model")
    tensors = load_safetensors(src / ADAPTER_WEIGHTS)
    own = {k for k in model.state_dict() if k.endswith(_ADAPTER_SUFFIXES)}
    absent = sorted(own - set(tensors))
    if absent:
        raise RuntimeError(f"load_lora: {ADAPTER_WEIGHTS} has no tensor for {absent}")
    try:
        model.load_state_dict(tensors, strict=False)
    except RuntimeError as err:
        raise RuntimeError(f"load_lora: adapter shapes do not fit this model (saved with r={config.r}): "
                           f"{err}") from err
    return config
