"""Model registry, ``from_pretrained`` / ``save_pretrained``.

Parity: astrai/model/automodel.py:16-95. ``from_pretrained(path)`` reads
``config.json``, picks the config class by ``model_type`` and the model class
from this registry, builds it with random init disabled (weights are about to
be overwritten) and loads ``model.safetensors``. Adds ``device``/``dtype``
arguments so large models are built directly where they will run.
"""

from __future__ import annotations

from contextlib import contextmanager
from pathlib import Path
from typing import Optional, Union

import torch
import torch.nn as nn

from astrai_b200.config.model_config import BaseModelConfig, ConfigFactory
from astrai_b200.factory import Registry
from astrai_b200.serialization import load_model_config, load_model_weights, save_model

_INIT_FNS = ("xavier_normal_", "xavier_uniform_", "kaiming_normal_", "kaiming_uniform_", "zeros_", "ones_",
             "constant_", "normal_", "uniform_", "trunc_normal_")


@contextmanager
def disable_random_init(enable: bool = True):
    """Turn nn.init.* into no-ops while a model whose weights will be loaded is built."""
    if not enable:
        yield
        return
    saved = {n: getattr(nn.init, n) for n in _INIT_FNS if hasattr(nn.init, n)}
    for n in saved:
        setattr(nn.init, n, lambda *a, **k: a[0] if a else None)
    try:
        yield
    finally:
        for n, fn in saved.items():
            setattr(nn.init, n, fn)


class AutoModel(Registry, nn.Module):
    _self_base = True

    def __init__(self, config: BaseModelConfig):
        nn.Module.__init__(self)
        self.config = config

    @classmethod
    def from_pretrained(cls, path: Union[str, Path], disable_random_init: bool = True, strict: bool = True,
                        device: Optional[Union[str, torch.device]] = None,
                        dtype: Optional[torch.dtype] = None) -> nn.Module:
        p = Path(path)
        if not (p / "config.json").exists():
            raise FileNotFoundError(f"Config file not found: {p / 'config.json'}")
        config = ConfigFactory.load(load_model_config(str(p)))
        model_cls = AutoModel.get_component_class(config.model_type or "autoregressive_lm")
        with _maybe_device(device), globals()["disable_random_init"](disable_random_init):
            model = model_cls(config)
        if (p / "model.safetensors").exists():
            model.load_state_dict(load_model_weights(str(p)), strict=strict)
        if dtype is not None:
            model = model.to(dtype=dtype)
        return model

    def save_pretrained(self, save_directory: Union[str, Path]) -> None:
        save_model(config=self.config.to_dict(), state_dict=self.state_dict(), save_directory=str(save_directory))


@contextmanager
def _maybe_device(device):
    if device is None:
        yield
    else:
        with torch.device(device):
            yield
