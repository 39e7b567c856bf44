"""Model registry plus ``from_pretrained`` / ``save_pretrained``.

Interface kept from the reference (astrai/model/automodel.py:16-95): ``AutoModel`` is both the
base class of the model families and their registry (``@AutoModel.register("...")``, keyed by
``config.json``'s ``model_type``), ``from_pretrained(path, disable_random_init=True,
strict=True)`` and ``save_pretrained(dir)`` over ``config.json`` + ``model.safetensors``.

Loading without paying for random init: the model is built on the ``meta`` device (no memory,
no init kernels), moved to real but uninitialised storage with ``to_empty``, and then filled.
Two things do not survive ``to_empty`` and are restored explicitly: parameters shared between
modules (a model lists them in :meth:`AutoModel.tied_parameters`) and non-persistent buffers
computed at construction (modules that own one implement ``reset_buffers()``).
``device`` / ``dtype`` place a large model directly where it will run.
"""

from __future__ import annotations

from pathlib import Path
from typing import List, Optional, Tuple, Union

import torch
import torch.nn as nn

from astrai_b200.config.model_config import BaseModelConfig, ConfigFactory
from astrai_b200.factory import Registry
from astrai_b200.serialization import load_model_config, load_model_weights, save_model

CONFIG_FILE = "config.json"
WEIGHTS_FILE = "model.safetensors"


def _materialise(model: nn.Module, device: torch.device) -> nn.Module:
    """meta-device ``model`` -> uninitialised storage on ``device``, with ties and computed buffers restored."""
    ties = model.tied_parameters() if isinstance(model, AutoModel) else []
    model.to_empty(device=device)
    for dst, src in ties:
        owner, _, name = dst.rpartition(".")
        setattr(model.get_submodule(owner) if owner else model, name, model.get_parameter(src))
    for m in model.modules():
        if hasattr(m, "reset_buffers"):
            m.reset_buffers()
    return model


class AutoModel(Registry, nn.Module):
    _self_base = True

    def __init__(self, config: BaseModelConfig):
        nn.Module.__init__(self)
        self.config = config

    def tied_parameters(self) -> List[Tuple[str, str]]:
        """``(alias, source)`` parameter paths that must stay one tensor; none by default."""
        return []

    @classmethod
    def from_pretrained(cls, path: Union[str, Path], disable_random_init: bool = True, strict: bool = True,
                        device: Optional[Union[str, torch.device]] = None,
                        dtype: Optional[torch.dtype] = None) -> nn.Module:
        """Build the model that ``path/config.json`` describes and load ``path/model.safetensors``
        into it (a missing weights file leaves the random init, or uninitialised memory when
        ``disable_random_init`` is set, which only makes sense with weights to load)."""
        src = Path(path)
        if not (src / CONFIG_FILE).is_file():
            raise FileNotFoundError(f"{src}: no {CONFIG_FILE}, so this is not a saved model directory")
        config = ConfigFactory.load(load_model_config(str(src)))
        family = AutoModel.get_component_class(config.model_type or "autoregressive_lm")
        target = torch.device(device) if device is not None else torch.device("cpu")
        if disable_random_init:
            with torch.device("meta"):
                model = family(config)
            _materialise(model, target)
        else:
            with torch.device(target):
                model = family(config)
        if (src / WEIGHTS_FILE).is_file():
            model.load_state_dict(load_model_weights(str(src)), strict=strict)
        return model if dtype is None else model.to(dtype=dtype)

    def save_pretrained(self, save_directory: Union[str, Path]) -> None:
        save_model(config=self.config.to_dict(), state_dict=self.state_dict(), save_directory=str(save_directory))
