from astrai_b200.serialization.checkpoint import (
    Checkpoint,
    load_json,
    load_model_config,
    load_model_weights,
    load_safetensors,
    load_state_dict,
    load_torch,
    save_json,
    save_model,
    save_safetensors,
    save_torch,
)
from astrai_b200.serialization.dataset import load_bin, load_bin_offsets, load_h5, save_bin, save_h5

__all__ = [
    "Checkpoint",
    "load_json",
    "load_model_config",
    "load_model_weights",
    "load_safetensors",
    "load_state_dict",
    "load_torch",
    "save_json",
    "save_model",
    "save_safetensors",
    "save_torch",
    "load_bin",
    "load_bin_offsets",
    "load_h5",
    "save_bin",
    "save_h5",
]
