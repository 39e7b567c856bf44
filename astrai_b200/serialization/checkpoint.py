"""Model and checkpoint files.

On-disk layout (shared with the reference so directories are interchangeable,
astrai/serialization/checkpoint.py:137-201):

    <dir>/config.json         model config
    <dir>/model.safetensors   full (unsharded) state dict
    <dir>/meta.json           epoch, consumed_samples, timestamp, + train config
    <dir>/<name>.pt           extra objects (optimizer, scheduler, ...)

Loads can be "rank-0 reads, everyone receives": with ``broadcast=True`` and an
initialised process group only rank 0 touches the file system. Tensors are
broadcast one by one (after a spec list) so no rank has to pickle the whole
model.
"""

from __future__ import annotations

import io
import json
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Dict, Optional, Union

import safetensors.torch as sft
import torch
import torch.distributed as dist

META_FILE = "meta.json"
CONFIG_FILE = "config.json"
WEIGHTS_FILE = "model.safetensors"

PathLike = Union[str, Path]


def _dist_on() -> bool:
    return dist.is_available() and dist.is_initialized()


def _rank() -> int:
    return dist.get_rank() if _dist_on() else 0


def _bcast_obj(obj: Any) -> Any:
    box = [obj]
    dist.broadcast_object_list(box, src=0)
    return box[0]


# ---------------------------------------------------------------- primitives
def save_safetensors(state_dict: Dict[str, torch.Tensor], path: PathLike) -> None:
    # safetensors refuses shared storage; tied weights are removed by the model
    clean = {k: v.detach().contiguous().cpu() for k, v in state_dict.items()}
    sft.save_file(clean, str(path))


def load_safetensors(path: PathLike, broadcast: bool = False) -> Dict[str, torch.Tensor]:
    if not (broadcast and _dist_on()):
        return sft.load_file(str(path))
    return _bcast_obj(sft.load_file(str(path)) if _rank() == 0 else None)


def save_json(data: Dict[str, Any], path: PathLike) -> None:
    with open(path, "w", encoding="utf-8") as fh:
        json.dump(data, fh, indent=2, ensure_ascii=False)


def load_json(path: PathLike, broadcast: bool = False) -> Dict[str, Any]:
    def read():
        with open(path, "r", encoding="utf-8") as fh:
            return json.load(fh)

    if not (broadcast and _dist_on()):
        return read()
    return _bcast_obj(read() if _rank() == 0 else None)


def save_torch(obj: Any, path: PathLike) -> None:
    torch.save(obj, str(path))


def load_torch(path: PathLike, broadcast: bool = False) -> Any:
    if not (broadcast and _dist_on()):
        return torch.load(str(path), map_location="cpu", weights_only=False)
    if _rank() == 0:
        blob = Path(path).read_bytes()
        n = torch.tensor([len(blob)], dtype=torch.long)
    else:
        blob, n = None, torch.zeros(1, dtype=torch.long)
    dist.broadcast(n, src=0)
    buf = torch.frombuffer(bytearray(blob), dtype=torch.uint8) if blob is not None else torch.empty(int(n.item()), dtype=torch.uint8)
    dist.broadcast(buf, src=0)
    return torch.load(io.BytesIO(buf.numpy().tobytes()), map_location="cpu", weights_only=False)


def load_state_dict(path: PathLike, broadcast: bool = False) -> Dict[str, torch.Tensor]:
    """Read a safetensors file; with ``broadcast`` only rank 0 reads it."""
    if not (broadcast and _dist_on()):
        return sft.load_file(str(path))
    sd = sft.load_file(str(path)) if _rank() == 0 else {}
    specs = _bcast_obj([(k, tuple(v.shape), str(v.dtype).rsplit(".", 1)[-1]) for k, v in sorted(sd.items())] if _rank() == 0 else None)
    out: Dict[str, torch.Tensor] = {}
    for name, shape, dt in specs:
        t = sd[name].contiguous() if _rank() == 0 else torch.empty(shape, dtype=getattr(torch, dt))
        dist.broadcast(t, src=0)
        out[name] = t
    return out


def save_model(config: Dict[str, Any], state_dict: Dict[str, torch.Tensor], save_directory: PathLike) -> None:
    d = Path(save_directory)
    d.mkdir(parents=True, exist_ok=True)
    save_json(config, d / CONFIG_FILE)
    save_safetensors(state_dict, d / WEIGHTS_FILE)


def load_model_config(save_directory: PathLike) -> Dict[str, Any]:
    return load_json(Path(save_directory) / CONFIG_FILE)


def load_model_weights(save_directory: PathLike) -> Dict[str, torch.Tensor]:
    return load_state_dict(Path(save_directory) / WEIGHTS_FILE)


# ---------------------------------------------------------------- checkpoint
@dataclass
class Checkpoint:
    state_dict: Dict[str, Any] = field(default_factory=dict)
    epoch: int = 0
    consumed_samples: int = 0
    extra: Dict[str, Any] = field(default_factory=dict)
    meta: Dict[str, Any] = field(default_factory=dict)
    config: Dict[str, Any] = field(default_factory=dict)

    def save(self, save_dir: PathLike) -> None:
        d = Path(save_dir)
        d.mkdir(parents=True, exist_ok=True)
        meta = {
            "epoch": self.epoch,
            "consumed_samples": self.consumed_samples,
            "timestamp": time.strftime("%Y-%m-%dT%H:%M:%S"),
        }
        meta.update(self.meta)
        save_json(meta, d / META_FILE)
        save_json(self.config, d / CONFIG_FILE)
        save_safetensors(self.state_dict, d / WEIGHTS_FILE)
        for name, obj in self.extra.items():
            save_torch(obj, d / f"{name}.pt")

    @classmethod
    def load(cls, save_dir: PathLike, broadcast: bool = False) -> "Checkpoint":
        d = Path(save_dir)
        meta = load_json(d / META_FILE, broadcast)
        config = load_json(d / CONFIG_FILE, broadcast) if (d / CONFIG_FILE).exists() else {}
        sd = load_state_dict(d / WEIGHTS_FILE, broadcast)
        extra = {p.stem: load_torch(p, broadcast) for p in sorted(d.glob("*.pt"))}
        return cls(
            state_dict=sd,
            epoch=meta.get("epoch", 0),
            consumed_samples=meta.get("consumed_samples", 0),
            extra=extra,
            meta=meta,
            config=config,
        )

    @classmethod
    def load_any(cls, save_dir: PathLike, broadcast: bool = False) -> Optional["Checkpoint"]:
        """A full checkpoint, a bare model directory, or None."""
        d = Path(save_dir)
        if (d / META_FILE).exists():
            return cls.load(d, broadcast)
        if (d / WEIGHTS_FILE).exists():
            cfg = load_json(d / CONFIG_FILE, broadcast) if (d / CONFIG_FILE).exists() else {}
            return cls(state_dict=load_state_dict(d / WEIGHTS_FILE, broadcast), config=cfg)
        return None
