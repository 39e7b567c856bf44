"""Token-shard files for datasets.

Two formats, matching the reference's on-disk layout
(astrai/serialization/dataset.py:14-123):

* ``bin``: ``<dir>/<key>.bin`` raw little-endian arrays + ``meta.json``
  ``{key: {"shape": [...], "dtype": "int32", "offsets": [...]?}}``. Keys listed
  in ``record_keys`` carry cumulative per-record offsets so single records can
  be sliced out of the concatenation. Loaded with ``np.memmap`` (copy-on-write)
  so shards larger than RAM stream from the page cache.
* ``h5``: one group per key, datasets ``data_{i}``. Needs ``h5py``; this image
  has none, so the functions raise a clear ImportError when it is missing.
"""

from __future__ import annotations

import json
import os
from pathlib import Path
from typing import Any, Dict, List, Optional

import numpy as np
import torch

try:  # optional dependency
    import h5py  # type: ignore
except Exception:  # pragma: no cover - exercised only where h5py is absent
    h5py = None


def _need_h5py():
    if h5py is None:
        raise ImportError("h5py is not installed; use the 'bin' or 'jsonl' storage format")


def save_h5(file_path: str, file_name: str, tensor_group: Dict[str, List[torch.Tensor]]) -> None:
    _need_h5py()
    os.makedirs(file_path, exist_ok=True)
    with h5py.File(os.path.join(file_path, f"{file_name}.h5"), "w") as f:
        for key, ts in tensor_group.items():
            g = f.create_group(key)
            for i, t in enumerate(ts):
                g.create_dataset(f"data_{i}", data=t.cpu().numpy())


def load_h5(file_path: str, share_memory: bool = True) -> Dict[str, List[torch.Tensor]]:
    _need_h5py()
    root = Path(file_path)
    files = [root] if root.is_file() else sorted(list(root.rglob("*.h5")) + list(root.rglob("*.hdf5")))
    out: Dict[str, List[torch.Tensor]] = {}
    for fp in files:
        with h5py.File(fp, "r") as f:
            for key in f.keys():
                g = f[key]
                names = sorted(g.keys(), key=lambda s: int(s.split("_")[-1]) if s.split("_")[-1].isdigit() else s)
                for n in names:
                    t = torch.from_numpy(g[n][:])
                    out.setdefault(key, []).append(t.share_memory_() if share_memory else t)
    return out


def save_bin(file_path: str, tensor_group: Dict[str, List[torch.Tensor]], record_keys: Optional[List[str]] = None) -> None:
    os.makedirs(file_path, exist_ok=True)
    rec = set(record_keys or ())
    meta: Dict[str, Any] = {}
    for key, ts in tensor_group.items():
        if ts and isinstance(ts[0], list):
            raise ValueError(f"Nested key '{key}' cannot be stored in bin format; use h5 or jsonl")
        cat = torch.cat([t.reshape(-1) if t.dim() == 0 else t for t in ts], 0) if ts else torch.zeros(0, dtype=torch.int32)
        entry: Dict[str, Any] = {"shape": list(cat.shape), "dtype": str(cat.dtype).rsplit(".", 1)[-1]}
        if key in rec:
            offs = [0]
            for t in ts:
                offs.append(offs[-1] + int(t.shape[0]))
            entry["offsets"] = offs
        meta[key] = entry
        cat.cpu().numpy().tofile(os.path.join(file_path, f"{key}.bin"))
    with open(os.path.join(file_path, "meta.json"), "w") as fh:
        json.dump(meta, fh)


def load_bin(file_path: str) -> Dict[str, List[torch.Tensor]]:
    with open(os.path.join(file_path, "meta.json")) as fh:
        meta = json.load(fh)
    out: Dict[str, List[torch.Tensor]] = {}
    for key, info in meta.items():
        shape = tuple(info["shape"])
        if int(np.prod(shape)) == 0:
            out[key] = [torch.zeros(shape, dtype=getattr(torch, info["dtype"]))]
            continue
        arr = np.memmap(os.path.join(file_path, f"{key}.bin"), dtype=info["dtype"], mode="c", shape=shape)
        out[key] = [torch.from_numpy(arr)]
    return out


def load_bin_offsets(file_path: str) -> Dict[str, List[int]]:
    with open(os.path.join(file_path, "meta.json")) as fh:
        meta = json.load(fh)
    return {k: v["offsets"] for k, v in meta.items() if "offsets" in v}
