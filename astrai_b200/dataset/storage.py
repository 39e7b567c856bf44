"""Token stores (parity: astrai/dataset/storage.py:71-664).

A store owns the tokens of a dataset and the sample-index arithmetic:

* stream mode (``window_size > 0``): all shards form one token stream; the
  number of samples is ``(total - 1 - w) // stride + 1`` and sample ``i``
  covers ``[begin, begin + w)`` with ``begin = min(i * stride, total - 1 - w)``
  (the +1 leaves room for the shifted next-token target). Slices spanning
  shards are stitched by bisecting cumulative shard lengths - shards are
  never concatenated in memory.
* record mode: per-record tensors (H5 / JSONL segments, or ``bin`` shards
  whose ``meta.json`` carries per-record offsets); ``len`` = record count.

Backends: ``bin`` (``np.memmap`` shards shared by all DataLoader workers
through the page cache), ``h5`` (requires h5py), ``jsonl`` (eager
tokenisation through a :class:`TokenizeTransform`, a ``dataset_config.json``
next to the files, the built-in chat ``messages`` config, or lazy per-record
tokenisation with ``processor=``). ``detect_format`` picks the backend from
the files present.
"""

from __future__ import annotations

import bisect
import json
import logging
from pathlib import Path
from typing import Callable, Dict, List, Optional, Tuple, Union

import torch

from astrai_b200.factory import Registry
from astrai_b200.serialization import load_bin, load_bin_offsets, load_h5

logger = logging.getLogger(__name__)


def detect_format(load_path: str) -> str:
    root = Path(load_path)
    if root.is_file():
        suf = root.suffix.lower()
        if suf in (".h5", ".hdf5"):
            return "h5"
        if suf == ".jsonl":
            return "jsonl"
        raise ValueError(f"Unsupported file format: {suf}")
    if any(root.rglob("*.h5")) or any(root.rglob("*.hdf5")):
        return "h5"
    if any(root.rglob("*.bin")) and any(root.rglob("meta.json")):
        return "bin"
    if any(root.rglob("*.jsonl")):
        return "jsonl"
    raise FileNotFoundError(f"No supported data files found at {load_path}")


class Store:
    """Common bookkeeping: segments per key, cumulative lengths, record offsets."""

    segments_are_records = False

    def __init__(self, window_size: int = 0, stride: Optional[int] = None):
        self._data: Dict[str, list] = {}
        self._cum: Dict[str, List[int]] = {}
        self._offsets: Dict[str, List[int]] = {}
        self._length = 0
        self._num_records = 0
        self._window_size = int(window_size)
        self._stride = int(stride) if stride else int(window_size)

    def load(self, path: str, **kwargs) -> None:  # pragma: no cover - abstract
        raise NotImplementedError

    # ------------------------------------------------------------------ properties
    @property
    def keys(self) -> List[str]:
        return list(self._data.keys())

    @property
    def window_size(self) -> int:
        return self._window_size

    @property
    def stride(self) -> int:
        return self._stride

    @property
    def token_count(self) -> int:
        return self._length

    @property
    def num_records(self) -> int:
        return self._num_records

    @property
    def num_samples(self) -> int:
        if self._window_size > 0 and self._length > 0:
            if self._length <= self._window_size:
                return 0
            return (self._length - 1 - self._window_size) // self._stride + 1
        return self._num_records

    def __len__(self) -> int:
        return self.num_samples

    def __getitem__(self, index: int) -> Dict[str, torch.Tensor]:
        n = self.num_samples
        if index < 0:
            index += n
        if not 0 <= index < n:
            raise IndexError(f"Store index out of range: {index}, num_samples={n}")
        if self._window_size > 0 and self._length > 0:
            b, e = self.sample_window(index)
            return {k: self.fetch(b, e, k) for k in self._stream_keys()}
        return self.fetch_record(index, list(self._data.keys()))

    def sample_window(self, index: int) -> Tuple[int, int]:
        if self._window_size <= 0:
            raise RuntimeError("sample_window() requires window_size > 0 (stream mode)")
        if self._length <= self._window_size:
            raise IndexError(f"Data too short for window: token_count={self._length}, window_size={self._window_size}")
        if not 0 <= index < self.num_samples:
            raise IndexError(f"Sample index out of range: {index}, num_samples={self.num_samples}")
        begin = min(index * self._stride, self._length - 1 - self._window_size)
        return begin, min(begin + self._window_size, self._length - 1)

    def _stream_keys(self) -> List[str]:
        return [k for k, v in self._data.items() if not (v and isinstance(v[0], list))]

    # ------------------------------------------------------------------ normalisation
    def _normalize(self, raw: Dict[str, list], offsets: Optional[Dict[str, List[int]]] = None) -> None:
        lengths = []
        for key, segs in raw.items():
            self._data[key] = segs
            if not segs:
                self._cum[key] = []
                lengths.append(0)
                continue
            if isinstance(segs[0], list):  # nested per-record groups (GRPO)
                self._cum[key] = []
                continue
            cum, tot = [], 0
            for t in segs:
                tot += int(t.shape[0])
                cum.append(tot)
            self._cum[key] = cum
            lengths.append(tot)
        self._length = min(lengths) if lengths else 0
        good: Dict[str, List[int]] = {}
        for key, off in (offsets or {}).items():
            segs = self._data.get(key, [])
            if len(segs) == 1 and len(off) > 1:
                good[key] = off
            elif len(segs) > 1:
                logger.warning("Key '%s' has %d segments with offsets; record mode disabled for it", key, len(segs))
        self._offsets = good
        if good:
            self._num_records = min(len(v) - 1 for v in good.values())
        elif self.segments_are_records:
            counts = [len(v) for v in self._data.values() if not (v and isinstance(v[0], list))]
            self._num_records = min(counts) if counts else 0
        else:
            self._num_records = 0

    # ------------------------------------------------------------------ access
    def fetch(self, begin: int, end: int, keys: Union[str, List[str]]):
        if not self._data:
            raise RuntimeError("Store not loaded")
        if not (0 <= begin < self._length and 0 <= end <= self._length):
            raise ValueError(f"Index out of bounds: begin={begin}, end={end}, length={self._length}")
        if isinstance(keys, str):
            return self._fetch_key(keys, begin, end)
        return {k: self._fetch_key(k, begin, end) for k in keys}

    def _fetch_key(self, key: str, begin: int, end: int) -> torch.Tensor:
        segs, cum = self._data[key], self._cum[key]
        first = bisect.bisect_right(cum, begin)
        last = bisect.bisect_left(cum, end)
        parts = []
        for i in range(first, last + 1):
            prev = cum[i - 1] if i > 0 else 0
            parts.append(segs[i][max(begin - prev, 0):min(end - prev, segs[i].shape[0])])
        return parts[0] if len(parts) == 1 else torch.cat(parts, 0)

    def fetch_record(self, index: int, keys: Union[str, List[str]]):
        if not 0 <= index < self._num_records:
            raise ValueError(f"Record index out of bounds: {index}, num_records={self._num_records}")
        if isinstance(keys, str):
            return self._record_key(keys, index)
        return {k: self._record_key(k, index) for k in keys}

    def _record_key(self, key: str, index: int):
        off = self._offsets.get(key)
        if off:
            end = off[index + 1] if index + 1 < len(off) else self._data[key][0].shape[0]
            return self._data[key][0][off[index]:end]
        return self._data[key][index]


Streamable = Store  # access traits are folded into Store
Recordable = Store


class StoreFactory(Registry["Store"]):
    pass


@StoreFactory.register("h5")
class H5Store(Store):
    segments_are_records = True

    def load(self, path: str, **kwargs) -> None:
        self._normalize(load_h5(path))


@StoreFactory.register("bin")
class MmapStore(Store):
    def __init__(self, window_size: int = 0, stride: Optional[int] = None):
        super().__init__(window_size, stride)
        self._mmap_refs: List[torch.Tensor] = []

    def load(self, path: str, **kwargs) -> None:
        root = Path(path)
        metas = sorted(root.rglob("meta.json")) if root.is_dir() else []
        if not metas:
            raise FileNotFoundError(f"No meta.json found under {path}")
        raw: Dict[str, List[torch.Tensor]] = {}
        offs: Dict[str, List[int]] = {}
        for m in metas:
            for k, ts in load_bin(str(m.parent)).items():
                raw.setdefault(k, []).extend(ts)
            for k, o in load_bin_offsets(str(m.parent)).items():
                offs.setdefault(k, []).extend(o)
        self._normalize(raw, offsets=offs or None)
        self._mmap_refs = [t for ts in self._data.values() for t in ts if isinstance(t, torch.Tensor)]


class JsonlSource:
    """Reads a .jsonl file or every *.jsonl of a directory (bad lines skipped)."""

    def __init__(self, path: str):
        self.path = Path(path)
        self._records: Optional[List[dict]] = None

    def load(self) -> List[dict]:
        if self._records is None:
            files = [self.path] if self.path.is_file() else sorted(self.path.glob("*.jsonl"))
            recs: List[dict] = []
            for f in files:
                with open(f, "r", encoding="utf-8") as fh:
                    for line in fh:
                        line = line.strip()
                        if not line:
                            continue
                        try:
                            recs.append(json.loads(line))
                        except json.JSONDecodeError:
                            logger.warning("Failed to parse JSON line in %s, skipping", f)
            self._records = recs
        return self._records


@StoreFactory.register("jsonl")
class JsonlStore(Store):
    CONFIG_NAME = "dataset_config.json"
    segments_are_records = True
    DEFAULT_MESSAGES_CONFIG = {
        "version": 1,
        "input": {"sections": [{"field": "messages", "action": "$role", "template": True}]},
        "mask": {"system": "mask", "user": "mask", "assistant": "train"},
        "mask_default": "mask",
        "output": {"position_ids_mode": "doc_reset"},
    }

    def __init__(self, window_size: int = 0, stride: Optional[int] = None):
        super().__init__(window_size, stride)
        self._source: Optional[JsonlSource] = None
        self._processor: Optional[Callable[[dict], Dict[str, torch.Tensor]]] = None
        self._keys_cache: Optional[List[str]] = None

    def load(self, path: str, transform=None, processor=None, **kwargs) -> None:
        self._source = JsonlSource(path)
        records = self._source.load()
        if processor is not None:
            self._processor = processor
            self._num_records = len(records)
            return
        if transform is None:
            from astrai_b200.config.preprocess_config import PipelineConfig
            from astrai_b200.preprocessing.pipeline import TokenizeTransform

            root = Path(path)
            cfg = root / self.CONFIG_NAME if root.is_dir() else None
            if cfg is not None and cfg.exists():
                transform = TokenizeTransform.from_config_file(str(cfg))
            else:
                tok = kwargs.get("tokenizer_path")
                if not tok:
                    raise FileNotFoundError(
                        f"JSONL dataset config not found. Expected {self.CONFIG_NAME} alongside *.jsonl files, pass "
                        "an explicit transform, processor= for lazy tokenisation, or tokenizer_path= for the "
                        "built-in messages config.")
                transform = TokenizeTransform(PipelineConfig.from_dict(self.DEFAULT_MESSAGES_CONFIG), tok)
        self._normalize(transform.apply(records))

    @property
    def keys(self) -> List[str]:
        if self._processor is not None:
            if self._keys_cache is None and self._num_records > 0:
                self._keys_cache = list(self._processor(self._source.load()[0]).keys())
            return self._keys_cache or []
        return list(self._data.keys())

    def fetch_record(self, index: int, keys):
        if self._processor is not None:
            if not 0 <= index < self._num_records:
                raise ValueError(f"Record index out of bounds: {index}, num_records={self._num_records}")
            data = self._processor(self._source.load()[index])
            return data[keys] if isinstance(keys, str) else {k: data[k] for k in keys}
        return super().fetch_record(index, keys)

    def fetch(self, begin: int, end: int, keys):
        if self._processor is not None:
            raise RuntimeError("JsonlStore in lazy (processor) mode does not support stream fetch(); "
                               "use fetch_record() instead.")
        return super().fetch(begin, end, keys)

    def __getitem__(self, index: int):
        if self._processor is not None:
            return self.fetch_record(index, self.keys)
        return super().__getitem__(index)
