"""Token stores: where a dataset's tokens live and how sample indices map onto them.

Public names kept from the reference (astrai/dataset/storage.py:71-664): ``Store``,
``StoreFactory`` (keys ``bin`` / ``h5`` / ``jsonl``), ``MmapStore``, ``H5Store``,
``JsonlStore``, ``JsonlSource``, ``detect_format``, and the store methods the datasets call
(``sample_window``, ``fetch``, ``fetch_record``, ``keys``, ``token_count``, ``num_records``,
``num_samples``).

Design. A store is a dict of *columns*, one per key:

* :class:`_StreamColumn` - the key's shards viewed as one token stream. Shard ends are kept
  as a prefix-sum array; a slice that spans shards is found with ``np.searchsorted`` and
  stitched from views, so shards are never concatenated in memory (``bin`` shards stay
  memory-mapped and shared by DataLoader workers through the page cache);
* :class:`_RecordColumn` - per-record access, either one tensor per record or one flat tensor
  cut at recorded offsets (``bin`` shards written with ``record_keys``);
* :class:`_NestedColumn` - a list of tensor lists per record (GRPO responses).

Stream mode (``window_size > 0``) is a contract shared with checkpoints (resuming at a sample
index must see the same tokens): with ``T`` stream tokens, ``w`` the window and ``s`` the
stride, there are ``(T - 1 - w) // s + 1`` samples, and sample ``i`` covers
``[b, b + w)`` with ``b = min(i * s, T - 1 - w)``; the spare token is the last target.
Record mode (``window_size == 0``): one sample per record.
"""

from __future__ import annotations

import json
import logging
from pathlib import Path
from typing import Callable, Dict, Iterable, List, Optional, Sequence, Tuple, Union

import numpy as np
import torch

from astrai_b200.factory import Registry
from astrai_b200.serialization import load_bin, load_bin_offsets, load_h5

logger = logging.getLogger(__name__)

Keys = Union[str, Sequence[str]]

_SUFFIX_FORMAT = {".h5": "h5", ".hdf5": "h5", ".jsonl": "jsonl"}


def detect_format(load_path: str) -> str:
    """``bin`` / ``h5`` / ``jsonl`` from a file's suffix or a directory's contents
    (h5 files win over bin shards, which win over jsonl files)."""
    root = Path(load_path)
    if root.is_file():
        fmt = _SUFFIX_FORMAT.get(root.suffix.lower())
        if fmt is None:
            raise ValueError(f"cannot tell the storage format of {root.name}: expected .h5, .hdf5 or .jsonl")
        return fmt
    found = {p.suffix.lower() for p in root.rglob("*") if p.is_file()}
    if ".h5" in found or ".hdf5" in found:
        return "h5"
    if ".bin" in found and any(root.rglob("meta.json")):
        return "bin"
    if ".jsonl" in found:
        return "jsonl"
    raise FileNotFoundError(f"{load_path}: no .h5/.hdf5 files, no .bin shards with meta.json and no .jsonl files")


# ---------------------------------------------------------------------------------------- columns
class _StreamColumn:
    """Shards of one key read as one stream of tokens."""

    def __init__(self, shards: Sequence[torch.Tensor]):
        self.shards = list(shards)
        self.ends = np.cumsum([int(t.shape[0]) for t in self.shards], dtype=np.int64)

    @property
    def total(self) -> int:
        return int(self.ends[-1]) if len(self.ends) else 0

    def span(self, begin: int, end: int) -> torch.Tensor:
        if end <= begin:
            return self.shards[0][:0]
        first = int(np.searchsorted(self.ends, begin, side="right"))
        last = int(np.searchsorted(self.ends, end, side="left"))
        pieces = []
        for s in range(first, min(last, len(self.shards) - 1) + 1):
            start = int(self.ends[s - 1]) if s else 0
            pieces.append(self.shards[s][max(begin - start, 0):end - start])
        return pieces[0] if len(pieces) == 1 else torch.cat(pieces)


class _RecordColumn:
    """Per-record tensors: a list of records, or one flat tensor cut at ``cuts`` (n + 1 offsets)."""

    def __init__(self, records: Sequence[torch.Tensor], cuts: Optional[Sequence[int]] = None):
        self.records = list(records)
        self.cuts = None if cuts is None else np.asarray(cuts, dtype=np.int64)

    def __len__(self) -> int:
        return len(self.cuts) - 1 if self.cuts is not None else len(self.records)

    def record(self, i: int) -> torch.Tensor:
        if self.cuts is None:
            return self.records[i]
        return self.records[0][int(self.cuts[i]):int(self.cuts[i + 1])]


class _NestedColumn(_RecordColumn):
    """Records that are lists of tensors (e.g. GRPO responses / masks per prompt)."""


# ---------------------------------------------------------------------------------------- store
class Store:
    """Columns of tokens plus the sample arithmetic of stream and record mode."""

    #: True where each loaded segment is one record (h5 groups, jsonl lines); bin shards are
    #: streams unless their meta.json carries record offsets
    segments_are_records = False

    def __init__(self, window_size: int = 0, stride: Optional[int] = None):
        self.window = max(int(window_size), 0)
        self.step = int(stride) if stride else self.window
        self.streams: Dict[str, _StreamColumn] = {}
        self.records: Dict[str, _RecordColumn] = {}
        self._order: List[str] = []

    def load(self, path: str, **kwargs) -> None:  # pragma: no cover - overridden by every backend
        raise NotImplementedError(f"{type(self).__name__} does not implement load()")

    # ------------------------------------------------------------------ building
    def _install(self, raw: Dict[str, list], cuts: Optional[Dict[str, Sequence[int]]] = None) -> None:
        """Turn ``{key: [segments]}`` (and optional per-key record offsets) into columns."""
        cuts = dict(cuts or {})
        self.streams, self.records, self._order = {}, {}, list(raw)
        for key, segs in raw.items():
            if segs and isinstance(segs[0], list):
                self.records[key] = _NestedColumn(segs)
                continue
            self.streams[key] = _StreamColumn(segs)
            if key in cuts:
                if len(segs) == 1 and len(cuts[key]) > 1:
                    self.records[key] = _RecordColumn(segs, cuts[key])
                else:
                    logger.warning("record offsets of %r ignored: they need exactly one shard, found %d",
                                   key, len(segs))
            elif self.segments_are_records:
                self.records[key] = _RecordColumn(segs)

    # ------------------------------------------------------------------ sizes
    @property
    def keys(self) -> List[str]:
        return list(self._order)

    @property
    def window_size(self) -> int:
        return self.window

    @property
    def stride(self) -> int:
        return self.step

    @property
    def token_count(self) -> int:
        """Tokens of the shortest stream key (0 when there is none)."""
        return min((c.total for c in self.streams.values()), default=0)

    @property
    def num_records(self) -> int:
        return min((len(c) for c in self.records.values()), default=0)

    @property
    def stream_mode(self) -> bool:
        return self.window > 0 and self.token_count > 0

    @property
    def num_samples(self) -> int:
        if not self.stream_mode:
            return self.num_records
        spare = self.token_count - 1 - self.window
        return spare // self.step + 1 if spare >= 0 else 0

    def __len__(self) -> int:
        return self.num_samples

    # ------------------------------------------------------------------ samples
    def sample_window(self, index: int) -> Tuple[int, int]:
        """Token range ``[begin, end)`` of stream sample ``index`` (the contract formula)."""
        if self.window <= 0:
            raise RuntimeError(f"{type(self).__name__} was built with window_size=0 (record mode): no windows")
        T, n = self.token_count, self.num_samples
        if n == 0:
            raise IndexError(f"{T} tokens cannot hold one window of {self.window} plus its target token")
        if not 0 <= index < n:
            raise IndexError(f"sample {index} requested from a store of {n} samples")
        begin = min(index * self.step, T - 1 - self.window)
        return begin, begin + self.window

    def __getitem__(self, index: int) -> Dict[str, torch.Tensor]:
        n = self.num_samples
        i = index + n if index < 0 else index
        if not 0 <= i < n:
            raise IndexError(f"sample {index} requested from a store of {n} samples")
        if self.stream_mode:
            begin, end = self.sample_window(i)
            return self.fetch(begin, end, list(self.streams))
        return self.fetch_record(i, self.keys)

    def fetch(self, begin: int, end: int, keys: Keys):
        """Stream tokens ``[begin, end)`` of one key (a tensor) or several (a dict)."""
        if not self.streams:
            raise RuntimeError(f"{type(self).__name__}: nothing loaded (call load() first)")
        T = self.token_count
        if not (0 <= begin < T and begin <= end <= T):
            raise ValueError(f"token range [{begin}, {end}) is outside the stream of {T} tokens")
        return self._pick(keys, lambda k: self._stream(k).span(begin, end))

    def fetch_record(self, index: int, keys: Keys):
        """Record ``index`` of one key (a tensor, or a list for nested keys) or several (a dict)."""
        n = self.num_records
        if not 0 <= index < n:
            raise ValueError(f"record {index} requested from a store of {n} records")
        return self._pick(keys, lambda k: self._record(k).record(index))

    # ------------------------------------------------------------------ helpers
    @staticmethod
    def _pick(keys: Keys, get: Callable[[str], object]):
        return get(keys) if isinstance(keys, str) else {k: get(k) for k in keys}

    def _stream(self, key: str) -> _StreamColumn:
        col = self.streams.get(key)
        if col is None:
            raise KeyError(f"{key!r} is not a stream key of this store (stream keys: {sorted(self.streams)})")
        return col

    def _record(self, key: str) -> _RecordColumn:
        col = self.records.get(key)
        if col is None:
            raise KeyError(f"{key!r} has no per-record layout in this store (record keys: {sorted(self.records)})")
        return col


# the reference splits access into mixins; here both are part of Store
Streamable = Store
Recordable = Store


class StoreFactory(Registry["Store"]):
    pass


@StoreFactory.register("h5")
class H5Store(Store):
    """``*.h5`` files (needs h5py): one group per key, one dataset per record."""

    segments_are_records = True

    def load(self, path: str, **kwargs) -> None:
        self._install(load_h5(path))


@StoreFactory.register("bin")
class MmapStore(Store):
    """Directories of ``meta.json`` + ``<key>.bin`` shards, memory-mapped copy-on-write."""

    def load(self, path: str, **kwargs) -> None:
        shard_dirs = sorted({m.parent for m in Path(path).rglob("meta.json")}) if Path(path).is_dir() else []
        if not shard_dirs:
            raise FileNotFoundError(f"{path}: no shard directory with a meta.json below it")
        raw: Dict[str, List[torch.Tensor]] = {}
        cuts: Dict[str, List[int]] = {}
        for d in shard_dirs:
            for key, tensors in load_bin(str(d)).items():
                raw.setdefault(key, []).extend(tensors)
            for key, offs in load_bin_offsets(str(d)).items():
                cuts.setdefault(key, []).extend(offs)
        self._install(raw, cuts)


class JsonlSource:
    """The records of one ``.jsonl`` file, or of every ``*.jsonl`` in a directory (sorted by name),
    read once and cached. Lines that are not valid JSON are skipped with a warning."""

    def __init__(self, path: str):
        self.path = Path(path)
        self._cache: Optional[List[dict]] = None

    def files(self) -> List[Path]:
        return [self.path] if self.path.is_file() else sorted(self.path.glob("*.jsonl"))

    def load(self) -> List[dict]:
        if self._cache is None:
            self._cache = [rec for f in self.files() for rec in self._parse(f)]
        return self._cache

    @staticmethod
    def _parse(file: Path) -> Iterable[dict]:
        with open(file, encoding="utf-8") as fh:
            for lineno, line in enumerate(fh, 1):
                if not line.strip():
                    continue
                try:
                    yield json.loads(line)
                except json.JSONDecodeError as err:
                    logger.warning("%s:%d skipped (%s)", file, lineno, err.msg)


@StoreFactory.register("jsonl")
class JsonlStore(Store):
    """Raw JSONL records, tokenised either eagerly at load time (a transform built from
    ``dataset_config.json`` next to the files, an explicit ``transform``, or the built-in chat
    ``messages`` config with ``tokenizer_path``), or lazily per record (``processor``)."""

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
        self.source: Optional[JsonlSource] = None
        self.processor: Optional[Callable[[dict], Dict[str, torch.Tensor]]] = None
        self._lazy_keys: Optional[List[str]] = None

    def load(self, path: str, transform=None, processor=None, **kwargs) -> None:
        self.source = JsonlSource(path)
        recs = self.source.load()
        if processor is not None:
            self.processor = processor
            return
        self._install((transform or self._find_transform(path, kwargs.get("tokenizer_path"))).apply(recs))

    def _find_transform(self, path: str, tokenizer_path: Optional[str]):
        from astrai_b200.config.preprocess_config import PipelineConfig
        from astrai_b200.preprocessing.pipeline import TokenizeTransform

        cfg = Path(path) / self.CONFIG_NAME
        if Path(path).is_dir() and cfg.exists():
            return TokenizeTransform.from_config_file(str(cfg))
        if tokenizer_path:
            return TokenizeTransform(PipelineConfig.from_dict(self.DEFAULT_MESSAGES_CONFIG), tokenizer_path)
        raise FileNotFoundError(f"{path}: don't know how to tokenise these records. Put a {self.CONFIG_NAME} next "
                                "to the .jsonl files, or pass transform=, processor= (lazy, per record) or "
                                "tokenizer_path= (chat 'messages' records)")

    # ------------------------------------------------------------------ lazy (processor) mode
    @property
    def lazy(self) -> bool:
        return self.processor is not None

    @property
    def keys(self) -> List[str]:
        if not self.lazy:
            return super().keys
        if self._lazy_keys is None:
            recs = self.source.load()
            self._lazy_keys = list(self.processor(recs[0])) if recs else []
        return list(self._lazy_keys)

    @property
    def num_records(self) -> int:
        return len(self.source.load()) if self.lazy else super().num_records

    def fetch_record(self, index: int, keys: Keys):
        if not self.lazy:
            return super().fetch_record(index, keys)
        n = self.num_records
        if not 0 <= index < n:
            raise ValueError(f"record {index} requested from a store of {n} records")
        out = self.processor(self.source.load()[index])
        return self._pick(keys, out.__getitem__)

    def fetch(self, begin: int, end: int, keys: Keys):
        if self.lazy:
            raise RuntimeError("a JsonlStore loaded with processor= tokenises one record at a time and has no "
                               "token stream; use fetch_record()")
        return super().fetch(begin, end, keys)
