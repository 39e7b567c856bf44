"""Offline JSONL -> token-shard pipeline, packing, position ids and writers.

Parity: astrai/preprocessing/{packing,position_id,writer,core,transform,pipeline}.py.

* packing (per shard, applied in lockstep to every per-token key):
  ``simple`` truncates; ``bfd`` best-fit-decreasing bins of at most
  ``max_packed_len`` tokens (sequences placed longest first into the bin with
  the least room that still fits); ``bfd_split`` first cuts over-long
  sequences into ``max_packed_len`` chunks;
* position ids: ``none``, ``doc_reset`` (restart at 0 per document - attached
  before packing so bins concatenate per-document ranges), ``continuous``
  (0..n over the packed shard);
* writers: ``bin`` -> ``out/<domain>/shard_XXXX/{key}.bin + meta.json``,
  ``h5`` -> ``out/<domain>/data_XXXX.h5``; a failed write removes the partial
  shard;
* :class:`Pipeline` streams records in batches (a batch that fails is retried
  record by record), buckets them by domain and flushes a shard every
  ``max_tokens_per_shard`` tokens;
* :class:`TokenizeTransform` applies the same record processing eagerly in
  memory for ``JsonlStore``.
"""

from __future__ import annotations

import json
import logging
import os
import shutil
from collections import defaultdict
from itertools import chain
from pathlib import Path
from typing import Dict, Iterator, List, Optional

import torch

from astrai_b200.config.preprocess_config import PipelineConfig
from astrai_b200.factory import Registry
from astrai_b200.preprocessing.builder import MaskBuilderFactory
from astrai_b200.serialization import save_bin, save_h5

logger = logging.getLogger(__name__)

_DTYPES = {"int32": torch.int32, "int64": torch.int64, "int16": torch.int16, "uint8": torch.uint8,
           "float32": torch.float32, "bool": torch.bool}


def filter_by_length(text: str, min_len: int = 50, max_len: int = 2_000_000) -> bool:
    return min_len <= len(text) <= max_len


# ----------------------------------------------------------------------------- packing
def _truncate(seq: List[int], max_len: int, mode: str) -> List[int]:
    if len(seq) <= max_len:
        return seq
    return seq[-max_len:] if mode == "keep_end" else seq[:max_len]


def plan_bfd(sequences: List[List[int]], max_packed_len: int, truncation_mode: str = "keep_start") -> List[List[int]]:
    """Best-fit decreasing: bins of original indices; capacity on truncated lengths."""
    order = sorted(range(len(sequences)), key=lambda i: len(sequences[i]), reverse=True)
    bins: List[List[int]] = []
    fill: List[int] = []
    for i in order:
        n = len(_truncate(sequences[i], max_packed_len, truncation_mode))
        best, best_room = None, max_packed_len + 1
        for b, f in enumerate(fill):
            room = max_packed_len - f
            if n <= room < best_room:
                best, best_room = b, room
        if best is None:
            bins.append([i])
            fill.append(n)
        else:
            bins[best].append(i)
            fill[best] += n
    return bins


class PackingStrategy:
    def apply(self, keys: Dict[str, list], max_packed_len: int, truncation_mode: str) -> Dict[str, list]:
        raise NotImplementedError


class PackingStrategyFactory(Registry["PackingStrategy"]):
    pass


@PackingStrategyFactory.register("simple")
class SimplePacking(PackingStrategy):
    def apply(self, keys, max_packed_len, truncation_mode):
        return {k: [_truncate(v, max_packed_len, truncation_mode) for v in vs] for k, vs in keys.items()}


@PackingStrategyFactory.register("bfd")
class BFDPacking(PackingStrategy):
    def apply(self, keys, max_packed_len, truncation_mode):
        seqs = keys.get("sequence", [])
        if not seqs:
            return keys
        bins = plan_bfd(seqs, max_packed_len, truncation_mode)
        return {k: [_truncate(list(chain.from_iterable(vs[i] for i in b)), max_packed_len, truncation_mode)
                    for b in bins] for k, vs in keys.items()}


@PackingStrategyFactory.register("bfd_split")
class BFDSplitPacking(BFDPacking):
    def apply(self, keys, max_packed_len, truncation_mode):
        seqs = keys.get("sequence", [])
        if not seqs or max_packed_len <= 0:
            return super().apply(keys, max_packed_len, truncation_mode)
        starts = [list(range(0, len(s), max_packed_len)) for s in seqs]
        split = {k: [v[s:s + max_packed_len] for v, st in zip(vs, starts) for s in st] for k, vs in keys.items()}
        return super().apply(split, max_packed_len, truncation_mode)


# ----------------------------------------------------------------------------- position ids
class PositionIdStrategy:
    def generate(self, sequences: List[List[int]]) -> List[int]:
        raise NotImplementedError


class PositionIdStrategyFactory(Registry["PositionIdStrategy"]):
    pass


@PositionIdStrategyFactory.register("none")
class NoPositionId(PositionIdStrategy):
    def generate(self, sequences):
        return []


@PositionIdStrategyFactory.register("doc_reset")
class DocResetPositionId(PositionIdStrategy):
    def generate(self, sequences):
        return [i for s in sequences for i in range(len(s))]


@PositionIdStrategyFactory.register("continuous")
class ContinuousPositionId(PositionIdStrategy):
    def generate(self, sequences):
        return list(range(sum(len(s) for s in sequences)))


# ----------------------------------------------------------------------------- writers
class StoreWriter:
    def save(self, output_dir: str, domain: str, shard_idx: int, tensors: Dict[str, List[torch.Tensor]]) -> None:
        raise NotImplementedError


class StoreWriterFactory(Registry["StoreWriter"]):
    pass


@StoreWriterFactory.register("bin")
class BinWriter(StoreWriter):
    def save(self, output_dir, domain, shard_idx, tensors):
        path = os.path.join(output_dir, domain, f"shard_{shard_idx:04d}")
        try:
            save_bin(path, tensors)
        except Exception:
            shutil.rmtree(path, ignore_errors=True)
            logger.error("Failed to write shard %s/shard_%04d, removed partial output", domain, shard_idx)
            raise


@StoreWriterFactory.register("h5")
class H5Writer(StoreWriter):
    def save(self, output_dir, domain, shard_idx, tensors):
        d = os.path.join(output_dir, domain)
        f = os.path.join(d, f"data_{shard_idx:04d}.h5")
        try:
            save_h5(d, f"data_{shard_idx:04d}", tensors)
        except Exception:
            if os.path.exists(f):
                os.remove(f)
            logger.error("Failed to write shard %s/data_%04d.h5, removed partial output", domain, shard_idx)
            raise


# ----------------------------------------------------------------------------- shared core
def build_preprocessing_components(config: PipelineConfig, tokenizer_path: str):
    from astrai_b200.tokenize import AutoTokenizer

    return (AutoTokenizer.from_pretrained(tokenizer_path), MaskBuilderFactory.create("sectioned"),
            PositionIdStrategyFactory.create(config.output.position_ids_mode))


def primary_ids(result: dict) -> List[int]:
    for v in result.values():
        if isinstance(v, list) and v and isinstance(v[0], int):
            return v
    return []


def infer_dtype(ids: list) -> torch.dtype:
    return torch.float32 if ids and isinstance(ids[0], float) else torch.int32


def iter_raw_records(records: List[dict], mask_builder, config, tokenizer) -> Iterator[dict]:
    for item in records:
        r = mask_builder.build(item, config, tokenizer)
        if r is None:
            continue
        r.pop("domain", None)
        if primary_ids(r):
            yield r


def to_per_record_tensors(raw: Dict[str, list]) -> Dict[str, list]:
    out: Dict[str, list] = {}
    for k, lst in raw.items():
        if lst and isinstance(lst[0], list):
            out[k] = [[torch.tensor(s, dtype=infer_dtype(s)) for s in ids] if ids and isinstance(ids[0], list)
                      else torch.tensor(ids, dtype=infer_dtype(ids)) for ids in lst]
        else:
            out[k] = [torch.tensor(list(chain.from_iterable(lst)), dtype=torch.int32)]
    return out


def build_position_ids(sequences: List[List[int]], strategy) -> Optional[List[int]]:
    return strategy.generate(sequences) or None


class TokenizeTransform:
    """In-memory record tokenisation for JsonlStore (same core as Pipeline)."""

    def __init__(self, config: PipelineConfig, tokenizer_path: str):
        self.config = config
        self.tokenizer, self.mask_builder, self.position_strategy = build_preprocessing_components(config,
                                                                                                  tokenizer_path)

    @classmethod
    def from_config_file(cls, config_path: str) -> "TokenizeTransform":
        raw = json.loads(Path(config_path).read_text(encoding="utf-8"))
        tok = raw.pop("tokenizer_path", None) or str(Path(config_path).parent)
        return cls(PipelineConfig.from_dict(raw), tok)

    def apply(self, records: List[dict]) -> Dict[str, list]:
        raw: Dict[str, list] = {}
        for r in iter_raw_records(records, self.mask_builder, self.config, self.tokenizer):
            ids = primary_ids(r)
            if self.config.output.position_ids_mode != "none" and "position_ids" not in r:
                pos = build_position_ids([ids], self.position_strategy)
                if pos:
                    r["position_ids"] = pos
            for k, v in r.items():
                raw.setdefault(k, []).append(v)
        t = to_per_record_tensors(raw)
        for k, vs in t.items():  # per-record lists keep one tensor per record
            if vs and not isinstance(vs[0], list) and len(raw[k]) > 1 and len(vs) == 1:
                t[k] = [torch.tensor(x, dtype=infer_dtype(x)) for x in raw[k]]
        return t


# ----------------------------------------------------------------------------- pipeline
class Pipeline:
    def __init__(self, config: PipelineConfig, input_paths: List[str], output_dir: str, tokenizer_path: str):
        os.makedirs(output_dir, exist_ok=True)
        self.config = config
        self.paths = list(input_paths)
        self.output_dir = output_dir
        self.tokenizer_path = tokenizer_path
        self.tokenizer, self.mask_builder, self._position_id = build_preprocessing_components(config, tokenizer_path)
        self._packer = PackingStrategyFactory.create(config.preprocessing.packing_strategy)
        self._writer = StoreWriterFactory.create(config.output.storage_format)

    def transform(self, item: dict) -> Optional[dict]:
        return self.mask_builder.build(item, self.config, self.tokenizer)

    def transform_batch(self, items: List[dict]) -> List[Optional[dict]]:
        return self.mask_builder.build_batch(items, self.config, self.tokenizer)

    def _items(self) -> Iterator[dict]:
        for path in self.paths:
            with open(path, "r", encoding="utf-8") as fh:
                if path.endswith(".json"):
                    data = json.load(fh)
                    yield from (data if isinstance(data, list) else [data])
                else:
                    for line in fh:
                        line = line.strip()
                        if line:
                            yield json.loads(line)

    def _batches(self, n: int):
        batch: List[dict] = []
        for it in self._items():
            batch.append(it)
            if len(batch) >= max(1, n):
                yield batch
                batch = []
        if batch:
            yield batch

    def run(self) -> Dict[str, int]:
        pp = self.config.preprocessing
        domains: Dict[str, Dict[str, list]] = defaultdict(lambda: defaultdict(list))
        shard_idx: Dict[str, int] = defaultdict(int)
        total = count = 0
        stop = False
        for items in self._batches(pp.batch_size):
            try:
                results = self.transform_batch(items)
            except Exception:
                logger.warning("Batch failed; retrying records individually", exc_info=True)
                results = []
                for it in items:
                    try:
                        results.append(self.transform(it))
                    except Exception:
                        logger.warning("Record failed, skipping", exc_info=True)
                        results.append(None)
            for r in results:
                if pp.max_items and count >= pp.max_items:
                    stop = True
                    break
                if r is None:
                    continue
                dom = r.pop("domain", "__default__")
                ids = primary_ids(r)
                if not ids:
                    continue
                bucket = domains[dom]
                for k in list(bucket.keys()):  # keep keys aligned across records
                    if k not in r:
                        bucket[k].append([0] * len(ids))
                for k, v in r.items():
                    bucket[k].append(v)
                count += 1
                total += len(ids)
                if total >= self.config.output.max_tokens_per_shard:
                    self._flush(domains, shard_idx)
                    domains.clear()
                    total = 0
            if stop:
                break
        if total > 0:
            self._flush(domains, shard_idx)
        return {"records": count, "shards": sum(shard_idx.values())}

    def _flush(self, domains, shard_idx) -> None:
        pp, mode = self.config.preprocessing, self.config.output.position_ids_mode
        for dom, keys in domains.items():
            keys = dict(keys)
            seqs = keys.get("sequence", [])
            if mode == "doc_reset" and seqs:
                keys["position_ids"] = [list(range(len(s))) for s in seqs]
            keys = self._packer.apply(keys, pp.max_packed_len, pp.truncation_mode)
            tensors: Dict[str, List[torch.Tensor]] = {}
            for k, lst in keys.items():
                dt = _DTYPES.get(self.config.output.dtype.get(k, "int32"), torch.int32)
                if lst and isinstance(lst[0], list):
                    tensors[k] = [torch.tensor(list(chain.from_iterable(x)) if x and isinstance(x[0], list) else x,
                                               dtype=dt) for x in lst]
                else:
                    tensors[k] = [torch.tensor(list(chain.from_iterable(lst)), dtype=dt)]
            if mode == "continuous" and keys.get("sequence"):
                pos = self._position_id.generate(keys["sequence"])
                if pos:
                    tensors["position_ids"] = [torch.tensor(pos, dtype=torch.int32)]
            self._writer.save(self.output_dir, dom, shard_idx[dom], tensors)
            shard_idx[dom] += 1
