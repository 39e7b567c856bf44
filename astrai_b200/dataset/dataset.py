"""Training datasets: a :class:`Store` plus the key mapping of one training type.

Public names kept from the reference (astrai/dataset/dataset.py:43-506): ``BaseDataset``,
``DatasetFactory`` (keys ``seq``, ``sft``, ``dpo``, ``grpo``), the four dataset classes,
``dpo_tokenize``, ``dpo_processor``, ``dpo_collate_fn`` and ``grpo_collate_fn``.

Each dataset class is declarative:

* window datasets (``seq``, ``sft``) list ``fields``: output name, store key, target shift
  (0 for inputs, 1 for next-token targets) and dtype. Sample ``i`` takes the store's window
  ``[b, e)`` for shift 0 and ``[b + 1, e + 1)`` for shift 1;
* record datasets (``dpo``, ``grpo``) list ``casts``: store key and dtype of one record's
  tensors (lists of tensors for GRPO's nested keys).

``DatasetFactory.load`` detects the storage format, picks the window (record types always
read whole records), builds a lazy DPO processor for raw JSONL when a tokenizer is given,
loads the store and wraps it.
"""

from __future__ import annotations

from functools import partial
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch
from torch.utils.data import Dataset

from astrai_b200.dataset.storage import Store, StoreFactory, detect_format
from astrai_b200.factory import Registry

# ---------------------------------------------------------------------------------------- DPO records


def _as_turns(prompt) -> List[dict]:
    """A prompt given as a string (one user turn), a message list, or anything else (stringified)."""
    if isinstance(prompt, list):
        return prompt
    return [{"role": "user", "content": prompt if isinstance(prompt, str) else str(prompt)}]


def _response_text(resp) -> Optional[str]:
    """A response given as a string or as a message list (contents joined)."""
    if isinstance(resp, str):
        return resp
    if isinstance(resp, list):
        return "".join(m.get("content", "") for m in resp if isinstance(m, dict))
    return None


def dpo_tokenize(record: dict, tokenizer, max_len: int = 2048) -> Optional[dict]:
    """One preference record -> token ids and response masks, or None if a field is missing.

    Accepted records: ``{"prompt" | "input": str or messages, "chosen": str or messages,
    "rejected": ...}``. The prompt is rendered with the generation prompt; each response is
    appended as one assistant turn. Masks are 1 on response tokens only; every list is cut
    to ``max_len``."""
    prompt = record.get("prompt") or record.get("input")
    answers = [_response_text(record.get("chosen")), _response_text(record.get("rejected"))]
    if prompt is None or None in answers:
        return None
    turns = _as_turns(prompt)
    n_prompt = min(len(tokenizer.apply_chat_template(turns, tokenize=True, add_generation_prompt=True)), max_len)
    out = {}
    for name, text in zip(("chosen", "rejected"), answers):
        ids = tokenizer.apply_chat_template(turns + [{"role": "assistant", "content": text}], tokenize=True,
                                            add_generation_prompt=False)[:max_len]
        out[name] = ids
        out[name + "_mask"] = [int(i >= n_prompt) for i in range(len(ids))]
    return out


def dpo_processor(record: dict, tokenizer, max_len: int = 2048) -> Dict[str, torch.Tensor]:
    """:func:`dpo_tokenize` as tensors (ids int32, masks bool); raises on an unusable record."""
    tok = dpo_tokenize(record, tokenizer, max_len=max_len)
    if tok is None:
        raise ValueError("DPO record needs 'prompt' (or 'input'), 'chosen' and 'rejected'; "
                         f"this one has {sorted(record)}")
    return {k: torch.tensor(v, dtype=torch.bool if k.endswith("_mask") else torch.int32) for k, v in tok.items()}


# ---------------------------------------------------------------------------------------- collate


def _pad_rows(rows: Sequence[torch.Tensor], width: int, dtype, left: bool = False) -> torch.Tensor:
    out = torch.zeros(len(rows), width, dtype=dtype)
    for i, r in enumerate(rows):
        n = r.shape[0]
        if n:
            (out[i, width - n:] if left else out[i, :n]).copy_(r)
    return out


def dpo_collate_fn(batch: List[Dict[str, torch.Tensor]]) -> Dict[str, torch.Tensor]:
    """Right-pad chosen / rejected ids and masks of a batch to one common length [B, S]."""
    width = max(s[k].shape[0] for s in batch for k in ("chosen", "rejected"))
    return {k: _pad_rows([s[k] for s in batch], width, torch.bool if k.endswith("_mask") else torch.long)
            for k in ("chosen", "rejected", "chosen_mask", "rejected_mask")}


def grpo_collate_fn(batch: List[Dict[str, torch.Tensor]]) -> Dict[str, torch.Tensor]:
    """Prompts left-padded to [B, P] (with ``prompt_mask``), the G responses per prompt and
    their masks right-padded to [B, G, R], rewards [B, G] (missing entries stay 0)."""
    G = len(batch[0]["responses"])
    P = max(s["prompts"].shape[0] for s in batch)
    R = max(r.shape[0] for s in batch for r in s["responses"])
    prompts = _pad_rows([s["prompts"] for s in batch], P, torch.long, left=True)
    pmask = _pad_rows([torch.ones(s["prompts"].shape[0], dtype=torch.bool) for s in batch], P, torch.bool,
                      left=True)
    resp = torch.zeros(len(batch), G, R, dtype=torch.long)
    masks = torch.zeros(len(batch), G, R, dtype=torch.bool)
    rewards = torch.zeros(len(batch), G)
    for i, s in enumerate(batch):
        resp[i, :len(s["responses"][:G])] = _pad_rows(s["responses"][:G], R, torch.long)
        masks[i, :len(s["masks"][:G])] = _pad_rows(s["masks"][:G], R, torch.bool)
        r = s["rewards"][:G]
        rewards[i, :r.shape[0]] = r
    return {"prompts": prompts, "prompt_mask": pmask, "responses": resp, "masks": masks, "rewards": rewards}


# ---------------------------------------------------------------------------------------- datasets


def validate_keys(store: Store, required: Sequence[str]) -> None:
    have = set(store.keys)
    missing = [k for k in required if k not in have]
    if missing:
        raise KeyError(f"the store lacks {missing} (it has {sorted(have)})")


class BaseDataset(Dataset):
    """A store checked for the keys this dataset reads."""

    required_keys: List[str] = []

    def __init__(self, store: Store):
        super().__init__()
        validate_keys(store, self.required_keys)
        self.store = store

    def __len__(self) -> int:
        return len(self.store)

    @property
    def keys(self) -> List[str]:
        return self.store.keys

    @property
    def token_count(self) -> int:
        return self.store.token_count

    def __getitem__(self, index: int) -> Dict[str, torch.Tensor]:  # pragma: no cover - per dataset
        raise NotImplementedError(f"{type(self).__name__} does not define samples")


class _WindowDataset(BaseDataset):
    #: (output name, store key, shift, dtype)
    fields: Tuple[Tuple[str, str, int, torch.dtype], ...] = ()

    def __init_subclass__(cls, **kw):
        super().__init_subclass__(**kw)
        cls.required_keys = sorted({key for _, key, _, _ in cls.fields})

    def __getitem__(self, index: int) -> Dict[str, torch.Tensor]:
        b, e = self.store.sample_window(index)
        return {name: self.store.fetch(b + shift, e + shift, key).to(dtype) for name, key, shift, dtype in self.fields}


class _RecordDataset(BaseDataset):
    #: (store key, dtype); nested keys come back as lists of tensors
    casts: Tuple[Tuple[str, torch.dtype], ...] = ()

    def __init_subclass__(cls, **kw):
        super().__init_subclass__(**kw)
        cls.required_keys = [k for k, _ in cls.casts]

    def __getitem__(self, index: int) -> Dict[str, torch.Tensor]:
        rec = self.store.fetch_record(index, self.required_keys)
        out = {}
        for key, dtype in self.casts:
            v = rec[key]
            out[key] = [t.to(dtype) for t in v] if isinstance(v, list) else v.to(dtype)
        return out


class DatasetFactory(Registry["BaseDataset"]):
    #: training types that read whole records, never windows
    RECORD_TYPES = ("dpo", "grpo")

    @classmethod
    def load(cls, train_type: str, load_path: Optional[str] = None, window_size: int = 0, stride: Optional[int] = None,
             storage_type: Optional[str] = None, tokenizer_path: Optional[str] = None, max_len: int = 2048,
             store: Optional[Store] = None, **kwargs) -> BaseDataset:
        """Dataset of ``train_type`` over ``store``, or over a store loaded from ``load_path``."""
        if store is None:
            if load_path is None:
                raise ValueError("DatasetFactory.load needs a load_path to read, or a ready store=")
            store = cls._open_store(train_type, load_path, window_size, stride, storage_type, tokenizer_path,
                                    max_len, kwargs)
        return cls.create(train_type, store=store)

    @classmethod
    def _open_store(cls, train_type, load_path, window_size, stride, storage_type, tokenizer_path, max_len,
                    load_kw) -> Store:
        fmt = storage_type or detect_format(load_path)
        window = 0 if train_type in cls.RECORD_TYPES else window_size
        st = StoreFactory.create(fmt, window_size=window, stride=(stride or window_size) if window else 0)
        kw = dict(load_kw)
        if fmt == "jsonl" and tokenizer_path:
            if train_type == "dpo":
                from astrai_b200.tokenize import AutoTokenizer

                kw["processor"] = partial(dpo_processor, tokenizer=AutoTokenizer.from_pretrained(tokenizer_path),
                                          max_len=max_len)
            elif train_type in ("seq", "sft"):
                kw.setdefault("tokenizer_path", tokenizer_path)
        st.load(load_path, **kw)
        return st


@DatasetFactory.register("seq")
class SEQDataset(_WindowDataset):
    fields = (("input_ids", "sequence", 0, torch.long), ("target_ids", "sequence", 1, torch.long))


@DatasetFactory.register("sft")
class SFTDataset(_WindowDataset):
    fields = (("input_ids", "sequence", 0, torch.long), ("target_ids", "sequence", 1, torch.long),
              ("position_ids", "position_ids", 0, torch.long), ("loss_mask", "loss_mask", 1, torch.bool))


@DatasetFactory.register("dpo")
class DPODataset(_RecordDataset):
    casts = (("chosen", torch.long), ("rejected", torch.long), ("chosen_mask", torch.bool),
             ("rejected_mask", torch.bool))

    def make_processor(self, tokenizer, max_len: int) -> Callable[[dict], Dict[str, torch.Tensor]]:
        return partial(dpo_processor, tokenizer=tokenizer, max_len=max_len)


@DatasetFactory.register("grpo")
class GRPODataset(_RecordDataset):
    casts = (("prompts", torch.long), ("responses", torch.long), ("masks", torch.bool), ("rewards", torch.float32))
