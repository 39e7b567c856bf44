"""Datasets per training type (parity: astrai/dataset/dataset.py:43-506).

* ``seq``  - stream windows; ``input_ids`` and the +1-shifted ``target_ids``;
* ``sft``  - as seq plus ``position_ids`` and the shifted ``loss_mask``;
* ``dpo``  - one preference pair per record (``chosen``, ``rejected`` and
  their masks); raw JSONL is tokenised lazily through the chat template;
* ``grpo`` - one prompt with G responses, masks and rewards per record.

``DatasetFactory.load(train_type, load_path, window_size, stride, ...)``
builds the store (format auto-detected) and the dataset; ``dpo_collate_fn``
right-pads pairs, ``grpo_collate_fn`` left-pads prompts and right-pads
responses.
"""

from __future__ import annotations

from functools import partial
from typing import Callable, Dict, List, Optional

import torch
from torch.utils.data import Dataset

from astrai_b200.dataset.storage import Store, StoreFactory, detect_format
from astrai_b200.factory import Registry


def _to_messages(v) -> list:
    if isinstance(v, str):
        return [{"role": "user", "content": v}]
    if isinstance(v, list):
        return v
    return [{"role": "user", "content": str(v)}]


def _text(v) -> Optional[str]:
    if v is None:
        return None
    if isinstance(v, str):
        return v
    if isinstance(v, list):
        return "".join(m.get("content", "") for m in v if isinstance(m, dict))
    return None


def dpo_tokenize(record: dict, tokenizer, max_len: int = 2048) -> Optional[dict]:
    """Prompt rendered with the generation prompt, chosen / rejected appended as
    one assistant turn; masks cover the response tokens only."""
    prompt = record.get("prompt") or record.get("input")
    ch, rj = _text(record.get("chosen")), _text(record.get("rejected"))
    if prompt is None or ch is None or rj is None:
        return None
    pm = _to_messages(prompt)
    p_ids = tokenizer.apply_chat_template(pm, tokenize=True, add_generation_prompt=True)
    c_ids = tokenizer.apply_chat_template(pm + [{"role": "assistant", "content": ch}], tokenize=True,
                                          add_generation_prompt=False)[:max_len]
    r_ids = tokenizer.apply_chat_template(pm + [{"role": "assistant", "content": rj}], tokenize=True,
                                          add_generation_prompt=False)[:max_len]
    pl = min(len(p_ids), max_len)

    def mask(ids):
        return ([0] * pl + [1] * max(0, len(ids) - pl))[:max_len]

    return {"chosen": c_ids, "rejected": r_ids, "chosen_mask": mask(c_ids), "rejected_mask": mask(r_ids)}


def dpo_processor(record: dict, tokenizer, max_len: int = 2048) -> Dict[str, torch.Tensor]:
    r = dpo_tokenize(record, tokenizer, max_len=max_len)
    if r is None:
        raise ValueError(f"Malformed DPO record: {list(record.keys())}")
    return {"chosen": torch.tensor(r["chosen"], dtype=torch.int32),
            "rejected": torch.tensor(r["rejected"], dtype=torch.int32),
            "chosen_mask": torch.tensor(r["chosen_mask"], dtype=torch.bool),
            "rejected_mask": torch.tensor(r["rejected_mask"], dtype=torch.bool)}


def dpo_collate_fn(batch: List[Dict[str, torch.Tensor]]) -> Dict[str, torch.Tensor]:
    B = len(batch)
    S = max(max(b["chosen"].size(0), b["rejected"].size(0)) for b in batch)
    out = {"chosen": torch.zeros(B, S, dtype=torch.long), "rejected": torch.zeros(B, S, dtype=torch.long),
           "chosen_mask": torch.zeros(B, S, dtype=torch.bool), "rejected_mask": torch.zeros(B, S, dtype=torch.bool)}
    for i, b in enumerate(batch):
        for k in ("chosen", "rejected"):
            n = b[k].size(0)
            out[k][i, :n] = b[k]
            out[k + "_mask"][i, :n] = b[k + "_mask"]
    return out


def grpo_collate_fn(batch: List[Dict[str, torch.Tensor]]) -> Dict[str, torch.Tensor]:
    B, G = len(batch), len(batch[0]["responses"])
    P = max(b["prompts"].size(0) for b in batch)
    R = max(r.size(0) for b in batch for r in b["responses"])
    prompts = torch.zeros(B, P, dtype=torch.long)
    pmask = torch.zeros(B, P, dtype=torch.bool)
    resp = torch.zeros(B, G, R, dtype=torch.long)
    masks = torch.zeros(B, G, R, dtype=torch.bool)
    rewards = torch.zeros(B, G, dtype=torch.float32)
    for i, b in enumerate(batch):
        n = b["prompts"].size(0)
        prompts[i, P - n:] = b["prompts"]
        pmask[i, P - n:] = True
        rewards[i, : b["rewards"].size(0)] = b["rewards"]
        for g in range(min(G, len(b["responses"]))):
            m = b["responses"][g].size(0)
            resp[i, g, :m] = b["responses"][g]
            if g < len(b["masks"]):
                masks[i, g, :m] = b["masks"][g]
    return {"prompts": prompts, "prompt_mask": pmask, "responses": resp, "masks": masks, "rewards": rewards}


def validate_keys(store: Store, required: List[str]) -> None:
    missing = [k for k in required if k not in set(store.keys)]
    if missing:
        raise KeyError(f"Store is missing required keys {missing}; available keys are {sorted(store.keys)}.")


class BaseDataset(Dataset):
    required_keys: List[str] = []

    def __init__(self, store: Store):
        super().__init__()
        self.store = store
        validate_keys(store, self.required_keys)

    def __len__(self) -> int:
        return len(self.store)

    @property
    def keys(self) -> List[str]:
        return self.store.keys

    @property
    def token_count(self) -> int:
        return self.store.token_count

    def __getitem__(self, index: int) -> Dict[str, torch.Tensor]:  # pragma: no cover - abstract
        raise NotImplementedError


class DatasetFactory(Registry["BaseDataset"]):
    @classmethod
    def load(cls, train_type: str, load_path: Optional[str] = None, window_size: int = 0, stride: Optional[int] = None,
             storage_type: Optional[str] = None, tokenizer_path: Optional[str] = None, max_len: int = 2048,
             store: Optional[Store] = None, **kwargs) -> BaseDataset:
        if store is not None:
            return cls.create(train_type, store=store)
        if load_path is None:
            raise ValueError("Either load_path or store must be provided")
        storage_type = storage_type or detect_format(load_path)
        stride = stride or window_size
        processor = cls._maybe_build_processor(train_type, storage_type, tokenizer_path, max_len)
        win = window_size if train_type in ("seq", "sft") else 0
        st = StoreFactory.create(storage_type, window_size=win, stride=stride if stride else win)
        if processor is not None:
            st.load(load_path, processor=processor, **kwargs)
        else:
            kw = dict(kwargs)
            if tokenizer_path and storage_type == "jsonl" and train_type in ("seq", "sft"):
                kw.setdefault("tokenizer_path", tokenizer_path)
            st.load(load_path, **kw)
        return cls.create(train_type, store=st)

    @staticmethod
    def _maybe_build_processor(train_type, storage_type, tokenizer_path, max_len) -> Optional[Callable]:
        if tokenizer_path is None or storage_type != "jsonl" or train_type != "dpo":
            return None
        from astrai_b200.tokenize import AutoTokenizer

        return partial(dpo_processor, tokenizer=AutoTokenizer.from_pretrained(tokenizer_path), max_len=max_len)


@DatasetFactory.register("seq")
class SEQDataset(BaseDataset):
    required_keys = ["sequence"]

    def __getitem__(self, index: int):
        b, e = self.store.sample_window(index)
        return {"input_ids": self.store.fetch(b, e, "sequence").to(torch.long),
                "target_ids": self.store.fetch(b + 1, e + 1, "sequence").to(torch.long)}


@DatasetFactory.register("sft")
class SFTDataset(BaseDataset):
    required_keys = ["sequence", "loss_mask", "position_ids"]

    def __getitem__(self, index: int):
        b, e = self.store.sample_window(index)
        return {"input_ids": self.store.fetch(b, e, "sequence").to(torch.long),
                "target_ids": self.store.fetch(b + 1, e + 1, "sequence").to(torch.long),
                "position_ids": self.store.fetch(b, e, "position_ids").to(torch.long),
                "loss_mask": self.store.fetch(b + 1, e + 1, "loss_mask").to(torch.bool)}


@DatasetFactory.register("dpo")
class DPODataset(BaseDataset):
    required_keys = ["chosen", "rejected", "chosen_mask", "rejected_mask"]

    def make_processor(self, tokenizer, max_len: int):
        return partial(dpo_processor, tokenizer=tokenizer, max_len=max_len)

    def __getitem__(self, index: int):
        r = self.store.fetch_record(index, self.required_keys)
        return {"chosen": r["chosen"].to(torch.long), "rejected": r["rejected"].to(torch.long),
                "chosen_mask": r["chosen_mask"].to(torch.bool), "rejected_mask": r["rejected_mask"].to(torch.bool)}


@DatasetFactory.register("grpo")
class GRPODataset(BaseDataset):
    required_keys = ["prompts", "responses", "masks", "rewards"]

    def __getitem__(self, index: int):
        r = self.store.fetch_record(index, self.required_keys)
        return {"prompts": r["prompts"].to(torch.long),
                "responses": [x.to(torch.long) for x in r["responses"]],
                "masks": [x.to(torch.bool) for x in r["masks"]],
                "rewards": r["rewards"].to(torch.float32)}
