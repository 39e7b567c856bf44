"""Online rollout for RL training (parity: astrai/trainer/rollout.py:26-421).

* ``RawRollout`` / ``RolloutResult`` - prompts ``[B, P]`` (left-padded) with
  mask, responses / response mask / behaviour log-probs ``[B, G, R]``, decoded
  texts, and (result) rewards ``[B, G]``.
* ``BaseRewardModel.score(prompts, responses) -> [B, G]``.
* ``RolloutGenerator`` renders chat prompts (``messages`` or
  ``instruction``/``input``/``output`` batches), expands each prompt G times
  and generates through ``InferenceScheduler.run_batch(return_logprobs=True)``
  - the same paged-KV continuous-batching path the server uses.
* ``RolloutRunner`` caches a scored rollout per prompt batch and refreshes it
  every ``rollout_interval`` optimizer steps; ``__call__`` returns
  ``(result, is_fresh)``; rewards are validated (shape, finite).
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch

_PAD = 0


@dataclass(kw_only=True)
class RawRollout:
    prompts: torch.Tensor
    prompt_mask: torch.Tensor
    responses: torch.Tensor
    response_mask: torch.Tensor
    logprobs_old: torch.Tensor
    prompt_texts: List[str] = field(default_factory=list)
    response_texts: List[List[str]] = field(default_factory=list)


@dataclass(kw_only=True)
class RolloutResult(RawRollout):
    rewards: torch.Tensor


class BaseRewardModel(ABC):
    @abstractmethod
    def score(self, prompts: List[str], responses: List[List[str]]) -> torch.Tensor: ...


class RolloutGenerator:
    def __init__(self, scheduler, tokenizer, max_tokens: int = 1024, group_size: int = 8, temperature: float = 1.0,
                 top_k: int = 0, top_p: float = 1.0, frequency_penalty: float = 0.0, rep_window: int = 64):
        self.scheduler = scheduler
        self.tokenizer = tokenizer
        self.max_tokens = max_tokens
        self.group_size = group_size
        self.temperature = temperature
        self.top_k = top_k
        self.top_p = top_p
        self.frequency_penalty = frequency_penalty
        self.rep_window = rep_window

    @torch.no_grad()
    def generate(self, batch: Dict) -> RawRollout:
        model = self.scheduler.model
        was = model.training
        model.eval()
        try:
            texts, prompt_ids = self._prepare_prompts(batch)
            return self.generate_from_ids(prompt_ids, texts)
        finally:
            model.train(was)

    def generate_from_ids(self, prompt_ids: List[List[int]], texts: Optional[List[str]] = None) -> RawRollout:
        B, G = len(prompt_ids), self.group_size
        flat = [list(ids) for ids in prompt_ids for _ in range(G)]
        results = self.scheduler.run_batch(flat, max_tokens=self.max_tokens, temperature=self.temperature,
                                           top_k=self.top_k, top_p=self.top_p,
                                           frequency_penalty=self.frequency_penalty, rep_window=self.rep_window,
                                           return_logprobs=True)
        if len(results) != B * G:
            raise RuntimeError(f"Rollout scheduler returned {len(results)} results, expected {B * G}")
        dev = self.scheduler.device
        R = max(1, max(len(t) for t, _ in results))
        P = max(len(x) for x in prompt_ids)
        prompts = torch.zeros(B, P, dtype=torch.long)
        pmask = torch.zeros(B, P, dtype=torch.bool)
        for i, ids in enumerate(prompt_ids):
            prompts[i, P - len(ids):] = torch.tensor(ids, dtype=torch.long)
            pmask[i, P - len(ids):] = True
        resp = torch.full((B, G, R), _PAD, dtype=torch.long)
        rmask = torch.zeros(B, G, R, dtype=torch.bool)
        lps = torch.zeros(B, G, R, dtype=torch.float32)
        rtexts: List[List[str]] = [[] for _ in range(B)]
        for k, (tok, lp) in enumerate(results):
            if len(tok) != len(lp):
                raise RuntimeError("Rollout scheduler returned misaligned token IDs and logprobs")
            i, g = divmod(k, G)
            n = len(tok)
            if n:
                resp[i, g, :n] = torch.tensor(tok, dtype=torch.long)
                rmask[i, g, :n] = True
                lps[i, g, :n] = torch.tensor(lp, dtype=torch.float32)
            rtexts[i].append(self.tokenizer.decode(tok, skip_special_tokens=True) if self.tokenizer else "")
        return RawRollout(prompts=prompts.to(dev), prompt_mask=pmask.to(dev), responses=resp.to(dev),
                          response_mask=rmask.to(dev), logprobs_old=lps.to(dev),
                          prompt_texts=texts or [""] * B, response_texts=rtexts)

    def _prepare_prompts(self, batch: Dict) -> Tuple[List[str], List[List[int]]]:
        if "messages" in batch:
            msgs = batch["messages"]
        elif "instruction" in batch:
            ins = batch["instruction"]
            n = len(ins)
            inp = batch.get("input") or [""] * n
            out = batch.get("output") or [""] * n
            msgs = [self._instruction_to_messages(a, b, c) for a, b, c in zip(ins, inp, out)]
        else:
            raise ValueError("Rollout batch must contain either 'messages' or 'instruction' "
                             f"(optionally 'input'/'output'); got keys: {list(batch.keys())}")
        texts = [self.tokenizer.apply_chat_template(m, tokenize=False, add_generation_prompt=True) for m in msgs]
        ids = [list(self.tokenizer.encode(t)) for t in texts]
        return texts, ids

    @staticmethod
    def _instruction_to_messages(instruction: str, inp: str = "", output: str = "") -> List[Dict[str, str]]:
        m = []
        if instruction:
            m.append({"role": "system", "content": instruction})
        if inp:
            m.append({"role": "user", "content": inp})
        if output:
            m.append({"role": "assistant", "content": output})
        return m


class RolloutRunner:
    def __init__(self, generator: RolloutGenerator, reward_model: BaseRewardModel, rollout_interval: int = 512):
        self.generator = generator
        self.reward_model = reward_model
        self.rollout_interval = rollout_interval
        self._cache: Optional[RolloutResult] = None
        self._cache_key = None
        self._steps_since_rollout = 0

    def step(self) -> None:
        self._steps_since_rollout += 1

    def clear_cache(self) -> None:
        self._cache = None
        self._cache_key = None

    @staticmethod
    def _batch_key(batch: Dict):
        def freeze(v):
            if isinstance(v, dict):
                return tuple(sorted((k, freeze(x)) for k, x in v.items()))
            if isinstance(v, (list, tuple)):
                return tuple(freeze(x) for x in v)
            if isinstance(v, torch.Tensor):
                return tuple(v.flatten().tolist())
            return v

        return tuple((f, freeze(batch[f])) for f in ("messages", "instruction", "input", "output", "prompt_ids")
                     if f in batch)

    def _score(self, raw: RawRollout) -> RolloutResult:
        r = self.reward_model.score(raw.prompt_texts, raw.response_texts)
        if not isinstance(r, torch.Tensor):
            r = torch.as_tensor(r, dtype=torch.float32)
        if tuple(r.shape) != tuple(raw.responses.shape[:2]):
            raise ValueError(f"Reward model returned shape {tuple(r.shape)}, expected {tuple(raw.responses.shape[:2])}")
        if not torch.isfinite(r).all():
            raise ValueError("Reward model returned non-finite values")
        return RolloutResult(prompts=raw.prompts, prompt_mask=raw.prompt_mask, responses=raw.responses,
                             response_mask=raw.response_mask, logprobs_old=raw.logprobs_old,
                             prompt_texts=raw.prompt_texts, response_texts=raw.response_texts,
                             rewards=r.to(device=raw.prompts.device, dtype=torch.float32))

    def __call__(self, batch: Dict) -> Tuple[RolloutResult, bool]:
        key = self._batch_key(batch)
        if self._cache is None or key != self._cache_key or self._steps_since_rollout >= self.rollout_interval:
            if "prompt_ids" in batch:
                raw = self.generator.generate_from_ids([list(map(int, p)) for p in batch["prompt_ids"]])
            else:
                raw = self.generator.generate(batch)
            self._cache = self._score(raw)
            self._cache_key = key
            self._steps_since_rollout = 0
            return self._cache, True
        return self._cache, False
