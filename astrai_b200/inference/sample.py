"""Token sampling: temperature -> top-k -> top-p -> frequency penalty -> draw.

API parity with astrai/inference/sample.py:18-375 (strategy classes,
``SamplingPipeline`` and ``sample()`` with the same arguments and order).

Execution differs: on CUDA ``sample()`` is ONE kernel launch per batch
(``_C.sample``) that reads each logits row once into registers, finds the
top-k and nucleus thresholds by bisection on the float bit pattern (no sort,
no ``topk``), applies the frequency penalty from the history window, draws
by inverse CDF with a counter-based RNG held on the device, and writes the
token and its log-probability under the final distribution. No host
synchronisation happens, so the call can be captured in a CUDA graph.
The strategy classes keep the reference's PyTorch semantics for any device.

Greedy decoding: a row whose temperature is exactly 0 takes the argmax of
the raw logits and reports its log-probability under softmax(raw logits).
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from typing import List, Optional, Tuple, Union

import torch
from torch import Tensor

Scalar = Union[float, int, Tensor]


class BaseSamplingStrategy(ABC):
    @abstractmethod
    def apply(self, logits: Tensor, filter_value: float = -float("inf"), input_ids: Optional[Tensor] = None,
              input_mask: Optional[Tensor] = None) -> Tensor:
        raise NotImplementedError


def _per_row(v: Scalar, logits: Tensor) -> Tensor:
    if isinstance(v, Tensor):
        return v.to(logits.device).reshape(-1, 1)
    return torch.full((logits.shape[0], 1), float(v), device=logits.device)


class TemperatureStrategy(BaseSamplingStrategy):
    def __init__(self, temperature: Scalar = 1.0):
        self.temperature = temperature

    def apply(self, logits, filter_value=-float("inf"), input_ids=None, input_mask=None):
        t = self.temperature
        if isinstance(t, Tensor):
            return logits / t.to(logits.device).reshape(-1, 1).clamp(min=1e-8)
        return logits / max(float(t), 1e-8) if t != 1.0 else logits


class TopKStrategy(BaseSamplingStrategy):
    """Keeps the k largest logits per row (0 disables)."""

    def __init__(self, top_k: Scalar = 0):
        self.top_k = top_k

    def apply(self, logits, filter_value=-float("inf"), input_ids=None, input_mask=None):
        k = _per_row(self.top_k, logits).long().clamp(min=0, max=logits.shape[-1])
        kmax = int(k.max())
        if kmax <= 0:
            return logits
        vals = torch.topk(logits, kmax, dim=-1).values
        thr = vals.gather(-1, (k - 1).clamp(min=0))
        thr = torch.where(k > 0, thr, torch.full_like(thr, -float("inf")))
        return logits.masked_fill(logits < thr, filter_value)


class TopPStrategy(BaseSamplingStrategy):
    """Nucleus filtering: keeps a token while the mass of more likely tokens
    is <= top_p (so the smallest set whose mass exceeds top_p survives)."""

    def __init__(self, top_p: Scalar = 1.0):
        self.top_p = top_p

    def apply(self, logits, filter_value=-float("inf"), input_ids=None, input_mask=None):
        p = _per_row(self.top_p, logits).to(torch.float32)
        if bool((p >= 1.0).all()):
            return logits
        srt, idx = torch.sort(logits, descending=True, dim=-1)
        cum = torch.softmax(srt.float(), dim=-1).cumsum(-1)
        remove = (cum - torch.softmax(srt.float(), dim=-1)) > p  # exclusive mass
        remove &= p < 1.0
        mask = torch.zeros_like(remove).scatter(-1, idx, remove)
        return logits.masked_fill(mask, filter_value)


class FrequencyPenaltyStrategy(BaseSamplingStrategy):
    """Subtracts ``penalty * count(token)`` over the history window."""

    def __init__(self, penalty: Scalar = 0.0):
        self.penalty = penalty

    def apply(self, logits, filter_value=-float("inf"), input_ids=None, input_mask=None):
        if input_ids is None:
            return logits
        pen = _per_row(self.penalty, logits).to(logits.dtype)
        if bool((pen == 0).all()):
            return logits
        ids = input_ids.to(logits.device).long()
        valid = (ids >= 0) & (ids < logits.shape[-1])
        if input_mask is not None:
            valid &= input_mask.to(logits.device).bool()
        counts = torch.zeros_like(logits)
        counts.scatter_add_(1, torch.where(valid, ids, 0), valid.to(logits.dtype))
        return logits - pen * counts


class SamplingPipeline(BaseSamplingStrategy):
    def __init__(self, strategies: List[BaseSamplingStrategy]):
        self.strategies = strategies

    def apply(self, logits, filter_value=-float("inf"), input_ids=None, input_mask=None):
        for s in self.strategies:
            logits = s.apply(logits, filter_value, input_ids, input_mask)
        return logits

    def _greedy_rows(self, logits: Tensor) -> Optional[Tensor]:
        first = self.strategies[0] if self.strategies else None
        if not isinstance(first, TemperatureStrategy):
            return None
        return _per_row(first.temperature, logits).reshape(-1) == 0

    @torch.inference_mode()
    def sample(self, logits: Tensor, filter_value: float = -float("inf"), input_ids: Optional[Tensor] = None,
               input_mask: Optional[Tensor] = None, return_logprobs: bool = False,
               generator: Optional[torch.Generator] = None):
        greedy = self._greedy_rows(logits)
        x = self.apply(logits.float().clone(), filter_value, input_ids, input_mask)
        logp = torch.log_softmax(x, dim=-1)
        tok = torch.multinomial(logp.exp().nan_to_num(0.0), 1, generator=generator).squeeze(-1)
        if greedy is not None and bool(greedy.any()):
            raw = logits.float()
            tok = torch.where(greedy, raw.argmax(-1), tok)
            logp = torch.where(greedy[:, None], torch.log_softmax(raw, -1), logp)
        if not return_logprobs:
            return tok
        return tok, logp.gather(-1, tok[:, None]).squeeze(-1)


class DeviceRNG:
    """Counter-based RNG state on the device: int64 ``(seed, counter)``.

    The sampling kernel hashes (seed, counter, row); :meth:`advance` bumps
    the counter on the stream, so successive captured graph replays draw
    fresh numbers without host involvement.
    """

    def __init__(self, device, seed: Optional[int] = None):
        if seed is None:
            seed = int(torch.randint(0, 2**62, (1,)).item())
        # a normal tensor even when first made under inference_mode (a later advance outside it is legal)
        with torch.inference_mode(False):
            self.state = torch.tensor([seed, 0], dtype=torch.int64, device=device)

    def advance(self) -> None:
        self.state[1:].add_(1)


_RNGS = {}


def _rng_for(device) -> DeviceRNG:
    key = str(device)
    if key not in _RNGS:
        _RNGS[key] = DeviceRNG(device)
    return _RNGS[key]


def _as_row_tensor(v: Scalar, rows: int, device, dtype) -> Tensor:
    if isinstance(v, Tensor):
        t = v.to(device=device, dtype=dtype).reshape(-1)
        return t.expand(rows).contiguous() if t.numel() == 1 else t.contiguous()
    return torch.full((rows,), v, device=device, dtype=dtype)


def fused_sample(logits: Tensor, temperature: Tensor, top_k: Tensor, top_p: Tensor, penalty: Tensor,
                 history: Optional[Tensor], rng: DeviceRNG, out_tok: Tensor,
                 out_logprob: Optional[Tensor] = None) -> None:
    """Graph-capturable sampling into preallocated outputs (CUDA).

    ``temperature/top_p/penalty`` fp32 [rows], ``top_k`` int32 [rows],
    ``history`` int64 [rows, H] padded with -1.
    """
    from astrai_b200.ops._ext import native

    native().sample(logits, temperature, top_k, top_p, penalty, history, rng.state, out_tok, out_logprob)
    rng.advance()


@torch.inference_mode()
def sample(logits: Tensor, temperature: Scalar = 1.0, top_k: Scalar = 0, top_p: Scalar = 1.0,
           frequency_penalty: Scalar = 0.0, input_ids: Optional[Tensor] = None, input_mask: Optional[Tensor] = None,
           filter_value: float = -float("inf"), return_logprobs: bool = False
           ) -> Union[Tensor, Tuple[Tensor, Tensor]]:
    """Sample one token per row of ``logits [batch, vocab]``.

    Same arguments and result as the reference ``sample()``; ``input_ids``
    is the history window (with ``input_mask`` marking real tokens).
    """
    if logits.is_cuda and logits.dim() == 2 and filter_value == -float("inf") and logits.dtype in (
            torch.float32, torch.bfloat16):
        rows, dev = logits.shape[0], logits.device
        hist = None
        if input_ids is not None:
            hist = input_ids.to(dev).long()
            if input_mask is not None:
                hist = hist.masked_fill(~input_mask.to(dev).bool(), -1)
            hist = hist.contiguous()
        tok = torch.empty(rows, dtype=torch.int64, device=dev)
        lp = torch.empty(rows, dtype=torch.float32, device=dev) if return_logprobs else None
        fused_sample(logits if logits.stride(-1) == 1 else logits.contiguous(),
                     _as_row_tensor(temperature, rows, dev, torch.float32),
                     _as_row_tensor(top_k, rows, dev, torch.int32),
                     _as_row_tensor(top_p, rows, dev, torch.float32),
                     _as_row_tensor(frequency_penalty, rows, dev, torch.float32), hist, _rng_for(dev), tok, lp)
        return (tok, lp) if return_logprobs else tok
    pipe = SamplingPipeline([TemperatureStrategy(temperature), TopKStrategy(top_k), TopPStrategy(top_p),
                             FrequencyPenaltyStrategy(frequency_penalty)])
    return pipe.sample(logits, filter_value, input_ids, input_mask, return_logprobs)
