"""Training strategies: seq / sft / dpo / grpo (+ online_dpo / online_grpo).

Loss definitions follow the reference (astrai/trainer/strategy.py):
* seq:  mean CE over all targets with label smoothing;
* sft:  CE over tokens with ``loss_mask`` (ignore_index -100), attention
        restricted to the document of each token (packed sequences);
* dpo:  ``-logsigmoid(beta * ((pi_c - pi_r) - (ref_c - ref_r)))`` with
        response-token log-prob sums (``reduction="sum"`` by default);
* grpo: group-normalised advantages ``(r - mean) / (std_biased + 1e-8)``,
        token-level PPO clip, k1 KL ``exp(ref-pol) - (ref-pol) - 1`` against a
        frozen reference, token mean over response tokens.

Differences that matter for speed: CE and token log-probs run in the fused
kernels on bf16 logits (no fp32 [tokens, vocab] copy); document and padding
masks are passed to attention as int32 segment ids instead of dense
``[B, 1, S, S]`` boolean masks; DPO runs policy/reference forwards on the
concatenated chosen+rejected batch as the reference does.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Callable, Dict, Optional, Union

import torch
import torch.nn as nn
import torch.nn.functional as F

from astrai_b200.factory import Registry
from astrai_b200.ops.loss import cross_entropy, token_logprobs


def create_ref_model(model_fn: Callable[[], nn.Module], state_dict: Dict[str, torch.Tensor]) -> nn.Module:
    ref = model_fn()
    ref.load_state_dict(state_dict)
    ref.requires_grad_(False)
    ref.eval()
    return ref


def move_to_device(batch: Dict[str, torch.Tensor], device) -> Dict[str, torch.Tensor]:
    return {k: (v.to(device, non_blocking=True) if isinstance(v, torch.Tensor) else v) for k, v in batch.items()}


def doc_ids_from_positions(position_ids: torch.Tensor) -> torch.Tensor:
    """Document index of every token: a new document starts where the position does not increase."""
    start = torch.zeros_like(position_ids[:, :1], dtype=torch.int32)
    bounds = (position_ids[:, 1:] <= position_ids[:, :-1]).to(torch.int32)
    return torch.cat([start, bounds.cumsum(1, dtype=torch.int32)], dim=1)


def make_doc_boundary_mask(position_ids: torch.Tensor) -> torch.Tensor:
    """Dense [B, 1, S, S] same-document & causal mask (reference API; the hot path uses segment ids)."""
    doc = doc_ids_from_positions(position_ids)
    S = position_ids.size(1)
    same = doc.unsqueeze(-1) == doc.unsqueeze(-2)
    causal = torch.tril(torch.ones(S, S, dtype=torch.bool, device=position_ids.device))
    return (same & causal).unsqueeze(1)


def padding_segments(valid: torch.Tensor) -> torch.Tensor:
    """Segment ids for key padding: valid tokens share id 0, each padding token gets a unique negative id."""
    B, S = valid.shape
    pad = -(torch.arange(S, device=valid.device, dtype=torch.int32) + 1).expand(B, S)
    return torch.where(valid.bool(), torch.zeros_like(pad), pad)


def get_logprobs(model, input_ids: torch.Tensor, attn_mask: Optional[torch.Tensor], loss_mask: torch.Tensor,
                 reduction: str, seg_ids: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Per-token log p(x_t | x_<t) of ``input_ids[:, 1:]``, masked by ``loss_mask[:, 1:]``.

    ``attn_mask`` may be a dense mask (reference API) or None with ``seg_ids``.
    """
    if reduction not in ("mean", "sum", "none"):
        raise ValueError(f"reduction must be one of ['mean', 'sum', 'none'], got '{reduction}'")
    tgt = input_ids[:, 1:]
    lm = loss_mask[:, 1:].to(torch.float32)
    if attn_mask is not None:
        am = attn_mask[:, :, :-1, :-1] if attn_mask.dim() == 4 else attn_mask[:, :-1]
        logits = model(input_ids[:, :-1], am)["logits"]
    else:
        logits = model(input_ids[:, :-1], seg_ids=None if seg_ids is None else seg_ids[:, :-1])["logits"]
    lp = token_logprobs(logits, tgt)
    if reduction == "mean":
        return (lp * lm).sum(-1) / lm.sum(-1).clamp(min=1.0)
    if reduction == "sum":
        return (lp * lm).sum(-1)
    return lp * lm


class BaseStrategy(ABC):
    """Offline strategies consume dataset batches; with a RolloutRunner injected
    (``set_rollout_runner``) they produce their own batches from rollouts."""

    # the loss of a fixed-shape batch is computed with device work only (see trainer/graph_step.py)
    cuda_graph_safe = False

    def __init__(self, model, device, **kwargs):
        self.model = model
        self.device = device
        self.executor = kwargs.pop("executor", None)
        self.extra_kwargs = kwargs
        self._rollout_runner = None

    @abstractmethod
    def compute_loss(self, batch: Dict[str, torch.Tensor]) -> torch.Tensor: ...

    def supports_online(self) -> bool:
        return False

    def set_rollout_runner(self, runner) -> None:
        self._rollout_runner = runner

    def prepare_from_rollout(self, result) -> Dict[str, torch.Tensor]:
        raise NotImplementedError(f"{type(self).__name__} does not support online rollout")

    def _on_rollout_refresh(self) -> None:
        pass

    def on_optimizer_step(self) -> None:
        if self._rollout_runner is not None:
            self._rollout_runner.step()

    def _add_aux(self, out: Dict[str, torch.Tensor], loss: torch.Tensor) -> torch.Tensor:
        aux = out.get("aux_loss") if isinstance(out, dict) else None
        return loss + aux if aux is not None else loss

    def __call__(self, batch: Dict[str, torch.Tensor]) -> torch.Tensor:
        if self._rollout_runner is None:
            return self.compute_loss(batch)
        result, fresh = self._rollout_runner(batch)
        if fresh:
            self._on_rollout_refresh()
        return self.compute_loss(self.prepare_from_rollout(result))


class StrategyFactory(Registry["BaseStrategy"]):
    pass


@StrategyFactory.register("seq")
class SEQStrategy(BaseStrategy):
    cuda_graph_safe = True

    def __init__(self, model, device, label_smoothing: float = 0.0, **kwargs):
        super().__init__(model, device, **kwargs)
        self.label_smoothing = label_smoothing

    def compute_loss(self, batch):
        batch = move_to_device(batch, self.device)
        out = self.model(input_ids=batch["input_ids"])
        loss = cross_entropy(out["logits"], batch["target_ids"], label_smoothing=self.label_smoothing)
        return self._add_aux(out, loss)


@StrategyFactory.register("sft")
class SFTStrategy(BaseStrategy):
    cuda_graph_safe = True

    def __init__(self, model, device, label_smoothing: float = 0.0, **kwargs):
        super().__init__(model, device, **kwargs)
        self.label_smoothing = label_smoothing

    def compute_loss(self, batch):
        batch = move_to_device(batch, self.device)
        pos = batch["position_ids"]
        target = batch["target_ids"].masked_fill(~batch["loss_mask"].bool(), -100)
        out = self.model(input_ids=batch["input_ids"], position_ids=pos, seg_ids=doc_ids_from_positions(pos))
        loss = cross_entropy(out["logits"], target, label_smoothing=self.label_smoothing, ignore_index=-100)
        return self._add_aux(out, loss)


@StrategyFactory.register("dpo")
class DPOStrategy(BaseStrategy):
    def __init__(self, model, device, ref_model, beta: float = 0.1, reduction: str = "sum", **kwargs):
        super().__init__(model, device, **kwargs)
        self.ref_model = ref_model
        self.beta = beta
        self.reduction = reduction

    def compute_loss(self, batch):
        batch = move_to_device(batch, self.device)
        ids = torch.cat([batch["chosen"], batch["rejected"]], 0)
        lmask = torch.cat([batch["chosen_mask"], batch["rejected_mask"]], 0)
        seg = padding_segments(ids.ne(0))  # key padding (token id 0) + causal
        lp = get_logprobs(self.model, ids, None, lmask, self.reduction, seg_ids=seg)
        with torch.no_grad():
            lr_ = get_logprobs(self.ref_model, ids, None, lmask, self.reduction, seg_ids=seg)
        n = batch["chosen"].shape[0]
        diff = (lp[:n] - lp[n:]) - (lr_[:n] - lr_[n:])
        return -F.logsigmoid(self.beta * diff).mean()

    def supports_online(self) -> bool:
        return True

    def prepare_from_rollout(self, result):
        best = result.rewards.argmax(-1)
        worst = result.rewards.argmin(-1)
        idx = torch.arange(result.responses.shape[0], device=result.responses.device)
        return {"chosen": result.responses[idx, best], "chosen_mask": result.response_mask[idx, best].float(),
                "rejected": result.responses[idx, worst], "rejected_mask": result.response_mask[idx, worst].float()}


@StrategyFactory.register("grpo")
class GRPOStrategy(BaseStrategy):
    def __init__(self, model, device, old_model, ref_model, clip_eps: float = 0.2, kl_coef: float = 0.01,
                 group_size: int = 4, **kwargs):
        super().__init__(model, device, **kwargs)
        self.old_model = old_model
        self.ref_model = ref_model
        self.clip_eps = clip_eps
        self.kl_coef = kl_coef
        self.group_size = group_size

    def sync_old_model(self) -> None:
        sd = self.executor.unwrap_model(self.model) if self.executor is not None else self.model.state_dict()
        if sd is not None:
            self.old_model.load_state_dict(sd)

    def compute_loss(self, batch):
        batch = move_to_device(batch, self.device)
        prompts, responses, masks, rewards = batch["prompts"], batch["responses"], batch["masks"], batch["rewards"]
        B, G, R = responses.shape
        resp = responses.reshape(-1, R)
        rmask = masks.reshape(-1, R)
        prompt = prompts.unsqueeze(1).expand(-1, G, -1).reshape(B * G, -1)
        pmask = batch.get("prompt_mask")
        if pmask is None:
            pmask = prompts.ne(0)
        pmask = pmask.unsqueeze(1).expand(-1, G, -1).reshape(B * G, -1)
        P = prompt.shape[1]
        seqs = torch.cat([prompt, resp], -1)
        loss_mask = torch.cat([torch.zeros_like(prompt, dtype=torch.bool), rmask.bool()], -1)
        seg = padding_segments(torch.cat([pmask.bool(), rmask.bool()], -1))
        pol = get_logprobs(self.model, seqs, None, loss_mask, "none", seg_ids=seg)[:, P - 1:]
        with torch.no_grad():
            old = get_logprobs(self.old_model, seqs, None, loss_mask, "none", seg_ids=seg)[:, P - 1:]
            ref = get_logprobs(self.ref_model, seqs, None, loss_mask, "none", seg_ids=seg)[:, P - 1:]
        pol, old, ref = pol.view(B, G, -1), old.view(B, G, -1), ref.view(B, G, -1)
        tm = rmask.view(B, G, -1).float()
        eps = 1e-8
        adv = ((rewards - rewards.mean(-1, keepdim=True)) / (rewards.std(-1, keepdim=True, unbiased=False) + eps))
        adv = adv.unsqueeze(-1)
        ratio = torch.exp(pol - old)
        surr = torch.min(ratio * adv, torch.clamp(ratio, 1 - self.clip_eps, 1 + self.clip_eps) * adv)
        cnt = tm.sum().clamp(min=1.0)
        policy_loss = (-surr * tm).sum() / cnt
        r = torch.exp(ref - pol)
        kl = r - torch.log(r + eps) - 1.0
        return policy_loss + self.kl_coef * (kl * tm).sum() / cnt

    def supports_online(self) -> bool:
        return True

    def prepare_from_rollout(self, result):
        return {"prompts": result.prompts, "prompt_mask": result.prompt_mask, "responses": result.responses,
                "masks": result.response_mask, "rewards": result.rewards}

    def _on_rollout_refresh(self) -> None:
        self.sync_old_model()


StrategyFactory.alias("online_grpo", "grpo")
StrategyFactory.alias("online_dpo", "dpo")
