"""Checkpoint and forward parity with the reference implementation (CPU, fp32).

A model saved by the reference's ``save_pretrained`` loads with this framework's
``AutoModel.from_pretrained`` and produces the same logits, and the reverse.
Skipped when the reference package is not installed under ``baseline/_ref``.
"""

import os
import sys
import types

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "astrai")), reason="reference not installed")

CFG = dict(vocab_size=256, hidden_size=64, num_attention_heads=4, num_key_value_heads=2, intermediate_size=128,
           max_position_embeddings=128, num_hidden_layers=2, rms_norm_eps=1e-5, rope_theta=10000.0)
VARIANTS = {"gqa": {}, "tied": {"tie_word_embeddings": True}, "qk_norm": {"use_qk_norm": True},
            "ntk": {"rope_scaling": {"type": "ntk", "factor": 2.0}},
            "moe": {"ffn_type": "moe", "n_routed_experts": 4, "n_shared_experts": 2, "n_activated_experts": 2},
            "mla": {"attn_type": "mla", "kv_lora_rank": 16, "qk_nope_head_dim": 8, "qk_rope_head_dim": 8,
                    "num_key_value_heads": 4},
            "gated": {"use_gated_attention": True}}


def _ref():
    sys.modules.setdefault("h5py", types.ModuleType("h5py"))
    if REF not in sys.path:
        sys.path.append(REF)
    import astrai.config
    import astrai.model

    return astrai.config, astrai.model


@pytest.mark.parametrize("name", sorted(VARIANTS))
def test_reference_checkpoint_loads_and_matches(name, tmp_path):
    from astrai_b200.models import AutoModel

    rcfg_mod, rmodel_mod = _ref()
    kw = {**CFG, **VARIANTS[name]}
    torch.manual_seed(0)
    ref = rmodel_mod.AutoRegressiveLM(rcfg_mod.AutoRegressiveLMConfig(**kw)).float().eval()
    ref.save_pretrained(str(tmp_path / "ref"))
    ours = AutoModel.from_pretrained(str(tmp_path / "ref")).float().eval()
    ids = torch.randint(0, CFG["vocab_size"], (2, 33), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        a = ref(ids)["logits"].float()
        b = ours(ids)["logits"].float()
    torch.testing.assert_close(b, a, atol=1e-4, rtol=1e-4)
    # and back: our save_pretrained loads in the reference
    ours.save_pretrained(str(tmp_path / "ours"))
    back = rmodel_mod.AutoModel.from_pretrained(str(tmp_path / "ours")).float().eval()
    with torch.no_grad():
        torch.testing.assert_close(back(ids)["logits"].float(), a, atol=1e-4, rtol=1e-4)


def test_training_trajectory_matches_reference(tmp_path):
    """BASELINE config 1 in one process: the same init, batches, AdamW(1e-4, wd 0.1), clip 1.0 and label
    smoothing 0.05 give the reference's loss trajectory (fp32 CPU)."""
    import torch.nn.functional as F

    from astrai_b200.models import AutoModel
    from astrai_b200.ops.loss import cross_entropy
    from astrai_b200.optim import FusedAdamW

    rcfg_mod, rmodel_mod = _ref()
    kw = dict(vocab_size=1024, hidden_size=256, num_attention_heads=8, num_key_value_heads=2, intermediate_size=688,
              max_position_embeddings=128, num_hidden_layers=4, rms_norm_eps=1e-5, rope_theta=10000.0,
              tie_word_embeddings=True)
    torch.manual_seed(3407)
    ref = rmodel_mod.AutoRegressiveLM(rcfg_mod.AutoRegressiveLMConfig(**kw)).float().train()
    ref.save_pretrained(str(tmp_path / "init"))
    ours = AutoModel.from_pretrained(str(tmp_path / "init")).float().train()
    opt_r = torch.optim.AdamW(ref.parameters(), lr=1e-4, weight_decay=0.1)
    opt_o = FusedAdamW(ours.parameters(), lr=1e-4, weight_decay=0.1)
    g = torch.Generator().manual_seed(3407)
    lr_, lo_ = [], []
    for _ in range(6):
        x = torch.randint(0, 1024, (2, 129), generator=g)
        lr = F.cross_entropy(ref(x[:, :-1])["logits"].reshape(-1, 1024).float(), x[:, 1:].reshape(-1),
                             label_smoothing=0.05)
        lo = cross_entropy(ours(x[:, :-1])["logits"], x[:, 1:], label_smoothing=0.05)
        for m, loss, opt in ((ref, lr, opt_r), (ours, lo, opt_o)):
            opt.zero_grad()
            loss.backward()
            torch.nn.utils.clip_grad_norm_(m.parameters(), 1.0)
            opt.step()
        lr_.append(lr.item())
        lo_.append(lo.item())
    assert max(abs(a - b) for a, b in zip(lr_, lo_)) < 1e-4, (lr_, lo_)


def _pair(tmp_path, kw=None):
    from astrai_b200.models import AutoModel

    rcfg_mod, rmodel_mod = _ref()
    torch.manual_seed(5)
    ref = rmodel_mod.AutoRegressiveLM(rcfg_mod.AutoRegressiveLMConfig(**(kw or CFG))).float()
    d = str(tmp_path / "m")
    ref.save_pretrained(d)
    return ref, AutoModel.from_pretrained(d).float(), rmodel_mod, d


@pytest.mark.parametrize("kind", ["seq", "sft", "dpo", "grpo"])
def test_strategy_losses_and_grads_match_reference(kind, tmp_path):
    """Each training strategy's loss and weight gradient equal the reference's on the same batch (the
    reference builds dense masks, this framework segment ids; both must mean the same attention)."""
    import copy

    from astrai_b200.models import AutoModel
    from astrai_b200.trainer.strategy import StrategyFactory

    ref, ours, rmod, d = _pair(tmp_path)
    from astrai.trainer.strategy import StrategyFactory as RefFactory

    g = torch.Generator().manual_seed(9)
    V, B, S = CFG["vocab_size"], 2, 24
    if kind in ("seq", "sft"):
        x = torch.randint(1, V, (B, S + 1), generator=g)
        batch = {"input_ids": x[:, :-1], "target_ids": x[:, 1:]}
        if kind == "sft":
            pos = torch.cat([torch.arange(10), torch.arange(S - 10)]).expand(B, -1).clone()  # two packed docs
            batch.update(position_ids=pos, loss_mask=torch.rand(B, S, generator=g) > 0.3)
        kw = {"label_smoothing": 0.05}
    elif kind == "dpo":
        ids = lambda: torch.randint(1, V, (B, S), generator=g)  # noqa: E731
        m = torch.zeros(B, S)
        m[:, S // 2:] = 1
        batch = {"chosen": ids(), "rejected": ids(), "chosen_mask": m.bool(), "rejected_mask": m.bool()}
        kw = {"beta": 0.1}
    else:
        G, P, R = 3, 8, 10
        batch = {"prompts": torch.randint(1, V, (B, P), generator=g),
                 "responses": torch.randint(1, V, (B, G, R), generator=g),
                 # responses are valid prefixes followed by padding, as rollouts produce them
                 "masks": torch.arange(R) < torch.randint(1, R + 1, (B, G, 1), generator=g),
                 "rewards": torch.rand(B, G, generator=g)}
        kw = {"clip_eps": 0.2, "kl_coef": 0.04, "group_size": G}
    extra_r, extra_o = {}, {}
    if kind in ("dpo", "grpo"):
        extra_r["ref_model"] = rmod.AutoModel.from_pretrained(d).float().eval()
        extra_o["ref_model"] = AutoModel.from_pretrained(d).float().eval()
        with torch.no_grad():  # a reference policy that differs from the trained one
            for p in list(extra_r["ref_model"].parameters()) + list(extra_o["ref_model"].parameters()):
                p.mul_(0.9)
    if kind == "grpo":
        extra_r["old_model"] = copy.deepcopy(extra_r["ref_model"])
        extra_o["old_model"] = copy.deepcopy(extra_o["ref_model"])
    sr = RefFactory.create(kind, model=ref, device="cpu", **kw, **extra_r)
    so = StrategyFactory.create(kind, model=ours, device="cpu", **kw, **extra_o)
    lr = sr.compute_loss({k: v.clone() for k, v in batch.items()})
    lo = so.compute_loss({k: v.clone() for k, v in batch.items()})
    torch.testing.assert_close(lo.detach(), lr.detach(), atol=2e-5, rtol=2e-4)
    lr.backward()
    lo.backward()
    gr = dict(ref.named_parameters())
    for n, p in ours.named_parameters():
        if n in gr and gr[n].grad is not None:
            torch.testing.assert_close(p.grad, gr[n].grad, atol=2e-5, rtol=2e-3)
