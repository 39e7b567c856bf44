"""The CUDA-graph micro-step (trainer/graph_step.py) against eager micro-steps: same losses and
weights over several optimizer steps, replays actually happen, the launch counter keeps counting,
and the Trainer runs with ``cuda_graph=True``."""

import copy

import pytest
import torch

pytestmark = pytest.mark.gpu


def _model():
    from astrai_b200.config import AutoRegressiveLMConfig
    from astrai_b200.models import AutoRegressiveLM

    cfg = AutoRegressiveLMConfig(vocab_size=512, hidden_size=256, num_hidden_layers=2, rms_norm_eps=1e-5,
                                 intermediate_size=512, tie_word_embeddings=False, max_position_embeddings=512,
                                 rope_theta=10000.0, num_attention_heads=2, num_key_value_heads=1)
    torch.manual_seed(0)
    return AutoRegressiveLM(cfg).to("cuda", torch.bfloat16)


def _loss_fn(model):
    from astrai_b200.ops.loss import cross_entropy

    def f(batch):
        batch = {k: v.to("cuda", non_blocking=True) for k, v in batch.items()}  # no-op for the static buffers
        out = model(input_ids=batch["input_ids"])
        return cross_entropy(out["logits"], batch["target_ids"])

    return f


def test_graphed_micro_step_matches_eager():
    from astrai_b200.ops._ext import native
    from astrai_b200.optim import FusedAdamW
    from astrai_b200.trainer.graph_step import GraphedMicroStep

    ma = _model()
    mb = copy.deepcopy(ma)
    oa, ob = FusedAdamW(ma.parameters(), lr=1e-3), FusedAdamW(mb.parameters(), lr=1e-3)
    accum = 2
    step_b = GraphedMicroStep(_loss_fn(mb), mb, torch.device("cuda"), scale=1.0 / accum, eager_calls=accum)
    fa = _loss_fn(ma)
    g = torch.Generator().manual_seed(1)
    data = torch.randint(0, 512, (5, accum, 2, 129), generator=g).pin_memory()
    la, lb = [], []
    for s in range(5):
        for mi in range(accum):
            x = data[s, mi]
            batch = {"input_ids": x[:, :-1], "target_ids": x[:, 1:]}
            loss = fa({k: v.cuda() for k, v in batch.items()})
            (loss / accum).backward()
            la.append(loss.detach().float())
            n0 = native().launch_count()
            lb.append(step_b(batch).float().clone())
            if step_b.replays and mi == accum - 1 and s == 4:
                assert native().launch_count() - n0 == step_b._launches > 0
        oa.step()
        ob.step()
        oa.zero_grad(set_to_none=False)
        ob.zero_grad(set_to_none=False)
    torch.cuda.synchronize()
    assert step_b.disabled_reason is None, step_b.disabled_reason
    assert step_b.replays == 5 * accum - accum - 1  # eager optimizer step, one captured call, then replays
    for a, b in zip(la, lb):
        assert abs(a.item() - b.item()) <= 1e-3 * abs(a.item())
    for pa, pb in zip(ma.parameters(), mb.parameters()):
        assert torch.allclose(pa.float(), pb.float(), rtol=1e-2, atol=1e-3)


def test_graphed_micro_step_recaptures_on_new_shapes():
    from astrai_b200.trainer.graph_step import GraphedMicroStep

    m = _model()
    step = GraphedMicroStep(_loss_fn(m), m, torch.device("cuda"), eager_calls=1)
    for seq in (64, 64, 64, 96, 96):
        x = torch.randint(0, 512, (2, seq + 1), device="cuda")
        loss = step({"input_ids": x[:, :-1], "target_ids": x[:, 1:]})
        assert torch.isfinite(loss).item()
    # call 1 eager, 2 capture (64), 3 replay, 4 capture (96), 5 replay
    assert step.replays == 2 and step._static["input_ids"].shape[1] == 96


def test_trainer_with_cuda_graph(tmp_path):
    import os

    from torch.utils.data import Dataset

    from astrai_b200.config import AutoRegressiveLMConfig, TrainConfig
    from astrai_b200.models import AutoRegressiveLM
    from astrai_b200.optim import FusedAdamW
    from astrai_b200.trainer import SchedulerFactory, Trainer

    class Seq(Dataset):
        def __init__(self):
            self.x = torch.randint(0, 512, (32, 65), generator=torch.Generator().manual_seed(0))

        def __len__(self):
            return len(self.x)

        def __getitem__(self, i):
            return {"input_ids": self.x[i, :-1], "target_ids": self.x[i, 1:]}

    cfg = AutoRegressiveLMConfig(vocab_size=512, hidden_size=256, num_hidden_layers=2, rms_norm_eps=1e-5,
                                 intermediate_size=512, tie_word_embeddings=False, max_position_embeddings=512,
                                 rope_theta=10000.0, num_attention_heads=2, num_key_value_heads=1)
    tc = TrainConfig(model_fn=lambda: AutoRegressiveLM(cfg).to(torch.bfloat16), strategy="seq", dataset=Seq(),
                     optimizer_fn=lambda m: FusedAdamW(m.parameters(), lr=1e-3),
                     scheduler_fn=lambda o: SchedulerFactory.create("cosine", o, warmup_steps=1, lr_decay_steps=10),
                     batch_per_device=2,
                     grad_accum_steps=2, ckpt_dir=os.path.join(tmp_path, "ck"), ckpt_interval=100,
                     log_dir=os.path.join(tmp_path, "logs"), device_type="cuda", nprocs=1, random_seed=7,
                     cuda_graph=True)
    t = Trainer(tc)
    t.train()
    runner = t.last_context.kwargs["graph_step"]
    assert runner is not None and runner.disabled_reason is None and runner.replays == 16 - 2 - 1
    assert torch.isfinite(t.last_context.loss if isinstance(t.last_context.loss, torch.Tensor)
                          else torch.tensor(t.last_context.loss)).all()
