"""CPU tests: Trainer loop, accumulation, checkpoint/resume after a failure,
schedules, strategies, and 2-rank gloo data parallelism."""

import json
import os

import pytest
import torch
from torch.utils.data import Dataset

from tests.conftest import TINY_CFG


class RandSeq(Dataset):
    def __init__(self, n, seq=16, vocab=512, seed=0):
        g = torch.Generator().manual_seed(seed)
        self.x = torch.randint(0, vocab, (n, seq + 1), generator=g)

    def __len__(self):
        return len(self.x)

    def __getitem__(self, i):
        return {"input_ids": self.x[i, :-1], "target_ids": self.x[i, 1:]}


class FailingSeq(RandSeq):
    """Raises after `stop_after` items: host-side fault injection."""

    def __init__(self, n, stop_after):
        super().__init__(n)
        self.stop_after, self.count = stop_after, 0

    def __getitem__(self, i):
        self.count += 1
        if self.count == self.stop_after:
            raise RuntimeError("Simulated failure")
        return super().__getitem__(i)


def make_cfg(ds, d, **kw):
    from astrai_b200.config import AutoRegressiveLMConfig, TrainConfig
    from astrai_b200.models import AutoRegressiveLM
    from astrai_b200.optim import FusedAdamW
    from astrai_b200.trainer import SchedulerFactory

    base = dict(model_fn=lambda: AutoRegressiveLM(AutoRegressiveLMConfig(**TINY_CFG)), strategy="seq", dataset=ds,
                optimizer_fn=lambda m: FusedAdamW(m.parameters(), lr=1e-3),
                scheduler_fn=lambda o: SchedulerFactory.create("cosine", o, warmup_steps=1, lr_decay_steps=10),
                batch_per_device=2, grad_accum_steps=2, ckpt_dir=os.path.join(d, "ck"), ckpt_interval=2,
                log_dir=os.path.join(d, "logs"), device_type="cpu", nprocs=1, random_seed=7)
    base.update(kw)
    return TrainConfig(**base)


def test_trainer_steps_checkpoints_metrics(tmpdir_path):
    from astrai_b200.trainer import Trainer

    t = Trainer(make_cfg(RandSeq(16), tmpdir_path, metrics=["loss", "grad_norm", "tokens_per_s", "mfu"]))
    t.train()
    ctx = t.last_context
    assert ctx.optimizer_step == 4 and ctx.consumed_samples == 16
    assert sorted(os.listdir(os.path.join(tmpdir_path, "ck"))) == ["epoch_0_step_2", "epoch_0_step_4"]
    meta = json.load(open(os.path.join(tmpdir_path, "ck", "epoch_0_step_4", "meta.json")))
    assert meta["consumed_samples"] == 16 and meta["batch_per_device"] == 2
    assert os.path.exists(os.path.join(tmpdir_path, "ck", "epoch_0_step_4", "optimizer.pt"))
    logs = os.listdir(os.path.join(tmpdir_path, "logs"))
    rows = [json.loads(x) for x in open(os.path.join(tmpdir_path, "logs", sorted(logs)[-1]))]
    assert any(r["type"] == "step" and "grad_norm" in r for r in rows)
    assert all(r["tokens_per_s"] > 0 and 0 < r["mfu"] < 1 for r in rows if r["type"] == "step")
    assert ctx.kwargs["tokens"] == 16 * (RandSeq(1).x.shape[1] - 1)


def test_failure_checkpoint_and_resume(tmpdir_path):
    from astrai_b200.trainer import Trainer

    with pytest.raises(RuntimeError, match="Simulated failure"):
        Trainer(make_cfg(FailingSeq(20, stop_after=7), tmpdir_path, ckpt_interval=100)).train()
    ck = os.listdir(os.path.join(tmpdir_path, "ck"))
    assert ck == ["epoch_0_step_1"]  # on_error checkpoint (4 samples consumed = 1 optimizer step)
    path = os.path.join(tmpdir_path, "ck", ck[0])
    t = Trainer(make_cfg(RandSeq(20), tmpdir_path, ckpt_interval=100))
    t.train(param_path=path, resume=True)
    assert t.last_context.consumed_samples == 20
    last = json.load(open(os.path.join(tmpdir_path, "ck", "epoch_0_step_5", "meta.json")))
    assert last["consumed_samples"] == 20


@pytest.mark.parametrize("kind,kw", [("cosine", dict(warmup_steps=3, lr_decay_steps=10)),
                                     ("sgdr", dict(warmup_steps=2, cycle_length=4, t_mult=2)),
                                     ("wsd", dict(warmup_steps=2, stable_steps=3, decay_steps=5))])
def test_schedules_and_state(kind, kw):
    from astrai_b200.trainer import SchedulerFactory

    p = torch.nn.Parameter(torch.zeros(1))
    opt = torch.optim.SGD([p], lr=1.0)
    s = SchedulerFactory.create(kind, opt, min_rate=0.1, **kw)
    lrs = []
    for _ in range(20):
        lrs.append(opt.param_groups[0]["lr"])
        opt.step()
        s.step()
    assert lrs[0] == pytest.approx(0.1)  # warmup floor
    assert max(lrs) == pytest.approx(1.0) and min(lrs) >= 0.1 - 1e-9
    sd = s.state_dict()
    s2 = SchedulerFactory.create(kind, torch.optim.SGD([p], lr=1.0), min_rate=0.5, **kw)
    s2.load_state_dict(sd)
    assert s2.min_rate == 0.1 and s2.last_epoch == s.last_epoch


def test_strategies_losses_and_grpo_properties():
    from astrai_b200.config import AutoRegressiveLMConfig
    from astrai_b200.models import AutoRegressiveLM
    from astrai_b200.trainer.strategy import StrategyFactory, create_ref_model

    torch.manual_seed(0)
    fn = lambda: AutoRegressiveLM(AutoRegressiveLMConfig(**TINY_CFG))  # noqa: E731
    m = fn()
    ref = create_ref_model(fn, m.state_dict())
    B, S = 2, 12
    sft = StrategyFactory.create("sft", model=m, device="cpu")
    batch = {"input_ids": torch.randint(0, 512, (B, S)), "target_ids": torch.randint(0, 512, (B, S)),
             "position_ids": torch.tensor([[0, 1, 2, 3, 0, 1, 2, 3, 4, 5, 6, 7]] * B),
             "loss_mask": torch.rand(B, S) > 0.3}
    l1 = sft(batch)
    l1.backward()
    assert torch.isfinite(l1)
    dpo = StrategyFactory.create("dpo", model=m, device="cpu", ref_model=ref, beta=0.1)
    ch = torch.randint(1, 512, (B, S))
    l2 = dpo({"chosen": ch, "rejected": torch.randint(1, 512, (B, S)), "chosen_mask": torch.ones(B, S),
              "rejected_mask": torch.ones(B, S)})
    assert abs(l2.item() - 0.6931) < 1e-3  # policy == reference at init -> -log(sigmoid(0))
    grpo = StrategyFactory.create("grpo", model=m, device="cpu", old_model=ref, ref_model=ref, group_size=3)
    b = {"prompts": torch.randint(1, 512, (B, 5)), "responses": torch.randint(1, 512, (B, 3, 4)),
         "masks": torch.ones(B, 3, 4, dtype=torch.bool), "rewards": torch.ones(B, 3)}
    l3 = grpo(b)
    assert abs(l3.item()) < 1e-5  # identical rewards -> zero advantage, KL 0 at init
    b["rewards"] = torch.rand(B, 3)
    l4 = grpo(b)
    l4.backward()
    assert torch.isfinite(l4)
    assert all(p.grad is None for p in ref.parameters())


def _ddp_worker(rank, world, port, out_dir):
    import torch.distributed as dist

    from astrai_b200.parallel import setup_parallel

    with setup_parallel(rank, world, rank, "gloo", "127.0.0.1", str(port), "cpu"):
        losses = run_config1(rank, world)
        dist.all_reduce(losses)  # global batch loss = mean of the equal-size rank losses
        losses /= world
        if rank == 0:
            torch.save(losses, os.path.join(out_dir, "ddp.pt"))
        dist.barrier()


CONFIG1 = dict(vocab_size=1024, hidden_size=256, num_hidden_layers=4, num_attention_heads=8, num_key_value_heads=2,
               intermediate_size=688, rms_norm_eps=1e-5, rope_theta=10000.0, tie_word_embeddings=True,
               max_position_embeddings=128)


def run_config1(rank, world, per_rank=2, steps=10):
    """fp32, tied, label smoothing 0.05, AdamW 1e-4 wd 0.1, clip 1.0."""
    from astrai_b200.config import AutoRegressiveLMConfig
    from astrai_b200.models import AutoRegressiveLM
    from astrai_b200.ops.loss import cross_entropy
    from astrai_b200.optim import FusedAdamW
    from astrai_b200.parallel import ExecutorFactory

    torch.manual_seed(3407)
    model = AutoRegressiveLM(AutoRegressiveLMConfig(**CONFIG1))
    ex = ExecutorFactory.create("ddp" if world > 1 else "none", grad_accum_steps=1)
    model = ex.wrap(model)
    opt = FusedAdamW(model.parameters(), lr=1e-4, weight_decay=0.1)
    g = torch.Generator().manual_seed(11)
    data = torch.randint(0, 1024, (steps, 4, 129), generator=g)
    losses = []
    for s in range(steps):
        x = data[s, rank * per_rank:(rank + 1) * per_rank]
        loss = cross_entropy(model(x[:, :-1])["logits"], x[:, 1:], label_smoothing=0.05)
        ex.backward(loss)  # sync step: gradients averaged across ranks
        ex.clip_grad_norm(model, 1.0)
        opt.step()
        opt.zero_grad()
        losses.append(loss.detach())
    return torch.stack(losses)


def test_config1_gloo_ddp_matches_single_process(tmpdir_path):
    import torch.multiprocessing as mp

    from astrai_b200.parallel import find_free_port

    port = find_free_port()
    mp.start_processes(_ddp_worker, args=(2, port, tmpdir_path), nprocs=2, start_method="spawn", join=True)
    ddp = torch.load(os.path.join(tmpdir_path, "ddp.pt"))
    single = run_config1(0, 1, per_rank=4)
    # averaged gradients of 2 x 2 samples == gradients of 4 samples: identical trajectories
    assert ddp.shape == (10,)
    torch.testing.assert_close(ddp, single, atol=2e-5, rtol=2e-5)


def _allreduce_worker(rank, world, port):
    import torch.distributed as dist

    from astrai_b200.parallel import get_rank, get_world_size, only_on_rank, setup_parallel

    with setup_parallel(rank, world, rank, "gloo", "127.0.0.1", str(port), "cpu"):
        t = torch.tensor([float(get_rank() + 1)])
        dist.all_reduce(t)
        assert t.item() == 3.0 and get_world_size() == 2
        out = only_on_rank(0, sync=True)(lambda: "r0")()
        assert (out == "r0") == (rank == 0)


def test_spawn_gloo_collectives():
    import torch.multiprocessing as mp

    from astrai_b200.parallel import find_free_port

    mp.start_processes(_allreduce_worker, args=(2, find_free_port()), nprocs=2, start_method="spawn", join=True)


def test_cli_train_flags_and_config(tmpdir_path, model_dir):
    import os

    from astrai_b200.cli.train import build_config, compute_total_steps, parse_args, scheduler_kwargs
    from astrai_b200.serialization import save_bin

    assert compute_total_steps(100, 2, 4, 2, 3) == (13 // 3) * 2
    assert scheduler_kwargs("wsd", 100, 0.1)["stable_steps"] == 72
    data = os.path.join(tmpdir_path, "data")
    save_bin(os.path.join(data, "shard"), {"sequence": [torch.randint(0, 500, (400,), dtype=torch.int32)]})
    args = parse_args(["--train_type", "seq", "--param_path", model_dir, "--data_root_path", data, "--window_size",
                       "32", "--device_type", "cpu", "--comm_backend", "fused", "--parallel_mode", "ddp"])
    cfg = build_config(args)
    assert cfg.executor_kwargs == {"comm_backend": "fused", "expert_parallel": False}
    assert cfg.strategy == "seq" and len(cfg.dataset) > 0


def test_profiler_callback_writes_trace(tmp_path):
    from astrai_b200.trainer.train_callback import CallbackFactory, nvtx_range

    cb = CallbackFactory.create("profiler", profile_dir=str(tmp_path), wait=0, warmup=1, active=1)
    cb.on_train_begin(None)
    for _ in range(3):
        with nvtx_range("forward"):
            torch.randn(32, 32) @ torch.randn(32, 32)
        cb.on_optimizer_step(None)
    cb.on_train_end(None)
    names = os.listdir(tmp_path)
    assert "kernels.txt" in names and any(n.startswith("trace_step") for n in names)


def test_cuda_graph_flag_falls_back_to_eager_on_cpu(tmpdir_path):
    """``cuda_graph=True`` off a CUDA device: the loop runs eagerly with the same results."""
    from astrai_b200.trainer import Trainer
    from astrai_b200.trainer.graph_step import GraphedMicroStep

    runs = []
    for flag in (False, True):
        torch.manual_seed(11)  # model init
        t = Trainer(make_cfg(RandSeq(8), os.path.join(tmpdir_path, str(flag)), cuda_graph=flag))
        t.train()
        runs.append(t.last_context)
    assert runs[1].kwargs["graph_step"] is None
    for pa, pb in zip(runs[0].model.parameters(), runs[1].model.parameters()):
        assert torch.equal(pa, pb)
    m = torch.nn.Linear(4, 4)
    step = GraphedMicroStep(lambda b: m(b["x"]).sum(), m, torch.device("cpu"))
    assert step.disabled_reason == "not a CUDA device"
    step({"x": torch.ones(2, 4)})
    assert m.weight.grad is not None and step.replays == 0
