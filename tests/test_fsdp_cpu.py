"""Sharded data parallelism on the CPU: the whole-tensor sharding plan of the fused FSDP backend
(pure host logic, identical on every rank) and the torch ``fully_shard`` executor on gloo ranks
against a single-process run over the same global batch."""

import os

import pytest
import torch
import torch.nn as nn

from astrai_b200.parallel.fsdp import ShardPlan, model_units


def _sizes(n=40, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [(f"p{i}", int(torch.randint(1, 5000, (1,), generator=g)) * 16) for i in range(n)]


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_plan_owns_every_parameter_once_and_balances(world):
    params = _sizes()
    plan = ShardPlan(params, world)
    assert len(plan.owner) == len(params) and all(0 <= r < world for r in plan.owner)
    owned = [plan.owned(r) for r in range(world)]
    assert sorted(i for o in owned for i in o) == list(range(len(params)))
    total = sum(b for _, b in params)
    assert sum(plan.load) == total
    # largest-first to the least-loaded rank: no rank exceeds the mean by more than the largest tensor
    assert max(plan.load) <= total / world + max(b for _, b in params)
    assert plan.imbalance() >= 1.0


def test_plan_layouts_are_aligned_and_disjoint():
    params = _sizes(25, seed=3)
    plan = ShardPlan(params, 4)
    spans = sorted((plan.grad_off[i], plan.grad_off[i] + b) for i, (_, b) in enumerate(params))
    for (a0, a1), (b0, _) in zip(spans, spans[1:]):
        assert a1 <= b0
    assert all(o % 256 == 0 for o in plan.grad_off) and spans[-1][1] <= plan.grad_bytes
    for r in range(4):
        own = sorted((plan.param_off[i], plan.param_off[i] + plan.nbytes[i]) for i in plan.owned(r))
        for (a0, a1), (b0, _) in zip(own, own[1:]):
            assert a1 <= b0
        assert all(o % 256 == 0 for o, _ in own)
        assert (own[-1][1] if own else 0) <= plan.param_bytes


def test_plan_is_a_function_of_sizes_and_world():
    params = _sizes(30, seed=7)
    a, b = ShardPlan(params, 5), ShardPlan(list(params), 5)
    assert a.owner == b.owner and a.param_off == b.param_off and a.grad_off == b.grad_off
    # ties go to the lowest rank: equal sizes are dealt round-robin
    eq = ShardPlan([(f"w{i}", 1024) for i in range(6)], 3)
    assert eq.owner == [0, 1, 2, 0, 1, 2]


class _Net(nn.Module):
    def __init__(self):
        super().__init__()
        self.inp = nn.Linear(16, 32)
        self.layers = nn.ModuleList([nn.Linear(32, 32) for _ in range(3)])
        self.out = nn.Linear(32, 4)

    def forward(self, x):
        x = self.inp(x)
        for layer in self.layers:
            x = torch.relu(layer(x))
        return self.out(x)


def test_units_are_the_reference_wrapping_units():
    units = model_units(_Net())
    assert len(units) == 5  # inp, 3 layers, out


def _batches(steps, world, per_rank=8):
    g = torch.Generator().manual_seed(123)
    return [torch.randn(world, per_rank, 16, generator=g) for _ in range(steps)]


def _plan_worker(rank, world, port, sizes, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = ShardPlan(sizes, world)
        got = [None] * world
        dist.all_gather_object(got, (plan.owner, plan.param_off, plan.grad_off))
        q.put(all(g == got[0] for g in got))
    finally:
        dist.destroy_process_group()


def test_plan_identical_on_every_gloo_rank():
    import torch.multiprocessing as mp

    from astrai_b200.parallel import find_free_port

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = 3
    mp.start_processes(_plan_worker, args=(world, find_free_port(), _sizes(33, seed=11), q), nprocs=world,
                       start_method="spawn", join=True)
    assert all(q.get() for _ in range(world))


def _fsdp_worker(rank, world, port, steps, q):
    import torch.distributed as dist

    from astrai_b200.parallel.executor import ExecutorFactory

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        model = _Net()
        ex = ExecutorFactory.create("fsdp2", grad_accum_steps=1)
        model = ex.wrap(model)
        opt = torch.optim.AdamW(model.parameters(), lr=1e-2, weight_decay=0.01)
        losses = []
        for xb in _batches(steps, world):
            loss = model(xb[rank]).pow(2).mean()
            loss.backward()
            ex.finish_step(model)
            opt.step()
            ex.after_optimizer_step()
            opt.zero_grad()
            t = loss.detach().clone()
            dist.all_reduce(t)
            losses.append(float(t) / world)
        sd = ex.unwrap_model(model)
        if rank == 0:
            q.put((losses, {k: v.detach().numpy().copy() for k, v in sd.items()}))  # by value
    finally:
        dist.destroy_process_group()


def test_torch_fsdp2_executor_on_gloo_matches_one_process():
    import torch.multiprocessing as mp

    from astrai_b200.parallel import find_free_port

    steps, world = 4, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.start_processes(_fsdp_worker, args=(world, find_free_port(), steps, q), nprocs=world, start_method="spawn",
                       join=True)
    losses, sd = q.get()
    torch.manual_seed(0)
    ref = _Net()
    opt = torch.optim.AdamW(ref.parameters(), lr=1e-2, weight_decay=0.01)
    ref_losses = []
    for xb in _batches(steps, world):
        # the mean over ranks of per-rank means = the mean over the global batch (equal rank batches)
        loss = torch.stack([ref(xb[r]).pow(2).mean() for r in range(world)]).mean()
        loss.backward()
        opt.step()
        opt.zero_grad()
        ref_losses.append(float(loss))
    assert losses == pytest.approx(ref_losses, rel=1e-4, abs=1e-6)
    for k, v in ref.state_dict().items():
        torch.testing.assert_close(torch.from_numpy(sd[k]), v, atol=1e-5, rtol=1e-4)
