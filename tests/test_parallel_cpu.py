"""CPU tests of the parallel layer's host logic: the fused all-reduce's
round / slice / chunk decomposition (host restatement of the kernel)."""

import torch


def test_allreduce_plan_covers_every_element_once_and_norm():
    from astrai_b200.parallel.symm import AllReducePlan, emulate_fused_allreduce

    for world, ctas, R, N in [(2, 3, 16 * 2 * 50, 8 * 777), (4, 2, 8 * 4 * 4096, 8 * 9000), (8, 5, 8 * 8 * 10, 8 * 13)]:
        plan = AllReducePlan(world, R, ctas)
        seen = torch.zeros(N, dtype=torch.int32)
        for rd in range(plan.rounds(N)):
            for s in range(world):
                for b in range(ctas):
                    for c0, c1 in plan.chunks(N, rd, s, b):
                        seen[c0:c1] += 1
        assert bool((seen == 1).all())
        g = torch.Generator().manual_seed(world)
        flats = [torch.randn(N, generator=g).to(torch.bfloat16) for _ in range(world)]
        outs, sq = emulate_fused_allreduce(flats, plan)
        want = (torch.stack([f.float() for f in flats]).sum(0) / world).to(torch.bfloat16)
        assert all(torch.equal(o, want) for o in outs)
        assert abs(sq - float(want.float().pow(2).sum())) <= 1e-3 * sq
        assert plan.off_gather + 4 * plan.R <= plan.nbytes


def _tp_worker(rank, world, port):
    import torch.distributed as dist

    from astrai_b200.parallel import ColumnParallelLinear, RowParallelLinear, setup_parallel

    with setup_parallel(rank, world, rank, "gloo", "127.0.0.1", str(port), "cpu"):
        torch.manual_seed(0)
        full = torch.nn.Linear(8, 6)
        x = torch.randn(3, 8, requires_grad=True)
        ref = full(x)
        ref.sum().backward()
        row = RowParallelLinear(None, 8, 6)
        row.load_state_dict(full.state_dict())
        xs = x.detach()[:, rank * 4:(rank + 1) * 4].clone().requires_grad_()
        y = row(xs)
        torch.testing.assert_close(y, ref.detach(), atol=1e-5, rtol=1e-5)
        y.sum().backward()
        torch.testing.assert_close(row.weight.grad, full.weight.grad[:, rank * 4:(rank + 1) * 4], atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(xs.grad, x.grad[:, rank * 4:(rank + 1) * 4], atol=1e-5, rtol=1e-5)
        col = ColumnParallelLinear(None, 8, 6)
        col.load_state_dict(full.state_dict())
        x2 = x.detach().clone().requires_grad_()
        z = col(x2)
        torch.testing.assert_close(z, ref.detach(), atol=1e-5, rtol=1e-5)
        z.sum().backward()
        torch.testing.assert_close(col.weight.grad, full.weight.grad[rank * 3:(rank + 1) * 3], atol=1e-5, rtol=1e-5)
        g = x2.grad.clone()
        dist.all_reduce(g)  # input gradient is the sum over the column shards
        torch.testing.assert_close(g, x.grad, atol=1e-5, rtol=1e-5)


def test_tensor_parallel_layers_gloo():
    import torch.multiprocessing as mp

    from astrai_b200.parallel import find_free_port

    mp.start_processes(_tp_worker, args=(2, find_free_port()), nprocs=2, start_method="spawn", join=True)
