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
