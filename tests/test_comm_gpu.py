"""Fused NVLink all-reduce on 2-4 GPUs (one process per GPU, NCCL bootstrap).

Checks the mean against an fp32 average of every rank's inputs, the squared
norm against the reduced values (and bitwise equal on every rank), repeated
calls (epochs), many rounds, the NCCL fallback for ineligible tensors, DDP
training with the fused backend against the NCCL backend, and the bounded
peer wait: a rank that never joins makes the other rank's kernel give up and
report kErrWaitPeer instead of hanging.
"""

import os
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu

NGPU = torch.cuda.device_count() if torch.cuda.is_available() else 0
need2 = pytest.mark.skipif(NGPU < 2, reason="needs 2 GPUs")


def _init(rank, world, port):
    import torch.distributed as dist

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120), device_id=torch.device("cuda", rank))
    return dist


def _ar_worker(rank, world, port):
    dist = _init(rank, world, port)
    try:
        from astrai_b200.ops._ext import native
        from astrai_b200.parallel.symm import FusedAllReduce

        native().read_error()
        ar = FusedAllReduce(round_elems=8 * world * 3000, ctas=8)  # many rounds per call
        sizes = [4096 * 8, 2048, 8 * 1000 + 8, 24, 13]  # 13 elements: NCCL fallback
        for it in range(3):
            g = torch.Generator(device="cuda").manual_seed(100 * it + rank)
            grads = [torch.randn(n, device="cuda", generator=g).to(torch.bfloat16) for n in sizes]
            ref = []
            for o in grads:
                lst = [torch.empty_like(o) for _ in range(world)]
                dist.all_gather(lst, o)
                ref.append(torch.stack([t.float() for t in lst]).sum(0) / world)
            sumsq = ar.all_reduce_mean(grads)
            torch.cuda.synchronize()
            for out, rf in zip(grads, ref):
                tol = rf.abs() * 2 ** -7 + 1e-6  # one bf16 rounding of the fp32 mean
                assert ((out.float() - rf).abs() <= tol).all()
            want = sum(float(o.float().pow(2).sum()) for o in grads)
            assert abs(float(sumsq) - want) <= 1e-4 * want
            allv = [torch.zeros(1, device="cuda") for _ in range(world)]
            dist.all_gather(allv, sumsq.clone())
            assert all(torch.equal(allv[0], v) for v in allv[:4] if v is not None), "norms differ across ranks"
        assert native().read_error() == 0
        ar.close()
    finally:
        dist.destroy_process_group()


def _ddp_worker(rank, world, port, backend, out_path):
    dist = _init(rank, world, port)
    try:
        from astrai_b200.config import AutoRegressiveLMConfig
        from astrai_b200.models import AutoRegressiveLM
        from astrai_b200.ops.loss import cross_entropy
        from astrai_b200.optim import FusedAdamW
        from astrai_b200.parallel import ExecutorFactory

        torch.manual_seed(0)
        cfg = AutoRegressiveLMConfig(vocab_size=1024, hidden_size=256, num_attention_heads=2, num_key_value_heads=1,
                                     intermediate_size=512, num_hidden_layers=2, max_position_embeddings=256)
        model = AutoRegressiveLM(cfg).cuda().to(torch.bfloat16)
        ex = ExecutorFactory.create("ddp", grad_accum_steps=1, comm_backend=backend)
        model = ex.wrap(model)
        opt = FusedAdamW(model.parameters(), lr=1e-3, weight_decay=0.1)
        g = torch.Generator(device="cuda").manual_seed(7 + rank)
        losses, norms = [], []
        for _ in range(4):
            x = torch.randint(0, 1024, (2, 129), device="cuda", generator=g)
            loss = cross_entropy(model(x[:, :-1])["logits"], x[:, 1:])
            ex.backward(loss)
            norms.append(float(ex.clip_grad_norm(model, 1.0)))
            opt.step()
            opt.zero_grad()
            losses.append(float(loss))
        if rank == 0:
            torch.save({"losses": losses, "norms": norms}, out_path)
    finally:
        dist.destroy_process_group()


def _timeout_worker(rank, world, port):
    dist = _init(rank, world, port)
    try:
        from astrai_b200.ops._ext import native
        from astrai_b200.parallel.symm import FusedAllReduce

        native().read_error()
        ar = FusedAllReduce(ctas=4, wait_s=0.5)
        grads = [torch.ones(4096, device="cuda", dtype=torch.bfloat16)]
        if rank == 0:  # rank 1 never joins this call: rank 0's bounded waits must expire
            ar.all_reduce_mean(grads)
            torch.cuda.synchronize()
            assert native().read_error() == 5  # kErrWaitPeer
        dist.barrier()
        ar.close()
    finally:
        dist.destroy_process_group()


def _sharded_muon_worker(rank, world, port, out_path):
    """Owner-sharded Muon (update applied to every rank's copy over NVLink) against the plain
    replicated Muon run on the same gradients: equal parameters, identical on every rank."""
    dist = _init(rank, world, port)
    try:
        from astrai_b200.ops._ext import native
        from astrai_b200.optim import Muon

        native().read_error()
        shapes = [(256, 512)] * 3 + [(512, 256)] * 2 + [(128, 128)] + [(64, 192)]
        torch.manual_seed(0)  # same initial weights and gradient stream on every rank
        init = [torch.randn(s, device="cuda").to(torch.bfloat16) * 0.05 for s in shapes]
        packed = torch.cat([init[0], init[1]])  # two packed views of one storage, as q/k/v are
        a = [torch.nn.Parameter(packed[:256]), torch.nn.Parameter(packed[256:])] + \
            [torch.nn.Parameter(t.clone()) for t in init[2:]]
        b = [torch.nn.Parameter(t.clone()) for t in init]
        kw = dict(lr=0.02, weight_decay=0.1, adjust_lr_fn="match_rms_adamw")
        opt_a = Muon(a, shard=True, **kw)
        opt_b = Muon(b, **kw)
        for step in range(3):
            for pa, pb in zip(a, b):
                g = torch.randn(pa.shape, device="cuda").to(torch.bfloat16)
                pa.grad, pb.grad = g.clone(), g.clone()
            opt_a.step()
            opt_b.step()
        torch.cuda.synchronize()
        assert native().read_error() == 0
        assert opt_a._arena is not None and all(opt_a._arena.holds(p) for p in a)
        assert a[1].data_ptr() == a[0].data_ptr() + a[0].numel() * 2, "packed views no longer adjacent"
        for pa, pb in zip(a, b):
            torch.testing.assert_close(pa.float(), pb.float(), atol=2e-3, rtol=2e-2)
        flat = torch.cat([p.detach().reshape(-1) for p in a])
        allv = [torch.empty_like(flat) for _ in range(world)]
        dist.all_gather(allv, flat)
        assert all(torch.equal(allv[0], v) for v in allv), "replicas differ across ranks"
        owned = sum(1 for p in a if len(opt_a.state.get(p, {})) > 0)
        counts = [torch.zeros(1, device="cuda") for _ in range(world)]
        dist.all_gather(counts, torch.tensor([float(owned)], device="cuda"))
        if rank == 0:
            torch.save({"owned": [int(c) for c in counts]}, out_path)
    finally:
        dist.destroy_process_group()


def _gather_worker(rank, world, port):
    """GEMM fused with the all-gather (epilogue stores into every rank's copy) against the local GEMM
    plus an NCCL all-gather: four calls with new inputs (the buffer is reused, so the flag handshake
    between calls is exercised), then the fused ColumnParallelLinear forward and backward."""
    dist = _init(rank, world, port)
    try:
        from astrai_b200.ops._ext import native
        from astrai_b200.parallel.module import ColumnParallelLinear, GatherGemm

        native().read_error()
        C = native()
        M, K, n = 1000, 512, 264
        gg = GatherGemm()
        for it in range(4):
            torch.manual_seed(100 * it + rank)
            x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
            w = (torch.randn(n, K, device="cuda") * 0.05).to(torch.bfloat16)
            y = gg(x, w)
            loc = torch.empty(M, n, device="cuda", dtype=torch.bfloat16)
            C.gemm(x, w, loc, None, 0, 0)
            parts = [torch.empty_like(loc) for _ in range(world)]
            dist.all_gather(parts, loc)
            torch.testing.assert_close(y, torch.cat(parts, dim=1), atol=0, rtol=0)
        torch.cuda.synchronize()
        assert native().read_error() == 0
        gg.close()
        torch.manual_seed(7)
        layers = [ColumnParallelLinear(None, 512, 1024, bias=False, fused=f).cuda().to(torch.bfloat16) for f in (1, 0)]
        layers[1].weight.data.copy_(layers[0].weight.data)
        torch.manual_seed(8 + rank)
        x0 = torch.randn(4, 300, 512, device="cuda").to(torch.bfloat16)
        g = torch.randn(4, 300, 1024, device="cuda").to(torch.bfloat16)
        outs = []
        for layer in layers:
            x = x0.clone().requires_grad_()
            y = layer(x)
            y.backward(g)
            outs.append((y, x.grad, layer.weight.grad))
        assert layers[0]._gg is not None and layers[1]._gg is None
        for a, b in zip(outs[0], outs[1]):
            torch.testing.assert_close(a.float(), b.float(), atol=2e-2, rtol=2e-2)
        torch.cuda.synchronize()
        assert native().read_error() == 0
        dist.barrier()
        layers[0]._gg.close()
    finally:
        dist.destroy_process_group()


def _reduce_worker(rank, world, port):
    """GEMM fused with the all-reduce (partials pushed to the row owners as tiles finish, owners sum
    and broadcast) against the local GEMM + an fp32 sum of every rank's bf16 partial; repeated calls
    and a row count that does not divide evenly; then RowParallelLinear fused vs NCCL, fwd and bwd."""
    dist = _init(rank, world, port)
    try:
        from astrai_b200.ops._ext import native
        from astrai_b200.parallel.module import ReduceGemm, RowParallelLinear

        native().read_error()
        C = native()
        rg = ReduceGemm()
        for it, (M, K, N) in enumerate([(1000, 256, 520), (1000, 256, 520), (777, 128, 264), (777, 128, 264)]):
            torch.manual_seed(100 * it + rank)
            x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
            w = (torch.randn(N, K, device="cuda") * 0.05).to(torch.bfloat16)
            y = rg(x, w)
            loc = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            C.gemm(x, w, loc, None, 0, 0)
            parts = [torch.empty_like(loc) for _ in range(world)]
            dist.all_gather(parts, loc)
            ref = torch.stack([t.float() for t in parts]).sum(0)
            torch.testing.assert_close(y.float(), ref, atol=1e-2, rtol=1e-2)
            same = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(same, y)
            assert all(torch.equal(same[0], t) for t in same), "ranks disagree on the reduced output"
        torch.cuda.synchronize()
        assert native().read_error() == 0
        rg.close()
        torch.manual_seed(9)
        layers = [RowParallelLinear(None, 1024, 512, bias=True, fused=f).cuda().to(torch.bfloat16) for f in (1, 0)]
        layers[1].weight.data.copy_(layers[0].weight.data)
        torch.manual_seed(10 + rank)
        x0 = torch.randn(3, 200, 1024 // world, device="cuda").to(torch.bfloat16)
        torch.manual_seed(11)
        g = torch.randn(3, 200, 512, device="cuda").to(torch.bfloat16)
        outs = []
        for layer in layers:
            x = x0.clone().requires_grad_()
            y = layer(x)
            y.backward(g)
            outs.append((y, x.grad, layer.weight.grad))
        assert layers[0]._rg is not None and layers[1]._rg is None
        for a, b in zip(outs[0], outs[1]):
            torch.testing.assert_close(a.float(), b.float(), atol=3e-2, rtol=2e-2)
        torch.cuda.synchronize()
        assert native().read_error() == 0
        dist.barrier()
        layers[0]._rg.close()
    finally:
        dist.destroy_process_group()


def _spawn(fn, world, *args):
    import torch.multiprocessing as mp

    from astrai_b200.parallel import find_free_port

    mp.start_processes(fn, args=(world, find_free_port()) + args, nprocs=world, start_method="spawn", join=True)


@need2
def test_gemm_fused_allreduce_matches_sum():
    _spawn(_reduce_worker, min(NGPU, 4))


@need2
def test_gemm_fused_allgather_matches_nccl():
    _spawn(_gather_worker, min(NGPU, 4))


@need2
def test_fused_allreduce_matches_fp32_mean():
    _spawn(_ar_worker, min(NGPU, 4))


@need2
def test_ddp_fused_backend_matches_nccl(tmp_path):
    world = 2
    _spawn(_ddp_worker, world, "nccl", str(tmp_path / "nccl.pt"))
    _spawn(_ddp_worker, world, "fused", str(tmp_path / "fused.pt"))
    a, b = torch.load(tmp_path / "nccl.pt"), torch.load(tmp_path / "fused.pt")
    for x, y in zip(a["losses"], b["losses"]):
        assert abs(x - y) <= 2e-2 * abs(x)
    for x, y in zip(a["norms"], b["norms"]):
        assert abs(x - y) <= 2e-2 * abs(x)


@need2
def test_fused_allreduce_bounded_wait_reports_missing_peer():
    _spawn(_timeout_worker, 2)


@need2
@pytest.mark.parametrize("chunk_bytes", [None, "1"])
def test_sharded_muon_matches_replicated(tmp_path, monkeypatch, chunk_bytes):
    """chunk_bytes "1": one matrix per Newton-Schulz launch, so a shape group's flag is raised only
    by its last launch (the ranks started here read the variable at import)."""
    if chunk_bytes is not None:
        monkeypatch.setenv("ASTRAI_NS_CHUNK_BYTES", chunk_bytes)
    _spawn(_sharded_muon_worker, 2, str(tmp_path / "owned.pt"))
    owned = torch.load(tmp_path / "owned.pt")["owned"]
    assert sum(owned) == 7 and all(n > 0 for n in owned)  # each matrix has exactly one owner
