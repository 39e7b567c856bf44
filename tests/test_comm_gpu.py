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


def _spawn(fn, world, *args):
    import torch.multiprocessing as mp

    from astrai_b200.parallel import find_free_port

    mp.start_processes(fn, args=(world, find_free_port()) + args, nprocs=world, start_method="spawn", join=True)


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
