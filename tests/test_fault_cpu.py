"""Host-side failure detection with gloo ranks on CPU: a rank that stops (no heartbeat), a rank
that records its failure, a rank that never reaches a barrier. No GPU is involved."""

import os
import time
from datetime import timedelta

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _init(rank, world, port):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=30))


def _write(path, text):
    with open(path, "w") as fh:
        fh.write(text)


def _dead_rank_worker(rank, world, port, out):
    from astrai_b200.parallel.health import Heartbeat, PeerFailure

    _init(rank, world, port)
    hb = Heartbeat(interval=0.1, timeout=1.0).start()
    hb.wait_all_alive(10.0)
    if rank == world - 1:
        hb.stop()  # this rank "dies": no more beats, no failure note
        time.sleep(6.0)
        return
    seen = "none"
    end = time.monotonic() + 8.0
    while time.monotonic() < end:
        try:
            hb.check()
        except PeerFailure as e:
            seen = ",".join(map(str, e.ranks)) + "|" + e.reasons[e.ranks[0]]
            break
        time.sleep(0.1)
    hb.stop()
    _write(os.path.join(out, f"r{rank}.txt"), seen)
    time.sleep(0.5)


def _failed_rank_worker(rank, world, port, out):
    from astrai_b200.parallel.health import Heartbeat, PeerFailure

    _init(rank, world, port)
    hb = Heartbeat(interval=0.1, timeout=30.0).start()
    hb.wait_all_alive(10.0)
    if rank == 1:
        hb.mark_failed("ValueError('boom at step 3')")
        hb.stop()
        time.sleep(3.0)
        return
    seen = "none"
    t0 = time.monotonic()
    while time.monotonic() - t0 < 5.0:
        try:
            hb.check()
        except PeerFailure as e:
            seen = f"{e.ranks}|{e.reasons[1]}|{time.monotonic() - t0:.2f}"
            break
        time.sleep(0.05)
    hb.stop()
    _write(os.path.join(out, f"r{rank}.txt"), seen)


def _barrier_worker(rank, world, port, out):
    from astrai_b200.parallel.health import PeerFailure, diagnosed_barrier

    _init(rank, world, port)
    if rank == 1:
        time.sleep(5.0)  # never reaches the barrier in time
        return
    try:
        diagnosed_barrier(timeout_s=1.5)
        seen = "passed"
    except PeerFailure as e:
        seen = ",".join(map(str, e.ranks))
    _write(os.path.join(out, f"r{rank}.txt"), seen)


def _run(fn, world, tmp_path):
    from astrai_b200.parallel import find_free_port

    mp.start_processes(fn, args=(world, find_free_port(), str(tmp_path)), nprocs=world, start_method="spawn",
                       join=True)


def _read(tmp_path, r):
    with open(tmp_path / f"r{r}.txt") as fh:
        return fh.read()


def test_heartbeat_names_a_rank_that_stopped(tmp_path):
    _run(_dead_rank_worker, 3, tmp_path)
    for r in (0, 1):
        ranks, reason = _read(tmp_path, r).split("|")
        assert ranks == "2" and "no heartbeat" in reason


def test_failure_note_reaches_peers_before_the_timeout(tmp_path):
    _run(_failed_rank_worker, 2, tmp_path)
    ranks, reason, secs = _read(tmp_path, 0).split("|")
    assert ranks == "[1]" and "boom at step 3" in reason and float(secs) < 2.0


def test_diagnosed_barrier_names_the_missing_rank(tmp_path):
    _run(_barrier_worker, 2, tmp_path)
    assert _read(tmp_path, 0) == "1"
