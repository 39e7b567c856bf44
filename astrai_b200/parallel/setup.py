"""Process launch and process-group plumbing.

Parity: astrai/parallel/setup.py. ``spawn_parallel_fn(func, world_size, ...)``
runs ``func(**kwargs)`` once per rank: in-process when the environment was
prepared by torchrun / torchelastic / an external launcher (RANK and
WORLD_SIZE set), else through ``torch.multiprocessing`` with one spawned
process per rank (all ranks are terminated if one fails). ``setup_parallel``
initialises the process group (``device_id`` bound for NCCL) and exports
LOCAL_RANK / WORLD_SIZE / LOCAL_DEVICE; ``only_on_rank(r, sync)`` runs a
function on one rank, optionally followed by a barrier.

Additions: a configurable process-group timeout (``ASTRAI_PG_TIMEOUT_S``,
default 1800 s) so ranks waiting for a dead peer fail instead of hanging, and
``heartbeat`` helpers used by failure detection (parallel/health.py).
"""

from __future__ import annotations

import os
import socket
from contextlib import contextmanager
from datetime import timedelta
from functools import wraps
from typing import Callable, Optional

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def find_free_port() -> str:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return str(s.getsockname()[1])


def get_current_device() -> str:
    return os.environ.get("LOCAL_DEVICE", "cuda" if torch.cuda.is_available() else "cpu")


def get_world_size() -> int:
    return dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1


def get_rank() -> int:
    return dist.get_rank() if dist.is_available() and dist.is_initialized() else 0


def _pg_timeout() -> timedelta:
    return timedelta(seconds=float(os.environ.get("ASTRAI_PG_TIMEOUT_S", "1800")))


@contextmanager
def setup_parallel(rank: int, world_size: int, local_rank: int, backend: str = "nccl",
                   master_addr: str = "localhost", master_port: str = "29500", device_type: str = "cuda"):
    if dist.is_available() and dist.is_initialized():
        os.environ.setdefault("LOCAL_DEVICE", str(torch.device(device_type, local_rank)))
        yield dist.group.WORLD
        return
    device = torch.device(device_type, local_rank) if device_type != "cpu" else torch.device("cpu")
    os.environ["LOCAL_RANK"] = str(local_rank)
    os.environ["WORLD_SIZE"] = str(world_size)
    os.environ["LOCAL_DEVICE"] = str(device)
    if device_type == "cuda" and torch.cuda.is_available():
        torch.cuda.set_device(local_rank)
    if world_size <= 1:
        yield None
        return
    os.environ["MASTER_ADDR"] = master_addr
    os.environ["MASTER_PORT"] = str(master_port)
    kw = dict(rank=rank, world_size=world_size, backend=backend, timeout=_pg_timeout())
    if backend in ("nccl", "ccl") and device.type != "cpu":
        kw["device_id"] = device
    dist.init_process_group(**kw)
    try:
        yield dist.group.WORLD
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def only_on_rank(rank: int, sync: bool = False):
    def deco(func):
        @wraps(func)
        def wrapper(*args, **kwargs):
            out = func(*args, **kwargs) if get_rank() == rank else None
            if sync and dist.is_available() and dist.is_initialized():
                dist.barrier()
            return out

        return wrapper

    return deco


def _run_rank(rank, world_size, backend, master_addr, master_port, device_type, func, kwargs):
    with setup_parallel(rank, world_size, rank, backend, master_addr, master_port, device_type):
        func(**kwargs)


def _detect_launcher() -> str:
    if dist.is_available() and dist.is_torchelastic_launched():
        return "torchelastic"
    if "LOCAL_WORLD_SIZE" in os.environ:
        return "torchrun"
    if "RANK" in os.environ and "WORLD_SIZE" in os.environ:
        return "external"
    return "local"


def spawn_parallel_fn(func: Callable, world_size: int, backend: str = "nccl", master_addr: str = "localhost",
                      master_port: Optional[str] = None, device_type: str = "cuda", start_method: str = "spawn",
                      **kwargs):
    if master_port is None:
        master_port = find_free_port()
    launcher = _detect_launcher()
    if launcher != "local":
        rank = int(os.environ["RANK"])
        ws = int(os.environ["WORLD_SIZE"])
        local = int(os.environ.get("LOCAL_RANK", rank))
        with setup_parallel(rank, ws, local, backend, os.environ.get("MASTER_ADDR", master_addr),
                            os.environ.get("MASTER_PORT", master_port), device_type):
            func(**kwargs)
        return
    args = (world_size, backend, master_addr, master_port, device_type, func, kwargs)
    if world_size == 1:
        _run_rank(0, *args)
        return
    ctx = mp.start_processes(_run_rank, args=args, nprocs=world_size, start_method=start_method, join=False)
    try:
        while not ctx.join():
            pass
    except BaseException:
        for p in ctx.processes:
            if p.is_alive():
                p.terminate()
        ctx.join()
        raise
