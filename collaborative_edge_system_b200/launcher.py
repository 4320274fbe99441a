"""Process-group start-up: one process per GPU (torchrun) or N local processes.

``init_distributed`` mirrors collab_infer ``distributed/launcher.py:55-96``
(environment variables, backend from ``$COLLAB_BACKEND``), defaulting to
NCCL when CUDA is present because the attention path runs on GPUs.
``launch_local`` spawns N processes on this host (gloo unless told
otherwise) and returns each rank's result; the multi-rank CPU tests use it.
"""

from __future__ import annotations

import os
import pickle
import socket
from datetime import timedelta
from typing import Any, Callable, Dict, List, Optional, Sequence

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def find_free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def init_distributed(backend: Optional[str] = None, *, timeout_s: float = 600.0) -> torch.device:
    """Initialise the default group from RANK/WORLD_SIZE/MASTER_*; return this rank's device."""
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", rank))
    backend = backend or os.environ.get("COLLAB_BACKEND") or ("nccl" if torch.cuda.is_available() else "gloo")
    device = torch.device("cpu")
    if torch.cuda.is_available():
        device = torch.device("cuda", local % torch.cuda.device_count())
        torch.cuda.set_device(device)
    if world > 1 and not dist.is_initialized():
        addr = os.environ.get("MASTER_ADDR", "127.0.0.1")
        port = int(os.environ.get("MASTER_PORT", 29500))
        kw = {"device_id": device} if backend == "nccl" else {}
        dist.init_process_group(backend, init_method=f"tcp://{addr}:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=timeout_s), **kw)
    return device


def _entry(rank: int, fn: Callable[..., Any], world: int, port: int, backend: str, args: Sequence[Any],
           threads: int, queue: Any, timeout_s: float, env: Optional[Dict[str, str]]) -> None:
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    if env:
        os.environ.update(env)
    torch.set_num_threads(max(1, threads))
    kw = {}
    if backend == "nccl":  # one GPU per rank, bound before the communicator is created
        dev = torch.device("cuda", rank % torch.cuda.device_count())
        torch.cuda.set_device(dev)
        kw["device_id"] = dev
    dist.init_process_group(backend, init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s), **kw)
    try:
        res = fn(rank, world, *args)
        if queue is not None:
            queue.put((rank, pickle.dumps(res)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def launch_local(fn: Callable[..., Any], world_size: int, args: Sequence[Any] = (), *, backend: str = "gloo",
                 threads_per_rank: Optional[int] = None, return_results: bool = False, timeout_s: float = 300.0,
                 env: Optional[Dict[str, str]] = None) -> Optional[List[Any]]:
    """Run ``fn(rank, world_size, *args)`` in ``world_size`` spawned processes (``launcher.py:139-197``)."""
    port = find_free_port()
    threads = threads_per_rank or max(1, (os.cpu_count() or 1) // world_size)
    ctx = mp.get_context("spawn")
    queue = ctx.SimpleQueue() if return_results else None
    os.environ.setdefault("TORCH_CPP_LOG_LEVEL", "ERROR")
    procs = mp.start_processes(_entry, args=(fn, world_size, port, backend, tuple(args), threads, queue, timeout_s, env),
                               nprocs=world_size, join=False, start_method="spawn")
    results: Dict[int, Any] = {}

    def drain() -> None:
        while queue is not None and not queue.empty():
            r, payload = queue.get()
            results[r] = pickle.loads(payload)

    while not procs.join(timeout=0.05):
        drain()
    drain()
    if not return_results:
        return None
    missing = [r for r in range(world_size) if r not in results]
    if missing:
        raise RuntimeError(f"ranks {missing} did not return a result")
    return [results[r] for r in range(world_size)]


__all__ = ["find_free_port", "init_distributed", "launch_local"]
