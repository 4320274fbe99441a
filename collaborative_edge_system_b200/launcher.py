"""Process-group start-up: one process per GPU under torchrun, or N local ranks for tests.

``init_distributed`` joins the job described by the ``RANK`` / ``WORLD_SIZE`` /
``LOCAL_RANK`` / ``MASTER_*`` environment (collab_infer
``distributed/launcher.py:55-96``), with NCCL as the default backend when
CUDA is present (``$COLLAB_BACKEND`` overrides it).

``launch_local`` runs ``fn(rank, world_size, *args)`` on N spawned ranks of
this host (collab_infer ``launcher.py:139-197``: same arguments and result
order).  Each rank writes its pickled result, or its traceback, into a
per-job directory; the parent watches the ranks, stops the whole job as soon
as one fails or the deadline passes, and raises with the failing rank's
traceback, so a dead rank never leaves its peers waiting in a collective.
"""

from __future__ import annotations

import os
import pickle
import shutil
import socket
import tempfile
import time
import traceback
from datetime import timedelta
from typing import Any, Callable, Dict, List, Optional, Sequence

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

_GRACE_S = 30.0  # beyond the process-group timeout, before the watchdog stops a job


def find_free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bind_device(local_rank: int) -> torch.device:
    if not torch.cuda.is_available():
        return torch.device("cpu")
    dev = torch.device("cuda", local_rank % torch.cuda.device_count())
    torch.cuda.set_device(dev)
    return dev


def init_distributed(backend: Optional[str] = None, *, timeout_s: float = 600.0) -> torch.device:
    """Join the job of the environment (no-op for one rank); returns this rank's device."""
    env = os.environ
    rank, world = int(env.get("RANK", 0)), int(env.get("WORLD_SIZE", 1))
    backend = backend or env.get("COLLAB_BACKEND") or ("nccl" if torch.cuda.is_available() else "gloo")
    device = _bind_device(int(env.get("LOCAL_RANK", rank)))
    if world > 1 and not dist.is_initialized():
        url = f"tcp://{env.get('MASTER_ADDR', '127.0.0.1')}:{int(env.get('MASTER_PORT', 29500))}"
        extra = {"device_id": device} if backend == "nccl" else {}
        dist.init_process_group(backend, init_method=url, rank=rank, world_size=world,
                                timeout=timedelta(seconds=timeout_s), **extra)
    return device


def _rank_main(rank: int, world: int, port: int, backend: str, fn: Callable[..., Any], args: Sequence[Any],
               threads: int, box: str, keep: bool, timeout_s: float, env: Optional[Dict[str, str]]) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    os.environ.update(env or {})
    torch.set_num_threads(max(1, threads))
    try:
        init_distributed(backend, timeout_s=timeout_s)
        value = fn(rank, world, *args)
        if world > 1:
            dist.barrier()  # every rank finished its collectives before any group is torn down
        payload = pickle.dumps(value if keep else None)
        tmp = os.path.join(box, f"{rank}.part")
        with open(tmp, "wb") as f:
            f.write(payload)
        os.replace(tmp, os.path.join(box, f"{rank}.ok"))
    except BaseException:
        with open(os.path.join(box, f"{rank}.err"), "w") as f:
            f.write(traceback.format_exc())
        raise
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def launch_local(fn: Callable[..., Any], world_size: int, args: Sequence[Any] = (), *, backend: str = "gloo",
                 threads_per_rank: Optional[int] = None, return_results: bool = False, timeout_s: float = 300.0,
                 env: Optional[Dict[str, str]] = None) -> Optional[List[Any]]:
    """Run ``fn(rank, world_size, *args)`` on ``world_size`` spawned ranks; returns the results in rank order
    when ``return_results`` is set.  ``fn`` must be importable by the children (a module-level function)."""
    threads = threads_per_rank or max(1, (os.cpu_count() or 1) // world_size)
    box = tempfile.mkdtemp(prefix="cea-ranks-")
    ctx = mp.get_context("spawn")
    os.environ.setdefault("TORCH_CPP_LOG_LEVEL", "ERROR")
    port = find_free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world_size, port, backend, fn, tuple(args), threads, box,
                                                  return_results, timeout_s, env), daemon=True)
             for r in range(world_size)]
    try:
        for p in procs:
            p.start()
        deadline = time.monotonic() + timeout_s + _GRACE_S
        failed: Optional[int] = None
        while any(p.is_alive() for p in procs):
            failed = next((r for r, p in enumerate(procs) if p.exitcode not in (None, 0)), None)
            if failed is not None or time.monotonic() > deadline:
                break
            time.sleep(0.02)
        stragglers = [r for r, p in enumerate(procs) if p.is_alive()]
        for r in stragglers:
            procs[r].terminate()
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()
                p.join()
        if failed is None:
            failed = next((r for r, p in enumerate(procs) if p.exitcode != 0 and r not in stragglers), None)
        if failed is not None:
            err = os.path.join(box, f"{failed}.err")
            detail = open(err).read() if os.path.exists(err) else f"exit code {procs[failed].exitcode}"
            raise RuntimeError(f"rank {failed} of {world_size} failed:\n{detail}")
        if stragglers:
            raise RuntimeError(f"ranks {stragglers} of {world_size} still ran after {timeout_s + _GRACE_S:.0f} s")
        missing = [r for r in range(world_size) if not os.path.exists(os.path.join(box, f"{r}.ok"))]
        if missing:
            raise RuntimeError(f"ranks {missing} did not report a result")
        if not return_results:
            return None
        results = []
        for r in range(world_size):
            with open(os.path.join(box, f"{r}.ok"), "rb") as f:
                results.append(pickle.load(f))
        return results
    finally:
        shutil.rmtree(box, ignore_errors=True)


__all__ = ["find_free_port", "init_distributed", "launch_local"]
