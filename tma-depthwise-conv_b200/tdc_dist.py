"""One process per GPU: process-group set-up, batch shards and max-over-ranks
timing for jobs that spread the depthwise conv over several GPUs of one node.

The operator has no exchange step: images are independent, so each rank
convolves its own shard of the batch with a replicated 3x3xC filter and no
collective touches the data path.  The process group is used only for the
barriers around a timed region and for reducing timings (max over ranks).
"""
from __future__ import annotations

import contextlib
import datetime
import os
import sys

import torch
import torch.distributed as dist


def env_rank() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment (1 process: 0, 1, 0)."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


@contextlib.contextmanager
def stdout_to_stderr():
    """Send file descriptor 1 to stderr for a while (communicator set-up prints
    a version banner on stdout, which must carry only the result line)."""
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        yield
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)


def init(backend: str, timeout_s: float = 120.0) -> tuple[int, int, int]:
    """Join the process group when WORLD_SIZE > 1 (rendezvous from MASTER_ADDR/PORT).

    The first barrier runs here, so the communicator exists (and has printed
    whatever it prints) before the caller writes to stdout."""
    rank, world, local = env_rank()
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kw = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        with stdout_to_stderr():
            dist.init_process_group(backend, rank=rank, world_size=world,
                                    timeout=datetime.timedelta(seconds=timeout_s), **kw)
            dist.barrier()
    return rank, world, local


def barrier() -> None:
    if dist.is_initialized():
        dist.barrier()


def max_over_ranks(value: float, device: torch.device | str = "cpu") -> float:
    """Largest `value` over all ranks (the job finishes when its slowest rank does)."""
    if not dist.is_initialized():
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, device: torch.device | str = "cpu") -> float:
    if not dist.is_initialized():
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def finalize() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()
