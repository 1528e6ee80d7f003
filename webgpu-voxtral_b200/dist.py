"""Process-group plumbing for multi-GPU runs (one process per GPU, torch.distributed).

torch.distributed is only the plumbing: rendezvous, barriers, the max-over-ranks
reduction of device timings and the broadcast of the NCCL unique id that the C ABI's
own communicator (vx_tp_init) is built from.  The data path never goes through torch.
"""
from __future__ import annotations

import datetime
import os
from typing import Optional

import torch
import torch.distributed as dist


def env_rank() -> tuple[int, int, int]:
    """(rank, local_rank, world_size) from the torchrun environment (1 process = 0, 0, 1)."""
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def init(backend: Optional[str] = None, timeout_s: float = 120.0, device: Optional[int] = None) -> bool:
    """Initialise the default process group when WORLD_SIZE > 1.  Returns True if distributed."""
    rank, local, world = env_rank()
    if world <= 1:
        return False
    if dist.is_initialized():
        return True
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29511")
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    kw = {}
    if backend == "nccl":
        torch.cuda.set_device(local if device is None else device)
        kw["device_id"] = torch.device("cuda", local if device is None else device)
    dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return True


def barrier():
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


def max_over_ranks(x: float) -> float:
    """Maximum of a host float over all ranks (device timings: the job ends with the slowest rank)."""
    if not (dist.is_available() and dist.is_initialized()):
        return float(x)
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")
    t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def min_over_ranks(x: float) -> float:
    """Minimum of a host float over all ranks (a rate: the job runs at its slowest rank)."""
    return -max_over_ranks(-float(x))


def sum_over_ranks(x: float) -> float:
    if not (dist.is_available() and dist.is_initialized()):
        return float(x)
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")
    t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def broadcast_bytes(payload: Optional[bytes], src: int = 0) -> bytes:
    """Broadcast a small byte string (e.g. a 128-byte NCCL unique id) from `src`."""
    if not (dist.is_available() and dist.is_initialized()):
        assert payload is not None
        return payload
    obj = [payload]
    dist.broadcast_object_list(obj, src=src)
    return obj[0]


def all_gather_bytes(payload: bytes) -> list:
    """Every rank's byte string, in rank order (e.g. 64-byte CUDA IPC handles)."""
    if not (dist.is_available() and dist.is_initialized()):
        return [payload]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, payload)
    return out


def shutdown():
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
