"""Session data parallelism across GPUs (one process per GPU).

Generation sessions are independent (their own noise, context window and
conditioning), so the frame path shards by session with no collective on the
data path: rank r of W takes sessions [r S/W, (r+1) S/W). The only cross-rank
traffic is control: barriers around timed regions and max/sum reductions of
scalars for reporting. This replaces the reference's single-process mesh
(`ttnn.open_mesh_device`, oasis_inference.py:1718-1722), whose multi-chip path
is tensor parallelism with `ttnn.all_reduce` (:1156, :1194).
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist


def shard_sessions(total: int, world: int, rank: int) -> tuple[int, int]:
    """First session and session count of `rank`; every rank gets the same count."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if total % world:
        raise ValueError(f"{total} sessions do not split evenly over {world} GPUs")
    per = total // world
    return rank * per, per


def init_from_env(backend: str | None = None) -> tuple[int, int, int]:
    """(rank, world, local_rank) from torchrun's environment; initialises the
    process group when world > 1 (NCCL on GPUs, gloo otherwise)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        else:
            dist.init_process_group(backend)
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return rank, world, local


def _reduce(value: float, op) -> float:
    if not dist.is_initialized():
        return float(value)
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=op)
    return float(t.item())


def max_over_ranks(value: float) -> float:
    """Largest value over all ranks (the job time of a data-parallel step)."""
    return _reduce(value, dist.ReduceOp.MAX)


def sum_over_ranks(value: float) -> float:
    return _reduce(value, dist.ReduceOp.SUM)


def gather_objects(obj) -> list:
    """obj of every rank, in rank order (a one-element list without a process group)."""
    if not dist.is_initialized():
        return [obj]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


def barrier() -> None:
    if dist.is_initialized():
        dist.barrier()
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        torch.cuda.synchronize()
