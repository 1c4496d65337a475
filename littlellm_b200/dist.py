"""Multi-GPU plumbing for the layer-op chain: one process per GPU.

The path shards by whole sequences with no exchange; torch.distributed
(NCCL on GPUs, gloo for the CPU tests) is used only for barriers, the
max-over-ranks timing and gathering outputs to rank 0 for verification.
"""
from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist


def env() -> tuple[int, int, int]:
    """(world, rank, local_rank) from the torchrun environment."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend: str, device: torch.device | None = None, timeout_s: float = 300.0) -> None:
    kwargs = {"timeout": timedelta(seconds=timeout_s)}
    if device is not None and backend == "nccl":
        kwargs["device_id"] = device
    dist.init_process_group(backend, **kwargs)


def shard_range(n_items: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of this rank's even share of n_items (items = sequences)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if n_items % world != 0:
        raise ValueError(f"{n_items} sequences do not split evenly over {world} ranks")
    per = n_items // world
    return rank * per, (rank + 1) * per


def max_over_ranks(value: float, device: torch.device | None = None) -> float:
    """Max of a float over all ranks (identity without a process group)."""
    if not (dist.is_available() and dist.is_initialized()):
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_rows(local: torch.Tensor) -> torch.Tensor | None:
    """Concatenates every rank's equally-shaped `local` rows, in rank order,
    on rank 0 (all_gather, so every rank takes the same collective steps);
    other ranks get None."""
    if not (dist.is_available() and dist.is_initialized()):
        return local
    parts = [torch.empty_like(local) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, local.contiguous())
    return torch.cat(parts, dim=0) if dist.get_rank() == 0 else None


def or_over_ranks(value: int, device: torch.device | None = None) -> int:
    """Bitwise OR of an int over all ranks (error flags)."""
    if not (dist.is_available() and dist.is_initialized()):
        return value
    bits = torch.tensor([(value >> b) & 1 for b in range(8)], dtype=torch.int32, device=device)
    dist.all_reduce(bits, op=dist.ReduceOp.MAX)
    return int(sum(int(v) << b for b, v in enumerate(bits.tolist())))
