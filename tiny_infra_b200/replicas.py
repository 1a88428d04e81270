"""Multi-GPU serving as independent replicas: one process per GPU, each with its own engine and
KV pool, no collective on the data path (a 0.5B model fits one GPU; the reference has no
multi-GPU path at all).  The host-side pieces:

* ``partition(n, world, rank)`` -- round-robin request assignment (request i goes to rank
  i % world);
* ``serve_partition(batcher, requests, world, rank)`` -- run this rank's share through its
  continuous batcher concurrently and return {request index: tokens};
* ``max_over_ranks`` / ``gather_to_rank0`` -- the two cross-rank steps a job needs around the
  data path: the job's time is the slowest rank's (all_reduce MAX), and results are collected
  on rank 0.  Both work with the nccl (GPU) and gloo (CPU) backends of torch.distributed.
"""
from __future__ import annotations

import asyncio

import torch
import torch.distributed as dist


def partition(n_items: int, world: int, rank: int) -> list[int]:
    """Indices of the items rank ``rank`` of ``world`` serves (round robin)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    return list(range(rank, n_items, world))


async def serve_partition(batcher, requests, world: int, rank: int, **gen_kw) -> dict:
    """``requests``: list of (prompt_tokens, max_new_tokens) for the whole job; this rank serves
    its round-robin share through ``batcher`` (whose ``run_loop`` must be running)."""
    mine = partition(len(requests), world, rank)
    outs = await asyncio.gather(*[batcher.generate(list(requests[i][0]), requests[i][1], **gen_kw)
                                  for i in mine])
    return dict(zip(mine, outs))


def _initialized() -> bool:
    return dist.is_available() and dist.is_initialized()


def max_over_ranks(value: float, device: torch.device | None = None) -> float:
    """The maximum of ``value`` over all ranks (the value itself without a process group)."""
    if not _initialized() or dist.get_world_size() == 1:
        return float(value)
    if device is None:
        device = torch.device("cpu") if dist.get_backend() == "gloo" else torch.device(
            "cuda", torch.cuda.current_device())
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_to_rank0(obj):
    """Every rank's ``obj`` in a list on rank 0 (None elsewhere)."""
    if not _initialized() or dist.get_world_size() == 1:
        return [obj]
    world = dist.get_world_size()
    out = [None] * world if dist.get_rank() == 0 else None
    dist.gather_object(obj, out, dst=0)
    return out
