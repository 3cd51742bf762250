"""Multi-GPU plumbing for the early-exit path: one process per GPU, rows
sharded by rank with no exchange on the data path.

The path shards naturally (every row is independent given the router
weights), so the only collectives are host-side bookkeeping: the max of the
ranks' device times for a benchmark, and the sum of per-rank exit counts
when global ExitStats are wanted (the reference has no distributed code; its
statistics are the per-process ones of python/TIDE/scheduler.py:12-36).
Backend "nccl" on GPUs, "gloo" for CPU processes.
"""
from __future__ import annotations

import datetime
import os
from typing import Tuple

import torch

from tide_b200.scheduler import ExitStats


def world_from_env() -> Tuple[int, int, int]:
    """(world size, rank, local rank) from the torchrun environment."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend: str | None = None, timeout_s: float = 300.0) -> Tuple[int, int, int]:
    """Join the process group when WORLD_SIZE > 1 and pin this process's GPU
    (local rank) when CUDA is present.  Rendezvous comes from MASTER_ADDR /
    MASTER_PORT; a short timeout makes ranks that wait for a dead peer fail."""
    world, rank, local = world_from_env()
    cuda = torch.cuda.is_available()
    if cuda:
        torch.cuda.set_device(local if world > 1 else 0)
    if world > 1:
        import torch.distributed as dist

        backend = backend or ("nccl" if cuda else "gloo")
        kw = {"device_id": torch.device("cuda", local)} if backend == "nccl" else {}
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return world, rank, local


def _device() -> torch.device:
    import torch.distributed as dist

    return torch.device("cuda") if dist.get_backend() == "nccl" else torch.device("cpu")


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(world: int, v: float) -> float:
    """Max of a per-rank scalar (device times of a timed region)."""
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device=_device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_counts(world: int, counts: torch.Tensor) -> torch.Tensor:
    """Element-wise sum over ranks of an int tensor of counts (e.g. the
    {survivors, exits} words of every checkpoint); returns a new tensor on
    the input's device."""
    if world == 1:
        return counts.clone()
    import torch.distributed as dist

    t = counts.to(_device(), torch.int64).clone()
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.to(counts.device, counts.dtype)


def global_stats(world: int, stats: ExitStats, layers=None) -> ExitStats:
    """ExitStats summed over ranks (same fields, same summary text).  `layers`
    lists every checkpoint layer (the same list on every rank: a rank records
    only the layers where some of its tokens exited, so its own keys can
    differ from another rank's); without it every rank must pass stats with
    the same keys.  Layers with no exit on any rank are left out, as in a
    single process."""
    layers = sorted(layers) if layers is not None else sorted(stats.exits_per_layer)
    local = torch.tensor([stats.total_tokens, stats.remaining_tokens]
                         + [stats.exits_per_layer.get(k, 0) for k in layers], dtype=torch.int64)
    tot = sum_counts(world, local).tolist()
    return ExitStats(total_tokens=int(tot[0]), remaining_tokens=int(tot[1]),
                     exits_per_layer={k: int(v) for k, v in zip(layers, tot[2:]) if v})


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous, balanced [start, end) of n rows (or sequences) for a rank:
    sizes differ by at most one and the ranges tile [0, n) in rank order."""
    if world < 1 or not (0 <= rank < world) or n < 0:
        raise ValueError(f"bad shard request n={n} world={world} rank={rank}")
    return n * rank // world, n * (rank + 1) // world


def all_gather_rows(world: int, rows: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Every rank's rows stacked in rank order ([world * n, ...]): the end-of-
    step gather of the output rows (or of rank-local lm_head results).  With
    NCCL on NVLink/NVSwitch it runs as one ncclAllGather."""
    if world == 1:
        return rows if out is None else out.copy_(rows)
    import torch.distributed as dist

    if out is None:
        out = torch.empty((world * rows.shape[0],) + tuple(rows.shape[1:]), dtype=rows.dtype,
                          device=rows.device)
    dist.all_gather_into_tensor(out, rows.contiguous())
    return out


def all_gather_counts(world: int, counts: torch.Tensor) -> torch.Tensor:
    """Per-rank exit counts of every rank, [world, ...] in rank order."""
    return all_gather_rows(world, counts.reshape(1, *counts.shape)).reshape(world, *counts.shape)

