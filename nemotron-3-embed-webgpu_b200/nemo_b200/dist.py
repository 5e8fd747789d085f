"""Rank plumbing for request-sharded runs (one process per GPU).

The encoder shards by request: every rank holds a full weight replica and runs
its own micro-batches, so the data path has no collective. The only
collectives are the timing barrier and the max-over-ranks reduction of the
measured time; both go through torch.distributed (NCCL on GPUs, gloo on CPU
for tests). These helpers keep that logic in one place.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta


@dataclass
class RankInfo:
    rank: int
    world: int
    local_rank: int


def rank_info() -> RankInfo:
    """RANK / WORLD_SIZE / LOCAL_RANK from the launcher's environment (1 rank if unset)."""
    return RankInfo(int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
                    int(os.environ.get("LOCAL_RANK", "0")))


def init(backend: str, timeout_s: float = 300.0, device=None) -> RankInfo:
    """Initialises the process group when WORLD_SIZE > 1 (short timeout: ranks that wait on a dead peer error out)."""
    info = rank_info()
    if info.world > 1:
        import torch.distributed as dist
        kw = {"timeout": timedelta(seconds=timeout_s)}
        if device is not None:
            kw["device_id"] = device
        dist.init_process_group(backend, **kw)
    return info


_CPU_GROUP = None


def cpu_barrier(info: RankInfo) -> None:
    """A barrier that puts no work on any GPU (gloo over the host). Ranks wait
    here while one rank uses every GPU of the box (head-parallel runs), so no
    other process has a collective kernel in flight on those GPUs."""
    global _CPU_GROUP
    if info.world == 1:
        return
    import torch.distributed as dist
    if _CPU_GROUP is None:
        _CPU_GROUP = dist.new_group(backend="gloo")
    dist.barrier(group=_CPU_GROUP)


def barrier(info: RankInfo) -> None:
    if info.world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(info: RankInfo, value: float, device: str = "cpu") -> float:
    """The largest of the ranks' values (device timing rule: max over ranks)."""
    if info.world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def throughput(world: int, steps: int, requests_per_step: int, seconds: float) -> float:
    """Whole-job requests/s: every rank ran `steps` steps of `requests_per_step` requests in at most `seconds`."""
    return world * steps * requests_per_step / seconds


def shard_requests(lengths: list[int], world: int) -> list[list[int]]:
    """Longest-first onto the rank with the fewest tokens (the C ABI's multi-device split, model.ts batches)."""
    order = sorted(range(len(lengths)), key=lambda i: -lengths[i])
    load = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: load[j])
        out[r].append(i)
        load[r] += lengths[i]
    return out


def shutdown(info: RankInfo) -> None:
    if info.world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
