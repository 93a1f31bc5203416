"""Data-parallel replicas for independent requests (one process per GPU, no data-path
collective).

π0.5 requests are independent: each GPU holds a full copy of the weights and serves its own
share of the requests; the only cross-process traffic is the timing barrier and the max of the
per-rank device times used to report whole-job throughput.
"""

from __future__ import annotations

from typing import List, Sequence


def shard_requests(n_requests: int, world: int, rank: int) -> List[int]:
    """Request indices served by `rank`: contiguous blocks, the first n % world ranks one longer,
    so the shards are disjoint, cover every request and differ in size by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if n_requests < 0:
        raise ValueError("negative request count")
    base, extra = divmod(n_requests, world)
    start = rank * base + min(rank, extra)
    return list(range(start, start + base + (1 if rank < extra else 0)))


def whole_job_throughput(local_ms: float, units: int, group=None) -> tuple:
    """(units per second over all ranks, max elapsed ms over ranks).

    `local_ms` is this rank's device time for its `units` (requests, chunks); the job ends when
    the slowest rank ends, so throughput = Σ units / max ms. With no process group (or one rank)
    the local values are returned."""
    import torch
    import torch.distributed as dist

    if group is None and not (dist.is_available() and dist.is_initialized()):
        return units / (local_ms / 1e3), float(local_ms)
    dev = torch.device("cpu")
    if dist.get_backend(group) == "nccl":
        dev = torch.device("cuda", torch.cuda.current_device())
    t = torch.tensor([float(local_ms), float(units)], dtype=torch.float64, device=dev)
    mx = t[:1].clone()
    dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
    tot = t[1:].clone()
    dist.all_reduce(tot, op=dist.ReduceOp.SUM, group=group)
    ms = float(mx.item())
    return float(tot.item()) / (ms / 1e3), ms


def gather_actions(local: Sequence, world: int, group=None) -> list:
    """All ranks' per-request results, in request order (rank-major, matching shard_requests)."""
    import torch.distributed as dist

    if world == 1:
        return list(local)
    out = [None] * world
    dist.all_gather_object(out, list(local), group=group)
    return [x for part in out for x in part]
