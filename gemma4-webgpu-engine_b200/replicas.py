"""One model replica per GPU: the request streams of a box split across independent processes.

The model (about 2.1 GB of weights with the per-layer-embedding table, about 0.9 GB streamed per
decode step) does not shard profitably, so a box runs one full replica per GPU and partitions
the sequences; nothing crosses between GPUs on the data path. The only cross-process steps are
host aggregation around a measurement: a barrier before timing, the slowest rank's time (max),
and the summed token count. These run on whatever process group the caller made (NCCL on the
GPU box, gloo in the CPU tests).
"""
from __future__ import annotations

import datetime


def replica_slice(n_items: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous share [start, stop) of n_items for `rank` of `world`: sizes differ by at most
    one, earlier ranks take the larger shares, and the shares tile 0..n_items exactly."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n_items < 0:
        raise ValueError("negative item count")
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def aggregate(torch, seconds: float, tokens: float, device=None) -> tuple[float, float]:
    """(max seconds over ranks, total tokens over ranks). Single process: the inputs back."""
    dist = torch.distributed
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return seconds, tokens
    t = torch.tensor([seconds], dtype=torch.float64, device=device)
    n = torch.tensor([tokens], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.all_reduce(n, op=dist.ReduceOp.SUM)
    return float(t.item()), float(n.item())


def init_group(torch, backend: str, timeout_s: float = 60.0, device=None) -> None:
    """Join the process group of a torchrun launch with a short timeout, so that a rank that
    never arrives ends the others' next collective with an error instead of a hang."""
    kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device is not None:
        kw["device_id"] = device
    torch.distributed.init_process_group(backend, **kw)
