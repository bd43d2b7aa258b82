"""Process-group plumbing of the multi-GPU runs: one process per GPU, ranks from the launcher's environment
(torchrun's RANK / LOCAL_RANK / WORLD_SIZE), a short collective timeout so that a rank which dies or hangs ends the
others' next collective with an error instead of a hang, and the reductions of per-rank scalars the runs need (the
max over ranks of a device time, the sum of work). The data path itself shards with no collective."""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass


@dataclass(frozen=True)
class RankInfo:
    rank: int
    world: int
    local: int


def rank_info(env=None) -> RankInfo:
    """The launcher's rank layout, validated: 1 <= WORLD_SIZE, 0 <= RANK < WORLD_SIZE, 0 <= LOCAL_RANK <= RANK.
    Missing variables mean a single process. Raises ValueError naming the inconsistent variable."""
    env = os.environ if env is None else env

    def num(name, default):
        raw = env.get(name, str(default))
        try:
            return int(raw)
        except ValueError:
            raise ValueError(f"{name}={raw!r} is not an integer") from None

    world, rank, local = num("WORLD_SIZE", 1), num("RANK", 0), num("LOCAL_RANK", 0)
    if world < 1:
        raise ValueError(f"WORLD_SIZE={world} must be >= 1")
    if not 0 <= rank < world:
        raise ValueError(f"RANK={rank} must be in [0, WORLD_SIZE={world})")
    if not 0 <= local <= rank:
        raise ValueError(f"LOCAL_RANK={local} must be in [0, RANK={rank}]")
    return RankInfo(rank, world, local)


def init(info: RankInfo, backend: str = "nccl", timeout_s: float = 120.0, device=None) -> None:
    """Joins the process group when world > 1 (MASTER_ADDR / MASTER_PORT from the environment). `timeout_s` bounds
    every collective: a peer that is gone or stuck turns into an exception on the others."""
    if info.world == 1:
        return
    import torch.distributed as dist

    kw = {"device_id": device} if device is not None and backend == "nccl" else {}
    dist.init_process_group(backend, rank=info.rank, world_size=info.world,
                            timeout=datetime.timedelta(seconds=timeout_s), **kw)


def _reduce(x: float, op: str, device) -> float:
    import torch
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def max_over_ranks(x: float, device=None) -> float:
    """Max of a per-rank scalar (a device time) over all ranks; the value itself with one process."""
    return _reduce(x, "max", device)


def sum_over_ranks(x: float, device=None) -> float:
    """Sum of a per-rank scalar (work done) over all ranks; the value itself with one process."""
    return _reduce(x, "sum", device)


def barrier() -> None:
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


def shutdown() -> None:
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
