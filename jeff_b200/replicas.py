"""Request-sharded replicas on the GPUs of one box (one process per GPU).

Requests are independent (the reference's engine/batched_path.py:5-7), so each GPU holds the full int4 base, every
adapter and its own prefix pool, and serves its own share of the calls; nothing crosses GPUs on the per-call path.
What does cross them, once at load and again on every adapter add or remove: rank 0's weights and adapter pool
rows, broadcast (NCCL over NVLink on the GPU box, gloo on the CPU for tests) into the other ranks' tensors of the
same shapes, in one fixed order (FastPath.tensors()). Timing across ranks is the maximum over ranks.

The process group is given a short timeout, so ranks that wait on a rank that died end with an error instead of
waiting for good."""

from __future__ import annotations

import datetime
import os
from collections.abc import Sequence

import torch


def world() -> tuple[int, int, int]:
    """(rank, world size, local rank) from the launcher's environment (1 process when unset)."""
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK",
                                                                                                           "0"))


def setup(backend: str = "nccl", timeout_s: float = 600.0) -> tuple[int, int, int]:
    """Join the process group when the world has more than one rank (NCCL: bind this rank's GPU first)."""
    rank, size, local = world()
    if size > 1:
        import torch.distributed as dist

        if backend == "nccl":
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
    elif backend == "nccl" and torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, size, local


def check_same_layout(tensors: Sequence[torch.Tensor]) -> None:
    """Every rank holds tensors of the same count, shapes and dtypes (a broadcast into a mismatched tensor would
    read or write the wrong bytes): compared through an all-gather of a small layout digest."""
    import torch.distributed as dist

    layout = [(tuple(t.shape), str(t.dtype)) for t in tensors]
    gathered: list = [None] * dist.get_world_size()
    dist.all_gather_object(gathered, layout)
    for r, other in enumerate(gathered):
        if other != layout:
            raise RuntimeError(f"Rank {r} holds a different tensor layout than rank {dist.get_rank()}: "
                               f"{len(other)} tensors against {len(layout)}")


def broadcast_tensors(tensors: Sequence[torch.Tensor], src: int = 0) -> None:
    """Copy rank `src`'s tensors into every rank's tensors of the same layout, in order."""
    import torch.distributed as dist

    check_same_layout(tensors)
    for t in tensors:
        dist.broadcast(t, src)


def barrier(size: int) -> None:
    if size > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, size: int, device: str | torch.device = "cuda") -> float:
    """The largest of every rank's value (a time: the job's time is its slowest rank's)."""
    if size == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def share(items: Sequence, rank: int, size: int) -> list:
    """This rank's share of a list of independent calls: every size-th item from position rank (calls keep their
    order within a rank; the union over ranks is the whole list, with no item on two ranks)."""
    return list(items[rank::size])
