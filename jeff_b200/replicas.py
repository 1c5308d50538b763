"""Request-sharded replicas on the GPUs of one box (one process per GPU).

Requests are independent (the reference's engine/batched_path.py:5-7), so each GPU holds the full int4 base, every
adapter and its own prefix pool, and serves its own share of the calls; nothing crosses GPUs on the per-call path.
What does cross them: once at load, rank 0's weights and adapter pool rows, broadcast (NCCL over NVLink on the GPU
box, gloo on the CPU for tests) into the other ranks' tensors of the same shapes, in one fixed order
(FastPath.tensors()); on each adapter add, that adapter's row only (FastPath.adapter_tensors(row)); on a remove,
nothing. Timing across ranks is the maximum over ranks.

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


def add_adapter_everywhere(fast, adapter, src: int = 0) -> int:
    """Add an adapter on every rank at once: each rank packs it into its lowest free row (the same row everywhere,
    since every rank adds and removes the same adapters in the same order), ranks other than `src` may pass a
    skeleton of the same shapes (synthetic.make_adapter(..., skeleton=True)), and `src`'s row is then broadcast
    into the others: the row's LoRA A and B of every group, its readout rows and temperature, and nothing else.
    Returns the row. Every rank must call this, in the same order."""
    import torch.distributed as dist

    # a rank whose own add fails still joins the gather, so no rank is left waiting in a collective
    try:
        index, failure = fast.add_adapter(adapter), None
    except Exception as error:  # noqa: BLE001 - reported to every rank below
        index, failure = None, f"{type(error).__name__}: {error}"
    outcomes: list = [None] * dist.get_world_size()
    dist.all_gather_object(outcomes, (index, failure))
    rows = [row for row, _ in outcomes]
    if len(set(rows)) != 1 or rows[0] is None:
        if index is not None:
            fast.remove_adapter(adapter.name)
        problems = "; ".join(f"rank {r}: {why}" for r, (_, why) in enumerate(outcomes) if why)
        raise RuntimeError(f"The ranks put adapter {adapter.name} in different rows {rows}"
                           f"{' (' + problems + ')' if problems else ''}; their adapter pools have drifted apart "
                           "(add and remove the same adapters on every rank, in the same order)")
    broadcast_tensors(fast.adapter_tensors(index), src)
    return index


def remove_adapter_everywhere(fast, name: str) -> None:
    """Remove an adapter on every rank (no data moves: the row is freed and its cached prefixes forgotten on each
    rank); every rank must call this, in the same order. A rank whose own removal fails still joins the exchange of
    outcomes, so no rank is left waiting in a collective; if any rank failed, every rank raises the same error."""
    size = _size()
    try:
        fast.remove_adapter(name)
        failure = None
    except Exception as error:  # noqa: BLE001 - reported to every rank below
        failure = f"{type(error).__name__}: {error}"
    if size == 1:
        if failure:
            raise RuntimeError(f"Removing adapter {name} failed: {failure}")
        return
    import torch.distributed as dist

    outcomes: list = [None] * size
    dist.all_gather_object(outcomes, failure)
    problems = "; ".join(f"rank {r}: {why}" for r, why in enumerate(outcomes) if why)
    if problems:
        raise RuntimeError(f"Removing adapter {name} failed on some ranks ({problems}); their adapter pools have "
                           "drifted apart (add and remove the same adapters on every rank, in the same order)")


def _size() -> int:
    import torch.distributed as dist

    return dist.get_world_size() if dist.is_initialized() else 1


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
