"""The multi-GPU host logic on the CPU: two gloo ranks (world size 2, 127.0.0.1) run what bench.py's replicas run
over NCCL, the layout check and broadcast of rank 0's weights and adapters into rank 1's skeleton tensors, the
max-over-ranks of a time, and the per-rank share of independent calls; plus the refusal when the ranks' tensor
layouts differ (both ranks raise; none waits)."""

from __future__ import annotations

import dataclasses
import os
import socket
import sys
import traceback
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


# host-only fields the device never receives (the oracle's dequantised copies and per-matrix adapter views)
HOST_ONLY = {"W", "matrices"}


def host_tensors(obj) -> list[torch.Tensor]:
    """Every tensor of a synthetic model or adapter that FastPath uploads, in a fixed order (dataclass fields in
    order, dicts by key)."""
    out: list[torch.Tensor] = []

    def walk(x) -> None:
        if isinstance(x, torch.Tensor):
            out.append(x)
        elif dataclasses.is_dataclass(x) and not isinstance(x, type):
            for f in dataclasses.fields(x):
                if f.name not in HOST_ONLY:
                    walk(getattr(x, f.name))
        elif isinstance(x, dict):
            for key in sorted(x, key=str):
                walk(x[key])
        elif isinstance(x, (list, tuple)):
            for item in x:
                walk(item)

    walk(obj)
    return out


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, port: int, mode: str, errors) -> None:
    try:
        sys.path.insert(0, str(ROOT))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                          LOCAL_RANK=str(rank))
        from jeff_b200 import replicas, synthetic

        r, size, _ = replicas.setup("gloo", timeout_s=60)
        assert (r, size) == (rank, 2)
        spec = synthetic.ModelSpec(layers=4, vocab=512, seed=7)
        skeleton = rank != 0
        model = synthetic.make_model(spec, skeleton=skeleton)
        adapters = [synthetic.make_adapter(model, i, seed=50 + i, skeleton=skeleton) for i in (1, 2)]
        tensors = host_tensors(model) + [t for ad in adapters for t in host_tensors(ad)]
        if mode == "mismatch" and rank == 1:
            tensors = tensors[:-1]
        try:
            replicas.broadcast_tensors(tensors, 0)
        except RuntimeError as error:
            if mode == "mismatch" and "different tensor layout" in str(error):
                replicas.barrier(size)
                import torch.distributed as dist

                dist.destroy_process_group()
                return
            raise
        assert mode == "ok", "a mismatched layout was not refused"
        want_model = synthetic.make_model(spec)
        want = host_tensors(want_model) + [t for i in (1, 2)
                                           for t in host_tensors(synthetic.make_adapter(want_model, i, seed=50 + i))]
        assert len(want) == len(tensors)
        for a, b in zip(tensors, want, strict=True):
            assert torch.equal(a, b)
        slowest = replicas.max_over_ranks(1.0 + rank, size, device="cpu")
        assert slowest == 2.0
        calls = list(range(10))
        mine = replicas.share(calls, rank, size)
        gathered: list = [None, None]
        import torch.distributed as dist

        dist.all_gather_object(gathered, mine)
        assert sorted(gathered[0] + gathered[1]) == calls and not set(gathered[0]) & set(gathered[1])
        replicas.barrier(size)
        dist.destroy_process_group()
    except BaseException:
        errors.put(f"rank {rank}: {traceback.format_exc()}")
        raise


@pytest.mark.parametrize("mode", ["ok", "mismatch"])
def test_two_gloo_ranks_broadcast_weights_and_reduce_times(mode: str) -> None:
    ctx = mp.get_context("spawn")
    errors = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, mode, errors)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    messages = []
    while not errors.empty():
        messages.append(errors.get())
    assert not messages, "\n".join(messages)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
