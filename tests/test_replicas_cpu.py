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


class RowPools:
    """FastPath's adapter rows on the CPU (FastPath itself needs the GPU): lowest-free-row placement as
    FastPath.add_adapter does it, and FastPath.adapter_tensors' row views over pools of the same kinds."""

    def __init__(self, max_adapters: int = 3) -> None:
        import bisect  # noqa: F401

        rows = max_adapters + 1
        self.max_adapters = max_adapters
        self.readout_pool = torch.zeros(rows, 8, 32, dtype=torch.bfloat16)
        self.temp_pool = torch.ones(rows)
        self.lins = [SimpleLin(rows, 16, 32, 64), SimpleLin(rows, 0, 32, 64), SimpleLin(rows, 32, 64, 32)]
        self.free_rows = list(range(1, rows))
        self.adapter_index: dict[str, int] = {}

    def add_adapter(self, adapter) -> int:
        index = self.free_rows.pop(0)
        for lin, (a, b) in zip((x for x in self.lins if x.rank), adapter.lora, strict=True):
            lin.lora_a[index].copy_(a)
            lin.lora_b[index].copy_(b)
        self.readout_pool[index].copy_(adapter.readout)
        self.temp_pool[index] = adapter.temperature
        self.adapter_index[adapter.name] = index
        return index

    def remove_adapter(self, name: str) -> None:
        import bisect

        bisect.insort(self.free_rows, self.adapter_index.pop(name))

    def adapter_tensors(self, index: int) -> list[torch.Tensor]:
        from jeff_b200.fast_path import FastPath

        return FastPath.adapter_tensors(self, index)   # the real method over these pools


class SimpleLin:
    def __init__(self, rows: int, rank: int, k: int, columns: int) -> None:
        self.rank = rank
        self.lora_a = torch.zeros(rows, rank, k, dtype=torch.bfloat16) if rank else None
        self.lora_b = torch.zeros(rows, columns, rank, dtype=torch.bfloat16) if rank else None


def small_adapter(name: str, seed: int, skeleton: bool):
    from types import SimpleNamespace

    g = torch.Generator().manual_seed(seed)

    def draw(*shape):
        return torch.zeros(*shape, dtype=torch.bfloat16) if skeleton else torch.randn(*shape, generator=g).to(
            torch.bfloat16)

    return SimpleNamespace(name=name, lora=[(draw(16, 32), draw(64, 16)), (draw(32, 64), draw(32, 32))],
                           readout=draw(8, 32), temperature=1.0 if skeleton else 0.5 + seed / 10)


def _adapter_rank_main(rank: int, port: int, errors) -> None:
    try:
        sys.path.insert(0, str(ROOT))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                          LOCAL_RANK=str(rank))
        import torch.distributed as dist

        from jeff_b200 import replicas

        replicas.setup("gloo", timeout_s=60)
        pools = RowPools()
        skeleton = rank != 0
        assert replicas.add_adapter_everywhere(pools, small_adapter("a", 1, skeleton)) == 1
        assert replicas.add_adapter_everywhere(pools, small_adapter("b", 2, skeleton)) == 2
        replicas.remove_adapter_everywhere(pools, "a")
        assert replicas.add_adapter_everywhere(pools, small_adapter("c", 3, skeleton)) == 1
        want = RowPools()
        want.add_adapter(small_adapter("c", 3, False))
        want.add_adapter(small_adapter("b", 2, False))
        for row in (1, 2):
            for got, exp in zip(pools.adapter_tensors(row), want.adapter_tensors(row), strict=True):
                assert torch.equal(got, exp), f"rank {rank} row {row}"
        # pools that drifted apart (rank 1 holds an extra adapter) are refused on both ranks
        if rank == 1:
            pools.add_adapter(small_adapter("local", 9, False))
        try:
            replicas.add_adapter_everywhere(pools, small_adapter("d", 4, skeleton))
            raise AssertionError("drifted pools were not refused")
        except RuntimeError as error:
            assert "different rows" in str(error)
        assert "d" not in pools.adapter_index
        # a removal that fails on one rank (rank 0 never loaded "local") raises on both, and neither is left waiting
        try:
            replicas.remove_adapter_everywhere(pools, "local")
            raise AssertionError("a removal that failed on rank 0 was not reported")
        except RuntimeError as error:
            assert "rank 0" in str(error) and "Removing adapter local" in str(error)
        replicas.barrier(2)
        dist.destroy_process_group()
    except BaseException:
        errors.put(f"rank {rank}: {traceback.format_exc()}")
        raise


def test_two_gloo_ranks_add_and_remove_adapters_by_row() -> None:
    ctx = mp.get_context("spawn")
    errors = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_adapter_rank_main, args=(r, port, errors)) for r in range(2)]
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
    assert all(p.exitcode == 0 for p in procs)
