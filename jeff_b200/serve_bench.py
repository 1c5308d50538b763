"""Configuration 5 of the reference benchmark: request-sharded serving load on the configuration 4 model.

    python -m jeff_b200.serve_bench [--calls N] [--load 0.9] [--window-ms 1] [--max-batch-rows 64]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 -m jeff_b200.serve_bench --gpus N

The calls (seed 5): Poisson arrivals; one of 32 adapters per call, Zipf(1.1) over the adapters' ranks; one of 64
distinct 512-token bound-context prefixes, uniform; a new-token count from the lognormal of mean 96 and sigma 0.8
(mu = ln 96 - 0.32), rounded, at least 1 and at most 1024; token ids uniform over the vocabulary; 2 to 32 options.

Serving: each GPU is one replica holding the base, all 32 adapters and its own prefix pool. A call goes to replica
int(sha256(adapter + prefix)) mod N, the reference router's sticky rule (apps/server/src/jeff_server/router.py:
_binding_key and EngineRouter.predict), so one prefix's states live on one GPU. Each replica batches its calls with
the reference scheduler's rule (runtime/python/src/jeff_runtime/scheduler.py, Scheduler._gather): a micro-batch
closes `window_ms` after its oldest waiting call arrived, or as soon as `max_batch_rows` calls wait, and takes at
most `max_batch_rows` calls in arrival order; the batch goes to B200Engine.predict_many as one group per adapter,
which runs it as graph replays per new-token bucket in the configuration's batch buckets of 1, 8, 16, 32 and 64 rows. A call's latency is the time
from its arrival to the end of the engine call that answered it. The reference's defaults are window 1 ms, 64 rows
(docs/operating.md: --batch-window-ms 1 --max-batch-rows 64).

The run is open loop and single threaded per replica: arrival times are fixed in advance, and between engine calls
the loop admits every call whose arrival time has passed, so a slow engine call makes the queue grow exactly as it
would with independent clients. Each call is prepared (engine.prepare) before the clock starts, standing in for the
reference's preparation threads, which prepare each request on arrival beside the GPU thread. Before timing, every
(adapter, prefix) pair of the stream is made resident (its prefix pass run) and every decision graph recorded, so
the timed runs see a warm pool (prefix misses are still counted). The run measures capacity first (a saturation stream: every call waiting at time 0), then replays an
open-loop stream at `load` x capacity, and prints one JSON line: decisions/s, p50/p99 latency, batch sizes."""

from __future__ import annotations

import argparse
import hashlib
import json
import math
import time
import zlib
from collections import deque
from collections.abc import Callable, Sequence
from dataclasses import dataclass

import numpy as np

ADAPTERS, PREFIXES, PREFIX_TOKENS = 32, 64, 512
CFG5_BATCH_BUCKETS = (1, 8, 16, 32, 64)   # the configuration's CUDA-graph batch buckets
MEAN_NEW, SIGMA_NEW, MAX_NEW = 96.0, 0.8, 1024


@dataclass
class Calls:
    """A call stream: arrival times (s), adapter numbers (1..32), prefix numbers, new token ids, option counts."""
    arrival: np.ndarray
    adapter: np.ndarray
    prefix: np.ndarray
    new_ids: list[np.ndarray]
    count: np.ndarray

    def __len__(self) -> int:
        return len(self.arrival)

    def subset(self, index: Sequence[int]) -> Calls:
        idx = np.asarray(index, dtype=np.int64)
        return Calls(self.arrival[idx], self.adapter[idx], self.prefix[idx], [self.new_ids[i] for i in idx],
                     self.count[idx])

    def at(self, arrival: np.ndarray) -> Calls:
        return Calls(np.asarray(arrival, dtype=np.float64), self.adapter, self.prefix, self.new_ids, self.count)


def rng(seed: int, name: str) -> np.random.Generator:
    return np.random.default_rng((seed * 1_000_003 + zlib.crc32(name.encode())) % (2**63))


def zipf_weights(n: int, s: float) -> np.ndarray:
    w = np.arange(1, n + 1, dtype=np.float64) ** -s
    return w / w.sum()


def make_calls(n: int, rate: float, seed: int = 5, vocab: int = 151936) -> Calls:
    """`n` calls of configuration 5 arriving as a Poisson process of `rate` calls/s (rate inf: all at time 0)."""
    g = rng(seed, "cfg5/calls")
    arrival = np.zeros(n) if math.isinf(rate) else np.cumsum(g.exponential(1.0 / rate, n))
    adapter = g.choice(ADAPTERS, size=n, p=zipf_weights(ADAPTERS, 1.1)) + 1
    prefix = g.integers(0, PREFIXES, n)
    mu = math.log(MEAN_NEW) - SIGMA_NEW ** 2 / 2
    lengths = np.clip(np.rint(g.lognormal(mu, SIGMA_NEW, n)), 1, MAX_NEW).astype(np.int64)
    ids = g.integers(0, vocab, int(lengths.sum()))
    offsets = np.concatenate([[0], np.cumsum(lengths)])
    new_ids = [ids[offsets[i]:offsets[i + 1]] for i in range(n)]
    count = g.integers(2, 33, n)
    return Calls(arrival, adapter, prefix, new_ids, count)


def prefix_ids(seed: int = 5, vocab: int = 151936) -> dict[str, list[int]]:
    """The 64 prefixes' token ids by prefix text."""
    return {prefix_text(j): rng(seed, f"cfg5/prefix/{j}").integers(0, vocab, PREFIX_TOKENS).tolist()
            for j in range(PREFIXES)}


def prefix_text(j: int) -> str:
    return f"cfg5 bound context {j}"


def adapter_id(a: int) -> str:
    return f"adapter-{a}"


def replica_of(adapter: str, prefix: str, replicas: int) -> int:
    """The replica a call goes to: the reference router's sticky hash of its binding (adapter and prefix)."""
    return int(hashlib.sha256((adapter + prefix).encode()).hexdigest(), 16) % replicas


def route(adapters: Sequence[int], prefixes: Sequence[int], replicas: int) -> list[list[int]]:
    """Each replica's calls (positions into the given adapter and prefix numbers), in order."""
    shares: list[list[int]] = [[] for _ in range(replicas)]
    for i, (a, p) in enumerate(zip(adapters, prefixes, strict=True)):
        shares[replica_of(adapter_id(int(a)), prefix_text(int(p)), replicas)].append(i)
    return shares


def rows_of(calls: Calls, index: Sequence[int]) -> list[dict]:
    return [{"prefix_text": prefix_text(int(calls.prefix[i])), "new_ids": calls.new_ids[i].tolist(),
             "count": int(calls.count[i])} for i in index]


@dataclass
class Served:
    done: np.ndarray          # completion time of each call (s after the stream's time 0)
    batches: int
    batch_rows: list[int]
    elapsed: float            # time 0 to the last completion
    prefix_misses: int
    passes: int


def serve(engine, calls: Calls, window_ms: float = 1.0, max_batch_rows: int = 64,
          clock: Callable[[], float] = time.perf_counter, sleep: Callable[[float], None] = time.sleep,
          prepared: Sequence | None = None) -> Served:
    """Answer `calls` (arrival-ordered) on `engine` with the micro-batching rule of the module docstring.
    `prepared`: each call's engine.prepare() result, made beforehand, as the reference scheduler has its clients'
    threads prepare each request on arrival (Scheduler.submit) while the GPU thread runs; a batch then joins its
    calls' prepared rows per adapter (Prepared.join, as Scheduler._run does). Without it, rows are prepared on the
    serving loop, inside the measured time."""
    n = len(calls)
    done = np.full(n, np.nan)
    queue: deque[int] = deque()
    window = window_ms / 1000.0
    nxt = 0
    batches, misses, passes = 0, 0, 0
    batch_rows: list[int] = []
    t0 = clock()

    def admit(now: float) -> None:
        nonlocal nxt
        while nxt < n and calls.arrival[nxt] <= now:
            queue.append(nxt)
            nxt += 1

    while nxt < n or queue:
        now = clock() - t0
        admit(now)
        if not queue:
            sleep(max(0.0, float(calls.arrival[nxt]) - now))
            continue
        close = float(calls.arrival[queue[0]]) + window
        while len(queue) < max_batch_rows:
            now = clock() - t0
            admit(now)
            if len(queue) >= max_batch_rows or now >= close:
                break
            upcoming = float(calls.arrival[nxt]) if nxt < n else math.inf
            sleep(max(0.0, min(close, upcoming) - now))
        batch = [queue.popleft() for _ in range(min(max_batch_rows, len(queue)))]
        groups: dict[int, list[int]] = {}
        for i in batch:
            groups.setdefault(int(calls.adapter[i]), []).append(i)
        if prepared is not None:
            work = [(adapter_id(a), type(prepared[members[0]]).join([prepared[i] for i in members]))
                    for a, members in groups.items()]
        else:
            work = [(adapter_id(a), engine.prepare(adapter_id(a), rows_of(calls, members)))
                    for a, members in groups.items()]
        results = engine.predict_many(work)
        finished = clock() - t0
        for (a, members), result in zip(groups.items(), results, strict=True):
            if isinstance(result, Exception):
                raise RuntimeError(f"adapter-{a}: {result}") from result
            for i in members:
                done[i] = finished
        timing = results[0].timing if results else {}
        misses += int(timing.get("prefix_misses", 0))
        passes += int(timing.get("passes", 0))
        batches += 1
        batch_rows.append(len(batch))
    return Served(done, batches, batch_rows, float(np.nanmax(done)) if n else 0.0, misses, passes)


def latency_ms(calls: Calls, served: Served) -> np.ndarray:
    return (served.done - calls.arrival) * 1000.0


def percentile(values: np.ndarray, q: float) -> float:
    return float(np.percentile(values, q)) if len(values) else float("nan")


# ---------------------------------------------------------------- the B200 run


def build_engine(rank: int, world: int, pool_prefixes: int):
    """The configuration 4 base with 32 rank-16 adapters on this GPU (rank 0 builds, the others receive by
    broadcast), a prefix pool for `pool_prefixes` 512-token prefixes, prefix text tokenised from the 64 prefixes."""
    import torch

    from jeff_b200 import synthetic
    from jeff_b200.batched_path import BatchedPath
    from jeff_b200.engine import B200Engine
    from jeff_b200.fast_path import FastPath

    skeleton = rank != 0
    model = synthetic.make_model(synthetic.ModelSpec(), skeleton=skeleton)
    fast = FastPath(model, max_adapters=ADAPTERS, base_readout=synthetic.base_head(model) if not skeleton else None,
                    pool_pages_count=2 + pool_prefixes * (50 + PREFIX_TOKENS // 32) + 64)
    ids = prefix_ids()
    path = BatchedPath(fast, tokenize=lambda text: ids[text], batch_buckets=CFG5_BATCH_BUCKETS)
    engine = B200Engine(paths=(fast, path), max_adapters=ADAPTERS)
    for a in range(1, ADAPTERS + 1):
        engine.add_adapter(adapter_id(a), synthetic.make_adapter(model, a, seed=1000 + a, skeleton=skeleton))
    if world > 1:
        from jeff_b200 import replicas

        replicas.broadcast_tensors(fast.tensors(), 0)
        torch.cuda.synchronize()
    return engine


def warm(engine, pairs: Sequence[tuple[int, int]]) -> float:
    """Make every (adapter, prefix) pair resident and record every decision graph; seconds taken."""
    started = time.perf_counter()
    engine.batched.record()
    pairs = sorted(set(pairs))
    for start in range(0, len(pairs), 64):
        groups: dict[int, list[dict]] = {}
        for a, p in pairs[start:start + 64]:
            groups.setdefault(a, []).append({"prefix_text": prefix_text(p), "new_ids": [1, 2, 3], "count": 2})
        engine.predict_many([(adapter_id(a), engine.prepare(adapter_id(a), rows)) for a, rows in groups.items()])
    return time.perf_counter() - started


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--calls", type=int, default=100_000)
    ap.add_argument("--capacity-calls", type=int, default=20_000)
    ap.add_argument("--load", type=float, default=0.9)
    ap.add_argument("--window-ms", type=float, default=1.0)
    ap.add_argument("--max-batch-rows", type=int, default=64)
    args = ap.parse_args()

    import torch

    from jeff_b200 import _lib, replicas

    rank, world, _ = replicas.setup("nccl", timeout_s=300)
    _lib.load()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but the launcher started {world} ranks")
    saturation = make_calls(args.capacity_calls, math.inf)
    stream = make_calls(args.calls, 1.0)            # arrival times rescaled to the offered rate below
    adapters = np.concatenate([saturation.adapter, stream.adapter])
    prefixes = np.concatenate([saturation.prefix, stream.prefix])
    pairs = [(int(adapters[i]), int(prefixes[i])) for i in route(adapters, prefixes, world)[rank]]
    engine = build_engine(rank, world, pool_prefixes=len(set(pairs)) + 16)
    warm_s = warm(engine, pairs)
    torch.cuda.synchronize()

    def run(calls: Calls) -> tuple[Served, Calls, float]:
        mine = calls.subset(route(calls.adapter, calls.prefix, world)[rank])
        ready = [engine.prepare(adapter_id(int(mine.adapter[i])), rows_of(mine, [i])) for i in range(len(mine))]
        replicas.barrier(world)
        served = serve(engine, mine, args.window_ms, args.max_batch_rows, prepared=ready)
        return served, mine, replicas.max_over_ranks(served.elapsed, world)

    sat_served, sat_mine, sat_elapsed = run(saturation)
    capacity = len(saturation) / sat_elapsed
    rate = args.load * capacity
    stream = stream.at(stream.arrival / rate)       # exponential gaps scale with 1 / rate; the draws are the same
    served, mine, elapsed = run(stream)
    lat = latency_ms(mine, served)
    gathered = [lat]
    stats = [(served.batches, sum(served.batch_rows), served.prefix_misses, served.passes)]
    if world > 1:
        import torch.distributed as dist

        gathered = [None] * world
        dist.all_gather_object(gathered, lat)
        stats = [None] * world
        dist.all_gather_object(stats, (served.batches, sum(served.batch_rows), served.prefix_misses, served.passes))
    if rank == 0:
        lat_all = np.concatenate(gathered)
        batches = sum(s[0] for s in stats)
        print(json.dumps({
            "config": {"workload": "cfg5: request-sharded serving load on the cfg4 model (24 layers int4 g128z), "
                                   "Poisson arrivals, 32 rank-16 adapters Zipf(1.1), 64 distinct 512-token prefixes, "
                                   "new tokens lognormal mean 96 sigma 0.8 cap 1024, options 2..32",
                       "calls": args.calls, "window_ms": args.window_ms, "max_batch_rows": args.max_batch_rows,
                       "routing": "sha256(adapter + prefix) mod replicas"},
            "n_gpus": world, "data": "synthetic",
            "capacity_decisions_per_s": capacity, "capacity_calls": len(saturation),
            "load": args.load, "offered_calls_per_s": rate,
            "decisions_per_s": len(stream) / elapsed,
            "p50_ms": percentile(lat_all, 50), "p99_ms": percentile(lat_all, 99), "max_ms": float(lat_all.max()),
            "mean_batch_rows": sum(s[1] for s in stats) / max(batches, 1), "batches": batches,
            "passes": sum(s[3] for s in stats), "prefix_misses_timed": sum(s[2] for s in stats),
            "warm_s": warm_s}), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
