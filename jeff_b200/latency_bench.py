"""Decision latency and pass throughput of the batched path, in the reference's own measurement shapes.

    python -m jeff_b200.latency_bench [--reps N]

The reference publishes two series for its batched decision path (results/step2b1/batch1_final.json and
throughput.json, summarised in docs/operating.md:240-244), measured on its own GPU with a bfloat16 base:
- batch-1 latency: one row over a 1,000-token cached prefix, N = 32 / 64 / 128 / 256 new tokens, 32 options, an
  adapter among 9 loaded; p50 wall time of a decide() call;
- throughput: rows per second for passes of B = 1 / 4 / 16 / 64 rows at N = 32 / 64 / 128.
This module measures the same shapes on this B200 build (configuration 4's int4 g128 + zero base, random-init
weights, 9 rank-16 adapters, one 1,000-token prefix per adapter made resident by the prefix pass first). Each timed
call goes through BatchedPath.decide: pinned host input, host-to-device copy, the recorded graph, the probabilities
back to the host. One JSON line per measurement."""

from __future__ import annotations

import argparse
import json
import statistics
import time

import torch

from jeff_b200 import synthetic
from jeff_b200.batched_path import BatchedPath, Row
from jeff_b200.fast_path import FastPath

ADAPTERS = 9
PREFIX_TOKENS = 1000
OPTIONS = 32


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=50)
    ap.add_argument("--profile", action="store_true",
                    help="run one batch-1 decision (N = 32) inside cudaProfilerStart/Stop (for ncu "
                         "--profile-from-start off) and exit")
    args = ap.parse_args()
    torch.cuda.set_device(0)
    model = synthetic.make_model(synthetic.ModelSpec())
    fast = FastPath(model, max_adapters=ADAPTERS, base_readout=synthetic.base_head(model),
                    pool_pages_count=2 + ADAPTERS * (50 + (PREFIX_TOKENS + 31) // 32) + 64)
    rows_of = [fast.add_adapter(synthetic.make_adapter(model, a, seed=1000 + a)) for a in range(1, ADAPTERS + 1)]
    g = torch.Generator().manual_seed(11)
    texts = {f"prefix {a}": torch.randint(0, 151936, (PREFIX_TOKENS,), generator=g).tolist() for a in range(ADAPTERS)}
    path = BatchedPath(fast, tokenize=lambda t: texts[t])
    shapes = [(1, 32), (1, 64), (1, 128), (1, 256)] + [(b, n) for n in (32, 64, 128) for b in (4, 16, 64)]
    path.record(shapes[:1] if args.profile else shapes)
    slots, _ = path.ensure_prefixes([(rows_of[a], f"prefix {a}") for a in range(ADAPTERS)], max_tokens=8192)

    def rows(b: int, n: int, seed: int) -> list[tuple[int, int, Row]]:
        gg = torch.Generator().manual_seed(seed)
        return [(rows_of[i % ADAPTERS], slots[i % ADAPTERS],
                 Row(f"prefix {i % ADAPTERS}", torch.randint(0, 151936, (n,), generator=gg).tolist(), OPTIONS))
                for i in range(b)]

    try:
        if args.profile:
            call = rows(1, 32, 1)
            for _ in range(3):
                path.decide(call)
            torch.cuda.synchronize()
            torch.cuda.profiler.start()
            path.decide(call)
            torch.cuda.synchronize()
            torch.cuda.profiler.stop()
            return
        for n in (32, 64, 128, 256):
            calls = [rows(1, n, 100 * n + r) for r in range(args.reps + 5)]
            for c in calls[:5]:
                path.decide(c)
            torch.cuda.synchronize()
            wall = []
            for c in calls[5:]:
                t0 = time.perf_counter()
                path.decide(c)
                wall.append((time.perf_counter() - t0) * 1e3)
            wall.sort()
            print(json.dumps({"measure": "batch-1 decision latency", "new_tokens": n, "prefix_tokens": PREFIX_TOKENS,
                              "options": OPTIONS, "adapters_loaded": ADAPTERS, "calls": len(wall),
                              "p50_ms": statistics.median(wall), "p90_ms": wall[int(0.9 * (len(wall) - 1))],
                              "min_ms": wall[0], "reference_p50_ms_rtx_pro_6000": {32: 2.41, 64: 2.70, 128: 3.01,
                                                                                    256: 3.89}[n]}), flush=True)
        reference = {32: {1: 414, 4: 1376, 16: 2600, 64: 3199}, 64: {1: 372, 4: 1033, 16: 1571, 64: 1851},
                     128: {1: 336, 4: 681, 16: 874, 64: 931}}
        for n in (32, 64, 128):
            for b in (1, 4, 16, 64):
                calls = [rows(b, n, 7 * b + n + r) for r in range(max(4, args.reps // 5) + 3)]
                for c in calls[:3]:
                    path.decide(c)
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                for c in calls[3:]:
                    path.decide(c)
                secs = time.perf_counter() - t0
                print(json.dumps({"measure": "pass throughput", "rows_per_pass": b, "new_tokens": n,
                                  "prefix_tokens": PREFIX_TOKENS, "rows_per_s": b * (len(calls) - 3) / secs,
                                  "reference_rows_per_s_rtx_pro_6000": reference[n][b]}), flush=True)
    finally:
        path.pool.unpin(slots)


if __name__ == "__main__":
    main()
