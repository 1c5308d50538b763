"""Benchmark of the B200 decision hot path, one JSON line on rank 0.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Workload ("step"): one batched decision pass of 64 calls x 128 new tokens on the int4 (group 128, bf16 scale and
zero) 24-layer hybrid base, each call on its adapter's shared 512-token prefix served from the paged prefix pool, 16
rank-16 adapters, option counts 2..32 (synthetic seeded data; no checkpoint or tokenizer exists offline).

- value: decisions/s with the packed inputs already in HBM (graph replays, CUDA events, W warm-up steps); the
  weights (264 MB) exceed the 126 MB L2, so every pass streams them from HBM.
- e2e: the same through BatchedPath.decide's pass (pinned host buffer -> H2D -> graph replay -> D2H probabilities).
- roofline: the dominant kernel, the tcgen05 W4A16 + LoRA product: its algorithmic FLOPs per launch over its
  average launch time, measured live by replaying a graph of the pass's 96 products with CUDA events.
- cpu_baseline: the reference's CPU standard path (the oracle restatement of DecisionModel.forward in float32, full
  prompt recomputed, as LocalEngine(backend="torch") runs it) on a bounded sample of calls.
- Multi-GPU: request-sharded replicas; rank 0 builds the weights and adapters and broadcasts them over NCCL at load;
  each rank runs its own 64 calls; no collective on the timed path except the barrier and the max-of-times reduce.

--impl reference: the reference's own CPU implementation of the path (the oracle port; the reference is Python
and cannot travel to the GPU box) on all host cores, one call per step, rank 0 only."""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

MEASURED_PEAKS = ROOT / "MEASURED_PEAKS.json"
METRIC = "decisions/sec (64x128-tok calls, int4+multi-LoRA)"
CALLS, NEW, PREFIX, ADAPTERS = 64, 128, 512, 16


def peaks() -> dict:
    if MEASURED_PEAKS.exists():
        d = json.loads(MEASURED_PEAKS.read_text())
        return {"hbm": d["hbm_gbs"], "bf16": d["bf16_tflops"], "bf16_sustained": d.get("bf16_tflops_sustained"),
                "source": "measured"}
    return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


class Clocks:
    """SM clock and throttle reasons sampled while the timed regions run: NVML every 20 ms (read-only queries), or
    nvidia-smi when NVML is not available."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, index: int) -> None:
        self.index = index
        self.samples: list[tuple[float, float, str]] = []
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._nvml = None
        try:
            import pynvml

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(index).uuid)
            handle = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            self._nvml = (pynvml, handle)
        except Exception:
            self._nvml = None

    def _sample_nvml(self) -> None:
        nv, h = self._nvml
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        active = [n for n, b in self.REASONS.items() if bits & b]
        self.samples.append((float(sm), float(mx), ",".join(active)))

    def _sample_smi(self) -> None:
        q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}", "--format=csv,noheader,nounits"],
                             capture_output=True, text=True, timeout=5)
        parts = [p.strip() for p in out.stdout.strip().split(",")]
        if len(parts) == 6:
            active = [n for n, v in zip(self.REASONS, parts[2:]) if v.lower() == "active"]
            self.samples.append((float(parts[0]), float(parts[1]), ",".join(active)))

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                self._sample_nvml() if self._nvml is not None else self._sample_smi()
            except Exception:
                if self._nvml is not None:
                    self._nvml = None
            self._stop.wait(0.02 if self._nvml is not None else 0.2)

    def __enter__(self) -> "Clocks":
        self._thread.start()
        return self

    def __exit__(self, *exc) -> None:
        self._stop.set()
        self._thread.join(timeout=10)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        reasons = sorted({r for _, _, a in self.samples for r in a.split(",") if r})
        return {"sm_mhz": statistics.median(s for s, _, _ in self.samples),
                "sm_max_mhz": max(m for _, m, _ in self.samples), "reasons": reasons, "samples": len(self.samples)}


def dist_setup(gpus: int) -> tuple[int, int, int]:
    from jeff_b200 import replicas

    return replicas.setup("nccl", timeout_s=600)


def barrier(world: int) -> None:
    from jeff_b200 import replicas

    replicas.barrier(world)


def max_over_ranks(value: float, world: int) -> float:
    from jeff_b200 import replicas

    return replicas.max_over_ranks(value, world, device="cuda")


# ---------------------------------------------------------------- the CPU baseline (oracle port of the standard path)


CPU_CHUNK = 8   # rows per forward of the reference's standard path (local_engine.py:641-661)


def cpu_chunk(rows) -> list[int]:
    """The calls of one CPU step: one adapter group of the pass, as the reference's standard path runs them (one
    adapter's rows at a time, local_engine.py:531-551, in forwards of at most CPU_CHUNK rows): the first group of the
    pass's mean group size (4 calls for 64 calls over 16 adapters), so that a step is a typical forward."""
    groups: dict[int, list[int]] = {}
    for i, a in enumerate(rows.adapters):
        groups.setdefault(a, []).append(i)
    mean = round(len(rows.adapters) / len(groups))
    pick = next((g for g in groups.values() if len(g) == mean), next(iter(groups.values())))
    return pick[:CPU_CHUNK]


def cpu_sample(model, adapters, rows, picks: list[int], threads: int) -> tuple[float, int]:
    """Seconds for one forward of the calls `picks` through the reference's standard path restated on the CPU
    (float32, each call's whole prompt, prefix + new tokens, recomputed: no prefix cache), as one chunk, and the
    thread count used."""
    from oracle import model_ref

    torch.set_num_threads(threads)
    gdn = sum(k == "linear_attention" for k in model.kinds)
    attn = len(model.kinds) - gdn
    batch = [model_ref.RowIn(rows.prefixes[i] + rows.new_ids[i], adapters[rows.adapters[i] - 1].lora,
                             adapters[rows.adapters[i] - 1].readout, adapters[rows.adapters[i] - 1].temperature,
                             rows.counts[i], model_ref.PrefixState.empty(gdn, attn)) for i in picks]
    started = time.perf_counter()
    with torch.inference_mode():
        model_ref.run_pass(model, batch, exact=True)
    return time.perf_counter() - started, threads


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args: argparse.Namespace) -> None:
    rank, world, _ = dist_setup(args.gpus)
    if rank != 0:
        return
    from jeff_b200 import synthetic

    model = synthetic.make_model(synthetic.ModelSpec())
    adapters = [synthetic.make_adapter(model, i, seed=1000 + i) for i in range(1, ADAPTERS + 1)]
    rows = synthetic.make_cfg4_rows(seed=4)
    threads = host_cores()
    picks = cpu_chunk(rows)
    for _ in range(args.warmup):
        cpu_sample(model, adapters, rows, picks, threads)
    times = [cpu_sample(model, adapters, rows, picks, threads)[0] for _ in range(args.steps)]
    sec = sum(times) / len(times)
    value = len(picks) / sec
    line = {"metric": METRIC, "value": value, "unit": "decisions/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": sec * 1000, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic", "impl": "reference",
            "config": {"workload": f"cfg4: one chunk of {len(picks)} calls of one adapter (each 512-token prefix + "
                                   "128 new tokens, whole prompt recomputed), the reference's standard-path chunking",
                       "model": "hybrid GDN/attention 24 layers, int4-g128z weights dequantised",
                       "global_batch": len(picks), "seq_len": PREFIX + NEW, "parallelism": "cpu"},
            "cpu_baseline": {"value": value, "unit": "decisions/s", "cores": threads, "kind": "port",
                             "sample": f"{args.steps} steps, each one forward of {len(picks)} calls (640 tokens "
                                       "each) of one adapter group"},
            "e2e": {"value": value, "unit": "decisions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- the B200 arm


def build_replica(rank: int, world: int):
    from jeff_b200 import synthetic
    from jeff_b200.fast_path import FastPath

    spec = synthetic.ModelSpec()
    skeleton = rank != 0
    model = synthetic.make_model(spec, skeleton=skeleton)
    adapters = [synthetic.make_adapter(model, i, seed=1000 + i, skeleton=skeleton) for i in range(1, ADAPTERS + 1)]
    head = synthetic.base_head(model) if not skeleton else None
    fast = FastPath(model, max_adapters=ADAPTERS, pool_pages_count=2 + ADAPTERS * 70 + 64,
                    base_readout=head)
    for ad in adapters:
        fast.add_adapter(ad)
    if world > 1:
        from jeff_b200 import replicas

        replicas.broadcast_tensors(fast.tensors(), 0)
        torch.cuda.synchronize()
    return model, adapters, fast


def products_graph(path, b: int, n: int):
    """A graph of the pass's 96 int4 products (with LoRA) in layer order on the workspace's buffers, their
    algorithmic FLOPs (2 m k out for the base, 2 m R (k + out) for the LoRA) and this library's launches in it."""
    f, ws = path.fast, path.ws
    t = b * n
    adapters = path.views(b, n)["adapters"]
    flops = 0

    def work() -> None:
        nonlocal flops
        flops = 0
        for layer in f.layers:
            for key, x in (("proj", ws.h[:t]), ("out", ws.y[:t]), ("mlp_in", ws.h[:t]), ("mlp_down", ws.act[:t])):
                lin = layer[key]
                y = {"proj": ws.pr[:t * lin.out].view(t, lin.out), "out": ws.d[:t], "mlp_in": ws.act[:t],
                     "mlp_down": ws.d[:t]}[key]
                lin(x, adapters, n, ws.mid, y)
                flops += 2 * t * lin.k * lin.out + 2 * t * lin.rank * (lin.k + lin.out)

    graph, _ = path._capture(work)
    return graph, flops, path.last_capture_launches


def traffic_from_profiles() -> float | None:
    """DRAM bytes per launch of the product kernel from the committed ncu summary (profiles/), when present."""
    p = ROOT / "profiles" / "w4a16_lora_kernel_cfg4.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["dram_bytes_per_launch"])
        except Exception:
            return None
    return None


def run_b200(args: argparse.Namespace) -> None:
    rank, world, local = dist_setup(args.gpus)
    from jeff_b200 import _lib, synthetic
    from jeff_b200.batched_path import BatchedPath, Row

    _lib.load()
    model, adapters, fast = build_replica(rank, world)
    rows = synthetic.make_cfg4_rows(seed=4 + 100 * rank)
    texts = {}
    for a, p in zip(rows.adapters, rows.prefixes):
        texts[f"cfg4 prefix of adapter {a}"] = p
    path = BatchedPath(fast, tokenize=lambda t: texts[t], max_tokens=CALLS * NEW, max_rows_per_pass=CALLS)
    index = [fast.index(f"adapter-{a}") for a in rows.adapters]
    keys = [(index[i], f"cfg4 prefix of adapter {rows.adapters[i]}") for i in range(CALLS)]
    slots, prefix_timing = path.ensure_prefixes(keys, max_tokens=8192)
    part = [(index[i], slots[i], Row(keys[i][1], rows.new_ids[i], rows.counts[i])) for i in range(CALLS)]
    lengths = [path.pool.length(s) for s in slots]
    graph, out = path.graph(CALLS, NEW)
    size = path.fill(CALLS, NEW, part, lengths)
    path.inp[:size].copy_(path.inp_host[:size])
    torch.cuda.synchronize()
    if args.profile:
        # one eager decision pass between cudaProfilerStart/Stop (ncu --profile-from-start off sees only it)
        torch.cuda.profiler.start()
        path.body(CALLS, NEW)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        return

    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # ---- value: inputs resident in HBM
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    with Clocks(local) as clocks:
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        end.record(stream)
        end.synchronize()
        barrier(world)
    ms = max_over_ranks(start.elapsed_time(end) / args.steps, world)
    value = CALLS * world / (ms / 1000.0)
    probs_first = out.clone()

    # ---- e2e: host buffers, H2D + replay + D2H every step
    for _ in range(args.warmup):
        path.run_pass(CALLS, NEW, part, lengths)
    barrier(world)
    torch.cuda.synchronize()
    e2e_times = []
    wall0 = time.perf_counter()
    for _ in range(args.steps):
        _, step_ms = path.run_pass(CALLS, NEW, part, lengths)
        e2e_times.append(step_ms)
    wall = (time.perf_counter() - wall0) / args.steps * 1000
    barrier(world)
    e2e_ms = max_over_ranks(max(sum(e2e_times) / len(e2e_times), wall), world)
    e2e_value = CALLS * world / (e2e_ms / 1000.0)
    deterministic = bool(torch.equal(probs_first, out))

    # ---- roofline of the dominant kernel (the int4 product), rank 0's GPU
    pg, flops, prod_launches = products_graph(path, CALLS, NEW)
    for _ in range(3):
        pg.replay()
    torch.cuda.synchronize()
    reps = max(3, args.steps)
    start.record(stream)
    for _ in range(reps):
        pg.replay()
    end.record(stream)
    end.synchronize()
    prod_ms = start.elapsed_time(end) / reps
    pk = peaks()
    achieved_tflops = flops / (prod_ms / 1000.0) / 1e12
    gemms = 96
    launches_per_pass = path.graph_launches.get((CALLS, NEW), 0)

    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": "decisions/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 (int4 weights, fp32 accumulate)", "data": "synthetic",
        "config": {"workload": "cfg4: 64 calls x 128 new tokens on 16 shared 512-token prefixes (pool), 16 rank-16 "
                               "adapters, int4 group-128 + bf16 scale/zero, 24 layers (18 GDN + 6 attention)",
                   "global_batch": CALLS * world, "seq_len": NEW, "prefix_tokens": PREFIX, "adapters": ADAPTERS,
                   "parallelism": f"replicas x{world}", "l2": "weights 264 MB > 126 MB L2 (no flush needed)"},
        "e2e": {"value": e2e_value, "unit": "decisions/s", "h2d_bytes_per_step": size * 4,
                "d2h_bytes_per_step": CALLS * 255 * 4},
        "gpu_launches": launches_per_pass * args.steps,
        "roofline": {"bound": "tensor", "kernel": "w4a16_lora_kernel (+ lora_shrink)", "achieved": achieved_tflops,
                     "peak": pk["bf16"], "unit": "TFLOP/s", "frac": achieved_tflops / pk["bf16"],
                     "peak_source": f"{pk['source']} bf16 burst", "traffic": traffic_from_profiles(),
                     "flops_per_pass": flops, "launches_per_pass": gemms, "products_ms_per_pass": prod_ms,
                     "launches_in_products_graph": prod_launches},
        "prefix_ms": prefix_timing["prefix_ms"], "deterministic_replays": deterministic,
    }
    if world == 1 and not args.no_cpu:
        picks = cpu_chunk(rows)
        sec, threads = cpu_sample(model, adapters, rows, picks, host_cores())
        line["cpu_baseline"] = {"value": len(picks) / sec, "unit": "decisions/s", "cores": threads, "kind": "port",
                                "sample": f"one forward of {len(picks)} calls of one adapter group (512 prefix + 128 "
                                          "new tokens each, fp32 standard path, the reference's chunking)"}
    line["clocks"] = clocks.summary()
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--profile", action="store_true",
                    help="run one eager pass inside cudaProfilerStart/Stop (for ncu --profile-from-start off) and exit")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    try:
        if args.impl == "reference":
            run_reference(args)
        else:
            run_b200(args)
    finally:
        if int(os.environ.get("WORLD_SIZE", "1")) > 1:
            import torch.distributed as dist

            if dist.is_initialized():
                dist.destroy_process_group()


if __name__ == "__main__":
    main()
