"""Kernel throughput of the hot path's roofline targets on synthetic inputs shaped like the benchmark's
configurations 1 and 3 (bench.py reports the whole decision pass; this reports single kernels against HBM).

    python -m jeff_b200.kernel_bench [--reps N]

cfg1: one int4 W4A16 + LoRA product: M 64 tokens, K 1024, N 3584, one rank-16 adapter, int4 group 128 with bf16
  scales and zeros. Algorithmic bytes per call 2,686,976 (words 1,835,008 + scales 57,344 + zeros 57,344 + x 131,072
  + y 458,752 + A 32,768 + B 114,688): HBM-bound. Timed as a CUDA graph of 256 calls cycling through enough distinct
  weight copies to exceed twice the 126 MB L2, so each call streams its weights from HBM; once through the persistent
  kernel (jb_int4_lora_product) and once through the small-pass route the batched path takes (the split entry: the
  warp-per-dot LoRA shrink and the weight-streaming kernel with its K slices one cluster).
small: the products of one batch-1 decision (32 new tokens, one row), each shape through both routes the same way.
cfg2: the projection sweep over one decoder layer (q 1024->2048, k and v 1024->512, o 2048->1024, gate and up
  1024->3584, down 3584->1024, q with its gate 1024->4096): 64 requests of 32 to 128 tokens packed into M = 4096 rows
  with one adapter id per token, 8 rank-16 adapters, int4 group 128 with bf16 scales and zeros. Per projection
  FLOPs 2MNK + 2M 16 (K + N) and algorithmic bytes K N / 2 + 2 (K / 128) N 2 + M K 2 + M N 2 + 8 16 (K + N) 2 + M 4:
  tensor-bound (400 to 1500 FLOP per byte), so each line gives TFLOP/s against the measured bf16 peak beside GB/s.
  Timed like cfg1, cycling through enough copies of x, the weights and y to exceed twice the L2.
cfg3: one Gated DeltaNet prefill layer: 64 rows x 256 new tokens, each from a pooled fp32 state ~ N(0, 0.1). The
  prep kernel (conv width 4 + SiLU + L2 norms + gates from the projection output) reads 201 MB of q/k/v inputs,
  1 MB of gates and 2.4 MB of convolution tails and writes 201 MB of q/k/v and 1.5 MB of g/beta; the chunked scan
  reads q, k, v (201 MB), g and beta (1.5 MB) and the states (67 MB) and writes o (67 MB): 337 MB. The fused mixer
  (jb_gdn_layer: prep, scan and gated norm in one launch) reads the projection output (270 MB: q | k | v | z | b | a),
  the tails and the states and writes y (67 MB): 406 MB, with q, k, v and o never in HBM.

One JSON line per kernel: milliseconds per call, GB/s of algorithmic bytes, and the fraction of the measured HBM copy
bandwidth (MEASURED_PEAKS.json beside the repository root when present); for cfg2 also TFLOP/s and the fraction of
the measured dense bf16 peak (the burst figure: each kernel is timed alone)."""

from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import torch

from jeff_b200 import constants as C
from jeff_b200 import int4, kernels, synthetic
from jeff_b200.prefix_pool import PrefixPool

ROOT = Path(__file__).resolve().parent.parent
L2_BYTES = 126 * 2**20


def hbm_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def tensor_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def timed(fn, reps: int) -> float:
    """Milliseconds per call of fn on the current stream (CUDA events, after 3 warm-up calls)."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        fn()
    end.record()
    end.synchronize()
    return start.elapsed_time(end) / reps


def cfg1(reps: int) -> dict:
    m, k, n, rank = 64, 1024, 3584, 16
    w = synthetic.normal(1, "cfg1/w", (n, k), 0.02)
    packed, _ = int4.quantize_pack(w, "g128z")
    per_copy = packed.words.numel() * 4 + packed.scales.numel() * 2 + packed.zeros.numel() * 2
    copies = math.ceil(2 * L2_BYTES / per_copy)
    dev = packed.to("cuda")
    words = [kernels.int4_repack(dev.words.clone()) for _ in range(copies)]
    scales = [dev.scales.clone() for _ in range(copies)]
    zeros = [dev.zeros.clone() for _ in range(copies)]
    a_pool = torch.zeros(2, rank, k, dtype=torch.bfloat16, device="cuda")
    b_pool = torch.zeros(2, packed.columns, rank, dtype=torch.bfloat16, device="cuda")
    a_pool[1] = synthetic.normal(1, "cfg1/a", (rank, k), 0.02).to(torch.bfloat16)
    b_pool[1, :n] = (2.0 * synthetic.normal(1, "cfg1/b", (n, rank), 0.01)).to(torch.bfloat16)
    adapters = torch.ones(1, dtype=torch.int32, device="cuda")
    x = synthetic.normal(1, "cfg1/x", (m, k), 1.0).to(torch.bfloat16).cuda()
    y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    mid = torch.empty(m, rank, dtype=torch.bfloat16, device="cuda")
    calls = 256

    def body() -> None:
        for i in range(calls):
            j = i % copies
            kernels.int4_product(x, words[j], scales[j], zeros[j], packed.group, n, a_pool, b_pool, adapters, m,
                                 mid=mid, y=y)

    body()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        body()
    ms = timed(graph.replay, reps) / calls
    scratch = (torch.empty(4 * 2**20, dtype=torch.float32, device="cuda"),
               torch.zeros(1024, dtype=torch.int32, device="cuda"))

    def body_small() -> None:
        for i in range(calls):
            j = i % copies
            kernels.int4_product(x, words[j], scales[j], zeros[j], packed.group, n, a_pool, b_pool, adapters, m,
                                 mid=mid, y=y, split=scratch)

    body_small()
    torch.cuda.synchronize()
    graph_small = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_small):
        body_small()
    small_ms = timed(graph_small.replay, reps) / calls
    algo = 1_835_008 + 57_344 + 57_344 + 131_072 + 458_752 + 32_768 + 114_688
    config = "cfg1 M64 K1024 N3584 rank16 g128z"
    return [{"kernel": "w4a16_lora (lora_shrink + w4a16_lora_kernel)", "config": config, "ms": ms, "bytes": algo,
             "weight_copies": copies},
            {"kernel": "small-pass route (lsh::dot_kernel + w4s::small_kernel, K slices one cluster)",
             "config": config, "ms": small_ms, "bytes": algo, "weight_copies": copies}]


def small(reps: int) -> list[dict]:
    """The products of one batch-1 decision (32 new tokens of one row, one adapter, configuration 4's int4 g128 + zero
    base), each shape as the batched path runs it at 32 tokens: the LoRA first factor (dot kernel) and the
    weight-streaming small-pass product through jb_int4_lora_product_split, beside the persistent kernel
    (jb_int4_lora_product) on the same call. Weights cycled past twice the L2 between calls; algorithmic bytes: the
    int4 words, scales and zeros, x, y, the adapter's A and B rows and mid."""
    m, rank_of = 32, {"in_proj": 48, "qkv": 48, "out_proj": 16, "o_proj": 16, "gate_up": 32, "down": 16}
    shapes = [("in_proj", 1024, C.GDN_PROJ), ("qkv", 1024, C.ATTN_PROJ), ("out_proj", 2048, 1024),
              ("o_proj", 2048, 1024), ("gate_up", 1024, 2 * C.INTER), ("down", C.INTER, 1024)]
    lines = []
    for name, k, n in shapes:
        rank = rank_of[name]
        packed, _ = int4.quantize_pack(synthetic.normal(1, f"small/{name}", (n, k), 0.02), "g128z")
        per_copy = packed.words.numel() * 4 + packed.scales.numel() * 2 + packed.zeros.numel() * 2
        copies = math.ceil(2 * L2_BYTES / per_copy)
        dev = packed.to("cuda")
        words = [kernels.int4_repack(dev.words.clone()) for _ in range(copies)]
        scales = [dev.scales.clone() for _ in range(copies)]
        zeros = [dev.zeros.clone() for _ in range(copies)]
        a_pool = (0.02 * torch.randn(2, rank, k, device="cuda")).to(torch.bfloat16)
        b_pool = (0.01 * torch.randn(2, packed.columns, rank, device="cuda")).to(torch.bfloat16)
        adapters = torch.ones(1, dtype=torch.int32, device="cuda")
        x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
        y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
        mid = torch.empty(m, rank, dtype=torch.bfloat16, device="cuda")
        scratch = (torch.empty(4 * 2**20, dtype=torch.float32, device="cuda"),
                   torch.zeros(1024, dtype=torch.int32, device="cuda"))
        calls = 64
        res = {}
        for route, split in (("persistent", None), ("small", scratch)):
            def body() -> None:
                for i in range(calls):
                    j = i % copies
                    kernels.int4_product(x, words[j], scales[j], zeros[j], packed.group, n, a_pool, b_pool, adapters,
                                         m, mid=mid, y=y, split=split)

            body()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                body()
            res[route] = timed(graph.replay, reps) / calls
            del graph
        algo = per_copy + m * k * 2 + m * n * 2 + rank * (k + n) * 2 + m * rank * 2
        lines.append({"kernel": "small-pass route (lsh::dot_kernel + w4s::small_kernel)",
                      "config": f"batch-1 {name} M{m} K{k} N{n} rank{rank} g128z", "ms": res["small"],
                      "persistent_ms": res["persistent"], "bytes": algo, "weight_copies": copies})
        del words, scales, zeros
        torch.cuda.empty_cache()
    lines.append({"kernel": "batch-1 products of a Gated DeltaNet layer (in_proj, out_proj, gate_up, down)",
                  "config": "batch-1 M32", "ms": sum(x["ms"] for x in lines if x["config"].split()[1] in
                                                      ("in_proj", "out_proj", "gate_up", "down")),
                  "persistent_ms": sum(x["persistent_ms"] for x in lines if x["config"].split()[1] in
                                       ("in_proj", "out_proj", "gate_up", "down")),
                  "bytes": sum(x["bytes"] for x in lines if x["config"].split()[1] in
                               ("in_proj", "out_proj", "gate_up", "down"))})
    return lines


def cfg2(reps: int) -> list[dict]:
    lengths = synthetic.cfg2_lengths()
    chosen = synthetic.cfg2_adapters()
    per_token = torch.tensor(chosen, dtype=torch.int32).repeat_interleave(torch.tensor(lengths)).cuda()
    m = sum(lengths)
    lines = []
    for name, k, n in synthetic.CFG2_SHAPES:
        proj = synthetic.cfg2_projection(name, k, n)
        packed = proj.packed
        per_copy = m * k * 2 + packed.words.numel() * 4 + 2 * packed.scales.numel() * 2 + m * n * 2
        copies = math.ceil(2 * L2_BYTES / per_copy)
        dev = packed.to("cuda")
        words = [kernels.int4_repack(dev.words.clone()) for _ in range(copies)]
        scales = [dev.scales.clone() for _ in range(copies)]
        zeros = [dev.zeros.clone() for _ in range(copies)]
        xs = [proj.x.cuda() for _ in range(copies)]
        ys = [torch.empty(m, n, dtype=torch.bfloat16, device="cuda") for _ in range(copies)]
        a_pool, b_pool = proj.lora_a.cuda(), proj.lora_b.cuda()
        mid = torch.empty(m, a_pool.shape[1], dtype=torch.bfloat16, device="cuda")
        calls = 8 * copies

        def body() -> None:
            for i in range(calls):
                j = i % copies
                kernels.int4_product(xs[j], words[j], scales[j], zeros[j], packed.group, n, a_pool, b_pool,
                                     per_token, 1, mid=mid, y=ys[j])

        body()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            body()
        ms = timed(graph.replay, reps) / calls

        def shrinks() -> None:
            for i in range(calls):
                kernels.lora_shrink(xs[i % copies], a_pool, per_token, 1, out=mid)

        shrinks()
        torch.cuda.synchronize()
        shrink_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(shrink_graph):
            shrinks()
        shrink_ms = timed(shrink_graph.replay, reps) / calls
        rank, n_adapters = a_pool.shape[1], a_pool.shape[0] - 1
        flops = 2 * m * n * k + 2 * m * rank * (k + n)
        algo = (k * n // 2 + 2 * (k // 128) * n * 2 + m * k * 2 + m * n * 2 + n_adapters * rank * (k + n) * 2
                + m * 4)
        lines.append({"kernel": "w4a16_lora (lora_shrink + w4a16_lora_kernel)",
                      "config": f"cfg2 {name} M{m} K{k} N{n} packed 64 requests, 8 rank-16 adapters, g128z",
                      "ms": ms, "shrink_ms": shrink_ms, "bytes": algo, "flops": flops, "copies": copies})
        del graph, shrink_graph, words, scales, zeros, xs, ys
        torch.cuda.empty_cache()
    lines.append({"kernel": "cfg2 sweep: the 8 projections one after another", "config": "cfg2 M4096 packed",
                  "ms": sum(x["ms"] for x in lines), "shrink_ms": sum(x["shrink_ms"] for x in lines),
                  "bytes": sum(x["bytes"] for x in lines),
                  "flops": sum(x["flops"] for x in lines)})
    return lines


def cfg3(reps: int) -> list[dict]:
    rows, n = 64, 256
    t = rows * n
    pool = PrefixPool(2 + rows * 51, "cuda")
    slots = [pool.reserve(1, f"cfg3 state {i}", 1) for i in range(rows)]
    g = torch.Generator(device="cuda").manual_seed(3)
    pool.state.normal_(0.0, 0.1, generator=g)
    pool.conv.normal_(0.0, 1.0, generator=g)
    tables = pool.tables.index_select(0, torch.tensor(slots, device="cuda")).contiguous()
    pr = torch.randn(t, C.GDN_PROJ, generator=g, device="cuda").to(torch.bfloat16)
    conv_w = (0.5 * torch.randn(4, C.QKV_DIM, generator=g, device="cuda")).to(torch.bfloat16).float().contiguous()
    a_neg = -torch.rand(C.NV, generator=g, device="cuda") * 16.0
    dt_bias = torch.ones(C.NV, device="cuda")
    outs = kernels.gdn_prep_rows(pr, pool, tables, 0, conv_w, a_neg, dt_bias, n)
    o = torch.empty_like(outs[2])
    prep_ms = timed(lambda: kernels.gdn_prep_rows(pr, pool, tables, 0, conv_w, a_neg, dt_bias, n, outs=outs), reps)
    q, k, v, gg, beta = outs
    scan_ms = timed(lambda: kernels.gdn_scan(q, k, v, gg, beta, pool, tables, 0, out=o, kernel="tc"), reps)
    chunk_ms = timed(lambda: kernels.gdn_scan(q, k, v, gg, beta, pool, tables, 0, out=o, kernel="chunk"), reps)
    gnorm = torch.ones(C.DV, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(t, C.NV * C.DV, dtype=torch.bfloat16, device="cuda")
    norm_ms = timed(lambda: kernels.gated_norm(o.view(t, C.NV, C.DV), pr, gnorm, out=y), reps)
    layer_ms = timed(lambda: kernels.gdn_layer(pr, pool, tables, 0, conv_w, a_neg, dt_bias, gnorm, n, out=y), reps)
    qkv = t * C.QKV_DIM * 2
    tails = rows * 3 * C.QKV_DIM * 2 + 4 * C.QKV_DIM * 4
    states = rows * C.NV * C.DK * C.DV * 4
    prep_bytes = qkv + t * 2 * C.NV * 2 + tails + qkv + t * C.NV * (4 + 2)
    scan_bytes = qkv + t * C.NV * (4 + 2) + states + t * C.NV * C.DV * 2
    norm_bytes = 3 * t * C.NV * C.DV * 2
    # the fused mixer reads the projection output's q | k | v | z | b | a, the tails, taps and states, writes y
    layer_bytes = t * C.GDN_PROJ * 2 + tails + states + t * C.NV * C.DV * 2
    config = "cfg3 64 rows x 256 tokens"
    return [{"kernel": "gdn prep_kernel", "config": config, "ms": prep_ms, "bytes": prep_bytes},
            {"kernel": "gdn scan_kernel (tcgen05 chunk scan from pooled state)", "config": config, "ms": scan_ms,
             "bytes": scan_bytes},
            {"kernel": "gdn chunk_kernel (mma.sync chunk scan from pooled state)", "config": config, "ms": chunk_ms,
             "bytes": scan_bytes},
            {"kernel": "gated_norm_kernel", "config": config, "ms": norm_ms, "bytes": norm_bytes},
            {"kernel": "gdn layer_kernel (prep + scan + gated norm fused)", "config": config, "ms": layer_ms,
             "bytes": layer_bytes, "unfused_ms": prep_ms + scan_ms + norm_ms}]


def cfg4_attention(reps: int) -> list[dict]:
    """Configuration 4's attention layer: 64 rows x 128 new tokens, each over its own 512-token prefix in pool pages;
    the tcgen05 kernel with the gate fused, and the mma.sync kernel + gate_mul. FLOPs: Q K^T and P V over each query's
    keys (the 512 prefix keys and its causal new keys); bytes: q, the new keys and values, the prefix pages' keys and
    values of this layer, the gates and y."""
    b, n, plen = 64, 128, 512
    pool = PrefixPool(2 + b * (50 + plen // 32) + 4, "cuda")
    slots = [pool.reserve(1, f"attention {r}", plen) for r in range(b)]
    g = torch.Generator(device="cuda").manual_seed(4)
    pool.kv.normal_(0.0, 1.0, generator=g)
    tables = pool.tables.index_select(0, torch.tensor(slots, device="cuda")).contiguous()
    pos = torch.full((b,), plen, dtype=torch.int32, device="cuda")
    t = b * n
    q = torch.randn(t, C.NQ, C.HD, generator=g, device="cuda").to(torch.bfloat16)
    kn = torch.randn(t, C.NKV, C.HD, generator=g, device="cuda").to(torch.bfloat16)
    vn = torch.randn(t, C.NKV, C.HD, generator=g, device="cuda").to(torch.bfloat16)
    pr = torch.randn(t, C.ATTN_PROJ, generator=g, device="cuda").to(torch.bfloat16)
    y = torch.empty(t, C.NQ * C.HD, dtype=torch.bfloat16, device="cuda")
    ao = torch.empty(t, C.NQ, C.HD, dtype=torch.bfloat16, device="cuda")
    tc_ms = timed(lambda: kernels.paged_attention_gated(q, pool, tables, 0, pos, kn, vn, n, pr, out=y), reps)

    def old() -> None:
        kernels.paged_attention(q, pool, tables, 0, pos, kn, vn, n, out=ao)
        kernels.gate_mul(ao, pr, out=y)

    old_ms = timed(old, reps)
    keys = b * C.NQ * sum(plen + i + 1 for i in range(n))          # (query, key) pairs
    flops = 4 * keys * C.HD
    bytes_ = t * C.NQ * C.HD * 2 * 3 + 2 * t * C.NKV * C.HD * 2 + b * plen * 2 * C.NKV * C.HD * 2
    config = "cfg4 attention: 64 rows x 128 new tokens over 512-token prefixes"
    return [{"kernel": "attention_kernel (tcgen05, gate fused)", "config": config, "ms": tc_ms, "bytes": bytes_,
             "flops": flops},
            {"kernel": "paged_attention_kernel (mma.sync) + gate_mul_kernel", "config": config, "ms": old_ms,
             "bytes": bytes_, "flops": flops}]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--only", choices=["cfg1", "cfg2", "cfg3", "attention", "small"], default=None)
    args = ap.parse_args()
    if not torch.cuda.is_available():
        raise SystemExit("kernel_bench needs a CUDA GPU")
    torch.cuda.set_device(0)
    peak, source = hbm_peak()
    tpeak, tsource = tensor_peak()
    runs = {"cfg1": lambda: cfg1(args.reps), "cfg2": lambda: cfg2(args.reps), "cfg3": lambda: cfg3(args.reps),
            "attention": lambda: cfg4_attention(args.reps), "small": lambda: small(args.reps)}
    chosen = [args.only] if args.only else list(runs)
    for line in [x for name in chosen for x in runs[name]()]:
        gbs = line["bytes"] / (line["ms"] / 1e3) / 1e9
        line.update(gbs=gbs, hbm_peak_gbs=peak, peak_source=source, frac=gbs / peak)
        if "flops" in line:
            tflops = line["flops"] / (line["ms"] / 1e3) / 1e12
            line.update(tflops=tflops, bf16_peak_tflops=tpeak, tensor_peak_source=tsource, tensor_frac=tflops / tpeak)
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
