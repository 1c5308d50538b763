"""The batched decision path on B200 (the reference's engine/batched_path.py BatchedPath, :177-752): one CUDA graph
replay answers up to 64 rows, each with its own adapter and cached prefix, on a FastPath's weights and pools.

A pass holds B rows of N new tokens (T = B * N, row after row), each row padded to N after its last real token;
every layer is causal, so padding never reaches a real token. One graph per (B, N), recorded on first use (or all
at start with record()); everything a graph reads per row comes from ONE packed int32 input buffer in device memory
(batched_path.py:45-50): [slot, adapter, prefix length, last, count] x B, then the B x N token ids, filled on the
host with numpy into a pinned twin and copied in with one copy; the probabilities (B x 255) come back in one copy.
All intermediate tensors live in one preallocated Workspace, so capture and replay allocate nothing.

Batched prefix passes (batched_path.py:291-349, :613-744): new prefixes are processed B at a time from the empty
state, each row writing its final Gated DeltaNet states, convolution tails and attention keys/values straight into its
own slot's pages (the kernels take the rows' page lists from the prefix input buffer).

Calls are serialised by the caller (the engine's GPU thread), adapter changes between passes."""

from __future__ import annotations

import time
from collections.abc import Callable, Sequence
from dataclasses import dataclass
from typing import Any

import numpy as np
import torch

from jeff_b200 import _lib
from jeff_b200 import constants as C
from jeff_b200 import kernels
from jeff_b200.fast_path import FastPath
from jeff_b200.prefix_pool import PAGE_TOKENS, SINK_PAGE, ZERO_PAGE

DT = torch.bfloat16
PASS_SHAPES = tuple((b, n) for n in C.NEW_BUCKETS for b in C.BATCH_BUCKETS if b * n <= C.MAX_PASS_TOKENS)
PREFIX_PASS_ROWS = {64: 16, 128: 32, 256: 16, 512: 8, 768: 4, 1024: 4, 1536: 4, 2048: 2, 3072: 2, 4096: 1,
                    6144: 1, 8192: 1}
PREFIX_META = 2


@dataclass
class Row:
    """One question ready for the fast path (the reference's prepare.Row): prefix text, new token ids, options."""
    prefix_text: str
    new_ids: list[int]
    count: int


def max_rows(n: int) -> int:
    return max(b for b in C.BATCH_BUCKETS if b * n <= C.MAX_PASS_TOKENS)


SPLIT_FLOATS = 8 * 2**20     # 32 MB: the slices of a 512-token pass's widest product
SPLIT_COUNTERS = 4096


class Workspace:
    """Every intermediate tensor of a pass of up to `tokens` tokens and `rows` rows."""

    def __init__(self, tokens: int, rows: int, width: int, max_rank: int, device: torch.device) -> None:
        def e(*shape: int, dtype: torch.dtype = DT) -> torch.Tensor:
            return torch.empty(*shape, dtype=dtype, device=device)

        self.tokens, self.rows = tokens, rows
        self.x = e(tokens, C.HIDDEN)
        self.h = e(tokens, C.HIDDEN)
        self.d = e(tokens, C.HIDDEN)
        self.pr = e(tokens * C.GDN_PROJ)
        self.q = e(tokens * C.NV * C.DK)
        self.k = e(tokens * C.NV * C.DK)
        self.v = e(tokens * C.NV * C.DV)
        self.g = e(tokens * C.NV, dtype=torch.float32)
        self.beta = e(tokens * C.NV)
        self.o = e(tokens * C.NV * C.DV)
        self.y = e(tokens, C.NQ * C.HD)
        self.aq = e(tokens, C.NQ, C.HD)
        self.ao = e(tokens, C.NQ, C.HD)
        self.kn = e(tokens, C.NKV, C.HD)
        self.vn = e(tokens, C.NKV, C.HD)
        self.act = e(tokens, C.INTER)
        self.mid = e(tokens * max(max_rank, 16))
        # split-K scratch of small passes' products (jb_int4_lora_product_split): fp32 slice sums and per-tile
        # counters, which start at zero and are left at zero by every product
        self.split = (torch.empty(SPLIT_FLOATS, dtype=torch.float32, device=device),
                      torch.zeros(SPLIT_COUNTERS, dtype=torch.int32, device=device))
        self.tables = torch.zeros(rows, width, dtype=torch.int32, device=device)
        self.zero_tables = torch.zeros(rows, width, dtype=torch.int32, device=device)
        self.zero_pos = torch.zeros(rows, dtype=torch.int32, device=device)
        self.hidden = e(rows, C.HIDDEN)
        self.probs = e(rows, C.READOUT_ROWS, dtype=torch.float32)


class BatchedPath:
    def __init__(self, fast: FastPath, tokenize: Callable[[str], list[int]] | None = None,
                 max_tokens: int = C.MAX_PASS_TOKENS, max_rows_per_pass: int = max(C.BATCH_BUCKETS),
                 batch_buckets: Sequence[int] = C.BATCH_BUCKETS) -> None:
        # the row counts decide() pads a decision pass to (one recorded graph per bucket and new-token bucket): the
        # reference's 1, 2, 4, ..., 64 by default; a deployment may record fewer (configuration 5: 1, 8, 16, 32, 64)
        if sorted(batch_buckets) != list(batch_buckets) or batch_buckets[0] != 1 or \
                batch_buckets[-1] != max(C.BATCH_BUCKETS):
            raise ValueError(f"batch buckets {list(batch_buckets)}: increasing, from 1 to {max(C.BATCH_BUCKETS)}")
        self.batch_buckets = tuple(batch_buckets)
        self.fast = fast
        self.pool = fast.prefixes
        # the Gated DeltaNet mixer: three launches (jb_gdn_prep_rows, jb_gdn_scan, jb_gated_norm) by default, or the
        # fused jb_gdn_layer (the same bits, tested). Measured on a B200 at configuration 3 the fused launch takes
        # 0.73 ms against 0.53 ms for the three: it saves the q, k, v and o traffic, but its prep and norm
        # instructions then run inside the scan's one 8-warp CTA per SM, which issues on 30% of cycles (latency
        # bound), where the separate prep kernel runs them at full occupancy. So the pass keeps the three launches.
        self.fused_gdn = False
        # the chunk scan of decision passes and of prefix passes: "tc" (tcgen05, the default), "chunk" (mma.sync) or
        # "recurrent" (token by token in fp32, no bf16 operands inside the rule)
        self.gdn_scan_kernel = "tc"
        # prefix states are cached and every later call on the prefix starts from them, so the prefix pass computes
        # them with the fp32 rule (no bf16 operands inside the chunk products; 1.5x the tcgen05 scan's prefix-pass
        # time, measured on a B200): on the 1,024 chained calls of configuration 4 this takes the decision/abstain
        # outcomes identical to the oracle's from 1,022 to 1,023 (both remaining differences within 0.01 of the
        # 0.8 threshold)
        self.gdn_prefix_scan_kernel = "recurrent"
        # passes too small to fill the GPU: products through jb_int4_lora_product_split (K slices for the smallest
        # passes' few-tile products) and the attention through jb_paged_attention_gated_split (the key walk in slices),
        # both on the workspace's split scratch
        self.split_k = True
        # attention: the tcgen05 kernel with the output gate fused (jb_paged_attention_gated); False runs the mma.sync
        # kernel and jb_gate_mul (the same result within the attention tolerance, tested)
        self.tc_attention = True
        self.tokenize = tokenize
        self.max_tokens = max_tokens
        dev = fast.device
        self.device = dev
        width = self.pool.width
        self.ws = Workspace(max_tokens, max_rows_per_pass, width, fast.max_rank, dev)
        self.ws.zero_tables[:, :self.pool.fixed_pages] = ZERO_PAGE
        size = max(C.META * b + b * n for b, n in PASS_SHAPES)
        self.inp = torch.zeros(size, dtype=torch.int32, device=dev)
        self.inp_host = torch.zeros(size, dtype=torch.int32).pin_memory()
        self.inp_np = self.inp_host.numpy()
        self.out_host = torch.zeros(max(C.BATCH_BUCKETS), C.READOUT_ROWS, dtype=torch.float32).pin_memory()
        # decide()'s passes, enqueued back to back: a second pinned input buffer (the two alternate, so one is
        # filled while the copy out of the other may still run), and pinned outputs and events per pass
        self.inp_host2 = torch.zeros(size, dtype=torch.int32).pin_memory()
        self.in_copied = [torch.cuda.Event(), torch.cuda.Event()]
        self.pass_out: list[torch.Tensor] = []
        self.pass_events: list[tuple[torch.cuda.Event, torch.cuda.Event]] = []
        psize = max((PREFIX_META + self._prefix_width(nb) + nb) * b for nb, cap in PREFIX_PASS_ROWS.items()
                    for b in C.BATCH_BUCKETS if b <= cap and b * nb <= max_tokens) if max_tokens >= 64 else 1
        self.prefix_inp = torch.zeros(psize, dtype=torch.int32, device=dev)
        self.prefix_inp_host = torch.zeros(psize, dtype=torch.int32).pin_memory()
        self.prefix_inp_np = self.prefix_inp_host.numpy()
        self.graphs: dict[tuple[int, int], tuple[torch.cuda.CUDAGraph, torch.Tensor]] = {}
        self.graph_launches: dict[tuple[int, int], int] = {}   # this library's kernels in each decision graph
        self.prefix_graphs: dict[tuple[int, int], torch.cuda.CUDAGraph] = {}
        self.graph_pool = torch.cuda.graph_pool_handle()
        self.stream = torch.cuda.Stream(device=dev)
        self.start = torch.cuda.Event(enable_timing=True)
        self.end = torch.cuda.Event(enable_timing=True)

    # ------------------------------------------------------------ input views

    def views(self, b: int, n: int) -> dict[str, torch.Tensor]:
        meta = self.inp[:C.META * b].view(C.META, b)
        return {"slots": meta[0], "adapters": meta[1], "pos": meta[2], "last": meta[3], "counts": meta[4],
                "ids": self.inp[C.META * b:C.META * b + b * n]}

    def _prefix_width(self, nb: int) -> int:
        return self.pool.fixed_pages + nb // PAGE_TOKENS

    def prefix_views(self, b: int, nb: int) -> dict[str, torch.Tensor]:
        w = self._prefix_width(nb)
        meta = self.prefix_inp[:PREFIX_META * b].view(PREFIX_META, b)
        pages = self.prefix_inp[PREFIX_META * b:(PREFIX_META + w) * b].view(b, w)
        ids = self.prefix_inp[(PREFIX_META + w) * b:(PREFIX_META + w + nb) * b]
        return {"adapters": meta[0], "lengths": meta[1], "pages": pages, "ids": ids}

    # ------------------------------------------------------------ the passes

    def _layers(self, x: torch.Tensor, adapters: torch.Tensor, n: int, t: int, gdn_tables: torch.Tensor,
                attn_tables: torch.Tensor, pos: torch.Tensor, last: torch.Tensor | None,
                real: torch.Tensor | None = None, out_tables: torch.Tensor | None = None,
                trace: list[torch.Tensor] | None = None, first: int = 0,
                stop: int | None = None) -> torch.Tensor | None:
        """Decoder layers first..stop-1 (all by default) over t tokens (rows of n), in place on the residual x;
        returns the last d. `trace` (eager runs only) receives each layer's residual stream bf16(x + d)."""
        f, ws, pool = self.fast, self.ws, self.pool
        b = t // n
        d: torch.Tensor | None = None
        gi = sum(1 for k in f.kinds[:first] if k == "linear_attention")
        ai = first - gi
        prefix = out_tables is not None
        stop = len(f.layers) if stop is None else stop
        for li in range(first, stop):
            layer = f.layers[li]
            _, h = kernels.add_rms(x, d, layer["norm_in"], xo=x, h=ws.h[:t])
            proj = layer["proj"]
            pr = proj(h, adapters, n, ws.mid, ws.pr[:t * proj.out].view(t, proj.out), split=ws.split if self.split_k else None)
            if layer["kind"] == "linear_attention" and self.fused_gdn:
                y = kernels.gdn_layer(pr, pool, gdn_tables, gi, layer["conv"], layer["a_neg"], layer["dt_bias"],
                                      layer["gnorm"], n, last=last, real=real, out_tables=out_tables,
                                      out=ws.y[:t, :C.NV * C.DV])
                gi += 1
            elif layer["kind"] == "linear_attention":
                size = t * C.NV * C.DK
                outs = (ws.q[:size].view(b, n, C.NV, C.DK), ws.k[:size].view(b, n, C.NV, C.DK),
                        ws.v[:size].view(b, n, C.NV, C.DV), ws.g[:t * C.NV].view(b, n, C.NV),
                        ws.beta[:t * C.NV].view(b, n, C.NV))
                q, k, v, g, beta = kernels.gdn_prep_rows(pr, pool, gdn_tables, gi, layer["conv"], layer["a_neg"],
                                                         layer["dt_bias"], n, real=real, out_tables=out_tables,
                                                         outs=outs)
                o = kernels.gdn_scan(q, k, v, g, beta, pool, gdn_tables, gi, last=last, out_tables=out_tables,
                                     kernel=self.gdn_prefix_scan_kernel if prefix else self.gdn_scan_kernel,
                                     out=ws.o[:size].view(b, n, C.NV, C.DV))
                y = kernels.gated_norm(o, pr, layer["gnorm"], out=ws.y[:t, :C.NV * C.DV])
                gi += 1
            else:
                kn, vn = ws.kn[:t], ws.vn[:t]
                aq = kernels.attn_prep_rows(pr, layer["q_w1"], layer["k_w1"], f.inv_freq, pos, kn, vn, n,
                                            out=ws.aq[:t])
                if prefix:
                    assert real is not None and out_tables is not None
                    kernels.kv_scatter(kn, vn, n, real, pool, out_tables, ai)
                    if li == len(f.layers) - 1:
                        return None   # the last layer: only its keys and values are kept
                if self.tc_attention:
                    y = kernels.paged_attention_gated(aq, pool, attn_tables, ai, pos, kn, vn, n, pr, out=ws.y[:t],
                                                      scratch=ws.split[0] if self.split_k else None)
                else:
                    ao = kernels.paged_attention(aq, pool, attn_tables, ai, pos, kn, vn, n, out=ws.ao[:t])
                    y = kernels.gate_mul(ao, pr, out=ws.y[:t])
                ai += 1
            d = layer["out"](y, adapters, n, ws.mid, ws.d[:t], split=ws.split if self.split_k else None)
            _, h = kernels.add_rms(x, d, layer["norm_post"], xo=x, h=ws.h[:t])
            act = layer["mlp_in"](h, adapters, n, ws.mid, ws.act[:t], split=ws.split if self.split_k else None)     # SwiGLU in the product's epilogue
            d = layer["mlp_down"](act, adapters, n, ws.mid, ws.d[:t], split=ws.split if self.split_k else None)
            if trace is not None:
                trace.append((x.float() + d.float()).to(DT))
        return d

    def body(self, b: int, n: int, trace: list[torch.Tensor] | None = None) -> torch.Tensor:
        """The recorded decision pass: B rows of N tokens from the packed input; returns probabilities (B, 255)."""
        f, ws = self.fast, self.ws
        v = self.views(b, n)
        t = b * n
        tables = ws.tables[:b]
        torch.index_select(self.pool.tables, 0, v["slots"], out=tables)
        x = kernels.embed(f.embed, v["ids"], out=ws.x[:t])
        d = self._layers(x, v["adapters"], n, t, tables, tables, v["pos"], v["last"], trace=trace)
        assert d is not None
        hidden = kernels.rms_last(x, d, v["last"], n, f.final_w1, out=ws.hidden[:b])
        return kernels.readout_rows(hidden, f.readout_pool, f.temp_pool, v["adapters"], v["counts"],
                                    out=ws.probs[:b])

    def prefix_body(self, b: int, nb: int) -> None:
        """The recorded prefix pass: B prefixes of at most nb tokens from the empty state, each row's state written
        into the pages its row of the prefix input lists (padding rows list the sink page only)."""
        f, ws = self.fast, self.ws
        if f.kinds[-1] != "full_attention":
            raise ValueError("The batched prefix pass expects the last layer to be an attention layer")
        v = self.prefix_views(b, nb)
        t = b * nb
        x = kernels.embed(f.embed, v["ids"], out=ws.x[:t])
        self._layers(x, v["adapters"], nb, t, ws.zero_tables[:b], ws.zero_tables[:b], ws.zero_pos[:b], None,
                     real=v["lengths"], out_tables=v["pages"])

    # ------------------------------------------------------------ graphs

    def _capture(self, work: Callable[[], Any]) -> tuple[torch.cuda.CUDAGraph, Any]:
        self.pool.sync()   # block tables current before capture (the captured pass only reads them)
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            for _ in range(2):
                work()
        self.stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        before = _lib.launches
        with torch.cuda.graph(graph, pool=self.graph_pool, stream=self.stream):
            out = work()
        self.last_capture_launches = _lib.launches - before
        torch.cuda.current_stream(self.device).wait_stream(self.stream)
        return graph, out

    def _pad_decision(self, b: int, n: int) -> None:
        meta = self.inp_np[:C.META * b].reshape(C.META, b)
        meta[:4] = 0
        meta[3] = n - 1
        meta[4] = 2
        self.inp_np[C.META * b:C.META * b + b * n] = 0
        self.inp[:C.META * b + b * n].copy_(self.inp_host[:C.META * b + b * n])

    def graph(self, b: int, n: int) -> tuple[torch.cuda.CUDAGraph, torch.Tensor]:
        if (b, n) not in self.graphs:
            if b * n > self.max_tokens:
                raise ValueError(f"A pass of {b} x {n} tokens exceeds this path's workspace ({self.max_tokens})")
            self._pad_decision(b, n)
            self.graphs[(b, n)] = self._capture(lambda: self.body(b, n))
            self.graph_launches[(b, n)] = self.last_capture_launches
        return self.graphs[(b, n)]

    def _pad_prefix(self, b: int, nb: int) -> None:
        w = self._prefix_width(nb)
        size = (PREFIX_META + w + nb) * b
        self.prefix_inp_np[:size] = 0
        self.prefix_inp_np[b:2 * b] = nb // 2
        self.prefix_inp_np[PREFIX_META * b:(PREFIX_META + w) * b] = SINK_PAGE
        self.prefix_inp[:size].copy_(self.prefix_inp_host[:size])

    def prefix_graph(self, b: int, nb: int) -> torch.cuda.CUDAGraph:
        if (b, nb) not in self.prefix_graphs:
            if b * nb > self.max_tokens:
                raise ValueError(f"A prefix pass of {b} x {nb} tokens exceeds this path's workspace")
            self._pad_prefix(b, nb)
            self.prefix_graphs[(b, nb)] = self._capture(lambda: self.prefix_body(b, nb))[0]
        return self.prefix_graphs[(b, nb)]

    def record(self, shapes: Sequence[tuple[int, int]] | None = None) -> float:
        """Record the decision graphs of `shapes` (by default every PASS_SHAPES shape of this path's batch buckets that
        the workspace holds)."""
        started = time.perf_counter()
        default = [s for s in PASS_SHAPES if s[0] * s[1] <= self.max_tokens and s[0] in self.batch_buckets]
        for b, n in shapes if shapes is not None else default:
            self.graph(b, n)
        torch.cuda.synchronize(self.device)
        return time.perf_counter() - started

    def trace_pass(self, b: int, n: int, part: Sequence[tuple[int, int, Row]],
                   lengths: Sequence[int]) -> tuple[torch.Tensor, list[torch.Tensor]]:
        """One pass run eagerly (no graph) with each layer's residual stream kept: (probs (B, 255), per layer
        (B * N, 1024) bf16). For parity tests."""
        size = self.fill(b, n, part, lengths)
        self.inp[:size].copy_(self.inp_host[:size])
        trace: list[torch.Tensor] = []
        probs = self.body(b, n, trace=trace).clone()
        torch.cuda.synchronize(self.device)
        return probs, trace

    def layer_pass(self, li: int, x_in: torch.Tensor, b: int, n: int, part: Sequence[tuple[int, int, Row]],
                   lengths: Sequence[int]) -> torch.Tensor:
        """Decoder layer `li` alone, eagerly, on the residual stream x_in (B * N, 1024) bf16 of the staged rows:
        returns its output residual stream bf16(x + d). For layer-local parity tests."""
        size = self.fill(b, n, part, lengths)
        self.inp[:size].copy_(self.inp_host[:size])
        v = self.views(b, n)
        t = b * n
        tables = self.ws.tables[:b]
        torch.index_select(self.pool.tables, 0, v["slots"], out=tables)
        x = self.ws.x[:t]
        x.copy_(x_in)
        d = self._layers(x, v["adapters"], n, t, tables, tables, v["pos"], v["last"], first=li, stop=li + 1)
        assert d is not None
        out = (x.float() + d.float()).to(DT)
        torch.cuda.synchronize(self.device)
        return out

    def last_layer_readout(self, x_in: torch.Tensor, b: int, n: int, part: Sequence[tuple[int, int, Row]],
                           lengths: Sequence[int]) -> torch.Tensor:
        """The last decoder layer, the final norm and the readout, eagerly, on the residual stream x_in (B * N, 1024)
        bf16 entering the last layer: probabilities (B, 255). For parity tests."""
        size = self.fill(b, n, part, lengths)
        self.inp[:size].copy_(self.inp_host[:size])
        f, ws = self.fast, self.ws
        v = self.views(b, n)
        t = b * n
        tables = ws.tables[:b]
        torch.index_select(self.pool.tables, 0, v["slots"], out=tables)
        x = ws.x[:t]
        x.copy_(x_in)
        li = len(f.layers) - 1
        d = self._layers(x, v["adapters"], n, t, tables, tables, v["pos"], v["last"], first=li, stop=li + 1)
        assert d is not None
        hidden = kernels.rms_last(x, d, v["last"], n, f.final_w1, out=ws.hidden[:b])
        probs = kernels.readout_rows(hidden, f.readout_pool, f.temp_pool, v["adapters"], v["counts"],
                                     out=ws.probs[:b]).clone()
        torch.cuda.synchronize(self.device)
        return probs

    # ------------------------------------------------------------ requests

    def fill(self, b: int, n: int, part: Sequence[tuple[int, int, Row]], lengths: Sequence[int],
             host: np.ndarray | None = None) -> int:
        """Stage rows into a pinned input buffer (`host`, by default the first; padding rows: slot 0, adapter 0, one
        token, one option)."""
        host = self.inp_np if host is None else host
        self.pool.sync()   # the pass reads the block tables of every reservation made before it
        size = C.META * b + b * n
        meta = host[:C.META * b].reshape(C.META, b)
        ids = host[C.META * b:size]
        meta[:4] = 0
        meta[4] = 1
        ids[:] = 0
        for j, (adapter, slot, row) in enumerate(part):
            real = len(row.new_ids)
            if real > n:
                raise AssertionError(f"{real} new tokens staged in a pass of {n}")
            ids[j * n:j * n + real] = row.new_ids
            meta[:, j] = (slot, adapter, lengths[j], real - 1, row.count)
        return size

    def run_pass(self, b: int, n: int, part: Sequence[tuple[int, int, Row]], lengths: Sequence[int]) -> tuple[
            np.ndarray, float]:
        """One pass: H2D of the packed input, graph replay, D2H of the probabilities. Returns (probs (B, 255), ms)."""
        graph, out = self.graph(b, n)
        size = self.fill(b, n, part, lengths)
        stream = torch.cuda.current_stream(self.device)
        self.start.record(stream)
        self.inp[:size].copy_(self.inp_host[:size], non_blocking=True)
        graph.replay()
        self.out_host[:b].copy_(out, non_blocking=True)
        self.end.record(stream)
        self.end.synchronize()
        return self.out_host[:b].numpy(), self.start.elapsed_time(self.end)

    def run_passes(self, passes: Sequence[tuple[int, int, Sequence[tuple[int, int, Row]], Sequence[int]]]
                   ) -> list[tuple[np.ndarray, float]]:
        """Several passes (b, n, rows, prefix lengths) enqueued back to back on the current stream, with one wait at
        the end instead of one per pass: pass i's input is staged in pinned buffer i % 2 while pass i - 1 runs (after
        the copy that last read that buffer is done), its probabilities come back into a pinned buffer of its own.
        Every graph is recorded before the first pass is enqueued. Returns (probs (B, 255), ms) per pass, in order;
        ms is the device time from the pass's input copy to its output copy."""
        for b, n, _, _ in passes:
            self.graph(b, n)
        while len(self.pass_out) < len(passes):
            self.pass_out.append(torch.zeros(max(C.BATCH_BUCKETS), C.READOUT_ROWS, dtype=torch.float32).pin_memory())
            self.pass_events.append((torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)))
        stream = torch.cuda.current_stream(self.device)
        hosts = ((self.inp_host, self.inp_np), (self.inp_host2, self.inp_host2.numpy()))
        for i, (b, n, part, lengths) in enumerate(passes):
            graph, out = self.graph(b, n)
            host, host_np = hosts[i % 2]
            if i >= 2:
                self.in_copied[i % 2].synchronize()
            size = self.fill(b, n, part, lengths, host_np)
            start, end = self.pass_events[i]
            start.record(stream)
            self.inp[:size].copy_(host[:size], non_blocking=True)
            self.in_copied[i % 2].record(stream)
            graph.replay()
            self.pass_out[i][:b].copy_(out, non_blocking=True)
            end.record(stream)
        results = []
        for i, (b, _, _, _) in enumerate(passes):
            start, end = self.pass_events[i]
            end.synchronize()
            results.append((self.pass_out[i][:b].numpy(), start.elapsed_time(end)))
        return results

    def _check(self, rows: Sequence[tuple[int, int, Row]]) -> list[int]:
        loaded = set(self.fast.adapter_index.values())
        lengths = []
        for i, (adapter, slot, row) in enumerate(rows):
            if adapter not in loaded:
                raise ValueError(f"Row {i}: adapter row {adapter} holds no loaded adapter (loaded rows: "
                                 f"{sorted(loaded)})")
            if slot != 0 and self.pool.key(slot) != (adapter, row.prefix_text):
                raise ValueError(f"Row {i}: prefix slot {slot} holds another prefix than the row's under adapter row "
                                 f"{adapter} (it holds adapter row {self.pool.key(slot)[0]}'s)")
            if not 1 <= len(row.new_ids) <= max(C.NEW_BUCKETS):
                raise ValueError(f"Row {i}: {len(row.new_ids)} new tokens; the batched path takes 1 to "
                                 f"{max(C.NEW_BUCKETS)}")
            if not 1 <= row.count <= C.READOUT_ROWS:
                raise ValueError(f"Row {i}: {row.count} answer options; the readout has 1 to {C.READOUT_ROWS}")
            lengths.append(self.pool.length(slot))
        return lengths

    def decide(self, rows: Sequence[tuple[int, int, Row]]) -> tuple[list[list[float]], list[int], dict[str, Any]]:
        """Each row's option probabilities, input tokens (prefix + new) and timing (batched_path.py:528-562):
        rows (adapter row, prefix slot, Row) grouped by new-token bucket, passes of at most max_rows(N) rows in the
        smallest batch bucket that holds them; results in the rows' order."""
        lengths = self._check(rows)
        by_bucket: dict[int, list[int]] = {}
        for i, (_, _, row) in enumerate(rows):
            by_bucket.setdefault(next(b for b in C.NEW_BUCKETS if b >= len(row.new_ids)), []).append(i)
        results: list[list[float]] = [[] for _ in rows]
        batch_rows, bucket, adapters_in_pass = [0] * len(rows), [0] * len(rows), [0] * len(rows)
        timing: dict[str, Any] = {"model_ms": 0.0, "new_tokens": sum(len(r.new_ids) for _, _, r in rows), "passes": 0}
        plan: list[tuple[int, int, list[int]]] = []
        for n, members in sorted(by_bucket.items()):
            cap = min(max_rows(n), self.ws.rows, self.max_tokens // n)
            for first in range(0, len(members), cap):
                part = members[first:first + cap]
                plan.append((next(bb for bb in self.batch_buckets if bb >= len(part)), n, part))
        done = self.run_passes([(b, n, [rows[i] for i in part], [lengths[i] for i in part]) for b, n, part in plan])
        for (_, n, part), (probs, ms) in zip(plan, done, strict=True):
            timing["model_ms"] += ms
            timing["passes"] += 1
            adapters = len({rows[i][0] for i in part})
            for j, i in enumerate(part):
                results[i] = probs[j, :rows[i][2].count].tolist()
                batch_rows[i], bucket[i], adapters_in_pass[i] = len(part), n, adapters
        timing.update(batch_rows=batch_rows, bucket=bucket, adapters_in_pass=adapters_in_pass)
        tokens = [lengths[i] + len(row.new_ids) for i, (_, _, row) in enumerate(rows)]
        return results, tokens, timing

    # ------------------------------------------------------------ prefixes

    def prefix_passes(self, nb: int, count: int) -> list[int]:
        """The batch buckets of the passes for `count` new prefixes of bucket nb: largest recorded size first."""
        cap = min(PREFIX_PASS_ROWS[nb], self.max_tokens // nb, self.ws.rows)
        sizes = [b for b in C.BATCH_BUCKETS if b <= cap]
        out = []
        while count > 0:
            b = next((s for s in sorted(sizes, reverse=True) if s <= count), None)
            b = b if b is not None else min(s for s in sizes if s >= count)
            out.append(b)
            count -= b
        return out

    def _prefix_pass(self, b: int, nb: int, part: Sequence[tuple[int, int, list[int]]]) -> float:
        graph = self.prefix_graph(b, nb)
        self.pool.sync()
        w = self._prefix_width(nb)
        size = (PREFIX_META + w + nb) * b
        meta = self.prefix_inp_np[:PREFIX_META * b].reshape(PREFIX_META, b)
        pages = self.prefix_inp_np[PREFIX_META * b:(PREFIX_META + w) * b].reshape(b, w)
        ids = self.prefix_inp_np[(PREFIX_META + w) * b:size]
        meta[:] = 0
        pages[:] = SINK_PAGE
        ids[:] = 0
        for j, (slot, adapter, toks) in enumerate(part):
            table = self.pool.block_table(slot)
            if len(toks) > nb or len(table) != self.pool.shapes.pages_per_prefix(len(toks)):
                raise AssertionError(f"Slot {slot}: a prefix of {len(toks)} tokens with {len(table)} pages staged in a "
                                     f"pass of {nb}")
            pages[j, :len(table)] = table
            ids[j * nb:j * nb + len(toks)] = toks
            meta[:, j] = (adapter, len(toks))
        stream = torch.cuda.current_stream(self.device)
        self.start.record(stream)
        self.prefix_inp[:size].copy_(self.prefix_inp_host[:size], non_blocking=True)
        graph.replay()
        self.end.record(stream)
        self.end.synchronize()
        return self.start.elapsed_time(self.end)

    def ensure_prefixes(self, rows: Sequence[tuple[int, str]], max_tokens: int) -> tuple[list[int], dict[str, Any]]:
        """Each row's prefix slot (adapter row, prefix text), pinned once per row (the caller unpins the list), with
        the prefixes not yet in the pool processed by batched prefix passes (the reference's ensure_prefixes,
        batched_path.py:613-698, same checks, messages and timing keys). All or nothing: if anything fails, every pin
        taken here is returned and every reservation whose prefix pass did not run is released."""
        pool = self.pool
        loaded = set(self.fast.adapter_index.values())
        bad = next((i for i, (adapter, _) in enumerate(rows) if adapter not in loaded), None)
        if bad is not None:
            raise ValueError(f"Row {bad}: adapter row {rows[bad][0]} holds no loaded adapter (loaded rows: "
                             f"{sorted(loaded)})")
        # distinct keys in first-appearance order, each with the rows that use it
        users: dict[tuple[int, str], list[int]] = {}
        for i, key in enumerate(rows):
            users.setdefault(tuple(key), []).append(i)          # type: ignore[arg-type]
        cached = {key: slot for key in users if (slot := pool.lookup(*key)) is not None}
        tokens: dict[tuple[int, str], list[int]] = {}
        for key in users:
            if key in cached:
                continue
            if self.tokenize is None:
                raise ValueError("This batched path has no tokenizer to process new prefixes")
            ids = list(self.tokenize(key[1]))
            if len(ids) > C.LONGEST_PREFIX_TOKENS:
                raise ValueError(f"The question's fixed part has {len(ids)} tokens; the fast path holds at most "
                                 f"{C.LONGEST_PREFIX_TOKENS}")
            if len(ids) >= max_tokens:
                raise ValueError(f"Question branch exceeds the {max_tokens}-token limit; no input was truncated.")
            tokens[key] = ids
        timing: dict[str, Any] = dict(prefix_ms=0.0, prefix_misses=len(tokens),
                                      prefix_hits=sum(len(users[k]) for k in cached),
                                      prefix_shared=sum(len(users[k]) - 1 for k in tokens), prefix_passes=0)
        claim = _Claim(pool)
        with claim:
            # cached prefixes first, so that reserving the new ones cannot evict them
            for key, slot in cached.items():
                claim.pin(slot, len(users[key]))
            slot_of = dict(cached)
            for key, ids in tokens.items():
                slot_of[key] = claim.reserve(key, len(ids), len(users[key]))
            buckets: dict[int, list[tuple[int, str]]] = {}
            for key, ids in tokens.items():
                buckets.setdefault(next(nb for nb in C.PREFIX_BUCKETS if nb >= max(len(ids), 1)), []).append(key)
            for nb in sorted(buckets):
                queue = buckets[nb]
                for b in self.prefix_passes(nb, len(queue)):
                    batch, queue = queue[:b], queue[b:]
                    timing["prefix_ms"] += self._prefix_pass(b, nb, [(slot_of[k], k[0], tokens[k]) for k in batch])
                    timing["prefix_passes"] += 1
                    claim.written(slot_of[k] for k in batch)
        return [slot_of[tuple(key)] for key in rows], timing     # type: ignore[index]


class _Claim:
    """The pins and reservations one ensure_prefixes call takes, undone together if the call fails: its pins are
    returned and the reservations whose prefix pass never ran are released (their pages hold nothing)."""

    def __init__(self, pool: Any) -> None:
        self.pool = pool
        self.pins: list[int] = []
        self.unwritten: set[int] = set()

    def pin(self, slot: int, times: int) -> None:
        self.pool.pin([slot] * times)
        self.pins += [slot] * times

    def reserve(self, key: tuple[int, str], tokens: int, times: int) -> int:
        slot = self.pool.reserve(key[0], key[1], tokens)
        self.unwritten.add(slot)
        self.pin(slot, times)
        return slot

    def written(self, slots: Any) -> None:
        self.unwritten.difference_update(slots)

    def __enter__(self) -> _Claim:
        return self

    def __exit__(self, kind: Any, error: Any, tb: Any) -> bool:
        if kind is not None:
            self.pool.unpin(self.pins)
            for slot in self.unwritten:
                self.pool.release(slot)
        return False
