"""The hot path's operators as the reference's fast path calls them, each one call into libjeffb200 (no Triton, no
CPU fallback). Names, arguments and returns follow the reference's engine modules:

- int4_product (int4_kernels.py:132-177), lora_shrink (fast_path.py:159-177): the fused W4A16 + multi-LoRA product;
- add_rms, gated_norm, gate_mul, silu_mul (fast_path.py:80-156), rms_last (batched_path.py:274-275), embed;
- gdn_prep_rows, gdn_scan (batched_kernels.py:89-261 and fla's chunk kernel), attn_prep_rows, paged_attention,
  kv_scatter (batched_kernels.py:302-486, batched_path.py:345-349), readout_rows (batched_kernels.py:492-559).

Every function launches on the current torch stream and allocates its outputs only when no `out` is given (the
recorded passes pass preallocated buffers, so graphs capture no allocation)."""

from __future__ import annotations

import torch

from jeff_b200 import _lib
from jeff_b200 import constants as C
from jeff_b200._lib import ptr, stream_ptr

DT = torch.bfloat16


def _check(t: torch.Tensor, name: str, dtype: torch.dtype, shape: tuple[int, ...] | None = None) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name}: expected a CUDA tensor, got one on {t.device}")
    if t.dtype != dtype:
        raise ValueError(f"{name}: expected {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name}: expected a contiguous tensor, got strides {t.stride()}")
    if shape is not None and tuple(t.shape) != shape:
        raise ValueError(f"{name}: expected shape {shape}, got {tuple(t.shape)}")


def _pass_rows(t: int, n: int) -> int:
    if n % 32 or t % n:
        raise ValueError(f"A pass of {t} tokens in rows of {n}: rows must be a multiple of 32 tokens, and the pass "
                         "whole rows")
    return t // n


# ---------------------------------------------------------------- int4 products


def int4_repack(words: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """The reference's kernel word layout -> this library's kernel layout (jb_int4_repack), on the device."""
    out = out if out is not None else torch.empty_like(words)
    _lib.call("jb_int4_repack", ptr(words), ptr(out), words.shape[0] * 8, words.shape[1], stream_ptr())
    return out


def int4_dequant(words: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor | None, group: int) -> torch.Tensor:
    """The packed group (kernel-layout words) dequantised on the device: (columns, k) bf16."""
    k, columns = words.shape[0] * 8, words.shape[1]
    out = torch.empty(columns, k, dtype=DT, device=words.device)
    _lib.call("jb_int4_dequant", ptr(words), ptr(scales), ptr(zeros), k, columns, group, ptr(out), stream_ptr())
    return out


def lora_shrink(x: torch.Tensor, lora_a: torch.Tensor, adapters: torch.Tensor, row_len: int,
                out: torch.Tensor | None = None) -> torch.Tensor:
    m, k = x.shape
    rank = lora_a.shape[1]
    mid = out if out is not None else torch.empty(m, rank, dtype=DT, device=x.device)
    _lib.call("jb_lora_shrink", ptr(x), m, k, ptr(lora_a), rank, lora_a.shape[0], ptr(adapters), row_len, ptr(mid),
              stream_ptr())
    return mid


def int4_product(x: torch.Tensor, words: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor | None, group: int,
                 out_features: int, lora_a: torch.Tensor | None, lora_b: torch.Tensor | None,
                 adapters: torch.Tensor | None, row_len: int, mid: torch.Tensor | None = None,
                 y: torch.Tensor | None = None, swiglu: bool = False, tmem_a: bool = False,
                 split: tuple[torch.Tensor, torch.Tensor] | None = None) -> torch.Tensor:
    """y (m, out) = bf16(x W^T + bf16(x A[a]^T) B[a]^T) for row a = adapters[t // row_len] of token t: the fused
    product of one group (module docstring); `words` in the kernel layout (int4_repack). lora_a (rows, R, k),
    lora_b (rows, columns, R) bf16, or None. swiglu: the group's columns are gate|up blocks of 64 and y (m, out / 2)
    receives bf16(bf16(silu(g)) u) (fast_path.silu_mul fused into the epilogue). tmem_a: the tensor-memory form of
    the product kernel (weights dequantised into tensor memory as the MMA's A operand; the same bits, measured
    slower), for rows of a multiple of 128 tokens. split (fp32 slices, int32 counters, the counters zero): the
    split-K form (jb_int4_lora_product_split), which the library uses when the pass's tiles are fewer than the SMs;
    the same result up to the order of the fp32 sums."""
    m, k = x.shape
    columns = words.shape[1]
    if words.shape[0] * 8 != k:
        raise ValueError(f"int4_product: x has {k} inputs, the weights {words.shape[0] * 8}")
    rank = 0 if lora_a is None else lora_a.shape[1]
    if y is None:
        y = torch.empty(m, out_features // 2 if swiglu else out_features, dtype=DT, device=x.device)
    if rank and mid is None:
        mid = torch.empty(m, rank, dtype=DT, device=x.device)
    args = (ptr(x), m, k, ptr(words), ptr(scales), ptr(zeros), group, columns, out_features, ptr(lora_a), ptr(lora_b),
            rank, 0 if lora_a is None else lora_a.shape[0], ptr(adapters), row_len, ptr(mid) if rank else None, ptr(y),
            y.stride(0), (1 if swiglu else 0) | (2 if tmem_a else 0))
    if split is None:
        _lib.call("jb_int4_lora_product", *args, stream_ptr())
    else:
        parts, counters = split
        _check(parts, "split partials", torch.float32)
        _check(counters, "split counters", torch.int32)
        _lib.call("jb_int4_lora_product_split", *args, ptr(parts), parts.numel(), ptr(counters), counters.numel(),
                  stream_ptr())
    return y


def w4a16_small(x: torch.Tensor, words: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor | None, group: int,
                out_features: int, mid: torch.Tensor | None, lora_b: torch.Tensor | None,
                adapters: torch.Tensor | None, row_len: int, split: int = 0, swiglu: bool = False,
                y: torch.Tensor | None = None) -> torch.Tensor:
    """The weight-streaming product for passes of at most 64 tokens in at most two LoRA rows (jb_w4a16_lora_small):
    y = bf16(x W^T + mid B[a]^T), mid the LoRA first factor (m, R) already computed (or None). split: K slices per
    128-column tile, one thread-block cluster (0: the library's choice)."""
    m, k = x.shape
    columns = words.shape[1]
    rank = 0 if mid is None else mid.shape[1]
    if y is None:
        y = torch.empty(m, out_features // 2 if swiglu else out_features, dtype=DT, device=x.device)
    _lib.call("jb_w4a16_lora_small", ptr(x), m, k, ptr(words), ptr(scales), ptr(zeros), group, columns, out_features,
              ptr(mid), ptr(lora_b), rank, 0 if lora_b is None else lora_b.shape[0], ptr(adapters), row_len, ptr(y),
              y.stride(0), 1 if swiglu else 0, split, stream_ptr())
    return y


# ---------------------------------------------------------------- norms and activations


def add_rms(x: torch.Tensor, d: torch.Tensor | None, w1: torch.Tensor, xo: torch.Tensor | None = None,
            h: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """(x + d, rms(x + d) * w1), w1 = 1 + weight float32 (fast_path.add_rms)."""
    rows, n = x.shape
    h = h if h is not None else torch.empty_like(x)
    if d is not None:
        xo = xo if xo is not None else torch.empty_like(x)
    else:
        xo = x
    _lib.call("jb_add_rms", ptr(x), ptr(d), ptr(w1), ptr(xo), ptr(h), rows, n, stream_ptr())
    return xo, h


def rms_last(x: torch.Tensor, d: torch.Tensor, last: torch.Tensor, row_len: int, w1: torch.Tensor,
             out: torch.Tensor | None = None) -> torch.Tensor:
    b = x.shape[0] // row_len
    hidden = out if out is not None else torch.empty(b, x.shape[1], dtype=DT, device=x.device)
    _lib.call("jb_rms_last", ptr(x), ptr(d), ptr(last), b, row_len, x.shape[1], ptr(w1), ptr(hidden), stream_ptr())
    return hidden


def embed(table: torch.Tensor, ids: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    t = ids.shape[0]
    x = out if out is not None else torch.empty(t, table.shape[1], dtype=DT, device=table.device)
    _lib.call("jb_embed", ptr(table), table.shape[0], table.shape[1], ptr(ids), t, ptr(x), stream_ptr())
    return x


def silu_mul(gu: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    rows = gu.shape[0]
    y = out if out is not None else torch.empty(rows, C.INTER, dtype=DT, device=gu.device)
    _lib.call("jb_silu_mul", ptr(gu), gu.stride(0), C.INTER, ptr(y), rows, stream_ptr())
    return y


def gate_mul(o: torch.Tensor, pr: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    rows = pr.shape[0]
    y = out if out is not None else torch.empty(rows, C.NQ * C.HD, dtype=DT, device=o.device)
    _lib.call("jb_gate_mul", ptr(o), ptr(pr), pr.stride(0), ptr(y), rows, stream_ptr())
    return y


def gated_norm(o: torch.Tensor, pr: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    rows = pr.shape[0]
    y = out if out is not None else torch.empty(rows, C.NV * C.DV, dtype=DT, device=o.device)
    _lib.call("jb_gated_norm", ptr(o), ptr(pr), pr.stride(0), C.QKV_DIM, ptr(w), ptr(y), rows, stream_ptr())
    return y


def readout_rows(hidden: torch.Tensor, readout_pool: torch.Tensor, temp_pool: torch.Tensor, adapters: torch.Tensor,
                 counts: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Each row's option probabilities (B, 255) fp32 (batched_kernels.readout_rows)."""
    b = hidden.shape[0]
    if temp_pool.dim() != 1 or temp_pool.dtype != torch.float32 or not temp_pool.is_contiguous():
        raise ValueError(f"readout_rows: temp_pool must be a contiguous float32 vector (one temperature per adapter "
                         f"row), got shape {tuple(temp_pool.shape)}, {temp_pool.dtype}")
    if readout_pool.shape[1:] != (C.READOUT_ROWS, C.HIDDEN) or not readout_pool.is_contiguous():
        raise ValueError(f"readout_rows: expected a contiguous readout_pool (adapters + 1, {C.READOUT_ROWS}, "
                         f"{C.HIDDEN}), got {tuple(readout_pool.shape)}")
    probs = out if out is not None else torch.empty(b, C.READOUT_ROWS, dtype=torch.float32, device=hidden.device)
    _lib.call("jb_readout_rows", ptr(hidden), ptr(readout_pool), readout_pool.shape[0], ptr(temp_pool), ptr(adapters),
              ptr(counts), b, ptr(probs), stream_ptr())
    return probs


# ---------------------------------------------------------------- Gated DeltaNet


def gdn_prep_rows(pr: torch.Tensor, pool, tables: torch.Tensor, gdn_layer: int, conv_w: torch.Tensor,
                  a_neg: torch.Tensor, dt_bias: torch.Tensor, n: int, real: torch.Tensor | None = None,
                  out_tables: torch.Tensor | None = None, outs: tuple | None = None) -> tuple[torch.Tensor, ...]:
    """q, k, v (B, n, 16, 128) bf16, g (B, n, 16) fp32, beta (B, n, 16) bf16 (batched_kernels.gdn_prep_rows).
    With real and out_tables (the prefix pass): padding tokens get g = beta = 0 and each row's conv tail goes to its
    output pages."""
    t = pr.shape[0]
    b = _pass_rows(t, n)
    shapes = pool.shapes
    if tables.dim() != 2 or tables.shape[0] < b or tables.shape[1] < shapes.fixed_pages or tables.dtype != torch.int32:
        raise ValueError(f"tables: expected int32 (rows >= {b}, width >= {shapes.fixed_pages}), got "
                         f"{tuple(tables.shape)} {tables.dtype}")
    if conv_w.shape != (4, C.QKV_DIM) or conv_w.dtype != torch.float32 or not conv_w.is_contiguous():
        raise ValueError(f"gdn_prep_rows: conv_w must be a contiguous float32 (4, {C.QKV_DIM}) tensor, got "
                         f"{tuple(conv_w.shape)}, {conv_w.dtype}")
    for name, vec in (("a", a_neg), ("dt_bias", dt_bias)):
        if vec.shape != (C.NV,) or vec.dtype != torch.float32 or not vec.is_contiguous():
            raise ValueError(f"{name}: expected a contiguous torch.float32 vector of {C.NV} entries, got shape "
                             f"{tuple(vec.shape)}, {vec.dtype}")
    dev = pr.device
    if outs is None:
        q = torch.empty(b, n, C.NV, C.DK, dtype=DT, device=dev)
        outs = (q, torch.empty_like(q), torch.empty_like(q), torch.empty(b, n, C.NV, dtype=torch.float32, device=dev),
                torch.empty(b, n, C.NV, dtype=DT, device=dev))
    q, k, v, g, beta = outs
    per = shapes.layers_per_conv_page
    _lib.call("jb_gdn_prep_rows", ptr(pr), pr.stride(0), t, n, ptr(pool.data), shapes.page_bytes, ptr(tables),
              tables.stride(0), shapes.state_pages + gdn_layer // per, gdn_layer % per, ptr(conv_w), ptr(a_neg),
              ptr(dt_bias), ptr(q), ptr(k), ptr(v), ptr(g), ptr(beta), ptr(real), ptr(out_tables),
              0 if out_tables is None else out_tables.stride(0), stream_ptr())
    return q, k, v, g, beta


def gdn_scan(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor, pool,
             tables: torch.Tensor, gdn_layer: int, last: torch.Tensor | None = None,
             out_tables: torch.Tensor | None = None, out: torch.Tensor | None = None,
             kernel: str = "tc") -> torch.Tensor:
    """The gated delta rule from each row's pooled state; o (B, n, 16, 128). kernel "tc" (64-token chunks, every
    chunk product a tcgen05 MMA with the state in tensor memory: fla's chunk_gated_delta_rule), "chunk" (the same
    chunks on mma.sync, the form the fused jb_gdn_layer shares bit for bit) or "recurrent" (token by token,
    batched_kernels.gdn_recurrent_slots)."""
    b, n = q.shape[:2]
    shapes = pool.shapes
    if tables.dim() != 2 or tables.shape[0] < b or tables.shape[1] < shapes.fixed_pages or tables.dtype != torch.int32:
        raise ValueError(f"tables: expected int32 (rows >= {b}, width >= {shapes.fixed_pages}), got "
                         f"{tuple(tables.shape)} {tables.dtype}")
    for name, x in (("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta)):
        if not x.is_contiguous():
            raise ValueError(f"gdn_scan: {name} must be contiguous")
    o = out if out is not None else torch.empty_like(v)
    name = {"tc": "jb_gdn_scan_tc", "chunk": "jb_gdn_scan", "recurrent": "jb_gdn_scan_recurrent"}[kernel]
    _lib.call(name, ptr(q), ptr(k), ptr(v), ptr(g), ptr(beta), ptr(o), b, n, ptr(pool.data),
              shapes.page_bytes, ptr(tables), tables.stride(0), shapes.state[0] * gdn_layer, shapes.heads_per_page,
              ptr(last), ptr(out_tables), 0 if out_tables is None else out_tables.stride(0), stream_ptr())
    return o


def gdn_layer(pr: torch.Tensor, pool, tables: torch.Tensor, gdn_layer: int, conv_w: torch.Tensor,
              a_neg: torch.Tensor, dt_bias: torch.Tensor, gnorm_w: torch.Tensor, n: int,
              last: torch.Tensor | None = None, real: torch.Tensor | None = None,
              out_tables: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """A Gated DeltaNet layer's mixer in one launch (gdn_prep_rows, the chunked rule and gated_norm fused): y
    (t, 2048) bf16 from the in_proj output pr (t, 8224), each row resuming from its pooled state and conv tail.
    last: the decision pass's last real token per row; real + out_tables: the prefix pass."""
    t = pr.shape[0]
    _pass_rows(t, n)
    shapes = pool.shapes
    if tables.dim() != 2 or tables.shape[0] < t // n or tables.shape[1] < shapes.fixed_pages or \
            tables.dtype != torch.int32:
        raise ValueError(f"tables: expected int32 (rows >= {t // n}, width >= {shapes.fixed_pages}), got "
                         f"{tuple(tables.shape)} {tables.dtype}")
    if conv_w.shape != (4, C.QKV_DIM) or conv_w.dtype != torch.float32 or not conv_w.is_contiguous():
        raise ValueError(f"gdn_layer: conv_w must be a contiguous float32 (4, {C.QKV_DIM}) tensor, got "
                         f"{tuple(conv_w.shape)}, {conv_w.dtype}")
    if gnorm_w.shape != (C.DV,) or gnorm_w.dtype != DT or not gnorm_w.is_contiguous():
        raise ValueError(f"gdn_layer: gnorm_w must be a contiguous bf16 ({C.DV},) vector")
    if pr.stride(1) != 1 or pr.shape[1] < C.GDN_PROJ:
        raise ValueError(f"gdn_layer: pr must be row-major with at least {C.GDN_PROJ} columns")
    y = out if out is not None else torch.empty(t, C.NV * C.DV, dtype=DT, device=pr.device)
    if y.stride(1) != 1 or y.shape[1] < C.NV * C.DV:
        raise ValueError("gdn_layer: out must be row-major with at least 2048 columns")
    per = shapes.layers_per_conv_page
    _lib.call("jb_gdn_layer", ptr(pr), pr.stride(0), t, n, ptr(pool.data), shapes.page_bytes, ptr(tables),
              tables.stride(0), shapes.state[0] * gdn_layer, shapes.heads_per_page, shapes.state_pages + gdn_layer // per,
              gdn_layer % per, ptr(conv_w), ptr(a_neg), ptr(dt_bias), ptr(gnorm_w), ptr(y), y.stride(0), ptr(last),
              ptr(real), ptr(out_tables), 0 if out_tables is None else out_tables.stride(0), stream_ptr())
    return y


# ---------------------------------------------------------------- attention


def attn_prep_rows(pr: torch.Tensor, q_w1: torch.Tensor, k_w1: torch.Tensor, inv_freq: torch.Tensor,
                   pos: torch.Tensor, kn: torch.Tensor, vn: torch.Tensor, n: int,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    t = pr.shape[0]
    _pass_rows(t, n)
    for name, x in (("kn", kn), ("vn", vn)):
        if tuple(x.shape) != (t, C.NKV, C.HD) or not x.is_contiguous():
            raise ValueError(f"attn_prep_rows: {name} must be a contiguous ({t}, {C.NKV}, {C.HD}) tensor")
    q = out if out is not None else torch.empty(t, C.NQ, C.HD, dtype=DT, device=pr.device)
    _lib.call("jb_attn_prep_rows", ptr(pr), pr.stride(0), t, n, ptr(q_w1), ptr(k_w1), ptr(inv_freq), ptr(pos), ptr(q),
              ptr(kn), ptr(vn), stream_ptr())
    return q


def paged_attention(q: torch.Tensor, pool, tables: torch.Tensor, attn_layer: int, pos: torch.Tensor,
                    kn: torch.Tensor, vn: torch.Tensor, n: int, out: torch.Tensor | None = None) -> torch.Tensor:
    t = q.shape[0]
    b = _pass_rows(t, n)
    width = pool.fixed_pages + pool.max_kv_pages
    if tables.dim() != 2 or tables.shape[0] < b or tables.shape[1] < width or tables.dtype != torch.int32:
        raise ValueError(f"tables: expected int32 (rows >= {b}, width >= {width}), got {tuple(tables.shape)} "
                         f"{tables.dtype}")
    for name, x in (("q", q), ("kn", kn), ("vn", vn)):
        if not x.is_contiguous():
            raise ValueError(f"paged_attention: {name} must be contiguous")
    o = out if out is not None else torch.empty(t, C.NQ, C.HD, dtype=DT, device=q.device)
    _lib.call("jb_paged_attention", ptr(q), ptr(pool.data), pool.shapes.page_bytes, ptr(tables), tables.stride(0),
              pool.fixed_pages, attn_layer, pool.shapes.attn_layers, ptr(pos), ptr(kn), ptr(vn), ptr(o), b, n,
              stream_ptr())
    return o


def paged_attention_gated(q: torch.Tensor, pool, tables: torch.Tensor, attn_layer: int, pos: torch.Tensor,
                          kn: torch.Tensor, vn: torch.Tensor, n: int, pr: torch.Tensor,
                          out: torch.Tensor | None = None, scratch: torch.Tensor | None = None) -> torch.Tensor:
    """Paged prefix-KV attention on tcgen05 with the output gate fused (paged_attention then gate_mul in one launch):
    y (t, 2048) bf16 = bf16(bf16(attention) * bf16(sigmoid(gate))), the gate half of each head's q_proj output in
    pr. scratch (fp32): the split walk's (jb_paged_attention_gated_split), which passes too small to fill the GPU
    spread over more CTAs."""
    t = q.shape[0]
    b = _pass_rows(t, n)
    width = pool.fixed_pages + pool.max_kv_pages
    if tables.dim() != 2 or tables.shape[0] < b or tables.shape[1] < width or tables.dtype != torch.int32:
        raise ValueError(f"tables: expected int32 (rows >= {b}, width >= {width}), got {tuple(tables.shape)} "
                         f"{tables.dtype}")
    for name, x in (("q", q), ("kn", kn), ("vn", vn)):
        if not x.is_contiguous():
            raise ValueError(f"paged_attention_gated: {name} must be contiguous")
    y = out if out is not None else torch.empty(t, C.NQ * C.HD, dtype=DT, device=q.device)
    args = (ptr(q), ptr(pool.data), pool.pages, pool.shapes.page_bytes, ptr(tables), tables.stride(0),
            pool.fixed_pages, attn_layer, pool.shapes.attn_layers, ptr(pos), ptr(kn), ptr(vn), ptr(pr), pr.stride(0),
            ptr(y), y.stride(0), b, n)
    if scratch is None:
        _lib.call("jb_paged_attention_gated", *args, stream_ptr())
    else:
        _check(scratch, "attention scratch", torch.float32)
        _lib.call("jb_paged_attention_gated_split", *args, ptr(scratch), scratch.numel(), stream_ptr())
    return y


def kv_scatter(kn: torch.Tensor, vn: torch.Tensor, n: int, real: torch.Tensor, pool, out_tables: torch.Tensor,
               attn_layer: int) -> None:
    b = kn.shape[0] // n
    _lib.call("jb_kv_scatter", ptr(kn), ptr(vn), b, n, ptr(real), ptr(pool.data), pool.shapes.page_bytes,
              ptr(out_tables), out_tables.stride(0), pool.fixed_pages, attn_layer, pool.shapes.attn_layers,
              stream_ptr())
