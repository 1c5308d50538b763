"""Each CUDA kernel of the hot path against the CPU oracle on the same seeded inputs (B200 only), in passes of
B = 1, 3 and 16 rows whose prefixes have mixed lengths (0, and lengths that are not multiples of 32), read through
block tables from a real prefix pool whose pages hold NaN past each prefix's end, so a read out of bounds shows up.

Tolerances follow the reference's kernel tests (runtime/python/tests/test_batched_kernels.py) and are stated per test:
one bfloat16 step is 2^-7 of the value at most; references that round the same values can land a step apart when
their float32 sums differ in the last bits. Integer work (unpack, dequantise) is bit-exact."""

from __future__ import annotations

import math
import random

import numpy as np
import pytest
import torch

from jeff_b200 import constants as C
from jeff_b200 import int4 as prod_int4
from jeff_b200 import kernels, synthetic
from jeff_b200.prefix_pool import PrefixPool
from oracle import int4_ref, model_ref

pytestmark = pytest.mark.gpu

BF16_STEP = 2.0 ** -7
PREFIX_LENGTHS = (0, 1, 7, 31, 32, 33, 45, 64, 100, 257, 513, 1000)
BATCHES = (1, 3, 16)


def bf(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).float()


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.fixture(scope="module")
def pool_fixture():
    """A pool with one random prefix per length (NaN past each prefix's end in its last key/value page), and the
    CPU copies of every prefix's state."""
    torch.manual_seed(0)
    pool = PrefixPool(2 + 60 * len(PREFIX_LENGTHS) + 600, "cuda")
    shapes = pool.shapes
    slots, states = {}, {}
    for i, p in enumerate(PREFIX_LENGTHS):
        slot = pool.reserve(1, f"prefix {i}", p)
        padded = math.ceil(p / 32) * 32
        kv = torch.randn(shapes.attn_layers, 2, padded, *shapes.kv).to(torch.bfloat16)
        kv[:, :, p:] = float("nan")
        conv = torch.randn(shapes.gdn_layers, *shapes.conv).to(torch.bfloat16)
        state = 0.5 * torch.randn(shapes.gdn_layers, *shapes.state)
        pool.write(slot, conv.cuda(), state.cuda(), kv.cuda())
        # write() pads partial pages with zeros: poison the tail of the last page explicitly
        if p % 32:
            table = pool.block_table(slot)
            last_page = table[shapes.fixed_pages + p // 32]
            pool.kv[last_page, :, :, p % 32:] = float("nan")
        slots[p] = slot
        states[slot] = (conv, state, kv[:, :, :p])
    states[0] = (torch.zeros(shapes.gdn_layers, *shapes.conv), torch.zeros(shapes.gdn_layers, *shapes.state),
                 torch.zeros(shapes.attn_layers, 2, 0, *shapes.kv))
    # pinned for the module: a test's own reservations must never evict them (they fail instead when pages run out)
    pool.pin(list(slots.values()))
    return pool, slots, states


def pass_slots(slots: dict[int, int], b: int, seed: int) -> list[int]:
    if b == 1:
        return [slots[33]]
    must = [0, slots[0], slots[33], slots[32], slots[1000]]
    rng = random.Random(seed)
    every = [0, *slots.values()]
    chosen = (must + [rng.choice(every) for _ in range(b)])[:b]
    rng.shuffle(chosen)
    return chosen


def tables_for(pool: PrefixPool, slots: list[int]) -> tuple[torch.Tensor, torch.Tensor]:
    idx = torch.tensor(slots, device="cuda")
    tables = pool.tables.index_select(0, idx).contiguous()
    pos = torch.tensor([pool.length(s) for s in slots], device="cuda", dtype=torch.int32)
    return tables, pos


# ---------------------------------------------------------------- int4


def test_int4_repack_permutes_nibbles() -> None:
    """The kernel word layout: input j of each word in nibble slot (j >> 1) + 4 (j & 1)."""
    words = torch.tensor([[0x76543210, -0x10000000]], dtype=torch.int32)
    got = kernels.int4_repack(words.cuda()).cpu()
    assert int(got[0, 0]) & 0xFFFFFFFF == 0x75316420
    assert int(got[0, 1]) & 0xFFFFFFFF == 0xF0000000


@pytest.mark.parametrize("fmt", ["g64", "g128z"])
def test_int4_dequant_is_bit_exact(fmt: str) -> None:
    w = synthetic.normal(7, f"dq/{fmt}", (330, 512), 0.02)
    packed, _ = prod_int4.quantize_pack(w, fmt)
    dev = packed.to("cuda")
    got = kernels.int4_dequant(kernels.int4_repack(dev.words), dev.scales, dev.zeros, packed.group)
    zb = None if packed.zeros is None else bits(packed.zeros)
    want = int4_ref.dequantize_kernel_layout(packed.words.numpy(), bits(packed.scales), zb, packed.group)
    assert np.array_equal(bits(got), want)


def exact_product(x: torch.Tensor, W: torch.Tensor, a_rows, b_rows, row_of: torch.Tensor):
    """float64 exact x W^T + bf16(x A^T) B^T per row, and the forward-error bound of a product rounded once
    (one bf16 step of the result, the float32 accumulation slack over k + rank terms, the mid's bf16 rounding)."""
    xd = x.double()
    exact = xd @ W.double().T
    mag = xd.abs() @ W.double().abs().T
    lora_round = torch.zeros_like(exact)
    for r in torch.unique(row_of).tolist():
        sel = row_of == r
        a, b = a_rows[r].double(), b_rows[r].double()
        mid = xd[sel] @ a.T
        exact[sel] += bf(mid.float()).double() @ b.T
        mag[sel] += (xd[sel].abs() @ a.abs().T) @ b.abs().T
        lora_round[sel] = 2.0 ** -9 * (mid.abs() @ b.abs().T)
    k = x.shape[1] + a_rows[0].shape[0]
    _, e = torch.frexp(exact.abs())
    step = torch.where(exact == 0, torch.zeros_like(exact), torch.ldexp(torch.ones_like(exact), e - 8))
    return exact, step + k * 2.0 ** -23 * mag + lora_round


@pytest.mark.parametrize("fmt", ["g128z", "g64"])
@pytest.mark.parametrize(("m", "k", "outs", "row_len"), [
    (64, 1024, [3584], 64),                       # configuration 1
    (128, 1024, [6144, 2048, 16, 16], 32),        # the Gated DeltaNet projection, 4 adapters per tile
    (256, 1024, [4096, 512, 512], 128),           # the attention projection (q+gate, k, v)
    (192, 2048, [1024], 64),                      # out_proj, ragged M (not a multiple of 128)
    (96, 3584, [1024], 32),                       # down_proj, k = 3584
    (2048, 1024, [3584], 128),                    # many tiles per persistent CTA
    (384, 1024, [1024], 128),                     # a tile whose second 128-row half lies past m
    (300, 1024, [2048], 1),                       # one adapter id per token: every adapter of the pool in a tile
    (288, 2048, [1024, 512], 48),                 # rows of 48 tokens: tiles and halves that span rows
])
def test_int4_lora_product_within_its_error_bound(fmt: str, m: int, k: int, outs: list[int], row_len: int) -> None:
    g = torch.Generator().manual_seed(m + k + len(outs))
    w = torch.randn(sum(outs), k, generator=g) * 0.02
    packed, W = prod_int4.quantize_pack(w, fmt)
    rank = 16 * min(len(outs), 3)
    rows = m // row_len
    pool_rows = 5
    a_pool = (torch.randn(pool_rows, rank, k, generator=g) * 0.02).to(torch.bfloat16)
    b_pool = torch.zeros(pool_rows, packed.columns, rank, dtype=torch.bfloat16)
    b_pool[:, :sum(outs)] = (torch.randn(pool_rows, sum(outs), rank, generator=g) * 0.02).to(torch.bfloat16)
    a_pool[0] = 0
    b_pool[0] = 0
    adapters = torch.randint(0, pool_rows, (rows,), generator=g, dtype=torch.int32)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    dev = packed.to("cuda")
    dev = prod_int4.PackedInt4(kernels.int4_repack(dev.words), dev.scales, dev.zeros, dev.group, dev.out)
    got = kernels.int4_product(x.cuda(), dev.words, dev.scales, dev.zeros, packed.group, sum(outs), a_pool.cuda(),
                               b_pool.cuda(), adapters.cuda(), row_len).cpu()
    row_of = adapters.long().repeat_interleave(row_len)
    exact, bound = exact_product(x.float(), W.float(), a_pool.float(), b_pool[:, :sum(outs)].float(), row_of)
    err = (got.double() - exact).abs()
    assert int((err > bound).sum()) == 0, f"worst at {(err / bound.clamp_min(1e-30)).max():.3g} x the bound"
    # and the same bits on a second run (no atomics: deterministic)
    again = kernels.int4_product(x.cuda(), dev.words, dev.scales, dev.zeros, packed.group, sum(outs), a_pool.cuda(),
                                 b_pool.cuda(), adapters.cuda(), row_len).cpu()
    assert torch.equal(got, again)


@pytest.mark.parametrize(("m", "k", "outs", "row_len"), [
    (32, 1024, [6144, 2048, 16, 16], 32),         # the Gated DeltaNet projection of a batch-1 pass (32 tokens)
    (32, 2048, [1024], 32),                       # out_proj: 8 tiles, K split 16 ways
    (32, 3584, [1024], 32),                       # down_proj, K = 3584
    (40, 1024, [4096, 512, 512], 8),              # ragged m, an adapter per 8 tokens
    (128, 1024, [3584], 32),                      # four batch-1 rows
    (512, 1024, [2048], 128),                     # two row tiles
])
def test_split_k_product_within_its_error_bound(m: int, k: int, outs: list[int], row_len: int) -> None:
    """jb_int4_lora_product_split: every output within the product's forward-error bound (the slices' fp32 sums in
    another order are covered by the same accumulation slack), the same bits on a second run, the tile counters
    back at zero, and within the bound of the unsplit product's result too."""
    g = torch.Generator().manual_seed(7 * m + k)
    w = torch.randn(sum(outs), k, generator=g) * 0.02
    packed, W = prod_int4.quantize_pack(w, "g128z")
    rank = 16 * min(len(outs), 3)
    pool_rows = 5
    a_pool = (torch.randn(pool_rows, rank, k, generator=g) * 0.02).to(torch.bfloat16)
    b_pool = torch.zeros(pool_rows, packed.columns, rank, dtype=torch.bfloat16)
    b_pool[:, :sum(outs)] = (torch.randn(pool_rows, sum(outs), rank, generator=g) * 0.02).to(torch.bfloat16)
    a_pool[0] = 0
    b_pool[0] = 0
    adapters = torch.randint(0, pool_rows, ((m + row_len - 1) // row_len,), generator=g, dtype=torch.int32)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    dev = packed.to("cuda")
    dev = prod_int4.PackedInt4(kernels.int4_repack(dev.words), dev.scales, dev.zeros, dev.group, dev.out)
    split = (torch.empty(4 * 2**20, dtype=torch.float32, device="cuda"),
             torch.zeros(1024, dtype=torch.int32, device="cuda"))
    args = (x.cuda(), dev.words, dev.scales, dev.zeros, packed.group, sum(outs), a_pool.cuda(), b_pool.cuda(),
            adapters.cuda(), row_len)
    got = kernels.int4_product(*args, split=split).cpu()
    row_of = adapters.long().repeat_interleave(row_len)[:m]
    exact, bound = exact_product(x.float(), W.float(), a_pool.float(), b_pool[:, :sum(outs)].float(), row_of)
    err = (got.double() - exact).abs()
    assert int((err > bound).sum()) == 0, f"worst at {(err / bound.clamp_min(1e-30)).max():.3g} x the bound"
    assert torch.equal(kernels.int4_product(*args, split=split).cpu(), got)
    assert not split[1].any()
    plain = kernels.int4_product(*args).cpu()
    assert int(((plain.double() - exact).abs() > bound).sum()) == 0


@pytest.mark.parametrize("m,k,outs,row_len,rank,split,fmt", [
    (1, 1024, [3584], 1, 16, 0, "g128z"),                     # one token, the library's choice of slices
    (16, 1024, [6144, 2048, 16, 16], 16, 48, 4, "g128z"),     # in_proj-like group, ragged last tile
    (32, 2048, [1024], 32, 16, 8, "g128z"),                   # out_proj, eight slices
    (32, 3584, [1024], 16, 32, 8, "g64"),                     # down_proj, two rows of two adapters, symmetric g64
    (16, 256, [1024], 16, 16, 1, "g128z"),                    # one slice: the persistent kernel's sums and order
    (64, 1024, [4096, 512, 512], 32, 16, 2, "g128z"),         # two rows of 32 tokens, two slices
    (40, 1024, [2048], 8, 0, 0, "g128z"),                     # no LoRA (ragged 48-token box)
])
def test_small_product_within_its_error_bound(m: int, k: int, outs: list[int], row_len: int, rank: int, split: int,
                                              fmt: str) -> None:
    """jb_w4a16_lora_small against the float64 product: every output within the product's forward-error bound and
    the same bits on a second run; with one slice, the same bits as the persistent kernel (jb_w4a16_lora: the same
    sums in the same K order)."""
    g = torch.Generator().manual_seed(11 * m + k + split)
    w = torch.randn(sum(outs), k, generator=g) * 0.02
    packed, W = prod_int4.quantize_pack(w, fmt)
    pool_rows = 5
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    adapters = torch.randint(0, pool_rows, ((m + row_len - 1) // row_len,), generator=g, dtype=torch.int32)
    if rank:
        a_pool = (torch.randn(pool_rows, rank, k, generator=g) * 0.02).to(torch.bfloat16)
        b_pool = torch.zeros(pool_rows, packed.columns, rank, dtype=torch.bfloat16)
        b_pool[:, :sum(outs)] = (torch.randn(pool_rows, sum(outs), rank, generator=g) * 0.02).to(torch.bfloat16)
        a_pool[0] = 0
        b_pool[0] = 0
        row_of = adapters.long().repeat_interleave(row_len)[:m]
        mid = torch.einsum("tk,trk->tr", x.float(), a_pool.float()[row_of]).to(torch.bfloat16)
    dev = packed.to("cuda")
    words = kernels.int4_repack(dev.words)
    zeros = dev.zeros if fmt == "g128z" else None
    args = (x.cuda(), words, dev.scales, zeros, packed.group, sum(outs), mid.cuda() if rank else None,
            b_pool.cuda() if rank else None, adapters.cuda(), row_len)
    got = kernels.w4a16_small(*args, split=split).cpu()
    exact = x.double() @ W.double().T
    mag = x.double().abs() @ W.double().abs().T
    if rank:
        b_rows = b_pool.double()[row_of][:, :sum(outs)]
        exact += torch.einsum("tr,tnr->tn", mid.double(), b_rows)
        mag += torch.einsum("tr,tnr->tn", mid.double().abs(), b_rows.abs())
    # one bf16 rounding of the result, the fp32 accumulation slack over k + rank terms (mid is an exact input here)
    _, e = torch.frexp(exact.abs())
    step = torch.where(exact == 0, torch.zeros_like(exact), torch.ldexp(torch.ones_like(exact), e - 8))
    bound = step + (k + rank) * 2.0 ** -23 * mag
    err = (got.double() - exact).abs()
    assert int((err > bound).sum()) == 0, f"worst at {(err / bound.clamp_min(1e-30)).max():.3g} x the bound"
    assert torch.equal(kernels.w4a16_small(*args, split=split).cpu(), got)
    if split == 1:
        plain = torch.empty(m, sum(outs), dtype=torch.bfloat16, device="cuda")
        kernels._lib.call("jb_w4a16_lora", kernels.ptr(args[0]), m, k, kernels.ptr(words), kernels.ptr(dev.scales),
                          kernels.ptr(zeros), packed.group, words.shape[1], sum(outs), kernels.ptr(args[6]),
                          kernels.ptr(args[7]), rank, pool_rows, kernels.ptr(args[8]), row_len, kernels.ptr(plain),
                          plain.stride(0), 0, kernels.stream_ptr())
        assert torch.equal(plain.cpu(), got)


def test_small_product_refuses_what_it_cannot_hold() -> None:
    """Three LoRA rows, a split that leaves a slice a ragged token count, and a slice too big for shared memory are
    refused before any launch (the split entry sends such passes to the persistent kernel instead)."""
    x = torch.zeros(48, 3584, dtype=torch.bfloat16, device="cuda")
    words = torch.zeros(3584 // 8, 1024, dtype=torch.int32, device="cuda")
    scales = torch.ones(3584 // 128, 1024, dtype=torch.bfloat16, device="cuda")
    mid = torch.zeros(48, 16, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(2, 1024, 16, dtype=torch.bfloat16, device="cuda")
    adp = torch.zeros(3, dtype=torch.int32, device="cuda")
    with pytest.raises(kernels._lib.ArgumentError, match="LoRA rows"):
        kernels.w4a16_small(x, words, scales, None, 128, 1024, mid, b, adp, 16)
    with pytest.raises(kernels._lib.ArgumentError, match="multiple of 4"):
        kernels.w4a16_small(x, words, scales, None, 128, 1024, None, None, None, 48, split=8)
    with pytest.raises(kernels._lib.ArgumentError, match="shared memory"):
        kernels.w4a16_small(x, words, scales, None, 128, 1024, None, None, None, 48, split=1)


def test_split_k_product_swiglu_epilogue() -> None:
    """The SwiGLU epilogue after the slices are added: a gate/up group of 8 tiles (so the 32-token pass is sliced),
    as the unsplit product's test bounds it (four bf16 steps, 5e-4 absolute near zero)."""
    from jeff_b200.fast_path import swiglu_order

    g = torch.Generator().manual_seed(78)
    m, k, inter, row_len, rank, pool_rows = 32, 2048, 512, 32, 32, 3
    w = torch.randn(2 * inter, k, generator=g) * 0.02
    packed, W = prod_int4.quantize_pack(w, "g128z")
    order = swiglu_order(inter)
    a_pool = (torch.randn(pool_rows, rank, k, generator=g) * 0.02).to(torch.bfloat16)
    b_pool = (torch.randn(pool_rows, 2 * inter, rank, generator=g) * 0.02).to(torch.bfloat16)
    adapters = torch.randint(0, pool_rows, (m // row_len,), generator=g, dtype=torch.int32)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    words = kernels.int4_repack(packed.words[:, order].contiguous().cuda())
    split = (torch.empty(4 * 2**20, dtype=torch.float32, device="cuda"),
             torch.zeros(1024, dtype=torch.int32, device="cuda"))
    got = kernels.int4_product(x.cuda(), words, packed.scales[:, order].contiguous().cuda(),
                               packed.zeros[:, order].contiguous().cuda(), packed.group, 2 * inter, a_pool.cuda(),
                               b_pool[:, order].contiguous().cuda(), adapters.cuda(), row_len, swiglu=True,
                               split=split).cpu().float()
    row_of = adapters.long().repeat_interleave(row_len)
    exact, _ = exact_product(x.float(), W.float(), a_pool.float(), b_pool.float(), row_of)
    gu = bf(exact.float())
    gate, up = gu[:, :inter], gu[:, inter:]
    want = bf(bf(gate * torch.sigmoid(gate)) * up)      # silu_mul (fast_path.py:141-156) of this narrower group
    torch.testing.assert_close(got, want, rtol=4 * BF16_STEP, atol=5e-4)
    assert not split[1].any()


@pytest.mark.parametrize("fmt", ["g128z", "g64"])
def test_int4_lora_product_swiglu_epilogue(fmt: str) -> None:
    """The gate/up group with the SwiGLU epilogue (columns interleaved in blocks of 64): y = bf16(bf16(silu(g)) u)
    of the rounded products. Against silu_mul of the exact products rounded to bf16: within four bf16 steps (a
    product within its error bound can round to the neighbouring bf16 value, moving g or u by one step), and 5e-4
    absolute where g or u is near zero (the products' float32 summation slack, about 1e-4 here, dominates there)."""
    from jeff_b200.fast_path import swiglu_order

    g = torch.Generator().manual_seed(77)
    m, k, inter, row_len, rank, pool_rows = 512, 1024, 3584, 128, 32, 3
    w = torch.randn(2 * inter, k, generator=g) * 0.02
    packed, W = prod_int4.quantize_pack(w, fmt)
    order = swiglu_order(inter)
    a_pool = (torch.randn(pool_rows, rank, k, generator=g) * 0.02).to(torch.bfloat16)
    b_pool = (torch.randn(pool_rows, 2 * inter, rank, generator=g) * 0.02).to(torch.bfloat16)
    adapters = torch.randint(0, pool_rows, (m // row_len,), generator=g, dtype=torch.int32)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    zeros = None if packed.zeros is None else packed.zeros[:, order].contiguous().cuda()
    words = kernels.int4_repack(packed.words[:, order].contiguous().cuda())
    got = kernels.int4_product(x.cuda(), words, packed.scales[:, order].contiguous().cuda(), zeros, packed.group,
                               2 * inter, a_pool.cuda(), b_pool[:, order].contiguous().cuda(), adapters.cuda(),
                               row_len, swiglu=True).cpu().float()
    row_of = adapters.long().repeat_interleave(row_len)
    exact, _ = exact_product(x.float(), W.float(), a_pool.float(), b_pool.float(), row_of)
    gu = bf(exact.float())
    want = model_ref.silu_mul(gu)
    torch.testing.assert_close(got, want, rtol=4 * BF16_STEP, atol=5e-4)


@pytest.mark.parametrize("fmt", ["g128z", "g64"])
@pytest.mark.parametrize(("m", "k", "out", "rank", "row_len", "swiglu"), [
    (64, 1024, 3584, 16, 64, False),        # configuration 1: one row for the whole pass
    (256, 1024, 8224, 48, 128, False),      # the Gated DeltaNet projection (columns not a multiple of 128)
    (384, 2048, 1024, 16, 128, False),      # out_proj
    (200, 3584, 1024, 16, 256, False),      # down_proj, K = 3584, m past the last full tile
    (512, 1024, 7168, 32, 128, True),       # gate|up with the SwiGLU epilogue
    (1000, 1024, 4608, 0, 128, False),      # no LoRA, ragged m
])
def test_tensor_memory_product_gives_the_bits_of_the_shared_memory_form(fmt: str, m: int, k: int, out: int,
                                                                         rank: int, row_len: int,
                                                                         swiglu: bool) -> None:
    """The tensor-memory form (JB_PRODUCT_TMEM_A: weights dequantised into tensor memory as the MMA's A operand,
    tokens as N) against the shared-memory form on the same inputs: every bit the same (each output is the same fp32
    sum in the same K order, rounded once), with and without LoRA and SwiGLU, both int4 formats, ragged m and
    columns. The shared-memory form is itself held to the float64 error bound above."""
    from jeff_b200.fast_path import swiglu_order

    g = torch.Generator().manual_seed(m + k + out + rank)
    w = torch.randn(out, k, generator=g) * 0.02
    packed, _ = prod_int4.quantize_pack(w, fmt)
    words, scales, zeros = packed.words, packed.scales, packed.zeros
    if swiglu:
        order = swiglu_order(out // 2)
        words, scales = words[:, order], scales[:, order]
        zeros = None if zeros is None else zeros[:, order]
    pool_rows = 4
    lora_a = lora_b = adapters = None
    if rank:
        lora_a = (torch.randn(pool_rows, rank, k, generator=g) * 0.02).to(torch.bfloat16).cuda()
        lora_b = torch.zeros(pool_rows, packed.columns, rank, dtype=torch.bfloat16)
        lora_b[:, :out] = (torch.randn(pool_rows, out, rank, generator=g) * 0.05).to(torch.bfloat16)
        lora_b = lora_b.cuda()
        adapters = torch.randint(-1, pool_rows + 1, (-(-m // row_len),), generator=g, dtype=torch.int32).cuda()
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    args = (x, kernels.int4_repack(words.contiguous().cuda()), scales.contiguous().cuda(),
            None if zeros is None else zeros.contiguous().cuda(), packed.group, out, lora_a, lora_b, adapters,
            row_len)
    tm = kernels.int4_product(*args, swiglu=swiglu, tmem_a=True)
    sm = kernels.int4_product(*args, swiglu=swiglu)
    assert torch.equal(tm.view(torch.int16), sm.view(torch.int16)), \
        f"{int((tm != sm).sum())} of {tm.numel()} outputs differ, max {float((tm.float() - sm.float()).abs().max())}"


@pytest.mark.parametrize(("m", "k", "rank", "row_len"), [
    (256, 1024, 48, 64),      # tcgen05 kernel: 128-token tiles of two adapters
    (512, 3584, 16, 128),     # tcgen05, K = 3584
    (208, 2048, 64, 64),      # tcgen05, m not a multiple of the 128-token tile
    (384, 1024, 32, 128),     # tcgen05
    (256, 1024, 48, 32),      # tcgen05, rows of 32 tokens: four adapters in a tile (two passes at rank 48)
    (96, 1024, 32, 16),       # small pass (dot kernel): rows of 16 tokens
    (96, 960, 16, 32),        # small pass: K not a multiple of 128
    (200, 1024, 16, 1),       # tcgen05, one adapter id per token: every adapter of the pool in a tile
    (240, 2048, 32, 48),      # tcgen05, rows of 48 tokens: tiles that span rows
    (100, 1024, 64, 7),       # small pass, rows of 7 tokens
    (32, 3584, 48, 32),       # small pass: a batch-1 row of the down projection's K
])
def test_lora_shrink_matches_the_oracle(m: int, k: int, rank: int, row_len: int) -> None:
    """mid = bf16(x A[a]^T) per row's adapter: within one bf16 step of the float32 product (summation order), and the
    same bits on a second call (fixed-order reductions)."""
    g = torch.Generator().manual_seed(m + k + rank)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    a_pool = (torch.randn(3, rank, k, generator=g) * 0.02).to(torch.bfloat16)
    rows = (m + row_len - 1) // row_len
    adapters = torch.randint(0, 3, (rows,), generator=g, dtype=torch.int32)
    got = kernels.lora_shrink(x.cuda(), a_pool.cuda(), adapters.cuda(), row_len).cpu()
    row_of = adapters.long().repeat_interleave(row_len)[:m]
    want = torch.stack([x[i].float() @ a_pool[row_of[i]].float().T for i in range(m)])
    torch.testing.assert_close(got.float(), bf(want), rtol=BF16_STEP, atol=1e-6)
    again = kernels.lora_shrink(x.cuda(), a_pool.cuda(), adapters.cuda(), row_len).cpu()
    assert torch.equal(got, again)


def test_lora_shrink_per_token_ids_give_the_bits_of_whole_rows() -> None:
    """The shrink with one adapter id per token (blocks of several adapters, one K pass per adapter) returns the
    same bits as with those tokens' rows of 64 (blocks of one adapter): a row's result depends on its own x and
    adapter only."""
    g = torch.Generator().manual_seed(11)
    m, k, rank, row_len = 256, 1024, 16, 64
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    a_pool = (torch.randn(4, rank, k, generator=g) * 0.02).to(torch.bfloat16).cuda()
    rows = torch.tensor([3, 1, 1, 2], dtype=torch.int32)
    whole = kernels.lora_shrink(x, a_pool, rows.cuda(), row_len)
    per_token = kernels.lora_shrink(x, a_pool, rows.repeat_interleave(row_len).cuda(), 1)
    assert np.array_equal(bits(whole), bits(per_token))


# ---------------------------------------------------------------- configuration 2: packed requests of mixed lengths


@pytest.fixture(scope="module")
def cfg2_pass() -> tuple[list[int], list[int], torch.Tensor]:
    lengths = synthetic.cfg2_lengths()
    chosen = synthetic.cfg2_adapters()
    per_token = torch.tensor(chosen, dtype=torch.int32).repeat_interleave(torch.tensor(lengths))
    return lengths, chosen, per_token


@pytest.mark.parametrize("shape", synthetic.CFG2_SHAPES, ids=[s[0] for s in synthetic.CFG2_SHAPES])
def test_cfg2_packed_projection_within_its_bound_and_equal_to_the_padded_pass(cfg2_pass, shape) -> None:
    """Configuration 2: 64 requests of 32 to 128 tokens packed into 4096 rows with one adapter id per token (row_len
    1: the gathered expand over each tile's adapters, shrink blocks of several adapters), 8 rank-16 adapters, int4
    group 128 with zeros. Every output lies within the error bound of the exact product (as above), and every row
    is bit for bit the row of the same request padded to a 128-token row (row_len 128: one adapter per 128-row half,
    the expand loaded by TMA): a row's bits depend on its own input and adapter only, however requests are laid
    out in the pass."""
    lengths, chosen, per_token = cfg2_pass
    name, k, n = shape
    proj = synthetic.cfg2_projection(name, k, n)
    words = kernels.int4_repack(proj.packed.words.cuda())
    scales, zeros = proj.packed.scales.cuda(), proj.packed.zeros.cuda()
    a_pool, b_pool = proj.lora_a.cuda(), proj.lora_b.cuda()
    got = kernels.int4_product(proj.x.cuda(), words, scales, zeros, proj.packed.group, n, a_pool, b_pool,
                               per_token.cuda(), 1).cpu()
    starts = np.cumsum([0, *lengths[:-1]]).tolist()
    padded = torch.zeros(len(lengths) * 128, k, dtype=torch.bfloat16)
    for i, (s0, ln) in enumerate(zip(starts, lengths, strict=True)):
        padded[128 * i:128 * i + ln] = proj.x[s0:s0 + ln]
    got_padded = kernels.int4_product(padded.cuda(), words, scales, zeros, proj.packed.group, n, a_pool, b_pool,
                                      torch.tensor(chosen, dtype=torch.int32).cuda(), 128).cpu()
    rows = torch.cat([torch.arange(128 * i, 128 * i + ln) for i, ln in enumerate(lengths)])
    assert np.array_equal(bits(got), bits(got_padded[rows]))
    exact, bound = exact_product(proj.x.float(), proj.W.float(), proj.lora_a.float(), proj.lora_b[:, :n].float(),
                                 per_token.long())
    err = (got.double() - exact).abs()
    assert int((err > bound).sum()) == 0, f"worst at {(err / bound.clamp_min(1e-30)).max():.3g} x the bound"


# ---------------------------------------------------------------- norms and activations


@pytest.mark.parametrize(("rows", "n"), [(96, 1024), (7, 1024), (5, 2048)])
def test_add_rms_and_rms_last_match_the_oracle(rows: int, n: int) -> None:
    """Rows of 1024 (the warp-per-row kernel, including a row count that leaves a block part empty) and of 2048
    (the block-per-row kernel): the sum bit-exact, the norm within one bf16 step."""
    g = torch.Generator().manual_seed(4 + rows)
    x = torch.randn(rows, n, generator=g).to(torch.bfloat16)
    d = torch.randn(rows, n, generator=g).to(torch.bfloat16)
    w = torch.randn(n, generator=g) * 0.1
    xo, h = kernels.add_rms(x.cuda(), d.cuda(), (1.0 + w).cuda())
    rx, rh = model_ref.add_rms(x.float(), d.float(), w)
    assert torch.equal(xo.cpu().float(), rx)     # one rounding of an exact sum
    torch.testing.assert_close(h.cpu().float(), rh, rtol=BF16_STEP, atol=1e-6)
    _, h0 = kernels.add_rms(x.cuda(), None, (1.0 + w).cuda())
    torch.testing.assert_close(h0.cpu().float(), model_ref.add_rms(x.float(), None, w)[1], rtol=BF16_STEP, atol=1e-6)
    if rows % 32:
        return
    last = torch.tensor([31, 0, 17], dtype=torch.int32)
    hid = kernels.rms_last(x.cuda(), d.cuda(), last.cuda(), 32, (1.0 + w).cuda()).cpu().float()
    at = torch.arange(3) * 32 + last.long()
    _, want = model_ref.add_rms(bf(x[at].float() + d[at].float()), None, w)
    torch.testing.assert_close(hid, want, rtol=BF16_STEP, atol=1e-6)


def test_activations_match_the_oracle() -> None:
    g = torch.Generator().manual_seed(5)
    gu = torch.randn(64, 2 * C.INTER, generator=g).to(torch.bfloat16)
    torch.testing.assert_close(kernels.silu_mul(gu.cuda()).cpu().float(), model_ref.silu_mul(gu.float()),
                               rtol=BF16_STEP, atol=1e-6)
    pr = torch.randn(64, C.ATTN_PROJ, generator=g).to(torch.bfloat16)
    o = torch.randn(64, C.NQ, C.HD, generator=g).to(torch.bfloat16)
    gate = pr.float()[:, :C.NQ * 2 * C.HD].view(64, C.NQ, 2 * C.HD)[:, :, C.HD:]
    torch.testing.assert_close(kernels.gate_mul(o.cuda(), pr.cuda()).cpu().float(),
                               model_ref.gate_mul(o.float(), gate), rtol=BF16_STEP, atol=1e-6)
    prg = torch.randn(64, C.GDN_PROJ, generator=g).to(torch.bfloat16)
    og = (0.3 * torch.randn(64, C.NV, C.DV, generator=g)).to(torch.bfloat16)
    wg = (1 + 0.1 * torch.randn(C.DV, generator=g)).to(torch.bfloat16)
    torch.testing.assert_close(kernels.gated_norm(og.cuda(), prg.cuda(), wg.cuda()).cpu().float(),
                               model_ref.gated_norm(og.float(), prg[:, C.QKV_DIM:C.QKV_DIM + C.Z_DIM], wg),
                               rtol=2 * BF16_STEP, atol=1e-5)
    table = torch.randn(500, 1024, generator=g).to(torch.bfloat16)
    ids = torch.randint(0, 500, (77,), generator=g, dtype=torch.int32)
    assert torch.equal(kernels.embed(table.cuda(), ids.cuda()).cpu(), table[ids.long()])


@pytest.mark.parametrize("b", BATCHES)
def test_readout_rows_match_the_oracle(b: int) -> None:
    g = torch.Generator().manual_seed(b)
    rng = random.Random(b)
    hidden = torch.randn(b, 1024, generator=g).to(torch.bfloat16)
    pool = (0.05 * torch.randn(6, 255, 1024, generator=g)).to(torch.bfloat16)
    temps = 0.5 + 1.5 * torch.rand(6, generator=g)
    adapters = torch.tensor([rng.randrange(6) for _ in range(b)], dtype=torch.int32)
    counts = torch.tensor(([1, 2, 255] + [rng.randrange(1, 256) for _ in range(b)])[:b], dtype=torch.int32)
    got = kernels.readout_rows(hidden.cuda(), pool.cuda(), temps.cuda(), adapters.cuda(), counts.cuda()).cpu()
    for r in range(b):
        want = model_ref.readout(hidden[r].float(), pool[adapters[r]], int(counts[r]), float(temps[adapters[r]]))
        torch.testing.assert_close(got[r], want, rtol=1e-3, atol=1e-5)
        assert not got[r, int(counts[r]):].any()


# ---------------------------------------------------------------- Gated DeltaNet


@pytest.mark.parametrize("b", BATCHES)
@pytest.mark.parametrize("n", [32, 64, 160])
@pytest.mark.parametrize("gdn_layer", [0, 13, 17])
def test_gdn_prep_rows_match_the_oracle(pool_fixture, b: int, n: int, gdn_layer: int) -> None:
    """q, k within two bf16 steps (the L2 norm's sum order), v and beta within one, g float32 within 1e-5."""
    pool, slots, states = pool_fixture
    ss = pass_slots(slots, b, seed=b * 100 + n + gdn_layer)
    tables, _ = tables_for(pool, ss)
    g = torch.Generator().manual_seed(gdn_layer)
    conv_w = bf(0.5 * torch.randn(4, C.QKV_DIM, generator=g)).contiguous()
    a_log = torch.randn(C.NV, generator=g)
    dt_bias = torch.randn(C.NV, generator=g)
    pr = torch.randn(b * n, C.GDN_PROJ, generator=g).to(torch.bfloat16)
    got = kernels.gdn_prep_rows(pr.cuda(), pool, tables, gdn_layer, conv_w.cuda(), (-torch.exp(a_log)).cuda(),
                                dt_bias.cuda(), n)
    for r in range(b):
        tail = states[ss[r]][0][gdn_layer]
        want = model_ref.gdn_prep(pr[r * n:(r + 1) * n], tail, conv_w.T, a_log, dt_bias)
        for name, x, y, rtol in zip("q k v".split(), got[:3], want[:3], (2 * BF16_STEP, 2 * BF16_STEP, BF16_STEP),
                                    strict=True):
            torch.testing.assert_close(x[r].cpu().float(), y, rtol=rtol, atol=1e-6, msg=lambda m, nm=name: f"{nm}: {m}")
        torch.testing.assert_close(got[3][r].cpu(), want[3], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(got[4][r].cpu().float(), want[4], rtol=BF16_STEP, atol=1e-6)


def test_gdn_prep_rows_prefix_mode_masks_padding_and_writes_conv_tails(pool_fixture) -> None:
    """The prefix pass's prep: tokens at or past a row's real length get g = beta = 0 (q, k, v as usual), and each
    row's last three real convolution inputs (from the cached tail when the row is shorter than three) go to its
    output pages, bit for bit."""
    pool, slots, states = pool_fixture
    ss = [slots[45], 0, slots[1000]]
    tables, _ = tables_for(pool, ss)
    b, n, gdn_layer = 3, 96, 5
    real = torch.tensor([96, 2, 57], dtype=torch.int32)
    g = torch.Generator().manual_seed(55)
    conv_w = bf(0.5 * torch.randn(4, C.QKV_DIM, generator=g)).contiguous()
    a_log = torch.randn(C.NV, generator=g)
    dt_bias = torch.randn(C.NV, generator=g)
    pr = torch.randn(b * n, C.GDN_PROJ, generator=g).to(torch.bfloat16)
    fresh = [pool.reserve(7, f"prep tail {i}", 64) for i in range(b)]
    pool.pin(fresh)
    try:
        out_tables, _ = tables_for(pool, fresh)
        got = kernels.gdn_prep_rows(pr.cuda(), pool, tables, gdn_layer, conv_w.cuda(), (-torch.exp(a_log)).cuda(),
                                    dt_bias.cuda(), n, real=real.cuda(), out_tables=out_tables)
        torch.cuda.synchronize()
        for r in range(b):
            rl = int(real[r])
            tail = states[ss[r]][0][gdn_layer]
            want = model_ref.gdn_prep(pr[r * n:(r + 1) * n], tail, conv_w.T, a_log, dt_bias)
            torch.testing.assert_close(got[2][r].cpu().float(), want[2], rtol=BF16_STEP, atol=1e-6)
            torch.testing.assert_close(got[3][r, :rl].cpu(), want[3][:rl], rtol=1e-5, atol=1e-6)
            assert not got[3][r, rl:].any() and not got[4][r, rl:].float().any()
            inputs = torch.cat([tail.to(torch.bfloat16), pr[r * n:(r + 1) * n, :C.QKV_DIM]])
            conv_out = pool.gather(fresh[r])[0][gdn_layer].cpu()
            assert torch.equal(conv_out, inputs[rl:rl + 3]), f"row {r}: conv tail"
    finally:
        pool.unpin(fresh)
        for slot in fresh:
            pool.release(slot)


GDN_RTOL, GDN_ATOL = 2.0 ** -6, 2.0 ** -9


def gdn_inputs(b: int, n: int, seed: int):
    g = torch.Generator().manual_seed(seed)

    def unit() -> torch.Tensor:
        x = torch.randn(b, n, C.NV, C.DK, generator=g)
        return (x / x.norm(dim=-1, keepdim=True)).to(torch.bfloat16)

    q, k = unit(), unit()
    v = torch.randn(b, n, C.NV, C.DV, generator=g).to(torch.bfloat16)
    gg = -0.5 * torch.nn.functional.softplus(torch.randn(b, n, C.NV, generator=g))
    beta = torch.sigmoid(torch.randn(b, n, C.NV, generator=g)).to(torch.bfloat16)
    return q, k, v, gg, beta


@pytest.mark.parametrize("kernel", ["tc", "chunk", "recurrent"])
@pytest.mark.parametrize("b", BATCHES)
@pytest.mark.parametrize("n", [32, 64, 160])
@pytest.mark.parametrize("gdn_layer", [0, 5, 17])
def test_gdn_scan_matches_the_oracle(pool_fixture, kernel: str, b: int, n: int, gdn_layer: int) -> None:
    """Each row from its own prefix state read in place (layer 5's heads straddle pages); n = 160 runs two whole
    64-token chunks and a partial one. GDN_RTOL, GDN_ATOL (the reference's: two bf16 steps at the largest outputs,
    set for fla's chunk kernel, whose bf16 operand roundings the chunk kernel shares); with a stop at the last real
    token, the real positions are bit for bit those without it and the padding positions zero."""
    pool, slots, states = pool_fixture
    ss = pass_slots(slots, b, seed=b * 7 + n + gdn_layer)
    tables, _ = tables_for(pool, ss)
    q, k, v, g, beta = gdn_inputs(b, n, seed=b + n + gdn_layer)
    got = kernels.gdn_scan(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), pool, tables, gdn_layer,
                           kernel=kernel)
    s0 = torch.stack([states[s][1][gdn_layer] for s in ss])
    want, _ = model_ref.gdn_scan(q.float(), k.float(), v.float(), g, beta.float(), s0)
    torch.testing.assert_close(got.cpu().float(), want, rtol=GDN_RTOL, atol=GDN_ATOL)
    rng = random.Random(b * n)
    last = torch.tensor([n - 1 if r == 0 else rng.randrange(n) for r in range(b)], dtype=torch.int32)
    stopped = kernels.gdn_scan(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), pool, tables, gdn_layer,
                               last=last.cuda(), kernel=kernel).cpu()
    for r in range(b):
        end = int(last[r]) + 1
        assert torch.equal(stopped[r, :end], got[r, :end].cpu())
        assert not stopped[r, end:].any()


@pytest.mark.parametrize("kernel", ["tc", "chunk", "recurrent"])
def test_gdn_scan_writes_the_final_state_into_the_output_pages(pool_fixture, kernel: str) -> None:
    """The prefix pass's final states: the recurrent kernel within float32 noise (rtol 1e-4); the two chunk kernels
    (tcgen05 and mma.sync), whose state products take bf16 operands, within 1e-2 norm-wise per head."""
    pool, slots, states = pool_fixture
    b, n = 3, 160
    ss = [slots[33], 0, slots[100]]
    tables, _ = tables_for(pool, ss)
    q, k, v, g, beta = gdn_inputs(b, n, seed=42)
    fresh = [pool.reserve(2, f"out {kernel} {i}", 40) for i in range(b)]
    pool.pin(fresh)
    out_tables = pool.tables.index_select(0, torch.tensor(fresh, device="cuda")).contiguous()
    kernels.gdn_scan(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), pool, tables, 7, out_tables=out_tables,
                     kernel=kernel)
    torch.cuda.synchronize()
    s0 = torch.stack([states[s][1][7] for s in ss])
    _, s_fin = model_ref.gdn_scan(q.float(), k.float(), v.float(), g, beta.float(), s0)
    pool.unpin(fresh)
    for i, slot in enumerate(fresh):
        got = pool.gather(slot)[1][7].cpu()
        if kernel == "recurrent":
            torch.testing.assert_close(got, s_fin[i], rtol=1e-4, atol=1e-5)
        else:
            for hh in range(16):
                assert model_ref.rel_error(got[hh], s_fin[i][hh]) < 1e-2
        pool.release(slot)


def gdn_layer_weights(seed: int):
    g = torch.Generator().manual_seed(seed)
    conv_w = bf(0.5 * torch.randn(4, C.QKV_DIM, generator=g)).contiguous()
    a_log = torch.randn(C.NV, generator=g)
    dt_bias = torch.randn(C.NV, generator=g)
    gnorm = (1.0 + 0.1 * torch.randn(C.DV, generator=g)).to(torch.bfloat16)
    return conv_w, a_log, dt_bias, gnorm, g


def three_kernels(pr, pool, tables, gdn_layer, conv_w, a_neg, dt_bias, gnorm, n, last=None, real=None,
                  out_tables=None, scan="chunk"):
    """jb_gdn_prep_rows, jb_gdn_scan (the mma.sync chunk form, which jb_gdn_layer shares bit for bit, unless `scan`
    names another) and jb_gated_norm in sequence."""
    q, k, v, g, beta = kernels.gdn_prep_rows(pr, pool, tables, gdn_layer, conv_w, a_neg, dt_bias, n, real=real,
                                             out_tables=out_tables)
    o = kernels.gdn_scan(q, k, v, g, beta, pool, tables, gdn_layer, last=last, out_tables=out_tables,
                         kernel=scan)
    return kernels.gated_norm(o.view(-1, C.NV, C.DV), pr, gnorm)


@pytest.mark.parametrize(("b", "n"), [(1, 32), (3, 96), (16, 160), (64, 128)])
@pytest.mark.parametrize("gdn_layer", [0, 5, 17])
def test_gdn_layer_is_bit_identical_to_prep_scan_and_norm(pool_fixture, b: int, n: int, gdn_layer: int) -> None:
    """The fused mixer (jb_gdn_layer) against jb_gdn_prep_rows + jb_gdn_scan + jb_gated_norm on the same inputs:
    every bit of y the same, for rows whose prefixes (states and conv tails read in place) have mixed lengths, with
    partial chunks (n = 32, 96, 160) and a stop at each row's last real token."""
    pool, slots, states = pool_fixture
    ss = pass_slots(slots, b, seed=b * 11 + n + gdn_layer)
    tables, _ = tables_for(pool, ss)
    conv_w, a_log, dt_bias, gnorm, g = gdn_layer_weights(gdn_layer + n)
    pr = torch.randn(b * n, C.GDN_PROJ, generator=g).to(torch.bfloat16).cuda()
    rng = random.Random(b * n + gdn_layer)
    last = torch.tensor([n - 1 if r == 0 else rng.randrange(n) for r in range(b)], dtype=torch.int32).cuda()
    args = (pr, pool, tables, gdn_layer, conv_w.cuda(), (-torch.exp(a_log)).cuda(), dt_bias.cuda(), gnorm.cuda(), n)
    want = three_kernels(*args, last=last)
    got = kernels.gdn_layer(*args, last=last)
    assert torch.equal(bits_t(got), bits_t(want))
    assert torch.equal(bits_t(kernels.gdn_layer(*args)), bits_t(three_kernels(*args)))


def bits_t(x: torch.Tensor) -> torch.Tensor:
    return x.contiguous().view(torch.int16)


def test_gdn_layer_prefix_mode_writes_the_same_pages(pool_fixture) -> None:
    """The prefix pass: padding tokens (from each row's real length) leave the state unchanged; each row's final
    state and last three real conv inputs go to its own pages. Fused and three-kernel runs write the same bits into
    two sets of fresh pages, and the same y."""
    pool, slots, states = pool_fixture
    ss = [slots[45], 0, slots[1000]]
    tables, _ = tables_for(pool, ss)
    b, n, gdn_layer = 3, 96, 11
    real = torch.tensor([96, 2, 57], dtype=torch.int32).cuda()
    conv_w, a_log, dt_bias, gnorm, g = gdn_layer_weights(99)
    pr = torch.randn(b * n, C.GDN_PROJ, generator=g).to(torch.bfloat16).cuda()
    args = (pr, pool, tables, gdn_layer, conv_w.cuda(), (-torch.exp(a_log)).cuda(), dt_bias.cuda(), gnorm.cuda(), n)
    sets = [[pool.reserve(8, f"layer pages {which} {i}", 64) for i in range(b)] for which in range(2)]
    for fresh in sets:
        pool.pin(fresh)
    try:
        ys = []
        for fresh, run in zip(sets, (three_kernels, kernels.gdn_layer), strict=True):
            out_tables, _ = tables_for(pool, fresh)
            ys.append(run(*args, real=real, out_tables=out_tables))
        torch.cuda.synchronize()
        assert torch.equal(bits_t(ys[0]), bits_t(ys[1]))
        for a, c in zip(*sets, strict=True):
            conv_a, state_a, _ = pool.gather(a)
            conv_c, state_c, _ = pool.gather(c)
            assert torch.equal(conv_a[gdn_layer], conv_c[gdn_layer])
            assert torch.equal(state_a[gdn_layer].view(torch.int32), state_c[gdn_layer].view(torch.int32))
    finally:
        for fresh in sets:
            pool.unpin(fresh)
            for slot in fresh:
                pool.release(slot)


@pytest.mark.parametrize("path", ["fused", "tc"])
def test_gdn_layer_at_configuration_3_matches_the_oracle(path: str) -> None:
    """path "fused": jb_gdn_layer; "tc": jb_gdn_prep_rows, the tcgen05 scan and jb_gated_norm (the pass's three
    launches). Configuration 3 as specified: 64 rows x 256 new tokens, each from a pooled fp32 state ~ N(0, 0.1) of 16 heads
    of 128 x 128 and a cached conv tail ~ N(0, 1); raw q | k | v ~ N(0, 1) bf16 through the width-4 conv (weights
    ~ N(0, 0.5)), SiLU and the L2 norm; beta = sigmoid(N(0, 1)); g = logsigmoid(N(2, 0.5)) (A_log = 0, dt_bias = 0,
    a = -N(2, 0.5), so -exp(A_log) softplus(a + dt_bias) = logsigmoid(-a)); z ~ N(0, 1). The fused layer's y
    against the oracle's prep, token-by-token fp32 rule and gated norm (run on this GPU as the checker): norm-wise
    relative error per (row, head) within 1e-2; the final states written by the prefix-mode run within 1e-2 per
    head (the chunk rule's bf16 operands)."""
    b, n = 64, 256
    shapes_pool = PrefixPool(2 + b * 50 * 2 + 4, "cuda")
    sh = shapes_pool.shapes
    g = torch.Generator().manual_seed(3)
    slots = [shapes_pool.reserve(1, f"cfg3 {r}", 0) for r in range(b)]
    outs = [shapes_pool.reserve(2, f"cfg3 out {r}", 0) for r in range(b)]
    states = 0.1 * torch.randn(b, sh.gdn_layers, *sh.state, generator=g)
    tails = torch.randn(b, sh.gdn_layers, *sh.conv, generator=g).to(torch.bfloat16)
    for r, slot in enumerate(slots):
        shapes_pool.write(slot, tails[r].cuda(), states[r].cuda(), torch.zeros(sh.attn_layers, 2, 0, *sh.kv))
    gdn_layer = 4
    tables, _ = tables_for(shapes_pool, slots)
    out_tables, _ = tables_for(shapes_pool, outs)
    conv_w = bf(0.5 * torch.randn(4, C.QKV_DIM, generator=g)).contiguous()
    a_log, dt_bias = torch.zeros(C.NV), torch.zeros(C.NV)
    gnorm = torch.ones(C.DV, dtype=torch.bfloat16)
    pr = torch.empty(b * n, C.GDN_PROJ)
    pr[:, :C.QKV_DIM + C.Z_DIM] = torch.randn(b * n, C.QKV_DIM + C.Z_DIM, generator=g)
    pr[:, C.QKV_DIM + C.Z_DIM:C.QKV_DIM + C.Z_DIM + C.NV] = torch.randn(b * n, C.NV, generator=g)
    pr[:, C.QKV_DIM + C.Z_DIM + C.NV:] = -(2.0 + 0.5 * torch.randn(b * n, C.NV, generator=g))
    pr = pr.to(torch.bfloat16).cuda()
    real = torch.full((b,), n, dtype=torch.int32).cuda()
    args = (pr, shapes_pool, tables, gdn_layer, conv_w.cuda(), torch.full((C.NV,), -1.0).cuda(), dt_bias.cuda(),
            gnorm.cuda(), n)
    if path == "fused":
        y = kernels.gdn_layer(*args, real=real, out_tables=out_tables)
    else:
        y = three_kernels(*args, real=real, out_tables=out_tables, scan="tc").view(b * n, C.NV * C.DV)
    torch.cuda.synchronize()
    worst_y, worst_s = 0.0, 0.0
    for r in range(b):
        rows = slice(r * n, (r + 1) * n)
        q, k, v, gg, beta = model_ref.gdn_prep(pr[rows].float(), tails[r][gdn_layer].cuda(), conv_w.T.cuda(),
                                               a_log.cuda(), dt_bias.cuda())
        o, s_fin = model_ref.gdn_scan(q[None], k[None], v[None], gg[None], beta[None],
                                      states[r][gdn_layer][None].cuda())
        want = model_ref.gated_norm(model_ref.bf(o[0]), pr[rows, C.QKV_DIM:C.QKV_DIM + C.Z_DIM], gnorm.cuda())
        got = y[rows].float().view(n, C.NV, C.DV)
        want = want.view(n, C.NV, C.DV)
        for hh in range(C.NV):
            worst_y = max(worst_y, model_ref.rel_error(got[:, hh], want[:, hh]))
        fin = shapes_pool.gather(outs[r])[1][gdn_layer]
        for hh in range(C.NV):
            worst_s = max(worst_s, model_ref.rel_error(fin[hh], s_fin[0][hh]))
    print(f"configuration 3 ({path}): worst per-(row, head) relative error of y {worst_y:.2e}, of the final state "
          f"{worst_s:.2e}")
    assert worst_y < 1e-2
    assert worst_s < 1e-2


# ---------------------------------------------------------------- attention


@pytest.mark.parametrize("b", BATCHES)
@pytest.mark.parametrize("n", [32, 64])
def test_attn_prep_rows_match_the_oracle(pool_fixture, b: int, n: int) -> None:
    """Within two bf16 steps (the GPU's cos and sin may move a rounded value by one step); values bit for bit."""
    pool, slots, _ = pool_fixture
    ss = pass_slots(slots, b, seed=b + n)
    _, pos = tables_for(pool, ss)
    g = torch.Generator().manual_seed(b + n)
    qn = 0.1 * torch.randn(C.HD, generator=g)
    kn_w = 0.1 * torch.randn(C.HD, generator=g)
    inv = model_ref.inv_freq()
    pr = torch.randn(b * n, C.ATTN_PROJ, generator=g).to(torch.bfloat16)
    kn = torch.empty(b * n, C.NKV, C.HD, dtype=torch.bfloat16, device="cuda")
    vn = torch.empty_like(kn)
    q = kernels.attn_prep_rows(pr.cuda(), (1 + qn).cuda(), (1 + kn_w).cuda(), inv.cuda(), pos, kn, vn, n).cpu()
    for r in range(b):
        rq, rk, rv, _ = model_ref.attn_prep(pr[r * n:(r + 1) * n], qn, kn_w, int(pos[r]))
        sl = slice(r * n, (r + 1) * n)
        torch.testing.assert_close(q[sl].float(), rq, rtol=2 * BF16_STEP, atol=2 * BF16_STEP)
        torch.testing.assert_close(kn.cpu()[sl].float(), rk, rtol=2 * BF16_STEP, atol=2 * BF16_STEP)
        assert torch.equal(vn.cpu()[sl].float(), rv)


ATTN_RTOL, ATTN_ATOL = 2.0 ** -6, 2.0 ** -8


def attention_inputs(t: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(t, C.NQ, C.HD, generator=g).to(torch.bfloat16)
    kn = torch.randn(t, C.NKV, C.HD, generator=g).to(torch.bfloat16)
    vn = torch.randn(t, C.NKV, C.HD, generator=g).to(torch.bfloat16)
    pr = torch.randn(t, C.ATTN_PROJ, generator=g).to(torch.bfloat16)   # the gate halves of q_proj are read
    return q, kn, vn, pr


def gated_oracle(q, kp, vp, kn, vn, pr_rows):
    """bf16(bf16(attention) * bf16(sigmoid(gate))) per token (the reference's paged_attention then gate_mul)."""
    o = model_ref.bf(model_ref.attention(q, kp, vp, kn, vn))
    gate = pr_rows[:, :C.NQ * 2 * C.HD].float().view(-1, C.NQ, 2 * C.HD)[:, :, C.HD:]
    return model_ref.gate_mul(o, gate)


@pytest.mark.parametrize("split", [False, True])
@pytest.mark.parametrize("b", BATCHES)
@pytest.mark.parametrize("n", [32, 64, 128])
def test_gated_attention_on_tensor_memory_matches_the_oracle(pool_fixture, b: int, n: int, split: bool) -> None:
    """The tcgen05 kernel (S and O in tensor memory, K / V pages by TMA, the gate fused): prefix keys read in place
    from pages that hold NaN past each prefix's end (those V rows must be zeroed, not multiplied by zero), prefixes of
    0 to 1,000 tokens (partial pages, a partial last tile of 64 keys), the new keys causally, attention layers 0 and 5.
    Against the oracle's attention and gate multiply within ATTN_RTOL (plus one bf16 step for the second rounding) and
    ATTN_ATOL; and against the mma.sync kernel + jb_gate_mul within twice that (each is within it of the exact
    result). split: the key walk in slices with a combine (jb_paged_attention_gated_split: up to 16 slices at one
    row, so short prefixes leave slices with no keys), the same bounds, and the same bits on a second call."""
    pool, slots, states = pool_fixture
    ss = pass_slots(slots, b, seed=b * 13 + n)
    tables, pos = tables_for(pool, ss)
    q, kn, vn, pr = attention_inputs(b * n, seed=b * 3 + n)
    scratch = torch.empty(4 * 2**20, dtype=torch.float32, device="cuda") if split else None
    for layer in (0, 5):
        got = kernels.paged_attention_gated(q.cuda(), pool, tables, layer, pos, kn.cuda(), vn.cuda(), n,
                                            pr.cuda(), scratch=scratch).cpu()
        if split:
            again = kernels.paged_attention_gated(q.cuda(), pool, tables, layer, pos, kn.cuda(), vn.cuda(), n,
                                                  pr.cuda(), scratch=scratch).cpu()
            assert torch.equal(got, again)
        assert not got.isnan().any(), "the kernel let a NaN past a prefix's last token into the sums"
        old = kernels.gate_mul(kernels.paged_attention(q.cuda(), pool, tables, layer, pos, kn.cuda(), vn.cuda(), n),
                               pr.cuda()).cpu()
        # two implementations each within the tolerance of the exact result: within twice it of each other
        torch.testing.assert_close(got.float(), old.float(), rtol=2 * (ATTN_RTOL + BF16_STEP), atol=2 * ATTN_ATOL)
        for r in range(b):
            kv = states[ss[r]][2][layer]
            sl = slice(r * n, (r + 1) * n)
            want = gated_oracle(q[sl], kv[0], kv[1], kn[sl], vn[sl], pr[sl])
            torch.testing.assert_close(got[sl].float(), want, rtol=ATTN_RTOL + BF16_STEP, atol=ATTN_ATOL)


def test_gated_attention_at_configuration_4() -> None:
    """Configuration 4's attention: 64 rows of 128 new tokens, each over its own 512-token prefix (16 pages of a pool
    written with random keys and values), both attention layers that bracket the layout (0 and 5); against the oracle
    run on this GPU as the checker, within ATTN_RTOL (+ one bf16 step) and ATTN_ATOL."""
    b, n, plen = 64, 128, 512
    pool = PrefixPool(2 + b * (50 + plen // 32) + 4, "cuda")
    sh = pool.shapes
    g = torch.Generator().manual_seed(4)
    slots = [pool.reserve(1, f"cfg4 attention {r}", plen) for r in range(b)]
    kvs = []
    for slot in slots:
        kv = torch.randn(sh.attn_layers, 2, plen, *sh.kv, generator=g).to(torch.bfloat16)
        pool.write(slot, torch.zeros(sh.gdn_layers, *sh.conv), torch.zeros(sh.gdn_layers, *sh.state), kv.cuda())
        kvs.append(kv.cuda())
    tables, pos = tables_for(pool, slots)
    q, kn, vn, pr = (x.cuda() for x in attention_inputs(b * n, seed=44))
    for layer in (0, 5):
        got = kernels.paged_attention_gated(q, pool, tables, layer, pos, kn, vn, n, pr)
        worst = 0.0
        for r in range(b):
            sl = slice(r * n, (r + 1) * n)
            want = gated_oracle(q[sl], kvs[r][layer, 0], kvs[r][layer, 1], kn[sl], vn[sl], pr[sl])
            torch.testing.assert_close(got[sl].float(), want, rtol=ATTN_RTOL + BF16_STEP, atol=ATTN_ATOL)
            worst = max(worst, float((got[sl].float() - want).abs().max()))
        print(f"configuration 4 attention layer {layer}: max |y - y_oracle| {worst:.2e}")


@pytest.mark.parametrize("b", BATCHES)
@pytest.mark.parametrize("n", [32, 64])
def test_paged_attention_matches_the_oracle(pool_fixture, b: int, n: int) -> None:
    """Prefix keys/values read in place (NaN past each prefix's end must not be read), then the new keys causally,
    attention layers 0 and 5; ATTN_RTOL, ATTN_ATOL (the reference's: P is rounded to bf16 before P V)."""
    pool, slots, states = pool_fixture
    ss = pass_slots(slots, b, seed=b * 11 + n)
    tables, pos = tables_for(pool, ss)
    g = torch.Generator().manual_seed(b + n)
    q = torch.randn(b * n, C.NQ, C.HD, generator=g).to(torch.bfloat16)
    kn = torch.randn(b * n, C.NKV, C.HD, generator=g).to(torch.bfloat16)
    vn = torch.randn(b * n, C.NKV, C.HD, generator=g).to(torch.bfloat16)
    for layer in (0, 5):
        got = kernels.paged_attention(q.cuda(), pool, tables, layer, pos, kn.cuda(), vn.cuda(), n).cpu()
        assert not got.isnan().any(), "the kernel read a NaN past a prefix's last token"
        for r in range(b):
            kv = states[ss[r]][2][layer]
            sl = slice(r * n, (r + 1) * n)
            want = model_ref.attention(q[sl], kv[0], kv[1], kn[sl], vn[sl])
            torch.testing.assert_close(got[sl].float(), want, rtol=ATTN_RTOL, atol=ATTN_ATOL)
