"""jb_int4_lora_product_static, the product that takes no scratch from its caller and allocates nothing, against
jb_int4_lora_product with a caller-allocated scratch, both called through the C ABI on the same inputs.

The file is named to be collected last, so the static scratch is first used after every other test has run (and,
alone, on a fresh process). Two calls in a row on different shapes check that what a previous call left in the
scratch never reaches a result: the shrink writes all of it that the expand reads."""

from __future__ import annotations

import pytest
import torch

from jeff_b200 import _lib
from jeff_b200 import int4 as prod_int4
from jeff_b200 import kernels

STATIC_MID_MAX = 1048576   # JB_PRODUCT_STATIC_MID_MAX


def _operands(seed: int, m: int, k: int, out: int, rank: int, row_len: int, pool_rows: int = 4):
    g = torch.Generator().manual_seed(seed)
    packed, _ = prod_int4.quantize_pack(torch.randn(out, k, generator=g) * 0.02, "g128z")
    a_pool = (torch.randn(pool_rows, rank, k, generator=g) * 0.02).to(torch.bfloat16)
    b_pool = torch.zeros(pool_rows, packed.columns, rank, dtype=torch.bfloat16)
    b_pool[:, :out] = (torch.randn(pool_rows, out, rank, generator=g) * 0.02).to(torch.bfloat16)
    adapters = torch.randint(0, pool_rows, (m // row_len,), generator=g, dtype=torch.int32)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    dev = packed.to("cuda")
    words = kernels.int4_repack(dev.words)
    return dict(x=x.cuda(), words=words, scales=dev.scales, zeros=dev.zeros, group=packed.group,
                columns=packed.columns, out=out, a=a_pool.cuda(), b=b_pool.cuda(), rank=rank, pool_rows=pool_rows,
                adapters=adapters.cuda(), row_len=row_len)


def _call(name: str, o: dict, mid: torch.Tensor | None) -> torch.Tensor:
    m, k = o["x"].shape
    y = torch.full((m, o["out"]), float("nan"), dtype=torch.bfloat16, device="cuda")
    p = _lib.ptr
    head = (p(o["x"]), m, k, p(o["words"]), p(o["scales"]), p(o["zeros"]), o["group"], o["columns"], o["out"],
            p(o["a"]), p(o["b"]), o["rank"], o["pool_rows"], p(o["adapters"]), o["row_len"])
    tail = (p(y), y.stride(0), 0, _lib.stream_ptr())
    if name == "jb_int4_lora_product":
        _lib.call(name, *head, p(mid), *tail)
    else:
        _lib.call(name, *head, *tail)
    return y


@pytest.mark.gpu
def test_static_product_matches_the_scratch_product_on_two_calls_in_a_row() -> None:
    """Bit for bit the product given a caller scratch: the same kernels run on the same inputs (the static entry
    point differs only in where the LoRA shrink's output lives), on two calls in a row that share the array."""
    torch.cuda.set_device(0)
    cases = [
        _operands(11, 1024, 1024, 3584, 16, 128),    # one adapter per 128-row half
        _operands(12, 256, 2048, 1024, 48, 32),      # four adapters per half, a smaller m than the call before
    ]
    for o in cases:
        mid = torch.empty(o["x"].shape[0], o["rank"], dtype=torch.bfloat16, device="cuda")
        want = _call("jb_int4_lora_product", o, mid)
        got = _call("jb_int4_lora_product_static", o, None)
        torch.cuda.synchronize()
        assert not torch.isnan(got).any()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_static_product_refuses_more_than_its_scratch() -> None:
    """m x rank beyond the static scratch is refused before anything reaches the device (runs without a GPU)."""
    _lib.load()
    p = 16
    m, rank = STATIC_MID_MAX // 64 + 16, 64
    with pytest.raises(_lib.ArgumentError, match="exceeds the static scratch"):
        _lib.call("jb_int4_lora_product_static", p, m, 1024, p, p, None, 128, 1024, 1024, p, p, rank, 2, p, 128,
                  p, 1024, 0, None)
