"""The seeded inputs of the reference benchmark's configuration 2 (the int4 + multi-LoRA projection sweep) on the
CPU: 64 request lengths in [32, 128] that sum to the 4096-token pass, one of 8 adapters per request, the projection
pools with row 0 as the base, and the same draws on every call."""

from __future__ import annotations

import pytest
import torch

from jeff_b200 import synthetic


def test_cfg2_lengths_fill_the_pass_inside_their_range() -> None:
    lengths = synthetic.cfg2_lengths()
    assert len(lengths) == 64 and sum(lengths) == 4096
    assert min(lengths) >= 32 and max(lengths) <= 128
    assert lengths == synthetic.cfg2_lengths()
    assert sum(synthetic.cfg2_lengths(total=64 * 128)) == 64 * 128
    assert set(synthetic.cfg2_lengths(total=64 * 32)) == {32}
    with pytest.raises(ValueError, match="cannot sum"):
        synthetic.cfg2_lengths(total=64 * 128 + 1)


def test_cfg2_adapters_are_pool_rows_one_to_eight() -> None:
    chosen = synthetic.cfg2_adapters()
    assert len(chosen) == 64 and set(chosen) <= set(range(1, 9)) and len(set(chosen)) == 8
    assert chosen == synthetic.cfg2_adapters()


def test_cfg2_projection_pools_and_shapes() -> None:
    proj = synthetic.cfg2_projection("k", 1024, 512, tokens=64)
    assert proj.packed.group == 128 and proj.packed.zeros is not None
    assert proj.lora_a.shape == (9, 16, 1024) and proj.lora_b.shape == (9, proj.packed.columns, 16)
    assert not proj.lora_a[0].any() and not proj.lora_b[0].any()
    assert proj.lora_a[1:].abs().sum(dim=(1, 2)).min() > 0
    assert proj.x.shape == (64, 1024) and proj.x.dtype == torch.bfloat16
    assert dict((name, (k, n)) for name, k, n in synthetic.CFG2_SHAPES)["down"] == (3584, 1024)
