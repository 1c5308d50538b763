"""The C ABI (include/jeffb200.h) on the CPU: the library loads without a GPU, exports every declared entry point,
and refuses bad arguments with JB_EINVAL and a message before touching the device."""

from __future__ import annotations

import ctypes

import pytest

from jeff_b200 import _lib


@pytest.fixture(scope="module")
def lib() -> ctypes.CDLL:
    from jeff_b200 import build

    build.build()
    return _lib.load()


def test_every_declared_entry_point_is_exported(lib: ctypes.CDLL) -> None:
    names = _lib.header_symbols()
    assert len(names) >= 19
    for name in names:
        assert hasattr(lib, name), name
    assert lib.jb_abi_version() == 2


def test_bad_arguments_are_refused_before_any_launch(lib: ctypes.CDLL) -> None:
    p = ctypes.c_void_p(16)
    # k not a multiple of 64
    assert lib.jb_w4a16_lora(p, 64, 100, p, p, None, 64, 128, 128, None, None, 0, 0, None, 64, p, 128, 0, None) == -1
    assert b"multiple of 64" in lib.jb_last_error()
    # group must be 64 or 128
    assert lib.jb_int4_dequant(p, p, None, 128, 128, 32, p, None) == -1
    assert b"group" in lib.jb_last_error()
    # a pass must hold whole rows
    assert lib.jb_gdn_prep_rows(p, 8224, 100, 32, p, 393216, p, 434, 48, 0, p, p, p, p, p, p, p, p, None, None, 0,
                                None) == -1
    assert b"rows of 32" in lib.jb_last_error()
    # rows whose length is not a multiple of 128 gather the LoRA expand from a per-tile set of at most 256 pool rows,
    # kept for at most 128 row tiles (32768 tokens)
    assert lib.jb_w4a16_lora(p, 128, 1024, p, p, None, 64, 128, 128, p, p, 16, 300, p, 1, p, 128, 0, None) == -1
    assert b"at most 256" in lib.jb_last_error()
    assert lib.jb_w4a16_lora(p, 40000, 1024, p, p, None, 64, 128, 128, p, p, 16, 3, p, 48, p, 128, 0, None) == -1
    assert b"at most 32768 tokens" in lib.jb_last_error()
    # pools of more than 256 rows take the mma.sync shrinks; with K not a multiple of 128 the 16-row one, whose blocks
    # hold one adapter each
    assert lib.jb_lora_shrink(p, 32, 64, p, 16, 300, p, 1, p, None) == -1
    assert b"multiples of 16" in lib.jb_last_error()
    with pytest.raises(_lib.ArgumentError, match="rank 20"):
        _lib.call("jb_lora_shrink", p, 32, 64, p, 20, 1, p, 32, p, None)


def test_small_pass_product_refusals(lib: ctypes.CDLL) -> None:
    """jb_w4a16_lora_small refuses, before any launch, what its one-wave cluster form cannot hold: more than two LoRA
    rows, a slice count that is not 1, 2, 4 or 8 or leaves a slice's CTA a ragged token count, and a slice whose K
    blocks do not fit in shared memory."""
    p = ctypes.c_void_p(16)
    small = lib.jb_w4a16_lora_small
    # 48 tokens in rows of 16: three LoRA rows
    assert small(p, 48, 3584, p, p, None, 128, 1024, 1024, p, p, 16, 2, p, 16, p, 1024, 0, 0, None) == -1
    assert b"LoRA rows" in lib.jb_last_error()
    # 48 tokens over 8 slices: 6 tokens per slice's CTA
    assert small(p, 48, 3584, p, p, None, 128, 1024, 1024, None, None, 0, 0, None, 48, p, 1024, 0, 8, None) == -1
    assert b"multiple of 4" in lib.jb_last_error()
    assert small(p, 48, 3584, p, p, None, 128, 1024, 1024, None, None, 0, 0, None, 48, p, 1024, 0, 3, None) == -1
    assert b"1, 2, 4 or 8" in lib.jb_last_error()
    # one slice of all 56 K blocks
    assert small(p, 48, 3584, p, p, None, 128, 1024, 1024, None, None, 0, 0, None, 48, p, 1024, 0, 1, None) == -1
    assert b"shared memory" in lib.jb_last_error()


def test_the_product_library_has_no_stage_trace(lib: ctypes.CDLL) -> None:
    """The trace read-outs exist only in measurement builds (-DJB_TRACE), not in the product library."""
    for name in ("jb_stage_trace_read", "jb_prod_trace_read", "jb_small_trace_read", "jb_small_span_read"):
        assert not hasattr(lib, name), name
